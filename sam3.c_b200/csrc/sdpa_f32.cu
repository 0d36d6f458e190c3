// sdpa_f32.cu - F32 scaled-dot-product attention for the backend vtable's
// SAM3_OP_SDPA on F32 tensors (cpu_sdpa.c:216-288: softmax(q.k^T/sqrt(hd)
// + mask).v with an online softmax over key tiles).
//
// The F32 graph is what the reference's sam3_vit_build hands a backend that
// is not Metal, so this kernel carries every attention FLOP of the drop-in
// path (110 GFLOP per global block, 12 per window block at 1008 px).  It is
// a flash-attention tile loop on the FP32 pipe (the vtable's bar is 1e-4,
// which the tensor-core kernels' 16-bit operands do not meet):
//   * one CTA = 64 queries of one (batch, head); 128 threads; thread
//     (qg = tid / 8, kg = tid % 8) owns queries qg*4 .. qg*4+3;
//   * per 64-key tile: S (4 queries x keys kg, kg+8, ..., kg+56) from Q and
//     K rows in shared memory (row pitch 68 floats: the 8 lanes of a phase
//     read 8 consecutive K rows without bank conflicts; the Q row is a
//     broadcast), row max / sum across the 8 lanes of a query by shuffles,
//     P written to shared memory, then O (4 queries x 8 of the head dims)
//     += P.V with V rows read as float4;
//   * the next K / V tile is fetched with cp.async once every thread is done
//     with the current one; three CTAs per SM hide the fetch.
// Tensors are addressed through (batch, head, row) strides, so the
// reference's [B,S,H,hd] -> permute(0,2,1,3) copies before and after SDPA
// (graph_helpers.c:840-880) become strides: the vtable hands this kernel
// the pre-permute views and the post-permute output.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "../../include/sam3cu.h"
#include "sam3cu_internal.h"

using namespace s3;

namespace {

constexpr int kBr = 64;      // queries per CTA
constexpr int kBc = 64;      // keys per tile
constexpr int kPitch = 68;   // shared row pitch (floats) of Q, K and P
constexpr int kThreads = 128;
#ifndef S3_SDPA_NBUF
#define S3_SDPA_NBUF 1
#endif
// K/V buffers: 2 = the next tile is fetched (cp.async) while the current one
// is used, 2 CTAs per SM; 1 = fetched after it, 3 CTAs per SM, the other
// CTAs covering the fetch.  Measured (global / window TFLOP/s): 2 -> 35.0 /
// 33.3, 1 -> 39.2 / 37.5.
constexpr int kNBuf = S3_SDPA_NBUF;

struct SdpaArgs {
  const float* q;
  const float* k;
  const float* v;
  const float* mask;  // [sq, sk] or null
  float* o;
  int64_t qb, qh, qs;  // element strides of Q (batch, head, row)
  int64_t kb, kh, ks;
  int64_t vb, vh, vs;
  int64_t ob, oh, os;
  int heads, sq, sk;
  float scale;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  const int n = valid ? 16 : 0;  // zero fill when out of range
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

// rows [r0, r0+64) x HD floats of a (row-strided) tensor into shared rows of
// `pitch` floats; rows past `nrows` are zero-filled.
template <int HD>
__device__ __forceinline__ void load_tile(float* sm, int pitch, const float* base, int64_t rs, int r0, int nrows) {
  constexpr int kVecPerRow = HD / 4;
  for (int i = threadIdx.x; i < kBr * kVecPerRow; i += kThreads) {
    const int r = i / kVecPerRow, c = (i % kVecPerRow) * 4;
    const bool ok = r0 + r < nrows;
    const float* src = base + static_cast<int64_t>(ok ? r0 + r : 0) * rs + c;
    cp_async16(sm + r * pitch + c, src, ok);
  }
}

template <int HD>
__global__ void __launch_bounds__(kThreads, kNBuf == 1 ? 3 : 2) sdpa_f32_tiled(SdpaArgs a) {
  constexpr int kDPer = HD / 8;  // head dims per thread in the P.V product
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  float* Qs = sm;                              // [64][68]
  float* Ks = Qs + kBr * kPitch;               // 2 x [64][68]
  float* Vs = Ks + kNBuf * kBc * kPitch;       // kNBuf x [64][HD]
  float* Ps = Vs + kNBuf * kBc * HD;           // [64][68]

  const int tid = threadIdx.x;
  const int qg = tid >> 3, kg = tid & 7;
  const int bh = blockIdx.y;
  const int b = bh / a.heads, h = bh % a.heads;
  const int q0 = blockIdx.x * kBr;
  const float* qbase = a.q + b * a.qb + h * a.qh;
  const float* kbase = a.k + b * a.kb + h * a.kh;
  const float* vbase = a.v + b * a.vb + h * a.vh;

  load_tile<HD>(Qs, kPitch, qbase, a.qs, q0, a.sq);
  load_tile<HD>(Ks, kPitch, kbase, a.ks, 0, a.sk);
  load_tile<HD>(Vs, HD, vbase, a.vs, 0, a.sk);
  cp_async_commit();

  float m[4], l[4], acc[4][kDPer];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -FLT_MAX;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kDPer; ++j) acc[i][j] = 0.f;
  }

  const int ntiles = (a.sk + kBc - 1) / kBc;
  for (int t = 0; t < ntiles; ++t) {
    const int buf = kNBuf == 2 ? (t & 1) : 0;
    cp_async_wait_all();
    __syncthreads();  // tile t visible; every thread is done with tile t-1
    if (kNBuf == 2 && t + 1 < ntiles) {
      load_tile<HD>(Ks + (buf ^ 1) * kBc * kPitch, kPitch, kbase, a.ks, (t + 1) * kBc, a.sk);
      load_tile<HD>(Vs + (buf ^ 1) * kBc * HD, HD, vbase, a.vs, (t + 1) * kBc, a.sk);
    }
    cp_async_commit();
    const float* Kt = Ks + buf * kBc * kPitch;
    const float* Vt = Vs + buf * kBc * HD;

    // S = Q K^T for queries qg*4+i, keys kg+8j
    float s[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) s[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < HD; d += 4) {
      float4 qv[4], kv[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(Qs + (qg * 4 + i) * kPitch + d);
#pragma unroll
      for (int j = 0; j < 8; ++j) kv[j] = *reinterpret_cast<const float4*>(Kt + (kg + 8 * j) * kPitch + d);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          s[i][j] = fmaf(qv[i].x, kv[j].x, s[i][j]);
          s[i][j] = fmaf(qv[i].y, kv[j].y, s[i][j]);
          s[i][j] = fmaf(qv[i].z, kv[j].z, s[i][j]);
          s[i][j] = fmaf(qv[i].w, kv[j].w, s[i][j]);
        }
    }

    // online softmax per query row across the 8 lanes kg = 0..7
    const int kbase_idx = t * kBc;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = q0 + qg * 4 + i;
      float mx = -FLT_MAX;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int kj = kbase_idx + kg + 8 * j;
        float v = s[i][j] * a.scale;
        if (a.mask && qi < a.sq && kj < a.sk) v += a.mask[static_cast<int64_t>(qi) * a.sk + kj];
        if (kj >= a.sk) v = -INFINITY;
        s[i][j] = v;
        mx = fmaxf(mx, v);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      const float mnew = fmaxf(m[i], mx);
      const float corr = expf(m[i] - mnew);  // 0 on the first tile (m = -FLT_MAX)
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float p = expf(s[i][j] - mnew);
        s[i][j] = p;
        sum += p;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      l[i] = l[i] * corr + sum;
      m[i] = mnew;
#pragma unroll
      for (int j = 0; j < kDPer; ++j) acc[i][j] *= corr;
#pragma unroll
      for (int j = 0; j < 8; ++j) Ps[(qg * 4 + i) * kPitch + kg + 8 * j] = s[i][j];
    }
    __syncwarp();  // the 8 lanes sharing a query row are in this warp

    // O += P V for queries qg*4+i, head dims (kg*4 + 32*c + e) for HD 64,
    // kg*4 + e for HD 32 (V rows are contiguous floats: float4 loads)
#pragma unroll 4
    for (int kk = 0; kk < kBc; kk += 4) {
      float4 pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = *reinterpret_cast<const float4*>(Ps + (qg * 4 + i) * kPitch + kk);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float* vr = Vt + (kk + u) * HD + kg * 4;
        float vv[kDPer];
#pragma unroll
        for (int c = 0; c < kDPer / 4; ++c) {
          const float4 x = *reinterpret_cast<const float4*>(vr + 32 * c);
          vv[4 * c] = x.x;
          vv[4 * c + 1] = x.y;
          vv[4 * c + 2] = x.z;
          vv[4 * c + 3] = x.w;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p = u == 0 ? pv[i].x : (u == 1 ? pv[i].y : (u == 2 ? pv[i].z : pv[i].w));
#pragma unroll
          for (int j = 0; j < kDPer; ++j) acc[i][j] = fmaf(p, vv[j], acc[i][j]);
        }
      }
    }
    if (kNBuf == 1 && t + 1 < ntiles) {  // one buffer: refill it once every thread is done with it
      __syncthreads();
      load_tile<HD>(Ks, kPitch, kbase, a.ks, (t + 1) * kBc, a.sk);
      load_tile<HD>(Vs, HD, vbase, a.vs, (t + 1) * kBc, a.sk);
      cp_async_commit();
    }
  }
  cp_async_wait_all();

  float* obase = a.o + b * a.ob + h * a.oh;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = q0 + qg * 4 + i;
    if (qi >= a.sq) continue;
    const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
    float* orow = obase + static_cast<int64_t>(qi) * a.os + kg * 4;
#pragma unroll
    for (int c = 0; c < kDPer / 4; ++c) {
      float4 x;
      x.x = acc[i][4 * c] * inv;
      x.y = acc[i][4 * c + 1] * inv;
      x.z = acc[i][4 * c + 2] * inv;
      x.w = acc[i][4 * c + 3] * inv;
      *reinterpret_cast<float4*>(orow + 32 * c) = x;
    }
  }
}

template <int HD>
constexpr int smem_bytes() {
  return static_cast<int>(sizeof(float)) * (kBr * kPitch + kNBuf * kBc * kPitch + kNBuf * kBc * HD + kBr * kPitch);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int sam3cu_sdpa_f32_strided(const float* q, const int64_t* q_strides, const float* k, const int64_t* k_strides,
                            const float* v, const int64_t* v_strides, const float* mask, float* o,
                            const int64_t* o_strides, int batch, int heads, int sq, int sk, int hd, void* stream) {
  if (!q || !k || !v || !o || !q_strides || !k_strides || !v_strides || !o_strides || batch <= 0 || heads <= 0 ||
      sq <= 0 || sk <= 0)
    return SAM3CU_EINVAL;
  if (hd != 64 && hd != 32) return SAM3CU_ESHAPE;
  if (static_cast<int64_t>(batch) * heads > 65535) return SAM3CU_ESHAPE;
  // 16-byte vector loads and stores: every base and stride a multiple of 4 floats
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return SAM3CU_ESHAPE;
  for (int i = 0; i < 3; ++i)
    if ((q_strides[i] | k_strides[i] | v_strides[i] | o_strides[i]) & 3) return SAM3CU_ESHAPE;
  SdpaArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.mask = mask;
  a.o = o;
  a.qb = q_strides[0], a.qh = q_strides[1], a.qs = q_strides[2];
  a.kb = k_strides[0], a.kh = k_strides[1], a.ks = k_strides[2];
  a.vb = v_strides[0], a.vh = v_strides[1], a.vs = v_strides[2];
  a.ob = o_strides[0], a.oh = o_strides[1], a.os = o_strides[2];
  a.heads = heads;
  a.sq = sq;
  a.sk = sk;
  a.scale = 1.0f / sqrtf(static_cast<float>(hd));
  dim3 grid((sq + kBr - 1) / kBr, batch * heads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  count_launches(1);
  if (hd == 64) {
    constexpr int sb = smem_bytes<64>();
    cudaFuncSetAttribute(sdpa_f32_tiled<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, sb);
    cudaFuncSetAttribute(sdpa_f32_tiled<64>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    sdpa_f32_tiled<64><<<grid, kThreads, sb, st>>>(a);
  } else {
    constexpr int sb = smem_bytes<32>();
    cudaFuncSetAttribute(sdpa_f32_tiled<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, sb);
    cudaFuncSetAttribute(sdpa_f32_tiled<32>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    sdpa_f32_tiled<32><<<grid, kThreads, sb, st>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? SAM3CU_OK : SAM3CU_ELAUNCH;
}

int sam3cu_sdpa_f32(const float* q, const float* k, const float* v, const float* mask, float* o, int bh, int sq,
                    int sk, int hd, void* stream) {
  if (bh <= 0 || sq <= 0 || sk <= 0 || hd <= 0) return SAM3CU_EINVAL;
  const int64_t qs[3] = {static_cast<int64_t>(sq) * hd, 0, hd};
  const int64_t ks[3] = {static_cast<int64_t>(sk) * hd, 0, hd};
  return sam3cu_sdpa_f32_strided(q, qs, k, ks, v, ks, mask, o, qs, bh, 1, sq, sk, hd, stream);
}

}  // extern "C"
