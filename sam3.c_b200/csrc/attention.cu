// attention.cu - fused multi-head attention forward for head_dim 64:
//   O = softmax(Q K^T / sqrt(64)) V  per (group, head)
// with online softmax over key tiles (the algorithm of cpu_sdpa.c:49-159,
// evaluated tile-wise on tensor cores).  Q/K/V are read straight out of the
// fused QKV projection output [rows, ldq] (Q at column h*64, K at E + h*64,
// V at 2E + h*64, already RoPE-rotated by the QKV GEMM epilogue) and O is
// written head-merged [rows, ldo], which is what the out-projection GEMM
// reads: the reference's SLICE / RESHAPE / PERMUTE nodes around SDPA
// (graph_helpers.c:721-882) become addressing.
//
// A "group" is a run of `seq` consecutive rows attending to each other: a
// 24x24 window (seq 576) when the token order is window-major, or a whole
// image (seq 5184) for global blocks.
//
// The production path is the tcgen05 kernel in attention_sm100.cu; this
// version computes on the warp-level bf16/fp16 MMA (m16n8k16, fp32
// accumulate): 4 warps x 16 query rows per CTA, 64-key tiles double-buffered
// through cp.async with an XOR-swizzled shared-memory layout.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "sam3cu_internal.h"
#include "sam3cu_internal.h"
#include "sm100_ptx.cuh"

namespace s3 {

S3_DEV_ERROR_ACCESSOR(dev_error_attn)

namespace {

constexpr int kQT = 64;   // query rows per CTA
constexpr int kKT = 64;   // keys per tile
constexpr int kHD = 64;   // head dim

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset in a 64x64 16-bit tile
  return row * 128 + ((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <bool kBf16>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if (kBf16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <bool kBf16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if (kBf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Load rows [row0, row0+64) x 64 columns (16-bit) of a strided matrix into
// a swizzled smem tile; rows >= nvalid are zero-filled.
__device__ __forceinline__ void load_tile(uint32_t sdst, const uint16_t* g, int64_t ld, int row0,
                                          int nvalid, int tid) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = tid + i * 128;  // 512 chunks of 16 B
    const int r = idx >> 3, c = idx & 7;
    const bool ok = (row0 + r) < nvalid;
    const uint16_t* src = g + static_cast<int64_t>(ok ? row0 + r : 0) * ld + c * 8;
    cp_async16(sdst + swz(r, c), src, ok);
  }
}

template <bool kBf16>
__global__ void __launch_bounds__(128) attn_fwd_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                                                       const uint16_t* __restrict__ v, int64_t ldq,
                                                       uint16_t* __restrict__ o, int64_t ldo, int seq,
                                                       int q_tiles, float scale_log2) {
  __shared__ __align__(1024) uint8_t smem[kQT * 128 + 4 * kKT * 128];
  const uint32_t sq = smem_u32(smem);
  const uint32_t sk0 = sq + kQT * 128;
  const uint32_t sv0 = sk0 + 2 * kKT * 128;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int group = blockIdx.x / q_tiles;
  const int qt = blockIdx.x % q_tiles;
  const int head = blockIdx.y;
  const int64_t grow0 = static_cast<int64_t>(group) * seq;  // first row of the group
  const uint16_t* qg = q + grow0 * ldq + head * kHD;
  const uint16_t* kg = k + grow0 * ldq + head * kHD;
  const uint16_t* vg = v + grow0 * ldq + head * kHD;

  load_tile(sq, qg, ldq, qt * kQT, seq, tid);
  load_tile(sk0, kg, ldq, 0, seq, tid);
  load_tile(sv0, vg, ldq, 0, seq, tid);
  cp_async_commit();

  const int n_kt = (seq + kKT - 1) / kKT;
  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  uint32_t qf[4][4];

  for (int t = 0; t < n_kt; ++t) {
    const int buf = t & 1;
    if (t + 1 < n_kt) {
      load_tile(sk0 + (buf ^ 1) * kKT * 128, kg, ldq, (t + 1) * kKT, seq, tid);
      load_tile(sv0 + (buf ^ 1) * kKT * 128, vg, ldq, (t + 1) * kKT, seq, tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(sq + swz(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const uint32_t sk = sk0 + buf * kKT * 128, sv = sv0 + buf * kKT * 128;
    // S = Q K^T for this warp's 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // pairs of 8-key blocks
        const int r = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sk + swz(r, c), b0, b1, b2, b3);
        mma16816<kBf16>(s[2 * jp], qf[kk], b0, b1);
        mma16816<kBf16>(s[2 * jp + 1], qf[kk], b2, b3);
      }
    }
    // mask keys beyond seq
    const int key0 = t * kKT;
    if (key0 + kKT > seq) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int kc = key0 + j * 8 + (lane & 3) * 2;
        if (kc >= seq) { s[j][0] = -INFINITY; s[j][2] = -INFINITY; }
        if (kc + 1 >= seq) { s[j][1] = -INFINITY; s[j][3] = -INFINITY; }
      }
    }
    // online softmax (rows g and g+8 of this warp)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fmaxf(s[j][2 * h], s[j][2 * h + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run[h], mx);
      const float corr = exp2f((m_run[h] - m_new) * scale_log2);
      m_run[h] = m_new;
      const float mb = m_new * scale_log2;
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s[j][2 * h] = exp2f(s[j][2 * h] * scale_log2 - mb);
        s[j][2 * h + 1] = exp2f(s[j][2 * h + 1] * scale_log2 - mb);
        sum += s[j][2 * h] + s[j][2 * h + 1];
      }
      l_run[h] = l_run[h] * corr + sum;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        acc[j][2 * h] *= corr;
        acc[j][2 * h + 1] *= corr;
      }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16-key chunks
      uint32_t pa[4];
      pa[0] = pack2<kBf16>(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack2<kBf16>(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack2<kBf16>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack2<kBf16>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // pairs of 8-wide d blocks
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = jp * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sv + swz(r, c), b0, b1, b2, b3);
        mma16816<kBf16>(acc[2 * jp], pa, b0, b1);
        mma16816<kBf16>(acc[2 * jp + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }
  // finalise: rows g and g+8 of this warp
  float l0 = l_run[0], l1 = l_run[1];
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int r0 = qt * kQT + warp * 16 + (lane >> 2);
  uint16_t* og = o + grow0 * ldo + head * kHD;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int col = j * 8 + (lane & 3) * 2;
    if (r0 < seq)
      *reinterpret_cast<uint32_t*>(og + static_cast<int64_t>(r0) * ldo + col) =
          pack2<kBf16>(acc[j][0] * inv0, acc[j][1] * inv0);
    if (r0 + 8 < seq)
      *reinterpret_cast<uint32_t*>(og + static_cast<int64_t>(r0 + 8) * ldo + col) =
          pack2<kBf16>(acc[j][2] * inv1, acc[j][3] * inv1);
  }
}

}  // namespace

// Warp-MMA version (kept as the comparison baseline; SAM3CU_ATTN=mma selects it).
int launch_attention_mma(const void* q, const void* k, const void* v, int64_t ldq, void* o, int64_t ldo,
                         int dtype, int n_groups, int seq, int heads, int head_dim, cudaStream_t st) {
  if (head_dim != kHD) return kErrShape;
  if (ldq % 8 || ldo % 8) return kErrShape;
  if (n_groups <= 0 || seq <= 0 || heads <= 0) return kOk;
  const int q_tiles = (seq + kQT - 1) / kQT;
  dim3 grid(n_groups * q_tiles, heads);
  count_launches(1);
  const float scale_log2 = (1.0f / sqrtf(static_cast<float>(head_dim))) * 1.4426950408889634f;
  if (dtype == kBF16)
    attn_fwd_kernel<true><<<grid, 128, 0, st>>>(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k),
                                                static_cast<const uint16_t*>(v), ldq, static_cast<uint16_t*>(o),
                                                ldo, seq, q_tiles, scale_log2);
  else if (dtype == kF16)
    attn_fwd_kernel<false><<<grid, 128, 0, st>>>(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k),
                                                 static_cast<const uint16_t*>(v), ldq, static_cast<uint16_t*>(o),
                                                 ldo, seq, q_tiles, scale_log2);
  else
    return kErrDtype;
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_attention(const void* q, const void* k, const void* v, int64_t ldq, void* o, int64_t ldo, int dtype,
                     int n_groups, int seq, int heads, int head_dim, cudaStream_t st) {
  static const int use_mma = [] {
    const char* e = getenv("SAM3CU_ATTN");
    return e && strcmp(e, "mma") == 0 ? 1 : 0;
  }();
  if (use_mma) return launch_attention_mma(q, k, v, ldq, o, ldo, dtype, n_groups, seq, heads, head_dim, st);
  return launch_attention_tc(q, k, v, ldq, o, ldo, dtype, n_groups, seq, heads, head_dim, st);
}

}  // namespace s3
