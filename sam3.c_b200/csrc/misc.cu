// misc.cu - HBM-bound kernels around the GEMMs: LayerNorm, patch im2col,
// row permutes, Q8 repack, dtype casts.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "io.cuh"
#include "misc.cuh"
#include "sam3cu_internal.h"
#include "sm100_ptx.cuh"
#include "gemm_sm100.cuh"

namespace s3 {

S3_DEV_ERROR_ACCESSOR(dev_error_misc)

namespace {


__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per row; the row lives in registers (NV float4 per lane, cols ==
// 128*NV).  Two-pass statistics exactly as cpu_layernorm.c:31-64: mean, then
// sum of squared deviations, inv_std = 1/sqrtf(var/cols + 1e-5).
template <int TI, int TO, int NV>
__global__ void __launch_bounds__(256) layernorm_rows(const void* __restrict__ x, void* __restrict__ y,
                                                      const float* __restrict__ g,
                                                      const float* __restrict__ b, int rows, int cols,
                                                      const int* __restrict__ out_row_map,
                                                      int out_row_period) {
  griddep_launch();  // the GEMM that follows may start its set-up
  griddep_wait();    // launched early behind a GEMM: its output is read below
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int64_t base = static_cast<int64_t>(warp) * cols;
  float4 v[NV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = IO<TI>::ld4(x, base + (i * 32 + lane) * 4);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  const float mean = warp_sum(s) / static_cast<float>(cols);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q += (a * a + bb * bb) + (c * c + d * d);
  }
  const float inv_std = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(cols) + 1e-5f);
  int orow = warp;
  if (out_row_map) orow = (warp / out_row_period) * out_row_period + out_row_map[warp % out_row_period];
  const int64_t obase = static_cast<int64_t>(orow) * cols;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    float4 r;
    r.x = (v[i].x - mean) * inv_std;
    r.y = (v[i].y - mean) * inv_std;
    r.z = (v[i].z - mean) * inv_std;
    r.w = (v[i].w - mean) * inv_std;
    if (g) {
      float4 gg = __ldg(reinterpret_cast<const float4*>(g + c));
      r.x *= gg.x; r.y *= gg.y; r.z *= gg.z; r.w *= gg.w;
    }
    if (b) {
      float4 bb = __ldg(reinterpret_cast<const float4*>(b + c));
      r.x += bb.x; r.y += bb.y; r.z += bb.z; r.w += bb.w;
    }
    IO<TO>::st4(y, obase + c, r);
  }
}

// Generic fallback (any cols, scalar, three passes over the row).
template <int TI, int TO>
__global__ void layernorm_rows_generic(const void* __restrict__ x, void* __restrict__ y,
                                       const float* __restrict__ g, const float* __restrict__ b,
                                       int rows, int cols) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  auto ld = [&](int64_t i) -> float {
    if (TI == kF32) return static_cast<const float*>(x)[i];
    if (TI == kBF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(x)[i]);
    return __half2float(static_cast<const __half*>(x)[i]);
  };
  const int64_t base = static_cast<int64_t>(warp) * cols;
  float s = 0.f;
  for (int c = lane; c < cols; c += 32) s += ld(base + c);
  const float mean = warp_sum(s) / static_cast<float>(cols);
  float q = 0.f;
  for (int c = lane; c < cols; c += 32) {
    float d = ld(base + c) - mean;
    q += d * d;
  }
  const float inv_std = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(cols) + 1e-5f);
  for (int c = lane; c < cols; c += 32) {
    float r = (ld(base + c) - mean) * inv_std;
    if (g) r *= g[c];
    if (b) r += b[c];
    if (TO == kF32) static_cast<float*>(y)[base + c] = r;
    else if (TO == kBF16) static_cast<__nv_bfloat16*>(y)[base + c] = __float2bfloat16_rn(r);
    else static_cast<__half*>(y)[base + c] = __float2half_rn(r);
  }
}

#ifndef S3_PDL_LN
#define S3_PDL_LN 0
#endif
// S3_PDL_LN: LayerNorm launched with programmatic dependent launch behind a
// GEMM (which then triggers its dependents after set-up)
#if S3_PDL_LN
#define S3_LN_LAUNCH(...) launch_pdl(__VA_ARGS__, blocks, 256, 0, st, x, y, g, b, rows, cols, map, period)
#else
#define S3_LN_LAUNCH(...) \
  (__VA_ARGS__<<<blocks, 256, 0, st>>>(x, y, g, b, rows, cols, map, period), \
   cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch)
#endif

template <int TI, int TO>
int ln_dispatch(const void* x, void* y, const float* g, const float* b, int rows, int cols,
                const int* map, int period, cudaStream_t st) {
  const int blocks = (rows + 7) / 8;
  const bool al = (cols % 128 == 0);
  if (al && cols == 1024)
    return S3_LN_LAUNCH(layernorm_rows<TI, TO, 8>);
  else if (al && cols == 512)
    return S3_LN_LAUNCH(layernorm_rows<TI, TO, 4>);
  else if (al && cols == 256)
    return S3_LN_LAUNCH(layernorm_rows<TI, TO, 2>);
  else if (al && cols == 128)
    return S3_LN_LAUNCH(layernorm_rows<TI, TO, 1>);
  else if (al && cols == 2048)
    return S3_LN_LAUNCH(layernorm_rows<TI, TO, 16>);
  else if (!map)
    layernorm_rows_generic<TI, TO><<<blocks, 256, 0, st>>>(x, y, g, b, rows, cols);
  else
    return kErrShape;
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

// Patch-embed im2col: image planar CHW [3, img, img] (per image) ->
// A[row, (ky*ps + kx)*3 + c] for the patch at raster position src_of_row[row
// % np] (so rows come out in whatever token order the map gives), K padded
// with zeros up to kpad.  Matches the OHWI weight layout of the reference's
// NHWC conv path (image_encoder.c:554-597).
template <int TO>
__global__ void patch_im2col(const float* __restrict__ img, void* __restrict__ a, int n_img, int img_sz,
                             int ps, int gs, int kpad, const int* __restrict__ src_of_row) {
  const int np = gs * gs;
  const int64_t total = static_cast<int64_t>(n_img) * np * kpad;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(i % kpad);
    const int64_t row = i / kpad;
    const int im = static_cast<int>(row / np);
    int p = static_cast<int>(row % np);
    if (src_of_row) p = src_of_row[p];
    float v = 0.f;
    const int kk = ps * ps * 3;
    if (k < kk) {
      const int c = k % 3, kx = (k / 3) % ps, ky = k / (3 * ps);
      const int py = p / gs, px = p % gs;
      v = img[((static_cast<int64_t>(im) * 3 + c) * img_sz + py * ps + ky) * img_sz + px * ps + kx];
    }
    if (TO == kBF16) static_cast<__nv_bfloat16*>(a)[i] = __float2bfloat16_rn(v);
    else if (TO == kF16) static_cast<__half*>(a)[i] = __float2half_rn(v);
    else static_cast<float*>(a)[i] = v;
  }
}

// The same for 16-bit output, one thread per (row, ky): it reads the three
// 14-float runs of image line py*ps + ky (one per channel) and writes the 42
// consecutive columns (ky*ps + kx)*3 + c as 21 packed pairs; thread ky == ps
// of a row zero-fills columns ps*ps*3 .. kpad.  32-bit index math; ps even.
template <int TO>
__global__ void patch_im2col16(const float* __restrict__ img, uint32_t* __restrict__ a, int rows, int img_sz,
                               int ps, int gs, int kpad, const int* __restrict__ src_of_row) {
  const int np = gs * gs;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = ps + 1;
  if (t >= rows * per_row) return;
  const int row = t / per_row, ky = t - row * per_row;
  uint32_t* arow = a + static_cast<int64_t>(row) * (kpad / 2);
  if (ky == ps) {  // zero padding of K
    for (int k2 = ps * ps * 3 / 2; k2 < kpad / 2; ++k2) arow[k2] = 0u;
    return;
  }
  const int im = row / np;
  int p = row - im * np;
  if (src_of_row) p = src_of_row[p];
  const int py = p / gs, px = p - py * gs;
  const int64_t plane = static_cast<int64_t>(img_sz) * img_sz;
  const float* src = img + static_cast<int64_t>(im) * 3 * plane + static_cast<int64_t>(py * ps + ky) * img_sz + px * ps;
  uint32_t* dst = arow + ky * ps * 3 / 2;
  float buf[2];
  int nb = 0, k2 = 0;
  for (int kx = 0; kx < ps; ++kx) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      buf[nb++] = __ldg(src + c * plane + kx);
      if (nb == 2) {
        uint32_t w;
        if (TO == kBF16) {
          __nv_bfloat162 h = __floats2bfloat162_rn(buf[0], buf[1]);
          w = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(buf[0], buf[1]);
          w = *reinterpret_cast<uint32_t*>(&h);
        }
        dst[k2++] = w;
        nb = 0;
      }
    }
  }
}

// Row gather: dst[(r/period)*period + r%period] = src[(r/period)*period +
// map[r%period]] for 16-byte vectors of `row_bytes`.
__global__ void gather_rows(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int rows,
                            int row_bytes, const int* __restrict__ map, int period) {
  const int vec = row_bytes / 16;
  const int64_t total = static_cast<int64_t>(rows) * vec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / vec), v = static_cast<int>(i % vec);
    const int sr = (r / period) * period + map[r % period];
    reinterpret_cast<uint4*>(dst + static_cast<int64_t>(r) * row_bytes)[v] =
        reinterpret_cast<const uint4*>(src + static_cast<int64_t>(sr) * row_bytes)[v];
  }
}

// Q8_0 blocks {f32 scale; i8 q[32]} (quant.h:30-33) over a flattened [N,K]
// weight, K % 32 == 0 -> int8 [N,K] + scales transposed [K/32, N].
__global__ void q8_repack(const uint8_t* __restrict__ blocks, int8_t* __restrict__ q, float* __restrict__ sc,
                          int N, int K) {
  const int kb = K / 32;
  const int64_t nblk = static_cast<int64_t>(N) * kb;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nblk;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint8_t* blk = blocks + b * 36;
    const int n = static_cast<int>(b / kb), j = static_cast<int>(b % kb);
    float s;
    memcpy(&s, blk, 4);
    sc[static_cast<int64_t>(j) * N + n] = s;
    int8_t* dst = q + static_cast<int64_t>(n) * K + j * 32;
#pragma unroll
    for (int i = 0; i < 32; ++i) dst[i] = static_cast<int8_t>(blk[4 + i]);
  }
}

// sam3_q8_quantize (quant.c:67-131) on the device, one block of 32 per
// thread: scale = absmax/127; q = roundf(x * (1/scale)) clamped to +-127;
// zero tail; scale 0 -> zero block.  IEEE division and roundf give the same
// bits as the reference's scalar path.
__global__ void q8_quantize_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst, int64_t n) {
  const int64_t nb = (n + 31) / 32;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nb;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t off = b * 32;
    const int cnt = static_cast<int>(n - off < 32 ? n - off : 32);
    float amax = 0.f;
    for (int i = 0; i < cnt; ++i) amax = fmaxf(amax, fabsf(src[off + i]));
    const float scale = __fdiv_rn(amax, 127.0f);
    uint8_t* blk = dst + b * 36;
    memcpy(blk, &scale, 4);
    const float inv = scale == 0.f ? 0.f : __fdiv_rn(1.0f, scale);
    for (int i = 0; i < 32; ++i) {
      int q = 0;
      if (scale != 0.f && i < cnt) {
        q = static_cast<int>(roundf(__fmul_rn(src[off + i], inv)));
        q = q > 127 ? 127 : (q < -127 ? -127 : q);
      }
      blk[4 + i] = static_cast<uint8_t>(static_cast<int8_t>(q));
    }
  }
}

// F32 -> 16-bit, 8 elements per thread (two 16-byte loads, one 16-byte store)
template <int TO>
__global__ void cast_f32_16_v8(const float4* __restrict__ x, uint4* __restrict__ y, int64_t n8) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 a = __ldg(x + 2 * i), b = __ldg(x + 2 * i + 1);
    uint32_t o[4];
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (TO == kBF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
        o[k] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
        o[k] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    y[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int TI, int TO>
__global__ void cast_kernel(const void* __restrict__ x, void* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v;
    if (TI == kF32) v = static_cast<const float*>(x)[i];
    else if (TI == kBF16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(x)[i]);
    else v = __half2float(static_cast<const __half*>(x)[i]);
    if (TO == kF32) static_cast<float*>(y)[i] = v;
    else if (TO == kBF16) static_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v);
    else static_cast<__half*>(y)[i] = __float2half_rn(v);
  }
}

int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  int cap = num_sms() * 16;
  return static_cast<int>(g < cap ? (g < 1 ? 1 : g) : cap);
}

}  // namespace

namespace {

// im2col for a dense KxK conv (zero padding) -> 16-bit columns: row
// (img, oy, ox), column (ky, kx, c) to match OHWI weights, zero-filled to
// kpad.  kChw: the input is planar CHW per image (the raw image), else NHWC.
template <int TI, int TO, bool kChw>
__global__ void conv_im2col(const void* __restrict__ x, void* __restrict__ a, int64_t total, int H, int W, int C,
                            int k, int stride, int pad, int OH, int OW, int kpad) {
  // grid-stride: the launcher caps the grid at 16 CTAs per SM
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total;  // total < 2^31 (launcher)
       i += gridDim.x * blockDim.x) {
  const int col = static_cast<int>(i % kpad);
  const unsigned row = i / kpad;
  const int ox = static_cast<int>(row % OW), oy = static_cast<int>((row / OW) % OH);
  const int64_t b = row / (static_cast<unsigned>(OW) * OH);
  float v = 0.f;
  if (col < k * k * C) {
    const int c = col % C, kx = (col / C) % k, ky = col / (C * k);
    const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
    if (iy >= 0 && iy < H && ix >= 0 && ix < W) {
      const int64_t src = kChw ? ((b * C + c) * H + iy) * W + ix : ((b * H + iy) * W + ix) * C + c;
      if (TI == kF32)
        v = static_cast<const float*>(x)[src];
      else if (TI == kBF16)
        v = __bfloat162float(static_cast<const __nv_bfloat16*>(x)[src]);
      else
        v = __half2float(static_cast<const __half*>(x)[src]);
    }
  }
  if (TO == kBF16)
    static_cast<__nv_bfloat16*>(a)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half*>(a)[i] = __float2half_rn(v);
  }
}

// 16-bit NHWC input with C % 8 == 0: one thread copies 8 channels (16
// bytes) of one tap; 32-bit index math (the launcher checks the count).
__global__ void conv_im2col_v8(const uint4* __restrict__ x, uint4* __restrict__ a, unsigned total, int H, int W,
                               int C8, int k, int stride, int pad, int OH, int OW, int kpad8, int kk8) {
  // grid-stride: the launcher caps the grid at 16 CTAs per SM
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
  const unsigned col = i % kpad8;
  const unsigned row = i / kpad8;
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (col < static_cast<unsigned>(kk8)) {
    const int c8 = col % C8, tap = col / C8;
    const int kx = tap % k, ky = tap / k;
    const int ox = row % OW, oy = (row / OW) % OH;
    const unsigned b = row / (static_cast<unsigned>(OW) * OH);
    const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
    if (iy >= 0 && iy < H && ix >= 0 && ix < W)
      v = __ldg(x + ((static_cast<int64_t>(b) * H + iy) * W + ix) * C8 + c8);
  }
  a[i] = v;
  }
}

}  // namespace

int launch_conv_im2col(const void* x, int tin, bool chw, void* a, int tout, int B, int H, int W, int C, int k,
                       int stride, int pad, int kpad, cudaStream_t st) {
  const int OH = (H + 2 * pad - k) / stride + 1, OW = (W + 2 * pad - k) / stride + 1;
  const int64_t total = static_cast<int64_t>(B) * OH * OW * kpad;
  if (!chw && tin == tout && tin != kF32 && C % 8 == 0 && kpad % 8 == 0) {
    const int64_t t8 = total / 8;
    if (t8 >= (1LL << 31)) return kErrShape;
    count_launches(1);
    conv_im2col_v8<<<grid_for(t8, 256), 256, 0, st>>>(static_cast<const uint4*>(x), static_cast<uint4*>(a),
                                                     static_cast<unsigned>(t8), H, W, C / 8, k, stride, pad, OH,
                                                     OW, kpad / 8, k * k * C / 8);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
  }
  if (total >= (1LL << 31)) return kErrShape;
  const int grid = grid_for(total, 256);
  count_launches(1);
#define S3_IC(TI, TO, CHW)                                                                               \
  if (tin == TI && tout == TO && chw == CHW) {                                                           \
    conv_im2col<TI, TO, CHW><<<grid, 256, 0, st>>>(x, a, total, H, W, C, k, stride, pad, OH, OW, kpad); \
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;                                         \
  }
  S3_IC(kF32, kBF16, true) S3_IC(kF32, kF16, true) S3_IC(kF32, kBF16, false) S3_IC(kF32, kF16, false)
  S3_IC(kBF16, kBF16, false) S3_IC(kF16, kF16, false)
#undef S3_IC
  return kErrDtype;
}

int launch_layernorm(const void* x, int tin, void* y, int tout, const float* g, const float* b, int rows,
                     int cols, const int* out_row_map, int out_row_period, cudaStream_t st) {
  if (rows <= 0) return kOk;
  if (cols <= 0) return kErrShape;
  count_launches(1);
#define S3_LN(TI, TO)                                                                       \
  if (tin == TI && tout == TO)                                                              \
    return ln_dispatch<TI, TO>(x, y, g, b, rows, cols, out_row_map, out_row_period, st);
  S3_LN(kF32, kF32) S3_LN(kF32, kBF16) S3_LN(kF32, kF16)
  S3_LN(kBF16, kF32) S3_LN(kBF16, kBF16) S3_LN(kF16, kF32) S3_LN(kF16, kF16)
#undef S3_LN
  return kErrDtype;
}

int launch_patch_im2col(const float* img, void* a, int tout, int n_img, int img_sz, int ps, int kpad,
                        const int* src_of_row, cudaStream_t st) {
  count_launches(1);
  const int gs = img_sz / ps;
  const int64_t rows = static_cast<int64_t>(n_img) * gs * gs;
  if ((tout == kBF16 || tout == kF16) && ps % 2 == 0 && kpad % 2 == 0 && rows * (ps + 1) < (1LL << 31)) {
    const int threads = static_cast<int>(rows * (ps + 1));
    if (tout == kBF16)
      patch_im2col16<kBF16><<<(threads + 255) / 256, 256, 0, st>>>(img, static_cast<uint32_t*>(a),
                                                                  static_cast<int>(rows), img_sz, ps, gs, kpad,
                                                                  src_of_row);
    else
      patch_im2col16<kF16><<<(threads + 255) / 256, 256, 0, st>>>(img, static_cast<uint32_t*>(a),
                                                                 static_cast<int>(rows), img_sz, ps, gs, kpad,
                                                                 src_of_row);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
  }
  const int64_t total = rows * kpad;
  const int grid = grid_for(total, 256);
  if (tout == kBF16) patch_im2col<kBF16><<<grid, 256, 0, st>>>(img, a, n_img, img_sz, ps, gs, kpad, src_of_row);
  else if (tout == kF16) patch_im2col<kF16><<<grid, 256, 0, st>>>(img, a, n_img, img_sz, ps, gs, kpad, src_of_row);
  else patch_im2col<kF32><<<grid, 256, 0, st>>>(img, a, n_img, img_sz, ps, gs, kpad, src_of_row);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_gather_rows(const void* src, void* dst, int rows, int row_bytes, const int* map, int period,
                       cudaStream_t st) {
  count_launches(1);
  if (row_bytes % 16) return kErrShape;
  const int64_t total = static_cast<int64_t>(rows) * (row_bytes / 16);
  gather_rows<<<grid_for(total, 256), 256, 0, st>>>(static_cast<const uint8_t*>(src),
                                                     static_cast<uint8_t*>(dst), rows, row_bytes, map,
                                                     period);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

namespace {

// Per output row n: the largest block scale m_n; scales of the row are
// multiplied by 2^e_n (exact) with e_n chosen so m_n * 2^e_n lies in
// [0.5, 1), and col_scale[n] = 2^-e_n undoes it after the GEMM.
__global__ void q8_row_shift_kernel(float* __restrict__ sc, float* __restrict__ col_scale, int N, int kb) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float m = 0.f;
  for (int j = 0; j < kb; ++j) m = fmaxf(m, fabsf(sc[static_cast<int64_t>(j) * N + n]));
  int e = 0;
  if (m > 0.f) {
    frexpf(m, &e);  // m = f * 2^e, f in [0.5, 1)
    e = -e;
  }
  const float up = ldexpf(1.0f, e);
  for (int j = 0; j < kb; ++j) sc[static_cast<int64_t>(j) * N + n] *= up;
  col_scale[n] = ldexpf(1.0f, -e);
}

}  // namespace

namespace {

// W16 [N, K] = int8 q [N, K] x scale of its 32-block (sc [K/32, N]); one
// thread per 16 values (one 16-byte load, two 16-byte stores).  mode 1
// (f16, scales row-shifted into f16's normal range): half2 arithmetic
// ((1024 + u) as f16 bits 0x64uu, minus 1152 exactly, times the scale
// rounded once); mode 0 (bf16) and 2 (f16, any scales): f32 arithmetic and
// one rounding.
__device__ __forceinline__ void q8_dequant_w16_one(const uint4* __restrict__ q, const float* __restrict__ sc,
                                                   uint4* __restrict__ w, int N, int K16, int64_t i, int f16) {
  const int n = static_cast<int>(i / K16), k16 = static_cast<int>(i - static_cast<int64_t>(n) * K16);
  const float s = __ldg(sc + static_cast<int64_t>(k16 >> 1) * N + n);
  const uint4 raw = __ldg(q + i);
  const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t out[8];
  if (f16 == 1) {
    const __half2 k1152 = __float2half2_rn(1152.0f), s2 = __float2half2_rn(s);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t u = words[j] ^ 0x80808080u;
      uint32_t h[2] = {__byte_perm(u, 0x64646464u, 0x4140), __byte_perm(u, 0x64646464u, 0x4342)};
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        __half2 v = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&h[k]), k1152), s2);
        out[2 * j + k] = *reinterpret_cast<uint32_t*>(&v);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t u = words[j] ^ 0x80808080u;
      float f[4];
#pragma unroll
      for (int b = 0; b < 4; ++b)
        f[b] = (__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650 + b)) - 8388736.0f) * s;
      if (f16) {
        __half2 a = __floats2half2_rn(f[0], f[1]), c = __floats2half2_rn(f[2], f[3]);
        out[2 * j] = *reinterpret_cast<uint32_t*>(&a);
        out[2 * j + 1] = *reinterpret_cast<uint32_t*>(&c);
      } else {
        __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]), c = __floats2bfloat162_rn(f[2], f[3]);
        out[2 * j] = *reinterpret_cast<uint32_t*>(&a);
        out[2 * j + 1] = *reinterpret_cast<uint32_t*>(&c);
      }
    }
  }
  w[2 * i] = make_uint4(out[0], out[1], out[2], out[3]);
  w[2 * i + 1] = make_uint4(out[4], out[5], out[6], out[7]);
}

__global__ void q8_dequant_w16_kernel(const uint4* __restrict__ q, const float* __restrict__ sc,
                                      uint4* __restrict__ w, int N, int K16, int64_t total, int f16) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < total) q8_dequant_w16_one(q, sc, w, N, K16, i, f16);
}

// Several weights in one launch: thread i works on the job whose range of
// 16-element groups holds it.
__global__ void q8_dequant_w16_multi_kernel(Q8DequantJobs jobs, int f16) {
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
#pragma unroll 1
  for (int j = 0; j < jobs.n; ++j) {
    const int64_t total = static_cast<int64_t>(jobs.job[j].N) * (jobs.job[j].K / 16);
    if (i < total) {
      q8_dequant_w16_one(reinterpret_cast<const uint4*>(jobs.job[j].q), jobs.job[j].sc,
                         static_cast<uint4*>(jobs.job[j].w), jobs.job[j].N, jobs.job[j].K / 16, i, f16);
      return;
    }
    i -= total;
  }
}

}  // namespace

namespace {
// F32 activations -> bf16 (8 per thread) and a Q8_0 weight -> bf16 (16
// values per thread) in one launch: the two inputs of an F32 x Q8_0 linear.
__global__ void q8_prep_kernel(const float4* __restrict__ x, uint4* __restrict__ xb, int64_t n8,
                               const uint4* __restrict__ q, const float* __restrict__ sc, uint4* __restrict__ w,
                               int N, int K16, int64_t total_w) {
  griddep_launch();  // the GEMM that follows may start its set-up
  // thread i: activation group i (8 values) and weight group i (16 values),
  // both in flight at once; no grid cap, one pass
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
  const bool has_x = i < n8;
  if (has_x) {
    a = __ldg(x + 2 * i);
    b = __ldg(x + 2 * i + 1);
  }
  if (i < total_w) q8_dequant_w16_one(q, sc, w, N, K16, i, 0);
  if (has_x) {
    __nv_bfloat162 h0 = __floats2bfloat162_rn(a.x, a.y), h1 = __floats2bfloat162_rn(a.z, a.w);
    __nv_bfloat162 h2 = __floats2bfloat162_rn(b.x, b.y), h3 = __floats2bfloat162_rn(b.z, b.w);
    xb[i] = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                       *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
  }
}
}  // namespace

int launch_q8_prep(const float* x, void* xb, int64_t nx, const int8_t* q, const float* sc, void* w, int N, int K,
                   cudaStream_t st) {
  if (nx % 8 || N <= 0 || K % 32 ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(xb) | reinterpret_cast<uintptr_t>(q) |
        reinterpret_cast<uintptr_t>(w)) & 15))
    return kErrShape;
  const int64_t total_w = static_cast<int64_t>(N) * (K / 16);
  const int64_t items = nx / 8 > total_w ? nx / 8 : total_w;
  const int64_t nblk = (items + 255) / 256;
  if (nblk >= (1LL << 31)) return kErrShape;
  count_launches(1);
  q8_prep_kernel<<<static_cast<unsigned>(nblk), 256, 0, st>>>(
      static_cast<const float4*>(static_cast<const void*>(x)), static_cast<uint4*>(xb), nx / 8,
      reinterpret_cast<const uint4*>(q), sc, static_cast<uint4*>(w), N, K / 16, total_w);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_q8_dequant_w16(const int8_t* q, const float* sc, void* w, int N, int K, int f16, cudaStream_t st) {
  if (N <= 0 || K % 32 || (reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return kErrShape;
  const int64_t total = static_cast<int64_t>(N) * (K / 16);
  count_launches(1);
  q8_dequant_w16_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const uint4*>(q), sc, static_cast<uint4*>(w), N, K / 16, total, f16);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_q8_dequant_w16_multi(const Q8DequantJobs& jobs, int f16, cudaStream_t st) {
  if (jobs.n <= 0 || jobs.n > Q8DequantJobs::kMax) return kErrShape;
  int64_t total = 0;
  for (int j = 0; j < jobs.n; ++j) {
    const Q8DequantJob& d = jobs.job[j];
    if (d.N <= 0 || d.K % 32 || (reinterpret_cast<uintptr_t>(d.q) & 15) || (reinterpret_cast<uintptr_t>(d.w) & 15))
      return kErrShape;
    total += static_cast<int64_t>(d.N) * (d.K / 16);
  }
  count_launches(1);
  q8_dequant_w16_multi_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(jobs, f16);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_q8_row_shift(float* sc, float* col_scale, int N, int K, cudaStream_t st) {
  if (N <= 0 || K % 32) return kErrShape;
  count_launches(1);
  q8_row_shift_kernel<<<(N + 255) / 256, 256, 0, st>>>(sc, col_scale, N, K / 32);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_q8_repack(const void* blocks, int8_t* q, float* sc, int N, int K, cudaStream_t st) {
  count_launches(1);
  if (K % 32) return kErrShape;
  const int64_t n = static_cast<int64_t>(N) * (K / 32);
  q8_repack<<<grid_for(n, 256), 256, 0, st>>>(static_cast<const uint8_t*>(blocks), q, sc, N, K);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_q8_quantize(const float* src, void* blocks, int64_t n, cudaStream_t st) {
  count_launches(1);
  q8_quantize_kernel<<<grid_for((n + 31) / 32, 256), 256, 0, st>>>(src, static_cast<uint8_t*>(blocks), n);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_cast(const void* x, int tin, void* y, int tout, int64_t n, cudaStream_t st) {
  count_launches(1);
  if (tin == kF32 && (tout == kBF16 || tout == kF16) && n % 8 == 0 &&
      !((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15)) {
    const int g8 = grid_for(n / 8, 256);
    if (tout == kBF16)
      cast_f32_16_v8<kBF16><<<g8, 256, 0, st>>>(static_cast<const float4*>(x), static_cast<uint4*>(y), n / 8);
    else
      cast_f32_16_v8<kF16><<<g8, 256, 0, st>>>(static_cast<const float4*>(x), static_cast<uint4*>(y), n / 8);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
  }
  const int grid = grid_for(n, 256);
#define S3_CAST(TI, TO) \
  if (tin == TI && tout == TO) { cast_kernel<TI, TO><<<grid, 256, 0, st>>>(x, y, n); return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch; }
  S3_CAST(kF32, kBF16) S3_CAST(kF32, kF16) S3_CAST(kBF16, kF32) S3_CAST(kF16, kF32) S3_CAST(kF32, kF32)
#undef S3_CAST
  return kErrDtype;
}

namespace {
// One thread waits until %globaltimer has advanced by `ns` (bounded by
// construction): parks a stream while the host enqueues work behind it.
__global__ void gpu_sleep_kernel(unsigned long long ns) {
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 >= ns) break;
    __nanosleep(10000);
  }
}
}  // namespace

int launch_gpu_sleep(unsigned long long ns, cudaStream_t st) {
  gpu_sleep_kernel<<<1, 1, 0, st>>>(ns);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace s3
