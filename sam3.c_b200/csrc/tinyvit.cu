// tinyvit.cu - TinyViT hot ops (image_encoder_tinyvit.c) on the B200 path.
//
// sam3cu_tvit_expand_bias        expand_attention_bias (:265-335), host
// sam3cu_tvit_window_attention   tvit_window_attention (:790-866) after the
//                                qkv linear: the reshape / slice / permute
//                                / scale / QK^T / +bias / softmax / .V /
//                                permute-back nodes as one tcgen05 kernel
// sam3cu_tvit_block_*            tvit_block_forward (:896-1052)
// sam3cu_tvit_mbconv_*           tvit_mbconv_forward (:682-720)
//
// The residual stream is NHWC f32 [images * H * W, C] in raster order, as
// in the reference.  Per TinyViTBlock (T = 16-bit activation type):
//   LN-gather  x -> xn T, rows in window-major order over the zero-padded
//              image (pad tokens are LayerNorm(0) = beta, as after the
//              reference's concat-with-zeros, :916-956)
//   QKV GEMM   xn . Wqkv^T + b -> qkv T [Tw, 3C] (per-head interleaved)
//   ATTN       window attention + relative position bias -> ao T [Tw, C]
//   PROJ GEMM  ao . Wproj^T + b -> p f32 [Tw, C]
//   UNPART     x[raster(t)] += p[t] for the tokens inside the image
//   DWCONV     3x3 depthwise conv of x with the BatchNorm folded into its
//              weights and bias -> lc f32
//   LN         lc -> xn T
//   FC1        xn . Wfc1^T + b, tanh-GELU -> h T
//   FC2        h . Wfc2^T + b + lc -> x f32
// Per MBConv (x f32 and its 16-bit copy xa):
//   CONV1      xa . W1'^T + b1', GELU -> h T        (1x1 conv, BN folded)
//   DWCONV     3x3 depthwise, BN folded, GELU -> h2 T
//   CONV3      h2 . W3'^T + b3' + x -> x f32        (in place, TMA reduce-add)
//   GELU       x = GELU(x), xa = T(x)
// BatchNorm folding: w' = w * s, b' = (b - mean) * s + beta with
// s = gamma / sqrtf(var + 1e-5) (cpu_batchnorm.c, eps 1e-5).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <memory>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/sam3cu.h"
#include "devbuf.cuh"
#include "gemm_sm100.cuh"
#include "io.cuh"
#include "misc.cuh"
#include "sam3cu_internal.h"

using namespace s3;

namespace {
cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int ck(cudaError_t e) { return e == cudaSuccess ? kOk : kErrCuda; }

int grid_1d(int64_t n, int block) {
  int64_t g = (n + block - 1) / block;
  return static_cast<int>(g < 1 ? 1 : (g > (1 << 30) ? (1 << 30) : g));
}

// Window-major padded token t of image b -> raster row of the unpadded
// image, or -1 for a padding token.
struct WinMap {
  int H, W, ws, nwx, n_tok, per_img;  // per_img = windows * ws * ws
  // t < 2^31 (the block forward checks its row count): 32-bit division
  __device__ __forceinline__ int64_t src_row(int64_t t64) const {
    const unsigned t = static_cast<unsigned>(t64);
    const unsigned b = t / per_img;
    const int r = static_cast<int>(t - b * per_img);
    const int w = r / n_tok, k = r - w * n_tok;
    const int py = (w / nwx) * ws + k / ws, px = (w % nwx) * ws + k % ws;
    if (py >= H || px >= W) return -1;
    return (static_cast<int64_t>(b) * H + py) * W + px;
  }
};

// LayerNorm of C-wide f32 rows (cpu_layernorm.c:31-64: mean, sum of squared
// deviations, 1/sqrtf(var/C + 1e-5), gamma, beta), one warp per output row;
// lane l holds columns l, l+32, ... (NE = C/32 of them).  With a window map
// the output row t reads source row map.src_row(t) (a zero row if -1).
template <int TO, int NE>
__global__ void __launch_bounds__(256) ln_rows_tvit(const float* __restrict__ x, void* __restrict__ y,
                                                    const float* __restrict__ g, const float* __restrict__ b,
                                                    int64_t rows, int C, WinMap map, int use_map) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t src = use_map ? map.src_row(row) : row;
  float v[NE];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NE; ++i) {
    v[i] = src >= 0 ? x[src * C + i * 32 + lane] : 0.f;
    s += v[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(C);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NE; ++i) {
    const float d = v[i] - mean;
    q += d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float inv_std = 1.0f / sqrtf(q / static_cast<float>(C) + 1e-5f);
#pragma unroll
  for (int i = 0; i < NE; ++i) {
    const int c = i * 32 + lane;
    float r = (v[i] - mean) * inv_std;
    if (g) r *= __ldg(g + c);
    if (b) r += __ldg(b + c);
    if (TO == kBF16)
      static_cast<__nv_bfloat16*>(y)[row * C + c] = __float2bfloat16_rn(r);
    else if (TO == kF16)
      static_cast<__half*>(y)[row * C + c] = __float2half_rn(r);
    else
      static_cast<float*>(y)[row * C + c] = r;
  }
}

template <int TO>
int ln_tvit_dispatch(const float* x, void* y, const float* g, const float* b, int64_t rows, int C,
                     const WinMap& m, int use_map, cudaStream_t st) {
  const int grid = grid_1d(rows * 32, 256);
  switch (C / 32) {
#define S3_CASE(NE)                                                                 \
  case NE:                                                                          \
    ln_rows_tvit<TO, NE><<<grid, 256, 0, st>>>(x, y, g, b, rows, C, m, use_map);    \
    break;
    S3_CASE(2) S3_CASE(3) S3_CASE(4) S3_CASE(6) S3_CASE(8) S3_CASE(9) S3_CASE(12) S3_CASE(16)
    S3_CASE(18) S3_CASE(24) S3_CASE(32)
#undef S3_CASE
    default:
      return kErrShape;
  }
  return ck(cudaGetLastError()) ? kErrLaunch : kOk;
}

int launch_ln_tvit(const float* x, void* y, int tout, const float* g, const float* b, int64_t rows, int C,
                   const WinMap* m, cudaStream_t st) {
  if (C % 32) return kErrShape;
  count_launches(1);
  WinMap mm{};
  if (m) mm = *m;
  const int use = m ? 1 : 0;
  if (tout == kBF16) return ln_tvit_dispatch<kBF16>(x, y, g, b, rows, C, mm, use, st);
  if (tout == kF16) return ln_tvit_dispatch<kF16>(x, y, g, b, rows, C, mm, use, st);
  return ln_tvit_dispatch<kF32>(x, y, g, b, rows, C, mm, use, st);
}

// x[map.src_row(t)] += p[t] for the tokens inside the image (f32, C % 4 == 0).
__global__ void unpartition_add(float* __restrict__ x, const float* __restrict__ p, int64_t rows, int C,
                                WinMap map) {
  const unsigned c4 = C / 4;
  const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;  // rows * C/4 < 2^31 (caller)
  if (i >= rows * c4) return;
  const unsigned t = i / c4;
  const int c = static_cast<int>(i - t * c4) * 4;
  const int64_t dst = map.src_row(t);
  if (dst < 0) return;
  const float4 a = *reinterpret_cast<const float4*>(p + static_cast<int64_t>(t) * C + c);
  float4* o = reinterpret_cast<float4*>(x + dst * C + c);
  float4 v = *o;
  v.x += a.x;
  v.y += a.y;
  v.z += a.z;
  v.w += a.w;
  *o = v;
}

__device__ __forceinline__ float gelu_f(float v) {
  // 0.5*x*(1+tanh(sqrt(2/pi)*(x+0.044715x^3))), cpu_gelu.c:23-36
  return 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v)));
}

// The same with the SFU's tanh.approx.f32 (relative error about 2^-11), for
// 16-bit outputs, whose rounding is coarser.
__device__ __forceinline__ float gelu_f16out(float v) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.7978845608f * (v + 0.044715f * v * v * v)));
  return 0.5f * v * (1.0f + t);
}
template <int TO>
__device__ __forceinline__ float gelu_out(float v) {
  return TO == kF32 ? gelu_f(v) : gelu_f16out(v);
}

// 3x3 depthwise conv, stride 1, zero padding 1, NHWC, four channels per
// thread; w9 [9][C] (tap-major, BatchNorm folded), bias [C]; optional GELU.
template <int TI, int TO, bool kGelu>
__global__ void dwconv3x3(const void* __restrict__ x, void* __restrict__ y, const float* __restrict__ w9,
                          const float* __restrict__ bias, int B, int H, int W, int C, int stride, int OH, int OW) {
  // 32-bit index math (the launcher checks B*OH*OW*C/4 < 2^31): 64-bit
  // division would dominate this memory-bound kernel
  const unsigned c4 = C / 4;
  const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
  const unsigned total = static_cast<unsigned>(B) * OH * OW * c4;
  if (i >= total) return;
  const int c = static_cast<int>(i % c4) * 4;
  const unsigned p = i / c4;  // output pixel
  const int ox = static_cast<int>(p % OW), oy = static_cast<int>((p / OW) % OH);
  const int64_t img = p / (static_cast<unsigned>(OH) * OW);
  const int yy = oy * stride, xx = ox * stride;  // input centre
  float4 acc = __ldg(reinterpret_cast<const float4*>(bias + c));
#pragma unroll
  for (int ky = 0; ky < 3; ++ky) {
    const int iy = yy + ky - 1;
    if (iy < 0 || iy >= H) continue;
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const int ix = xx + kx - 1;
      if (ix < 0 || ix >= W) continue;
      const float4 v = IO<TI>::ld4(x, ((img * H + iy) * W + ix) * C + c);
      const float4 k = __ldg(reinterpret_cast<const float4*>(w9 + (ky * 3 + kx) * C + c));
      acc.x = fmaf(v.x, k.x, acc.x);
      acc.y = fmaf(v.y, k.y, acc.y);
      acc.z = fmaf(v.z, k.z, acc.z);
      acc.w = fmaf(v.w, k.w, acc.w);
    }
  }
  if (kGelu) {
    acc.x = gelu_out<TO>(acc.x);
    acc.y = gelu_out<TO>(acc.y);
    acc.z = gelu_out<TO>(acc.z);
    acc.w = gelu_out<TO>(acc.w);
  }
  IO<TO>::st4(y, static_cast<int64_t>(p) * C + c, acc);
}

// The same conv, each thread computing kRows consecutive output rows of one
// column and 4 channels: the three input rows under the 3x3 window stay in
// registers, so each further output row loads one new input row (stride 1)
// or two (stride 2) instead of three, and each input value is read about
// 1.3x (stride 1) rather than 9x.  kS: the stride.
template <int TI, int TO, bool kGelu, int kS>
__global__ void dwconv3x3_rows(const void* __restrict__ x, void* __restrict__ y, const float* __restrict__ w9,
                               const float* __restrict__ bias, int H, int W, int C, int OH, int OW, int row_blocks,
                               unsigned total) {
  constexpr int kRows = 8;
  const unsigned c4 = C / 4;
  const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int c = static_cast<int>(i % c4) * 4;
  unsigned q = i / c4;
  const int ox = static_cast<int>(q % OW);
  q /= OW;
  const int oy0 = static_cast<int>(q % row_blocks) * kRows;
  const unsigned img = q / row_blocks;
  float4 k[9];
#pragma unroll
  for (int t = 0; t < 9; ++t) k[t] = __ldg(reinterpret_cast<const float4*>(w9 + t * C + c));
  const float4 b4 = __ldg(reinterpret_cast<const float4*>(bias + c));
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  // the three horizontal neighbours (zero outside the image) of input row iy
  auto load_row = [&](int iy, float4 (&r)[3]) {
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const int ix = ox * kS + kx - 1;
      r[kx] = (iy >= 0 && iy < H && ix >= 0 && ix < W)
                  ? IO<TI>::ld4(x, ((static_cast<int64_t>(img) * H + iy) * W + ix) * C + c)
                  : zero;
    }
  };
  auto fma4 = [](float4& a, const float4& v, const float4& w) {
    a.x = fmaf(v.x, w.x, a.x);
    a.y = fmaf(v.y, w.y, a.y);
    a.z = fmaf(v.z, w.z, a.z);
    a.w = fmaf(v.w, w.w, a.w);
  };
  float4 r0[3], r1[3], r2[3];
  load_row(oy0 * kS - 1, r0);
  if (kS == 1) load_row(oy0, r1);
#pragma unroll
  for (int rr = 0; rr < kRows; ++rr) {
    // no early exit: rows past the image load zeros and skip the store, so
    // the fully unrolled loop can issue later rows' loads early
    const int oy = oy0 + rr;
    if (kS == 1) {
      load_row(oy + 1, r2);
    } else {
      load_row(oy * 2, r1);
      load_row(oy * 2 + 1, r2);
    }
    float4 acc = b4;
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      fma4(acc, r0[kx], k[kx]);
      fma4(acc, r1[kx], k[3 + kx]);
      fma4(acc, r2[kx], k[6 + kx]);
    }
    if (kGelu) {
      acc.x = gelu_out<TO>(acc.x);
      acc.y = gelu_out<TO>(acc.y);
      acc.z = gelu_out<TO>(acc.z);
      acc.w = gelu_out<TO>(acc.w);
    }
    if (oy < OH) IO<TO>::st4(y, ((static_cast<int64_t>(img) * OH + oy) * OW + ox) * C + c, acc);
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      if (kS == 1) {
        r0[kx] = r1[kx];
        r1[kx] = r2[kx];
      } else {
        r0[kx] = r2[kx];
      }
    }
  }
}

// Stride-1 row kernel for the memory-bound MBConv pass (4 channels of one
// column per thread, kRows output rows): every input the thread needs,
// (kRows + 2) rows x 3 columns, is loaded up front in its storage type (8
// bytes for 16-bit data), so kRows * 3 + 6 independent loads are in flight
// per thread instead of the three of one row; the BatchNorm-folded taps and
// the bias come from shared memory.  ncu of the register-tap version showed
// DRAM at 10% of peak, 24% of warps active and long-scoreboard stalls: a
// latency-bound pass.  The grid is a few CTAs per SM, each loading the
// [9][C] taps once and striding over (channels, column, row block, image).
template <int TI>
struct DwRaw {
  using T = uint2;  // four 16-bit values
  static __device__ __forceinline__ T ld(const void* p, int64_t i) {
    return __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p) + i));
  }
  static __device__ __forceinline__ float4 f4(const T& r) {
    if (TI == kBF16) {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
      return make_float4(a.x, a.y, b.x, b.y);
    }
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  static __device__ __forceinline__ T zero() { return make_uint2(0u, 0u); }
};
template <>
struct DwRaw<kF32> {
  using T = float4;
  static __device__ __forceinline__ T ld(const void* p, int64_t i) {
    return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i));
  }
  static __device__ __forceinline__ float4 f4(const T& r) { return r; }
  static __device__ __forceinline__ T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
};

template <int TI, int TO, bool kGelu, int kRows>
__global__ void __launch_bounds__(256, 2) dwconv3x3_rows_smem(const void* __restrict__ x, void* __restrict__ y,
                                                           const float* __restrict__ w9,
                                                           const float* __restrict__ bias, int H, int W, int C,
                                                           int row_blocks, unsigned total) {
  using R = DwRaw<TI>;
  extern __shared__ float4 sm4[];
  float* sw = reinterpret_cast<float*>(sm4);  // [9][C] taps, then [C] bias
  for (int t = threadIdx.x; t < 10 * C / 4; t += blockDim.x)
    sm4[t] = __ldg(reinterpret_cast<const float4*>(t < 9 * C / 4 ? w9 + 4 * t : bias + 4 * t - 9 * C));
  __syncthreads();
  const unsigned c4 = C / 4;
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int c = static_cast<int>(i % c4) * 4;
    unsigned q = i / c4;
    const int ox = static_cast<int>(q % W);
    q /= W;
    const int oy0 = static_cast<int>(q % row_blocks) * kRows;
    const unsigned img = q / row_blocks;
    const float4* k = reinterpret_cast<const float4*>(sw + c);  // tap t at k[t * c4]
    typename R::T raw[kRows + 2][3];
#pragma unroll
    for (int r = 0; r < kRows + 2; ++r) {
      const int iy = oy0 + r - 1;
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const int ix = ox + kx - 1;
        raw[r][kx] = (iy >= 0 && iy < H && ix >= 0 && ix < W)
                         ? R::ld(x, ((static_cast<int64_t>(img) * H + iy) * W + ix) * C + c)
                         : R::zero();
      }
    }
#pragma unroll
    for (int rr = 0; rr < kRows; ++rr) {
      const int oy = oy0 + rr;
      float4 acc = k[9 * c4];  // bias
#pragma unroll
      for (int ky = 0; ky < 3; ++ky)
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
          const float4 v = R::f4(raw[rr + ky][kx]), w = k[(3 * ky + kx) * c4];
          acc.x = fmaf(v.x, w.x, acc.x);
          acc.y = fmaf(v.y, w.y, acc.y);
          acc.z = fmaf(v.z, w.z, acc.z);
          acc.w = fmaf(v.w, w.w, acc.w);
        }
      if (kGelu) {
        acc.x = gelu_out<TO>(acc.x);
        acc.y = gelu_out<TO>(acc.y);
        acc.z = gelu_out<TO>(acc.z);
        acc.w = gelu_out<TO>(acc.w);
      }
      if (oy < H) IO<TO>::st4(y, ((static_cast<int64_t>(img) * H + oy) * W + ox) * C + c, acc);
    }
  }
}

// 3x3 depthwise conv, zero padding 1, stride 1 or 2 (output (H-1)/s+1).
int launch_dwconv3x3(const void* x, int tin, void* y, int tout, const float* w9, const float* bias, int B,
                     int H, int W, int C, bool gelu, cudaStream_t st, int stride = 1) {
  if (C % 4 || stride < 1) return kErrShape;
  const int OH = (H - 1) / stride + 1, OW = (W - 1) / stride + 1;
  // stride 1: the row kernel (F32 blocks 0.369 -> 0.284 ms at 32 images);
  // stride 2: one output per thread measured faster (0.475 vs 0.904 ms per
  // launch; TinyViT 940 vs 919 images/s)
  static const bool old_rows = [] {  // S3CU_DWCONV=regs: taps in registers (A/B measurements)
    const char* e = getenv("S3CU_DWCONV");
    return e && strcmp(e, "regs") == 0;
  }();
  if (stride == 1 && !old_rows && 10 * C * 4 <= 48 * 1024) {
#ifndef S3_DW_ROWS16  // measured at 32 images, F16 (TinyViT images/s): 2 -> 926, 4 -> 956, 6 -> 966, 8 -> 964
#define S3_DW_ROWS16 6
#endif
    constexpr int kR16 = S3_DW_ROWS16, kR32 = 4;  // output rows per thread (16-bit / F32 input)
    const int rows = tin == kF32 ? kR32 : kR16;
    const int row_blocks = (OH + rows - 1) / rows;
    const int64_t total = static_cast<int64_t>(B) * row_blocks * OW * (C / 4);
    if (total >= (1LL << 31)) return kErrShape;
    count_launches(1);
    const int64_t want = (total + 255) / 256;
    const int grid = static_cast<int>(want < 8LL * num_sms() ? want : 8LL * num_sms());
    const unsigned t = static_cast<unsigned>(total);
    const size_t smem = static_cast<size_t>(10) * C * 4;
#define S3_DWS(TI, TO)                                                                                        \
  if (tin == TI && tout == TO) {                                                                              \
    constexpr int R_ = TI == kF32 ? kR32 : kR16;                                                              \
    if (gelu)                                                                                                 \
      dwconv3x3_rows_smem<TI, TO, true, R_><<<grid, 256, smem, st>>>(x, y, w9, bias, H, W, C, row_blocks, t); \
    else                                                                                                      \
      dwconv3x3_rows_smem<TI, TO, false, R_><<<grid, 256, smem, st>>>(x, y, w9, bias, H, W, C, row_blocks, t); \
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;                                              \
  }
    S3_DWS(kF32, kF32) S3_DWS(kBF16, kBF16) S3_DWS(kF16, kF16) S3_DWS(kF32, kBF16) S3_DWS(kF32, kF16)
#undef S3_DWS
    return kErrDtype;
  }
  if (stride == 1) {
    const int row_blocks = (OH + 7) / 8;
    const int64_t total = static_cast<int64_t>(B) * row_blocks * OW * (C / 4);
    if (total >= (1LL << 31)) return kErrShape;
    count_launches(1);
    const int grid = grid_1d(total, 256);
    const unsigned t = static_cast<unsigned>(total);
#define S3_DWR(TI, TO)                                                                                    \
  if (tin == TI && tout == TO) {                                                                          \
    if (stride == 1) {                                                                                    \
      if (gelu)                                                                                           \
        dwconv3x3_rows<TI, TO, true, 1><<<grid, 256, 0, st>>>(x, y, w9, bias, H, W, C, OH, OW, row_blocks, t);  \
      else                                                                                                \
        dwconv3x3_rows<TI, TO, false, 1><<<grid, 256, 0, st>>>(x, y, w9, bias, H, W, C, OH, OW, row_blocks, t); \
    } else {                                                                                              \
      if (gelu)                                                                                           \
        dwconv3x3_rows<TI, TO, true, 2><<<grid, 256, 0, st>>>(x, y, w9, bias, H, W, C, OH, OW, row_blocks, t);  \
      else                                                                                                \
        dwconv3x3_rows<TI, TO, false, 2><<<grid, 256, 0, st>>>(x, y, w9, bias, H, W, C, OH, OW, row_blocks, t); \
    }                                                                                                     \
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;                                          \
  }
    S3_DWR(kF32, kF32) S3_DWR(kBF16, kBF16) S3_DWR(kF16, kF16) S3_DWR(kF32, kBF16) S3_DWR(kF32, kF16)
#undef S3_DWR
    return kErrDtype;
  }
  const int64_t total = static_cast<int64_t>(B) * OH * OW * (C / 4);
  if (total >= (1LL << 31)) return kErrShape;
  count_launches(1);
  const int grid = grid_1d(total, 256);
#define S3_DW(TI, TO)                                                                            \
  if (tin == TI && tout == TO) {                                                                 \
    if (gelu)                                                                                    \
      dwconv3x3<TI, TO, true><<<grid, 256, 0, st>>>(x, y, w9, bias, B, H, W, C, stride, OH, OW);  \
    else                                                                                         \
      dwconv3x3<TI, TO, false><<<grid, 256, 0, st>>>(x, y, w9, bias, B, H, W, C, stride, OH, OW); \
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;                                 \
  }
  S3_DW(kF32, kF32) S3_DW(kBF16, kBF16) S3_DW(kF16, kF16) S3_DW(kF32, kBF16) S3_DW(kF32, kF16)
#undef S3_DW
  return kErrDtype;
}

// x = GELU(x) in place (f32) and xa = x as 16-bit.
template <int TO>
__global__ void gelu_cast(float* __restrict__ x, void* __restrict__ xa, int64_t n4) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  float4 v = reinterpret_cast<float4*>(x)[i];
  v.x = gelu_f(v.x);
  v.y = gelu_f(v.y);
  v.z = gelu_f(v.z);
  v.w = gelu_f(v.w);
  reinterpret_cast<float4*>(x)[i] = v;
  IO<TO>::st4(xa, i * 4, v);
}

// Fold eval-mode BatchNorm into a conv/linear with out_ch output rows of
// `per` weights each: w[o][...] *= s_o, b_o = (b_o - mean_o) * s_o + beta_o.
void fold_bn(std::vector<float>& w, std::vector<float>& b, int out_ch, int per, const float* cb,
             const float* gamma, const float* beta, const float* mean, const float* var) {
  b.assign(out_ch, 0.f);
  for (int o = 0; o < out_ch; ++o) {
    float bias = cb ? cb[o] : 0.f;
    float s = 1.f;
    if (mean && var) {
      s = 1.0f / sqrtf(var[o] + 1e-5f);
      if (gamma) s *= gamma[o];
      bias = (bias - mean[o]) * s + (beta ? beta[o] : 0.f);
    }
    for (int k = 0; k < per; ++k) w[static_cast<size_t>(o) * per + k] *= s;
    b[o] = bias;
  }
}

int upload(DevBuf& d, const void* h, size_t bytes, cudaStream_t st) {
  if (!d.alloc(bytes)) return kErrNoMem;
  return ck(cudaMemcpyAsync(d.p, h, bytes, cudaMemcpyHostToDevice, st));
}

// f32 host [N, K] -> device 16-bit [N, K]
int upload_w16(DevBuf& d, const float* h, int N, int K, int dt, cudaStream_t st) {
  DevBuf tmp;
  const size_t n = static_cast<size_t>(N) * K;
  int rc = upload(tmp, h, n * 4, st);
  if (rc) return rc;
  if (!d.alloc(n * 2)) return kErrNoMem;
  if ((rc = launch_cast(tmp.p, kF32, d.p, dt, static_cast<int64_t>(n), st))) return rc;
  return ck(cudaStreamSynchronize(st));
}

// Depthwise 3x3 weights [C,3,3,1] (OHWI) with BN folded -> device [9][C].
int upload_dw(DevBuf& w9, DevBuf& bias, int C, const float* w, const float* cb, const float* g, const float* be,
              const float* mean, const float* var, cudaStream_t st) {
  std::vector<float> wf(w, w + static_cast<size_t>(C) * 9), bf;
  fold_bn(wf, bf, C, 9, cb, g, be, mean, var);
  std::vector<float> t(static_cast<size_t>(9) * C);
  for (int c = 0; c < C; ++c)
    for (int k = 0; k < 9; ++k) t[static_cast<size_t>(k) * C + c] = wf[static_cast<size_t>(c) * 9 + k];
  int rc = upload(w9, t.data(), t.size() * 4, st);
  if (rc) return rc;
  if ((rc = upload(bias, bf.data(), bf.size() * 4, st))) return rc;
  return ck(cudaStreamSynchronize(st));
}

EpiParams epi(void* out, int out_type, int ldo, const float* bias) {
  EpiParams e;
  memset(&e, 0, sizeof(e));
  e.out = out;
  e.out_type = out_type;
  e.ldo = ldo;
  e.bias = bias;
  return e;
}

// Grow-only scratch buffer.
int ensure(DevBuf& d, size_t bytes) {
  if (d.p && d.bytes >= bytes) return kOk;
  if (d.p) {
    cudaFree(d.p);
    d.p = nullptr;
  }
  return d.alloc(bytes) ? kOk : kErrNoMem;
}

// A dense conv (OHWI weights [OC, k, k, IC]) with its BatchNorm folded, run
// as (im2col +) GEMM: W 16-bit [OC, kpad], bias f32 [OC].
struct DenseConv {
  int oc = 0, ic = 0, k = 1, stride = 1, pad = 0, kpad = 0;
  DevBuf w, b;
};

int make_dense_conv(DenseConv& cv, const sam3cu_tvit_conv_weights& cw, int oc, int ic, int k, int stride, int pad,
                    int act, cudaStream_t st) {
  if (!cw.w) return kErrShape;
  cv.oc = oc;
  cv.ic = ic;
  cv.k = k;
  cv.stride = stride;
  cv.pad = pad;
  const int kk = k * k * ic;
  cv.kpad = (kk + 7) / 8 * 8;  // 16-byte GEMM rows
  std::vector<float> wf(cw.w, cw.w + static_cast<size_t>(oc) * kk), bf;
  fold_bn(wf, bf, oc, kk, cw.b, cw.bn_w, cw.bn_b, cw.bn_mean, cw.bn_var);
  std::vector<float> wp(static_cast<size_t>(oc) * cv.kpad, 0.f);
  for (int o = 0; o < oc; ++o)
    std::copy(wf.begin() + static_cast<size_t>(o) * kk, wf.begin() + static_cast<size_t>(o + 1) * kk,
              wp.begin() + static_cast<size_t>(o) * cv.kpad);
  int rc = upload_w16(cv.w, wp.data(), oc, cv.kpad, act, st);
  if (!rc) rc = upload(cv.b, bf.data(), bf.size() * 4, st);
  return rc;
}

// Depthwise 3x3 weights + folded BN from the conv-weights struct.
int make_dw_conv(DevBuf& w9, DevBuf& bias, int C, const sam3cu_tvit_conv_weights& cw, cudaStream_t st) {
  if (!cw.w) return kErrShape;
  return upload_dw(w9, bias, C, cw.w, cw.b, cw.bn_w, cw.bn_b, cw.bn_mean, cw.bn_var, st);
}

}  // namespace

struct sam3cu_tvit_block {
  int C = 0, heads = 0, ws = 0, mlp = 0, act = kBF16;
  DevBuf ln1_w, ln1_b, qkv_w, qkv_b, proj_w, proj_b, bias;  // bias [heads, N, bias_ld]
  int bias_ld = 0;
  DevBuf bias_tile;  // N <= 64: per 128-row tile of 128/N windows, block-diagonal
  int bias_tile_ld = 0;
  DevBuf dw_w9, dw_b, ln2_w, ln2_b, fc1_w, fc1_b, fc2_w, fc2_b;
  DevBuf xn, qkv, ao, pr, lc, h;  // scratch
};

struct sam3cu_tvit_mbconv {
  int C = 0, mid = 0, act = kBF16;
  DevBuf w1, b1, dw_w9, dw_b, w3, b3;
  DevBuf xa, h, h2;  // scratch
};

struct sam3cu_tinyvit {
  sam3cu_tinyvit_config c{};
  int act = kBF16, max_batch = 0, grid = 0;
  cudaStream_t stream = nullptr;
  DenseConv pe0, pe1;
  std::vector<sam3cu_tvit_mbconv*> mb;                 // layer 0
  std::vector<std::vector<sam3cu_tvit_block*>> blocks;  // layers >= 1
  struct Merge {
    DenseConv c1, c3;
    DevBuf dw_w9, dw_b;
  } pm[SAM3CU_TVIT_MAX_LAYERS];
  DenseConv head1, head2;
  DevBuf img, out, a, x, xa, col, h, h2;  // staging and scratch
  ~sam3cu_tinyvit() {
    for (auto* m : mb) sam3cu_tvit_mbconv_destroy(m);
    for (auto& l : blocks)
      for (auto* b : l) sam3cu_tvit_block_destroy(b);
    if (stream) {
      cudaStreamSynchronize(stream);
      cudaStreamDestroy(stream);
    }
  }
};

extern "C" {

int sam3cu_tvit_expand_bias(const float* compact, int heads, int n_offsets, int ws, float* out, int out_ld) {
  if (!compact || !out || heads <= 0 || ws <= 0 || ws > 64) return SAM3CU_EINVAL;
  const int n = ws * ws;
  if (out_ld < n) return SAM3CU_EINVAL;
  // offset (|dy|, |dx|) -> index, numbered in the order the position pairs
  // (p1 row-major, then p2 row-major) first meet it
  std::vector<int> index(static_cast<size_t>(n), -1);
  int count = 0;
  for (int p1 = 0; p1 < n; ++p1)
    for (int p2 = 0; p2 < n; ++p2) {
      const int key = std::abs(p1 / ws - p2 / ws) * ws + std::abs(p1 % ws - p2 % ws);
      if (index[key] < 0) index[key] = count++;
    }
  if (count != n_offsets) return SAM3CU_EINVAL;
  for (int h = 0; h < heads; ++h)
    for (int p1 = 0; p1 < n; ++p1) {
      float* row = out + (static_cast<size_t>(h) * n + p1) * out_ld;
      for (int p2 = 0; p2 < n; ++p2) {
        const int key = std::abs(p1 / ws - p2 / ws) * ws + std::abs(p1 % ws - p2 % ws);
        row[p2] = compact[static_cast<size_t>(h) * n_offsets + index[key]];
      }
      for (int p2 = n; p2 < out_ld; ++p2) row[p2] = 0.f;
    }
  return SAM3CU_OK;
}

int sam3cu_tvit_window_attention(const void* qkv, int64_t ld_qkv, void* out, int64_t ld_out, int dtype,
                                 int n_windows, int n_tokens, int heads, int head_dim, const float* bias,
                                 int bias_ld, void* stream) {
  if (!qkv || !out || n_windows < 0 || n_tokens < 0 || heads <= 0) return SAM3CU_EINVAL;
  if (dtype != SAM3CU_BF16 && dtype != SAM3CU_F16) return SAM3CU_EDTYPE;
  if (ld_qkv < 3LL * heads * head_dim || ld_out < static_cast<int64_t>(heads) * head_dim) return SAM3CU_EINVAL;
  const size_t es = 2;
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.q = qkv;
  a.k = static_cast<const uint8_t*>(qkv) + head_dim * es;
  a.v = static_cast<const uint8_t*>(qkv) + 2 * head_dim * es;
  a.ldq = ld_qkv;
  a.in_hstride = 3 * head_dim;
  a.o = out;
  a.ldo = ld_out;
  a.o_hstride = head_dim;
  a.dtype = dtype;
  a.n_groups = n_windows;
  a.seq = n_tokens;
  a.heads = heads;
  a.head_dim = head_dim;
  a.bias = bias;
  a.bias_ld = bias_ld;
  a.scale = 0.f;  // 1/sqrt(head_dim), applied to the scores (the reference scales q)
  return launch_attention_tc_ex(a, as_stream(stream));
}

sam3cu_tvit_block* sam3cu_tvit_block_create(int dim, int heads, int ws, int mlp_dim, int dtype,
                                            const struct sam3cu_tvit_block_weights* w, int* status) {
  int rc = SAM3CU_OK;
  auto fail = [&](int r) -> sam3cu_tvit_block* {
    if (status) *status = r;
    return nullptr;
  };
  if (!w || dim <= 0 || heads <= 0 || dim % heads || ws <= 0 || ws > 16 || mlp_dim <= 0) return fail(SAM3CU_EINVAL);
  if (dtype != SAM3CU_BF16 && dtype != SAM3CU_F16) return fail(SAM3CU_EDTYPE);
  const int hd = dim / heads;
  if ((hd != 32 && hd != 64) || dim % 32 || mlp_dim % 8) return fail(SAM3CU_EINVAL);
  if (!w->qkv_w || !w->proj_w || !w->lc_w || !w->fc1_w || !w->fc2_w) return fail(SAM3CU_EINVAL);
  auto* b = new sam3cu_tvit_block();
  b->C = dim;
  b->heads = heads;
  b->ws = ws;
  b->mlp = mlp_dim;
  b->act = dtype == SAM3CU_F16 ? kF16 : kBF16;
  cudaStream_t st = nullptr;
  const int C = dim, N = ws * ws;
  auto vec = [&](DevBuf& d, const float* h, int n) {  // optional f32 vector (nullptr -> null buffer)
    if (!h || rc) return;
    rc = upload(d, h, static_cast<size_t>(n) * 4, st);
  };
  vec(b->ln1_w, w->attn_norm_w, C);
  vec(b->ln1_b, w->attn_norm_b, C);
  vec(b->qkv_b, w->qkv_b, 3 * C);
  vec(b->proj_b, w->proj_b, C);
  vec(b->ln2_w, w->mlp_norm_w, C);
  vec(b->ln2_b, w->mlp_norm_b, C);
  vec(b->fc1_b, w->fc1_b, mlp_dim);
  vec(b->fc2_b, w->fc2_b, C);
  if (!rc) rc = upload_w16(b->qkv_w, w->qkv_w, 3 * C, C, b->act, st);
  if (!rc) rc = upload_w16(b->proj_w, w->proj_w, C, C, b->act, st);
  if (!rc) rc = upload_w16(b->fc1_w, w->fc1_w, mlp_dim, C, b->act, st);
  if (!rc) rc = upload_w16(b->fc2_w, w->fc2_w, C, mlp_dim, b->act, st);
  if (!rc) rc = upload_dw(b->dw_w9, b->dw_b, C, w->lc_w, w->lc_b, w->lc_bn_w, w->lc_bn_b, w->lc_bn_mean,
                          w->lc_bn_var, st);
  if (!rc && w->attn_bias) {
    b->bias_ld = (N + 3) / 4 * 4;
    std::vector<float> dense(static_cast<size_t>(heads) * N * b->bias_ld);
    rc = sam3cu_tvit_expand_bias(w->attn_bias, heads, w->attn_bias_offsets, ws, dense.data(), b->bias_ld);
    if (!rc) rc = upload(b->bias, dense.data(), dense.size() * 4, st);
    if (!rc && N <= 64) {  // several windows share one attention tile
      const int G = 128 / N, R = G * N;
      b->bias_tile_ld = (R + 3) / 4 * 4;
      std::vector<float> tile(static_cast<size_t>(heads) * R * b->bias_tile_ld, -INFINITY);
      for (int h = 0; h < heads; ++h)
        for (int i = 0; i < R; ++i)
          for (int j = 0; j < R; ++j)
            if (i / N == j / N)
              tile[(static_cast<size_t>(h) * R + i) * b->bias_tile_ld + j] =
                  dense[(static_cast<size_t>(h) * N + i % N) * b->bias_ld + j % N];
      rc = upload(b->bias_tile, tile.data(), tile.size() * 4, st);
    }
  }
  if (!rc) rc = ck(cudaDeviceSynchronize());
  if (rc) {
    delete b;
    return fail(rc);
  }
  if (status) *status = SAM3CU_OK;
  return b;
}

void sam3cu_tvit_block_destroy(sam3cu_tvit_block* b) { delete b; }

int sam3cu_tvit_block_forward(sam3cu_tvit_block* b, float* x, int n_images, int H, int W, void* stream) {
  if (!b || !x || n_images <= 0 || H <= 0 || W <= 0) return SAM3CU_EINVAL;
  cudaStream_t st = as_stream(stream);
  const int C = b->C, ws = b->ws, N = ws * ws, hd = C / b->heads;
  const int nwy = (H + ws - 1) / ws, nwx = (W + ws - 1) / ws;
  const int64_t per_img = static_cast<int64_t>(nwy) * nwx * N;
  const int64_t Tw = per_img * n_images, Th = static_cast<int64_t>(n_images) * H * W;
  if (Tw > 0x7fffffffLL || Th * b->mlp > (1LL << 40)) return SAM3CU_EINVAL;
  const size_t es = 2;
  int rc;
  if ((rc = ensure(b->xn, static_cast<size_t>(std::max(Tw, Th)) * C * es)) ||
      (rc = ensure(b->qkv, static_cast<size_t>(Tw) * 3 * C * es)) ||
      (rc = ensure(b->ao, static_cast<size_t>(Tw) * C * es)) || (rc = ensure(b->pr, static_cast<size_t>(Tw) * C * 4)) ||
      (rc = ensure(b->lc, static_cast<size_t>(Th) * C * 4)) ||
      (rc = ensure(b->h, static_cast<size_t>(Th) * b->mlp * es)))
    return rc;
  WinMap m{H, W, ws, nwx, N, static_cast<int>(per_img)};
  // window attention half (tvit_window_attention inside tvit_block_forward)
  if ((rc = launch_ln_tvit(x, b->xn.p, b->act, b->ln1_w.as<float>(), b->ln1_b.as<float>(), Tw, C, &m, st)))
    return rc;
  EpiParams e = epi(b->qkv.p, b->act, 3 * C, b->qkv_b.as<float>());
  if ((rc = launch_gemm(b->xn.p, C, b->qkv_w.p, C, nullptr, nullptr, b->act, GemmShape{static_cast<int>(Tw), 3 * C, C},
                        e, st, 0)))
    return rc;
  {
    AttnArgs a;
    memset(&a, 0, sizeof(a));
    a.q = b->qkv.p;
    a.k = b->qkv.as<uint8_t>() + hd * es;
    a.v = b->qkv.as<uint8_t>() + 2 * hd * es;
    a.ldq = 3 * C;
    a.in_hstride = 3 * hd;
    a.o = b->ao.p;
    a.ldo = C;
    a.o_hstride = hd;
    a.dtype = b->act;
    a.n_groups = static_cast<int>(Tw / N);
    a.seq = N;
    a.heads = b->heads;
    a.head_dim = hd;
    a.bias = b->bias.as<float>();
    a.bias_ld = b->bias_ld;
    a.bias_tile = b->bias_tile.as<float>();
    a.bias_tile_ld = b->bias_tile_ld;
    if ((rc = launch_attention_tc_ex(a, st))) return rc;
  }
  e = epi(b->pr.p, kOutF32, C, b->proj_b.as<float>());
  if ((rc = launch_gemm(b->ao.p, C, b->proj_w.p, C, nullptr, nullptr, b->act, GemmShape{static_cast<int>(Tw), C, C},
                        e, st, 0)))
    return rc;
  if (Tw * (C / 4) >= (1LL << 31)) return SAM3CU_EINVAL;
  count_launches(1);
  unpartition_add<<<grid_1d(Tw * (C / 4), 256), 256, 0, st>>>(x, b->pr.as<float>(), Tw, C, m);
  if ((rc = ck(cudaGetLastError()))) return kErrLaunch;
  // local conv (3x3 depthwise + BN) and the MLP
  if ((rc = launch_dwconv3x3(x, kF32, b->lc.p, kF32, b->dw_w9.as<float>(), b->dw_b.as<float>(), n_images, H, W, C,
                             false, st)))
    return rc;
  if ((rc = launch_ln_tvit(b->lc.as<float>(), b->xn.p, b->act, b->ln2_w.as<float>(), b->ln2_b.as<float>(), Th, C,
                           nullptr, st)))
    return rc;
  e = epi(b->h.p, b->act, b->mlp, b->fc1_b.as<float>());
  e.act = 1;
  if ((rc = launch_gemm(b->xn.p, C, b->fc1_w.p, C, nullptr, nullptr, b->act,
                        GemmShape{static_cast<int>(Th), b->mlp, C}, e, st, 0)))
    return rc;
  e = epi(x, kOutF32, C, b->fc2_b.as<float>());
  e.residual = b->lc.as<float>();
  e.ldr = C;
  return launch_gemm(b->h.p, b->mlp, b->fc2_w.p, b->mlp, nullptr, nullptr, b->act,
                     GemmShape{static_cast<int>(Th), C, b->mlp}, e, st, 0);
}

sam3cu_tvit_mbconv* sam3cu_tvit_mbconv_create(int dim, int mid_dim, int dtype,
                                              const struct sam3cu_tvit_mbconv_weights* w, int* status) {
  auto fail = [&](int r) -> sam3cu_tvit_mbconv* {
    if (status) *status = r;
    return nullptr;
  };
  if (!w || dim <= 0 || mid_dim <= 0 || dim % 8 || mid_dim % 8) return fail(SAM3CU_EINVAL);
  if (!w->conv1_w || !w->conv2_w || !w->conv3_w) return fail(SAM3CU_EINVAL);
  if (dtype != SAM3CU_BF16 && dtype != SAM3CU_F16) return fail(SAM3CU_EDTYPE);
  auto* m = new sam3cu_tvit_mbconv();
  m->C = dim;
  m->mid = mid_dim;
  m->act = dtype == SAM3CU_F16 ? kF16 : kBF16;
  cudaStream_t st = nullptr;
  int rc = kOk;
  std::vector<float> wf, bf;
  // conv1 1x1 [mid, 1, 1, C] == linear [mid, C]; conv3 [C, 1, 1, mid]
  wf.assign(w->conv1_w, w->conv1_w + static_cast<size_t>(mid_dim) * dim);
  fold_bn(wf, bf, mid_dim, dim, w->conv1_b, w->bn1_w, w->bn1_b, w->bn1_mean, w->bn1_var);
  rc = upload_w16(m->w1, wf.data(), mid_dim, dim, m->act, st);
  if (!rc) rc = upload(m->b1, bf.data(), bf.size() * 4, st);
  if (!rc) {
    wf.assign(w->conv3_w, w->conv3_w + static_cast<size_t>(dim) * mid_dim);
    fold_bn(wf, bf, dim, mid_dim, w->conv3_b, w->bn3_w, w->bn3_b, w->bn3_mean, w->bn3_var);
    rc = upload_w16(m->w3, wf.data(), dim, mid_dim, m->act, st);
  }
  if (!rc) rc = upload(m->b3, bf.data(), bf.size() * 4, st);
  if (!rc) rc = upload_dw(m->dw_w9, m->dw_b, mid_dim, w->conv2_w, w->conv2_b, w->bn2_w, w->bn2_b, w->bn2_mean,
                          w->bn2_var, st);
  if (!rc) rc = ck(cudaDeviceSynchronize());
  if (rc) {
    delete m;
    return fail(rc);
  }
  if (status) *status = SAM3CU_OK;
  return m;
}

void sam3cu_tvit_mbconv_destroy(sam3cu_tvit_mbconv* m) { delete m; }

int sam3cu_tvit_mbconv_forward(sam3cu_tvit_mbconv* m, float* x, int n_images, int H, int W, void* stream) {
  if (!m || !x || n_images <= 0 || H <= 0 || W <= 0) return SAM3CU_EINVAL;
  cudaStream_t st = as_stream(stream);
  const int64_t Th = static_cast<int64_t>(n_images) * H * W;
  if (Th > 0x7fffffffLL) return SAM3CU_EINVAL;
  const size_t es = 2;
  int rc;
  if ((rc = ensure(m->xa, static_cast<size_t>(Th) * m->C * es)) ||
      (rc = ensure(m->h, static_cast<size_t>(Th) * m->mid * es)) ||
      (rc = ensure(m->h2, static_cast<size_t>(Th) * m->mid * es)))
    return rc;
  const int M = static_cast<int>(Th);
  if ((rc = launch_cast(x, kF32, m->xa.p, m->act, Th * m->C, st))) return rc;
  EpiParams e = epi(m->h.p, m->act, m->mid, m->b1.as<float>());
  e.act = 1;
  if ((rc = launch_gemm(m->xa.p, m->C, m->w1.p, m->C, nullptr, nullptr, m->act, GemmShape{M, m->mid, m->C}, e, st,
                        0)))
    return rc;
  if ((rc = launch_dwconv3x3(m->h.p, m->act, m->h2.p, m->act, m->dw_w9.as<float>(), m->dw_b.as<float>(), n_images,
                             H, W, m->mid, true, st)))
    return rc;
  e = epi(x, kOutF32, m->C, m->b3.as<float>());
  e.residual = x;  // in place: x += conv3(...) (TMA reduce-add)
  e.ldr = m->C;
  if ((rc = launch_gemm(m->h2.p, m->mid, m->w3.p, m->mid, nullptr, nullptr, m->act, GemmShape{M, m->C, m->mid}, e,
                        st, 0)))
    return rc;
  count_launches(1);
  const int64_t n4 = Th * m->C / 4;
  if (m->act == kF16)
    gelu_cast<kF16><<<grid_1d(n4, 256), 256, 0, st>>>(x, m->xa.p, n4);
  else
    gelu_cast<kBF16><<<grid_1d(n4, 256), 256, 0, st>>>(x, m->xa.p, n4);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

namespace {

// y[M, oc] = im2col(x) . W^T + b (optionally GELU), as one GEMM; a 1x1,
// stride-1 conv reads the 16-bit NHWC input directly.
int run_conv(sam3cu_tinyvit* t, const DenseConv& cv, const void* x, int tin, bool chw, int n, int H, int W,
             void* y, int out_type, int act_gelu) {
  const int OH = (H + 2 * cv.pad - cv.k) / cv.stride + 1, OW = (W + 2 * cv.pad - cv.k) / cv.stride + 1;
  const int64_t M = static_cast<int64_t>(n) * OH * OW;
  if (M > 0x7fffffffLL) return kErrShape;
  const void* a = x;
  int rc;
  if (cv.k != 1 || cv.stride != 1 || chw || tin == kF32 || cv.kpad != cv.ic) {
    if ((rc = ensure(t->col, static_cast<size_t>(M) * cv.kpad * 2))) return rc;
    if ((rc = launch_conv_im2col(x, tin, chw, t->col.p, t->act, n, H, W, cv.ic, cv.k, cv.stride, cv.pad, cv.kpad,
                                 t->stream)))
      return rc;
    a = t->col.p;
  }
  EpiParams e = epi(y, out_type, cv.oc, cv.b.as<float>());
  e.act = act_gelu;
  return launch_gemm(a, cv.kpad, cv.w.p, cv.kpad, nullptr, nullptr, t->act, GemmShape{static_cast<int>(M), cv.oc, cv.kpad},
                     e, t->stream, 0);
}

int tinyvit_forward(sam3cu_tinyvit* t, const float* images, int n, float* out) {
  const auto& c = t->c;
  const int S = c.img_size, H1 = (S - 1) / 2 + 1, H2 = (H1 - 1) / 2 + 1;
  const int C0 = c.embed_dims[0];
  int rc;
  // patch embed: 3x3/2 conv + BN + GELU (CHW image read in place), 3x3/2 conv + BN
  if ((rc = ensure(t->a, static_cast<size_t>(n) * H1 * H1 * t->pe0.oc * 2))) return rc;
  if ((rc = run_conv(t, t->pe0, images, kF32, true, n, S, S, t->a.p, t->act, 1))) return rc;
  size_t xmax = static_cast<size_t>(n) * H2 * H2 * C0;
  if ((rc = ensure(t->x, xmax * 4))) return rc;
  if ((rc = run_conv(t, t->pe1, t->a.p, t->act, false, n, H1, H1, t->x.p, kOutF32, 0))) return rc;
  int H = H2, C = C0;
  for (int l = 0; l < c.n_layers; ++l) {
    if (l == 0) {
      for (auto* m : t->mb)
        if ((rc = sam3cu_tvit_mbconv_forward(m, t->x.as<float>(), n, H, H, t->stream))) return rc;
    } else {
      for (auto* b : t->blocks[l])
        if ((rc = sam3cu_tvit_block_forward(b, t->x.as<float>(), n, H, H, t->stream))) return rc;
    }
    if (l == c.n_layers - 1) break;
    // PatchMerging (tvit_patch_merging, :726-750): 1x1 + BN, GELU;
    // 3x3 depthwise stride 2 + BN, GELU; 1x1 + BN
    const auto& pm = t->pm[l];
    const int Cn = c.embed_dims[l + 1], Hn = (H - 1) / 2 + 1;
    const int64_t P = static_cast<int64_t>(n) * H * H, Pn = static_cast<int64_t>(n) * Hn * Hn;
    if ((rc = ensure(t->xa, static_cast<size_t>(P) * C * 2)) || (rc = ensure(t->h, static_cast<size_t>(P) * Cn * 2)) ||
        (rc = ensure(t->h2, static_cast<size_t>(Pn) * Cn * 2)))
      return rc;
    if ((rc = launch_cast(t->x.p, kF32, t->xa.p, t->act, P * C, t->stream))) return rc;
    if ((rc = run_conv(t, pm.c1, t->xa.p, t->act, false, n, H, H, t->h.p, t->act, 1))) return rc;
    if ((rc = launch_dwconv3x3(t->h.p, t->act, t->h2.p, t->act, pm.dw_w9.as<float>(), pm.dw_b.as<float>(), n, H, H,
                               Cn, true, t->stream, 2)))
      return rc;
    if ((rc = ensure(t->x, static_cast<size_t>(Pn) * Cn * 4))) return rc;
    if ((rc = run_conv(t, pm.c3, t->h2.p, t->act, false, n, Hn, Hn, t->x.p, kOutF32, 0))) return rc;
    H = Hn;
    C = Cn;
  }
  // head: 1x1 conv + BN, GELU; 3x3 conv + bias (:1230-1262)
  const int64_t P = static_cast<int64_t>(n) * H * H;
  if ((rc = ensure(t->xa, static_cast<size_t>(P) * C * 2)) ||
      (rc = ensure(t->h, static_cast<size_t>(P) * c.embed_dim * 2)))
    return rc;
  if ((rc = launch_cast(t->x.p, kF32, t->xa.p, t->act, P * C, t->stream))) return rc;
  if ((rc = run_conv(t, t->head1, t->xa.p, t->act, false, n, H, H, t->h.p, t->act, 1))) return rc;
  return run_conv(t, t->head2, t->h.p, t->act, false, n, H, H, out, kOutF32, 0);
}

}  // namespace

sam3cu_tinyvit* sam3cu_tinyvit_create(const struct sam3cu_tinyvit_config* cfg, const struct sam3cu_tinyvit_weights* w,
                                      int dtype, int max_batch, int* status) {
  int dummy;
  int* st_p = status ? status : &dummy;
  auto fail = [&](int r) -> sam3cu_tinyvit* {
    *st_p = r;
    return nullptr;
  };
  if (!cfg || !w || max_batch <= 0 || cfg->n_layers < 2 || cfg->n_layers > SAM3CU_TVIT_MAX_LAYERS ||
      cfg->img_size < 8 || cfg->embed_dim <= 0 || cfg->embed_dim % 8 || cfg->mlp_ratio <= 0)
    return fail(SAM3CU_EINVAL);
  if (dtype != SAM3CU_BF16 && dtype != SAM3CU_F16) return fail(SAM3CU_EDTYPE);
  for (int l = 0; l < cfg->n_layers; ++l)
    if (cfg->embed_dims[l] <= 0 || cfg->embed_dims[l] % 32 || cfg->depths[l] < 0 ||
        (l == 0 ? !w->layers[0].conv_blocks && cfg->depths[0] > 0 : !w->layers[l].blocks && cfg->depths[l] > 0))
      return fail(SAM3CU_EINVAL);
  std::unique_ptr<sam3cu_tinyvit> t(new sam3cu_tinyvit());
  t->c = *cfg;
  t->act = dtype == SAM3CU_F16 ? kF16 : kBF16;
  t->max_batch = max_batch;
  int h = cfg->img_size;
  h = (h - 1) / 2 + 1;
  h = (h - 1) / 2 + 1;
  for (int l = 0; l + 1 < cfg->n_layers; ++l) h = (h - 1) / 2 + 1;
  t->grid = h;
  if (cudaStreamCreateWithFlags(&t->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(SAM3CU_ECUDA);
  cudaStream_t st = t->stream;
  const int C0 = cfg->embed_dims[0], Ch = C0 / 2;  // patch embed: 3 -> C0/2 -> C0
  int rc = make_dense_conv(t->pe0, w->patch_embed_0, Ch, 3, 3, 2, 1, t->act, st);
  if (!rc) rc = make_dense_conv(t->pe1, w->patch_embed_1, C0, Ch, 3, 2, 1, t->act, st);
  for (int b = 0; !rc && b < cfg->depths[0]; ++b) {
    sam3cu_tvit_mbconv* m = sam3cu_tvit_mbconv_create(C0, C0 * cfg->mlp_ratio, dtype, &w->layers[0].conv_blocks[b], &rc);
    if (m) t->mb.push_back(m);
  }
  t->blocks.resize(cfg->n_layers);
  for (int l = 1; !rc && l < cfg->n_layers; ++l)
    for (int b = 0; !rc && b < cfg->depths[l]; ++b) {
      const int C = cfg->embed_dims[l];
      sam3cu_tvit_block* blk = sam3cu_tvit_block_create(C, cfg->num_heads[l], cfg->window_sizes[l],
                                                        C * cfg->mlp_ratio, dtype, &w->layers[l].blocks[b], &rc);
      if (blk) t->blocks[l].push_back(blk);
    }
  for (int l = 0; !rc && l + 1 < cfg->n_layers; ++l) {
    const int C = cfg->embed_dims[l], Cn = cfg->embed_dims[l + 1];
    const auto& lw = w->layers[l];
    rc = make_dense_conv(t->pm[l].c1, lw.pm_conv1, Cn, C, 1, 1, 0, t->act, st);
    if (!rc) rc = make_dw_conv(t->pm[l].dw_w9, t->pm[l].dw_b, Cn, lw.pm_conv2, st);
    if (!rc) rc = make_dense_conv(t->pm[l].c3, lw.pm_conv3, Cn, Cn, 1, 1, 0, t->act, st);
  }
  if (!rc) {
    const int CL = cfg->embed_dims[cfg->n_layers - 1];
    sam3cu_tvit_conv_weights h1 = w->proj_conv1;  // the head's BN is its own struct
    h1.b = nullptr;                               // and its 1x1 conv has no bias (:1239-1241)
    h1.bn_w = w->proj_bn.bn_w;
    h1.bn_b = w->proj_bn.bn_b;
    h1.bn_mean = w->proj_bn.bn_mean;
    h1.bn_var = w->proj_bn.bn_var;
    rc = make_dense_conv(t->head1, h1, cfg->embed_dim, CL, 1, 1, 0, t->act, st);
    if (!rc) rc = make_dense_conv(t->head2, w->proj_conv2, cfg->embed_dim, cfg->embed_dim, 3, 1, 1, t->act, st);
  }
  if (!rc) rc = ck(cudaStreamSynchronize(st));
  if (rc) return fail(rc);
  *st_p = SAM3CU_OK;
  return t.release();
}

int sam3cu_tinyvit_grid(const sam3cu_tinyvit* t) { return t ? t->grid : 0; }

void sam3cu_tinyvit_destroy(sam3cu_tinyvit* t) { delete t; }

int sam3cu_tinyvit_encode(sam3cu_tinyvit* t, const float* images, int n, float* out, int on_device) {
  if (!t || !images || !out || n <= 0 || n > t->max_batch) return SAM3CU_EINVAL;
  const size_t in_bytes = static_cast<size_t>(n) * 3 * t->c.img_size * t->c.img_size * 4;
  const size_t out_bytes = static_cast<size_t>(n) * t->grid * t->grid * t->c.embed_dim * 4;
  int rc;
  if (on_device) {
    rc = tinyvit_forward(t, images, n, out);
  } else {
    if ((rc = ensure(t->img, in_bytes)) || (rc = ensure(t->out, out_bytes))) return rc;
    if (cudaMemcpyAsync(t->img.p, images, in_bytes, cudaMemcpyHostToDevice, t->stream) != cudaSuccess)
      return SAM3CU_ECUDA;
    rc = tinyvit_forward(t, t->img.as<float>(), n, t->out.as<float>());
    if (!rc && cudaMemcpyAsync(out, t->out.p, out_bytes, cudaMemcpyDeviceToHost, t->stream) != cudaSuccess)
      rc = SAM3CU_ECUDA;
  }
  if (cudaStreamSynchronize(t->stream) != cudaSuccess) return SAM3CU_ECUDA;
  return rc;
}

}  // extern "C"
