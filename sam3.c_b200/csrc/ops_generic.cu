// ops_generic.cu - the remaining graph ops of the encoder path as device
// kernels, for the per-node lowering of the backend vtable (cuda_backend.c):
// permute/transpose, slice, broadcast add, GELU, RoPE, cast, an F32
// attention (with the optional additive mask of SAM3_OP_SDPA), NHWC im2col
// for CONV2D and Q8_0 dequantisation.  Plus the device-memory and stream
// helpers the C11 backend shell calls.  These are HBM-bound elementwise
// kernels; the hot GEMM / attention / LayerNorm work lives in the fused
// kernels.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "../../include/sam3cu.h"
#include "sam3cu_internal.h"

using namespace s3;

namespace {

template <int T>
__device__ __forceinline__ float ld(const void* p, int64_t i) {
  if (T == kF32) return static_cast<const float*>(p)[i];
  if (T == kBF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}
template <int T>
__device__ __forceinline__ void st(void* p, int64_t i, float v) {
  if (T == kF32) static_cast<float*>(p)[i] = v;
  else if (T == kBF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(p)[i] = __float2half_rn(v);
}

int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  const int cap = num_sms() * 16;
  return static_cast<int>(g < 1 ? 1 : (g < cap ? g : cap));
}

int rc_launch() { return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch; }

cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

#define GRID_LOOP(i, n)                                                                   \
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < (n); \
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)

// out[o] = in[src(o)] for a permutation of up to 4 dims (cpu_transpose.c).
template <typename E>
__global__ void permute_kernel(const E* __restrict__ in, E* __restrict__ out, int64_t n, int4 odims, int4 istr) {
  GRID_LOOP(o, n) {
    int64_t r = o;
    const int c3 = static_cast<int>(r % odims.w); r /= odims.w;
    const int c2 = static_cast<int>(r % odims.z); r /= odims.z;
    const int c1 = static_cast<int>(r % odims.y); r /= odims.y;
    const int c0 = static_cast<int>(r);
    out[o] = in[static_cast<int64_t>(c0) * istr.x + static_cast<int64_t>(c1) * istr.y +
                static_cast<int64_t>(c2) * istr.z + static_cast<int64_t>(c3) * istr.w];
  }
}

// Slice along an axis: view as [outer, len, inner] (cpu_slice.c).
template <typename E>
__global__ void slice_kernel(const E* __restrict__ in, E* __restrict__ out, int64_t n, int64_t inner,
                             int64_t len_out, int64_t len_in, int64_t start) {
  GRID_LOOP(o, n) {
    const int64_t i = o % inner, r = o / inner;
    const int64_t k = r % len_out, outer = r / len_out;
    out[o] = in[(outer * len_in + start + k) * inner + i];
  }
}

// out[i] = a[i] + b[i % nb]  (same shape, row [N] broadcast, scalar;
// cpu_elementwise.c:28-62 / :472-495)
template <int T>
__global__ void add_kernel(const void* a, const void* b, void* out, int64_t n, int64_t nb) {
  GRID_LOOP(i, n) st<T>(out, i, ld<T>(a, i) + ld<T>(b, i % nb));
}

// tanh-GELU (cpu_gelu.c:23-36)
template <int T>
__global__ void gelu_kernel(const void* x, void* y, int64_t n) {
  GRID_LOOP(i, n) {
    const float v = ld<T>(x, i);
    const float inner = 0.7978845608f * (v + 0.044715f * v * v * v);
    st<T>(y, i, 0.5f * v * (1.0f + tanhf(inner)));
  }
}

// RoPE on [batch, seq, heads, hd] with F32 [seq, hd/2] tables (cpu_rope.c).
// Row r = (b, s) of heads*hd elements starts at r*ldx in x and r*ldy in y,
// so a column slice of a wider matrix (the Q or K third of the fused QKV
// output) is rotated where it lies.
template <int T>
__global__ void rope_kernel(const void* x, int64_t ldx, const float* __restrict__ cs, const float* __restrict__ sn,
                            void* y, int64_t ldy, int64_t npairs, int seq, int heads, int half) {
  GRID_LOOP(p, npairs) {
    const int d = static_cast<int>(p % half);
    const int64_t bsh = p / half;
    const int64_t row = bsh / heads;
    const int s = static_cast<int>(row % seq);
    const int64_t col = (bsh % heads) * 2 * half + 2 * d;
    const float c = cs[s * half + d], si = sn[s * half + d];
    const float x0 = ld<T>(x, row * ldx + col), x1 = ld<T>(x, row * ldx + col + 1);
    st<T>(y, row * ldy + col, x0 * c - x1 * si);
    st<T>(y, row * ldy + col + 1, x0 * si + x1 * c);
  }
}

template <int TI, int TO>
__global__ void cast_any(const void* x, void* y, int64_t n) {
  GRID_LOOP(i, n) st<TO>(y, i, ld<TI>(x, i));
}

// NHWC im2col for CONV2D with OHWI weights (cpu_conv2d.c): row (n, oy, ox),
// column (ky, kx, c), zero padding, K padded with zeros to kpad.
template <int T>
__global__ void im2col_nhwc(const void* x, void* a, int64_t n, int H, int W, int C, int kh, int kw, int stride,
                            int pad, int OH, int OW, int kpad) {
  GRID_LOOP(i, n) {
    const int kcol = static_cast<int>(i % kpad);
    const int64_t row = i / kpad;
    const int ox = static_cast<int>(row % OW);
    const int oy = static_cast<int>((row / OW) % OH);
    const int64_t b = row / (static_cast<int64_t>(OW) * OH);
    float val = 0.f;
    if (kcol < kh * kw * C) {
      const int c = kcol % C, kx = (kcol / C) % kw, ky = kcol / (C * kw);
      const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
      if (iy >= 0 && iy < H && ix >= 0 && ix < W)
        val = ld<T>(x, ((b * H + iy) * W + ix) * C + c);
    }
    st<T>(a, i, val);
  }
}

// Q8_0 blocks -> F32 (quant.c:134-151)
__global__ void q8_dequant_kernel(const uint8_t* __restrict__ blocks, float* __restrict__ out, int64_t n) {
  GRID_LOOP(i, n) {
    const uint8_t* blk = blocks + (i / 32) * 36;
    float s;
    memcpy(&s, blk, 4);
    out[i] = static_cast<float>(static_cast<int8_t>(blk[4 + i % 32])) * s;
  }
}

// elementwise product with trailing-suffix broadcast (cpu_elementwise.c)
template <int T>
__global__ void mul_kernel(const void* a, const void* b, void* out, int64_t n, int64_t nb) {
  GRID_LOOP(i, n) st<T>(out, i, ld<T>(a, i) * ld<T>(b, i % nb));
}

// Row softmax, one warp per row (cpu_softmax.c:29-47: max, expf(x - max),
// sum, times 1/sum), f32 arithmetic.
template <int T>
__global__ void softmax_rows(const void* x, void* y, int64_t rows, int cols) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t base = row * cols;
  float mx = -FLT_MAX;
  for (int c = lane; c < cols; c += 32) mx = fmaxf(mx, ld<T>(x, base + c));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int c = lane; c < cols; c += 32) sum += expf(ld<T>(x, base + c) - mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.0f / sum;
  for (int c = lane; c < cols; c += 32) st<T>(y, base + c, expf(ld<T>(x, base + c) - mx) * inv);
}

// Batched C[b] = A[b] [M,K] . B[b] [K,N], f32 accumulation in k order,
// 16x16 tiles through shared memory (the 4-D MATMUL of TinyViT's window
// attention; the encoder's large GEMMs use the tcgen05 kernels instead).
template <int T>
__global__ void bmm_kernel(const void* a, const void* b, void* c, int M, int K, int N) {
  __shared__ float as[16][17], bs[16][17];
  const int bz = blockIdx.z;
  const int row = blockIdx.y * 16 + threadIdx.y, col = blockIdx.x * 16 + threadIdx.x;
  const int64_t ao = static_cast<int64_t>(bz) * M * K, bo = static_cast<int64_t>(bz) * K * N;
  float acc = 0.f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    const int ka = k0 + threadIdx.x, kb = k0 + threadIdx.y;
    as[threadIdx.y][threadIdx.x] = (row < M && ka < K) ? ld<T>(a, ao + static_cast<int64_t>(row) * K + ka) : 0.f;
    bs[threadIdx.y][threadIdx.x] = (kb < K && col < N) ? ld<T>(b, bo + static_cast<int64_t>(kb) * N + col) : 0.f;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) acc += as[threadIdx.y][k] * bs[k][threadIdx.x];
    __syncthreads();
  }
  if (row < M && col < N) st<T>(c, static_cast<int64_t>(bz) * M * N + static_cast<int64_t>(row) * N + col, acc);
}

// Eval BatchNorm over the last dim (cpu_batchnorm.c: inv_std = 1/sqrtf(var
// + 1e-5), (x - mean) * inv_std * gamma + beta; gamma / beta optional).
template <int T>
__global__ void batchnorm_kernel(const void* x, void* y, int64_t n, int C, const float* __restrict__ g,
                                 const float* __restrict__ b, const float* __restrict__ mean,
                                 const float* __restrict__ var) {
  GRID_LOOP(i, n) {
    const int c = static_cast<int>(i % C);
    float v = (ld<T>(x, i) - mean[c]) * (1.0f / sqrtf(var[c] + 1e-5f));
    if (g) v *= g[c];
    if (b) v += b[c];
    st<T>(y, i, v);
  }
}

// Grouped NHWC conv with OHWI weights [OC, KH, KW, C/groups], direct
// (cpu_conv2d.c:320-420 with groups > 1: depthwise convs), f32 accumulation
// over (ky, kx, c).
template <int T>
__global__ void conv2d_grouped(const void* x, const void* w, void* y, int64_t n, int H, int W, int C, int OC, int KH,
                               int KW, int stride, int pad, int OH, int OW, int groups) {
  const int cpg_in = C / groups, cpg_out = OC / groups;
  GRID_LOOP(i, n) {
    const int oc = static_cast<int>(i % OC);
    int64_t p = i / OC;
    const int ox = static_cast<int>(p % OW), oy = static_cast<int>((p / OW) % OH);
    const int64_t b = p / (static_cast<int64_t>(OW) * OH);
    const int g = oc / cpg_out;
    float acc = 0.f;
    for (int ky = 0; ky < KH; ++ky) {
      const int iy = oy * stride - pad + ky;
      if (iy < 0 || iy >= H) continue;
      for (int kx = 0; kx < KW; ++kx) {
        const int ix = ox * stride - pad + kx;
        if (ix < 0 || ix >= W) continue;
        const int64_t xo = ((b * H + iy) * W + ix) * C + g * cpg_in;
        const int64_t wo = ((static_cast<int64_t>(oc) * KH + ky) * KW + kx) * cpg_in;
        for (int c = 0; c < cpg_in; ++c) acc += ld<T>(x, xo + c) * ld<T>(w, wo + c);
      }
    }
    st<T>(y, i, acc);
  }
}

// Direct transposed conv, NHWC x OHWI [OC, KH, KW, C] (cpu_conv_transpose2d.c:
// output (oh, ow) gathers input (ih, iw) with oh + pad - kh = ih * stride),
// f32 accumulation.
template <int T>
__global__ void conv_transpose2d_direct(const void* x, const void* w, void* y, int64_t n, int H, int W, int C,
                                        int OC, int KH, int KW, int stride, int pad, int OH, int OW) {
  GRID_LOOP(i, n) {
    const int oc = static_cast<int>(i % OC);
    int64_t p = i / OC;
    const int ow = static_cast<int>(p % OW), oh = static_cast<int>((p / OW) % OH);
    const int64_t b = p / (static_cast<int64_t>(OW) * OH);
    float acc = 0.f;
    for (int kh = 0; kh < KH; ++kh) {
      const int ho = oh + pad - kh;
      if (ho < 0 || ho % stride) continue;
      const int ih = ho / stride;
      if (ih >= H) continue;
      for (int kw = 0; kw < KW; ++kw) {
        const int wo = ow + pad - kw;
        if (wo < 0 || wo % stride) continue;
        const int iw = wo / stride;
        if (iw >= W) continue;
        const int64_t xo = ((b * H + ih) * W + iw) * C;
        const int64_t wofs = ((static_cast<int64_t>(oc) * KH + kh) * KW + kw) * C;
        for (int c = 0; c < C; ++c) acc += ld<T>(x, xo + c) * ld<T>(w, wofs + c);
      }
    }
    st<T>(y, i, acc);
  }
}

// y[b, h*k + ky, w*k + kx, oc] = g[(b, h, w), (ky*k + kx)*OC + oc]: the
// pixel shuffle after a stride-k, kernel-k transposed conv run as one GEMM.
template <typename E>
__global__ void convt_shuffle(const E* __restrict__ g, E* __restrict__ y, int64_t n, int H, int W, int k, int OC) {
  GRID_LOOP(i, n) {
    const int oc = static_cast<int>(i % OC);
    int64_t p = i / OC;
    const int OW = W * k, OH = H * k;
    const int ox = static_cast<int>(p % OW), oy = static_cast<int>((p / OW) % OH);
    const int64_t b = p / (static_cast<int64_t>(OW) * OH);
    const int hh = oy / k, ky = oy % k, ww = ox / k, kx = ox % k;
    y[i] = g[((b * H + hh) * W + ww) * static_cast<int64_t>(k * k * OC) + (ky * k + kx) * OC + oc];
  }
}

// NHWC max pool, kernel k, stride s, no padding (cpu_maxpool2d.c).
template <int T>
__global__ void maxpool_nhwc(const void* x, void* y, int64_t n, int H, int W, int C, int k, int s, int OH, int OW) {
  GRID_LOOP(i, n) {
    const int c = static_cast<int>(i % C);
    int64_t p = i / C;
    const int ox = static_cast<int>(p % OW), oy = static_cast<int>((p / OW) % OH);
    const int64_t b = p / (static_cast<int64_t>(OW) * OH);
    float m = -FLT_MAX;
    for (int ky = 0; ky < k; ++ky)
      for (int kx = 0; kx < k; ++kx) {
        const int iy = oy * s + ky, ix = ox * s + kx;
        if (iy < H && ix < W) m = fmaxf(m, ld<T>(x, ((b * H + iy) * W + ix) * C + c));
      }
    st<T>(y, i, m);
  }
}

}  // namespace

extern "C" {

int sam3cu_dev_alloc(void** p, size_t bytes) {
  return cudaMalloc(p, bytes ? bytes : 16) == cudaSuccess ? SAM3CU_OK : SAM3CU_ENOMEM;
}
int sam3cu_dev_free(void* p) { return cudaFree(p) == cudaSuccess ? SAM3CU_OK : SAM3CU_ECUDA; }
int sam3cu_stream_create(void** s) {
  cudaStream_t st;
  if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return SAM3CU_ECUDA;
  *s = st;
  return SAM3CU_OK;
}
int sam3cu_stream_destroy(void* s) { return cudaStreamDestroy(S(s)) == cudaSuccess ? SAM3CU_OK : SAM3CU_ECUDA; }
int sam3cu_stream_sync(void* s) { return cudaStreamSynchronize(S(s)) == cudaSuccess ? SAM3CU_OK : SAM3CU_ECUDA; }
int sam3cu_host_alloc_pinned(void** p, size_t bytes) {
  return cudaMallocHost(p, bytes ? bytes : 16) == cudaSuccess ? SAM3CU_OK : SAM3CU_ENOMEM;
}
int sam3cu_host_free_pinned(void* p) { return cudaFreeHost(p) == cudaSuccess ? SAM3CU_OK : SAM3CU_ECUDA; }
int sam3cu_event_create(void** e) {
  cudaEvent_t ev;
  if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return SAM3CU_ECUDA;
  *e = ev;
  return SAM3CU_OK;
}
int sam3cu_event_destroy(void* e) { return cudaEventDestroy(static_cast<cudaEvent_t>(e)) == cudaSuccess ? SAM3CU_OK : SAM3CU_ECUDA; }
int sam3cu_event_record(void* e, void* s) {
  return cudaEventRecord(static_cast<cudaEvent_t>(e), S(s)) == cudaSuccess ? SAM3CU_OK : SAM3CU_ECUDA;
}
int sam3cu_event_sync(void* e) { return cudaEventSynchronize(static_cast<cudaEvent_t>(e)) == cudaSuccess ? SAM3CU_OK : SAM3CU_ECUDA; }
int sam3cu_memcpy_h2d(void* dst, const void* src, size_t n, void* s) {
  return cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, S(s)) == cudaSuccess ? SAM3CU_OK : SAM3CU_ECUDA;
}
int sam3cu_memcpy_d2h(void* dst, const void* src, size_t n, void* s) {
  return cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, S(s)) == cudaSuccess ? SAM3CU_OK : SAM3CU_ECUDA;
}
int sam3cu_memcpy_d2d(void* dst, const void* src, size_t n, void* s) {
  return cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToDevice, S(s)) == cudaSuccess ? SAM3CU_OK : SAM3CU_ECUDA;
}

int sam3cu_gather_strided(const void* src, void* dst, int elem_size, int n_dims, const int* dims,
                          const int64_t* strides, void* stream) {
  if (!src || !dst || n_dims < 1 || n_dims > 4) return SAM3CU_EINVAL;
  int d[4] = {1, 1, 1, 1};
  int64_t st[4] = {0, 0, 0, 0};
  const int off = 4 - n_dims;
  for (int i = 0; i < n_dims; ++i) {
    if (dims[i] <= 0 || strides[i] < 0 || strides[i] >= (1ll << 31)) return SAM3CU_ESHAPE;
    d[off + i] = dims[i];
    st[off + i] = strides[i];
  }
  const int64_t n = static_cast<int64_t>(d[0]) * d[1] * d[2] * d[3];
  if (n >= (1ll << 31)) return SAM3CU_ESHAPE;
  int4 odims = make_int4(d[0], d[1], d[2], d[3]);
  int4 istr = make_int4(static_cast<int>(st[0]), static_cast<int>(st[1]), static_cast<int>(st[2]),
                        static_cast<int>(st[3]));
  count_launches(1);
  const int g = grid_for(n, 256);
  if (elem_size == 4) permute_kernel<uint32_t><<<g, 256, 0, S(stream)>>>(static_cast<const uint32_t*>(src), static_cast<uint32_t*>(dst), n, odims, istr);
  else if (elem_size == 2) permute_kernel<uint16_t><<<g, 256, 0, S(stream)>>>(static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), n, odims, istr);
  else if (elem_size == 1) permute_kernel<uint8_t><<<g, 256, 0, S(stream)>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), n, odims, istr);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_permute(const void* src, void* dst, int elem_size, int n_dims, const int* dims, const int* perm,
                   void* stream) {
  if (!src || !dst || n_dims < 1 || n_dims > 4) return SAM3CU_EINVAL;
  int d[4] = {1, 1, 1, 1}, p[4] = {0, 1, 2, 3};
  const int off = 4 - n_dims;
  for (int i = 0; i < n_dims; ++i) {
    d[off + i] = dims[i];
    if (perm[i] < 0 || perm[i] >= n_dims) return SAM3CU_EINVAL;
    p[off + i] = perm[i] + off;
  }
  int64_t istride[4];
  istride[3] = 1;
  for (int i = 2; i >= 0; --i) istride[i] = istride[i + 1] * d[i + 1];
  int4 odims = make_int4(d[p[0]], d[p[1]], d[p[2]], d[p[3]]);
  int4 istr = make_int4(static_cast<int>(istride[p[0]]), static_cast<int>(istride[p[1]]),
                        static_cast<int>(istride[p[2]]), static_cast<int>(istride[p[3]]));
  const int64_t n = static_cast<int64_t>(d[0]) * d[1] * d[2] * d[3];
  if (n >= (1ll << 31)) return SAM3CU_ESHAPE;
  count_launches(1);
  const int g = grid_for(n, 256);
  if (elem_size == 4) permute_kernel<uint32_t><<<g, 256, 0, S(stream)>>>(static_cast<const uint32_t*>(src), static_cast<uint32_t*>(dst), n, odims, istr);
  else if (elem_size == 2) permute_kernel<uint16_t><<<g, 256, 0, S(stream)>>>(static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), n, odims, istr);
  else if (elem_size == 1) permute_kernel<uint8_t><<<g, 256, 0, S(stream)>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), n, odims, istr);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_slice(const void* src, void* dst, int elem_size, int n_dims, const int* dims, int axis, int start,
                 int end, void* stream) {
  if (!src || !dst || n_dims < 1 || n_dims > 4 || axis < 0 || axis >= n_dims) return SAM3CU_EINVAL;
  if (start < 0 || end > dims[axis] || start >= end) return SAM3CU_EINVAL;
  int64_t inner = 1, outer = 1;
  for (int i = axis + 1; i < n_dims; ++i) inner *= dims[i];
  for (int i = 0; i < axis; ++i) outer *= dims[i];
  const int64_t n = outer * (end - start) * inner;
  count_launches(1);
  const int g = grid_for(n, 256);
  if (elem_size == 4) slice_kernel<uint32_t><<<g, 256, 0, S(stream)>>>(static_cast<const uint32_t*>(src), static_cast<uint32_t*>(dst), n, inner, end - start, dims[axis], start);
  else if (elem_size == 2) slice_kernel<uint16_t><<<g, 256, 0, S(stream)>>>(static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), n, inner, end - start, dims[axis], start);
  else if (elem_size == 1) slice_kernel<uint8_t><<<g, 256, 0, S(stream)>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), n, inner, end - start, dims[axis], start);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_add(const void* a, const void* b, void* out, int dtype, int64_t n, int64_t nb, void* stream) {
  if (!a || !b || !out || n < 0 || nb <= 0 || n % nb) return SAM3CU_EINVAL;
  if (n == 0) return SAM3CU_OK;
  count_launches(1);
  const int g = grid_for(n, 256);
  if (dtype == kF32) add_kernel<kF32><<<g, 256, 0, S(stream)>>>(a, b, out, n, nb);
  else if (dtype == kBF16) add_kernel<kBF16><<<g, 256, 0, S(stream)>>>(a, b, out, n, nb);
  else if (dtype == kF16) add_kernel<kF16><<<g, 256, 0, S(stream)>>>(a, b, out, n, nb);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_gelu(const void* x, void* y, int dtype, int64_t n, void* stream) {
  if (!x || !y || n < 0) return SAM3CU_EINVAL;
  if (n == 0) return SAM3CU_OK;
  count_launches(1);
  const int g = grid_for(n, 256);
  if (dtype == kF32) gelu_kernel<kF32><<<g, 256, 0, S(stream)>>>(x, y, n);
  else if (dtype == kBF16) gelu_kernel<kBF16><<<g, 256, 0, S(stream)>>>(x, y, n);
  else if (dtype == kF16) gelu_kernel<kF16><<<g, 256, 0, S(stream)>>>(x, y, n);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_rope_rows(const void* x, int64_t ldx, const float* cos_t, const float* sin_t, void* y, int64_t ldy,
                     int dtype, int batch, int seq, int heads, int hd, void* stream) {
  if (!x || !y || !cos_t || !sin_t || hd % 2 || batch <= 0 || seq <= 0 || heads <= 0) return SAM3CU_EINVAL;
  if (ldx < static_cast<int64_t>(heads) * hd || ldy < static_cast<int64_t>(heads) * hd) return SAM3CU_EINVAL;
  const int64_t np = static_cast<int64_t>(batch) * seq * heads * (hd / 2);
  count_launches(1);
  const int g = grid_for(np, 256);
  cudaStream_t st = S(stream);
  if (dtype == kF32) rope_kernel<kF32><<<g, 256, 0, st>>>(x, ldx, cos_t, sin_t, y, ldy, np, seq, heads, hd / 2);
  else if (dtype == kBF16) rope_kernel<kBF16><<<g, 256, 0, st>>>(x, ldx, cos_t, sin_t, y, ldy, np, seq, heads, hd / 2);
  else if (dtype == kF16) rope_kernel<kF16><<<g, 256, 0, st>>>(x, ldx, cos_t, sin_t, y, ldy, np, seq, heads, hd / 2);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_rope(const void* x, const float* cos_t, const float* sin_t, void* y, int dtype, int batch, int seq,
                int heads, int hd, void* stream) {
  const int64_t ld = static_cast<int64_t>(heads) * hd;
  return sam3cu_rope_rows(x, ld, cos_t, sin_t, y, ld, dtype, batch, seq, heads, hd, stream);
}

int sam3cu_cast(const void* x, int xdt, void* y, int ydt, int64_t n, void* stream) {
  if (!x || !y || n < 0) return SAM3CU_EINVAL;
  if (n == 0) return SAM3CU_OK;
  count_launches(1);
  const int g = grid_for(n, 256);
#define S3_C(A, B) if (xdt == A && ydt == B) { cast_any<A, B><<<g, 256, 0, S(stream)>>>(x, y, n); return rc_launch(); }
  S3_C(kF32, kF32) S3_C(kF32, kBF16) S3_C(kF32, kF16) S3_C(kBF16, kF32) S3_C(kBF16, kBF16) S3_C(kBF16, kF16)
  S3_C(kF16, kF32) S3_C(kF16, kBF16) S3_C(kF16, kF16)
#undef S3_C
  return SAM3CU_EDTYPE;
}


int sam3cu_im2col_nhwc(const void* x, void* a, int dtype, int n, int H, int W, int C, int kh, int kw, int stride,
                       int pad, int kpad, void* stream) {
  if (!x || !a || stride <= 0 || kh <= 0 || kw <= 0 || kpad < kh * kw * C) return SAM3CU_EINVAL;
  const int OH = (H + 2 * pad - kh) / stride + 1, OW = (W + 2 * pad - kw) / stride + 1;
  if (OH <= 0 || OW <= 0) return SAM3CU_EINVAL;
  const int64_t total = static_cast<int64_t>(n) * OH * OW * kpad;
  count_launches(1);
  const int g = grid_for(total, 256);
  if (dtype == kF32) im2col_nhwc<kF32><<<g, 256, 0, S(stream)>>>(x, a, total, H, W, C, kh, kw, stride, pad, OH, OW, kpad);
  else if (dtype == kBF16) im2col_nhwc<kBF16><<<g, 256, 0, S(stream)>>>(x, a, total, H, W, C, kh, kw, stride, pad, OH, OW, kpad);
  else if (dtype == kF16) im2col_nhwc<kF16><<<g, 256, 0, S(stream)>>>(x, a, total, H, W, C, kh, kw, stride, pad, OH, OW, kpad);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_q8_dequantize(const void* blocks, float* out, int64_t n, void* stream) {
  if (!blocks || !out || n <= 0) return SAM3CU_EINVAL;
  count_launches(1);
  q8_dequant_kernel<<<grid_for(n, 256), 256, 0, S(stream)>>>(static_cast<const uint8_t*>(blocks), out, n);
  return rc_launch();
}

int sam3cu_mul(const void* a, const void* b, void* out, int dtype, int64_t n, int64_t nb, void* stream) {
  if (!a || !b || !out || n < 0 || nb <= 0 || n % nb) return SAM3CU_EINVAL;
  count_launches(1);
  const int g = grid_for(n, 256);
  if (dtype == kF32) mul_kernel<kF32><<<g, 256, 0, S(stream)>>>(a, b, out, n, nb);
  else if (dtype == kBF16) mul_kernel<kBF16><<<g, 256, 0, S(stream)>>>(a, b, out, n, nb);
  else if (dtype == kF16) mul_kernel<kF16><<<g, 256, 0, S(stream)>>>(a, b, out, n, nb);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_softmax(const void* x, void* y, int dtype, int64_t rows, int cols, void* stream) {
  if (!x || !y || rows < 0 || cols <= 0) return SAM3CU_EINVAL;
  if (!rows) return SAM3CU_OK;
  count_launches(1);
  const unsigned g = static_cast<unsigned>((rows * 32 + 255) / 256);
  if (dtype == kF32) softmax_rows<kF32><<<g, 256, 0, S(stream)>>>(x, y, rows, cols);
  else if (dtype == kBF16) softmax_rows<kBF16><<<g, 256, 0, S(stream)>>>(x, y, rows, cols);
  else if (dtype == kF16) softmax_rows<kF16><<<g, 256, 0, S(stream)>>>(x, y, rows, cols);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_bmm(const void* a, const void* b, void* c, int dtype, int batch, int M, int K, int N, void* stream) {
  if (!a || !b || !c || batch <= 0 || M <= 0 || K <= 0 || N <= 0 || batch > 65535) return SAM3CU_EINVAL;
  count_launches(1);
  const dim3 grid((N + 15) / 16, (M + 15) / 16, batch), block(16, 16);
  if (dtype == kF32) bmm_kernel<kF32><<<grid, block, 0, S(stream)>>>(a, b, c, M, K, N);
  else if (dtype == kBF16) bmm_kernel<kBF16><<<grid, block, 0, S(stream)>>>(a, b, c, M, K, N);
  else if (dtype == kF16) bmm_kernel<kF16><<<grid, block, 0, S(stream)>>>(a, b, c, M, K, N);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_batchnorm(const void* x, void* y, int dtype, int64_t n, int C, const float* gamma, const float* beta,
                     const float* mean, const float* var, void* stream) {
  if (!x || !y || !mean || !var || C <= 0 || n % C) return SAM3CU_EINVAL;
  count_launches(1);
  const int g = grid_for(n, 256);
  if (dtype == kF32) batchnorm_kernel<kF32><<<g, 256, 0, S(stream)>>>(x, y, n, C, gamma, beta, mean, var);
  else if (dtype == kBF16) batchnorm_kernel<kBF16><<<g, 256, 0, S(stream)>>>(x, y, n, C, gamma, beta, mean, var);
  else if (dtype == kF16) batchnorm_kernel<kF16><<<g, 256, 0, S(stream)>>>(x, y, n, C, gamma, beta, mean, var);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_conv2d_grouped_nhwc(const void* x, const void* w, void* y, int dtype, int n, int H, int W, int C, int OC,
                               int KH, int KW, int stride, int pad, int groups, void* stream) {
  if (!x || !w || !y || groups <= 0 || C % groups || OC % groups || stride <= 0) return SAM3CU_EINVAL;
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0) return SAM3CU_EINVAL;
  const int64_t total = static_cast<int64_t>(n) * OH * OW * OC;
  count_launches(1);
  const int g = grid_for(total, 256);
  if (dtype == kF32)
    conv2d_grouped<kF32><<<g, 256, 0, S(stream)>>>(x, w, y, total, H, W, C, OC, KH, KW, stride, pad, OH, OW, groups);
  else if (dtype == kBF16)
    conv2d_grouped<kBF16><<<g, 256, 0, S(stream)>>>(x, w, y, total, H, W, C, OC, KH, KW, stride, pad, OH, OW, groups);
  else if (dtype == kF16)
    conv2d_grouped<kF16><<<g, 256, 0, S(stream)>>>(x, w, y, total, H, W, C, OC, KH, KW, stride, pad, OH, OW, groups);
  else
    return SAM3CU_EDTYPE;
  return rc_launch();
}

int sam3cu_memcpy2d_d2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t rows,
                        void* stream) {
  if (!dst || !src) return SAM3CU_EINVAL;
  if (!rows || !width) return SAM3CU_OK;
  return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, cudaMemcpyDeviceToDevice, S(stream)) ==
                 cudaSuccess
             ? SAM3CU_OK
             : SAM3CU_ECUDA;
}

int sam3cu_conv_transpose2d_nhwc(const void* x, const void* w, void* y, int dtype, int n, int H, int W, int C,
                                  int OC, int KH, int KW, int stride, int pad, void* stream) {
  if (!x || !w || !y || stride <= 0 || pad < 0) return SAM3CU_EINVAL;
  const int OH = (H - 1) * stride - 2 * pad + KH, OW = (W - 1) * stride - 2 * pad + KW;
  if (OH <= 0 || OW <= 0) return SAM3CU_EINVAL;
  const int64_t total = static_cast<int64_t>(n) * OH * OW * OC;
  count_launches(1);
  const int g = grid_for(total, 256);
#define S3_CT(TT)                                                                                        \
  conv_transpose2d_direct<TT><<<g, 256, 0, S(stream)>>>(x, w, y, total, H, W, C, OC, KH, KW, stride, pad, OH, OW)
  if (dtype == kF32) S3_CT(kF32);
  else if (dtype == kBF16) S3_CT(kBF16);
  else if (dtype == kF16) S3_CT(kF16);
  else return SAM3CU_EDTYPE;
#undef S3_CT
  return rc_launch();
}

int sam3cu_convt_shuffle(const void* g, void* y, int elem_size, int n, int H, int W, int k, int OC, void* stream) {
  if (!g || !y || k <= 0 || OC <= 0) return SAM3CU_EINVAL;
  const int64_t total = static_cast<int64_t>(n) * H * k * W * k * OC;
  count_launches(1);
  const int gr = grid_for(total, 256);
  if (elem_size == 4)
    convt_shuffle<float><<<gr, 256, 0, S(stream)>>>(static_cast<const float*>(g), static_cast<float*>(y), total, H, W,
                                                    k, OC);
  else if (elem_size == 2)
    convt_shuffle<uint16_t><<<gr, 256, 0, S(stream)>>>(static_cast<const uint16_t*>(g), static_cast<uint16_t*>(y),
                                                       total, H, W, k, OC);
  else
    return SAM3CU_EINVAL;
  return rc_launch();
}

int sam3cu_maxpool2d_nhwc(const void* x, void* y, int dtype, int n, int H, int W, int C, int k, int s, void* stream) {
  if (!x || !y || k <= 0 || s <= 0) return SAM3CU_EINVAL;
  const int OH = (H - k) / s + 1, OW = (W - k) / s + 1;
  if (OH <= 0 || OW <= 0) return SAM3CU_EINVAL;
  const int64_t total = static_cast<int64_t>(n) * OH * OW * C;
  count_launches(1);
  const int g = grid_for(total, 256);
  if (dtype == kF32) maxpool_nhwc<kF32><<<g, 256, 0, S(stream)>>>(x, y, total, H, W, C, k, s, OH, OW);
  else if (dtype == kBF16) maxpool_nhwc<kBF16><<<g, 256, 0, S(stream)>>>(x, y, total, H, W, C, k, s, OH, OW);
  else if (dtype == kF16) maxpool_nhwc<kF16><<<g, 256, 0, S(stream)>>>(x, y, total, H, W, C, k, s, OH, OW);
  else return SAM3CU_EDTYPE;
  return rc_launch();
}

}  // extern "C"
