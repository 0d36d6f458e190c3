// capi.cu - extern "C" single-op entry points of include/sam3cu.h.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "../../include/sam3cu.h"
#include "gemm_sm100.cuh"
#include "misc.cuh"
#include "sam3cu_internal.h"

using namespace s3;

namespace {

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// The library's own stream-ordered pool for per-call temporaries (the
// 16-bit copies of a Q8_0 weight and of F32 activations): its release
// threshold keeps freed memory mapped, so a steady stream of calls does not
// map and unmap device memory (the default pool returns it at every
// synchronisation).  One pool per device, created on first use.
cudaMemPool_t call_pool() {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!pools[dev]) {
    cudaMemPoolProps props;
    memset(&props, 0, sizeof(props));
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t p = nullptr;
    if (cudaMemPoolCreate(&p, &props) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    uint64_t keep = ~0ull;
    cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
    pools[dev] = p;
  }
  return pools[dev];
}

cudaError_t pool_alloc(void** p, size_t n, cudaStream_t st) {
  cudaMemPool_t pool = call_pool();
  return pool ? cudaMallocFromPoolAsync(p, n, pool, st) : cudaMallocAsync(p, n, st);
}

int linear_common(const void* x, int x_dtype, const void* w, const int8_t* q, const float* sc, const float* bias,
                  const float* residual, void* y, int y_dtype, int M, int K, int N, int act, void* stream) {
  if (!x || !y || (!w && !q) || M < 0 || K <= 0 || N <= 0) return SAM3CU_EINVAL;
  if (x_dtype != SAM3CU_BF16 && x_dtype != SAM3CU_F16 && x_dtype != SAM3CU_F32) return SAM3CU_EDTYPE;
  if (x_dtype == SAM3CU_F32 && q) {
    // F32 activations x Q8_0 weights (cpu_matmul_q8.c:168-235 takes F32 A):
    // A is rounded to BF16 in a stream-ordered buffer inside the call, then
    // the 16-bit path below runs (Q8's own rounding dominates the error)
    if (!x || !y || M < 0 || K <= 0 || N <= 0) return SAM3CU_EINVAL;
    if (M == 0) return SAM3CU_OK;
    cudaStream_t st = as_stream(stream);
    void* xb = nullptr;
    const size_t nb = (static_cast<size_t>(M) * K * 2 + 255) & ~static_cast<size_t>(255);
    if (M >= 2048 && K % 32 == 0 && ((static_cast<int64_t>(M) * K) % 8) == 0) {
      // large M: the activations and the dequantised weight in one buffer,
      // made by one launch, then the 16-bit GEMM
      const size_t nw = static_cast<size_t>(N) * K * 2;
      if (pool_alloc(&xb, nb + nw, st) == cudaSuccess) {
        void* w16 = static_cast<char*>(xb) + nb;
        int rc = launch_q8_prep(static_cast<const float*>(x), xb, static_cast<int64_t>(M) * K, q, sc, w16, N, K,
                                st);
        if (!rc) rc = linear_common(xb, SAM3CU_BF16, w16, nullptr, nullptr, bias, residual, y, y_dtype, M, K, N,
                                    act, stream);
        cudaFreeAsync(xb, st);
        if (rc != kErrShape) return rc;  // misaligned operands: the general path below
        xb = nullptr;
      } else {
        cudaGetLastError();
      }
    }
    if (pool_alloc(&xb, nb, st) != cudaSuccess) {
      cudaGetLastError();
      return SAM3CU_ENOMEM2;
    }
    int rc = sam3cu_cast(x, SAM3CU_F32, xb, SAM3CU_BF16, static_cast<int64_t>(M) * K, stream);
    if (!rc) rc = linear_common(xb, SAM3CU_BF16, w, q, sc, bias, residual, y, y_dtype, M, K, N, act, stream);
    cudaFreeAsync(xb, st);
    return rc;
  }
  if (y_dtype != SAM3CU_F32 && y_dtype != SAM3CU_BF16 && y_dtype != SAM3CU_F16) return SAM3CU_EDTYPE;
  if (act != SAM3CU_ACT_NONE && act != SAM3CU_ACT_GELU_TANH) return SAM3CU_EINVAL;
  if (residual == y && y_dtype != SAM3CU_F32) return SAM3CU_EINVAL;
  EpiParams ep;
  memset(&ep, 0, sizeof(ep));
  ep.out = y;
  ep.out_type = y_dtype;
  ep.ldo = N;
  ep.bias = bias;
  ep.act = act;
  ep.residual = residual;
  ep.ldr = N;
  GemmShape shp{M, N, K};
  cudaStream_t st = as_stream(stream);
  // Large M with Q8 weights: dequantise W once into a stream-ordered 16-bit
  // buffer and run the 16-bit GEMM on it (an in-GEMM dequantiser converts W
  // again for every row tile); small M keeps the in-GEMM path.
  if (q && M >= 2048 && K % 32 == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0) {
    void* w16 = nullptr;
    if (pool_alloc(&w16, static_cast<size_t>(N) * K * 2, st) == cudaSuccess) {
      int rc = launch_q8_dequant_w16(q, sc, w16, N, K, x_dtype == SAM3CU_F16 ? 2 : 0, st);
      if (!rc) rc = launch_gemm(x, K, w16, K, nullptr, nullptr, x_dtype, shp, ep, st, 0);
      cudaFreeAsync(w16, st);
      return rc;
    }
    cudaGetLastError();  // no pool memory: fall through to the in-GEMM dequantiser
  }
  return launch_gemm(x, K, w, K, q, sc, x_dtype, shp, ep, st, 0);
}

}  // namespace

extern "C" {

int sam3cu_init(int device) {
  if (cudaSetDevice(device) != cudaSuccess) return SAM3CU_EBACKEND;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0) return SAM3CU_EBACKEND;  // built for sm_100a only
  return cudaFree(nullptr) == cudaSuccess ? SAM3CU_OK : SAM3CU_EBACKEND;
}

const char* sam3cu_strerror(int s) {
  switch (s) {
    case SAM3CU_OK: return "ok";
    case SAM3CU_EINVAL: return "invalid argument";
    case SAM3CU_ENOMEM: return "out of memory";
    case SAM3CU_EBACKEND: return "backend / device unavailable";
    case SAM3CU_EDTYPE: return "unsupported dtype";
    case SAM3CU_ESHAPE: return "unsupported shape or alignment";
    case SAM3CU_ETMA: return "TMA descriptor creation failed";
    case SAM3CU_ELAUNCH: return "kernel launch failed";
    case SAM3CU_ECUDA: return "CUDA runtime error";
    case SAM3CU_EDEVICE: return "device-side wait timed out";
    case SAM3CU_EDTYPE2: return "unsupported dtype combination";
    case SAM3CU_ENOMEM2: return "device allocation failed";
    case SAM3CU_ESCRATCH: return "request exceeds the fixed static scratch buffer";
    case SAM3CU_EIO: return "I/O error";
    case SAM3CU_EMODEL: return "malformed .sam3 weight file or missing / mis-shaped tensor";
    case SAM3CU_ENOENT: return "tensor not in the weight file";
    default: return "unknown status";
  }
}

unsigned int sam3cu_last_device_error(void) {
  cudaDeviceSynchronize();
  unsigned int a = dev_error_gemm(), b = dev_error_attn(), c = dev_error_misc(), d = dev_error_attn_tc(),
               e = dev_error_gemm2();
  return a ? a : (b ? b : (c ? c : (d ? d : e)));
}

uint64_t sam3cu_launch_count(int reset) {
  uint64_t v = count_launches(0);
  if (reset) count_launches(-static_cast<int64_t>(v));
  return v;
}

int sam3cu_linear(const void* x, int x_dtype, const void* w, const float* bias, const float* residual, void* y,
                  int y_dtype, int M, int K, int N, int act, void* stream) {
  return linear_common(x, x_dtype, w, nullptr, nullptr, bias, residual, y, y_dtype, M, K, N, act, stream);
}

int sam3cu_linear_q8(const void* x, int x_dtype, const int8_t* q, const float* scales, const float* bias,
                     const float* residual, void* y, int y_dtype, int M, int K, int N, int act, void* stream) {
  if (!q || !scales) return SAM3CU_EINVAL;
  return linear_common(x, x_dtype, nullptr, q, scales, bias, residual, y, y_dtype, M, K, N, act, stream);
}

int sam3cu_q8_repack(const void* blocks, int N, int K, int8_t* q, float* scales, void* stream) {
  if (!blocks || !q || !scales || N <= 0 || K <= 0) return SAM3CU_EINVAL;
  return launch_q8_repack(blocks, q, scales, N, K, as_stream(stream));
}

int sam3cu_q8_quantize(const float* src, void* blocks, int64_t n, void* stream) {
  if (!src || !blocks || n <= 0) return SAM3CU_EINVAL;
  return launch_q8_quantize(src, blocks, n, as_stream(stream));
}

int sam3cu_layernorm(const void* x, int x_dtype, const float* gamma, const float* beta, void* y, int y_dtype,
                     int rows, int cols, void* stream) {
  if (!x || !y || rows < 0 || cols <= 0) return SAM3CU_EINVAL;
  if (x != y || x_dtype == y_dtype) {
    // in-place is safe: each warp holds its whole row before writing
  } else {
    return SAM3CU_EINVAL;
  }
  return launch_layernorm(x, x_dtype, y, y_dtype, gamma, beta, rows, cols, nullptr, 0, as_stream(stream));
}

int sam3cu_sdpa(const void* q, const void* k, const void* v, int64_t ld_qkv, void* o, int64_t ld_o, int dtype,
                int n_groups, int seq, int heads, int head_dim, void* stream) {
  if (!q || !k || !v || !o) return SAM3CU_EINVAL;
  if (dtype != SAM3CU_BF16 && dtype != SAM3CU_F16) return SAM3CU_EDTYPE;
  return launch_attention(q, k, v, ld_qkv, o, ld_o, dtype, n_groups, seq, heads, head_dim, as_stream(stream));
}

}  // extern "C"
