// conv_noalloc.cu - a CONV2D entry point that allocates no device memory.
//
// The backend's CONV2D lowering (cuda_backend.c) allocates a column buffer
// for the im2col step on every call.  Some callers cannot let a library
// allocate: hosts that reserve all device memory up front in their own pool
// (inference servers with a caching allocator, fixed-budget embedded
// deployments) and latency-critical loops, where cudaMalloc / cudaFree would
// synchronise the device or fragment the pool.  This variant keeps its
// column buffer in a file-scope device array instead, sized once for the
// whole process.
//
// Limits and sharing rules:
//   * kScratchBytes (32 MiB) per GPU that loads the library, held until the
//     process exits.  A call whose column buffer (plus padded weight, if the
//     filter size is not a multiple of the vector width) does not fit is
//     rejected with SAM3CU_ESCRATCH.
//   * Every call on a device shares the one array; calls whose kernels can
//     overlap on the GPU (different streams without ordering between them)
//     race on it.  Serialise them on one stream.
//   * The array keeps the previous call's contents; nothing in it needs to
//     start at zero, because im2col writes every element it later reads
//     (padding columns and out-of-image taps included).
//   * Every call looks up the array's device address with
//     cudaGetSymbolAddress for the current device and context (a host-side
//     lookup, no device work), so the address stays right after
//     cudaDeviceReset or under a context other than the primary one.  The
//     first call on a device also loads the module there: make that first
//     call before any stream capture.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <climits>

#include "../../include/sam3cu.h"
#include "sam3cu_internal.h"

namespace {

constexpr size_t kScratchBytes = 32ull << 20;

// Device-side scratch.  In host code this name is only a stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_conv_scratch[kScratchBytes];

// Device address of g_conv_scratch in the current device's current context,
// or nullptr on failure.  Looked up on every call: the address belongs to the
// context that loaded the module, and a cached copy would go stale when that
// context is replaced (cudaDeviceReset, a cuCtxCreate'd context).
void* scratch_for_current_device() {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_conv_scratch);
  if (e != cudaSuccess) {
    int dev = -1;
    cudaGetDevice(&dev);
    fprintf(stderr, "[sam3cu] cudaGetSymbolAddress(conv scratch) failed on device %d: %s\n", dev,
            cudaGetErrorString(e));
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

}  // namespace

extern "C" {

int sam3cu_conv2d_nhwc_noalloc(const void* x, const void* w, const float* bias, void* y, int dtype, int n, int H,
                               int W, int C, int OC, int kh, int kw, int stride, int pad, void* stream) {
  if (!x || !w || !y || n <= 0 || H <= 0 || W <= 0 || C <= 0 || OC <= 0 || kh <= 0 || kw <= 0 || stride <= 0 ||
      pad < 0)
    return SAM3CU_EINVAL;
  if (dtype != SAM3CU_F32 && dtype != SAM3CU_BF16 && dtype != SAM3CU_F16) return SAM3CU_EDTYPE;
  // Sizes in 64-bit arithmetic, range-checked before any is narrowed to int.
  const int64_t OH = (static_cast<int64_t>(H) + 2 * static_cast<int64_t>(pad) - kh) / stride + 1;
  const int64_t OW = (static_cast<int64_t>(W) + 2 * static_cast<int64_t>(pad) - kw) / stride + 1;
  if (OH <= 0 || OW <= 0 || OH > INT_MAX || OW > INT_MAX) return SAM3CU_EINVAL;
  const size_t es = dtype == SAM3CU_F32 ? 4 : 2;
  const int64_t kk = static_cast<int64_t>(kh) * kw * C;
  const int64_t al = dtype == SAM3CU_F32 ? 4 : 8;  // GEMM row pitch: 16 bytes
  const int64_t kpad = (kk + al - 1) / al * al;
  if (kpad > INT_MAX) return SAM3CU_EINVAL;
  const uint64_t rows = static_cast<uint64_t>(n) * static_cast<uint64_t>(OH) * static_cast<uint64_t>(OW);
  if (rows > 0x7fffffffull) return SAM3CU_EINVAL;
  const uint64_t col_bytes = (rows * static_cast<uint64_t>(kpad) * es + 255) & ~static_cast<uint64_t>(255);
  const uint64_t wpad_bytes = kpad != kk ? static_cast<uint64_t>(OC) * static_cast<uint64_t>(kpad) * es : 0;
  if (col_bytes + wpad_bytes > kScratchBytes) {
    fprintf(stderr,
            "[sam3cu] conv2d_nhwc_noalloc: needs %llu bytes of scratch, the static buffer holds %zu "
            "(split the batch)\n",
            static_cast<unsigned long long>(col_bytes + wpad_bytes), kScratchBytes);
    return SAM3CU_ESCRATCH;
  }
  uint8_t* scratch = static_cast<uint8_t*>(scratch_for_current_device());
  if (!scratch) return SAM3CU_ECUDA;
  void* col = scratch;
  int rc = sam3cu_im2col_nhwc(x, col, dtype, n, H, W, C, kh, kw, stride, pad, static_cast<int>(kpad), stream);
  if (rc) return rc;
  const void* wk = w;
  if (kpad != kk) {  // weight rows [OC, kk] -> [OC, kpad] with zero columns
    void* wpad = scratch + col_bytes;
    rc = sam3cu_im2col_nhwc(w, wpad, dtype, OC, 1, 1, static_cast<int>(kk), 1, 1, 1, 0, static_cast<int>(kpad),
                           stream);
    if (rc) return rc;
    wk = wpad;
  }
  return sam3cu_linear(col, dtype, wk, bias, nullptr, y, dtype, static_cast<int>(rows), static_cast<int>(kpad), OC,
                       SAM3CU_ACT_NONE,
                       stream);
}

}  // extern "C"
