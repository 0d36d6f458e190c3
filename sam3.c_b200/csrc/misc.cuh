// misc.cuh - launchers of the HBM-bound helper kernels (misc.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "sam3cu_internal.h"

namespace s3 {

int launch_layernorm(const void* x, int tin, void* y, int tout, const float* g, const float* b, int rows,
                     int cols, const int* out_row_map, int out_row_period, cudaStream_t st);
int launch_patch_im2col(const float* img, void* a, int tout, int n_img, int img_sz, int ps, int kpad,
                        const int* src_of_row, cudaStream_t st);
int launch_gather_rows(const void* src, void* dst, int rows, int row_bytes, const int* map, int period,
                       cudaStream_t st);
int launch_q8_repack(const void* blocks, int8_t* q, float* sc, int N, int K, cudaStream_t st);
int launch_q8_row_shift(float* sc, float* col_scale, int N, int K, cudaStream_t st);
// 16-bit W [N, K] from int8 q [N, K] and scales [K/32, N].  mode: 0 bf16,
// 1 f16 from row-shifted scales (half2 arithmetic), 2 f16 from any scales
int launch_q8_dequant_w16(const int8_t* q, const float* sc, void* w, int N, int K, int mode, cudaStream_t st);
// x F32 [nx] -> xb bf16 and Q8_0 W (int8 [N,K] + scales [K/32,N]) -> w bf16
// [N,K], in one launch (the inputs of an F32 x Q8_0 linear)
int launch_q8_prep(const float* x, void* xb, int64_t nx, const int8_t* q, const float* sc, void* w, int N, int K,
                   cudaStream_t st);
// The same for up to four weights in one launch (one pass over all of them).
struct Q8DequantJob {
  const int8_t* q;
  const float* sc;
  void* w;
  int N, K;
};
struct Q8DequantJobs {
  static constexpr int kMax = 4;
  Q8DequantJob job[kMax];
  int n;
};
int launch_q8_dequant_w16_multi(const Q8DequantJobs& jobs, int mode, cudaStream_t st);
int launch_cast(const void* x, int tin, void* y, int tout, int64_t n, cudaStream_t st);
// im2col of a dense KxK conv (zero padding) into 16-bit columns (row
// (img, oy, ox), column (ky, kx, c), zero-filled to kpad); chw: planar CHW
// input per image, else NHWC; a 16-byte path for 16-bit NHWC, C % 8 == 0
int launch_conv_im2col(const void* x, int tin, bool chw, void* a, int tout, int B, int H, int W, int C, int k,
                       int stride, int pad, int kpad, cudaStream_t st);

// Park the stream for `ns` nanoseconds of device time (measurement runs: the
// host enqueues the launches being timed meanwhile, so no host gap is timed).
int launch_gpu_sleep(unsigned long long ns, cudaStream_t st);

}  // namespace s3
