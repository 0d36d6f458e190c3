// selftest.cu - exercises the bounded-wait failure path on the device.
//
// Every mbarrier wait in the library gives up after a time limit, records a
// device error word and lets the kernel return, so a stuck pipeline never
// hangs the GPU and the context stays usable.  This entry point proves that
// path on demand: one CTA waits on an mbarrier that nothing ever arrives on,
// with a short limit, and must come back with the error recorded.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/sam3cu.h"
#include "sam3cu_internal.h"
#include "sm100_ptx.cuh"

namespace s3 {

S3_DEV_ERROR_ACCESSOR(dev_error_selftest)

namespace {

__global__ void wait_never_arrives(unsigned long long limit_ns, int* returned) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  // phase 0 of a fresh barrier with an arrival count of 1: nobody arrives
  const bool completed = mbar_wait_ns(&bar, 0, kErrSelfTest, nullptr, limit_ns);
  if (threadIdx.x == 0) *returned = completed ? 2 : 1;
}

}  // namespace
}  // namespace s3

extern "C" int sam3cu_selftest_wait_timeout(unsigned long long limit_ns, int* timed_out) {
  using namespace s3;
  if (!timed_out) return SAM3CU_EINVAL;
  *timed_out = 0;
  if (limit_ns < 1000000ull) limit_ns = 1000000ull;           // >= 1 ms
  if (limit_ns > kWaitLimitNs) limit_ns = kWaitLimitNs;       // <= the library's own limit
  int* d = nullptr;
  if (cudaMalloc(&d, sizeof(int)) != cudaSuccess) return SAM3CU_ENOMEM;
  int rc = SAM3CU_OK;
  int h = 0;
  cudaMemset(d, 0, sizeof(int));
  count_launches(1);
  wait_never_arrives<<<1, 32>>>(limit_ns, d);
  if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(&h, d, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = SAM3CU_ECUDA;
  cudaFree(d);
  const unsigned err = dev_error_selftest();  // reads and clears the word
  if (rc == SAM3CU_OK) *timed_out = (h == 1 && err == kErrSelfTest) ? 1 : 0;
  return rc;
}
