// devbuf.cuh - an owning device allocation (freed on destruction).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>

namespace s3 {

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  bool alloc(size_t n) {
    bytes = n;
    return cudaMalloc(&p, n ? n : 16) == cudaSuccess;
  }
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

}  // namespace s3
