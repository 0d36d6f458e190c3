// tinyvit.cu - TinyViT hot ops (image_encoder_tinyvit.c) on the B200 path.
//
// sam3cu_tvit_expand_bias        expand_attention_bias (:265-335), host
// sam3cu_tvit_window_attention   tvit_window_attention (:790-866) after the
//                                qkv linear: the reshape / slice / permute
//                                / scale / QK^T / +bias / softmax / .V /
//                                permute-back nodes as one tcgen05 kernel
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/sam3cu.h"
#include "sam3cu_internal.h"

using namespace s3;

namespace {
cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
}  // namespace

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

}  // extern "C"
