// sam3cu_internal.h - declarations shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace s3 {

// Library status codes (negative, mirrored in include/sam3cu.h).
enum : int {
  kOk = 0,
  kErrShape = -101,    // unsupported shape / alignment
  kErrTma = -102,      // tensor map creation failed
  kErrLaunch = -103,   // kernel launch failed
  kErrCuda = -104,     // CUDA runtime error
  kErrDevice = -105,   // device-side bounded wait gave up
  kErrDtype = -106,    // unsupported dtype
  kErrNoMem = -107,
};

// Element types: the reference's enum sam3_dtype codes (sam3_types.h:47-54).
enum : int { kF32 = 0, kF16 = 1, kBF16 = 2, kQ8 = 5 };

struct GemmShape;
struct EpiParams;

int num_sms();
// Add `delta` to the library-wide kernel launch counter; returns the new value.
uint64_t count_launches(int64_t delta);
int launch_q8_quantize(const float* src, void* blocks, int64_t n, cudaStream_t st);
unsigned int dev_error_gemm();
unsigned int dev_error_attn();
unsigned int dev_error_misc();
int launch_attention_tc(const void* q, const void* k, const void* v, int64_t ldq, void* o, int64_t ldo, int dtype,
                        int n_groups, int seq, int heads, int head_dim, cudaStream_t st);
// General form of the tcgen05 attention: head_dim 32 or 64, heads at any
// column stride in Q/K/V (in_hstride, e.g. 3*head_dim for a per-head
// interleaved q|k|v layout) and in O (o_hstride), an optional additive f32
// bias [heads, seq, bias_ld] and an explicit scale (<= 0: 1/sqrt(head_dim)).
struct AttnArgs {
  const void *q, *k, *v;
  int64_t ldq;
  int in_hstride;
  void* o;
  int64_t ldo;
  int o_hstride;
  int dtype;
  int n_groups, seq, heads, head_dim;
  const float* bias;
  int bias_ld;
  float scale;
  // optional: for seq <= 64, the bias laid out per 128-row tile of
  // floor(128/seq) groups, [heads, (128/seq)*seq, bias_tile_ld], -inf
  // between different groups; lets short groups share a tile
  const float* bias_tile;
  int bias_tile_ld;
};
int launch_attention_tc_ex(const AttnArgs& a, cudaStream_t st);
unsigned int dev_error_attn_tc();
unsigned int dev_error_gemm2();
int launch_attention(const void* q, const void* k, const void* v, int64_t ldq, void* o, int64_t ldo, int dtype,
                     int n_groups, int seq, int heads, int head_dim, cudaStream_t st);
int launch_gemm(const void* A, int lda, const void* W, int ldw, const int8_t* q8, const float* q8_scales,
                int ab_dtype, GemmShape shp, const EpiParams& ep, cudaStream_t stream, int max_ctas);

}  // namespace s3
