// gemm_sm100.cuh - persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   Y[M,N] = epilogue( A[M,K] . W[N,K]^T )
//
// This is the whole of sam3.c's `gh_linear` (TRANSPOSE(W) -> MATMUL ->
// ADD(bias), src/model/graph_helpers.c:297-322) plus what the encoder does
// right after it (tanh-GELU, residual ADD, RoPE on Q/K, window un-partition),
// in one kernel.  W is consumed as stored, [N,K] K-major, so the reference's
// per-call weight transpose disappears.
//
// CTA layout (192 threads, 1 CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A and W tiles -> kStages-deep smem ring
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma into TMEM;
//               owns TMEM allocation (2 accumulators x BN fp32 columns)
//   warps 2..    epilogue (8 warps; 4 with Q8 W): tcgen05.ld TMEM ->
//               registers -> fused ops -> HBM.  Warp w reads TMEM lane
//               quarter w % 4 (the hardware restriction) and, with 8 warps,
//               one half of the tile's columns.
// The two TMEM accumulators let the epilogue of tile i overlap the main loop
// of tile i+1.
//
// B operand sources (template kBMode):
//   kBTma16  W is bf16/fp16 [N,K]: loaded by TMA with the 128-byte swizzle.
//   kBQ8     W is Q8_0 repacked as int8 [N,K] + fp32 scales [N,K/32]
//            (same blocks as the reference's sam3_q8_block, quant.h:30-33):
//            TMA brings the int8 tile and scales, four converter warps
//            dequantise (q * scale -> bf16) straight into the swizzled
//            operand layout in shared memory.
//   kBF32    A and W are F32: "3xTF32".  TMA brings 32-wide F32 tiles
//            (128-byte rows, same swizzle), four converter warps split
//            every element x in place into hi = x with the low 13 mantissa
//            bits cleared (exact in TF32) and lo = x - hi (exact in F32),
//            and the MMA warp issues hi.hi + hi.lo + lo.hi with
//            kind::tf32, an F32 product to about 2^-22 relative.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "sm100_ptx.cuh"

namespace s3 {

enum OutType : int { kOutF32 = 0, kOutF16 = 1, kOutBF16 = 2 };  // = sam3_dtype codes
enum BMode : int { kBTma16 = 0, kBQ8 = 1, kBF32 = 2 };

// How the epilogue writes a chunk:
//   kEpiDirect    per-thread vector stores (every fused op, any layout)
//   kEpiTmaStore  swizzled smem staging + TMA bulk store (no row remap; a
//                 residual other than the output is added in registers)
//   kEpiTmaAdd    staging + TMA bulk reduce-add into the f32 output, which
//                 is the residual (in-place x += linear(...))
enum EpiMode : int { kEpiDirect = 0, kEpiTmaStore = 1, kEpiTmaAdd = 2 };

// Fused epilogue description.  All pointers are device pointers.
struct EpiParams {
  void* out;             // [M, ldo] (row index possibly remapped)
  int out_type;          // OutType
  int ldo;
  const float* col_scale;  // [N] or null: multiplies the accumulator first
                           // (undoes the per-row scale shift of fast Q8 W)
  const float* bias;     // [N] or null
  int act;               // 0 none, 1 tanh-GELU (cpu_gelu.c:23-36)
  const float* residual; // [M, ldr] fp32 added last, may alias out
  int ldr;
  int res_row_period;    // >0: residual row = row % period (pos-embed tiling)
  // RoPE on output columns [0, rope_cols): interleaved pairs within 64-wide
  // heads rotated by (cos, sin) of row p = row % rope_period
  // (cpu_rope.c:35-110).  The table is pair-major, rope_cs[d * period + p]
  // for pair d in [0, 32), so that the 32 lanes of a warp (32 consecutive
  // rows) read one contiguous 256-byte run per pair.
  const float2* rope_cs;
  int rope_cols;
  int rope_period;
  // Output row remap: stored row = (row / period) * period + map[row % period]
  const int* out_row_map;
  int out_row_period;
};

struct GemmShape {
  int M, N, K;
};

// Implicit-GEMM 3x3 convolution (stride 1, padding 1) on the pair kernel:
// A is read straight from the NHWC input through a 4-D tensor map, each
// CTA's 128 rows being a block of 4 image rows x 32 columns; K runs over
// (ky, kx, 64-channel slice).  Needs H % 4 == 0, W % 32 == 0, C % 64 == 0.
struct ConvGeom {
  int on;         // 0: plain GEMM
  int H, W, C;    // input = output spatial size, channels
  int n_img;
  int n_bx, n_by;  // 32-column / 4-row blocks per image
};

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;          // 64 x 16-bit = 128 B rows (SWIZZLE_128B)
constexpr int kStages16 = 4;      // smem ring depth, 16-bit W
constexpr int kStagesQ8 = 4;      // smem ring depth, Q8 W (A + int8 + scales per stage)
constexpr int kUmmaK = 16;
constexpr int kATileBytes = kBM * kBK * 2;   // 16 KiB
constexpr int kBTileBytes = kBN * kBK * 2;   // 32 KiB
constexpr int kQ8TileBytes = kBN * kBK;      // 16 KiB int8
constexpr int kQ8ScaleBytes = kBN * (kBK / 32) * 4;  // 2 KiB, scales stored [K/32, N]
constexpr int kTmemCols = 2 * kBN;           // 512: double-buffered accumulator

template <int kBMode>
struct GemmCfg {
  // 16-bit W: 2 + 8 epilogue warps; Q8 W: 2 + 4 epilogue + 4 converter warps
  static constexpr bool kConv = kBMode != kBTma16;  // converter warps present
  static constexpr int kEpiWarps = kConv ? 4 : 8;
  static constexpr int kConvThreads = kBMode == kBQ8 ? 256 : (kConv ? 128 : 0);
  static constexpr int kThreads = 64 + kEpiWarps * 32 + kConvThreads;
  static constexpr int kStages = kBMode == kBQ8 ? kStagesQ8 : (kBMode == kBF32 ? 2 : kStages16);
  // K elements per stage (always 128-byte operand rows) and per MMA
  static constexpr int kBKe = kBMode == kBF32 ? 32 : 64;
  static constexpr int kUmmaKe = kBMode == kBF32 ? 8 : 16;
  // 16-bit stage: A | W.  F32 stage: A_hi | W_hi | A_lo | W_lo.  Q8 stage:
  // A | int8 W | scales (34 KiB); the dequantised 16-bit W tiles live in a
  // separate 2-deep ring so conversion is decoupled from the TMA ring.
  static constexpr int kStageBytes =
      kBMode == kBQ8 ? kATileBytes + kQ8TileBytes + kQ8ScaleBytes
                     : kATileBytes + kBTileBytes + (kBMode == kBF32 ? kATileBytes + kBTileBytes : 0);
  static constexpr int kBRing = kBMode == kBQ8 ? 2 : 0;
  static constexpr int kStageOutBytes = 32 * 32 * 4;  // per epilogue warp: one 32x32 chunk
  static constexpr int kSmemBytes = kStages * kStageBytes + kBRing * kBTileBytes + kEpiWarps * kStageOutBytes +
                                    1024 /*align*/ + 256 /*barriers*/;
};

// Launch with programmatic stream serialisation (the kernel's set-up may
// overlap the end of the previous kernel in the stream; the kernel calls
// griddep_wait() before it reads anything that kernel wrote).
// S3CU_PDL=0 launches normally.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, int threads, int smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...) == cudaSuccess ? 0 : -103;  // kErrLaunch
}

// K slices per output tile the pair kernel uses (1 unless `additive`: an
// in-place F32 reduce-add epilogue without activation or RoPE).
int pair_splits(const GemmShape& shp, bool additive, int pairs);

// y[n*H*W, OC] = conv3x3(x NHWC [n, H, W, C], w [OC, 3, 3, C] OHWI) + bias
// as an implicit GEMM on the pair kernel (gemm2_sm100.cu); x / w 16-bit of
// dtype ab_dtype, y of ep.out_type (TMA store).  Returns kErrShape when the
// shape does not qualify (see ConvGeom), the caller then takes im2col.
int launch_conv3x3_implicit(const void* x, const void* w, int ab_dtype, int n, int H, int W, int C, int OC,
                            const EpiParams& ep, cudaStream_t stream);

// 2-SM pair launch (gemm2_sm100.cu); shapes validated by launch_gemm.
int launch_gemm_pair(const void* A, int lda, const void* W, int ldw, bool bf, GemmShape shp, const EpiParams& ep,
                     const CUtensorMap& to, int mode, cudaStream_t stream, int max_ctas);

}  // namespace s3
