// gemm2_sm100.cu - the 16-bit linear on CTA pairs (tcgen05 cta_group::2).
//
// Same contract and fused epilogue as gemm_kernel<kBTma16> (gemm_sm100.cu),
// but every output tile is 256 x 256 and is computed by a pair of CTAs on
// two SMs (a cluster of 2):
//   * each CTA TMA-loads its own 128 rows of A and its own 128 rows (N) of
//     W into its shared memory; the transaction bytes of both CTAs count on
//     the leader's (cluster rank 0) barrier;
//   * the leader's MMA thread issues tcgen05.mma.cta_group::2 256x256x16:
//     A rows and W halves are read from both CTAs' shared memory at the
//     same offsets, each CTA's TMEM receives its 128 rows x 256 columns;
//   * commits release the stage / accumulator in both CTAs.
// Per SM this halves the W bytes that shared memory must deliver per MMA
// (the reason a 1-SM 128x256 tile cannot run the tensor core at its rate),
// and with 32 KiB stages the ring is 6 deep.  No multicast loads are used.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "gemm_epilogue.cuh"
#include "gemm_sm100.cuh"
#include "sam3cu_internal.h"
#include "tma_host.cuh"

namespace s3 {

S3_DEV_ERROR_ACCESSOR(dev_error_gemm2)

namespace {

constexpr int kPM = 128;                 // rows per CTA (256 per pair)
constexpr int kPN = 256;                 // output columns per tile (the 128-column variant: kN)
constexpr int kPK = 64;
constexpr int kPStages = 6;
constexpr int kPTile = kPM * kPK * 2;    // 16 KiB: A tile (or W half-tile of a 256-column tile)
constexpr int kPEpiWarps = 8;
constexpr int kPThreads = 64 + kPEpiWarps * 32;
constexpr int kPOut = 32 * 32 * 4;
// Per tile width kN (256, or 128 for shapes whose 256-column tiles fill the
// last wave of CTA pairs poorly): W half-tile bytes, stage bytes, smem, TMEM.
template <int kN>
struct PairCfg {
  static constexpr int kWTile = (kN / 2) * kPK * 2;
  static constexpr int kStage = kPTile + kWTile;
  static constexpr int kSmem = kPStages * kStage + kPEpiWarps * kPOut + 1024 + 256;
  static constexpr int kTmemCols = 2 * kN;
};

template <int kN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 const __grid_constant__ CUtensorMap tmap_o, GemmShape shp, EpiParams ep, uint32_t idesc,
                 int epi_mode, int splits, ConvGeom cg) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using PC = PairCfg<kN>;
  uint8_t* stage_out = smem + kPStages * PC::kStage;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(stage_out + kPEpiWarps * kPOut);
  uint64_t* empty_bar = full_bar + kPStages;
  uint64_t* accf_bar = empty_bar + kPStages;  // [2]
  uint64_t* acce_bar = accf_bar + 2;          // [2] (leader's counts both CTAs)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  // conv: one M tile = two 128-pixel blocks (this CTA's = 2 * tile + rank)
  const int m_tiles = cg.on ? (cg.n_img * cg.n_by * cg.n_bx + 1) / 2 : (shp.M + 2 * kPM - 1) / (2 * kPM);
  const int n_tiles = (shp.N + kN - 1) / kN;
  // conv block b -> (image, first output row, first column, flat output row)
  auto conv_block = [&](int b, int& img, int& y0, int& x0) {
    const int bx = b % cg.n_bx, t = b / cg.n_bx;
    x0 = bx * 32;
    y0 = (t % cg.n_by) * 4;
    img = t / cg.n_by;
  };
  // split-K (splits > 1, reduce-add epilogue only): work item t covers
  // output tile t / splits and K slice t % splits; slice 0 adds the bias
  const int num_tiles = m_tiles * n_tiles * splits;
  const int k_iters = (shp.K + kPK - 1) / kPK;
  auto k_begin = [&](int tile) { return (tile % splits) * k_iters / splits; };
  auto k_end = [&](int tile) { return (tile % splits + 1) * k_iters / splits; };
  auto stage_a = [&](int s) { return smem + s * PC::kStage; };
  auto stage_b = [&](int s) { return smem + s * PC::kStage + kPTile; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], 2 * kPEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, PC::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers and TMEM exist before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
#if defined(S3_PDL_LN) && S3_PDL_LN
  griddep_launch();  // a LayerNorm launched behind this GEMM may start (it waits for completion)
#endif
  griddep_wait();  // set-up done; from here on the inputs of the previous kernel are read

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs): own A rows, own W half; the
    // whole warp runs the loop, one elected lane issues the copies
    {
      if (elect_one()) {
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
      }
      __syncwarp();
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        const int mn = tile / splits;
        const int m0 = (mn / n_tiles) * 2 * kPM + rank * kPM;
        const int n0 = (mn % n_tiles) * kN + rank * (kN / 2);
        int cimg = 0, cy0 = 0, cx0 = 0;
        if (cg.on) conv_block((mn / n_tiles) * 2 + rank, cimg, cy0, cx0);
        const int cchunks = cg.C / kPK;
        for (int kt = k_begin(tile); kt < k_end(tile); ++kt, ++it) {
          const int s = it % kPStages;
          const uint32_t ph = (it / kPStages) & 1;
          if (!mbar_wait_warp(&empty_bar[s], ph ^ 1, kErrStageFree, abort_flag)) { ok = false; break; }
          const uint32_t lead_full = mapa_shared(smem_u32(&full_bar[s]), 0);
          if (elect_one()) {
            if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * PC::kStage);  // both CTAs' bytes
            if (cg.on) {  // tap (ky, kx), channels c0..c0+63, shifted by the padding
              const int tap = kt / cchunks, c0 = (kt - tap * cchunks) * kPK;
              tma_load_4d_pair(stage_a(s), &tmap_a, lead_full, c0, cx0 + tap % 3 - 1, cy0 + tap / 3 - 1, cimg);
            } else {
              tma_load_2d_pair(stage_a(s), &tmap_a, lead_full, kt * kPK, m0);
            }
            tma_load_2d_pair(stage_b(s), &tmap_b, lead_full, kt * kPK, n0);
          }
          __syncwarp();
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the pair leader's whole warp runs the loop
    // (operands stay warp-uniform), one elected lane issues each MMA / commit
    if (rank == 0) {
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs, ++local) {
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait_warp(&acce_bar[acc], aph ^ 1, kErrAccFree, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kN;
        const int kt0 = k_begin(tile);
        for (int kt = kt0; kt < k_end(tile); ++kt, ++it) {
          const int s = it % kPStages;
          const uint32_t ph = (it / kPStages) & 1;
          if (!mbar_wait_warp(&full_bar[s], ph, kErrTmaWait, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sdesc_sw128(smem_u32(stage_a(s)));
          const uint64_t bdesc = make_sdesc_sw128(smem_u32(stage_b(s)));
#pragma unroll
          for (int k = 0; k < kPK / kUmmaK; ++k)
            umma_ss_pair_warp(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kt != kt0 || k) ? 1u : 0u);
          // free the stage in both CTAs once these MMAs have read it
          umma_commit_pair_warp(mapa_shared(smem_u32(&empty_bar[s]), 0));
          umma_commit_pair_warp(mapa_shared(smem_u32(&empty_bar[s]), 1));
        }
        if (ok) {
          umma_commit_pair_warp(mapa_shared(smem_u32(&accf_bar[acc]), 0));
          umma_commit_pair_warp(mapa_shared(smem_u32(&accf_bar[acc]), 1));
        }
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows
    const int quarter = warp & 3;
    constexpr int kChunks = kN / 32 / (kPEpiWarps / 4);
    const int half = (warp - 2) / 4;
    uint8_t* my_stage = stage_out + (warp - 2) * kPOut;
    const uint32_t lead_acce0 = mapa_shared(smem_u32(&acce_bar[0]), 0);
    const uint32_t lead_acce1 = mapa_shared(smem_u32(&acce_bar[1]), 0);
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs, ++local) {
      const int mn = tile / splits;
      int m0 = (mn / n_tiles) * 2 * kPM + rank * kPM;
      const int n0 = (mn % n_tiles) * kN;
      const bool first_slice = tile % splits == 0;
      // conv: this warp's 32 rows are output row y0 + quarter, columns x0..x0+31
      int conv_row = 0;
      if (cg.on) {
        int cimg, cy0, cx0;
        conv_block((mn / n_tiles) * 2 + rank, cimg, cy0, cx0);
        conv_row = (cimg * cg.H + cy0 + quarter) * cg.W + cx0;
        m0 = conv_row - quarter * 32;  // so that m0 + quarter * 32 below is conv_row
      }
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      int got = 0;
      if (lane == 0) got = mbar_wait(&accf_bar[acc], aph, kErrAccFull, abort_flag) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      tc_fence_after();
      const int row = m0 + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kN;
#pragma unroll 1
      for (int cc = 0; cc < kChunks; ++cc) {
        const int c = half * kChunks + cc;
        const int col0 = n0 + c * 32;
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        tmem_ld_wait();
        if (col0 >= shp.N) continue;  // warp-uniform
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (epi_mode == kEpiDirect) {
          if (row < shp.M) {
            epilogue_math(ep, v, row, col0, shp.N, first_slice);
            epilogue_store_direct(ep, v, row, col0, shp.N);
          }
        } else {
          epilogue_math(ep, v, row < shp.M ? row : shp.M - 1, col0, shp.N, first_slice);
          // a residual other than the destination (e.g. the periodic pos-embed)
          if (epi_mode == kEpiTmaStore && ep.residual)
            epilogue_residual(ep, v, row < shp.M ? row : shp.M - 1, col0, shp.N);
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
          stage_chunk(my_stage, v, lane, epi_mode == kEpiTmaAdd ? kOutF32 : ep.out_type);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (epi_mode == kEpiTmaAdd)
              tma_reduce_add_2d(&tmap_o, my_stage, col0, m0 + quarter * 32);
            else
              tma_store_2d(&tmap_o, my_stage, col0, m0 + quarter * 32);
            bulk_commit();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&acce_bar[acc]);
        else
          mbar_arrive_cluster(acc ? lead_acce1 : lead_acce0);
      }
    }
    if (lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, PC::kTmemCols);
  }
}

}  // namespace

// K slices per output tile for the pair kernel.  Only an epilogue that adds
// into an F32 destination (TMA reduce-add) with nothing non-linear after the
// bias can take partial sums; then the count (at most 4, each slice at
// least 16 K-iterations: shorter slices measured slower) that best fills the
// last wave of `pairs` CTA pairs is used, the smaller on a tie.  Example,
// M = 5184 (one image), N = 1024: 84 tiles fill 57% of two waves of 74
// pairs; fc2 (K = 4736) takes 4 slices (91%): 896 -> 1025 TFLOP/s.  The
// partial sums reach the destination in no fixed order, so such results are
// reproducible to F32 rounding, not bit for bit.
int pair_splits(const GemmShape& shp, bool additive, int pairs) {
  if (!additive || pairs <= 0) return 1;
  static const int max_splits = [] {  // S3CU_GEMM_MAX_SPLITS caps it (measurements)
    const char* e = getenv("S3CU_GEMM_MAX_SPLITS");
    return e ? atoi(e) : 4;
  }();
  const long tiles = static_cast<long>((shp.M + 2 * kPM - 1) / (2 * kPM)) * ((shp.N + kPN - 1) / kPN);
  const int k_iters = (shp.K + kPK - 1) / kPK;
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= max_splits; ++s) {
    if (s > 1 && k_iters / s < 16) break;
    const long work = tiles * s;
    const double eff = static_cast<double>(work) / (static_cast<double>((work + pairs - 1) / pairs) * pairs);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

// Pair launch of the 16-bit linear; the caller has validated shapes and
// alignment (launch_gemm).  Returns kOk, kErrTma or kErrLaunch.
int launch_gemm_pair(const void* A, int lda, const void* W, int ldw, bool bf, GemmShape shp, const EpiParams& ep,
                     const CUtensorMap& to, int mode, cudaStream_t stream, int max_ctas) {
  const CUtensorMapDataType dt = bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, A, dt, 2, shp.M, shp.K, lda, kPM, kPK, CU_TENSOR_MAP_SWIZZLE_128B)) return kErrTma;
  const int m_tiles = (shp.M + 2 * kPM - 1) / (2 * kPM);
  const int cap = (max_ctas > 0 ? max_ctas : num_sms()) / 2;
  const int splits = pair_splits(shp, mode == kEpiTmaAdd && ep.act == 0 && ep.rope_cols == 0, cap);
  // 128-column tiles (S3CU_GEMM_N128=1, or =-1: when 256-column ones leave
  // the last wave of pairs poorly filled and the narrower tiles fill it
  // clearly better; no split-K).  Off by default: at one image (M = 5184)
  // they measured slower despite the fuller waves, QKV 1098 -> 869 and fc1
  // 1119 -> 882 TFLOP/s, so a tile's fixed costs outweigh the wave gain.
  auto wave_eff = [&](long tiles) {
    return static_cast<double>(tiles) / (static_cast<double>((tiles + cap - 1) / cap) * cap);
  };
  static const int n128 = [] {  // S3CU_GEMM_N128=0 / 1 / -1: never / always / by waves
    const char* e = getenv("S3CU_GEMM_N128");
    return e ? atoi(e) : 0;
  }();
  const long t256 = static_cast<long>(m_tiles) * ((shp.N + 255) / 256) * splits;
  const long t128 = static_cast<long>(m_tiles) * ((shp.N + 127) / 128);
  const bool narrow = splits == 1 && shp.N % 128 == 0 &&
                      (n128 >= 0 ? n128 == 1 : wave_eff(t128) > wave_eff(t256) + 0.05);
  ConvGeom off;
  memset(&off, 0, sizeof(off));
  if (narrow) {
    using PC = PairCfg<128>;
    if (!make_tmap_2d(&tb, W, dt, 2, shp.N, shp.K, ldw, 64, kPK, CU_TENSOR_MAP_SWIZZLE_128B)) return kErrTma;
    const long pairs = t128 < cap ? t128 : cap;
    const uint32_t idesc = make_idesc(bf ? 1u : 0u, 2 * kPM, 128);
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(gemm2_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, PC::kSmem);
      attr = true;
    }
    return launch_pdl(gemm2_kernel<128>, static_cast<int>(2 * pairs), kPThreads, PC::kSmem, stream, ta, tb, to, shp,
                      ep, idesc, mode, 1, off);
  }
  using PC = PairCfg<kPN>;
  if (!make_tmap_2d(&tb, W, dt, 2, shp.N, shp.K, ldw, kPN / 2, kPK, CU_TENSOR_MAP_SWIZZLE_128B)) return kErrTma;
  const long pairs = t256 < cap ? t256 : cap;
  const uint32_t idesc = make_idesc(bf ? 1u : 0u, 2 * kPM, kPN);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemm2_kernel<kPN>, cudaFuncAttributeMaxDynamicSharedMemorySize, PC::kSmem);
    attr = true;
  }
  return launch_pdl(gemm2_kernel<kPN>, static_cast<int>(2 * pairs), kPThreads, PC::kSmem, stream, ta, tb, to, shp,
                    ep, idesc, mode, splits, off);
}

int launch_conv3x3_implicit(const void* x, const void* w, int ab_dtype, int n, int H, int W, int C, int OC,
                            const EpiParams& ep, cudaStream_t stream) {
  if ((ab_dtype != kBF16 && ab_dtype != kF16) || n <= 0 || H % 4 || W % 32 || C % kPK || OC % 8 ||
      ep.residual || ep.out_row_map || ep.rope_cols || ep.ldo != OC)
    return kErrShape;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(ep.out)) & 15)
    return kErrShape;
  const int64_t rows = static_cast<int64_t>(n) * H * W;
  if (rows >= (1LL << 31) || static_cast<int64_t>(9) * C >= (1LL << 31)) return kErrShape;
  const bool bf = ab_dtype == kBF16;
  const CUtensorMapDataType dt = bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb, to;
  // A: 64 channels x 32 columns x 4 rows of one image per 128-row operand tile
  if (!make_tmap_nhwc(&ta, x, dt, 2, n, H, W, C, kPK, 32, 4, CU_TENSOR_MAP_SWIZZLE_128B)) return kErrTma;
  if (!make_tmap_2d(&tb, w, dt, 2, OC, 9 * C, 9 * C, kPN / 2, kPK, CU_TENSOR_MAP_SWIZZLE_128B)) return kErrTma;
  const bool f32 = ep.out_type == kOutF32;
  const CUtensorMapDataType odt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                      : (ep.out_type == kOutBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  if (!make_tmap_2d(&to, ep.out, odt, f32 ? 4 : 2, rows, OC, OC, 32, 32,
                    f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
    return kErrTma;
  ConvGeom cg;
  cg.on = 1;
  cg.H = H;
  cg.W = W;
  cg.C = C;
  cg.n_img = n;
  cg.n_bx = W / 32;
  cg.n_by = H / 4;
  const GemmShape shp{static_cast<int>(rows), OC, 9 * C};
  const int m_tiles = (n * cg.n_by * cg.n_bx + 1) / 2, n_tiles = (OC + kPN - 1) / kPN;
  int pairs = m_tiles * n_tiles;
  const int cap = num_sms() / 2;
  if (pairs > cap) pairs = cap;
  const uint32_t idesc = make_idesc(bf ? 1u : 0u, 2 * kPM, kPN);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemm2_kernel<kPN>, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg<kPN>::kSmem);
    attr = true;
  }
  count_launches(1);
  return launch_pdl(gemm2_kernel<kPN>, 2 * pairs, kPThreads, PairCfg<kPN>::kSmem, stream, ta, tb, to, shp, ep, idesc, kEpiTmaStore,
                    1, cg);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace s3
