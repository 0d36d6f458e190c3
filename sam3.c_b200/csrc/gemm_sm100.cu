// gemm_sm100.cu - tcgen05 GEMM kernel bodies and launchers (see gemm_sm100.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <cstdlib>

#include "gemm_sm100.cuh"
#include "gemm_epilogue.cuh"
#include "sam3cu_internal.h"
#include "tma_host.cuh"

namespace s3 {

S3_DEV_ERROR_ACCESSOR(dev_error_gemm)

namespace {

// Split the F32 A and W tiles of one stage (16 KiB + 32 KiB, contiguous
// at `hi`) in place into hi = x & ~0x1fff (a TF32 value) and lo = x - hi,
// written at the same offset of the lo region (so the swizzled layout is
// kept).  128 threads, 16-byte vectors.
__device__ __forceinline__ void split_tf32_tile(uint8_t* hi, uint8_t* lo, int t) {
  constexpr int kVec = (kATileBytes + kBTileBytes) / 16;
#pragma unroll 4
  for (int i = t; i < kVec; i += 128) {
    float4 x = reinterpret_cast<float4*>(hi)[i];
    float4 h, l;
    h.x = __uint_as_float(__float_as_uint(x.x) & 0xffffe000u);
    h.y = __uint_as_float(__float_as_uint(x.y) & 0xffffe000u);
    h.z = __uint_as_float(__float_as_uint(x.z) & 0xffffe000u);
    h.w = __uint_as_float(__float_as_uint(x.w) & 0xffffe000u);
    l.x = x.x - h.x;
    l.y = x.y - h.y;
    l.z = x.z - h.z;
    l.w = x.w - h.w;
    reinterpret_cast<float4*>(hi)[i] = h;
    reinterpret_cast<float4*>(lo)[i] = l;
  }
}

// float(q) for the 4 signed bytes of `raw`, without int->float conversion
// instructions (they issue at a quarter rate): each byte, offset by 128,
// is permuted into the low mantissa byte of 2^23 and 2^23 + 128 is
// subtracted; exact for every int8.
__device__ __forceinline__ void i8x4_to_f32(uint32_t raw, float (&f)[4]) {
  const uint32_t u = raw ^ 0x80808080u;  // b + 128 as unsigned bytes
  f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
  f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
  f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
  f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
}

// Dequantise one k-tile of Q8 W (int8 [kBN rows x 64] + scales [2][kBN]) to
// 16-bit values in the 128-byte-swizzled K-major layout the MMA reads:
// value = float(q) * scale rounded to nearest even (as sam3_q8_dequantize
// then an RNE cast).  kT threads; thread t handles 16-byte chunk (t & 7)
// of rows (t>>3)+(kT/8)i for kT threads.
template <bool kBf16, int kT>
__device__ __forceinline__ void q8_dequant_tile(const int8_t* q, const float* sc, uint8_t* dst,
                                                int t) {
  const int c = t & 7;
#pragma unroll 4
  for (int i = 0; i < kBN / (kT >= 8 ? kT / 8 : 1); ++i) {  // kT = 0: not instantiated for use
    const int n = (t >> 3) + (kT / 8) * i;
    const uint2 raw = *reinterpret_cast<const uint2*>(q + n * kBK + c * 8);
    const float s = sc[(c >> 2) * kBN + n];
    float f[8];
    i8x4_to_f32(raw.x, *reinterpret_cast<float(*)[4]>(f));
    i8x4_to_f32(raw.y, *reinterpret_cast<float(*)[4]>(f + 4));
#pragma unroll
    for (int k = 0; k < 8; ++k) f[k] *= s;
    uint4 w;
    if (kBf16) {  // one cvt.rn.bf16x2.f32 per pair (integer rounding would load the ALU pipe)
      w.x = pack_bf16(f[0], f[1]);
      w.y = pack_bf16(f[2], f[3]);
      w.z = pack_bf16(f[4], f[5]);
      w.w = pack_bf16(f[6], f[7]);
    } else {
      w.x = pack_f16(f[0], f[1]);
      w.y = pack_f16(f[2], f[3]);
      w.z = pack_f16(f[4], f[5]);
      w.w = pack_f16(f[6], f[7]);
    }
    *reinterpret_cast<uint4*>(dst + n * 128 + ((c ^ (n & 7)) << 4)) = w;
  }
}

// Fast path for f16 operands: every value is made in half2 arithmetic.  Byte
// u = q + 128 is permuted under the f16 exponent of 1024 (bits 0x64uu =
// 1024 + u, exact), 1152 is subtracted (exact: q as f16), and the product
// with the block scale is rounded once to f16.  The scales carry a
// per-row power-of-two shift that keeps them in f16's normal range; the
// GEMM epilogue divides it out (EpiParams::col_scale).
template <int kT>
__device__ __forceinline__ void q8_dequant_tile_h2(const int8_t* q, const float* sc, uint8_t* dst, int t) {
  const int c = t & 7;
  const __half2 k1152 = __float2half2_rn(1152.0f);
#pragma unroll 4
  for (int i = 0; i < kBN / (kT >= 8 ? kT / 8 : 1); ++i) {  // kT = 0: not instantiated for use
    const int n = (t >> 3) + (kT / 8) * i;
    const uint2 raw = *reinterpret_cast<const uint2*>(q + n * kBK + c * 8);
    const __half2 s = __float2half2_rn(sc[(c >> 2) * kBN + n]);
    const uint32_t u0 = raw.x ^ 0x80808080u, u1 = raw.y ^ 0x80808080u;
    uint32_t h[4] = {__byte_perm(u0, 0x64646464u, 0x4140), __byte_perm(u0, 0x64646464u, 0x4342),
                     __byte_perm(u1, 0x64646464u, 0x4140), __byte_perm(u1, 0x64646464u, 0x4342)};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __half2 v = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&h[k]), k1152), s);
      h[k] = *reinterpret_cast<uint32_t*>(&v);
    }
    *reinterpret_cast<uint4*>(dst + n * 128 + ((c ^ (n & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
  }
}

// The (tile, K range) segments one CTA processes.  Plain: whole tiles
// blockIdx.x, blockIdx.x + gridDim.x, ...  Stream-K (`sk`, in-place F32
// reduce-add epilogues only): the tiles x k-iterations of the problem are
// cut into gridDim.x equal contiguous ranges, one per CTA, so every CTA
// gets the same MMA work whatever the tile count; a tile whose K range is
// split between CTAs is finished by the reduce-adds of its pieces (the
// bias with the piece that starts at k = 0).  Every role walks the same
// sequence.
struct Segs {
  int64_t pos, end;
  int k_iters, tile, kb, ke;
  bool sk;
  __device__ __forceinline__ void init(bool sk_, int num_tiles, int k_iters_) {
    sk = sk_;
    k_iters = k_iters_;
    const int64_t total = static_cast<int64_t>(num_tiles) * k_iters;
    if (sk) {
      pos = total * blockIdx.x / gridDim.x;
      end = total * (blockIdx.x + 1) / gridDim.x;
    } else {
      pos = static_cast<int64_t>(blockIdx.x) * k_iters;
      end = total;
    }
    if (pos < end) set();
  }
  __device__ __forceinline__ bool valid() const { return pos < end; }
  __device__ __forceinline__ void set() {
    tile = static_cast<int>(pos / k_iters);
    kb = static_cast<int>(pos % k_iters);
    const int64_t rem = end - pos;
    ke = (sk && rem < k_iters - kb) ? kb + static_cast<int>(rem) : k_iters;
  }
  __device__ __forceinline__ void advance() {
    pos += sk ? static_cast<int64_t>(ke - kb) : static_cast<int64_t>(gridDim.x) * k_iters;
    if (pos < end) set();
  }
};

template <int kBMode>
__global__ void __launch_bounds__(GemmCfg<kBMode>::kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                const __grid_constant__ CUtensorMap tmap_s, const __grid_constant__ CUtensorMap tmap_o,
                GemmShape shp, EpiParams ep, uint32_t idesc, int b_is_bf16, int epi_mode, int streamk) {
  using Cfg = GemmCfg<kBMode>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bring = smem + S * Cfg::kStageBytes;                  // Q8: dequantised W ring
  uint8_t* stage_out = bring + Cfg::kBRing * kBTileBytes;       // kEpiWarps x 4 KiB
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(stage_out + Cfg::kEpiWarps * Cfg::kStageOutBytes);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* conv_bar = empty_bar + S;   // F32: stage split; Q8: [2] ring slot ready
  uint64_t* bemp_bar = conv_bar + S;    // Q8: [2] ring slot consumed by the MMAs
  uint64_t* accf_bar = bemp_bar + 2;    // [2] accumulator committed
  uint64_t* acce_bar = accf_bar + 2;    // [2] accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (shp.M + kBM - 1) / kBM;
  const int n_tiles = (shp.N + kBN - 1) / kBN;
  const int num_tiles = m_tiles * n_tiles;
  constexpr int BKe = Cfg::kBKe;
  const int k_iters = (shp.K + BKe - 1) / BKe;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&conv_bar[s], Cfg::kConvThreads);
    }
    for (int b = 0; b < 2; ++b) mbar_init(&bemp_bar[b], 1);
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], Cfg::kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
#if defined(S3_PDL_LN) && S3_PDL_LN
  griddep_launch();  // a LayerNorm launched behind this GEMM may start (it waits for completion)
#endif
  griddep_wait();  // set-up done; from here on the inputs of the previous kernel are read

  auto stage_a = [&](int s) { return smem + s * Cfg::kStageBytes; };
  // W operand of k-iteration `it`: in the stage, or (Q8) in ring slot it & 1
  auto stage_b = [&](int s) { return smem + s * Cfg::kStageBytes + kATileBytes; };
  auto ring_b = [&](uint32_t it) { return bring + (it & 1) * kBTileBytes; };
  // F32: lo half of the stage; Q8: int8 tile and scales
  auto stage_q = [&](int s) {
    return smem + s * Cfg::kStageBytes + kATileBytes + (kBMode == kBQ8 ? 0 : kBTileBytes);
  };
  auto stage_sc = [&](int s) { return smem + s * Cfg::kStageBytes + kATileBytes + kQ8TileBytes; };

  if (warp == 0) {
    // ---------------- TMA producer: the whole warp runs the loop, one
    // elected lane issues the copies
    {
      if (elect_one()) {
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
        if (kBMode == kBQ8) tma_prefetch_desc(&tmap_s);
      }
      __syncwarp();
      uint32_t it = 0;
      bool ok = true;
      Segs sg;
      for (sg.init(streamk != 0, num_tiles, k_iters); sg.valid() && ok; sg.advance()) {
        const int m0 = (sg.tile / n_tiles) * kBM;  // N-fastest: A rows stay in L2
        const int n0 = (sg.tile % n_tiles) * kBN;
        for (int kt = sg.kb; kt < sg.ke; ++kt, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait_warp(&empty_bar[s], ph ^ 1, kErrStageFree, abort_flag)) { ok = false; break; }
          if (elect_one()) {
            if (kBMode == kBQ8) {
              mbar_arrive_expect_tx(&full_bar[s], kATileBytes + kQ8TileBytes + kQ8ScaleBytes);
              tma_load_2d(stage_a(s), &tmap_a, &full_bar[s], kt * kBK, m0);
              tma_load_2d(stage_q(s), &tmap_b, &full_bar[s], kt * kBK, n0);
              tma_load_2d(stage_sc(s), &tmap_s, &full_bar[s], n0, kt * (kBK / 32));
            } else {
              mbar_arrive_expect_tx(&full_bar[s], kATileBytes + kBTileBytes);
              tma_load_2d(stage_a(s), &tmap_a, &full_bar[s], kt * BKe, m0);
              tma_load_2d(stage_b(s), &tmap_b, &full_bar[s], kt * BKe, n0);
            }
          }
          __syncwarp();
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the whole warp runs the loop (operands
    // stay warp-uniform), one elected lane issues each MMA / commit
    {
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      Segs sg;
      for (sg.init(streamk != 0, num_tiles, k_iters); sg.valid() && ok; sg.advance(), ++local) {
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait_warp(&acce_bar[acc], aph ^ 1, kErrAccFree, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int kt = sg.kb; kt < sg.ke; ++kt, ++it) {
          const int kr = kt - sg.kb;  // 0 on the segment's first k-iteration: overwrite the accumulator
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          uint64_t* ready = kBMode == kBQ8 ? &conv_bar[it & 1] : (Cfg::kConv ? &conv_bar[s] : &full_bar[s]);
          const uint32_t rph = kBMode == kBQ8 ? (it >> 1) & 1 : ph;
          if (!mbar_wait_warp(ready, rph, kErrTmaWait, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sdesc_sw128(smem_u32(stage_a(s)));
          const uint64_t bdesc = make_sdesc_sw128(smem_u32(kBMode == kBQ8 ? ring_b(it) : stage_b(s)));
          if constexpr (kBMode == kBF32) {
            // 3xTF32: lo terms first, hi.hi last; 8 TF32 = 32 bytes per MMA
            const uint64_t aldesc = make_sdesc_sw128(smem_u32(stage_q(s)));
            const uint64_t bldesc = make_sdesc_sw128(smem_u32(stage_q(s) + kATileBytes));
#pragma unroll
            for (int k = 0; k < BKe / Cfg::kUmmaKe; ++k) {
              umma_ss_warp<1>(d_tmem, aldesc + 2 * k, bdesc + 2 * k, idesc, (kr | k) ? 1u : 0u);
              umma_ss_warp<1>(d_tmem, adesc + 2 * k, bldesc + 2 * k, idesc, 1u);
              umma_ss_warp<1>(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, 1u);
            }
          } else {
#pragma unroll
            for (int k = 0; k < BKe / Cfg::kUmmaKe; ++k) {
              // advance 16 elements = 32 bytes = 2 (16-byte units) along K
              umma_ss_warp<0>(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kr | k) ? 1u : 0u);
            }
          }
          umma_commit_warp(&empty_bar[s]);  // frees the smem stage when these MMAs finish
          if (kBMode == kBQ8) umma_commit_warp(&bemp_bar[it & 1]);  // and the ring slot
        }
        if (ok) umma_commit_warp(&accf_bar[acc]);
      }
    }
  } else if (warp < 2 + Cfg::kEpiWarps) {
    // ---------------- epilogue: warp w -> TMEM lane quarter w % 4, column
    // range [half * kBN / H, (half + 1) * kBN / H) with H = kEpiWarps / 4
    const int quarter = warp & 3;
    constexpr int kHalves = Cfg::kEpiWarps / 4;
    constexpr int kChunks = kBN / 32 / kHalves;
    const int half = (warp - 2) / 4;
    uint8_t* my_stage = stage_out + (warp - 2) * Cfg::kStageOutBytes;
    int local = 0;
    Segs sg;
    for (sg.init(streamk != 0, num_tiles, k_iters); sg.valid(); sg.advance(), ++local) {
      const int m0 = (sg.tile / n_tiles) * kBM;
      const int n0 = (sg.tile % n_tiles) * kBN;
      const bool first_k = sg.kb == 0;  // the bias goes with the piece at k = 0
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      // one lane waits, the warp follows its verdict (tcgen05.ld is .aligned)
      int got = 0;
      if (lane == 0) got = mbar_wait(&accf_bar[acc], aph, kErrAccFull, abort_flag) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      tc_fence_after();
      const int row = m0 + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN;
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
            epilogue_math(ep, v, row, col0, shp.N, first_k);
            epilogue_store_direct(ep, v, row, col0, shp.N);
          }
        } else {
          // rows >= M and columns >= N are clipped by the TMA store
          epilogue_math(ep, v, row < shp.M ? row : shp.M - 1, col0, shp.N, first_k);
          // a residual other than the destination (e.g. the periodic pos-embed)
          if (epi_mode == kEpiTmaStore && ep.residual)
            epilogue_residual(ep, v, row < shp.M ? row : shp.M - 1, col0, shp.N);
          if (lane == 0) bulk_wait_read<0>();  // previous chunk's smem read done
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
      if (lane == 0) mbar_arrive(&acce_bar[acc]);
    }
    if (lane == 0) bulk_wait<0>();  // all stores of this warp complete
  } else if (Cfg::kConv) {
    // ---------------- converters (4 warps): Q8 dequant or TF32 hi/lo split
    const int t = threadIdx.x - 32 * (2 + Cfg::kEpiWarps);
    uint32_t it = 0;
    bool ok = true;
    Segs sg;
    for (sg.init(streamk != 0, num_tiles, k_iters); sg.valid() && ok; sg.advance()) {
      for (int kt = sg.kb; kt < sg.ke; ++kt, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(&full_bar[s], ph, kErrTmaWait, abort_flag)) { ok = false; break; }
        if constexpr (kBMode == kBF32) {
          split_tf32_tile(stage_a(s), stage_q(s), t);
          fence_proxy_async_smem();  // make generic-proxy writes visible to tcgen05
          mbar_arrive(&conv_bar[s]);
        } else {
          // ring slot free once the MMAs of iteration it - 2 finished
          if (!mbar_wait(&bemp_bar[it & 1], ((it >> 1) & 1) ^ 1, kErrStageFree, abort_flag)) { ok = false; break; }
          const int8_t* q = reinterpret_cast<const int8_t*>(stage_q(s));
          const float* sc = reinterpret_cast<const float*>(stage_sc(s));
          if (b_is_bf16)
            q8_dequant_tile<true, Cfg::kConvThreads>(q, sc, ring_b(it), t);
          else if (ep.col_scale)  // shifted scales: half2 arithmetic
            q8_dequant_tile_h2<Cfg::kConvThreads>(q, sc, ring_b(it), t);
          else
            q8_dequant_tile<false, Cfg::kConvThreads>(q, sc, ring_b(it), t);
          fence_proxy_async_smem();  // make generic-proxy writes visible to tcgen05
          mbar_arrive(&conv_bar[it & 1]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

int g_num_sms = 0;




// 2-SM pair tiles (gemm2_sm100.cu) for the 16-bit path unless SAM3CU_GEMM=1sm
// or the problem is too small to keep the SMs busy with 256x256 tiles.
bool use_pair_gemm(const GemmShape& shp, bool additive) {
  static const int mode = [] {
    const char* e = getenv("SAM3CU_GEMM");
    return e && strcmp(e, "1sm") == 0 ? 0 : 1;
  }();
  if (!mode) return false;
  const long pairs = static_cast<long>((shp.M + 255) / 256) * ((shp.N + 255) / 256) *
                     pair_splits(shp, additive, num_sms() / 2);
  return pairs >= num_sms();  // at least two waves of pairs (K slices included)
}
std::atomic<uint64_t> g_launches{0};

}  // namespace

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("S3CU_PDL");
    return !(e && atoi(e) == 0);
  }();
  return on;
}

uint64_t count_launches(int64_t delta) {
  return g_launches.fetch_add(static_cast<uint64_t>(delta)) + static_cast<uint64_t>(delta);
}

int num_sms() {
  if (!g_num_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return g_num_sms;
}

// Launch Y = epi(A . W^T).  ab_dtype: kBF16 or kF16 (A and 16-bit W share it).
// W: 16-bit [N, ldw] or (q8 != null) int8 [N, K] + scales [K/32, N].
int launch_gemm(const void* A, int lda, const void* W, int ldw, const int8_t* q8, const float* q8_scales,
                int ab_dtype, GemmShape shp, const EpiParams& ep, cudaStream_t stream, int max_ctas) {
  if (ab_dtype != kBF16 && ab_dtype != kF16 && ab_dtype != kF32) return kErrDtype;
  const bool bf = ab_dtype == kBF16, f32in = ab_dtype == kF32;
  if (f32in && q8) return kErrDtype;
  if (shp.M <= 0 || shp.N <= 0 || shp.K <= 0) return 0;
  // TMA: 16-byte row pitch
  if (f32in ? (shp.K % 4 != 0 || lda % 4 != 0) : (shp.K % 8 != 0 || lda % 8 != 0)) return kErrShape;
  if (ep.rope_cols > 0 && (ep.rope_period <= 0 || !ep.rope_cs)) return kErrShape;
  if (ep.out_row_map && ep.out_row_period <= 0) return kErrShape;
  // vector epilogue stores/loads: 16-byte aligned rows
  if (ep.ldo % (ep.out_type == kOutF32 ? 4 : 8) != 0) return kErrShape;
  if (ep.residual && ep.ldr % 4 != 0) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(ep.out) | reinterpret_cast<uintptr_t>(ep.residual) |
       reinterpret_cast<uintptr_t>(ep.bias)) & 15u)
    return kErrShape;
  const CUtensorMapDataType dt = f32in ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : (bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  const int es = f32in ? 4 : 2;
  const int bke = f32in ? GemmCfg<kBF32>::kBKe : kBK;  // 128-byte operand rows either way
  CUtensorMap ta, tb, ts;
  memset(&ts, 0, sizeof(ts));
  if (!make_tmap_2d(&ta, A, dt, es, shp.M, shp.K, lda, kBM, bke, CU_TENSOR_MAP_SWIZZLE_128B))
    return kErrTma;
  const int m_tiles = (shp.M + kBM - 1) / kBM, n_tiles = (shp.N + kBN - 1) / kBN;
  int grid = m_tiles * n_tiles;
  int cap = max_ctas > 0 ? max_ctas : num_sms();
  if (grid > cap) grid = cap;
  const uint32_t idesc = make_idesc(f32in ? 2u : (bf ? 1u : 0u), kBM, kBN);
  // epilogue write path (see EpiMode)
  CUtensorMap to;
  memset(&to, 0, sizeof(to));
  int mode = kEpiDirect;
  if (!ep.out_row_map) {
    if (!ep.residual || ep.residual != ep.out)
      mode = kEpiTmaStore;  // a separate residual is added in registers
    else if (ep.out_type == kOutF32 && ep.ldr == ep.ldo && ep.res_row_period == 0)
      mode = kEpiTmaAdd;
  }
  if (mode != kEpiDirect) {
    const bool f32 = ep.out_type == kOutF32;
    const CUtensorMapDataType odt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                        : (ep.out_type == kOutBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    if (!make_tmap_2d(&to, ep.out, odt, f32 ? 4 : 2, shp.M, shp.N, ep.ldo, 32, 32,
                      f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
      mode = kEpiDirect;  // e.g. an output base that is not 16-byte aligned
  }
  count_launches(1);
  if (!q8 && !f32in && use_pair_gemm(shp, mode == kEpiTmaAdd && ep.act == 0 && ep.rope_cols == 0)) {
    if (ldw % 8 != 0) return kErrShape;
    return launch_gemm_pair(A, lda, W, ldw, bf, shp, ep, to, mode, stream, max_ctas);
  }
  // Stream-K for the in-place F32 reduce-add linears (no activation / RoPE)
  // of the 3xTF32 kernel whose tile count fills the last wave poorly, e.g.
  // proj at one image: 164 tiles of 128x256 on 148 SMs ran as 1.1 waves.
  // Every CTA then gets the same number of k-iterations (Segs).  Measured at
  // M = 5184: F32 proj 81 -> 135 TFLOP/s, fc2 102 -> 183.  The 16-bit
  // kernels do not gain (BF16 proj 515 -> 497: its reduce-add traffic, which
  // stream-K doubles, bounds it), so they keep whole tiles.
  // S3CU_GEMM_STREAMK=0 disables it, =2 also enables it for 16-bit operands.
  static const int sk_mode = [] {
    const char* e = getenv("S3CU_GEMM_STREAMK");
    return e ? atoi(e) : 1;
  }();
  int streamk = 0;
  {
    const int tiles = m_tiles * n_tiles;
    const int k_iters = (shp.K + bke - 1) / bke;
    if ((sk_mode >= 2 || (sk_mode == 1 && f32in)) && mode == kEpiTmaAdd && ep.act == 0 && ep.rope_cols == 0 && k_iters >= 8 &&
        static_cast<int64_t>(tiles) * k_iters >= 4LL * cap) {
      const int waves = (tiles + cap - 1) / cap;
      const double eff = static_cast<double>(tiles) / (static_cast<double>(waves) * cap);
      if (eff < 0.85) {
        streamk = 1;
        grid = cap;
      }
    }
  }
  if (q8) {
    if (shp.K % 64 != 0) return kErrShape;
    if (!make_tmap_2d(&tb, q8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, shp.N, shp.K, shp.K, kBN, kBK,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
      return kErrTma;
    if (!make_tmap_2d(&ts, q8_scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, shp.K / 32, shp.N, shp.N,
                      kBK / 32, kBN, CU_TENSOR_MAP_SWIZZLE_NONE))
      return kErrTma;
    constexpr int smem = GemmCfg<kBQ8>::kSmemBytes;
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(gemm_kernel<kBQ8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      attr = true;
    }
    return launch_pdl(gemm_kernel<kBQ8>, grid, GemmCfg<kBQ8>::kThreads, smem, stream, ta, tb, ts, to, shp, ep, idesc,
                      bf ? 1 : 0, mode, streamk);
  } else if (f32in) {
    if (ldw % 4 != 0) return kErrShape;
    if (!make_tmap_2d(&tb, W, dt, 4, shp.N, shp.K, ldw, kBN, bke, CU_TENSOR_MAP_SWIZZLE_128B))
      return kErrTma;
    constexpr int smem = GemmCfg<kBF32>::kSmemBytes;
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(gemm_kernel<kBF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      attr = true;
    }
    return launch_pdl(gemm_kernel<kBF32>, grid, GemmCfg<kBF32>::kThreads, smem, stream, ta, tb, ts, to, shp, ep,
                      idesc, 0, mode, streamk);
  } else {
    if (ldw % 8 != 0) return kErrShape;
    if (!make_tmap_2d(&tb, W, dt, 2, shp.N, shp.K, ldw, kBN, kBK, CU_TENSOR_MAP_SWIZZLE_128B))
      return kErrTma;
    constexpr int smem = GemmCfg<kBTma16>::kSmemBytes;
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(gemm_kernel<kBTma16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      attr = true;
    }
    return launch_pdl(gemm_kernel<kBTma16>, grid, GemmCfg<kBTma16>::kThreads, smem, stream, ta, tb, ts, to, shp,
                      ep, idesc, bf ? 1 : 0, mode, streamk);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : kErrLaunch;
}

}  // namespace s3
