// attention_sm100.cu - tcgen05 flash attention, head_dim 64, bf16 / fp16.
//
//   O = softmax(Q K^T / 8) V   per (group of `seq` rows, head)
//
// The online-softmax algorithm of cpu_sdpa.c:49-159 (running max, running
// sum, rescale of the partial output), evaluated on 128x128 tiles with the
// fifth-generation tensor cores:
//
//   S_j   = Q K_j^T          tcgen05.mma 128x128x64 -> TMEM (128 columns)
//   P_j   = exp2(S_j*c - m)  softmax warps: one thread per query row, P
//                            packed to 16-bit pairs in TMEM (64 columns)
//   O    += P_j V_j          tcgen05.mma 128x64x128, A = P from TMEM,
//                            B = V as stored (MN-major), accumulator in TMEM
//
// Keeping P in TMEM leaves shared memory to Q and the K/V ring: per 128-key
// tile the tensor cores read 48 KiB of operands from shared memory (Q, K,
// V) instead of 80 KiB plus the 32 KiB P store, and shared-memory bandwidth
// is what limits a head_dim-64 tile.
//
// CTA = 6 warps, two CTAs per SM (112 KiB smem, 256 TMEM columns and
// 192 threads x 168 registers each):
//   warp 0     TMA (Q tile once, K_j / V_j through a 3-stage ring);
//              allocates TMEM
//   warp 1     MMA issue (the whole warp; one elected lane issues)
//   warps 2-5  softmax and the output epilogue; warp w owns TMEM lane
//              quarter w % 4, i.e. query rows 32*(w%4) .. +31: a thread
//              holds its whole 128-key S row, so the row maximum and sum
//              need no exchange.  (S3_ATTN_SPLIT=2 builds the variant with
//              two warps per quarter, each exponentiating one 64-key half;
//              it measured slower on the 5184-token case.)
// A softmax thread copies its S row to registers and releases S at once,
// so S_{j+1} = Q K_{j+1}^T runs on the tensor cores during the softmax of
// tile j; the two CTAs of an SM interleave on the exponential units.
// The output is rescaled lazily: only when a row maximum grows by more than
// 2^8 is O read back from TMEM, multiplied and stored (tcgen05.ld / st);
// otherwise exponentials are taken against the stale maximum (values up to
// 256 are exact enough in fp32 and bf16).  Every mbarrier wait is bounded.
//
// attn_tc_persist_kernel is the same pipeline with a persistent grid for
// short groups (the 576-token windows): each CTA loops over work items
// (query tile, group, head) with barrier phases running on across items,
// so the next item's Q load and first S MMA overlap the current item's last
// softmax and output epilogue; q_empty gates the Q buffer and o_empty the O
// accumulator.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "sam3cu_internal.h"
#include "sm100_ptx.cuh"
#include "tma_host.cuh"

namespace s3 {

S3_DEV_ERROR_ACCESSOR(dev_error_attn_tc)

namespace {

constexpr int kQ = 128;                  // query rows per CTA
#ifndef S3_ATTN_KV
#define S3_ATTN_KV 128
#endif
constexpr int kKV = S3_ATTN_KV;          // keys per tile
static_assert(kKV == 64 || kKV == 128, "64- or 128-key tiles");
// 128-key tiles: S [0,128), O [128,192), P [192,256) in the CTA's 256 TMEM
// columns, one buffer each.  64-key tiles leave room to double-buffer S and
// P: S0 [0,64) S1 [64,128), O [128,192), P0 [192,224) P1 [224,256), so the
// softmax of tile j+1 neither waits for S_j to be released nor for P_j to
// be consumed (P.V of tile j).
constexpr int kNB = kKV == 64 ? 2 : 1;   // S / P buffers
constexpr int kStages = kKV == 64 ? 6 : 3;  // K/V ring depth (same bytes)
constexpr int kTmemCols = 256;

// Per head dimension: a Q, K or V tile is 128 rows of kD 16-bit elements,
// 128-byte rows (kD 64, 128-byte swizzle) or 64-byte rows (kD 32, 64-byte
// swizzle).
template <int kD>
struct HeadCfg {
  static constexpr int kRowBytes = kD * 2;
  static constexpr int kTile = kQ * kRowBytes;     // Q tile
  static constexpr int kKVTile = kKV * kRowBytes;  // K or V tile
  static constexpr int kSmem = kTile + 2 * kStages * kKVTile;  // Q | K0 V0 | K1 V1 | ...
  static_assert(kD == 32 || kD == 64, "head_dim 32 or 64");
};
#ifndef S3_ATTN_SPLIT
#define S3_ATTN_SPLIT 1
#endif
// Softmax warps per lane quarter: 2 = each row split into two 64-key halves
// (8 softmax warps), 1 = a whole 128-key row per thread (4 softmax warps).
constexpr int kSplit = S3_ATTN_SPLIT;
constexpr int kSoftWarps = 4 * kSplit;
constexpr int kThreads = 64 + 32 * kSoftWarps;  // 2 control warps + softmax
constexpr int kHalf = kKV / kSplit;             // keys per softmax warp
static_assert(kSplit == 1 || kNB == 1, "split softmax rows only with single-buffered S and P");
#ifndef S3_ATTN_PSTORE
#define S3_ATTN_PSTORE 8
#endif
constexpr int kPStore = S3_ATTN_PSTORE;         // P columns per tcgen05.st
constexpr float kRescaleLog2 = 8.0f;     // lazy rescale threshold (x256)


__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf) {
  if (bf) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two f32 lanes in one 64-bit register for the packed f32x2 operations.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fadd2_rm(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

#ifndef S3_ATTN_POLY
#define S3_ATTN_POLY 0
#endif
// Of every 8 key pairs a softmax thread exponentiates, this many take
// exp2_poly2 (FMA pipe) instead of two MUFU ex2 (16 results per clock per
// SM).  Measured at 8 images (global / window TFLOP/s): 0 -> 706 / 437,
// 1 -> 724 / 417, 2 -> 687 / 418, 3 -> 617 / 398: the softmax is bound by
// its dependency chain more than by the exponential unit, so 0 is kept.
constexpr int kPolyPairs = S3_ATTN_POLY;

// 2^x for a pair of exponents x <= 8 on the FMA pipe: x = n + f with
// n = floor(x) (round-down add of 1.5*2^23, which leaves n in the low
// mantissa bits), 2^f on [0, 1) by a degree-3 polynomial fitted here for
// relative error (max 7.5e-5, below the 16-bit rounding of P), and n added
// to the exponent field.  Exponents below -126 (masked keys: -inf) are
// clamped to -126, whose result is 2^-126 or a denormal: zero once P is
// rounded to fp16, and negligible in bf16 P and in the row sum.  (At -127
// the exponent field of a p(f) < 1 would wrap.)
__device__ __forceinline__ void exp2_poly2(uint64_t x2, float& p0, float& p1) {
  float x0, x1;
  f2unpack(x2, x0, x1);
  const uint64_t xc = f2pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t t = fadd2_rm(xc, f2pack(12582912.f, 12582912.f));  // floor(x) + 1.5*2^23
  const uint64_t n = fadd2(t, f2pack(-12582912.f, -12582912.f));    // floor(x), exact
  const uint64_t f = ffma2(n, f2pack(-1.f, -1.f), xc);               // x - floor(x), exact
  uint64_t p = ffma2(f, f2pack(0.07802403f, 0.07802403f), f2pack(0.22606707f, 0.22606707f));
  p = ffma2(p, f, f2pack(0.69583398f, 0.69583398f));
  p = ffma2(p, f, f2pack(0.99992514f, 0.99992514f));
  float q0, q1, t0, t1;
  f2unpack(p, q0, q1);
  f2unpack(t, t0, t1);
  p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Maximum of 64 values: four chains of three-input max.
__device__ __forceinline__ float max64(const float* v) {
  float m[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
  for (int c = 4; c < 64; c += 8) {
#pragma unroll
    for (int k = 0; k < 4; ++k) m[k] = max3(m[k], v[c + 2 * k], v[c + 2 * k + 1]);
  }
  return fmaxf(max3(m[0], m[1], m[2]), m[3]);
}

// Swap one float per row with the warp holding the other column half of
// the same rows (TMEM column tX + half, then read tX + (half ^ 1)); tX is
// any two free columns.  The two
// named-barrier passes order the store before the partner's load and the
// load before the next store.
__device__ __forceinline__ float pair_exchange(uint32_t tX, uint32_t lane_off, int half, float v, int quarter) {
  tmem_st_32x32b_x1(tX + lane_off + half, __float_as_uint(v));
  tmem_st_wait();
  tc_fence_before();
  asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
  tc_fence_after();
  const float other = __uint_as_float(tmem_ld_32x32b_x1(tX + lane_off + (half ^ 1)));
  tmem_ld_wait();
  tc_fence_before();
  asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
  tc_fence_after();
  return other;
}

// Maximum of 128 values: eight independent chains of three-input max
// (the softmax is latency-bound, so short chains matter).
__device__ __forceinline__ float max128(const float* v) {
  float m[8] = {v[0], v[1], v[2], v[3], v[64], v[65], v[66], v[67]};
#pragma unroll
  for (int c = 4; c < 64; c += 8) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      m[k] = max3(m[k], v[c + 2 * k], v[c + 2 * k + 1]);
      m[4 + k] = max3(m[4 + k], v[64 + c + 2 * k], v[64 + c + 2 * k + 1]);
    }
  }
  return fmaxf(fmaxf(max3(m[0], m[1], m[2]), m[3]), fmaxf(max3(m[4], m[5], m[6]), m[7]));
}

// Bounded wait by lane 0, verdict broadcast to the warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, unsigned err, volatile int* abort_flag,
                                          int lane) {
  int ok = 0;
  if (lane == 0) ok = mbar_wait(bar, parity, err, abort_flag) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Kernel arguments beyond the tensor maps.
struct AttnParams {
  uint16_t* o;         // output rows [groups * seq, ldo]; head h at column h * o_hstride
  int64_t ldo;
  int o_hstride;
  int in_hstride;      // column distance between heads in the Q/K/V maps
  int seq;             // rows (tokens) per group
  int q_tiles;         // ceil(seq / 128)
  int pack;            // > 1: this many whole groups share one 128-row tile
                       // (block-diagonal attention, seq <= 64); q_tiles = 1
  int n_groups;
  int n_x;             // work items per head: query tiles of all groups
  int n_items;         // n_x * heads (persistent kernel)
  float scale;         // softmax scale (1/sqrt(head_dim))
  float scale_log2;    // scale * log2(e)
  const float* bias;   // optional additive bias [heads, seq, bias_ld] f32, or with
                       // pack > 1 the per-tile table [heads, pack*seq, bias_ld]
  int bias_ld;         // multiple of 4
};

// Two CTAs of 10 warps per SM: 5 warps per SM sub-partition, whose
// register file holds 16K entries: about 100 registers per thread.
// kBf16: Q/K/V/P/O are bf16, else f16.  kD: head dim.  kBias: an additive
// f32 bias [head, query, key] joins the scaled scores before the softmax
// (TinyViT's relative position bias, image_encoder_tinyvit.c:842-846).
template <bool kBf16, int kD, bool kBias>
__global__ void __launch_bounds__(kThreads, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const AttnParams prm) {
  using HC = HeadCfg<kD>;
  constexpr int kTile = HC::kTile;
  constexpr int kOHalf = kD / kSplit;  // O columns per softmax warp
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint64_t bars[10 + 2 * kStages];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag_s;
  uint64_t* q_full = &bars[0];
  uint64_t* o_full = &bars[1];
  uint64_t* s_full = &bars[2];               // [kNB]
  uint64_t* s_empty = &bars[4];              // [kNB]
  uint64_t* p_full = &bars[6];               // [kNB]
  uint64_t* p_empty = &bars[8];              // [kNB]
  uint64_t* kv_full = &bars[10];             // [kStages]
  uint64_t* kv_empty = &bars[10 + kStages];  // [kStages]
  volatile int* abort_flag = &abort_flag_s;

  const int seq = prm.seq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const bool packed = prm.pack > 1;
  const int group = packed ? blockIdx.x * prm.pack : blockIdx.x / prm.q_tiles;
  const int qt = packed ? 0 : blockIdx.x % prm.q_tiles;
  const int row0 = group * seq;  // first row of the (first) group in the [rows, ld] matrices
  // rows / keys of this CTA: one group, or up to `pack` consecutive groups
  const int span = packed ? min(prm.pack, prm.n_groups - group) * seq : seq;
  const int n_kv = (span + kKV - 1) / kKV;
  const int hx = head * prm.in_hstride;  // column of this head in the Q/K/V maps

  if ((smem_u32(smem) & 1023u) != 0) {  // the swizzled layouts need 1 KiB alignment
    if (threadIdx.x == 0) atomicCAS(&g_dev_error, 0u, static_cast<unsigned>(kErrTmemAlloc));
    return;
  }
  uint8_t* sQ = smem;
  auto sK = [&](int st) { return smem + kTile + 2 * st * HC::kKVTile; };
  auto sV = [&](int st) { return smem + kTile + (2 * st + 1) * HC::kKVTile; };
  auto sdesc_k = [](uint32_t a) { return kD == 64 ? make_sdesc_sw128(a) : make_sdesc_sw64(a); };
  auto sdesc_mn = [](uint32_t a) { return kD == 64 ? make_sdesc_sw128_mn(a) : make_sdesc_sw64_mn(a); };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int b = 0; b < kNB; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], kSoftWarps);
      mbar_init(&p_full[b], kSoftWarps);
      mbar_init(&p_empty[b], 1);
    }
    mbar_init(o_full, 1);
    abort_flag_s = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t tO = tmem + 128;
  auto tS = [&](int b) { return tmem + static_cast<uint32_t>(b * kKV); };
  auto tP = [&](int b) { return tmem + 192u + static_cast<uint32_t>(b * (kKV / 2)); };

  if (warp == 0) {
    // TMA producer: the whole warp runs the loop, one elected lane issues
    if (elect_one()) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_arrive_expect_tx(q_full, kTile);
      tma_load_2d(sQ, &tq, q_full, hx, row0 + qt * kQ);
    }
    __syncwarp();
    for (int j = 0; j < n_kv; ++j) {
      const int st = j % kStages;
      if (!mbar_wait_warp(&kv_empty[st], ((j / kStages) & 1) ^ 1, kErrStageFree, abort_flag)) break;
      if (elect_one()) {
        mbar_arrive_expect_tx(&kv_full[st], 2 * HC::kKVTile);
        tma_load_2d(sK(st), &tk, &kv_full[st], hx, row0 + j * kKV);
        tma_load_2d(sV(st), &tv, &kv_full[st], hx, row0 + j * kKV);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // MMA issuer: the whole warp runs the loop (operands stay warp-uniform),
    // one elected lane issues each tcgen05.mma / commit
    const uint32_t fmt = kBf16 ? 1u : 0u;
    const uint32_t idesc_pv = make_idesc(fmt, kQ, kD, 1u);
    bool ok = mbar_wait_warp(q_full, 0, kErrTmaWait, abort_flag);
    const uint64_t qdesc = sdesc_k(smem_u32(sQ));
    auto keys_in = [&](int j) {  // keys of tile j, rounded up to a multiple of 16
      const int left = span - j * kKV;
      return left >= kKV ? kKV : ((left + 15) & ~15);
    };
    // S_j = Q K_j^T into TMEM once K_j landed and the softmax read S_{j-1}
    auto issue_s = [&](int j) -> bool {
      const int st = j % kStages, b = j % kNB;
      if (!mbar_wait_warp(&kv_full[st], (j / kStages) & 1, kErrTmaWait, abort_flag)) return false;
      if (!mbar_wait_warp(&s_empty[b], ((j / kNB) & 1) ^ 1, kErrAccFree, abort_flag)) return false;
      tc_fence_after();
      const uint64_t kdesc = sdesc_k(smem_u32(sK(st)));
      const uint32_t idesc_s = make_idesc(fmt, kQ, keys_in(j));
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk)  // 16 elements = 32 bytes along K
        umma_ss_warp(tS(b), qdesc + 2 * kk, kdesc + 2 * kk, idesc_s, kk ? 1u : 0u);
      umma_commit_warp(&s_full[b]);
      return true;
    };
    if (ok) ok = issue_s(0);
    if (ok && kNB == 2 && n_kv > 1) ok = issue_s(1);
    for (int j = 0; ok && j < n_kv; ++j) {
      // the next S = Q K^T runs while the softmax of tile j is computed
      // (double-buffered: S_{j+1} is already issued, S_{j+2} follows P_j.V_j)
      if (kNB == 1 && j + 1 < n_kv && !issue_s(j + 1)) break;
      const int pb = j % kNB;
      if (!mbar_wait_warp(&p_full[pb], (j / kNB) & 1, kErrAccFull, abort_flag)) break;
      tc_fence_after();
      const int st = j % kStages, n = keys_in(j);
      const uint64_t vdesc = sdesc_mn(smem_u32(sV(st)));
      constexpr uint32_t kVStep = 16 * HC::kRowBytes >> 4;  // 16 keys of V, in descriptor units
      if (n == kKV) {
#pragma unroll
        for (int kk = 0; kk < kKV / 16; ++kk)  // A = P from TMEM: 16 keys = 8 columns
          umma_ts_warp(tO, tP(pb) + kk * 8, vdesc + kk * kVStep, idesc_pv, (j | kk) ? 1u : 0u);
      } else {
        for (int kk = 0; kk < n / 16; ++kk)
          umma_ts_warp(tO, tP(pb) + kk * 8, vdesc + kk * kVStep, idesc_pv, (j | kk) ? 1u : 0u);
      }
      umma_commit_warp(&p_empty[pb]);
      umma_commit_warp(&kv_empty[st]);
      if (kNB == 2 && j + 2 < n_kv && !issue_s(j + 2)) break;
    }
    umma_commit_warp(o_full);
  } else {
    // ------------------------------------------------ softmax + epilogue
    // warp w: TMEM lane quarter w % 4 (hardware rule), column half (w-2)/4
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t scol = half * kHalf;  // first S column / key of this warp
    // With a bias the scores are scaled (and biased) on load; the softmax
    // then works on them with the plain log2(e) factor.
    const float sl2 = kBias ? 1.4426950408889634f : prm.scale_log2;
    // packed tiles: this row's group occupies keys [klo, klo + seq) of the
    // tile; with a bias the table is per tile row (block-diagonal, -inf
    // between groups), so it carries the mask itself
    const int qrow_t = min(qt * kQ + r, span - 1);
    const int klo = packed ? (qrow_t / seq) * seq : 0;
    const int brows = packed ? prm.pack * seq : seq;  // rows of the bias table per head
    const int kend = packed ? span : seq;             // keys that exist in this tile
    const float* brow = nullptr;
    if constexpr (kBias) brow = prm.bias + (static_cast<int64_t>(head) * brows + qrow_t) * prm.bias_ld;
    // S columns [c0, c0+64) of key tile j -> sv (scaled and biased if kBias,
    // keys >= seq set to -inf)
    int sb = 0;  // S buffer of the current tile
    auto load_s = [&](float* sv, uint32_t* su, uint32_t c0, int kfirst) {
#pragma unroll
      for (int c = 0; c < kHalf / 32; ++c)
        tmem_ld_32x32b_x32(tS(sb) + lane_off + c0 + c * 32, *reinterpret_cast<uint32_t(*)[32]>(su + c * 32));
      tmem_ld_wait();
      if constexpr (kBias) {
#pragma unroll
        for (int c = 0; c < kHalf; c += 4) {
          if (kfirst + c < kend) {  // bias rows are padded to a multiple of 4
            const float4 b = __ldg(reinterpret_cast<const float4*>(brow + kfirst + c));
            sv[c] = fmaf(sv[c], prm.scale, b.x);
            sv[c + 1] = fmaf(sv[c + 1], prm.scale, b.y);
            sv[c + 2] = fmaf(sv[c + 2], prm.scale, b.z);
            sv[c + 3] = fmaf(sv[c + 3], prm.scale, b.w);
          }
        }
      } else if (packed) {  // block-diagonal: keys of the row's own group only
#pragma unroll
        for (int c = 0; c < kHalf; ++c) {
          const int k = kfirst + c - klo;
          if (k < 0 || k >= seq) sv[c] = -INFINITY;
        }
      }
      if (kfirst + kHalf > kend) {  // ragged last tile: keys >= kend do not exist
#pragma unroll
        for (int c = 0; c < kHalf; ++c)
          if (kfirst + c >= kend) sv[c] = -INFINITY;
      }
    };
    auto max_row = [](const float* v) { return kHalf == 64 ? max64(v) : fmaxf(max64(v), max64(v + 64)); };
    float m_used = -INFINITY, l = 0.f;
    // A warp whose 32 query rows all lie past the group end (the last query
    // tile of a 576-token window) only keeps the barrier protocol going.
    const bool rows_live = qt * kQ + quarter * 32 < span;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      sb = j % kNB;
      if (!warp_wait(&s_full[sb], (j / kNB) & 1, kErrAccFull, abort_flag, lane)) { ok = false; break; }
      tc_fence_after();
      const int kb = j * kKV + scol;
      // keys of this half exist (the ragged last tile of a window has none
      // in its upper half; P.V then reads only the lower half of P)
      const bool live = rows_live && kb < span;
      uint32_t su[kHalf];  // S bits, loaded in place
      float* sv = reinterpret_cast<float*>(su);
      float mt = -INFINITY;
      if (kSplit == 2 && rows_live) {
        // maximum of the other key half first (its values are discarded)
        const int kbo = j * kKV + (scol ^ kHalf);
        if (kbo < span) {
          load_s(sv, su, scol ^ kHalf, kbo);
          mt = max_row(sv);
        }
      }
      if (live) load_s(sv, su, scol, kb);  // this warp's 64 S columns
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);  // S may be overwritten
      if (live) mt = fmaxf(mt, max_row(sv));
      const bool need = (mt - m_used) * sl2 > kRescaleLog2;
      // P buffer sb is free once the P.V of tile j - kNB finished (with one
      // buffer: the previous P.V, which also leaves O quiescent)
      if (j >= kNB && !warp_wait(&p_empty[sb], ((j / kNB) & 1) ^ 1, kErrAccFree, abort_flag, lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (__any_sync(0xffffffffu, need)) {  // same rows, same verdict in both halves
        const float m_new = fmaxf(m_used, mt);
        const float corr = (m_used == -INFINITY) ? 0.f : ex2((m_used - m_new) * sl2);
        l *= corr;
        m_used = m_new;
        // two buffers: O is quiescent once the P.V of tile j - 1 finished too
        if (kNB == 2 && j > 0 &&
            !warp_wait(&p_empty[(j - 1) % kNB], ((j - 1) / kNB) & 1, kErrAccFree, abort_flag, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (j > 0) {  // this half rescales O columns [kOHalf*half, kOHalf*(half+1))
#pragma unroll
          for (int c = 0; c < kOHalf / 8; ++c) {  // 8 columns at a time: few live registers
            uint32_t u[8];
            tmem_ld_32x32b_x8(tO + lane_off + half * kOHalf + c * 8, u);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 8; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * corr);
            tmem_st_32x32b_x8(tO + lane_off + half * kOHalf + c * 8, u);
          }
          tmem_st_wait();
        }
      }
      // P = exp2(S*c - m) -> 16-bit pairs into TMEM columns 192 + 32*half
      if (live) {
        const float mb = m_used * sl2;
        // e = S*c - m and the row sums on packed f32x2 lanes (keys c, c+1)
        const uint64_t sc2 = f2pack(sl2, sl2), nmb2 = f2pack(-mb, -mb);
        uint64_t l2[2] = {f2pack(0.f, 0.f), f2pack(0.f, 0.f)};
#pragma unroll
        for (int c0 = 0; c0 < kHalf; c0 += 2 * kPStore) {  // 2*kPStore keys -> kPStore P columns
          uint32_t pk[kPStore];
#pragma unroll
          for (int c = c0; c < c0 + 2 * kPStore; c += 2) {
            const uint64_t e2 = ffma2(f2pack(sv[c], sv[c + 1]), sc2, nmb2);
            float p0, p1;
            if (((c - c0) / 2) % 8 < kPolyPairs) {
              exp2_poly2(e2, p0, p1);
            } else {
              float e0, e1;
              f2unpack(e2, e0, e1);
              p0 = ex2(e0);
              p1 = ex2(e1);
            }
            l2[(c >> 1) & 1] = fadd2(l2[(c >> 1) & 1], f2pack(p0, p1));
            pk[(c - c0) / 2] = pack2(p0, p1, kBf16);
          }
          const uint32_t ta = tP(sb) + lane_off + half * (kHalf / 2) + c0 / 2;
          if constexpr (kPStore == 8)
            tmem_st_32x32b_x8(ta, *reinterpret_cast<const uint32_t(*)[8]>(pk));
          else if constexpr (kPStore == 16)
            tmem_st_32x32b_x16(ta, *reinterpret_cast<const uint32_t(*)[16]>(pk));
          else
            tmem_st_32x32b_x32(ta, *reinterpret_cast<const uint32_t(*)[32]>(pk));
        }
        float a0, a1;
        f2unpack(fadd2(l2[0], l2[1]), a0, a1);
        l += a0 + a1;
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    // all MMAs done: O complete, S columns free for the row-sum exchange
    // (both warps of a quarter reach the exchange, also after an abort)
    const bool o_ok = ok && warp_wait(o_full, 0, kErrAccFull, abort_flag, lane);
    tc_fence_after();
    if (kSplit == 2 && rows_live) l += pair_exchange(tS(0), lane_off, half, l, quarter);
    if (o_ok) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int qrow = qt * kQ + r;
      uint16_t* orow = prm.o + static_cast<int64_t>(row0 + qrow) * prm.ldo + head * prm.o_hstride + half * kOHalf;
#pragma unroll
      for (int c0 = 0; c0 < kOHalf; c0 += 16) {  // 16 output columns at a time
        uint32_t u[16];
        tmem_ld_32x32b_x16(tO + lane_off + half * kOHalf + c0, u);
        tmem_ld_wait();
        if (qrow < span) {
#pragma unroll
          for (int q4 = 0; q4 < 2; ++q4) {
            uint4 w;
            w.x = pack2(__uint_as_float(u[q4 * 8 + 0]) * inv, __uint_as_float(u[q4 * 8 + 1]) * inv, kBf16);
            w.y = pack2(__uint_as_float(u[q4 * 8 + 2]) * inv, __uint_as_float(u[q4 * 8 + 3]) * inv, kBf16);
            w.z = pack2(__uint_as_float(u[q4 * 8 + 4]) * inv, __uint_as_float(u[q4 * 8 + 5]) * inv, kBf16);
            w.w = pack2(__uint_as_float(u[q4 * 8 + 6]) * inv, __uint_as_float(u[q4 * 8 + 7]) * inv, kBf16);
            *reinterpret_cast<uint4*>(orow + c0 + q4 * 8) = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// What one work item (one 128-row query tile of one group, one head) covers.
struct AttnItem {
  int head, qt, row0, span, n_kv;
};
__device__ __forceinline__ AttnItem attn_item(const AttnParams& prm, int item) {
  AttnItem it;
  const int x = item % prm.n_x;
  it.head = item / prm.n_x;
  const bool packed = prm.pack > 1;
  const int group = packed ? x * prm.pack : x / prm.q_tiles;
  it.qt = packed ? 0 : x % prm.q_tiles;
  it.row0 = group * prm.seq;  // first row of the (first) group in the [rows, ld] matrices
  // rows / keys of this item: one group, or up to `pack` consecutive groups
  it.span = packed ? min(prm.pack, prm.n_groups - group) * prm.seq : prm.seq;
  it.n_kv = (it.span + kKV - 1) / kKV;
  return it;
}

// Two CTAs of 6 warps per SM.  Each CTA loops over work items
// blockIdx.x, blockIdx.x + gridDim.x, ...: the next item's Q load and first
// S = QK^T overlap the current item's last softmax and output epilogue.
// kBf16: Q/K/V/P/O are bf16, else f16.  kD: head dim.  kBias: an additive
// f32 bias [head, query, key] joins the scaled scores before the softmax
// (TinyViT's relative position bias, image_encoder_tinyvit.c:842-846).
template <bool kBf16, int kD, bool kBias>
__global__ void __launch_bounds__(kThreads, 2)
    attn_tc_persist_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const AttnParams prm) {
  using HC = HeadCfg<kD>;
  constexpr int kTile = HC::kTile;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint64_t bars[12 + 2 * kStages];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag_s;
  uint64_t* q_full = &bars[0];
  uint64_t* o_full = &bars[1];
  uint64_t* q_empty = &bars[2];              // all S MMAs of an item done: Q may be replaced
  uint64_t* o_empty = &bars[3];              // the epilogue read O: the next item may overwrite it
  uint64_t* s_full = &bars[4];               // [kNB]
  uint64_t* s_empty = &bars[6];              // [kNB]
  uint64_t* p_full = &bars[8];               // [kNB]
  uint64_t* p_empty = &bars[10];             // [kNB]
  uint64_t* kv_full = &bars[12];             // [kStages]
  uint64_t* kv_empty = &bars[12 + kStages];  // [kStages]
  volatile int* abort_flag = &abort_flag_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool packed = prm.pack > 1;
  const int kItemEnd = prm.n_items;

  if ((smem_u32(smem) & 1023u) != 0) {  // the swizzled layouts need 1 KiB alignment
    if (threadIdx.x == 0) atomicCAS(&g_dev_error, 0u, static_cast<unsigned>(kErrTmemAlloc));
    return;
  }
  uint8_t* sQ = smem;
  auto sK = [&](int st) { return smem + kTile + 2 * st * HC::kKVTile; };
  auto sV = [&](int st) { return smem + kTile + (2 * st + 1) * HC::kKVTile; };
  auto sdesc_k = [](uint32_t a) { return kD == 64 ? make_sdesc_sw128(a) : make_sdesc_sw64(a); };
  auto sdesc_mn = [](uint32_t a) { return kD == 64 ? make_sdesc_sw128_mn(a) : make_sdesc_sw64_mn(a); };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int b = 0; b < kNB; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], kSoftWarps);
      mbar_init(&p_full[b], kSoftWarps);
      mbar_init(&p_empty[b], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(o_empty, kSoftWarps);
    abort_flag_s = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t tO = tmem + 128;
  auto tS = [&](int b) { return tmem + static_cast<uint32_t>(b * kKV); };
  auto tP = [&](int b) { return tmem + 192u + static_cast<uint32_t>(b * (kKV / 2)); };

  if (warp == 0) {
    // TMA producer: the whole warp runs the loop, one elected lane issues
    if (elect_one()) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
    }
    __syncwarp();
    int t = 0;  // K/V tiles loaded so far, over all items of this CTA
    bool ok = true;
    for (int item = blockIdx.x, n = 0; ok && item < kItemEnd; item += gridDim.x, ++n) {
      const AttnItem it = attn_item(prm, item);
      const int hx = it.head * prm.in_hstride;  // column of this head in the Q/K/V maps
      // Q of the previous item is in use until its last S MMA completed
      if (n > 0 && !mbar_wait_warp(q_empty, (n - 1) & 1, kErrStageFree, abort_flag)) break;
      if (elect_one()) {
        mbar_arrive_expect_tx(q_full, kTile);
        tma_load_2d(sQ, &tq, q_full, hx, it.row0 + it.qt * kQ);
      }
      __syncwarp();
      for (int j = 0; j < it.n_kv; ++j, ++t) {
        const int st = t % kStages;
        if (!mbar_wait_warp(&kv_empty[st], ((t / kStages) & 1) ^ 1, kErrStageFree, abort_flag)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          mbar_arrive_expect_tx(&kv_full[st], 2 * HC::kKVTile);
          tma_load_2d(sK(st), &tk, &kv_full[st], hx, it.row0 + j * kKV);
          tma_load_2d(sV(st), &tv, &kv_full[st], hx, it.row0 + j * kKV);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // MMA issuer: the whole warp runs the loop (operands stay warp-uniform),
    // one elected lane issues each tcgen05.mma / commit
    const uint32_t fmt = kBf16 ? 1u : 0u;
    const uint32_t idesc_pv = make_idesc(fmt, kQ, kD, 1u);
    const uint64_t qdesc = sdesc_k(smem_u32(sQ));
    int t = 0;  // K/V tiles consumed over all items: ring stage and S / P phases
    bool ok = true;
    for (int item = blockIdx.x, n = 0; ok && item < kItemEnd; item += gridDim.x, ++n) {
      const AttnItem it = attn_item(prm, item);
      auto keys_in = [&](int j) {  // keys of tile j, rounded up to a multiple of 16
        const int left = it.span - j * kKV;
        return left >= kKV ? kKV : ((left + 15) & ~15);
      };
      // S_j = Q K_j^T into TMEM once K_j landed and the softmax read S_{j-1}
      auto issue_s = [&](int j, int tt) -> bool {
        const int st = tt % kStages, b = tt % kNB;
        if (!mbar_wait_warp(&kv_full[st], (tt / kStages) & 1, kErrTmaWait, abort_flag)) return false;
        if (!mbar_wait_warp(&s_empty[b], ((tt / kNB) & 1) ^ 1, kErrAccFree, abort_flag)) return false;
        tc_fence_after();
        const uint64_t kdesc = sdesc_k(smem_u32(sK(st)));
        const uint32_t idesc_s = make_idesc(fmt, kQ, keys_in(j));
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)  // 16 elements = 32 bytes along K
          umma_ss_warp(tS(b), qdesc + 2 * kk, kdesc + 2 * kk, idesc_s, kk ? 1u : 0u);
        umma_commit_warp(&s_full[b]);
        if (j == it.n_kv - 1) umma_commit_warp(q_empty);  // the item's last read of Q
        return true;
      };
      if (!mbar_wait_warp(q_full, n & 1, kErrTmaWait, abort_flag) || !issue_s(0, t)) break;
      if (kNB == 2 && it.n_kv > 1 && !issue_s(1, t + 1)) break;
      for (int j = 0; j < it.n_kv; ++j, ++t) {
        // the next S = Q K^T runs while the softmax of tile j is computed
        // (double-buffered: S_{j+1} is already issued, S_{j+2} follows P_j.V_j)
        if (kNB == 1 && j + 1 < it.n_kv && !issue_s(j + 1, t + 1)) { ok = false; break; }
        const int pb = t % kNB;
        if (!mbar_wait_warp(&p_full[pb], (t / kNB) & 1, kErrAccFull, abort_flag)) { ok = false; break; }
        // the first P.V of an item overwrites O: the epilogue of the previous
        // item must have read it
        if (j == 0 && n > 0 && !mbar_wait_warp(o_empty, (n - 1) & 1, kErrAccFree, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int st = t % kStages, nk = keys_in(j);
        const uint64_t vdesc = sdesc_mn(smem_u32(sV(st)));
        constexpr uint32_t kVStep = 16 * HC::kRowBytes >> 4;  // 16 keys of V, in descriptor units
        if (nk == kKV) {
#pragma unroll
          for (int kk = 0; kk < kKV / 16; ++kk)  // A = P from TMEM: 16 keys = 8 columns
            umma_ts_warp(tO, tP(pb) + kk * 8, vdesc + kk * kVStep, idesc_pv, (j | kk) ? 1u : 0u);
        } else {
          for (int kk = 0; kk < nk / 16; ++kk)
            umma_ts_warp(tO, tP(pb) + kk * 8, vdesc + kk * kVStep, idesc_pv, (j | kk) ? 1u : 0u);
        }
        umma_commit_warp(&p_empty[pb]);
        umma_commit_warp(&kv_empty[st]);
        if (kNB == 2 && j + 2 < it.n_kv && !issue_s(j + 2, t + 2)) { ok = false; break; }
      }
      if (ok) umma_commit_warp(o_full);
    }
  } else {
    // ------------------------------------------------ softmax + epilogue
    // warp w: TMEM lane quarter w % 4 (hardware rule): query rows
    // 32*(w%4) .. +31; a thread holds its whole 128-key S row, so the row
    // maximum and sum need no exchange
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    // With a bias the scores are scaled (and biased) on load; the softmax
    // then works on them with the plain log2(e) factor.
    const float sl2 = kBias ? 1.4426950408889634f : prm.scale_log2;
    int t = 0;  // S / P phases over all items
    bool ok = true;
    for (int item = blockIdx.x, n = 0; ok && item < kItemEnd; item += gridDim.x, ++n) {
      const AttnItem it = attn_item(prm, item);
      const int span = it.span;
      // packed tiles: this row's group occupies keys [klo, klo + seq) of the
      // tile; with a bias the table is per tile row (block-diagonal, -inf
      // between groups), so it carries the mask itself
      const int qrow_t = min(it.qt * kQ + r, span - 1);
      const int klo = packed ? (qrow_t / prm.seq) * prm.seq : 0;
      const int brows = packed ? prm.pack * prm.seq : prm.seq;  // rows of the bias table per head
      const int kend = packed ? span : prm.seq;                 // keys that exist in this tile
      const float* brow = nullptr;
      if constexpr (kBias) brow = prm.bias + (static_cast<int64_t>(it.head) * brows + qrow_t) * prm.bias_ld;
      // S columns of key tile j -> sv (scaled and biased if kBias, keys >= seq
      // set to -inf)
      auto load_s = [&](float* sv, uint32_t* su, int kfirst, int b) {
#pragma unroll
        for (int c = 0; c < kKV / 32; ++c)
          tmem_ld_32x32b_x32(tS(b) + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(su + c * 32));
        tmem_ld_wait();
        if constexpr (kBias) {
#pragma unroll
          for (int c = 0; c < kKV; c += 4) {
            if (kfirst + c < kend) {  // bias rows are padded to a multiple of 4
              const float4 b = __ldg(reinterpret_cast<const float4*>(brow + kfirst + c));
              sv[c] = fmaf(sv[c], prm.scale, b.x);
              sv[c + 1] = fmaf(sv[c + 1], prm.scale, b.y);
              sv[c + 2] = fmaf(sv[c + 2], prm.scale, b.z);
              sv[c + 3] = fmaf(sv[c + 3], prm.scale, b.w);
            }
          }
        } else if (packed) {  // block-diagonal: keys of the row's own group only
#pragma unroll
          for (int c = 0; c < kKV; ++c) {
            const int k = kfirst + c - klo;
            if (k < 0 || k >= prm.seq) sv[c] = -INFINITY;
          }
        }
        if (kfirst + kKV > kend) {  // ragged last tile: keys >= kend do not exist
#pragma unroll
          for (int c = 0; c < kKV; ++c)
            if (kfirst + c >= kend) sv[c] = -INFINITY;
        }
      };
      float m_used = -INFINITY, l = 0.f;
      // A warp whose 32 query rows all lie past the group end (the last query
      // tile of a 576-token window) only keeps the barrier protocol going.
      const bool live = it.qt * kQ + quarter * 32 < span;
      for (int j = 0; j < it.n_kv; ++j, ++t) {
        const int sb = t % kNB;
        if (!warp_wait(&s_full[sb], (t / kNB) & 1, kErrAccFull, abort_flag, lane)) { ok = false; break; }
        tc_fence_after();
        uint32_t su[kKV];  // S bits, loaded in place
        float* sv = reinterpret_cast<float*>(su);
        if (live) load_s(sv, su, j * kKV, sb);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[sb]);  // S may be overwritten
        const float mt = live ? (kKV == 64 ? max64(sv) : max128(sv)) : -INFINITY;
        const bool need = (mt - m_used) * sl2 > kRescaleLog2;
        // P buffer sb is free once the P.V of tile t - kNB finished (one
        // buffer: the previous P.V, which also leaves O quiescent; for j = 0
        // that P.V may belong to the previous item, finished before its
        // o_full)
        if (t >= kNB && !warp_wait(&p_empty[sb], ((t / kNB) & 1) ^ 1, kErrAccFree, abort_flag, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
          const float m_new = fmaxf(m_used, mt);
          const float corr = (m_used == -INFINITY) ? 0.f : ex2((m_used - m_new) * sl2);
          l *= corr;
          m_used = m_new;
          // two buffers: O is quiescent once the P.V of tile t - 1 finished too
          if (kNB == 2 && j > 0 &&
              !warp_wait(&p_empty[(t - 1) % kNB], ((t - 1) / kNB) & 1, kErrAccFree, abort_flag, lane)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (j > 0) {
#pragma unroll
            for (int c = 0; c < kD / 8; ++c) {  // 8 columns at a time: few live registers
              uint32_t u[8];
              tmem_ld_32x32b_x8(tO + lane_off + c * 8, u);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 8; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * corr);
              tmem_st_32x32b_x8(tO + lane_off + c * 8, u);
            }
            tmem_st_wait();
          }
        }
        // P = exp2(S*c - m) -> 16-bit pairs into TMEM columns 192..255
        if (live) {
          const float mb = m_used * sl2;
          // e = S*c - m and the row sums on packed f32x2 lanes (keys c, c+1)
          const uint64_t sc2 = f2pack(sl2, sl2), nmb2 = f2pack(-mb, -mb);
          uint64_t l2[2] = {f2pack(0.f, 0.f), f2pack(0.f, 0.f)};
#pragma unroll
          for (int c0 = 0; c0 < kKV; c0 += 16) {  // 16 keys -> 8 P columns
            uint32_t pk[8];
#pragma unroll
            for (int c = c0; c < c0 + 16; c += 2) {
              const uint64_t e2 = ffma2(f2pack(sv[c], sv[c + 1]), sc2, nmb2);
              float p0, p1;
              if ((c - c0) / 2 < kPolyPairs) {
                exp2_poly2(e2, p0, p1);
              } else {
                float e0, e1;
                f2unpack(e2, e0, e1);
                p0 = ex2(e0);
                p1 = ex2(e1);
              }
              l2[(c >> 1) & 1] = fadd2(l2[(c >> 1) & 1], f2pack(p0, p1));
              pk[(c - c0) / 2] = pack2(p0, p1, kBf16);
            }
            tmem_st_32x32b_x8(tP(sb) + lane_off + c0 / 2, *reinterpret_cast<const uint32_t(*)[8]>(pk));
          }
          float a0, a1;
          f2unpack(fadd2(l2[0], l2[1]), a0, a1);
          l += a0 + a1;
          tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[sb]);
      }
      // all MMAs of the item done: O complete
      if (!ok || !warp_wait(o_full, n & 1, kErrAccFull, abort_flag, lane)) break;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int qrow = it.qt * kQ + r;
      uint16_t* orow = prm.o + static_cast<int64_t>(it.row0 + qrow) * prm.ldo + it.head * prm.o_hstride;
#pragma unroll
      for (int c0 = 0; c0 < kD; c0 += 16) {  // 16 output columns at a time
        uint32_t u[16];
        tmem_ld_32x32b_x16(tO + lane_off + c0, u);
        tmem_ld_wait();
        if (qrow < span) {
#pragma unroll
          for (int q4 = 0; q4 < 2; ++q4) {
            uint4 w;
            w.x = pack2(__uint_as_float(u[q4 * 8 + 0]) * inv, __uint_as_float(u[q4 * 8 + 1]) * inv, kBf16);
            w.y = pack2(__uint_as_float(u[q4 * 8 + 2]) * inv, __uint_as_float(u[q4 * 8 + 3]) * inv, kBf16);
            w.z = pack2(__uint_as_float(u[q4 * 8 + 4]) * inv, __uint_as_float(u[q4 * 8 + 5]) * inv, kBf16);
            w.w = pack2(__uint_as_float(u[q4 * 8 + 6]) * inv, __uint_as_float(u[q4 * 8 + 7]) * inv, kBf16);
            *reinterpret_cast<uint4*>(orow + c0 + q4 * 8) = w;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);  // O may be overwritten by the next item
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// [rows, width] 16-bit matrix of row pitch ld, boxes of 128 rows x head_dim
// columns (128- or 64-byte swizzle, matching the kernel's descriptors).
bool make_head_map(CUtensorMap* m, const void* base, int dtype, int64_t rows, int64_t width, int64_t ld,
                   int head_dim, int box_rows) {
  const CUtensorMapDataType dt = dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return make_tmap_2d(m, base, dt, 2, rows, width, ld, box_rows, head_dim,
                      head_dim == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

template <bool kBf16, int kD, bool kBias>
int launch_variant(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnParams& prm,
                   dim3 grid, bool persist, cudaStream_t st) {
  constexpr int smem = HeadCfg<kD>::kSmem;
  static bool done = false;
  if (!done) {
    for (const void* f : {reinterpret_cast<const void*>(attn_tc_kernel<kBf16, kD, kBias>),
                          reinterpret_cast<const void*>(attn_tc_persist_kernel<kBf16, kD, kBias>)}) {
      cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      // full shared-memory carveout, so two CTAs fit on one SM
      cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    }
    done = true;
  }
  if (persist)
    attn_tc_persist_kernel<kBf16, kD, kBias><<<grid, kThreads, smem, st>>>(mq, mk, mv, prm);
  else
    attn_tc_kernel<kBf16, kD, kBias><<<grid, kThreads, smem, st>>>(mq, mk, mv, prm);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

int launch_attention_tc_ex(const AttnArgs& a, cudaStream_t st) {
  if (a.head_dim != 64 && a.head_dim != 32) return kErrShape;
  if (a.dtype != kBF16 && a.dtype != kF16) return kErrDtype;
  const int in_hs = a.in_hstride > 0 ? a.in_hstride : a.head_dim;
  const int o_hs = a.o_hstride > 0 ? a.o_hstride : a.head_dim;
  // TMA: 16-byte row pitch and column starts; vector output stores
  if (a.ldq % 8 || a.ldo % 8 || in_hs % 8 || o_hs % 8 || (reinterpret_cast<uintptr_t>(a.o) & 15)) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v)) & 15)
    return kErrShape;
  if (a.bias && (a.bias_ld % 4 || a.bias_ld < a.seq || (reinterpret_cast<uintptr_t>(a.bias) & 15))) return kErrShape;
  if (a.n_groups <= 0 || a.seq <= 0 || a.heads <= 0) return kOk;
  const int64_t rows = static_cast<int64_t>(a.n_groups) * a.seq;
  if (rows > 0x7fffffffLL) return kErrShape;
  const int64_t width = static_cast<int64_t>(a.heads - 1) * in_hs + a.head_dim;  // last head ends here
  CUtensorMap mq, mk, mv;
  if (!make_head_map(&mq, a.q, a.dtype, rows, width, a.ldq, a.head_dim, kQ) ||
      !make_head_map(&mk, a.k, a.dtype, rows, width, a.ldq, a.head_dim, kKV) ||
      !make_head_map(&mv, a.v, a.dtype, rows, width, a.ldq, a.head_dim, kKV))
    return kErrTma;
  AttnParams prm;
  prm.o = static_cast<uint16_t*>(a.o);
  prm.ldo = a.ldo;
  prm.o_hstride = o_hs;
  prm.in_hstride = in_hs;
  prm.seq = a.seq;
  prm.q_tiles = (a.seq + kQ - 1) / kQ;
  prm.n_groups = a.n_groups;
  prm.scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf(static_cast<float>(a.head_dim));
  prm.scale_log2 = prm.scale * 1.4426950408889634f;
  prm.bias = a.bias;
  prm.bias_ld = a.bias_ld;
  // short groups (TinyViT's 7x7 windows): several per 128-row tile, when
  // there is no bias or the caller supplies the per-tile bias table
  prm.pack = (a.seq <= kQ / 2 && (!a.bias || a.bias_tile)) ? kQ / a.seq : 1;
  if (prm.pack > 1 && a.bias_tile) {
    if (a.bias_tile_ld % 4 || a.bias_tile_ld < prm.pack * a.seq || (reinterpret_cast<uintptr_t>(a.bias_tile) & 15))
      return kErrShape;
    prm.bias = a.bias_tile;
    prm.bias_ld = a.bias_tile_ld;
  }
  prm.n_x = prm.pack > 1 ? (a.n_groups + prm.pack - 1) / prm.pack : a.n_groups * prm.q_tiles;
  if (static_cast<int64_t>(prm.n_x) * a.heads > 0x7fffffffLL) return kErrShape;
  prm.n_items = prm.n_x * a.heads;
  // Short items (windows: a few key tiles each) go to the persistent kernel:
  // two resident CTAs per SM loop over them, so one item's prologue and
  // epilogue overlap the next; long items (global attention) keep one CTA
  // each, which the hardware schedules dynamically.  S3CU_ATTN_PERSIST=0/1
  // forces the choice (for measurements).  Measured at 8 images: window
  // attention 417 -> 438 TFLOP/s; global unchanged.
  static const int force = [] {
    const char* e = getenv("S3CU_ATTN_PERSIST");
    return e ? atoi(e) : -1;
  }();
  const int n_kv = ((prm.pack > 1 ? prm.pack * a.seq : a.seq) + 127) / 128;  // in 128-key units
  // (Not with a bias: the biased variant spills in the persistent form and
  // measured slower on TinyViT.)
  const bool persist = force >= 0 ? force != 0 : (n_kv <= 8 && !a.bias);
  const int ctas = 2 * num_sms();
  dim3 grid = persist ? dim3(prm.n_items < ctas ? prm.n_items : ctas)
                      : dim3(prm.n_x, a.heads);
  count_launches(1);
  const bool bf = a.dtype == kBF16, b = a.bias != nullptr;
  if (a.head_dim == 64) {
    if (b) return bf ? launch_variant<true, 64, true>(mq, mk, mv, prm, grid, persist, st)
                     : launch_variant<false, 64, true>(mq, mk, mv, prm, grid, persist, st);
    return bf ? launch_variant<true, 64, false>(mq, mk, mv, prm, grid, persist, st)
              : launch_variant<false, 64, false>(mq, mk, mv, prm, grid, persist, st);
  }
  if (b) return bf ? launch_variant<true, 32, true>(mq, mk, mv, prm, grid, persist, st)
                   : launch_variant<false, 32, true>(mq, mk, mv, prm, grid, persist, st);
  return bf ? launch_variant<true, 32, false>(mq, mk, mv, prm, grid, persist, st)
            : launch_variant<false, 32, false>(mq, mk, mv, prm, grid, persist, st);
}

int launch_attention_tc(const void* q, const void* k, const void* v, int64_t ldq, void* o, int64_t ldo, int dtype,
                        int n_groups, int seq, int heads, int head_dim, cudaStream_t st) {
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.q = q;
  a.k = k;
  a.v = v;
  a.ldq = ldq;
  a.o = o;
  a.ldo = ldo;
  a.dtype = dtype;
  a.n_groups = n_groups;
  a.seq = seq;
  a.heads = heads;
  a.head_dim = head_dim;
  return launch_attention_tc_ex(a, st);
}

}  // namespace s3
