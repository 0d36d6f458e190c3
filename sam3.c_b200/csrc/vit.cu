// vit.cu - the sam3.c ViT image encoder (sam3_vit_build,
// src/model/image_encoder.c:513-963) lowered to fused sm_100a kernels.
//
// Token order.  The residual stream is kept in WINDOW-MAJOR order for the
// whole forward: row r of an image is window r / (ws*ws), slot r % (ws*ws).
// The reference instead partitions and un-partitions every windowed block
// (gh_window_partition / gh_window_unpartition, graph_helpers.c:444-514,
// two full-activation permutes per block).  LayerNorm and the MLP act per
// token and global attention attends over all tokens of an image, so only
// two things depend on the order: the global RoPE position of a row (looked
// up through win_to_raster) and the final output (written back in raster
// order by the last GEMM's epilogue).  The permutation therefore costs
// nothing at run time.
//
// Per block (M = images * 5184 rows; T = bf16 or f16):
//   LN1      x f32 -> xn T
//   QKV GEMM xn . Wqkv^T + b, RoPE on Q and K columns -> qkv T [M, 3e]
//   SDPA     per (window|image, head) -> ao T [M, e]
//   PROJ     ao . Wproj^T + b + x -> x f32
//   LN2      x -> xn T
//   FC1      xn . Wfc1^T + b, tanh-GELU -> h T [M, mlp]
//   FC2      h . Wfc2^T + b + x -> x f32 (last block: raster-order output)
// Embedding: im2col (rows in window order) -> GEMM + bias + tiled pos-embed
// -> ln_pre in place.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

#include "../../include/sam3cu.h"
#include "devbuf.cuh"
#include "gemm_sm100.cuh"
#include "misc.cuh"
#include "sam3_file.h"
#include "sam3cu_internal.h"

namespace s3 {
namespace {

constexpr int kMaxLayers = 32;

bool is_global_block(int i) { return i == 7 || i == 15 || i == 23 || i == 31; }


struct Linear {
  DevBuf w;      // 16-bit [N, K] (or unused for Q8)
  DevBuf q;      // int8 [N, K]
  DevBuf sc;     // f32 [K/32, N] (row-shifted for f16 activations, see cs)
  DevBuf cs;     // f32 [N]: 2^-shift of each output row, applied in the epilogue
  DevBuf bias;   // f32 [N]
  int N = 0, K = 0;
};

struct Block {
  DevBuf ln1_w, ln1_b, ln2_w, ln2_b;
  Linear qkv, proj, fc1, fc2;
};

// One weight as the host holds it: up to three parts of n elements each
// (the q, k, v tensors fuse_3 concatenates, image_encoder.c:223-265), each
// in one reference dtype (F32, F16, BF16 or Q8_0).  p == nullptr: zeros.
struct WPart {
  const void* p = nullptr;
  int dt = kF32;
};
struct WSrc {
  WPart part[3];
  int nparts = 1;
  int64_t n = 0;
};
struct VitSrc {
  WSrc patch_w, patch_b, pos_raw, ln_pre_w, ln_pre_b;
  struct BlockSrc {
    WSrc ln1_w, ln1_b, qkv_w, qkv_b, proj_w, proj_b, ln2_w, ln2_b, fc1_w, fc1_b, fc2_w, fc2_b;
  } blocks[kMaxLayers];
};

}  // namespace
}  // namespace s3

struct sam3cu_vit {
  sam3cu_vit_config c{};
  int wdtype = 0;       // SAM3CU_BF16 / F16 / Q8_0
  int act = 0;          // activation dtype kBF16 / kF16
  int max_batch = 0;
  int gs = 0, np = 0, kpad = 0;
  cudaStream_t stream = nullptr;
  s3::Block blocks[s3::kMaxLayers];
  s3::Linear patch;
  s3::DevBuf ln_pre_w, ln_pre_b, pos_win;        // pos_win: tiled pos-embed [np, e] f32, window order
  s3::DevBuf rope_win, rope_glo;  // float2 (cos, sin), pair-major: [32][positions]
  s3::DevBuf win_to_raster;                      // int [np]
  s3::DevBuf raster_to_win;                      // int [np]
  // activations
  s3::DevBuf x, xn, qkv, ao, h;
  s3::DevBuf wq;  // Q8_0 weights: 16-bit dequantised W of two blocks' four linears (two slots)
  // Q8_0: block i+1's weights are dequantised on `side` while block i runs
  cudaStream_t side = nullptr;
  cudaEvent_t ev_wfree[2] = {}, ev_wready[2] = {}, ev_fork = nullptr;
  // image / feature staging for host-buffer encodes: two sets, so that one
  // chunk's copies overlap the next chunk's compute (img2/out2 on demand)
  s3::DevBuf img, out, img2, out2;
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  cudaEvent_t ev_in[2] = {}, ev_done[2] = {}, ev_out[2] = {};
  // CUDA graphs, one per (batch size, input, output) in use
  struct Graph {
    int n;
    const float* in;
    float* out;
    cudaGraphExec_t exec;
    int nodes;
  };
  std::vector<Graph> graphs;
  int launches_per_block = 7;
  // optional per-launch profiling (sam3cu_vit_profile): kind of each launch
  std::vector<int>* prof_kinds = nullptr;
  std::vector<cudaEvent_t>* prof_events = nullptr;
};

namespace s3 {
namespace {

int ck(cudaError_t e) { return e == cudaSuccess ? kOk : kErrCuda; }

size_t dt_bytes(int dt, int64_t n) {
  switch (dt) {
    case kF32: return static_cast<size_t>(n) * 4;
    case kF16:
    case kBF16: return static_cast<size_t>(n) * 2;
    case kQ8: return static_cast<size_t>((n + 31) / 32) * 36;
    default: return 0;
  }
}

// Stage a weight as F32 on the device.  The host bytes go up as stored and
// are converted there: F16/BF16 are widened, Q8_0 blocks dequantised
// (sam3_q8_dequantize, quant.c:134-151).  Parts land back to back, which is
// fuse_3's concatenation (image_encoder.c:223-265).
int stage_f32(DevBuf& d, const WSrc& s, cudaStream_t st) {
  const int64_t total = s.n * s.nparts;
  if (!d.alloc(static_cast<size_t>(total) * 4)) return kErrNoMem;
  for (int i = 0; i < s.nparts; ++i) {
    const WPart& p = s.part[i];
    float* dst = d.as<float>() + i * s.n;
    if (!p.p) {
      if (cudaMemsetAsync(dst, 0, static_cast<size_t>(s.n) * 4, st) != cudaSuccess) return kErrCuda;
      continue;
    }
    if (p.dt == kF32) {
      if (cudaMemcpyAsync(dst, p.p, static_cast<size_t>(s.n) * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return kErrCuda;
      continue;
    }
    const size_t nb = dt_bytes(p.dt, s.n);
    if (!nb) return kErrDtype;
    DevBuf raw;
    if (!raw.alloc(nb)) return kErrNoMem;
    if (cudaMemcpyAsync(raw.p, p.p, nb, cudaMemcpyHostToDevice, st) != cudaSuccess) return kErrCuda;
    const int rc = p.dt == kQ8 ? sam3cu_q8_dequantize(raw.p, dst, s.n, st)
                               : launch_cast(raw.p, p.dt, dst, kF32, s.n, st);
    if (rc) return rc;
    if (cudaStreamSynchronize(st) != cudaSuccess) return kErrCuda;  // raw is freed on scope exit
  }
  return kOk;
}

// Upload a weight to a new device buffer as f32.
int upload_f32(DevBuf& d, const WSrc& s, cudaStream_t st) {
  const int rc = stage_f32(d, s, st);
  return rc ? rc : ck(cudaStreamSynchronize(st));
}

// Upload a host f32 table [n].
int upload_f32(DevBuf& d, const float* h, size_t n, cudaStream_t st) {
  WSrc s;
  s.part[0].p = h;
  s.n = static_cast<int64_t>(n);
  return upload_f32(d, s, st);
}

// Upload a weight [N,K] (row pitch K) to a device [N, ldk] 16-bit matrix
// (zero-padded columns K..ldk).
int upload_w16(DevBuf& d, const WSrc& s, int N, int K, int ldk, int dt, cudaStream_t st) {
  DevBuf tmp, pad;
  int rc = stage_f32(tmp, s, st);
  if (rc) return rc;
  const DevBuf* src = &tmp;
  if (ldk != K) {
    if (!pad.alloc(static_cast<size_t>(N) * ldk * 4)) return kErrNoMem;
    if (cudaMemsetAsync(pad.p, 0, pad.bytes, st) != cudaSuccess) return kErrCuda;
    if (cudaMemcpy2DAsync(pad.p, static_cast<size_t>(ldk) * 4, tmp.p, static_cast<size_t>(K) * 4,
                          static_cast<size_t>(K) * 4, N, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return kErrCuda;
    src = &pad;
  }
  if (!d.alloc(static_cast<size_t>(N) * ldk * 2)) return kErrNoMem;
  rc = launch_cast(src->p, kF32, d.p, dt, static_cast<int64_t>(N) * ldk, st);
  if (rc) return rc;
  return ck(cudaStreamSynchronize(st));  // tmp / pad are freed on return
}

int upload_linear(Linear& L, const WSrc& w, const WSrc& b, int N, int K, int wdtype, int act, cudaStream_t st) {
  L.N = N;
  L.K = K;
  int rc = upload_f32(L.bias, b, st);
  if (rc) return rc;
  if (wdtype == SAM3CU_Q8_0) {
    DevBuf blocks;
    const int64_t n = static_cast<int64_t>(N) * K;
    if (!blocks.alloc((n / 32) * 36)) return kErrNoMem;
    bool all_q8 = w.n % 32 == 0;
    for (int i = 0; i < w.nparts; ++i) all_q8 = all_q8 && w.part[i].p && w.part[i].dt == kQ8;
    if (all_q8) {
      // already Q8_0 (a quantised .sam3 file): the blocks go up as stored and
      // are only repacked; nothing is requantised
      const size_t pb = dt_bytes(kQ8, w.n);
      for (int i = 0; i < w.nparts; ++i)
        if (cudaMemcpyAsync(static_cast<uint8_t*>(blocks.p) + i * pb, w.part[i].p, pb, cudaMemcpyHostToDevice,
                            st) != cudaSuccess)
          return kErrCuda;
    } else {
      DevBuf tmp;
      if ((rc = stage_f32(tmp, w, st))) return rc;
      if ((rc = launch_q8_quantize(tmp.as<float>(), blocks.p, n, st))) return rc;
      if ((rc = ck(cudaStreamSynchronize(st)))) return rc;
    }
    if (!L.q.alloc(n) || !L.sc.alloc((n / 32) * 4)) return kErrNoMem;
    if ((rc = launch_q8_repack(blocks.p, L.q.as<int8_t>(), L.sc.as<float>(), N, K, st))) return rc;
    // f16 activations: scales shifted per row into f16's normal range for the
    // half2 dequantiser, the shift undone in the GEMM epilogue (bf16
    // activations dequantise in f32 arithmetic and need no shift)
    if (act == kF16) {
      if (!L.cs.alloc(static_cast<size_t>(N) * 4)) return kErrNoMem;
      if ((rc = launch_q8_row_shift(L.sc.as<float>(), L.cs.as<float>(), N, K, st))) return rc;
    }
    return ck(cudaStreamSynchronize(st));
  }
  return upload_w16(L.w, w, N, K, K, wdtype == SAM3CU_F16 ? kF16 : kBF16, st);
}

EpiParams epi_default() {
  EpiParams e;
  memset(&e, 0, sizeof(e));
  return e;
}

// Q8_0 weights are dequantised once per call into v->wq (16-bit [N, K],
// at most 9.7 MB, so it stays in L2) and the 16-bit GEMM runs on that: a
// dequantiser inside the GEMM would redo the conversion for every one of
// the M/256 row tiles.  The HBM copy of W stays int8.
// w16: for a Q8_0 linear, its dequantised 16-bit W (dequant_block).
int run_linear(sam3cu_vit* v, const Linear& L, const void* a, int lda, int M, const EpiParams& ep_in,
               const void* w16 = nullptr) {
  GemmShape shp{M, L.N, L.K};
  if (L.q.p) {
    if (!w16) return kErrShape;
    EpiParams ep = ep_in;
    ep.col_scale = L.cs.p ? L.cs.as<float>() : nullptr;  // undoes the per-row scale shift (f16)
    return launch_gemm(a, lda, w16, L.K, nullptr, nullptr, v->act, shp, ep, v->stream, 0);
  }
  const EpiParams& ep = ep_in;
  return launch_gemm(a, lda, L.w.p, L.K, nullptr, nullptr, v->act, shp, ep, v->stream, 0);
}

// Q8_0 weights: the four linears of a block are dequantised in one launch at
// the start of the block into consecutive 16-bit slots of v->wq (27.8 MB at
// the ViT-L sizes, so the GEMMs read them from L2); slot[k] = qkv, proj,
// fc1, fc2.
// the 16-bit slots of block B's linears in half `buf` of v->wq
void slot_ptrs(sam3cu_vit* v, const Block& B, const void* (&slot)[4], int buf) {
  const Linear* L[4] = {&B.qkv, &B.proj, &B.fc1, &B.fc2};
  uint8_t* p = static_cast<uint8_t*>(v->wq.p) + static_cast<size_t>(buf) * (v->wq.bytes / 2);
  for (int k = 0; k < 4; ++k) {
    slot[k] = p;
    p += static_cast<size_t>(L[k]->N) * L[k]->K * 2;
  }
}

int dequant_block(sam3cu_vit* v, const Block& B, const void* (&slot)[4], int buf = 0,
                  cudaStream_t st = nullptr) {
  const Linear* L[4] = {&B.qkv, &B.proj, &B.fc1, &B.fc2};
  Q8DequantJobs jobs;
  jobs.n = 4;
  uint8_t* p = static_cast<uint8_t*>(v->wq.p) + static_cast<size_t>(buf) * (v->wq.bytes / 2);
  for (int k = 0; k < 4; ++k) {
    jobs.job[k] = Q8DequantJob{L[k]->q.as<int8_t>(), L[k]->sc.as<float>(), p, L[k]->N, L[k]->K};
    slot[k] = p;
    p += static_cast<size_t>(L[k]->N) * L[k]->K * 2;
  }
  return launch_q8_dequant_w16_multi(jobs, v->act == kF16 ? 1 : 0, st ? st : v->stream);
}

// Q8_0, overlapped: block i's slot (i % 2) is filled on the side stream
// while block i-1 runs on the main stream.  ev_wready[b]: slot b holds the
// next block's weights; ev_wfree[b]: the block that used slot b finished
// its last GEMM.  (Profiling runs dequantise in line on the main stream.)
int dequant_ahead(sam3cu_vit* v, int i) {
  if (i >= v->c.depth) return kOk;
  const int b = i & 1;
  const void* unused[4];
  if (i >= 2 && cudaStreamWaitEvent(v->side, v->ev_wfree[b], 0) != cudaSuccess) return kErrCuda;
  int rc = dequant_block(v, v->blocks[i], unused, b, v->side);
  if (!rc && cudaEventRecord(v->ev_wready[b], v->side) != cudaSuccess) rc = kErrCuda;
  return rc;
}

// Launch kinds of the profiling runs: the detailed kinds of
// sam3cu_vit_profile_detail (enum sam3cu_prof_kind), summed into GEMM /
// attention / LayerNorm / other for sam3cu_vit_profile.
enum ProfKind {
  kProfPatch = SAM3CU_PROF_PATCH,
  kProfQkv = SAM3CU_PROF_QKV,
  kProfProj = SAM3CU_PROF_PROJ,
  kProfFc1 = SAM3CU_PROF_FC1,
  kProfFc2 = SAM3CU_PROF_FC2,
  kProfDequant = SAM3CU_PROF_DEQUANT,
  kProfAttnWin = SAM3CU_PROF_ATTN_WINDOW,
  kProfAttnGlob = SAM3CU_PROF_ATTN_GLOBAL,
  kProfLn = SAM3CU_PROF_LAYERNORM,
  kProfOther = SAM3CU_PROF_OTHER,
  kProfKinds = SAM3CU_PROF_KINDS
};
int coarse_kind(int k) {
  if (k <= kProfDequant) return 0;  // GEMM (the Q8_0 dequantisation included)
  if (k <= kProfAttnGlob) return 1;
  return k == kProfLn ? 2 : 3;
}

// Record an event after a launch of the given kind (profiling runs only).
void tick(sam3cu_vit* v, int kind) {
  if (!v->prof_events) return;
  cudaEvent_t e;
  cudaEventCreate(&e);
  cudaEventRecord(e, v->stream);
  v->prof_events->push_back(e);
  v->prof_kinds->push_back(kind);
}

// Enqueue the whole forward for n images: images (device, CHW f32) -> out
// (device, [n, np, e] f32 raster order).
int forward(sam3cu_vit* v, const float* images, int n, float* out) {
  const sam3cu_vit_config& c = v->c;
  const int e = c.embed_dim, np = v->np, M = n * np, ws = c.window_size, hd = e / c.n_heads;
  const int nw = v->gs / ws;
  const int* w2r = v->win_to_raster.as<int>();
  int rc;
  // ---- patch embed + bias + pos-embed (window order) -> x; ln_pre in place
  void* acol = v->h.p;  // im2col scratch aliases the MLP hidden buffer
  tick(v, kProfOther);  // start marker
  if ((rc = launch_patch_im2col(images, acol, v->act, n, c.img_size, c.patch_size, v->kpad, w2r, v->stream)))
    return rc;
  tick(v, kProfOther);
  {
    EpiParams ep = epi_default();
    ep.out = v->x.p;
    ep.out_type = kOutF32;
    ep.ldo = e;
    ep.bias = v->patch.bias.as<float>();
    ep.residual = v->pos_win.as<float>();
    ep.ldr = e;
    ep.res_row_period = np;
    if ((rc = run_linear(v, v->patch, acol, v->kpad, M, ep))) return rc;
    tick(v, kProfPatch);
  }
  if ((rc = launch_layernorm(v->x.p, kF32, v->x.p, kF32, v->ln_pre_w.as<float>(), v->ln_pre_b.as<float>(), M, e,
                             nullptr, 0, v->stream)))
    return rc;
  tick(v, kProfLn);
  if (c.depth == 0)
    return launch_gather_rows(v->x.p, out, M, e * 4, v->raster_to_win.as<int>(), np, v->stream);
  static const bool ahead_on = [] {  // SAM3CU_Q8_AHEAD=0: dequantise in line (A/B measurements)
    const char* e = getenv("SAM3CU_Q8_AHEAD");
    return !(e && atoi(e) == 0);
  }();
  const bool q8_ahead = ahead_on && v->wdtype == SAM3CU_Q8_0 && !v->prof_events && v->side;
  if (q8_ahead) {  // fork the side stream off the main one; blocks 0 and 1 first
    if (cudaEventRecord(v->ev_fork, v->stream) != cudaSuccess ||
        cudaStreamWaitEvent(v->side, v->ev_fork, 0) != cudaSuccess)
      return kErrCuda;
    if ((rc = dequant_ahead(v, 0)) || (rc = dequant_ahead(v, 1))) return rc;
  }
  for (int i = 0; i < c.depth; ++i) {
    const Block& B = v->blocks[i];
    const bool glob = is_global_block(i);
    const bool last = i == c.depth - 1;
    const void* w16[4] = {nullptr, nullptr, nullptr, nullptr};
    if (q8_ahead) {
      slot_ptrs(v, B, w16, i & 1);
      if (cudaStreamWaitEvent(v->stream, v->ev_wready[i & 1], 0) != cudaSuccess) return kErrCuda;
    } else if (v->wdtype == SAM3CU_Q8_0) {
      if ((rc = dequant_block(v, B, w16))) return rc;
      tick(v, kProfDequant);
    }
    if ((rc = launch_layernorm(v->x.p, kF32, v->xn.p, v->act, B.ln1_w.as<float>(), B.ln1_b.as<float>(), M, e,
                               nullptr, 0, v->stream)))
      return rc;
    tick(v, kProfLn);
    {
      EpiParams ep = epi_default();
      ep.out = v->qkv.p;
      ep.out_type = v->act;
      ep.ldo = 3 * e;
      ep.bias = B.qkv.bias.as<float>();
      ep.rope_cols = 2 * e;
      if (glob) {
        ep.rope_cs = v->rope_glo.as<float2>();
        ep.rope_period = np;
      } else {
        ep.rope_cs = v->rope_win.as<float2>();
        ep.rope_period = ws * ws;
      }
      if ((rc = run_linear(v, B.qkv, v->xn.p, e, M, ep, w16[0]))) return rc;
      tick(v, kProfQkv);
    }
    {
      const uint16_t* qkv = v->qkv.as<uint16_t>();
      const int groups = glob ? n : n * nw * nw;
      const int seq = glob ? np : ws * ws;
      if ((rc = launch_attention(qkv, qkv + e, qkv + 2 * e, 3 * e, v->ao.p, e, v->act, groups, seq, c.n_heads, hd,
                                 v->stream)))
        return rc;
      tick(v, glob ? kProfAttnGlob : kProfAttnWin);
    }
    {
      EpiParams ep = epi_default();
      ep.out = v->x.p;
      ep.out_type = kOutF32;
      ep.ldo = e;
      ep.bias = B.proj.bias.as<float>();
      ep.residual = v->x.as<float>();
      ep.ldr = e;
      if ((rc = run_linear(v, B.proj, v->ao.p, e, M, ep, w16[1]))) return rc;
      tick(v, kProfProj);
    }
    if ((rc = launch_layernorm(v->x.p, kF32, v->xn.p, v->act, B.ln2_w.as<float>(), B.ln2_b.as<float>(), M, e,
                               nullptr, 0, v->stream)))
      return rc;
    tick(v, kProfLn);
    {
      EpiParams ep = epi_default();
      ep.out = v->h.p;
      ep.out_type = v->act;
      ep.ldo = c.mlp_dim;
      ep.bias = B.fc1.bias.as<float>();
      ep.act = 1;
      if ((rc = run_linear(v, B.fc1, v->xn.p, e, M, ep, w16[2]))) return rc;
      tick(v, kProfFc1);
    }
    {
      EpiParams ep = epi_default();
      ep.out = last ? static_cast<void*>(out) : v->x.p;
      ep.out_type = kOutF32;
      ep.ldo = e;
      ep.bias = B.fc2.bias.as<float>();
      ep.residual = v->x.as<float>();
      ep.ldr = e;
      if (last) {
        ep.out_row_map = w2r;
        ep.out_row_period = np;
      }
      if ((rc = run_linear(v, B.fc2, v->h.p, c.mlp_dim, M, ep, w16[3]))) return rc;
      tick(v, kProfFc2);
    }
    if (q8_ahead) {  // slot i % 2 is free: the side stream fills it with block i + 2
      if (cudaEventRecord(v->ev_wfree[i & 1], v->stream) != cudaSuccess) return kErrCuda;
      if ((rc = dequant_ahead(v, i + 2))) return rc;
    }
  }
  if (q8_ahead) {  // join: the side stream's last work precedes the end of the forward
    if (cudaEventRecord(v->ev_fork, v->side) != cudaSuccess ||
        cudaStreamWaitEvent(v->stream, v->ev_fork, 0) != cudaSuccess)
      return kErrCuda;
  }
  return kOk;
}

void host_rope_table(int n_pos, int grid_w, int hd, float scale, std::vector<float>& cs, std::vector<float>& sn) {
  // precompute_rope_table (image_encoder.c:55-115): column (x) frequencies
  // first, then row (y); 16 frequencies 1/10000^(4i/hd).
  const int half = hd / 2, quarter = hd / 4;
  cs.assign(static_cast<size_t>(n_pos) * half, 0.f);
  sn.assign(cs.size(), 0.f);
  std::vector<float> fr(quarter);
  for (int i = 0; i < quarter; ++i) fr[i] = 1.0f / powf(10000.0f, static_cast<float>(i * 4) / static_cast<float>(hd));
  const int gh = n_pos / grid_w;
  for (int py = 0; py < gh; ++py)
    for (int px = 0; px < grid_w; ++px) {
      const int p = py * grid_w + px;
      const float sy = static_cast<float>(py) * scale, sx = static_cast<float>(px) * scale;
      for (int i = 0; i < quarter; ++i) {
        cs[p * half + i] = cosf(sx * fr[i]);
        sn[p * half + i] = sinf(sx * fr[i]);
        cs[p * half + quarter + i] = cosf(sy * fr[i]);
        sn[p * half + quarter + i] = sinf(sy * fr[i]);
      }
    }
}

int vit_setup(sam3cu_vit* v, const VitSrc& w) {
  const sam3cu_vit_config& c = v->c;
  const int e = c.embed_dim, ps = c.patch_size, ws = c.window_size;
  cudaStream_t st = v->stream;
  int rc;
  v->gs = c.img_size / ps;
  v->np = v->gs * v->gs;
  const int np = v->np, gs = v->gs, nw = gs / ws;
  v->kpad = ((ps * ps * 3 + 63) / 64) * 64;
  // token order maps
  std::vector<int> w2r(np);
  for (int r = 0; r < np; ++r) {
    const int win = r / (ws * ws), slot = r % (ws * ws);
    const int wy = win / nw, wx = win % nw, cy = slot / ws, cx = slot % ws;
    w2r[r] = (wy * ws + cy) * gs + wx * ws + cx;
  }
  if (!v->win_to_raster.alloc(np * 4)) return kErrNoMem;
  if ((rc = ck(cudaMemcpyAsync(v->win_to_raster.p, w2r.data(), np * 4, cudaMemcpyHostToDevice, st)))) return rc;
  std::vector<int> r2w(np);
  for (int r = 0; r < np; ++r) r2w[w2r[r]] = r;
  if (!v->raster_to_win.alloc(np * 4)) return kErrNoMem;
  if ((rc = ck(cudaMemcpyAsync(v->raster_to_win.p, r2w.data(), np * 4, cudaMemcpyHostToDevice, st)))) return rc;
  if ((rc = ck(cudaStreamSynchronize(st)))) return rc;
  // RoPE tables: window-local (scale 1) and global (scale ws/gs)
  std::vector<float> cs, sn;
  // Epilogue layout: (cos, sin) pairs, pair-major, indexed by the GEMM row
  // (window-local slot, resp. the window-major token index of a global block).
  const int half = e / c.n_heads / 2;
  std::vector<float> tab;
  auto pair_major = [&](int n, const int* row_pos) {
    tab.assign(static_cast<size_t>(half) * n * 2, 0.f);
    for (int d = 0; d < half; ++d)
      for (int r = 0; r < n; ++r) {
        const int p = row_pos ? row_pos[r] : r;
        tab[(static_cast<size_t>(d) * n + r) * 2] = cs[static_cast<size_t>(p) * half + d];
        tab[(static_cast<size_t>(d) * n + r) * 2 + 1] = sn[static_cast<size_t>(p) * half + d];
      }
  };
  host_rope_table(ws * ws, ws, e / c.n_heads, 1.0f, cs, sn);
  pair_major(ws * ws, nullptr);
  if ((rc = upload_f32(v->rope_win, tab.data(), tab.size(), st))) return rc;
  host_rope_table(np, gs, e / c.n_heads, static_cast<float>(ws) / static_cast<float>(gs), cs, sn);
  pair_major(np, w2r.data());
  if ((rc = upload_f32(v->rope_glo, tab.data(), tab.size(), st))) return rc;
  if ((rc = cudaStreamSynchronize(st) == cudaSuccess ? kOk : kErrCuda)) return rc;
  // tiled pos-embed in window order (tile_pos_embed, image_encoder.c:167-218):
  // row r takes raw row 1 + (py % 24) * 24 + (px % 24), gathered on device
  {
    std::vector<int> src_row(np);
    for (int r = 0; r < np; ++r) {
      const int rp = w2r[r], py = rp / gs, px = rp % gs;
      src_row[r] = 1 + (py % 24) * 24 + (px % 24);
    }
    DevBuf raw, map;
    if ((rc = stage_f32(raw, w.pos_raw, st))) return rc;
    if (!map.alloc(np * 4) || !v->pos_win.alloc(static_cast<size_t>(np) * e * 4)) return kErrNoMem;
    if ((rc = ck(cudaMemcpyAsync(map.p, src_row.data(), np * 4, cudaMemcpyHostToDevice, st)))) return rc;
    if ((rc = launch_gather_rows(raw.p, v->pos_win.p, np, e * 4, map.as<int>(), np, st))) return rc;
    if ((rc = ck(cudaStreamSynchronize(st)))) return rc;
  }
  if ((rc = upload_f32(v->ln_pre_w, w.ln_pre_w, st))) return rc;
  if ((rc = upload_f32(v->ln_pre_b, w.ln_pre_b, st))) return rc;
  // patch embedding as a GEMM: W [e, ps*ps*3] OHWI, K padded to kpad.  It
  // always runs with 16-bit weights; a Q8_0 patch weight (the converter
  // quantises every float tensor of >= 1024 elements, cli_convert.c:340-352)
  // is dequantised on upload.
  v->patch.N = e;
  v->patch.K = v->kpad;
  if ((rc = upload_f32(v->patch.bias, w.patch_b, st))) return rc;
  if ((rc = upload_w16(v->patch.w, w.patch_w, e, ps * ps * 3, v->kpad, v->act, st))) return rc;
  for (int i = 0; i < c.depth; ++i) {
    const VitSrc::BlockSrc& bw = w.blocks[i];
    Block& B = v->blocks[i];
    if ((rc = upload_f32(B.ln1_w, bw.ln1_w, st)) || (rc = upload_f32(B.ln1_b, bw.ln1_b, st)) ||
        (rc = upload_f32(B.ln2_w, bw.ln2_w, st)) || (rc = upload_f32(B.ln2_b, bw.ln2_b, st)))
      return rc;
    if ((rc = upload_linear(B.qkv, bw.qkv_w, bw.qkv_b, 3 * e, e, v->wdtype, v->act, st))) return rc;
    if ((rc = upload_linear(B.proj, bw.proj_w, bw.proj_b, e, e, v->wdtype, v->act, st))) return rc;
    if ((rc = upload_linear(B.fc1, bw.fc1_w, bw.fc1_b, c.mlp_dim, e, v->wdtype, v->act, st))) return rc;
    if ((rc = upload_linear(B.fc2, bw.fc2_w, bw.fc2_b, e, c.mlp_dim, v->wdtype, v->act, st))) return rc;
  }
  // activations for max_batch images
  const size_t M = static_cast<size_t>(v->max_batch) * np;
  const size_t hcols = static_cast<size_t>(c.mlp_dim) > static_cast<size_t>(v->kpad) ? c.mlp_dim : v->kpad;
  if (!v->x.alloc(M * e * 4) || !v->xn.alloc(M * e * 2) || !v->qkv.alloc(M * 3 * e * 2) ||
      !v->ao.alloc(M * e * 2) || !v->h.alloc(M * hcols * 2) ||
      !v->img.alloc(static_cast<size_t>(v->max_batch) * 3 * c.img_size * c.img_size * 4) ||
      !v->out.alloc(M * e * 4))
    return kErrNoMem;
  if (v->wdtype == SAM3CU_Q8_0) {  // two blocks' four dequantised linears
    const size_t wsum = (static_cast<size_t>(4) * e + 2 * static_cast<size_t>(c.mlp_dim)) * e * 2;
    if (!v->wq.alloc(2 * wsum)) return kErrNoMem;
    if (cudaStreamCreateWithFlags(&v->side, cudaStreamNonBlocking) != cudaSuccess) return kErrCuda;
    for (int b = 0; b < 2; ++b)
      if (cudaEventCreateWithFlags(&v->ev_wfree[b], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&v->ev_wready[b], cudaEventDisableTiming) != cudaSuccess)
        return kErrCuda;
    if (cudaEventCreateWithFlags(&v->ev_fork, cudaEventDisableTiming) != cudaSuccess) return kErrCuda;
  }
  return ck(cudaStreamSynchronize(st));
}


sam3cu_vit* vit_create(const sam3cu_vit_config* cfg, const VitSrc& w, int weight_dtype, int max_batch,
                       int* status_p) {
  *status_p = kOk;
  if (!cfg || max_batch <= 0 || cfg->depth < 0 || cfg->depth > kMaxLayers || cfg->n_heads <= 0 ||
      cfg->embed_dim / cfg->n_heads != 64 || cfg->embed_dim % 64 || cfg->mlp_dim % 64 || cfg->patch_size <= 0 ||
      cfg->window_size <= 0 || cfg->img_size % cfg->patch_size ||
      (cfg->img_size / cfg->patch_size) % cfg->window_size) {
    *status_p = SAM3CU_EINVAL;
    return nullptr;
  }
  if (weight_dtype != SAM3CU_BF16 && weight_dtype != SAM3CU_F16 && weight_dtype != SAM3CU_Q8_0) {
    *status_p = SAM3CU_EDTYPE;
    return nullptr;
  }
  std::unique_ptr<sam3cu_vit> v(new sam3cu_vit());
  v->c = *cfg;
  v->wdtype = weight_dtype;
  // Q8_0 weights pair with bf16 activations: the weights are dequantised
  // (f32 arithmetic, one rounding) on a side stream and the GEMMs then run
  // exactly as the BF16 encoder's.  SAM3CU_Q8_ACT=f16 selects f16
  // activations instead (half2 dequantisation with per-row scale shifts,
  // undone in the GEMM epilogue), which measured slower at one image.
  static const bool q8_f16 = [] {
    const char* e = getenv("SAM3CU_Q8_ACT");
    return e && strcmp(e, "f16") == 0;
  }();
  v->act = (weight_dtype == SAM3CU_F16 || (weight_dtype == SAM3CU_Q8_0 && q8_f16)) ? kF16 : kBF16;
  v->max_batch = max_batch;
  if (cudaStreamCreateWithFlags(&v->stream, cudaStreamNonBlocking) != cudaSuccess) {
    *status_p = kErrCuda;
    return nullptr;
  }
  int rc = vit_setup(v.get(), w);
  if (rc) {
    cudaStreamSynchronize(v->stream);
    cudaStreamDestroy(v->stream);
    *status_p = rc;
    return nullptr;
  }
  return v.release();
}

// Tensor names of the reference's ViT weights (image_encoder.c:155, 346-452).
#define VIT_P "detector_model.vision_encoder.backbone."

// A file tensor as a weight part, checked to hold n elements (the reference
// sam3_vit_load does not check shapes; a mis-sized tensor here is an error).
int file_part(const Sam3File& f, const char* name, int64_t n, bool optional, WPart& out) {
  const Sam3FileDesc* d = f.find(name);
  if (!d) return optional ? static_cast<int>(kOk) : static_cast<int>(SAM3CU_EMODEL);
  if (Sam3File::numel(d) != n) return SAM3CU_EMODEL;
  const int dt = static_cast<int>(d->dtype);
  if (dt != kF32 && dt != kF16 && dt != kBF16 && dt != kQ8) return SAM3CU_EDTYPE;
  if (d->data_size < dt_bytes(dt, n)) return SAM3CU_EMODEL;
  out.p = f.tensor_data(d);
  out.dt = dt;
  return kOk;
}

int file_src(const Sam3File& f, const char* name, int64_t n, WSrc& s, bool optional = false) {
  s = WSrc();
  s.n = n;
  return file_part(f, name, n, optional, s.part[0]);
}

// fuse_3 (image_encoder.c:223-265): q, k, v concatenated in that order
int file_src3(const Sam3File& f, int layer, const char* what, int64_t n, WSrc& s) {
  static const char* qkv[3] = {"q_proj", "k_proj", "v_proj"};
  s = WSrc();
  s.n = n;
  s.nparts = 3;
  char name[160];
  for (int j = 0; j < 3; ++j) {
    snprintf(name, sizeof(name), VIT_P "layers.%d.attention.%s.%s", layer, qkv[j], what);
    const int rc = file_part(f, name, n, false, s.part[j]);
    if (rc) return rc;
  }
  return kOk;
}

// The encoder shape a file holds, for callers that pass no config.
int config_from_file(const Sam3File& f, sam3cu_vit_config& c) {
  const Sam3FileDesc* pw = f.find(VIT_P "embeddings.patch_embeddings.projection.weight");
  const Sam3FileDesc* fc1 = f.find(VIT_P "layers.0.mlp.fc1.weight");
  if (!pw || !fc1 || pw->n_dims != 4 || fc1->n_dims != 2) return SAM3CU_EMODEL;
  c.embed_dim = pw->dims[0];
  c.patch_size = pw->dims[1];
  c.mlp_dim = fc1->dims[0];
  c.img_size = f.hdr->image_size;
  c.n_heads = c.embed_dim / 64;
  c.window_size = 24;
  c.depth = 0;
  char name[160];
  for (int i = 0; i < kMaxLayers; ++i) {
    snprintf(name, sizeof(name), VIT_P "layers.%d.layer_norm1.weight", i);
    if (!f.find(name)) break;
    c.depth = i + 1;
  }
  return kOk;
}

int vit_src_from_file(const Sam3File& f, const sam3cu_vit_config& c, VitSrc& src) {
  const int64_t e = c.embed_dim, m = c.mlp_dim, ps = c.patch_size;
  int rc;
  if ((rc = file_src(f, VIT_P "embeddings.patch_embeddings.projection.weight", e * ps * ps * 3, src.patch_w)) ||
      (rc = file_src(f, VIT_P "embeddings.patch_embeddings.projection.bias", e, src.patch_b, true)) ||
      (rc = file_src(f, VIT_P "embeddings.position_embedding.weight", 577 * e, src.pos_raw)) ||
      (rc = file_src(f, VIT_P "layer_norm.weight", e, src.ln_pre_w)) ||
      (rc = file_src(f, VIT_P "layer_norm.bias", e, src.ln_pre_b)))
    return rc;
  char name[160];
  auto one = [&](int i, const char* what, int64_t n, WSrc& s) {
    snprintf(name, sizeof(name), VIT_P "layers.%d.%s", i, what);
    return file_src(f, name, n, s);
  };
  for (int i = 0; i < c.depth; ++i) {
    VitSrc::BlockSrc& b = src.blocks[i];
    if ((rc = one(i, "layer_norm1.weight", e, b.ln1_w)) || (rc = one(i, "layer_norm1.bias", e, b.ln1_b)) ||
        (rc = file_src3(f, i, "weight", e * e, b.qkv_w)) || (rc = file_src3(f, i, "bias", e, b.qkv_b)) ||
        (rc = one(i, "attention.o_proj.weight", e * e, b.proj_w)) ||
        (rc = one(i, "attention.o_proj.bias", e, b.proj_b)) ||
        (rc = one(i, "layer_norm2.weight", e, b.ln2_w)) || (rc = one(i, "layer_norm2.bias", e, b.ln2_b)) ||
        (rc = one(i, "mlp.fc1.weight", m * e, b.fc1_w)) || (rc = one(i, "mlp.fc1.bias", m, b.fc1_b)) ||
        (rc = one(i, "mlp.fc2.weight", e * m, b.fc2_w)) || (rc = one(i, "mlp.fc2.bias", e, b.fc2_b)))
      return rc;
  }
  return kOk;
}

WSrc f32src(const float* p, int64_t n) {
  WSrc s;
  s.part[0].p = p;
  s.n = n;
  return s;
}

}  // namespace
}  // namespace s3

using namespace s3;

extern "C" {

sam3cu_vit* sam3cu_vit_create(const sam3cu_vit_config* cfg, const sam3cu_vit_weights* w, int weight_dtype,
                              int max_batch, int* status) {
  int st_dummy;
  int* status_p = status ? status : &st_dummy;
  if (!cfg || !w || cfg->depth < 0 || cfg->depth > kMaxLayers) {
    *status_p = SAM3CU_EINVAL;
    return nullptr;
  }
  const int64_t e = cfg->embed_dim, m = cfg->mlp_dim, ps = cfg->patch_size;
  VitSrc src;
  src.patch_w = f32src(w->patch_w, e * ps * ps * 3);
  src.patch_b = f32src(w->patch_b, e);
  src.pos_raw = f32src(w->pos_raw, 577 * e);
  src.ln_pre_w = f32src(w->ln_pre_w, e);
  src.ln_pre_b = f32src(w->ln_pre_b, e);
  for (int i = 0; i < cfg->depth; ++i) {
    const sam3cu_vit_block_weights& b = w->blocks[i];
    VitSrc::BlockSrc& d = src.blocks[i];
    d.ln1_w = f32src(b.ln1_w, e);
    d.ln1_b = f32src(b.ln1_b, e);
    d.ln2_w = f32src(b.ln2_w, e);
    d.ln2_b = f32src(b.ln2_b, e);
    d.qkv_w = f32src(b.qkv_w, 3 * e * e);
    d.qkv_b = f32src(b.qkv_b, 3 * e);
    d.proj_w = f32src(b.proj_w, e * e);
    d.proj_b = f32src(b.proj_b, e);
    d.fc1_w = f32src(b.fc1_w, m * e);
    d.fc1_b = f32src(b.fc1_b, m);
    d.fc2_w = f32src(b.fc2_w, e * m);
    d.fc2_b = f32src(b.fc2_b, e);
  }
  return vit_create(cfg, src, weight_dtype, max_batch, status_p);
}

sam3cu_vit* sam3cu_vit_create_from_sam3(const void* image, size_t bytes, const sam3cu_vit_config* cfg,
                                        int weight_dtype, int max_batch, int* status) {
  int st_dummy;
  int* status_p = status ? status : &st_dummy;
  Sam3File f;
  int rc = f.open(image, bytes);
  sam3cu_vit_config c{};
  if (!rc) {
    if (cfg) c = *cfg;
    else rc = config_from_file(f, c);
  }
  if (!rc && (c.depth < 0 || c.depth > kMaxLayers || c.embed_dim <= 0 || c.patch_size <= 0)) rc = SAM3CU_EINVAL;
  VitSrc src;
  if (!rc) rc = vit_src_from_file(f, c, src);
  if (rc) {
    *status_p = rc;
    return nullptr;
  }
  return vit_create(&c, src, weight_dtype, max_batch, status_p);
}

int sam3cu_vit_get_config(const sam3cu_vit* v, sam3cu_vit_config* cfg) {
  if (!v || !cfg) return SAM3CU_EINVAL;
  *cfg = v->c;
  return kOk;
}

void sam3cu_vit_destroy(sam3cu_vit* v) {
  if (!v) return;
  if (v->stream) cudaStreamSynchronize(v->stream);
  for (cudaStream_t s : {v->copy_in, v->copy_out})
    if (s) {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  for (int b = 0; b < 2; ++b)
    for (cudaEvent_t e : {v->ev_in[b], v->ev_done[b], v->ev_out[b]})
      if (e) cudaEventDestroy(e);
  for (auto& g : v->graphs) cudaGraphExecDestroy(g.exec);
  if (v->side) {
    cudaStreamSynchronize(v->side);
    cudaStreamDestroy(v->side);
  }
  for (int b = 0; b < 2; ++b)
    for (cudaEvent_t e : {v->ev_wfree[b], v->ev_wready[b]})
      if (e) cudaEventDestroy(e);
  if (v->ev_fork) cudaEventDestroy(v->ev_fork);
  if (v->stream) cudaStreamDestroy(v->stream);
  delete v;
}

void* sam3cu_vit_stream(sam3cu_vit* v) { return v ? v->stream : nullptr; }

int sam3cu_vit_profile_detail(sam3cu_vit* v, const float* images, int n, float* out, double* ms, int* counts) {
  if (!v || n <= 0 || n > v->max_batch || !images || !out || !ms || !counts) return SAM3CU_EINVAL;
  std::vector<int> kinds;
  std::vector<cudaEvent_t> evs;
  v->prof_kinds = &kinds;
  v->prof_events = &evs;
  // The GPU waits 30 ms while every launch and event is enqueued, so the
  // per-launch intervals hold device time only (with one image the kernels
  // are shorter than the host's per-launch work).
  int rc = launch_gpu_sleep(30000000ull, v->stream);
  if (!rc) rc = forward(v, images, n, out);
  v->prof_kinds = nullptr;
  v->prof_events = nullptr;
  cudaError_t ce = cudaStreamSynchronize(v->stream);
  for (int k = 0; k < kProfKinds; ++k) {
    ms[k] = 0.0;
    counts[k] = 0;
  }
  for (size_t i = 1; i < evs.size(); ++i) {
    float t = 0.f;
    cudaEventElapsedTime(&t, evs[i - 1], evs[i]);
    ms[kinds[i]] += t;
    counts[kinds[i]] += 1;
  }
  for (auto e : evs) cudaEventDestroy(e);
  if (rc) return rc;
  return ce == cudaSuccess ? kOk : kErrCuda;
}

int sam3cu_vit_profile(sam3cu_vit* v, const float* images, int n, float* out, double* ms, int* counts) {
  if (!ms || !counts) return SAM3CU_EINVAL;
  double fms[kProfKinds];
  int fc[kProfKinds];
  const int rc = sam3cu_vit_profile_detail(v, images, n, out, fms, fc);
  for (int k = 0; k < 4; ++k) {
    ms[k] = 0.0;
    counts[k] = 0;
  }
  if (rc) return rc;
  for (int k = 0; k < kProfKinds; ++k) {
    ms[coarse_kind(k)] += fms[k];
    counts[coarse_kind(k)] += fc[k];
  }
  return kOk;
}

int sam3cu_vit_launches_per_encode(sam3cu_vit* v, int n) {
  (void)n;
  if (!v) return 0;
  // Q8_0: one dequantisation launch for the 4 linears of a block
  return 3 + (v->wdtype == SAM3CU_Q8_0 ? 8 : 7) * v->c.depth + (v->c.depth == 0 ? 1 : 0);
}

// Enqueue through a CUDA graph captured once per (batch size, in, out)
// triple (a few are kept); falls back to direct launches if capture fails.
int sam3cu_vit_encode_async(sam3cu_vit* v, const float* images, int n, float* out) {
  if (!v || n <= 0 || n > v->max_batch || !images || !out) return SAM3CU_EINVAL;
  sam3cu_vit::Graph* hit = nullptr;
  for (auto& g : v->graphs)
    if (g.n == n && g.in == images && g.out == out) hit = &g;
  if (!hit) {
    constexpr size_t kMaxGraphs = 8;
    if (v->graphs.size() >= kMaxGraphs) {  // drop the oldest
      cudaGraphExecDestroy(v->graphs.front().exec);
      v->graphs.erase(v->graphs.begin());
    }
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(v->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      cudaGetLastError();
      return forward(v, images, n, out);  // direct launches count themselves
    }
    const uint64_t before = count_launches(0);
    int rc = forward(v, images, n, out);
    cudaError_t ce = cudaStreamEndCapture(v->stream, &g);
    count_launches(-static_cast<int64_t>(count_launches(0) - before));  // captured, not launched
    if (rc || ce != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
      return rc ? rc : kErrCuda;
    }
    size_t nodes = 0;
    cudaGraphGetNodes(g, nullptr, &nodes);
    cudaGraphExec_t ge = nullptr;
    ce = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return kErrCuda;
    v->graphs.push_back({n, images, out, ge, static_cast<int>(nodes)});
    hit = &v->graphs.back();
  }
  count_launches(hit->nodes);
  return cudaGraphLaunch(hit->exec, v->stream) == cudaSuccess ? kOk : kErrLaunch;
}

namespace {

// Copy streams, events and the second staging set for pipelined
// host-buffer encodes (created on first use).
int ensure_pipeline(sam3cu_vit* v) {
  if (v->copy_in) return kOk;
  const size_t in_bytes = static_cast<size_t>(v->max_batch) * 3 * v->c.img_size * v->c.img_size * 4;
  const size_t out_bytes = static_cast<size_t>(v->max_batch) * v->np * v->c.embed_dim * 4;
  if (!v->img2.alloc(in_bytes) || !v->out2.alloc(out_bytes)) return kErrNoMem;
  for (int b = 0; b < 2; ++b)
    for (cudaEvent_t* e : {&v->ev_in[b], &v->ev_done[b], &v->ev_out[b]})
      if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) return kErrCuda;
  if (cudaStreamCreateWithFlags(&v->copy_in, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&v->copy_out, cudaStreamNonBlocking) != cudaSuccess)
    return kErrCuda;
  return kOk;
}

}  // namespace

// Host buffers: n may exceed max_batch.  The images are encoded in chunks of
// max_batch; chunk i uses staging set i % 2, its H2D copy runs on copy_in
// and its D2H copy on copy_out, so with pinned host memory the copies of
// one chunk overlap the compute of the next.  Events order each staging
// set: H2D(i) after compute(i-2) read it, compute(i) after H2D(i) and after
// D2H(i-2) drained its output buffer, D2H(i) after compute(i).
int sam3cu_vit_encode(sam3cu_vit* v, const float* images, int n, float* out, int on_device) {
  if (!v || n <= 0 || !images || !out) return SAM3CU_EINVAL;
  if (on_device) {
    if (n > v->max_batch) return SAM3CU_EINVAL;
    const int rc = sam3cu_vit_encode_async(v, images, n, out);
    if (cudaStreamSynchronize(v->stream) != cudaSuccess) return kErrCuda;
    return rc;
  }
  const size_t img_elems = static_cast<size_t>(3) * v->c.img_size * v->c.img_size;
  const size_t out_elems = static_cast<size_t>(v->np) * v->c.embed_dim;
  // Chunks of max_batch; a batch of 4 .. max_batch images is split in two, so
  // the copies of one half overlap the other half's compute (a single chunk
  // would expose all of its H2D and D2H time).
  const int cs = (n <= v->max_batch && n >= 4) ? (n + 1) / 2 : v->max_batch;
  const int chunks = (n + cs - 1) / cs;
  int rc = kOk;
  if (chunks == 1) {  // a single chunk has nothing to overlap with
    if (cudaMemcpyAsync(v->img.p, images, n * img_elems * 4, cudaMemcpyHostToDevice, v->stream) != cudaSuccess)
      return kErrCuda;
    rc = sam3cu_vit_encode_async(v, v->img.as<float>(), n, v->out.as<float>());
    if (!rc && cudaMemcpyAsync(out, v->out.p, n * out_elems * 4, cudaMemcpyDeviceToHost, v->stream) != cudaSuccess)
      rc = kErrCuda;
    if (cudaStreamSynchronize(v->stream) != cudaSuccess) return kErrCuda;
    return rc;
  }
  if ((rc = ensure_pipeline(v))) return rc;
  for (int i = 0; i < chunks && !rc; ++i) {
    const int b = i & 1, first = i * cs;
    const int cn = std::min(cs, n - first);
    float* img = (b ? v->img2 : v->img).as<float>();
    float* feat = (b ? v->out2 : v->out).as<float>();
    if (i >= 2 && cudaStreamWaitEvent(v->copy_in, v->ev_done[b], 0) != cudaSuccess) rc = kErrCuda;
    if (!rc && cudaMemcpyAsync(img, images + first * img_elems, cn * img_elems * 4, cudaMemcpyHostToDevice,
                               v->copy_in) != cudaSuccess)
      rc = kErrCuda;
    if (!rc && cudaEventRecord(v->ev_in[b], v->copy_in) != cudaSuccess) rc = kErrCuda;
    if (!rc && cudaStreamWaitEvent(v->stream, v->ev_in[b], 0) != cudaSuccess) rc = kErrCuda;
    if (!rc && i >= 2 && cudaStreamWaitEvent(v->stream, v->ev_out[b], 0) != cudaSuccess) rc = kErrCuda;
    if (!rc) rc = sam3cu_vit_encode_async(v, img, cn, feat);
    if (!rc && cudaEventRecord(v->ev_done[b], v->stream) != cudaSuccess) rc = kErrCuda;
    if (!rc && cudaStreamWaitEvent(v->copy_out, v->ev_done[b], 0) != cudaSuccess) rc = kErrCuda;
    if (!rc && cudaMemcpyAsync(out + first * out_elems, feat, cn * out_elems * 4, cudaMemcpyDeviceToHost,
                               v->copy_out) != cudaSuccess)
      rc = kErrCuda;
    if (!rc && cudaEventRecord(v->ev_out[b], v->copy_out) != cudaSuccess) rc = kErrCuda;
  }
  const bool sync_ok = cudaStreamSynchronize(v->stream) == cudaSuccess &&
                       cudaStreamSynchronize(v->copy_in) == cudaSuccess &&
                       cudaStreamSynchronize(v->copy_out) == cudaSuccess;
  if (!sync_ok) return kErrCuda;
  return rc;
}

}  // extern "C"
