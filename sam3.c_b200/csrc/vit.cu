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
#include <cstring>
#include <memory>
#include <vector>

#include "../../include/sam3cu.h"
#include "devbuf.cuh"
#include "gemm_sm100.cuh"
#include "misc.cuh"
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
  s3::DevBuf wq;  // Q8_0 weights: 16-bit dequantised W of the current linear
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

// Upload host f32 [n] to a new device buffer as f32.
int upload_f32(DevBuf& d, const float* h, size_t n, cudaStream_t st) {
  if (!d.alloc(n * 4)) return kErrNoMem;
  if (!h) return ck(cudaMemsetAsync(d.p, 0, n * 4, st));
  return ck(cudaMemcpyAsync(d.p, h, n * 4, cudaMemcpyHostToDevice, st));
}

// Upload host f32 [N,K] (row pitch K) to a device [N, ldk] 16-bit matrix
// (zero-padded columns K..ldk).
int upload_w16(DevBuf& d, const float* h, int N, int K, int ldk, int dt, cudaStream_t st) {
  DevBuf tmp;
  if (!tmp.alloc(static_cast<size_t>(N) * ldk * 4)) return kErrNoMem;
  if (ldk != K) {
    if (cudaMemsetAsync(tmp.p, 0, tmp.bytes, st) != cudaSuccess) return kErrCuda;
    if (cudaMemcpy2DAsync(tmp.p, static_cast<size_t>(ldk) * 4, h, static_cast<size_t>(K) * 4,
                          static_cast<size_t>(K) * 4, N, cudaMemcpyHostToDevice, st) != cudaSuccess)
      return kErrCuda;
  } else if (cudaMemcpyAsync(tmp.p, h, tmp.bytes, cudaMemcpyHostToDevice, st) != cudaSuccess) {
    return kErrCuda;
  }
  if (!d.alloc(static_cast<size_t>(N) * ldk * 2)) return kErrNoMem;
  int rc = launch_cast(tmp.p, kF32, d.p, dt, static_cast<int64_t>(N) * ldk, st);
  if (rc) return rc;
  return ck(cudaStreamSynchronize(st));  // tmp is freed on return
}

int upload_linear(Linear& L, const float* w, const float* b, int N, int K, int wdtype, cudaStream_t st) {
  L.N = N;
  L.K = K;
  int rc = upload_f32(L.bias, b, N, st);
  if (rc) return rc;
  if (wdtype == SAM3CU_Q8_0) {
    DevBuf tmp, blocks;
    const int64_t n = static_cast<int64_t>(N) * K;
    if (!tmp.alloc(n * 4) || !blocks.alloc((n / 32) * 36)) return kErrNoMem;
    if (cudaMemcpyAsync(tmp.p, w, n * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) return kErrCuda;
    if ((rc = launch_q8_quantize(tmp.as<float>(), blocks.p, n, st))) return rc;
    if (!L.q.alloc(n) || !L.sc.alloc((n / 32) * 4)) return kErrNoMem;
    if ((rc = launch_q8_repack(blocks.p, L.q.as<int8_t>(), L.sc.as<float>(), N, K, st))) return rc;
    // f16 activations: scales shifted per row into f16's normal range for the
    // half2 dequantiser, the shift undone in the GEMM epilogue
    if (!L.cs.alloc(static_cast<size_t>(N) * 4)) return kErrNoMem;
    if ((rc = launch_q8_row_shift(L.sc.as<float>(), L.cs.as<float>(), N, K, st))) return rc;
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
int run_linear(sam3cu_vit* v, const Linear& L, const void* a, int lda, int M, const EpiParams& ep_in) {
  GemmShape shp{M, L.N, L.K};
  if (L.q.p) {
    int rc = launch_q8_dequant_w16(L.q.as<int8_t>(), L.sc.as<float>(), v->wq.p, L.N, L.K, v->act == kF16 ? 1 : 0,
                                   v->stream);
    if (rc) return rc;
    EpiParams ep = ep_in;
    ep.col_scale = L.cs.as<float>();  // undoes the per-row scale shift
    return launch_gemm(a, lda, v->wq.p, L.K, nullptr, nullptr, v->act, shp, ep, v->stream, 0);
  }
  const EpiParams& ep = ep_in;
  return launch_gemm(a, lda, L.w.p, L.K, nullptr, nullptr, v->act, shp, ep, v->stream, 0);
}

enum ProfKind { kProfGemm = 0, kProfAttn = 1, kProfLn = 2, kProfOther = 3, kProfKinds = 4 };

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
    tick(v, kProfGemm);
  }
  if ((rc = launch_layernorm(v->x.p, kF32, v->x.p, kF32, v->ln_pre_w.as<float>(), v->ln_pre_b.as<float>(), M, e,
                             nullptr, 0, v->stream)))
    return rc;
  tick(v, kProfLn);
  if (c.depth == 0)
    return launch_gather_rows(v->x.p, out, M, e * 4, v->raster_to_win.as<int>(), np, v->stream);
  for (int i = 0; i < c.depth; ++i) {
    const Block& B = v->blocks[i];
    const bool glob = is_global_block(i);
    const bool last = i == c.depth - 1;
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
      if ((rc = run_linear(v, B.qkv, v->xn.p, e, M, ep))) return rc;
      tick(v, kProfGemm);
    }
    {
      const uint16_t* qkv = v->qkv.as<uint16_t>();
      const int groups = glob ? n : n * nw * nw;
      const int seq = glob ? np : ws * ws;
      if ((rc = launch_attention(qkv, qkv + e, qkv + 2 * e, 3 * e, v->ao.p, e, v->act, groups, seq, c.n_heads, hd,
                                 v->stream)))
        return rc;
      tick(v, kProfAttn);
    }
    {
      EpiParams ep = epi_default();
      ep.out = v->x.p;
      ep.out_type = kOutF32;
      ep.ldo = e;
      ep.bias = B.proj.bias.as<float>();
      ep.residual = v->x.as<float>();
      ep.ldr = e;
      if ((rc = run_linear(v, B.proj, v->ao.p, e, M, ep))) return rc;
      tick(v, kProfGemm);
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
      if ((rc = run_linear(v, B.fc1, v->xn.p, e, M, ep))) return rc;
      tick(v, kProfGemm);
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
      if ((rc = run_linear(v, B.fc2, v->h.p, c.mlp_dim, M, ep))) return rc;
      tick(v, kProfGemm);
    }
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

int vit_setup(sam3cu_vit* v, const sam3cu_vit_weights* w) {
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
  // tiled pos-embed in window order (tile_pos_embed, image_encoder.c:167-218)
  {
    std::vector<float> pos(static_cast<size_t>(np) * e);
    for (int r = 0; r < np; ++r) {
      const int rp = w2r[r], py = rp / gs, px = rp % gs;
      const float* src = w->pos_raw + static_cast<size_t>(1 + (py % 24) * 24 + (px % 24)) * e;
      memcpy(&pos[static_cast<size_t>(r) * e], src, e * 4);
    }
    if ((rc = upload_f32(v->pos_win, pos.data(), pos.size(), st))) return rc;
    if ((rc = ck(cudaStreamSynchronize(st)))) return rc;
  }
  if ((rc = upload_f32(v->ln_pre_w, w->ln_pre_w, e, st))) return rc;
  if ((rc = upload_f32(v->ln_pre_b, w->ln_pre_b, e, st))) return rc;
  // patch embedding as a GEMM: W [e, ps*ps*3] OHWI, K padded to kpad.
  // It always runs with 16-bit weights (the reference's conv weight stays
  // F32 in a Q8 file: the converter quantises only 2-D linears).
  v->patch.N = e;
  v->patch.K = v->kpad;
  if ((rc = upload_f32(v->patch.bias, w->patch_b, e, st))) return rc;
  if ((rc = upload_w16(v->patch.w, w->patch_w, e, ps * ps * 3, v->kpad, v->act, st))) return rc;
  for (int i = 0; i < c.depth; ++i) {
    const sam3cu_vit_block_weights& bw = w->blocks[i];
    Block& B = v->blocks[i];
    if ((rc = upload_f32(B.ln1_w, bw.ln1_w, e, st)) || (rc = upload_f32(B.ln1_b, bw.ln1_b, e, st)) ||
        (rc = upload_f32(B.ln2_w, bw.ln2_w, e, st)) || (rc = upload_f32(B.ln2_b, bw.ln2_b, e, st)))
      return rc;
    if ((rc = upload_linear(B.qkv, bw.qkv_w, bw.qkv_b, 3 * e, e, v->wdtype, st))) return rc;
    if ((rc = upload_linear(B.proj, bw.proj_w, bw.proj_b, e, e, v->wdtype, st))) return rc;
    if ((rc = upload_linear(B.fc1, bw.fc1_w, bw.fc1_b, c.mlp_dim, e, v->wdtype, st))) return rc;
    if ((rc = upload_linear(B.fc2, bw.fc2_w, bw.fc2_b, e, c.mlp_dim, v->wdtype, st))) return rc;
  }
  // activations for max_batch images
  const size_t M = static_cast<size_t>(v->max_batch) * np;
  const size_t hcols = static_cast<size_t>(c.mlp_dim) > static_cast<size_t>(v->kpad) ? c.mlp_dim : v->kpad;
  if (!v->x.alloc(M * e * 4) || !v->xn.alloc(M * e * 2) || !v->qkv.alloc(M * 3 * e * 2) ||
      !v->ao.alloc(M * e * 2) || !v->h.alloc(M * hcols * 2) ||
      !v->img.alloc(static_cast<size_t>(v->max_batch) * 3 * c.img_size * c.img_size * 4) ||
      !v->out.alloc(M * e * 4))
    return kErrNoMem;
  if (v->wdtype == SAM3CU_Q8_0) {  // largest linear: fc1 / fc2 (or QKV)
    const size_t wmax = std::max(static_cast<size_t>(c.mlp_dim), static_cast<size_t>(3 * e)) * e * 2;
    if (!v->wq.alloc(wmax)) return kErrNoMem;
  }
  return ck(cudaStreamSynchronize(st));
}

}  // namespace
}  // namespace s3

using namespace s3;

extern "C" {

sam3cu_vit* sam3cu_vit_create(const sam3cu_vit_config* cfg, const sam3cu_vit_weights* w, int weight_dtype,
                              int max_batch, int* status) {
  int st_dummy;
  int* status_p = status ? status : &st_dummy;
  *status_p = kOk;
  if (!cfg || !w || max_batch <= 0 || cfg->depth < 0 || cfg->depth > kMaxLayers || cfg->n_heads <= 0 ||
      cfg->embed_dim / cfg->n_heads != 64 || cfg->embed_dim % 64 || cfg->mlp_dim % 64 ||
      cfg->img_size % cfg->patch_size || (cfg->img_size / cfg->patch_size) % cfg->window_size) {
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
  // Q8_0 weights pair with f16 activations: the int8 tiles are dequantised in
  // half2 arithmetic (gemm_sm100.cu), and f16 keeps 3 more mantissa bits
  v->act = (weight_dtype == SAM3CU_F16 || weight_dtype == SAM3CU_Q8_0) ? kF16 : kBF16;
  v->max_batch = max_batch;
  if (cudaStreamCreateWithFlags(&v->stream, cudaStreamNonBlocking) != cudaSuccess) {
    *status_p = kErrCuda;
    return nullptr;
  }
  int rc = vit_setup(v.get(), w);
  if (rc) {
    *status_p = rc;
    return nullptr;
  }
  return v.release();
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
  if (v->stream) cudaStreamDestroy(v->stream);
  delete v;
}

void* sam3cu_vit_stream(sam3cu_vit* v) { return v ? v->stream : nullptr; }

int sam3cu_vit_profile(sam3cu_vit* v, const float* images, int n, float* out, double* ms, int* counts) {
  if (!v || n <= 0 || n > v->max_batch || !images || !out || !ms || !counts) return SAM3CU_EINVAL;
  std::vector<int> kinds;
  std::vector<cudaEvent_t> evs;
  v->prof_kinds = &kinds;
  v->prof_events = &evs;
  int rc = forward(v, images, n, out);
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

int sam3cu_vit_launches_per_encode(sam3cu_vit* v, int n) {
  (void)n;
  if (!v) return 0;
  // Q8_0: one dequantisation launch before each of the 4 linears of a block
  return 3 + (v->wdtype == SAM3CU_Q8_0 ? 11 : 7) * v->c.depth + (v->c.depth == 0 ? 1 : 0);
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
  const int chunks = (n + v->max_batch - 1) / v->max_batch;
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
    const int b = i & 1, first = i * v->max_batch;
    const int cn = std::min(v->max_batch, n - first);
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
