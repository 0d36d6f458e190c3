// neck.cu - the SAM3 FPN neck (src/model/necks.c: sam3_neck_init /
// sam3_neck_build) as fused sm_100a kernels.
//
// Per scale stage (necks.c:24-145; the stage kind follows the scale factor
// as in sam3_neck_init, necks.c:165-177):
//   4x    ConvT(dim -> dim/2, k2 s2) + GELU, ConvT(dim/2 -> dim/4, k2 s2),
//         Conv1x1(dim/4 -> d), Conv3x3(d -> d, pad 1)
//   2x    ConvT(dim -> dim/2, k2 s2), Conv1x1(dim/2 -> d), Conv3x3
//   1x    Conv1x1(dim -> d), Conv3x3
//   0.5x  MaxPool(k2 s2), Conv1x1(dim -> d), Conv3x3
// every conv with its bias.  Lowering (T = the 16-bit compute type):
//   ConvT k2 s2  one GEMM [n*H*W, C] x Wt[(ky, kx, oc), C]^T with the bias
//                (replicated per (ky, kx)) and the GELU in the epilogue, then
//                a pixel shuffle to [n, 2H, 2W, oc]; Wt is the OHWI weight
//                permuted once at creation
//   Conv1x1      GEMM with the bias in the epilogue
//   Conv3x3      an implicit GEMM reading the NHWC map directly when the map
//                tiles into 4x32-pixel blocks (the 288x288 stage; no im2col
//                buffer), else 16-byte NHWC im2col + GEMM; bias fused, written
//                F32 straight into the caller's output (the reference's
//                outputs are F32)
// The input features [n, grid*grid, dim] F32 are cast to T once and shared
// by all stages.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

#include "../../include/sam3cu.h"
#include "devbuf.cuh"
#include "gemm_sm100.cuh"
#include "misc.cuh"
#include "sam3cu_internal.h"

using namespace s3;

namespace {

int ck(cudaError_t e) { return e == cudaSuccess ? kOk : kErrCuda; }

// S3CU_NECK_IM2COL=1 keeps every 3x3 conv on im2col + GEMM (measurements).
const bool g_no_implicit = [] {
  const char* e = getenv("S3CU_NECK_IM2COL");
  return e && atoi(e) != 0;
}();

struct NeckLayer {
  int kind = 0;  // 0 ConvT k2 s2, 1 Conv1x1, 2 Conv3x3
  int ci = 0, co = 0;
  bool gelu = false;
  DevBuf w;     // 16-bit: ConvT [(ky, kx, oc), ci]; Conv [co, k*k*ci] (OHWI rows)
  DevBuf bias;  // f32: ConvT [4 * co] (replicated), Conv [co]
};

struct NeckStage {
  float scale = 1.f;
  bool maxpool = false;
  int n_layers = 0;
  NeckLayer layer[4];
  int out_hw = 0;
};

// 16-bit copy of host f32 values.
int upload16(DevBuf& d, const std::vector<float>& h, int dt, cudaStream_t st) {
  DevBuf tmp;
  if (!tmp.alloc(h.size() * 4) || !d.alloc(h.size() * 2)) return kErrNoMem;
  int rc = ck(cudaMemcpyAsync(tmp.p, h.data(), h.size() * 4, cudaMemcpyHostToDevice, st));
  if (!rc) rc = launch_cast(tmp.p, kF32, d.p, dt, static_cast<int64_t>(h.size()), st);
  if (!rc) rc = ck(cudaStreamSynchronize(st));
  return rc;
}

int upload32(DevBuf& d, const std::vector<float>& h, cudaStream_t st) {
  if (!d.alloc(h.size() * 4)) return kErrNoMem;
  int rc = ck(cudaMemcpyAsync(d.p, h.data(), h.size() * 4, cudaMemcpyHostToDevice, st));
  return rc ? rc : ck(cudaStreamSynchronize(st));
}

}  // namespace

struct sam3cu_neck {
  int d_model = 0, dim = 0, grid = 0, n_scales = 0, act = kBF16, max_batch = 0;
  NeckStage stage[4];
  cudaStream_t stream = nullptr;
  DevBuf x16;          // [B * grid^2, dim] T
  DevBuf ga, gb, col;  // scratch: GEMM outputs / shuffled maps, and im2col columns
};

namespace {

EpiParams epi(void* out, int out_type, int ldo, const float* bias, int act) {
  EpiParams e;
  memset(&e, 0, sizeof(e));
  e.out = out;
  e.out_type = out_type;
  e.ldo = ldo;
  e.bias = bias;
  e.act = act;
  return e;
}

int neck_setup(sam3cu_neck* nk, const float* scales, const sam3cu_neck_weights* w) {
  cudaStream_t st = nk->stream;
  const int d = nk->d_model, dim = nk->dim;
  size_t g_max = 0, col_max = 0;  // elements per image
  int rc;
  for (int i = 0; i < nk->n_scales; ++i) {
    NeckStage& S = nk->stage[i];
    const float sf = scales[i];
    S.scale = sf;
    S.maxpool = sf < 0.75f;
    const int n_t = sf >= 3.5f ? 2 : (sf >= 1.5f ? 1 : 0);
    int H = S.maxpool ? (nk->grid - 2) / 2 + 1 : nk->grid, C = dim;
    int j = 0;
    for (int t = 0; t < n_t; ++t, ++j) {
      NeckLayer& L = S.layer[j];
      L.kind = 0;
      L.ci = C;
      L.co = C / 2;
      L.gelu = sf >= 3.5f && t == 0;  // gelu_after[0] of the 4x stage (necks.c:38-41)
      if (!w->conv_w[i][j] || L.co % 8 || L.ci % 8) return SAM3CU_EINVAL;
      // OHWI [co, 2, 2, ci] -> rows (ky, kx, oc)
      std::vector<float> wt(static_cast<size_t>(4) * L.co * L.ci), bt(static_cast<size_t>(4) * L.co, 0.f);
      for (int oc = 0; oc < L.co; ++oc)
        for (int k = 0; k < 4; ++k) {
          memcpy(&wt[(static_cast<size_t>(k) * L.co + oc) * L.ci],
                 w->conv_w[i][j] + (static_cast<size_t>(oc) * 4 + k) * L.ci, static_cast<size_t>(L.ci) * 4);
          if (w->conv_b[i][j]) bt[static_cast<size_t>(k) * L.co + oc] = w->conv_b[i][j][oc];
        }
      if ((rc = upload16(L.w, wt, nk->act, st)) || (rc = upload32(L.bias, bt, st))) return rc;
      g_max = std::max(g_max, static_cast<size_t>(H) * H * 4 * L.co);
      H *= 2;
      C = L.co;
    }
    for (int c = 0; c < 2; ++c, ++j) {
      NeckLayer& L = S.layer[j];
      L.kind = c ? 2 : 1;
      L.ci = c ? d : C;
      L.co = d;
      const int k = c ? 3 : 1;
      if (!w->conv_w[i][j] || L.ci % 8) return SAM3CU_EINVAL;
      std::vector<float> wt(w->conv_w[i][j], w->conv_w[i][j] + static_cast<size_t>(L.co) * k * k * L.ci);
      std::vector<float> bt(static_cast<size_t>(L.co), 0.f);
      if (w->conv_b[i][j]) memcpy(bt.data(), w->conv_b[i][j], static_cast<size_t>(L.co) * 4);
      if ((rc = upload16(L.w, wt, nk->act, st)) || (rc = upload32(L.bias, bt, st))) return rc;
      // the 3x3 conv needs im2col columns unless it runs as an implicit GEMM
      // (launch_conv3x3_implicit: H % 4 == 0, W % 32 == 0, C % 64 == 0)
      const bool implicit = !g_no_implicit && H % 4 == 0 && H % 32 == 0 && d % 64 == 0;
      if (c == 0) g_max = std::max(g_max, static_cast<size_t>(H) * H * d);
      else if (!implicit) col_max = std::max(col_max, static_cast<size_t>(H) * H * 9 * d);
    }
    S.n_layers = j;
    S.out_hw = H;
    // maxpool output and shuffled maps share the scratch sizes bounded above
    g_max = std::max(g_max, static_cast<size_t>(H) * H * C);
  }
  const size_t B = static_cast<size_t>(nk->max_batch);
  if (!nk->x16.alloc(B * nk->grid * nk->grid * dim * 2) || !nk->ga.alloc(B * g_max * 2) ||
      !nk->gb.alloc(B * g_max * 2) || !nk->col.alloc(B * col_max * 2))
    return kErrNoMem;
  return kOk;
}

int neck_run(sam3cu_neck* nk, const float* feat, int n, float* const* outs) {
  cudaStream_t st = nk->stream;
  const int dim = nk->dim, d = nk->d_model, T = nk->act;
  int rc = launch_cast(feat, kF32, nk->x16.p, T, static_cast<int64_t>(n) * nk->grid * nk->grid * dim, st);
  if (rc) return rc;
  for (int i = 0; i < nk->n_scales; ++i) {
    NeckStage& S = nk->stage[i];
    const void* cur = nk->x16.p;
    int H = nk->grid, C = dim;
    void* bufs[2] = {nk->ga.p, nk->gb.p};
    int nb = 0;
    if (S.maxpool) {
      if ((rc = sam3cu_maxpool2d_nhwc(cur, bufs[nb], T, n, H, H, C, 2, 2, st))) return rc;
      cur = bufs[nb];
      nb ^= 1;
      H = (H - 2) / 2 + 1;
    }
    for (int j = 0; j < S.n_layers; ++j) {
      NeckLayer& L = S.layer[j];
      const int M = n * H * H;
      if (L.kind == 0) {  // ConvT: GEMM into bufs[nb], shuffle into bufs[nb ^ 1]
        GemmShape shp{M, 4 * L.co, L.ci};
        if ((rc = launch_gemm(cur, L.ci, L.w.p, L.ci, nullptr, nullptr, T, shp,
                              epi(bufs[nb], T, 4 * L.co, L.bias.as<float>(), L.gelu ? 1 : 0), st, 0)))
          return rc;
        if ((rc = sam3cu_convt_shuffle(bufs[nb], bufs[nb ^ 1], 2, n, H, H, 2, L.co, st))) return rc;
        cur = bufs[nb ^ 1];
        H *= 2;
        C = L.co;
      } else if (L.kind == 1) {  // Conv1x1
        GemmShape shp{M, L.co, L.ci};
        if ((rc = launch_gemm(cur, L.ci, L.w.p, L.ci, nullptr, nullptr, T, shp,
                              epi(bufs[nb], T, L.co, L.bias.as<float>(), 0), st, 0)))
          return rc;
        cur = bufs[nb];
        nb ^= 1;
        C = L.co;
      } else {  // Conv3x3, pad 1 -> F32 output
        const int kk = 9 * C;
        // implicit GEMM straight from the NHWC map when the shape tiles into
        // 4x32-pixel blocks (the 288x288 stage); im2col + GEMM otherwise
        if (!g_no_implicit && H % 4 == 0 && H % 32 == 0 && C % 64 == 0) {
          rc = launch_conv3x3_implicit(cur, L.w.p, T, n, H, H, C, d, epi(outs[i], kOutF32, d, L.bias.as<float>(), 0),
                                       st);
          if (rc) return rc;  // the columns for this size were not allocated
          continue;
        }
        if ((rc = launch_conv_im2col(cur, T, false, nk->col.p, T, n, H, H, C, 3, 1, 1, kk, st))) return rc;
        GemmShape shp{M, d, kk};
        if ((rc = launch_gemm(nk->col.p, kk, L.w.p, kk, nullptr, nullptr, T, shp,
                              epi(outs[i], kOutF32, d, L.bias.as<float>(), 0), st, 0)))
          return rc;
      }
    }
  }
  return kOk;
}

}  // namespace

extern "C" {

sam3cu_neck* sam3cu_neck_create(int d_model, int dim, int grid, int n_scales, const float* scales,
                                const sam3cu_neck_weights* w, int dtype, int max_batch, int* status) {
  int st_dummy;
  int* status_p = status ? status : &st_dummy;
  *status_p = kOk;
  if (!scales || !w || n_scales < 1 || n_scales > 4 || d_model <= 0 || d_model % 8 || dim <= 0 || dim % 32 ||
      grid < 2 || max_batch <= 0) {
    *status_p = SAM3CU_EINVAL;
    return nullptr;
  }
  if (dtype != SAM3CU_BF16 && dtype != SAM3CU_F16) {
    *status_p = SAM3CU_EDTYPE;
    return nullptr;
  }
  std::unique_ptr<sam3cu_neck> nk(new sam3cu_neck());
  nk->d_model = d_model;
  nk->dim = dim;
  nk->grid = grid;
  nk->n_scales = n_scales;
  nk->act = dtype;
  nk->max_batch = max_batch;
  if (cudaStreamCreateWithFlags(&nk->stream, cudaStreamNonBlocking) != cudaSuccess) {
    *status_p = kErrCuda;
    return nullptr;
  }
  const int rc = neck_setup(nk.get(), scales, w);
  if (rc) {
    cudaStreamDestroy(nk->stream);
    *status_p = rc;
    return nullptr;
  }
  return nk.release();
}

int sam3cu_neck_out_size(const sam3cu_neck* nk, int i) {
  if (!nk || i < 0 || i >= nk->n_scales) return SAM3CU_EINVAL;
  return nk->stage[i].out_hw;
}

void* sam3cu_neck_stream(sam3cu_neck* nk) { return nk ? nk->stream : nullptr; }

int sam3cu_neck_forward_async(sam3cu_neck* nk, const float* feat, int n_images, float* const* outs) {
  if (!nk || !feat || !outs || n_images <= 0 || n_images > nk->max_batch) return SAM3CU_EINVAL;
  for (int i = 0; i < nk->n_scales; ++i)
    if (!outs[i]) return SAM3CU_EINVAL;
  return neck_run(nk, feat, n_images, outs);
}

int sam3cu_neck_forward(sam3cu_neck* nk, const float* feat, int n_images, float* const* outs) {
  const int rc = sam3cu_neck_forward_async(nk, feat, n_images, outs);
  if (rc) return rc;
  return cudaStreamSynchronize(nk->stream) == cudaSuccess ? kOk : kErrCuda;
}

void sam3cu_neck_destroy(sam3cu_neck* nk) {
  if (!nk) return;
  if (nk->stream) {
    cudaStreamSynchronize(nk->stream);
    cudaStreamDestroy(nk->stream);
  }
  delete nk;
}

}  // extern "C"
