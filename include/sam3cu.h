/*
 * include/sam3cu.h - C ABI of the B200 (sm_100a) backend for sam3.c's image
 * encoder hot path.  Plain pointers and sizes only; no CUDA or torch types
 * (streams are passed as `void *` holding a cudaStream_t, NULL = the
 * library's default stream).
 *
 * Reference interfaces each entry point replaces (paths inside sam3.c):
 *   sam3cu_linear / sam3cu_linear_q8
 *       gh_linear = TRANSPOSE(W) -> MATMUL -> ADD(bias)
 *       (src/model/graph_helpers.c:297-322) evaluated by cpu_kernel_matmul
 *       (src/backend/cpu/kernels/cpu_matmul.c:196-257), _bf16
 *       (cpu_matmul_bf16.c:183-251), _f16 (cpu_matmul_f16.c) and the F32 x
 *       Q8_0 kernel (cpu_matmul_q8.c:168-235), plus the activation node of
 *       gh_mlp (graph_helpers.c:1258-1278, tanh-GELU cpu_gelu.c:23-36) and
 *       the residual ADD of the ViT block (image_encoder.c:868,896).
 *   sam3cu_layernorm
 *       SAM3_OP_LAYERNORM, cpu_kernel_layernorm (cpu_layernorm.c:210-254).
 *   sam3cu_sdpa
 *       SAM3_OP_SDPA, cpu_kernel_sdpa (cpu_sdpa.c:216-288), with the
 *       surrounding SLICE/PERMUTE of gh_multihead_attention_rope
 *       (graph_helpers.c:721-882) folded into strides.
 *   sam3cu_q8_quantize
 *       sam3_q8_quantize (src/core/quant.c:67-131), bit-identical output.
 *   sam3cu_vit_*
 *       sam3_vit_init / sam3_vit_load / sam3_vit_build
 *       (src/model/image_encoder.h:112-173, image_encoder.c:513-963): the
 *       whole encoder forward lowered to fused kernels on one GPU.
 *   sam3cu_tvit_*
 *       the TinyViT hot ops of image_encoder_tinyvit.c: the relative
 *       position bias expansion (expand_attention_bias :265-335), the window
 *       attention after the qkv linear (tvit_window_attention :790-866),
 *       the TinyViTBlock (tvit_block_forward :896-1052) and the MBConv
 *       block (tvit_mbconv_forward :682-720).
 *   sam3_cuda_backend_ops (include/sam3cu_backend.h)
 *       the backend vtable struct sam3_backend_ops (src/backend/backend.h:29-56).
 *
 * Every function returns 0 on success or a negative SAM3CU_E* code; the
 * codes -1..-7 are the reference's enum sam3_error values.
 */
#ifndef SAM3CU_H
#define SAM3CU_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SAM3CU_API __attribute__((visibility("default")))
#else
#define SAM3CU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types: the reference's enum sam3_dtype codes (sam3_types.h:47-54). */
enum sam3cu_dtype {
	SAM3CU_F32  = 0,
	SAM3CU_F16  = 1,
	SAM3CU_BF16 = 2,
	SAM3CU_Q8_0 = 5,
};

enum sam3cu_status {
	SAM3CU_OK        = 0,
	SAM3CU_EINVAL    = -1,   /* = SAM3_EINVAL */
	SAM3CU_ENOMEM    = -2,   /* = SAM3_ENOMEM */
	SAM3CU_EIO       = -3,   /* = SAM3_EIO */
	SAM3CU_EBACKEND  = -4,   /* = SAM3_EBACKEND */
	SAM3CU_EMODEL    = -5,   /* = SAM3_EMODEL: malformed weight file */
	SAM3CU_EDTYPE    = -6,   /* = SAM3_EDTYPE */
	SAM3CU_ESHAPE    = -101, /* shape/alignment the kernels do not take */
	SAM3CU_ETMA      = -102, /* TMA descriptor creation failed */
	SAM3CU_ELAUNCH   = -103, /* kernel launch failed */
	SAM3CU_ECUDA     = -104, /* CUDA runtime error */
	SAM3CU_EDEVICE   = -105, /* a device-side bounded wait gave up */
	SAM3CU_EDTYPE2   = -106, /* unsupported dtype combination */
	SAM3CU_ENOMEM2   = -107, /* device allocation failed */
	SAM3CU_ESCRATCH  = -108, /* request exceeds a fixed static scratch buffer */
	SAM3CU_ENOENT    = -109, /* tensor name not in a .sam3 file */
};

/* Activation fused into a linear's epilogue. */
enum sam3cu_act {
	SAM3CU_ACT_NONE = 0,
	SAM3CU_ACT_GELU_TANH = 1, /* 0.5x(1+tanh(0.7978845608(x+0.044715x^3))) */
};

/* Select and initialise a CUDA device for the calling thread. */
SAM3CU_API int sam3cu_init(int device);

/* Human-readable text for a status code. */
SAM3CU_API const char *sam3cu_strerror(int status);

/* Synchronise the device and return (and clear) the first nonzero
 * device-side error word recorded by any kernel; 0 if none. */
SAM3CU_API unsigned int sam3cu_last_device_error(void);

/* Number of kernel launches this library issued since the last reset. */
SAM3CU_API uint64_t sam3cu_launch_count(int reset);

/*
 * y[M,N] = act(x[M,K] . w[N,K]^T + bias[N]) + residual[M,N]
 *
 * x, w: device, same type: SAM3CU_BF16 or SAM3CU_F16 (K % 8 == 0), or
 * SAM3CU_F32 (K % 4 == 0; computed as 3xTF32 on the tensor cores, about
 * 2^-22 relative per product), row-major.  bias/residual: device F32 or NULL; residual may
 * equal y when y is F32.  y_dtype: SAM3CU_F32, _BF16 or _F16.  act: enum
 * sam3cu_act.  FP32 accumulation on the tensor cores.
 */
SAM3CU_API int sam3cu_linear(const void *x, int x_dtype, const void *w, const float *bias,
		  const float *residual, void *y, int y_dtype, int M, int K,
		  int N, int act, void *stream);

/*
 * Same as sam3cu_linear with a Q8_0 weight, already repacked on the device
 * by sam3cu_q8_repack: q [N,K] int8 and scales [K/32, N] F32.  K % 64 == 0.
 * x is BF16 or F16 (the weight is dequantised to that type on chip), or
 * F32 as cpu_kernel_matmul_q8 takes it (cpu_matmul_q8.c:168-235): F32 x is
 * rounded to BF16 inside the call, in a stream-ordered buffer.
 */
SAM3CU_API int sam3cu_linear_q8(const void *x, int x_dtype, const int8_t *q,
		     const float *scales, const float *bias,
		     const float *residual, void *y, int y_dtype, int M, int K,
		     int N, int act, void *stream);

/*
 * Repack reference Q8_0 blocks ({float scale; int8 q[32]}, 36 bytes,
 * quant.h:30-33) of a flattened [N,K] weight (K % 32 == 0, so each block is
 * 32 consecutive K of one row) into q [N,K] int8 + scales [K/32, N] F32.
 * All pointers device.
 */
SAM3CU_API int sam3cu_q8_repack(const void *blocks, int N, int K, int8_t *q,
		     float *scales, void *stream);

/* Quantise n F32 values (device) to Q8_0 blocks (device), bit-identical to
 * sam3_q8_quantize (quant.c:67-131). */
SAM3CU_API int sam3cu_q8_quantize(const float *src, void *blocks, int64_t n,
		       void *stream);

/* Row LayerNorm, eps 1e-5, two-pass statistics in F32 (cpu_layernorm.c).
 * x/y: device, dtypes F32/BF16/F16; gamma/beta: device F32 or NULL. */
SAM3CU_API int sam3cu_layernorm(const void *x, int x_dtype, const float *gamma,
		     const float *beta, void *y, int y_dtype, int rows,
		     int cols, void *stream);

/*
 * Multi-head attention O = softmax(Q K^T / sqrt(head_dim)) V over groups of
 * `seq` consecutive rows.  Q, K, V, O device, dtype BF16 or F16; head h of
 * row r lives at column h*head_dim of a row of ld_qkv (Q, K, V) / ld_o (O)
 * elements.  head_dim must be 64.
 */
SAM3CU_API int sam3cu_sdpa(const void *q, const void *k, const void *v, int64_t ld_qkv,
		void *o, int64_t ld_o, int dtype, int n_groups, int seq,
		int heads, int head_dim, void *stream);

/*
 * Failure-path self test (no reference counterpart).  Launches one CTA that
 * waits on an mbarrier nothing ever arrives on, bounded by limit_ns
 * (clamped to [1 ms, 2 s]).  On return *timed_out is 1 when the wait gave up,
 * recorded its device error code and let the kernel finish, i.e. the path
 * every pipeline wait in the library takes instead of hanging.  The device
 * error word is cleared again, and the context stays usable.
 */
SAM3CU_API int sam3cu_selftest_wait_timeout(unsigned long long limit_ns, int *timed_out);

/* ------------------------------------------------------------- TinyViT */

/*
 * Expand TinyViT's compact relative position bias [heads, n_offsets]
 * (n_offsets = distinct (|dy|, |dx|) pairs of a ws x ws window, numbered in
 * first-seen order) into the dense [heads, ws*ws, out_ld] table, as
 * expand_attention_bias (image_encoder_tinyvit.c:265-335) does for
 * out_ld = ws*ws.  Host memory; out_ld >= ws*ws, extra columns are zeroed.
 * Returns SAM3CU_EINVAL if n_offsets does not match ws.
 */
SAM3CU_API int sam3cu_tvit_expand_bias(const float *compact, int heads, int n_offsets, int ws,
		float *out, int out_ld);

/*
 * TinyViT window attention after the qkv linear (tvit_window_attention,
 * image_encoder_tinyvit.c:790-866): qkv [n_windows * n_tokens, ld_qkv] in
 * the per-head interleaved layout (head h: q, k, v at columns
 * h*3*hd + {0, hd, 2*hd}), scores (q/sqrt(hd))·kᵀ + bias[h], softmax,
 * ·v, written to out [n_windows * n_tokens, ld_out] with head h at columns
 * h*hd (the permute-back layout before proj).  bias: device f32
 * [heads, n_tokens, bias_ld] (sam3cu_tvit_expand_bias), bias_ld a multiple
 * of 4, or NULL.  dtype F16 or BF16, head_dim 32 or 64; device pointers.
 */
SAM3CU_API int sam3cu_tvit_window_attention(const void *qkv, int64_t ld_qkv, void *out, int64_t ld_out,
		int dtype, int n_windows, int n_tokens, int heads, int head_dim,
		const float *bias, int bias_ld, void *stream);

/*
 * One TinyViTBlock (tvit_block_forward, image_encoder_tinyvit.c:896-1052)
 * on device: x [n_images, H, W, dim] NHWC f32, updated in place.  Weights
 * are host F32 in the reference's layouts (sam3_tvit_block): linears
 * [out, in], attn_bias the compact [heads, attn_bias_offsets] table,
 * lc_w the depthwise [dim, 3, 3, 1] (OHWI) conv with its BatchNorm.
 * Any pointer but qkv_w, proj_w, lc_w, fc1_w, fc2_w may be NULL (absent).
 * dtype (BF16 / F16) is the type of the GEMM and attention operands;
 * accumulation and the residual stream stay f32.
 */
struct sam3cu_tvit_block_weights {
	const float *attn_norm_w, *attn_norm_b, *qkv_w, *qkv_b, *proj_w, *proj_b;
	const float *attn_bias;
	int attn_bias_offsets;
	const float *lc_w, *lc_b, *lc_bn_w, *lc_bn_b, *lc_bn_mean, *lc_bn_var;
	const float *mlp_norm_w, *mlp_norm_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
};
typedef struct sam3cu_tvit_block sam3cu_tvit_block;
SAM3CU_API sam3cu_tvit_block *sam3cu_tvit_block_create(int dim, int heads, int window_size,
		int mlp_dim, int dtype, const struct sam3cu_tvit_block_weights *w, int *status);
SAM3CU_API int sam3cu_tvit_block_forward(sam3cu_tvit_block *blk, float *x, int n_images,
		int H, int W, void *stream);
SAM3CU_API void sam3cu_tvit_block_destroy(sam3cu_tvit_block *blk);

/*
 * One MBConv block (tvit_mbconv_forward, image_encoder_tinyvit.c:682-720)
 * on device: conv1 1x1 + BN, GELU, depthwise 3x3 + BN, GELU, conv3 1x1 +
 * BN, + shortcut, GELU; x [n_images, H, W, dim] NHWC f32 in place.  conv1_w
 * [mid, 1, 1, dim], conv2_w [mid, 3, 3, 1], conv3_w [dim, 1, 1, mid]
 * (OHWI); conv biases and BN tensors may be NULL.
 */
struct sam3cu_tvit_mbconv_weights {
	const float *conv1_w, *conv1_b, *bn1_w, *bn1_b, *bn1_mean, *bn1_var;
	const float *conv2_w, *conv2_b, *bn2_w, *bn2_b, *bn2_mean, *bn2_var;
	const float *conv3_w, *conv3_b, *bn3_w, *bn3_b, *bn3_mean, *bn3_var;
};
typedef struct sam3cu_tvit_mbconv sam3cu_tvit_mbconv;
SAM3CU_API sam3cu_tvit_mbconv *sam3cu_tvit_mbconv_create(int dim, int mid_dim, int dtype,
		const struct sam3cu_tvit_mbconv_weights *w, int *status);
SAM3CU_API int sam3cu_tvit_mbconv_forward(sam3cu_tvit_mbconv *mb, float *x, int n_images,
		int H, int W, void *stream);
SAM3CU_API void sam3cu_tvit_mbconv_destroy(sam3cu_tvit_mbconv *mb);

/*
 * Whole TinyViT backbone (sam3_tinyvit_build, image_encoder_tinyvit.c:1058-1290)
 * on device.
 *   image [3, S, S] F32 -> patch embed (3x3/2 conv + BN + GELU, 3x3/2 conv
 *   + BN) -> layer 0: MBConv blocks -> PatchMerging -> layers 1..: TinyViT
 *   blocks, PatchMerging after every layer but the last -> head (1x1 conv,
 *   BN, GELU, 3x3 conv + bias) -> features [grid*grid, embed_dim] F32.
 * Conv weights are OHWI [OC, k, k, IC/groups] with optional bias and BN,
 * as struct sam3_tvit_conv_weights (image_encoder_tinyvit.h:37-44).
 */
struct sam3cu_tvit_conv_weights {
	const float *w, *b, *bn_w, *bn_b, *bn_mean, *bn_var;
};
#define SAM3CU_TVIT_MAX_LAYERS 4
struct sam3cu_tinyvit_config {
	int img_size;          /* 1008 */
	int n_layers;          /* 4 */
	int embed_dims[SAM3CU_TVIT_MAX_LAYERS];    /* 96, 192, 384, 576 */
	int depths[SAM3CU_TVIT_MAX_LAYERS];        /* 2, 2, 6, 2 */
	int num_heads[SAM3CU_TVIT_MAX_LAYERS];     /* 3, 6, 12, 18 */
	int window_sizes[SAM3CU_TVIT_MAX_LAYERS];  /* 7, 7, 14, 7 */
	int embed_dim;         /* head output, 1024 */
	int mlp_ratio;         /* 4 */
};
struct sam3cu_tinyvit_layer_weights {
	const struct sam3cu_tvit_mbconv_weights *conv_blocks;  /* layer 0: depths[0] entries */
	const struct sam3cu_tvit_block_weights *blocks;        /* layers >= 1: depths[l] entries */
	struct sam3cu_tvit_conv_weights pm_conv1, pm_conv2, pm_conv3;  /* PatchMerging */
};
struct sam3cu_tinyvit_weights {
	struct sam3cu_tvit_conv_weights patch_embed_0, patch_embed_1;
	struct sam3cu_tinyvit_layer_weights layers[SAM3CU_TVIT_MAX_LAYERS];
	struct sam3cu_tvit_conv_weights proj_conv1, proj_bn, proj_conv2;
};
typedef struct sam3cu_tinyvit sam3cu_tinyvit;
SAM3CU_API sam3cu_tinyvit *sam3cu_tinyvit_create(const struct sam3cu_tinyvit_config *cfg,
		const struct sam3cu_tinyvit_weights *w, int dtype, int max_batch, int *status);
/* images [n, 3, S, S] F32 -> out [n, grid*grid, embed_dim] F32; device
 * pointers when on_device, else host pointers; n <= max_batch. */
SAM3CU_API int sam3cu_tinyvit_encode(sam3cu_tinyvit *tv, const float *images, int n_images,
		float *out, int on_device);
SAM3CU_API int sam3cu_tinyvit_grid(const sam3cu_tinyvit *tv);
SAM3CU_API void sam3cu_tinyvit_destroy(sam3cu_tinyvit *tv);

/* ------------------------------------------- per-node ops (backend vtable)
 * Device helpers and the remaining encoder-graph ops, used by the
 * sam3_backend_ops lowering in cuda_backend.c.  dtype arguments take
 * SAM3CU_F32 / _F16 / _BF16; pointers are device pointers unless named
 * host.  Each replaces the CPU kernel named beside it. */

SAM3CU_API int sam3cu_dev_alloc(void **p, size_t bytes);
SAM3CU_API int sam3cu_dev_free(void *p);
SAM3CU_API int sam3cu_stream_create(void **stream);
SAM3CU_API int sam3cu_stream_destroy(void *stream);
SAM3CU_API int sam3cu_stream_sync(void *stream);
SAM3CU_API int sam3cu_memcpy_h2d(void *dst, const void *host_src, size_t n, void *stream);
SAM3CU_API int sam3cu_memcpy_d2h(void *host_dst, const void *src, size_t n, void *stream);
SAM3CU_API int sam3cu_memcpy_d2d(void *dst, const void *src, size_t n, void *stream);
/* page-locked host staging buffers and events for the backend's host
 * transfers (cudaMallocHost / cudaEvent*, no timing) */
SAM3CU_API int sam3cu_host_alloc_pinned(void **p, size_t bytes);
SAM3CU_API int sam3cu_host_free_pinned(void *p);
SAM3CU_API int sam3cu_event_create(void **event);
SAM3CU_API int sam3cu_event_destroy(void *event);
SAM3CU_API int sam3cu_event_record(void *event, void *stream);
SAM3CU_API int sam3cu_event_sync(void *event);

/* Strided gather into a contiguous tensor: dst[i0,..,i3] =
 * src[sum_k i_k * strides[k]] (element strides, up to 4 dims).  The
 * backend's lowering keeps PERMUTE / SLICE / RESHAPE results as strided
 * views and calls this only where a consumer needs contiguous data
 * (cpu_transpose.c:312-387, cpu_slice.c). */
SAM3CU_API int sam3cu_gather_strided(const void *src, void *dst, int elem_size, int n_dims,
				     const int *dims, const int64_t *strides, void *stream);

/* TRANSPOSE / PERMUTE of up to 4 dims (cpu_transpose.c:312-387):
 * out dims[i] = dims[perm[i]]; elem_size 1, 2 or 4 bytes. */
SAM3CU_API int sam3cu_permute(const void *src, void *dst, int elem_size, int n_dims,
			      const int *dims, const int *perm, void *stream);

/* SLICE [start, end) along axis (cpu_slice.c). */
SAM3CU_API int sam3cu_slice(const void *src, void *dst, int elem_size, int n_dims,
			    const int *dims, int axis, int start, int end, void *stream);

/* ADD out[i] = a[i] + b[i % nb] for nb = n, last dim or 1
 * (cpu_elementwise.c:28-62, :472-495). */
SAM3CU_API int sam3cu_add(const void *a, const void *b, void *out, int dtype, int64_t n,
			  int64_t nb, void *stream);

/* GELU, tanh form (cpu_gelu.c:23-36). */
SAM3CU_API int sam3cu_gelu(const void *x, void *y, int dtype, int64_t n, void *stream);

/* ROPE on [batch, seq, heads, hd] with F32 [seq, hd/2] cos/sin tables
 * (cpu_rope.c:35-110). */
SAM3CU_API int sam3cu_rope(const void *x, const float *cos_t, const float *sin_t, void *y,
			   int dtype, int batch, int seq, int heads, int hd, void *stream);

/* ROPE as above on row-strided data: row (b, s) of heads*hd elements
 * starts at (b*seq + s)*ldx in x and (b*seq + s)*ldy in y (element
 * strides).  Lets the backend rotate the Q / K column slices of the fused
 * QKV output without materialising the SLICE (graph_helpers.c:771-800). */
SAM3CU_API int sam3cu_rope_rows(const void *x, int64_t ldx, const float *cos_t,
				const float *sin_t, void *y, int64_t ldy, int dtype, int batch,
				int seq, int heads, int hd, void *stream);

/* CAST between F32, F16 and BF16 (cpu_cast.c), round to nearest even. */
SAM3CU_API int sam3cu_cast(const void *x, int x_dtype, void *y, int y_dtype, int64_t n,
			   void *stream);

/* F32 SDPA on contiguous [bh, s, hd] (hd 32 or 64) with an optional
 * additive [sq, sk] mask (cpu_sdpa.c:216-288, same online softmax). */
SAM3CU_API int sam3cu_sdpa_f32(const float *q, const float *k, const float *v,
			       const float *mask, float *o, int bh, int sq, int sk, int hd,
			       void *stream);

/* F32 SDPA (cpu_sdpa.c:216-288) on strided tensors: element (b, h, s, d)
 * of Q lies at q[b*qs[0] + h*qs[1] + s*qs[2] + d] (K, V, O likewise), so the
 * [B,S,H,hd] <-> [B,H,S,hd] permutes around gh_multihead_attention_rope's
 * SDPA (graph_helpers.c:840-880) need no copies.  hd 32 or 64; pointers
 * 16-byte aligned, strides multiples of 4; optional additive [sq, sk] mask
 * shared by every (b, h). */
SAM3CU_API int sam3cu_sdpa_f32_strided(const float *q, const int64_t *q_strides,
				       const float *k, const int64_t *k_strides,
				       const float *v, const int64_t *v_strides,
				       const float *mask, float *o, const int64_t *o_strides,
				       int batch, int heads, int sq, int sk, int hd,
				       void *stream);

/* Elementwise a * b with b broadcast over a trailing suffix of a's dims
 * (n % nb == 0): SAM3_OP_MUL (cpu_elementwise.c). */
SAM3CU_API int sam3cu_mul(const void *a, const void *b, void *out, int dtype, int64_t n,
			  int64_t nb, void *stream);
/* Softmax over the last dim: SAM3_OP_SOFTMAX (cpu_softmax.c:29-47). */
SAM3CU_API int sam3cu_softmax(const void *x, void *y, int dtype, int64_t rows, int cols,
			      void *stream);
/* Batched C[b] = A[b][M,K] . B[b][K,N], f32 accumulation: the N-D MATMUL
 * TinyViT's window attention emits (image_encoder_tinyvit.c:836-854). */
SAM3CU_API int sam3cu_bmm(const void *a, const void *b, void *c, int dtype, int batch, int M,
			  int K, int N, void *stream);
/* Eval BatchNorm over the last dim: SAM3_OP_BATCHNORM (cpu_batchnorm.c);
 * gamma / beta may be NULL. */
SAM3CU_API int sam3cu_batchnorm(const void *x, void *y, int dtype, int64_t n, int C,
				const float *gamma, const float *beta, const float *mean,
				const float *var, void *stream);
/* Grouped NHWC conv with OHWI weights [OC,KH,KW,C/groups] (cpu_conv2d.c,
 * groups > 1: the depthwise convs of TinyViT). */
SAM3CU_API int sam3cu_conv2d_grouped_nhwc(const void *x, const void *w, void *y, int dtype,
		int n, int H, int W, int C, int OC, int KH, int KW, int stride, int pad,
		int groups, void *stream);
/* Transposed conv NHWC x OHWI [OC,KH,KW,C] (cpu_conv_transpose2d.c): direct
 * kernel, any stride / padding; output (H-1)*stride - 2*pad + KH. */
SAM3CU_API int sam3cu_conv_transpose2d_nhwc(const void *x, const void *w, void *y, int dtype,
		int n, int H, int W, int C, int OC, int KH, int KW, int stride, int pad,
		void *stream);
/* Pixel shuffle after a kernel-k, stride-k transposed conv run as a GEMM:
 * g [n*H*W, k*k*OC] (columns (ky, kx, oc)) -> y [n, H*k, W*k, OC]. */
SAM3CU_API int sam3cu_convt_shuffle(const void *g, void *y, int elem_size, int n, int H, int W,
				    int k, int OC, void *stream);
/* NHWC max pool, kernel k, stride s, no padding (cpu_maxpool2d.c). */
SAM3CU_API int sam3cu_maxpool2d_nhwc(const void *x, void *y, int dtype, int n, int H, int W,
				     int C, int k, int s, void *stream);
/* Device-to-device 2-D copy (rows of width bytes), for CONCAT. */
SAM3CU_API int sam3cu_memcpy2d_d2d(void *dst, size_t dpitch, const void *src, size_t spitch,
				   size_t width, size_t rows, void *stream);

/* NHWC im2col for CONV2D with OHWI weights (cpu_conv2d.c): rows (n,oy,ox),
 * columns (ky,kx,c) zero-padded to kpad. */
SAM3CU_API int sam3cu_im2col_nhwc(const void *x, void *a, int dtype, int n, int H, int W,
				  int C, int kh, int kw, int stride, int pad, int kpad,
				  void *stream);

/*
 * CONV2D without any device allocation.  No counterpart in the reference:
 * it exists for callers that cannot let a library allocate device memory
 * (hosts that reserve all GPU memory in their own pool, fixed-budget
 * deployments, latency-critical loops where cudaMalloc/cudaFree would
 * synchronise the device).  Same computation as the backend's CONV2D
 * lowering: NHWC input x [n,H,W,C], OHWI weight w [OC,kh,kw,C], groups 1,
 * optional F32 bias [OC], output y [n,OH,OW,OC]; dtype F32, BF16 or F16
 * (all device pointers).  The im2col column buffer lives in a static 32 MiB
 * device array that every GPU loading the library holds until exit;
 * requests that need more return SAM3CU_ESCRATCH (split the batch).  All
 * calls share that array: calls that can overlap on the GPU race, so order
 * them on one stream.  Each call resolves the array's address in the
 * current context (cudaGetSymbolAddress, host side only); the first call on
 * a device also loads the module there, so make it before any stream
 * capture.
 */
SAM3CU_API int sam3cu_conv2d_nhwc_noalloc(const void *x, const void *w, const float *bias,
					  void *y, int dtype, int n, int H, int W, int C,
					  int OC, int kh, int kw, int stride, int pad,
					  void *stream);

/* Q8_0 blocks -> F32 (sam3_q8_dequantize, quant.c:134-151). */
SAM3CU_API int sam3cu_q8_dequantize(const void *blocks, float *out, int64_t n, void *stream);

/* ---------------------------------------------------------------- ViT */

struct sam3cu_vit_config {
	int img_size;    /* 1008 */
	int patch_size;  /* 14 */
	int embed_dim;   /* 1024 */
	int depth;       /* 32; blocks 7, 15, 23, 31 are global */
	int n_heads;     /* 16 (head_dim must be 64) */
	int window_size; /* 24 */
	int mlp_dim;     /* 4736 */
};

/* One block's weights, HOST F32 in the reference layouts
 * (image_encoder.h:76-86): W [out,in] row-major, QKV fused [3e, e]. */
struct sam3cu_vit_block_weights {
	const float *ln1_w, *ln1_b, *qkv_w, *qkv_b, *proj_w, *proj_b;
	const float *ln2_w, *ln2_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
};

struct sam3cu_vit_weights {
	const float *patch_w;  /* [e, ps, ps, 3] OHWI */
	const float *patch_b;  /* [e] */
	const float *pos_raw;  /* [1, 24*24+1, e], CLS row first */
	const float *ln_pre_w, *ln_pre_b;
	struct sam3cu_vit_block_weights blocks[32];
};

typedef struct sam3cu_vit sam3cu_vit;

/*
 * Create an encoder on the current device and upload its weights.
 * weight_dtype: SAM3CU_BF16 or SAM3CU_F16 (weights rounded RNE, activations
 * in the same type, residual stream F32) or SAM3CU_Q8_0 (linear weights
 * quantised exactly as sam3_q8_quantize, activations BF16).  max_batch
 * bounds the images per sam3cu_vit_encode call (activation memory is
 * allocated once for it).  Returns NULL on failure (see *status).
 */
SAM3CU_API sam3cu_vit *sam3cu_vit_create(const struct sam3cu_vit_config *cfg,
			      const struct sam3cu_vit_weights *w,
			      int weight_dtype, int max_batch, int *status);

SAM3CU_API void sam3cu_vit_destroy(sam3cu_vit *vit);

/*
 * Encode n_images planar CHW F32 images (normalised, [n, 3, img, img]) into
 * features [n, np, e] F32 in raster patch order (the layout sam3_vit_build
 * returns).  images/out: device pointers when on_device != 0 (then
 * n_images <= max_batch), else host pointers.  With host pointers any
 * n_images is accepted: the batch is encoded in chunks of max_batch (a batch
 * of 4 .. max_batch images in two halves), and with page-locked host memory
 * each chunk's copies overlap the neighbouring chunks' compute (two staging
 * sets, separate copy streams).  Blocks until done.
 */
SAM3CU_API int sam3cu_vit_encode(sam3cu_vit *vit, const float *images, int n_images,
		      float *out, int on_device);

/* Device-resident variant for callers that time or pipeline: enqueue on the
 * encoder's stream only (images/out device), return without waiting. */
SAM3CU_API int sam3cu_vit_encode_async(sam3cu_vit *vit, const float *images,
			    int n_images, float *out);

/* cudaStream_t of the encoder, as void *. */
SAM3CU_API void *sam3cu_vit_stream(sam3cu_vit *vit);

/*
 * Run one encode with direct launches (no graph) and a CUDA event after
 * every launch; ms[k] / counts[k] receive the total device time and launch
 * count per kind: 0 GEMM, 1 attention, 2 LayerNorm, 3 other.  images/out
 * device.  For measurement only: the per-launch events serialise nothing
 * but add a little host overhead.
 */
SAM3CU_API int sam3cu_vit_profile(sam3cu_vit *vit, const float *images,
				  int n_images, float *out, double *ms,
				  int *counts);

/* Launch kinds of sam3cu_vit_profile_detail. */
enum sam3cu_prof_kind {
	SAM3CU_PROF_PATCH = 0,        /* patch-embedding GEMM */
	SAM3CU_PROF_QKV = 1,
	SAM3CU_PROF_PROJ = 2,
	SAM3CU_PROF_FC1 = 3,
	SAM3CU_PROF_FC2 = 4,
	SAM3CU_PROF_DEQUANT = 5,      /* Q8_0: a block's weights to 16-bit */
	SAM3CU_PROF_ATTN_WINDOW = 6,
	SAM3CU_PROF_ATTN_GLOBAL = 7,
	SAM3CU_PROF_LAYERNORM = 8,
	SAM3CU_PROF_OTHER = 9,
	SAM3CU_PROF_KINDS = 10
};

/* As sam3cu_vit_profile with ms / counts of SAM3CU_PROF_KINDS entries, one
 * per enum sam3cu_prof_kind (sam3cu_vit_profile sums kinds 0-5 as GEMM,
 * 6-7 as attention).  No counterpart in the reference. */
SAM3CU_API int sam3cu_vit_profile_detail(sam3cu_vit *vit, const float *images,
					 int n_images, float *out, double *ms,
					 int *counts);

/* Kernel launches one encode of n_images enqueues. */
SAM3CU_API int sam3cu_vit_launches_per_encode(sam3cu_vit *vit, int n_images);

/* ---------------------------------------------------------------- FPN neck */

/*
 * The SAM3 FPN neck: sam3_neck_init + sam3_neck_build (src/model/necks.c:
 * 150-178, 260-360) as fused kernels.  Per scale factor (>= 3.5: two k2s2
 * ConvTranspose with GELU after the first; >= 1.5: one; >= 0.75: none;
 * below: a 2x2 max pool first), then Conv1x1 to d_model and Conv3x3 (pad 1),
 * each with its bias.  Weights are HOST F32 in the reference layouts
 * (struct sam3_neck, necks.h): conv_w[stage][layer] OHWI in build order,
 * conv_b[stage][layer] (NULL: zero).  dtype: SAM3CU_BF16 or SAM3CU_F16,
 * the compute type (F32 accumulation); dim % 32 == 0, d_model % 8 == 0.
 */
struct sam3cu_neck_weights {
	const float *conv_w[4][4];
	const float *conv_b[4][4];
};
typedef struct sam3cu_neck sam3cu_neck;
SAM3CU_API sam3cu_neck *sam3cu_neck_create(int d_model, int dim, int grid, int n_scales,
					   const float *scales,
					   const struct sam3cu_neck_weights *w, int dtype,
					   int max_batch, int *status);
/* Output side length of stage i (outputs are [n, H_i, H_i, d_model]). */
SAM3CU_API int sam3cu_neck_out_size(const sam3cu_neck *nk, int i);
/* feat: device [n, grid*grid, dim] F32 (the ViT output layout); outs[i]:
 * device F32 [n, H_i, H_i, d_model].  Blocks until done. */
SAM3CU_API int sam3cu_neck_forward(sam3cu_neck *nk, const float *feat, int n_images,
				   float *const *outs);
/* The same, enqueued on the neck's stream without waiting. */
SAM3CU_API int sam3cu_neck_forward_async(sam3cu_neck *nk, const float *feat, int n_images,
					 float *const *outs);
/* cudaStream_t of the neck, as void *. */
SAM3CU_API void *sam3cu_neck_stream(sam3cu_neck *nk);
SAM3CU_API void sam3cu_neck_destroy(sam3cu_neck *nk);

/* ------------------------------------------------------ .sam3 weight files */

/*
 * Validate a .sam3 file image (the bytes sam3_weight_open maps,
 * src/core/weight.c:303-470; format src/core/weight.h:26-72): magic, version
 * 3 or 4, tensor table and every tensor's data range inside the image.
 * Returns SAM3CU_EMODEL for a malformed image.  Host only, no device work.
 */
SAM3CU_API int sam3cu_sam3_check(const void *image, size_t bytes, uint32_t *n_tensors,
				 uint32_t *version);

/*
 * sam3_weight_find + sam3_weight_to_tensor (weight.c:505-558) on a file
 * image: dtype (enum sam3_dtype), n_dims, dims[4], the tensor's byte offset
 * from the start of the IMAGE and its byte size.  SAM3CU_ENOENT if absent.
 */
SAM3CU_API int sam3cu_sam3_find(const void *image, size_t bytes, const char *name, int *dtype,
				int *n_dims, int *dims, uint64_t *data_offset, uint64_t *nbytes);

/*
 * sam3_vit_load (src/model/image_encoder.c:223-456) + sam3cu_vit_create from
 * a .sam3 file image: the detector_model.vision_encoder.backbone.* tensors
 * are found by the reference's names and uploaded AS STORED (F32, F16, BF16
 * or Q8_0, the dtypes sam3_convert writes), then converted on the device.
 * Q8_0 linear weights going to a SAM3CU_Q8_0 encoder are only repacked,
 * never requantised, so the int8 payload of the file is what the GEMMs
 * read; a Q8_0 tensor anywhere else (the converter quantises every float
 * tensor of >= 1024 elements, tools/cli_convert.c:340-352, LayerNorm gains
 * and biases included) is dequantised to F32.  q/k/v are concatenated into
 * the fused QKV as fuse_3 does.
 * cfg NULL: the shape is taken from the file (embed_dim and patch_size from
 * the patch weight, mlp_dim from layer 0's fc1, depth from the layers
 * present, img_size from the header; 64-wide heads, window 24).
 * A missing or mis-sized tensor returns SAM3CU_EMODEL (the reference warns
 * and continues with an uninitialised tensor, graph_helpers.c:143), except
 * the patch bias, which is optional and zero when absent, as in the
 * reference (image_encoder.c:271-297).  The image may be freed after the
 * call returns.
 */
SAM3CU_API sam3cu_vit *sam3cu_vit_create_from_sam3(const void *image, size_t bytes,
						   const struct sam3cu_vit_config *cfg,
						   int weight_dtype, int max_batch, int *status);

/* The shape an encoder was created with (after sam3cu_vit_create_from_sam3
 * with cfg NULL: the one read from the file).  No counterpart in the
 * reference, whose struct sam3_vit is caller-visible. */
SAM3CU_API int sam3cu_vit_get_config(const sam3cu_vit *vit, struct sam3cu_vit_config *cfg);

#ifdef __cplusplus
}
#endif

#endif /* SAM3CU_H */
