/*
 * oracle/ref_harness.c - flat C entry points onto the UNMODIFIED reference
 * CPU backend of sam3.c.
 *
 * TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
 * the reference's own sources (read where they lie, never copied) into
 * oracle/_ref/libsam3_ref.so.  Tests use it to pin the CPU restatement in
 * oracle/oracle.c; bench.py's reference arm times it as the CPU baseline.
 *
 * Each entry point builds the same single-node or full graph the reference
 * builds and evaluates it through the reference's own CPU kernels and thread
 * pool, so what runs is the reference's arithmetic, not ours.
 */
#include <stdlib.h>
#include <string.h>

#include "sam3/sam3_types.h"
#include "core/alloc.h"
#include "core/graph.h"
#include "core/quant.h"
#include "core/tensor.h"
#include "backend/backend.h"
#include "backend/cpu/cpu_backend.h"
#include "backend/cpu/kernels/cpu_kernels.h"
#include "model/graph_helpers.h"
#include "model/image_encoder.h"
#include "util/threadpool.h"
#include "util/log.h"

static struct sam3_threadpool *g_pool;

/* Create (or re-create) the reference thread pool with n threads; n <= 0
 * lets the reference auto-detect the core count (threadpool.c:52-74).
 * Returns the thread count in use. */
int ref_set_threads(int n)
{
	if (g_pool)
		sam3_threadpool_free(g_pool);
	g_pool = sam3_threadpool_create(n > 0 ? n : 0);
	return g_pool ? sam3_threadpool_n_threads(g_pool) : 0;
}

void ref_quiet(void)
{
	sam3_log_set_level(SAM3_LOG_ERROR);
}

static struct sam3_threadpool *pool(void)
{
	if (!g_pool)
		ref_set_threads(0);
	return g_pool;
}

static void wrap(struct sam3_tensor *t, enum sam3_dtype dt, int nd,
		 const int *dims, void *data, size_t nbytes)
{
	memset(t, 0, sizeof(*t));
	t->dtype = dt;
	t->n_dims = nd;
	for (int i = 0; i < nd; i++)
		t->dims[i] = dims[i];
	sam3_tensor_compute_strides(t);
	t->data = data;
	t->nbytes = nbytes;
}

/* C[M,N] = A[M,K] . B[K,N] through the reference kernel for the dtype:
 * dt 0 F32 (cpu_matmul.c), 1 F16 (cpu_matmul_f16.c), 2 BF16
 * (cpu_matmul_bf16.c).  16-bit operands are raw bit patterns. */
int ref_matmul(int dt, const void *a, const void *b, void *c, int M, int K,
	       int N)
{
	static const enum sam3_dtype map[3] = {SAM3_DTYPE_F32, SAM3_DTYPE_F16,
					       SAM3_DTYPE_BF16};
	size_t es = dt == 0 ? 4 : 2;
	struct sam3_tensor ta, tb, tc;
	wrap(&ta, map[dt], 2, (int[]){M, K}, (void *)a, es * M * K);
	wrap(&tb, map[dt], 2, (int[]){K, N}, (void *)b, es * K * N);
	wrap(&tc, map[dt], 2, (int[]){M, N}, c, es * M * N);
	struct sam3_node node;
	memset(&node, 0, sizeof(node));
	node.op = SAM3_OP_MATMUL;
	node.inputs[0] = &ta;
	node.inputs[1] = &tb;
	node.n_inputs = 2;
	node.output = &tc;
	if (dt == 0)
		return cpu_kernel_matmul(&node, pool());
	if (dt == 1)
		return cpu_kernel_matmul_f16(&node, pool());
	return cpu_kernel_matmul_bf16(&node, pool());
}

/* C[M,N] F32 = A[M,K] F32 . B[K,N] Q8_0 (blocks over the flattened [K,N]
 * tensor), through cpu_kernel_matmul_q8 (cpu_matmul_q8.c:168-235). */
int ref_matmul_q8(const float *a, const void *bq, float *c, int M, int K,
		  int N)
{
	struct sam3_tensor ta, tb, tc;
	wrap(&ta, SAM3_DTYPE_F32, 2, (int[]){M, K}, (void *)a, 4ul * M * K);
	wrap(&tb, SAM3_DTYPE_Q8_0, 2, (int[]){K, N}, (void *)bq,
	     sam3_q8_nbytes(K * N));
	wrap(&tc, SAM3_DTYPE_F32, 2, (int[]){M, N}, c, 4ul * M * N);
	struct sam3_node node;
	memset(&node, 0, sizeof(node));
	node.op = SAM3_OP_MATMUL;
	node.inputs[0] = &ta;
	node.inputs[1] = &tb;
	node.n_inputs = 2;
	node.output = &tc;
	return cpu_kernel_matmul_q8(&node, pool());
}

void ref_q8_quantize(const float *src, void *dst, int n)
{
	sam3_q8_quantize(src, (struct sam3_q8_block *)dst, n);
}

void ref_q8_dequantize(const void *src, float *dst, int n)
{
	sam3_q8_dequantize((const struct sam3_q8_block *)src, dst, n);
}

/* Elementwise/row ops on F32 through the reference kernels. */
int ref_gelu(const float *x, float *y, int n)
{
	struct sam3_tensor tx, ty;
	wrap(&tx, SAM3_DTYPE_F32, 1, (int[]){n}, (void *)x, 4ul * n);
	wrap(&ty, SAM3_DTYPE_F32, 1, (int[]){n}, y, 4ul * n);
	struct sam3_node node;
	memset(&node, 0, sizeof(node));
	node.op = SAM3_OP_GELU;
	node.inputs[0] = &tx;
	node.n_inputs = 1;
	node.output = &ty;
	return cpu_kernel_gelu(&node, pool());
}

int ref_layernorm(const float *x, const float *g, const float *b, float *y,
		  int rows, int cols)
{
	struct sam3_tensor tx, tg, tb, ty;
	wrap(&tx, SAM3_DTYPE_F32, 2, (int[]){rows, cols}, (void *)x,
	     4ul * rows * cols);
	wrap(&ty, SAM3_DTYPE_F32, 2, (int[]){rows, cols}, y, 4ul * rows * cols);
	struct sam3_node node;
	memset(&node, 0, sizeof(node));
	node.op = SAM3_OP_LAYERNORM;
	node.inputs[0] = &tx;
	node.n_inputs = 1;
	if (g) {
		wrap(&tg, SAM3_DTYPE_F32, 1, (int[]){cols}, (void *)g, 4ul * cols);
		node.inputs[1] = &tg;
		node.n_inputs = 2;
	}
	if (g && b) {
		wrap(&tb, SAM3_DTYPE_F32, 1, (int[]){cols}, (void *)b, 4ul * cols);
		node.inputs[2] = &tb;
		node.n_inputs = 3;
	}
	node.output = &ty;
	return cpu_kernel_layernorm(&node, pool());
}

int ref_rope(const float *x, const float *cs, const float *sn, float *y,
	     int batch, int seq, int heads, int hd)
{
	struct sam3_tensor tx, tc, ts, ty;
	int d4[] = {batch, seq, heads, hd};
	size_t nb = 4ul * batch * seq * heads * hd;
	wrap(&tx, SAM3_DTYPE_F32, 4, d4, (void *)x, nb);
	wrap(&ty, SAM3_DTYPE_F32, 4, d4, y, nb);
	wrap(&tc, SAM3_DTYPE_F32, 2, (int[]){seq, hd / 2}, (void *)cs,
	     2ul * seq * hd);
	wrap(&ts, SAM3_DTYPE_F32, 2, (int[]){seq, hd / 2}, (void *)sn,
	     2ul * seq * hd);
	struct sam3_node node;
	memset(&node, 0, sizeof(node));
	node.op = SAM3_OP_ROPE;
	node.inputs[0] = &tx;
	node.inputs[1] = &tc;
	node.inputs[2] = &ts;
	node.n_inputs = 3;
	node.output = &ty;
	node.params[0] = hd;
	return cpu_kernel_rope(&node, pool());
}

/* SDPA on [B, H, S, hd] contiguous F32 (cpu_sdpa.c:216-288). */
int ref_sdpa(const float *q, const float *k, const float *v, float *o, int B,
	     int H, int S, int hd)
{
	struct sam3_tensor tq, tk, tv, to;
	int d4[] = {B, H, S, hd};
	size_t nb = 4ul * B * H * S * hd;
	wrap(&tq, SAM3_DTYPE_F32, 4, d4, (void *)q, nb);
	wrap(&tk, SAM3_DTYPE_F32, 4, d4, (void *)k, nb);
	wrap(&tv, SAM3_DTYPE_F32, 4, d4, (void *)v, nb);
	wrap(&to, SAM3_DTYPE_F32, 4, d4, o, nb);
	struct sam3_node node;
	memset(&node, 0, sizeof(node));
	node.op = SAM3_OP_SDPA;
	node.inputs[0] = &tq;
	node.inputs[1] = &tk;
	node.inputs[2] = &tv;
	node.n_inputs = 3;
	node.output = &to;
	node.params[0] = hd;
	return cpu_kernel_sdpa(&node, pool());
}

/* Weight pointers for ref_vit_encode, F32 in the reference's own layouts
 * (image_encoder.h:34-86): per block ln1 w/b, qkv w [3e,e] / b [3e], proj
 * w [e,e] / b, ln2 w/b, fc1 w [m,e] / b [m], fc2 w [e,m] / b [e]. */
struct ref_vit_block_w {
	const float *ln1_w, *ln1_b, *qkv_w, *qkv_b, *proj_w, *proj_b;
	const float *ln2_w, *ln2_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
};

struct ref_vit_w {
	const float *patch_w, *patch_b, *pos_raw, *ln_pre_w, *ln_pre_b;
	struct ref_vit_block_w blocks[32];
};

static void put(struct sam3_tensor *t, const float *src)
{
	memcpy(t->data, src, t->nbytes);
}

/* Full sam3_vit_build (image_encoder.c:513-963) on the reference CPU
 * backend.  image: planar CHW [3,img,img] F32, already normalised.
 * out: [np, e] F32.  Returns 0 on success. */
struct sam3_backend *ref_make_backend(const struct sam3_backend_ops *ops,
					 size_t be_size, int be_type)
{
	if (!ops)
		return sam3_backend_init(SAM3_BACKEND_CPU);
	/* what sam3_backend_init does for a registered type (backend.c:36-78) */
	struct sam3_backend *be = calloc(1, be_size);
	if (!be)
		return NULL;
	be->type = (enum sam3_backend_type)be_type;
	be->ops = ops;
	if (be->ops->init(be) != SAM3_OK) {
		free(be);
		return NULL;
	}
	return be;
}

static int vit_encode_impl(int img_size, int patch_size, int embed_dim,
			   int depth, int n_heads, int window_size, int mlp_dim,
			   const struct ref_vit_w *w, const float *image,
			   float *out, const struct sam3_backend_ops *ops,
			   size_t be_size, int be_type);

int ref_vit_encode(int img_size, int patch_size, int embed_dim, int depth,
		   int n_heads, int window_size, int mlp_dim,
		   const struct ref_vit_w *w, const float *image, float *out)
{
	return vit_encode_impl(img_size, patch_size, embed_dim, depth, n_heads,
			       window_size, mlp_dim, w, image, out, NULL, 0, 0);
}

/* The reference's own sam3_vit_build driving another backend through its
 * vtable (ops = sam3_cuda_backend_ops(), be_size = its instance size). */
int ref_vit_encode_backend(int img_size, int patch_size, int embed_dim,
			   int depth, int n_heads, int window_size,
			   int mlp_dim, const struct ref_vit_w *w,
			   const float *image, float *out, const void *ops,
			   size_t be_size, int be_type)
{
	return vit_encode_impl(img_size, patch_size, embed_dim, depth, n_heads,
			       window_size, mlp_dim, w, image, out, ops,
			       be_size, be_type);
}

static int vit_encode_impl(int img_size, int patch_size, int embed_dim,
			   int depth, int n_heads, int window_size, int mlp_dim,
			   const struct ref_vit_w *w, const float *image,
			   float *out, const struct sam3_backend_ops *ops,
			   size_t be_size, int be_type)
{
	struct sam3_arena model, scratch, persist;
	struct sam3_vit *vit = calloc(1, sizeof(*vit));
	int gs = img_size / patch_size, np = gs * gs;
	size_t wbytes = 4ul * ((size_t)depth * (4ul * embed_dim * embed_dim +
		2ul * mlp_dim * embed_dim + 10ul * embed_dim + mlp_dim) +
		(size_t)embed_dim * patch_size * patch_size * 3 +
		577ul * embed_dim + 4ul * embed_dim + 4ul * np * 64);
	/* per-block-batch scratch of sam3_vit_build (two blocks per graph on
	 * the CPU backend, image_encoder.c:701-712), with headroom */
	size_t sbytes = 4ul * np * ((size_t)mlp_dim * 24 + embed_dim * 160) +
			(512ul << 20);
	int rc = -1;
	if (!vit || sam3_arena_init(&model, wbytes * 2 + (64ul << 20)) ||
	    sam3_arena_init(&scratch, sbytes) ||
	    sam3_arena_init(&persist, 8ul * np * embed_dim + (16ul << 20)))
		return -2;
	struct sam3_backend *be = ref_make_backend(ops, be_size, be_type);
	if (!be)
		goto done;
	sam3_vit_init(vit, img_size, patch_size, embed_dim, depth, n_heads,
		      window_size, mlp_dim, &model);
	if (sam3_vit_load(vit, NULL, &model) != SAM3_OK)
		goto done;
	put(vit->patch_embed_w, w->patch_w);
	put(vit->patch_embed_b, w->patch_b);
	put(vit->raw_pos_embed, w->pos_raw);
	put(vit->ln_pre_w, w->ln_pre_w);
	put(vit->ln_pre_b, w->ln_pre_b);
	for (int i = 0; i < depth; i++) {
		const struct ref_vit_block_w *b = &w->blocks[i];
		put(vit->layers[i].ln1_w, b->ln1_w);
		put(vit->layers[i].ln1_b, b->ln1_b);
		put(vit->layers[i].qkv_w, b->qkv_w);
		put(vit->layers[i].qkv_b, b->qkv_b);
		put(vit->layers[i].proj_w, b->proj_w);
		put(vit->layers[i].proj_b, b->proj_b);
		put(vit->layers[i].ln2_w, b->ln2_w);
		put(vit->layers[i].ln2_b, b->ln2_b);
		put(vit->layers[i].mlp_fc1_w, b->fc1_w);
		put(vit->layers[i].mlp_fc1_b, b->fc1_b);
		put(vit->layers[i].mlp_fc2_w, b->fc2_w);
		put(vit->layers[i].mlp_fc2_b, b->fc2_b);
	}
	{
		struct sam3_tensor *img;
		int dims[] = {3, img_size, img_size};
		img = gh_alloc_tensor(&persist, SAM3_DTYPE_F32, 3, dims);
		if (!img)
			goto done;
		memcpy(img->data, image, img->nbytes);
		struct sam3_tensor *res = sam3_vit_build(vit, be, img, &scratch,
							 &persist, NULL);
		if (!res)
			goto done;
		memcpy(out, res->data, 4ul * np * embed_dim);
		rc = 0;
	}
done:
	if (be) {
		if (ops) {
			be->ops->free(be);
			free(be);
		} else {
			sam3_backend_free(be);
		}
	}
	sam3_arena_free(&model);
	sam3_arena_free(&scratch);
	sam3_arena_free(&persist);
	free(vit);
	return rc;
}

/* gh_linear (TRANSPOSE(W) -> MATMUL -> ADD(bias)) and optionally tanh-GELU,
 * built by the reference's graph helpers on tensors of dtype dt (0 F32,
 * 1 F16, 2 BF16; 16-bit data as bit patterns), evaluated by the given
 * backend (NULL ops = the reference CPU backend).  x [M,K], w [N,K],
 * b [N] (or NULL), y [M,N].  Returns 0 on success. */
int ref_linear_graph(int dt, const void *x, const void *wt, const void *b,
		     void *y, int M, int K, int N, int gelu, const void *ops,
		     size_t be_size, int be_type)
{
	static const enum sam3_dtype map[3] = {SAM3_DTYPE_F32, SAM3_DTYPE_F16,
					       SAM3_DTYPE_BF16};
	size_t es = dt == 0 ? 4 : 2;
	struct sam3_arena a;
	if (sam3_arena_init(&a, 64ul << 20))
		return -2;
	struct sam3_graph *g = calloc(1, sizeof(*g));
	struct sam3_backend *be = ref_make_backend(ops, be_size, be_type);
	int rc = -1;
	if (!g || !be)
		goto out;
	sam3_graph_init(g);
	struct sam3_tensor *tx = gh_tensor_wrap(&a, map[dt], 2, (int[]){M, K}, (void *)x);
	struct sam3_tensor *tw = gh_tensor_wrap(&a, map[dt], 2, (int[]){N, K}, (void *)wt);
	struct sam3_tensor *tb = b ? gh_tensor_wrap(&a, map[dt], 1, (int[]){N}, (void *)b) : NULL;
	struct sam3_tensor *r = gh_linear(g, &a, tx, tw, tb);
	if (r && gelu) {
		struct sam3_tensor *o = gh_alloc_tensor(&a, map[dt], 2, (int[]){M, N});
		r = o ? sam3_graph_add_op(g, SAM3_OP_GELU, (struct sam3_tensor *[]){r}, 1, o) : NULL;
	}
	if (!r)
		goto out;
	if (be->ops->graph_eval(be, g) != SAM3_OK)
		goto out;
	memcpy(y, r->data, es * (size_t)M * N);
	rc = 0;
out:
	if (be) {
		if (ops) {
			be->ops->free(be);
			free(be);
		} else {
			sam3_backend_free(be);
		}
	}
	free(g);
	sam3_arena_free(&a);
	return rc;
}

/* A single-node graph of `op` (LAYERNORM with gamma/beta, SDPA [B,H,S,hd],
 * ROPE [B,S,H,hd] + [S,hd/2] tables, MATMUL A[M,K].B[K,N] incl. F32 x
 * Q8_0, SLICE, TRANSPOSE 4-D permute, CONV2D NHWC x OHWI, ADD) evaluated
 * by the given backend.  ins: up to 4 host tensors described by dtype /
 * n_dims / dims; params: node params.  Output shape/dtype given. */
struct ref_tdesc {
	int dtype, n_dims, dims[4];
	const void *data;
};

int ref_node_graph(int op, int n_in, const struct ref_tdesc *ins,
		   const struct ref_tdesc *outd, void *out_data,
		   const int *params, const void *ops, size_t be_size,
		   int be_type)
{
	struct sam3_arena a;
	if (sam3_arena_init(&a, 512ul << 20))
		return -2;
	struct sam3_graph *g = calloc(1, sizeof(*g));
	struct sam3_backend *be = ref_make_backend(ops, be_size, be_type);
	int rc = -1;
	if (!g || !be)
		goto out;
	sam3_graph_init(g);
	struct sam3_tensor *in[6] = {0};
	for (int i = 0; i < n_in; i++)
		in[i] = gh_tensor_wrap(&a, (enum sam3_dtype)ins[i].dtype,
				       ins[i].n_dims, ins[i].dims,
				       (void *)ins[i].data);
	struct sam3_tensor *o = gh_alloc_tensor(&a, (enum sam3_dtype)outd->dtype,
						outd->n_dims, outd->dims);
	if (!o || !sam3_graph_add_op(g, (enum sam3_op)op, in, n_in, o))
		goto out;
	for (int i = 0; i < 4; i++)
		g->nodes[0].params[i] = params ? params[i] : 0;
	if (be->ops->graph_eval(be, g) != SAM3_OK)
		goto out;
	memcpy(out_data, o->data, o->nbytes);
	rc = 0;
out:
	if (be) {
		if (ops) {
			be->ops->free(be);
			free(be);
		} else {
			sam3_backend_free(be);
		}
	}
	free(g);
	sam3_arena_free(&a);
	return rc;
}
