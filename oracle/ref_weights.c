/*
 * oracle/ref_weights.c - TEST INFRASTRUCTURE: .sam3 weight files written and
 * read by the reference's own code (src/core/weight.c, compiled from the
 * reference sources by oracle/Makefile), and the reference ViT loaded from
 * such a file (sam3_vit_load with a real sam3_weight_file).
 *
 * The tests use these to pin the CUDA library's .sam3 reader and its
 * file-driven encoder against the reference's writer, reader and loader.
 */
#include <stdlib.h>
#include <string.h>

#include "sam3/sam3_types.h"
#include "backend/backend.h"
#include "core/alloc.h"
#include "core/half.h"
#include "core/quant.h"
#include "core/weight.h"
#include "model/graph_helpers.h"
#include "model/image_encoder.h"

/* One tensor handed to the writer: host bytes in dtype (F32, F16 or BF16). */
struct rw_tensor {
	const char *name;
	int dtype;
	int n_dims;
	int dims[SAM3_MAX_DIMS];
	const void *data;
};

struct rw_state {
	const struct rw_tensor *t;
	int n;
	int quantize;
};

static size_t rw_numel(const struct rw_tensor *t)
{
	size_t n = 1;
	for (int d = 0; d < t->n_dims; d++)
		n *= (size_t)t->dims[d];
	return n;
}

/* the converter's rule (tools/cli_convert.c:340-352, threshold 1024 set at
 * :597): every F32/F16/BF16 tensor of >= 1024 elements becomes Q8_0 */
static int rw_quantised(const struct rw_state *s, const struct rw_tensor *t)
{
	return s->quantize && rw_numel(t) >= 1024 &&
	       (t->dtype == SAM3_DTYPE_F32 || t->dtype == SAM3_DTYPE_F16 ||
		t->dtype == SAM3_DTYPE_BF16);
}

static enum sam3_error rw_open(struct weight_reader *r, const char *path)
{
	(void)r;
	(void)path;
	return SAM3_OK;
}

static int rw_n_tensors(struct weight_reader *r)
{
	return ((struct rw_state *)r->impl)->n;
}

static enum sam3_error rw_info(struct weight_reader *r, int idx,
			       struct weight_tensor_info *info)
{
	struct rw_state *s = r->impl;
	const struct rw_tensor *t = &s->t[idx];
	memset(info, 0, sizeof(*info));
	info->name = t->name;
	info->n_dims = t->n_dims;
	for (int d = 0; d < t->n_dims; d++)
		info->dims[d] = t->dims[d];
	if (rw_quantised(s, t)) {
		info->dtype = SAM3_DTYPE_Q8_0;
		info->nbytes = sam3_q8_nbytes((int)rw_numel(t));
	} else {
		info->dtype = (enum sam3_dtype)t->dtype;
		info->nbytes = rw_numel(t) * sam3_dtype_size(info->dtype);
	}
	return SAM3_OK;
}

static enum sam3_error rw_read(struct weight_reader *r, int idx, void *dst,
			       size_t dst_size)
{
	struct rw_state *s = r->impl;
	const struct rw_tensor *t = &s->t[idx];
	size_t n = rw_numel(t);
	if (!rw_quantised(s, t)) {
		size_t nb = n * sam3_dtype_size((enum sam3_dtype)t->dtype);
		if (nb > dst_size)
			return SAM3_EINVAL;
		memcpy(dst, t->data, nb);
		return SAM3_OK;
	}
	/* as qr_read_tensor_data (cli_convert.c:357-425): widen, then
	 * sam3_q8_quantize */
	float *f = malloc(n * sizeof(float));
	if (!f)
		return SAM3_ENOMEM;
	for (size_t i = 0; i < n; i++) {
		if (t->dtype == SAM3_DTYPE_F32)
			f[i] = ((const float *)t->data)[i];
		else if (t->dtype == SAM3_DTYPE_F16)
			f[i] = fp16_to_f32(((const uint16_t *)t->data)[i]);
		else
			f[i] = bf16_to_f32(((const uint16_t *)t->data)[i]);
	}
	sam3_q8_quantize(f, (struct sam3_q8_block *)dst, (int)n);
	free(f);
	return SAM3_OK;
}

static void rw_close(struct weight_reader *r)
{
	(void)r;
}

static const struct weight_reader_ops rw_ops = {
	rw_open, rw_n_tensors, rw_info, rw_read, rw_close,
};

/* Write a .sam3 file with the reference's sam3_weight_write.  Returns the
 * sam3_error code. */
int ref_write_sam3(const char *path, const struct rw_tensor *t, int n,
		   int quantize, int image_size, int encoder_dim, int n_layers)
{
	struct rw_state s = {t, n, quantize};
	struct weight_reader r = {&rw_ops, &s};
	struct sam3_model_config cfg;
	memset(&cfg, 0, sizeof(cfg));
	cfg.image_size = image_size;
	cfg.encoder_dim = encoder_dim;
	cfg.n_encoder_layers = n_layers;
	return sam3_weight_write(path, &cfg, &r);
}

/* sam3_weight_open + sam3_weight_find on a file: the descriptor's fields
 * and its data offset from the start of the mapping.  Returns 0, 1 when the
 * tensor is absent, or the (negative) sam3_error of sam3_weight_open. */
int ref_find_sam3(const char *path, const char *name, int *dtype,
		  int *n_dims, int *dims, unsigned long long *offset,
		  unsigned long long *nbytes)
{
	struct sam3_weight_file wf;
	memset(&wf, 0, sizeof(wf));
	enum sam3_error err = sam3_weight_open(&wf, path);
	if (err != SAM3_OK)
		return (int)err;
	const struct sam3_weight_tensor_desc *d = sam3_weight_find(&wf, name);
	int rc = 1;
	if (d) {
		*dtype = (int)d->dtype;
		*n_dims = (int)d->n_dims;
		for (int i = 0; i < SAM3_MAX_DIMS; i++)
			dims[i] = d->dims[i];
		*offset = (unsigned long long)((const char *)
			sam3_weight_tensor_data(&wf, d) - (const char *)wf.mapped);
		*nbytes = d->data_size;
		rc = 0;
	}
	sam3_weight_close(&wf);
	return rc;
}

/* sam3_weight_open alone: its status for a (possibly malformed) file. */
int ref_open_sam3(const char *path)
{
	struct sam3_weight_file wf;
	memset(&wf, 0, sizeof(wf));
	enum sam3_error err = sam3_weight_open(&wf, path);
	if (err == SAM3_OK)
		sam3_weight_close(&wf);
	return (int)err;
}

struct sam3_backend *ref_make_backend(const struct sam3_backend_ops *ops,
				      size_t be_size, int be_type);

/* The reference encoder the way an application runs it: sam3_weight_open,
 * sam3_vit_init, sam3_vit_load(vit, &wf, ...), sam3_vit_build on the CPU
 * backend.  image: planar CHW [3,img,img] F32, normalised; out [np, e] F32.
 * Returns 0 on success. */
int ref_vit_encode_file(const char *path, int img_size, int patch_size,
			int embed_dim, int depth, int n_heads, int window_size,
			int mlp_dim, const float *image, float *out)
{
	struct sam3_weight_file wf;
	struct sam3_arena model, scratch, persist;
	struct sam3_vit *vit = calloc(1, sizeof(*vit));
	int gs = img_size / patch_size, np = gs * gs;
	size_t sbytes = 4ul * np * ((size_t)mlp_dim * 24 + embed_dim * 160) +
			(512ul << 20);
	int rc = -1;
	memset(&wf, 0, sizeof(wf));
	if (!vit || sam3_weight_open(&wf, path) != SAM3_OK) {
		free(vit);
		return -3;
	}
	/* weights stay in the mapping; the arena holds headers, fused QKV and
	 * the RoPE / pos-embed tables */
	size_t mbytes = 4ul * (size_t)depth * (3ul * embed_dim * embed_dim +
		3ul * embed_dim) + 4ul * np * (embed_dim + 128) + (64ul << 20);
	if (sam3_arena_init(&model, mbytes) || sam3_arena_init(&scratch, sbytes) ||
	    sam3_arena_init(&persist, 8ul * np * embed_dim + (16ul << 20))) {
		sam3_weight_close(&wf);
		free(vit);
		return -2;
	}
	struct sam3_backend *be = ref_make_backend(NULL, 0, 0);
	if (!be)
		goto done;
	sam3_vit_init(vit, img_size, patch_size, embed_dim, depth, n_heads,
		      window_size, mlp_dim, &model);
	if (sam3_vit_load(vit, &wf, &model) != SAM3_OK)
		goto done;
	{
		int dims[] = {3, img_size, img_size};
		struct sam3_tensor *img = gh_alloc_tensor(&persist, SAM3_DTYPE_F32,
							  3, dims);
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
	if (be)
		sam3_backend_free(be);
	sam3_arena_free(&model);
	sam3_arena_free(&scratch);
	sam3_arena_free(&persist);
	sam3_weight_close(&wf);
	free(vit);
	return rc;
}
