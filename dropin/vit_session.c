/*
 * vit_session.c - the reference's image encoder driving the CUDA backend,
 * the way sam3.c itself would once the backend is registered.
 *
 * The encoder graph is built by the UNMODIFIED reference model code
 * (sam3_vit_init / sam3_vit_load / sam3_vit_build, image_encoder.c:223-963,
 * compiled from the sam3.c sources by dropin/Makefile) and evaluated through
 * the vtable that sam3_cuda_backend_ops() returns (include/sam3cu_backend.h).
 * A session keeps the model, its arenas and the backend alive across
 * images, as a sam3_ctx does between sam3_set_image calls, so the weights
 * are uploaded to the device once and each encode pays only what the
 * reference's call sequence costs: its graph evaluations, the host <->
 * device copies of the image and of the residual stream between graphs,
 * and the final read-back.
 *
 * This file is the measurement harness of the drop-in path (bench.py's
 * dropin leg, tests/test_dropin_gpu.py); it is not part of libsam3cu.
 */
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "sam3/sam3_types.h"
#include "core/alloc.h"
#include "core/graph.h"
#include "core/tensor.h"
#include "backend/backend.h"
#include "model/image_encoder.h"
#include "model/graph_helpers.h"

#include "../include/sam3cu_backend.h"

struct dropin_vit {
	struct sam3_vit     vit;
	struct sam3_arena   model, scratch, persist;
	struct sam3_backend *be;
	int                 np, e, img;
};

/* the backend instance, as sam3_backend_init makes it for a registered
 * type (backend.c:36-78): zeroed subclass, base first, then ops->init */
static struct sam3_backend *make_backend(int device)
{
	struct sam3_cuda_backend *cb = calloc(1, sizeof(*cb));
	if (!cb)
		return NULL;
	/* the value SAM3_BACKEND_CUDA takes once appended to the reference's
	 * enum sam3_backend_type (backend.h:22-25) */
	cb->base.type = (enum sam3_backend_type)(SAM3_BACKEND_METAL + 1);
	cb->base.ops = sam3_cuda_backend_ops();
	cb->device = device;
	if (cb->base.ops->init(&cb->base) != SAM3_OK) {
		free(cb);
		return NULL;
	}
	return &cb->base;
}

static void fill(struct sam3_tensor *t, const float *src)
{
	memcpy(t->data, src, t->nbytes);
}

void dropin_vit_free(struct dropin_vit *s)
{
	if (!s)
		return;
	if (s->be) {
		s->be->ops->free(s->be);
		free(s->be);
	}
	sam3_arena_free(&s->model);
	sam3_arena_free(&s->scratch);
	sam3_arena_free(&s->persist);
	free(s);
}

/*
 * cfg: img_size, patch_size, embed_dim, depth, n_heads, window_size, mlp_dim.
 * w:   5 + 12*depth host F32 arrays in this order: patch_w (OHWI), patch_b,
 *      pos_raw [1,577,e], ln_pre_w, ln_pre_b, then per block ln1_w, ln1_b,
 *      qkv_w [3e,e], qkv_b, proj_w, proj_b, ln2_w, ln2_b, fc1_w, fc1_b,
 *      fc2_w, fc2_b (the tensors of sam3_vit_load, image_encoder.c:346-452).
 */
struct dropin_vit *dropin_vit_create(const int *cfg, const float *const *w, int device)
{
	struct dropin_vit *s = calloc(1, sizeof(*s));
	if (!s)
		return NULL;
	int img = cfg[0], ps = cfg[1], e = cfg[2], depth = cfg[3], mlp = cfg[6];
	int gs = img / ps, np = gs * gs;
	size_t wbytes = 4ul * ((size_t)depth * (4ul * e * e + 2ul * mlp * e + 10ul * e + mlp) +
			       (size_t)e * ps * ps * 3 + 577ul * e + 4ul * e + 4ul * np * 64);
	/* the CPU-style scratch of sam3_vit_build: every node output gets a
	 * host buffer (two blocks per graph, image_encoder.c:701-712) */
	size_t sbytes = 4ul * np * ((size_t)mlp * 24 + e * 160) + (512ul << 20);
	s->np = np;
	s->e = e;
	s->img = img;
	if (sam3_arena_init(&s->model, wbytes * 2 + (64ul << 20)) ||
	    sam3_arena_init(&s->scratch, sbytes) ||
	    sam3_arena_init(&s->persist, 8ul * np * e + 4ul * 3 * img * img + (16ul << 20)))
		goto fail;
	s->be = make_backend(device);
	if (!s->be)
		goto fail;
	sam3_vit_init(&s->vit, img, ps, e, depth, cfg[4], cfg[5], mlp, &s->model);
	if (sam3_vit_load(&s->vit, NULL, &s->model) != SAM3_OK)
		goto fail;
	fill(s->vit.patch_embed_w, w[0]);
	fill(s->vit.patch_embed_b, w[1]);
	fill(s->vit.raw_pos_embed, w[2]);
	fill(s->vit.ln_pre_w, w[3]);
	fill(s->vit.ln_pre_b, w[4]);
	for (int i = 0; i < depth; i++) {
		const float *const *b = w + 5 + 12 * i;
		__typeof__(s->vit.layers[0]) *L = &s->vit.layers[i];
		fill(L->ln1_w, b[0]);
		fill(L->ln1_b, b[1]);
		fill(L->qkv_w, b[2]);
		fill(L->qkv_b, b[3]);
		fill(L->proj_w, b[4]);
		fill(L->proj_b, b[5]);
		fill(L->ln2_w, b[6]);
		fill(L->ln2_b, b[7]);
		fill(L->mlp_fc1_w, b[8]);
		fill(L->mlp_fc1_b, b[9]);
		fill(L->mlp_fc2_w, b[10]);
		fill(L->mlp_fc2_b, b[11]);
	}
	return s;
fail:
	dropin_vit_free(s);
	return NULL;
}

/*
 * One image through sam3_vit_build: image planar CHW [3,img,img] F32
 * (normalised), out [np, e] F32.  Returns 0, or the failing step's code.
 * *seconds receives the host wall time of the sam3_vit_build call alone
 * (graph building, evaluation, copies; not the final memcpy into out).
 */
int dropin_vit_encode(struct dropin_vit *s, const float *image, float *out, double *seconds)
{
	sam3_arena_reset(&s->persist);
	sam3_arena_reset(&s->scratch);
	int dims[] = {3, s->img, s->img};
	struct sam3_tensor *img = gh_alloc_tensor(&s->persist, SAM3_DTYPE_F32, 3, dims);
	if (!img)
		return -2;
	memcpy(img->data, image, img->nbytes);
	struct timespec t0, t1;
	clock_gettime(CLOCK_MONOTONIC, &t0);
	struct sam3_tensor *res = sam3_vit_build(&s->vit, s->be, img, &s->scratch, &s->persist, NULL);
	clock_gettime(CLOCK_MONOTONIC, &t1);
	if (!res)
		return -1;
	if (seconds)
		*seconds = (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
	memcpy(out, res->data, 4ul * s->np * s->e);
	return 0;
}

/* print and reset the backend's SAM3CU_VTABLE_PROFILE counters */
void dropin_vit_profile_dump(struct dropin_vit *s)
{
	sam3cu_backend_profile_dump(s->be);
}
