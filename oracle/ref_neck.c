/*
 * oracle/ref_neck.c - TEST INFRASTRUCTURE: runs the reference's FPN neck
 * (src/model/necks.c: sam3_neck_init / sam3_neck_build, compiled from the
 * reference sources by oracle/Makefile) through a backend, with weights
 * supplied by the tests instead of a .sam3 file.
 */
#include <stdlib.h>
#include <string.h>

#include "backend/backend.h"
#include "backend/cpu/cpu_backend.h"
#include "core/alloc.h"
#include "core/graph.h"
#include "model/graph_helpers.h"
#include "model/necks.h"

struct sam3_backend *ref_make_backend(const struct sam3_backend_ops *ops,
				      size_t be_size, int be_type);

/* The reference CPU backend with the scratch capacity its header asks for
 * on full-size necks (cpu_backend.h:26-31: >= 1 GiB for the 3x3 conv on
 * 288x288x256); what sam3_backend_init does otherwise (backend.c:30-75). */
static struct sam3_backend *cpu_backend_big_scratch(void)
{
	struct sam3_cpu_backend *cpu = calloc(1, sizeof(*cpu));
	if (!cpu)
		return NULL;
	cpu->base.type = SAM3_BACKEND_CPU;
	cpu->base.ops = sam3_cpu_backend_ops();
	cpu->scratch_capacity = 2ul << 30;
	if (cpu->base.ops->init(&cpu->base) != SAM3_OK) {
		free(cpu);
		return NULL;
	}
	return &cpu->base;
}

/* conv (transpose) weights per stage and layer: OHWI [OC, k, k, IC] F32,
 * biases [OC] */
struct rn_weights {
	const float *w[SAM3_NECK_MAX_SCALES][SAM3_NECK_MAX_CONVS];
	const float *b[SAM3_NECK_MAX_SCALES][SAM3_NECK_MAX_CONVS];
};

/* features [grid*grid, dim] F32 -> outs[i] [H_i, W_i, d_model] F32.
 * ops NULL: the reference CPU backend.  Returns 0 on success. */
int ref_neck_run(int d_model, int dim, int grid, int n_scales,
		 const float *scales, const struct rn_weights *w,
		 const float *feat, float *const *outs, const void *ops,
		 size_t be_size, int be_type)
{
	struct sam3_neck neck;
	struct sam3_arena a;
	struct sam3_graph *g = calloc(1, sizeof(*g));
	int rc = -1;
	if (!g || sam3_arena_init(&a, 3ul << 30)) {
		free(g);
		return -2;
	}
	struct sam3_backend *be = ops ? ref_make_backend(ops, be_size, be_type)
				      : cpu_backend_big_scratch();
	if (!be)
		goto done;
	if (sam3_neck_init(&neck, d_model, dim, grid, n_scales, scales) != SAM3_OK ||
	    sam3_neck_load(&neck, NULL, &a) != SAM3_OK)
		goto done;
	for (int i = 0; i < n_scales; i++)
		for (int j = 0; j < neck.stages[i].n_convs; j++) {
			if (w->w[i][j])
				memcpy(neck.stages[i].conv_w[j]->data, w->w[i][j],
				       neck.stages[i].conv_w[j]->nbytes);
			if (w->b[i][j])
				memcpy(neck.stages[i].conv_b[j]->data, w->b[i][j],
				       neck.stages[i].conv_b[j]->nbytes);
		}
	sam3_graph_init(g);
	int fdims[2] = {grid * grid, dim};
	struct sam3_tensor *f = gh_alloc_tensor(&a, SAM3_DTYPE_F32, 2, fdims);
	struct sam3_tensor *o[SAM3_NECK_MAX_SCALES] = {0};
	if (!f)
		goto done;
	memcpy(f->data, feat, f->nbytes);
	if (sam3_neck_build(&neck, g, f, o, &a) != SAM3_OK)
		goto done;
	if (be->ops->graph_eval(be, g) != SAM3_OK)
		goto done;
	for (int i = 0; i < n_scales; i++)
		memcpy(outs[i], o[i]->data, o[i]->nbytes);
	rc = 0;
done:
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
