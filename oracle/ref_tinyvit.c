/*
 * oracle/ref_tinyvit.c - TEST INFRASTRUCTURE: exposes the reference's
 * static TinyViT helpers to the parity tests.
 *
 * The reference source file is compiled as part of this translation unit
 * (it is included, not copied), so its file-static functions, such as
 * expand_attention_bias (image_encoder_tinyvit.c:265-335), can be called
 * unmodified.
 */
#include "model/image_encoder_tinyvit.c"

/* Dense [heads, ws*ws, ws*ws] bias from the compact [heads, n_off] table,
 * by the reference's own expand_attention_bias.  Returns 0 on success. */
int ref_tvit_expand_bias(const float *compact, int heads, int n_off, int ws,
			 float *out)
{
	struct sam3_arena a;
	if (sam3_arena_init(&a, 64ul << 20))
		return -2;
	int dims[2] = {heads, n_off};
	struct sam3_tensor *c = gh_tensor_wrap(&a, SAM3_DTYPE_F32, 2, dims,
					       (void *)compact);
	int rc = -1;
	struct sam3_tensor *e = c ? expand_attention_bias(c, &a, heads, ws) : NULL;
	if (e) {
		memcpy(out, e->data, e->nbytes);
		rc = 0;
	}
	sam3_arena_free(&a);
	return rc;
}

/* ---- sam3_tinyvit_build through a backend ------------------------------ */

struct sam3_backend *ref_make_backend(const struct sam3_backend_ops *ops,
				      size_t be_size, int be_type);

/* Weight tree with the layouts of the CUDA library's sam3cu_tinyvit_*
 * structs (and oracle.c's orc_tinyvit_*), so the tests build it once. */
struct rt_conv { const float *w, *b, *bn_w, *bn_b, *bn_mean, *bn_var; };
struct rt_block {
	const float *attn_norm_w, *attn_norm_b, *qkv_w, *qkv_b, *proj_w,
		*proj_b, *attn_bias;
	int attn_bias_offsets;
	const float *lc_w, *lc_b, *lc_bn_w, *lc_bn_b, *lc_bn_mean, *lc_bn_var;
	const float *mlp_norm_w, *mlp_norm_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
};
struct rt_mb {
	struct { const float *w, *b, *bn_w, *bn_b, *bn_mean, *bn_var; } c[3];
};
struct rt_cfg {
	int img_size, n_layers, embed_dims[4], depths[4], num_heads[4],
	    window_sizes[4], embed_dim, mlp_ratio;
};
struct rt_layer {
	const struct rt_mb *conv_blocks;
	const struct rt_block *blocks;
	struct rt_conv pm_conv1, pm_conv2, pm_conv3;
};
struct rt_weights {
	struct rt_conv patch_embed_0, patch_embed_1;
	struct rt_layer layers[4];
	struct rt_conv proj_conv1, proj_bn, proj_conv2;
};

static void rt_put(struct sam3_tensor *t, const float *src)
{
	if (t && src)
		memcpy(t->data, src, t->nbytes);
}

static void rt_put_conv(struct sam3_tvit_conv_weights *cw, const float *w,
			const float *b, const float *g, const float *be,
			const float *mu, const float *var)
{
	rt_put(cw->conv_w, w);
	rt_put(cw->conv_b, b);
	rt_put(cw->bn_w, g);
	rt_put(cw->bn_b, be);
	rt_put(cw->bn_mean, mu);
	rt_put(cw->bn_var, var);
}

/* The reference's own sam3_tinyvit_init / _load (weight file NULL: zeroed
 * tensors, then filled from `w`) / _build, evaluated by the backend given
 * by ops (NULL: the reference CPU backend).  image [3, S, S]; out
 * [grid*grid, embed_dim].  Returns 0 on success. */
int ref_tinyvit_encode(const struct rt_cfg *c, const struct rt_weights *w,
		       const float *image, float *out, const void *ops,
		       size_t be_size, int be_type)
{
	struct sam3_tinyvit tv;
	struct sam3_arena model, scratch, persist;
	int rc = -1;
	if (sam3_arena_init(&model, 1ul << 30))
		return -2;
	if (sam3_arena_init(&scratch, 2ul << 30)) {
		sam3_arena_free(&model);
		return -2;
	}
	if (sam3_arena_init(&persist, 256ul << 20)) {
		sam3_arena_free(&model);
		sam3_arena_free(&scratch);
		return -2;
	}
	struct sam3_backend *be = ref_make_backend(ops, be_size, be_type);
	if (!be)
		goto done;
	if (sam3_tinyvit_init(&tv, c->embed_dims, c->depths, c->num_heads,
			      c->window_sizes, c->n_layers, c->img_size,
			      c->embed_dim, c->mlp_ratio) != SAM3_OK)
		goto done;
	if (sam3_tinyvit_load(&tv, NULL, &model) != SAM3_OK)
		goto done;
	const struct rt_conv *p;
	p = &w->patch_embed_0;
	rt_put_conv(&tv.patch_embed_0, p->w, p->b, p->bn_w, p->bn_b, p->bn_mean, p->bn_var);
	p = &w->patch_embed_1;
	rt_put_conv(&tv.patch_embed_1, p->w, p->b, p->bn_w, p->bn_b, p->bn_mean, p->bn_var);
	for (int l = 0; l < c->n_layers; l++) {
		struct sam3_tvit_layer *L = &tv.layers[l];
		const struct rt_layer *lw = &w->layers[l];
		for (int b = 0; b < L->n_blocks; b++) {
			struct sam3_tvit_block *B = &L->blocks[b];
			if (B->is_conv_block) {
				const struct rt_mb *mb = &lw->conv_blocks[b];
				struct sam3_tvit_conv_weights *cv[3] = {
					&B->mbconv.conv1, &B->mbconv.conv2, &B->mbconv.conv3};
				for (int k = 0; k < 3; k++)
					rt_put_conv(cv[k], mb->c[k].w, mb->c[k].b, mb->c[k].bn_w,
						    mb->c[k].bn_b, mb->c[k].bn_mean,
						    mb->c[k].bn_var);
				continue;
			}
			const struct rt_block *bw = &lw->blocks[b];
			struct sam3_tvit_attention *at = &B->attn;
			rt_put(at->norm_w, bw->attn_norm_w);
			rt_put(at->norm_b, bw->attn_norm_b);
			rt_put(at->qkv_w, bw->qkv_w);
			rt_put(at->qkv_b, bw->qkv_b);
			rt_put(at->proj_w, bw->proj_w);
			rt_put(at->proj_b, bw->proj_b);
			if (bw->attn_bias) {  /* expand with the reference's own helper */
				int dims[2] = {L->n_heads, bw->attn_bias_offsets};
				struct sam3_tensor *cmp = gh_tensor_wrap(
					&model, SAM3_DTYPE_F32, 2, dims, (void *)bw->attn_bias);
				struct sam3_tensor *e = cmp ? expand_attention_bias(
					cmp, &model, L->n_heads, L->window_size) : NULL;
				if (!e)
					goto done;
				memcpy(at->attn_bias->data, e->data, e->nbytes);
			}
			rt_put_conv(&B->local_conv, bw->lc_w, bw->lc_b, bw->lc_bn_w,
				    bw->lc_bn_b, bw->lc_bn_mean, bw->lc_bn_var);
			rt_put(B->mlp_norm_w, bw->mlp_norm_w);
			rt_put(B->mlp_norm_b, bw->mlp_norm_b);
			rt_put(B->mlp_fc1_w, bw->fc1_w);
			rt_put(B->mlp_fc1_b, bw->fc1_b);
			rt_put(B->mlp_fc2_w, bw->fc2_w);
			rt_put(B->mlp_fc2_b, bw->fc2_b);
		}
		if (L->has_downsample) {
			const struct rt_conv *q[3] = {&lw->pm_conv1, &lw->pm_conv2, &lw->pm_conv3};
			struct sam3_tvit_conv_weights *cv[3] = {
				&L->downsample.conv1, &L->downsample.conv2, &L->downsample.conv3};
			for (int k = 0; k < 3; k++)
				rt_put_conv(cv[k], q[k]->w, q[k]->b, q[k]->bn_w, q[k]->bn_b,
					    q[k]->bn_mean, q[k]->bn_var);
		}
	}
	p = &w->proj_conv1;
	rt_put(tv.proj_conv1.conv_w, p->w);
	p = &w->proj_bn;
	rt_put(tv.proj_bn.bn_w, p->bn_w);
	rt_put(tv.proj_bn.bn_b, p->bn_b);
	rt_put(tv.proj_bn.bn_mean, p->bn_mean);
	rt_put(tv.proj_bn.bn_var, p->bn_var);
	p = &w->proj_conv2;
	rt_put(tv.proj_conv2.conv_w, p->w);
	rt_put(tv.proj_conv2.conv_b, p->b);
	{
		int idims[3] = {3, c->img_size, c->img_size};
		struct sam3_tensor *img = gh_tensor_wrap(&scratch, SAM3_DTYPE_F32, 3,
							 idims, (void *)image);
		/* the build resets `scratch` between stages; keep the image in
		 * the persist arena */
		struct sam3_tensor *ip = gh_alloc_tensor(&persist, SAM3_DTYPE_F32, 3, idims);
		if (!img || !ip)
			goto done;
		memcpy(ip->data, image, ip->nbytes);
		struct sam3_tensor *r = sam3_tinyvit_build(&tv, be, ip, &scratch, &persist, NULL);
		if (!r)
			goto done;
		memcpy(out, r->data, r->nbytes);
	}
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
	sam3_arena_free(&model);
	sam3_arena_free(&scratch);
	sam3_arena_free(&persist);
	return rc;
}
