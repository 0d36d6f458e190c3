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
