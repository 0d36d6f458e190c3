/*
 * oracle/oracle.c - CPU restatement of sam3.c's image-encoder hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * backend: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg load it.  The product library (libsam3cu.so) never links or calls it.
 *
 * Every function restates one reference routine in plain C with FP32
 * arithmetic, citing the reference file:line it follows (paths are relative
 * to the sam3.c project root).  The restatement is pinned against the
 * reference itself (oracle/_ref/libsam3_ref.so, built from the reference
 * sources by oracle/Makefile) and against the known-answer values of the
 * reference's own tests (tests/test_oracle_pin.py).
 *
 * Deliberate differences from the reference CPU backend, each a fix the
 * north star asks for:
 *   - F16 GEMM accumulates in FP32 (the reference's x86 kernel re-rounds the
 *     accumulator to fp16 after every k, cpu_matmul_f16.c:87-93).
 *   - Q8_0 linears compute x . dequant(W)^T (the reference's gh_linear path
 *     transposes a Q8 tensor with element size 0, tensor.c:40, and so reads
 *     unrelated bytes).
 *
 * Threading: OpenMP over rows; results do not depend on the thread count
 * (each output element is produced by exactly one thread in a fixed order).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define Q8_BLOCK 32

/* Q8_0 block as stored by the reference: {float scale; int8 data[32]},
 * 36 bytes (src/core/quant.h:30-33). */
struct orc_q8_block {
	float  scale;
	int8_t data[Q8_BLOCK];
};

int orc_num_threads(int n)
{
#ifdef _OPENMP
	if (n > 0)
		omp_set_num_threads(n);
	return omp_get_max_threads();
#else
	(void)n;
	return 1;
#endif
}

/* ---- number formats (src/core/half.h:51-210) -------------------------- */

/* f32 -> bf16 bits, round to nearest even; NaN kept quiet (half.h:181-210). */
uint16_t orc_f32_to_bf16(float f)
{
	uint32_t u;
	memcpy(&u, &f, 4);
	if ((u & 0x7fffffffu) > 0x7f800000u)
		return (uint16_t)((u >> 16) | 0x40);
	u += 0x7fffu + ((u >> 16) & 1u);
	return (uint16_t)(u >> 16);
}

float orc_bf16_to_f32(uint16_t b)
{
	uint32_t u = (uint32_t)b << 16;
	float f;
	memcpy(&f, &u, 4);
	return f;
}

/* f32 -> IEEE fp16 bits, round to nearest even, with subnormals
 * (half.h:98-160).  Written from the IEEE-754 binary16 definition. */
uint16_t orc_f32_to_fp16(float f)
{
	uint32_t u;
	memcpy(&u, &f, 4);
	uint32_t sign = (u >> 16) & 0x8000u;
	uint32_t absu = u & 0x7fffffffu;
	if (absu > 0x7f800000u)
		return (uint16_t)(sign | 0x7e00u);
	if (absu >= 0x477ff000u) /* rounds to >= 65520 -> inf */
		return (uint16_t)(sign | 0x7c00u);
	if (absu < 0x38800000u) { /* below 2^-14: subnormal or zero */
		float af;
		memcpy(&af, &absu, 4);
		/* scale so that one fp16 subnormal ulp (2^-24) becomes 1.0 */
		float s = af * 16777216.0f;
		uint32_t q = (uint32_t)lrintf(s); /* RNE under default mode */
		return (uint16_t)(sign | q);
	}
	uint32_t mant = absu & 0x7fffffu;
	int32_t exp = (int32_t)(absu >> 23) - 127 + 15;
	uint32_t h = ((uint32_t)exp << 10) | (mant >> 13);
	uint32_t rem = mant & 0x1fffu;
	if (rem > 0x1000u || (rem == 0x1000u && (h & 1u)))
		h += 1;
	return (uint16_t)(sign | h);
}

float orc_fp16_to_f32(uint16_t h)
{
	uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
	uint32_t exp = (h >> 10) & 0x1fu;
	uint32_t mant = h & 0x3ffu;
	float f;
	if (exp == 0) {
		f = (float)mant * (1.0f / 16777216.0f);
		uint32_t u;
		memcpy(&u, &f, 4);
		u |= sign;
		memcpy(&f, &u, 4);
		return f;
	}
	uint32_t u;
	if (exp == 31)
		u = sign | 0x7f800000u | (mant << 13);
	else
		u = sign | ((exp - 15 + 127) << 23) | (mant << 13);
	memcpy(&f, &u, 4);
	return f;
}

void orc_round_bf16(const float *src, float *dst, int64_t n)
{
	for (int64_t i = 0; i < n; i++)
		dst[i] = orc_bf16_to_f32(orc_f32_to_bf16(src[i]));
}

void orc_round_fp16(const float *src, float *dst, int64_t n)
{
	for (int64_t i = 0; i < n; i++)
		dst[i] = orc_fp16_to_f32(orc_f32_to_fp16(src[i]));
}

/* ---- Q8_0 (src/core/quant.c:67-151) ----------------------------------- */

/* Blocks of 32 over the flattened tensor; scale = absmax/127; q =
 * roundf(x * (1/scale)) clamped to +-127; zero tail; scale 0 -> zero block
 * (quant.c:67-131). */
void orc_q8_quantize(const float *src, struct orc_q8_block *dst, int64_t n)
{
	int64_t nb = (n + Q8_BLOCK - 1) / Q8_BLOCK;
	for (int64_t b = 0; b < nb; b++) {
		int64_t off = b * Q8_BLOCK;
		int cnt = (int)((n - off) < Q8_BLOCK ? (n - off) : Q8_BLOCK);
		float amax = 0.0f;
		for (int i = 0; i < cnt; i++) {
			float a = fabsf(src[off + i]);
			if (a > amax)
				amax = a;
		}
		float scale = amax / 127.0f;
		dst[b].scale = scale;
		memset(dst[b].data, 0, Q8_BLOCK);
		if (scale == 0.0f)
			continue;
		float inv = 1.0f / scale;
		for (int i = 0; i < cnt; i++) {
			int q = (int)roundf(src[off + i] * inv);
			if (q > 127) q = 127;
			if (q < -127) q = -127;
			dst[b].data[i] = (int8_t)q;
		}
	}
}

/* value = data[i] * scale (quant.c:134-151). */
void orc_q8_dequantize(const struct orc_q8_block *src, float *dst, int64_t n)
{
	for (int64_t i = 0; i < n; i++) {
		const struct orc_q8_block *blk = &src[i / Q8_BLOCK];
		dst[i] = (float)blk->data[i % Q8_BLOCK] * blk->scale;
	}
}

/* ---- GELU (src/backend/cpu/kernels/cpu_gelu.c:23-36) ------------------ */

static inline float gelu_tanh(float x)
{
	float inner = 0.7978845608f * (x + 0.044715f * x * x * x);
	return 0.5f * x * (1.0f + tanhf(inner));
}

void orc_gelu(const float *x, float *y, int64_t n)
{
	for (int64_t i = 0; i < n; i++)
		y[i] = gelu_tanh(x[i]);
}

/* ---- Linear: gh_linear = TRANSPOSE(W) -> MATMUL -> ADD(bias) ----------
 * (src/model/graph_helpers.c:297-322; MATMUL cpu_matmul.c:196-257,
 *  bias ADD cpu_elementwise.c broadcast over the last dim).
 *
 * y[M,N] = x[M,K] . W[N,K]^T (+ b[N]) (then GELU if act==1) (+ res[M,N]).
 * FP32 accumulation in k order, as the reference kernels accumulate.
 * act: 0 none, 1 tanh-GELU (gh_mlp's activation node, graph_helpers.c).
 */
void orc_linear(const float *x, const float *w, const float *b,
		const float *res, float *y, int M, int K, int N, int act)
{
#pragma omp parallel for schedule(static)
	for (int i = 0; i < M; i++) {
		const float *xr = x + (int64_t)i * K;
		for (int j = 0; j < N; j++) {
			const float *wr = w + (int64_t)j * K;
			float acc = 0.0f;
			for (int k = 0; k < K; k++)
				acc += xr[k] * wr[k];
			if (b)
				acc += b[j];
			if (act == 1)
				acc = gelu_tanh(acc);
			if (res)
				acc += res[(int64_t)i * N + j];
			y[(int64_t)i * N + j] = acc;
		}
	}
}

/* Q8_0 weight [N,K] quantised along the flattened tensor, i.e. 32
 * consecutive K of one output row per block when K % 32 == 0 (the
 * converter's rule, tools/cli_convert.c).  y = x . dequant(W)^T (+b). */
void orc_linear_q8(const float *x, const struct orc_q8_block *wq,
		   const float *b, const float *res, float *y,
		   int M, int K, int N, int act)
{
	float *w = (float *)malloc(sizeof(float) * (size_t)N * K);
	orc_q8_dequantize(wq, w, (int64_t)N * K);
	orc_linear(x, w, b, res, y, M, K, N, act);
	free(w);
}

/* ---- LayerNorm (src/backend/cpu/kernels/cpu_layernorm.c:31-64) --------
 * mean, then sum of squared deviations, inv_std = 1/sqrtf(var/cols+1e-5),
 * then (x-mean)*inv_std*gamma+beta; gamma/beta optional. */
void orc_layernorm(const float *x, const float *g, const float *b, float *y,
		   int rows, int cols)
{
#pragma omp parallel for schedule(static)
	for (int r = 0; r < rows; r++) {
		const float *in = x + (int64_t)r * cols;
		float *out = y + (int64_t)r * cols;
		float sum = 0.0f;
		for (int j = 0; j < cols; j++)
			sum += in[j];
		float mean = sum / (float)cols;
		float vs = 0.0f;
		for (int j = 0; j < cols; j++) {
			float d = in[j] - mean;
			vs += d * d;
		}
		float inv_std = 1.0f / sqrtf(vs / (float)cols + 1e-5f);
		for (int j = 0; j < cols; j++) {
			float v = (in[j] - mean) * inv_std;
			if (g)
				v *= g[j];
			if (b)
				v += b[j];
			out[j] = v;
		}
	}
}

/* ---- RoPE ---------------------------------------------------------------
 * Table (src/model/image_encoder.c:55-115): 16 frequencies
 * 1/theta^(4i/hd); entry i<hd/4 uses the column (x) position * scale,
 * entry hd/4+i the row (y) position * scale; table [n_pos, hd/2]. */
void orc_rope_table(int n_pos, int grid_w, int head_dim, float scale,
		    float theta, float *cos_out, float *sin_out)
{
	int half = head_dim / 2, quarter = head_dim / 4;
	float freqs[64];
	for (int i = 0; i < quarter; i++)
		freqs[i] = 1.0f / powf(theta, (float)(i * 4) / (float)head_dim);
	int grid_h = n_pos / grid_w;
	for (int py = 0; py < grid_h; py++) {
		for (int px = 0; px < grid_w; px++) {
			int pos = py * grid_w + px;
			float sy = (float)py * scale, sx = (float)px * scale;
			for (int i = 0; i < quarter; i++) {
				cos_out[pos * half + i] = cosf(sx * freqs[i]);
				sin_out[pos * half + i] = sinf(sx * freqs[i]);
				cos_out[pos * half + quarter + i] = cosf(sy * freqs[i]);
				sin_out[pos * half + quarter + i] = sinf(sy * freqs[i]);
			}
		}
	}
}

/* Interleaved-pair rotation on [batch, seq, heads, hd] with a [seq, hd/2]
 * table (src/backend/cpu/kernels/cpu_rope.c:35-110).  x and y may alias. */
void orc_rope(const float *x, const float *cs, const float *sn, float *y,
	      int batch, int seq, int heads, int hd)
{
	int half = hd / 2;
#pragma omp parallel for schedule(static)
	for (int bs = 0; bs < batch * seq; bs++) {
		int s = bs % seq;
		for (int h = 0; h < heads; h++) {
			int64_t off = ((int64_t)bs * heads + h) * hd;
			for (int d = 0; d < half; d++) {
				float x0 = x[off + 2 * d], x1 = x[off + 2 * d + 1];
				float c = cs[s * half + d], si = sn[s * half + d];
				y[off + 2 * d] = x0 * c - x1 * si;
				y[off + 2 * d + 1] = x0 * si + x1 * c;
			}
		}
	}
}

/* ---- SDPA (src/backend/cpu/kernels/cpu_sdpa.c:49-159) -----------------
 * Per query row, online softmax over keys in order; scale 1/sqrt(hd);
 * q/k/v/o contiguous [BH, S, hd].  No mask on the encoder path. */
void orc_sdpa(const float *q, const float *k, const float *v, float *o,
	      int BH, int S, int hd)
{
	float scale = 1.0f / sqrtf((float)hd);
#pragma omp parallel for schedule(dynamic, 16)
	for (int64_t idx = 0; idx < (int64_t)BH * S; idx++) {
		int64_t bh = idx / S;
		const float *qr = q + idx * hd;
		const float *K = k + bh * (int64_t)S * hd;
		const float *V = v + bh * (int64_t)S * hd;
		float *out = o + idx * hd;
		float mx = -FLT_MAX, sum = 0.0f;
		for (int d = 0; d < hd; d++)
			out[d] = 0.0f;
		for (int j = 0; j < S; j++) {
			float sc = 0.0f;
			for (int d = 0; d < hd; d++)
				sc += qr[d] * K[(int64_t)j * hd + d];
			sc *= scale;
			if (sc > mx) {
				float corr = expf(mx - sc);
				sum *= corr;
				for (int d = 0; d < hd; d++)
					out[d] *= corr;
				mx = sc;
			}
			float w = expf(sc - mx);
			for (int d = 0; d < hd; d++)
				out[d] += w * V[(int64_t)j * hd + d];
			sum += w;
		}
		if (sum > 0.0f) {
			float inv = 1.0f / sum;
			for (int d = 0; d < hd; d++)
				out[d] *= inv;
		}
	}
}

/* ---- ViT encoder (src/model/image_encoder.c:513-963) -------------------- */

/* Configuration of sam3_vit (image_encoder.h:34-46); global blocks are the
 * fixed indices {7,15,23,31} (image_encoder.c:35). */
struct orc_vit_cfg {
	int img_size, patch_size, embed_dim, depth, n_heads, window_size,
	    mlp_dim;
};

/* Weights of one block, F32 [out,in] row-major; QKV fused [3e, e]
 * (image_encoder.c:223-259, 346-452). */
struct orc_vit_block {
	const float *ln1_w, *ln1_b, *qkv_w, *qkv_b, *proj_w, *proj_b;
	const float *ln2_w, *ln2_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
};

struct orc_vit_weights {
	const float *patch_w;  /* [e, ps, ps, 3] OHWI (image_encoder.c:266-278) */
	const float *patch_b;  /* [e] */
	const float *pos_raw;  /* [1, 24*24+1, e], CLS first (:294-306) */
	const float *ln_pre_w, *ln_pre_b;
	struct orc_vit_block blocks[32];
};

static int is_global_block(int i)
{
	return i == 7 || i == 15 || i == 23 || i == 31;
}

/* Window partition as a row permutation (graph_helpers.c:444-475):
 * token (py,px) -> window (py/ws)*nw + px/ws, slot (py%ws)*ws + px%ws. */
static void window_partition(const float *x, float *y, int gs, int ws, int e)
{
	int nw = gs / ws;
	for (int py = 0; py < gs; py++)
		for (int px = 0; px < gs; px++) {
			int win = (py / ws) * nw + px / ws;
			int slot = (py % ws) * ws + px % ws;
			memcpy(y + ((int64_t)win * ws * ws + slot) * e,
			       x + ((int64_t)py * gs + px) * e,
			       sizeof(float) * e);
		}
}

static void window_unpartition(const float *y, float *x, int gs, int ws,
			       int e)
{
	int nw = gs / ws;
	for (int py = 0; py < gs; py++)
		for (int px = 0; px < gs; px++) {
			int win = (py / ws) * nw + px / ws;
			int slot = (py % ws) * ws + px % ws;
			memcpy(x + ((int64_t)py * gs + px) * e,
			       y + ((int64_t)win * ws * ws + slot) * e,
			       sizeof(float) * e);
		}
}

/* gh_multihead_attention_rope (graph_helpers.c:721-882) on x[B*S, e]:
 * QKV linear, split Q|K|V columns, RoPE on Q and K with the [S, hd/2]
 * table, per-head SDPA, merge heads, out projection. */
static void mha_rope(const float *x, float *out, int B, int S, int e,
		     int heads, const struct orc_vit_block *w,
		     const float *cs, const float *sn)
{
	int hd = e / heads;
	int64_t bs = (int64_t)B * S;
	float *qkv = (float *)malloc(sizeof(float) * bs * 3 * e);
	float *q = (float *)malloc(sizeof(float) * bs * e);
	float *k = (float *)malloc(sizeof(float) * bs * e);
	float *v = (float *)malloc(sizeof(float) * bs * e);
	float *o = (float *)malloc(sizeof(float) * bs * e);
	orc_linear(x, w->qkv_w, w->qkv_b, NULL, qkv, (int)bs, e, 3 * e, 0);
	/* Slice (SLICE axis 1) then permute [B,S,H,hd] -> [B,H,S,hd]. */
	float *tq = (float *)malloc(sizeof(float) * bs * e);
	float *tk = (float *)malloc(sizeof(float) * bs * e);
	for (int64_t r = 0; r < bs; r++) {
		memcpy(tq + r * e, qkv + r * 3 * e, sizeof(float) * e);
		memcpy(tk + r * e, qkv + r * 3 * e + e, sizeof(float) * e);
	}
	orc_rope(tq, cs, sn, tq, B, S, heads, hd);
	orc_rope(tk, cs, sn, tk, B, S, heads, hd);
	for (int b = 0; b < B; b++)
		for (int s = 0; s < S; s++)
			for (int h = 0; h < heads; h++) {
				int64_t src = ((int64_t)b * S + s) * e + h * hd;
				int64_t dst = (((int64_t)b * heads + h) * S + s) * hd;
				memcpy(q + dst, tq + src, sizeof(float) * hd);
				memcpy(k + dst, tk + src, sizeof(float) * hd);
				memcpy(v + dst, qkv + ((int64_t)b * S + s) * 3 * e
					   + 2 * e + h * hd, sizeof(float) * hd);
			}
	orc_sdpa(q, k, v, o, B * heads, S, hd);
	/* permute back [B,H,S,hd] -> [B,S,H,hd] -> [B*S, e] */
	for (int b = 0; b < B; b++)
		for (int s = 0; s < S; s++)
			for (int h = 0; h < heads; h++)
				memcpy(tq + ((int64_t)b * S + s) * e + h * hd,
				       o + (((int64_t)b * heads + h) * S + s) * hd,
				       sizeof(float) * hd);
	orc_linear(tq, w->proj_w, w->proj_b, NULL, out, (int)bs, e, e, 0);
	free(qkv); free(q); free(k); free(v); free(o); free(tq); free(tk);
}

/* One pre-norm block in place on x[np, e] (image_encoder.c:755-900). */
void orc_vit_block_forward(const struct orc_vit_cfg *c,
			   const struct orc_vit_block *w, int is_global,
			   float *x, const float *glo_cos, const float *glo_sin,
			   const float *win_cos, const float *win_sin)
{
	int gs = c->img_size / c->patch_size, e = c->embed_dim;
	int np = gs * gs, ws = c->window_size;
	float *xn = (float *)malloc(sizeof(float) * (size_t)np * e);
	float *att = (float *)malloc(sizeof(float) * (size_t)np * e);
	float *h = (float *)malloc(sizeof(float) * (size_t)np * c->mlp_dim);
	orc_layernorm(x, w->ln1_w, w->ln1_b, xn, np, e);
	if (is_global) {
		mha_rope(xn, att, 1, np, e, c->n_heads, w, glo_cos, glo_sin);
	} else {
		float *xw = (float *)malloc(sizeof(float) * (size_t)np * e);
		float *aw = (float *)malloc(sizeof(float) * (size_t)np * e);
		int nw = gs / ws;
		window_partition(xn, xw, gs, ws, e);
		mha_rope(xw, aw, nw * nw, ws * ws, e, c->n_heads, w, win_cos,
			 win_sin);
		window_unpartition(aw, att, gs, ws, e);
		free(xw); free(aw);
	}
	for (int64_t i = 0; i < (int64_t)np * e; i++)
		x[i] += att[i];
	orc_layernorm(x, w->ln2_w, w->ln2_b, xn, np, e);
	orc_linear(xn, w->fc1_w, w->fc1_b, NULL, h, np, e, c->mlp_dim, 1);
	orc_linear(h, w->fc2_w, w->fc2_b, x, x, np, c->mlp_dim, e, 0);
	free(xn); free(att); free(h);
}

/* Patch embed (conv ps x ps stride ps, NHWC input, OHWI weight) + bias +
 * tiled pos-embed (24x24 pretrain grid tiled, CLS stripped,
 * image_encoder.c:167-218) + ln_pre (image_encoder.c:554-662).
 * image: planar CHW [3, img, img] F32 (already normalised). */
void orc_vit_embed(const struct orc_vit_cfg *c,
		   const struct orc_vit_weights *w, const float *image,
		   float *x)
{
	int ps = c->patch_size, img = c->img_size, gs = img / ps;
	int e = c->embed_dim, np = gs * gs;
#pragma omp parallel for schedule(static)
	for (int p = 0; p < np; p++) {
		int py = p / gs, px = p % gs;
		float *xr = x + (int64_t)p * e;
		for (int o = 0; o < e; o++) {
			float acc = 0.0f;
			const float *wo = w->patch_w + (int64_t)o * ps * ps * 3;
			for (int ky = 0; ky < ps; ky++)
				for (int kx = 0; kx < ps; kx++)
					for (int ch = 0; ch < 3; ch++)
						acc += image[((int64_t)ch * img + py * ps + ky) * img
							     + px * ps + kx]
						       * wo[(ky * ps + kx) * 3 + ch];
			xr[o] = acc + w->patch_b[o];
		}
		int sy = py % 24, sx = px % 24;
		const float *pr = w->pos_raw + (int64_t)(1 + sy * 24 + sx) * e;
		for (int o = 0; o < e; o++)
			xr[o] += pr[o];
	}
	orc_layernorm(x, w->ln_pre_w, w->ln_pre_b, x, np, e);
}

/* Full sam3_vit_build forward: embed, then every block; the output has no
 * final norm (image_encoder.c:950-962).  x: [np, e] F32 out. */
void orc_vit_forward(const struct orc_vit_cfg *c,
		     const struct orc_vit_weights *w, const float *image,
		     float *x)
{
	int gs = c->img_size / c->patch_size, ws = c->window_size;
	int hd = c->embed_dim / c->n_heads;
	int np = gs * gs;
	float *gc = (float *)malloc(sizeof(float) * np * hd / 2);
	float *gsn = (float *)malloc(sizeof(float) * np * hd / 2);
	float *wc = (float *)malloc(sizeof(float) * ws * ws * hd / 2);
	float *wsn = (float *)malloc(sizeof(float) * ws * ws * hd / 2);
	orc_rope_table(np, gs, hd, (float)ws / (float)gs, 10000.0f, gc, gsn);
	orc_rope_table(ws * ws, ws, hd, 1.0f, 10000.0f, wc, wsn);
	orc_vit_embed(c, w, image, x);
	for (int i = 0; i < c->depth; i++)
		orc_vit_block_forward(c, &w->blocks[i], is_global_block(i), x,
				      gc, gsn, wc, wsn);
	free(gc); free(gsn); free(wc); free(wsn);
}

/* ---- TinyViT (src/model/image_encoder_tinyvit.c) ------------------------ */

/* expand_attention_bias (:265-335): compact [heads, n_off] -> dense
 * [heads, N, N], N = ws*ws; offsets (|dy|, |dx|) numbered in the order the
 * position pairs (p1, p2), both row-major, first meet them.  Returns the
 * number of distinct offsets found (the caller checks it against n_off). */
int orc_tvit_expand_bias(const float *compact, int heads, int n_off, int ws,
			 float *out)
{
	int N = ws * ws, count = 0;
	int *idx = malloc(sizeof(int) * (size_t)N);
	for (int i = 0; i < N; i++)
		idx[i] = -1;
	for (int p1 = 0; p1 < N; p1++)
		for (int p2 = 0; p2 < N; p2++) {
			int key = abs(p1 / ws - p2 / ws) * ws +
				  abs(p1 % ws - p2 % ws);
			if (idx[key] < 0)
				idx[key] = count++;
		}
	if (count == n_off)
		for (int h = 0; h < heads; h++)
			for (int p1 = 0; p1 < N; p1++)
				for (int p2 = 0; p2 < N; p2++) {
					int key = abs(p1 / ws - p2 / ws) * ws +
						  abs(p1 % ws - p2 % ws);
					out[((int64_t)h * N + p1) * N + p2] =
						compact[(int64_t)h * n_off +
							idx[key]];
				}
	free(idx);
	return count;
}

/* Row softmax (cpu_softmax.c:29-47): max, expf(x - max), sum, * 1/sum. */
static void softmax_row(float *x, int n)
{
	float mx = -FLT_MAX, sum = 0.0f;
	for (int j = 0; j < n; j++)
		if (x[j] > mx)
			mx = x[j];
	for (int j = 0; j < n; j++) {
		x[j] = expf(x[j] - mx);
		sum += x[j];
	}
	float inv = 1.0f / sum;
	for (int j = 0; j < n; j++)
		x[j] *= inv;
}

/* tvit_window_attention (:790-866) after the qkv linear.  qkv
 * [nw*N, 3*heads*hd] in the per-head interleaved layout (reshape to
 * [nw, N, heads, 3*hd], slices at 0, hd, 2*hd on the last dim :796-809);
 * Q scaled by 1/sqrt(hd) (:823-833), scores Q.K^T + bias[h] (:836-846),
 * softmax (:849), .V (:854), permuted back to out [nw*N, heads*hd]. */
void orc_tvit_window_attention(const float *qkv, int nw, int N, int heads,
			       int hd, const float *bias, float *out)
{
	const int C = heads * hd, ld = 3 * C;
	const float scale = 1.0f / sqrtf((float)hd);
#pragma omp parallel for schedule(dynamic, 1)
	for (int64_t wh = 0; wh < (int64_t)nw * heads; wh++) {
		const int w = (int)(wh / heads), h = (int)(wh % heads);
		const float *base = qkv + (int64_t)w * N * ld + h * 3 * hd;
		float *q = malloc(sizeof(float) * (size_t)N * hd);
		float *s = malloc(sizeof(float) * (size_t)N);
		for (int i = 0; i < N; i++)
			for (int d = 0; d < hd; d++)
				q[i * hd + d] = base[(int64_t)i * ld + d] * scale;
		for (int i = 0; i < N; i++) {
			for (int j = 0; j < N; j++) {
				float acc = 0.0f;
				const float *kr = base + (int64_t)j * ld + hd;
				for (int d = 0; d < hd; d++)
					acc += q[i * hd + d] * kr[d];
				s[j] = acc + (bias ? bias[((int64_t)h * N + i) * N + j] : 0.0f);
			}
			softmax_row(s, N);
			float *o = out + ((int64_t)w * N + i) * C + h * hd;
			for (int d = 0; d < hd; d++) {
				float acc = 0.0f;
				for (int j = 0; j < N; j++)
					acc += s[j] * base[(int64_t)j * ld + 2 * hd + d];
				o[d] = acc;
			}
		}
		free(q);
		free(s);
	}
}

/* tvit_conv_bn (:655-674) for the depthwise 3x3 convs: conv2d NHWC with
 * OHWI weight [C,3,3,1], pad 1, groups C, stride 1 or 2 (cpu_conv2d.c:320-420;
 * output (H-1)/s+1), optional conv bias, then eval BatchNorm
 * (cpu_batchnorm.c: (x - mean) * 1/sqrtf(var + 1e-5) * gamma + beta), then
 * tanh-GELU if gelu. */
void orc_dwconv3x3_bn_s(const float *x, int B, int H, int W, int C, int stride,
			const float *w, const float *cb, const float *bn_w,
			const float *bn_b, const float *bn_mean,
			const float *bn_var, int gelu, float *y)
{
	const int OH = (H - 1) / stride + 1, OW = (W - 1) / stride + 1;
#pragma omp parallel for schedule(static)
	for (int64_t p = 0; p < (int64_t)B * OH * OW; p++) {
		int b = (int)(p / ((int64_t)OH * OW)), oy = (int)(p / OW % OH),
		    ox = (int)(p % OW);
		for (int c = 0; c < C; c++) {
			float acc = 0.0f;
			for (int ky = 0; ky < 3; ky++)
				for (int kx = 0; kx < 3; kx++) {
					int iy = oy * stride + ky - 1,
					    ix = ox * stride + kx - 1;
					if (iy < 0 || iy >= H || ix < 0 || ix >= W)
						continue;
					acc += x[(((int64_t)b * H + iy) * W + ix) * C + c] *
					       w[(c * 3 + ky) * 3 + kx];
				}
			if (cb)
				acc += cb[c];
			if (bn_mean) {
				float inv = 1.0f / sqrtf(bn_var[c] + 1e-5f);
				acc = (acc - bn_mean[c]) * inv;
				if (bn_w)
					acc *= bn_w[c];
				if (bn_b)
					acc += bn_b[c];
			}
			y[p * C + c] = gelu ? gelu_tanh(acc) : acc;
		}
	}
}

void orc_dwconv3x3_bn(const float *x, int B, int H, int W, int C,
		      const float *w, const float *cb, const float *bn_w,
		      const float *bn_b, const float *bn_mean,
		      const float *bn_var, int gelu, float *y)
{
	orc_dwconv3x3_bn_s(x, B, H, W, C, 1, w, cb, bn_w, bn_b, bn_mean, bn_var,
			   gelu, y);
}

/* Dense conv2d (cpu_conv2d.c:320-420, groups 1): OHWI weight [OC,k,k,IC],
 * zero padding, NHWC input (or planar CHW when chw), f32 accumulation over
 * (ky, kx, c); then optional bias, eval BatchNorm and tanh-GELU, as
 * tvit_conv_bn / gh_conv2d chain them.  y [B, OH, OW, OC]. */
void orc_conv2d_bn(const float *x, int chw, int B, int H, int W, int IC, int OC,
		   int k, int stride, int pad, const float *w, const float *cb,
		   const float *bn_w, const float *bn_b, const float *bn_mean,
		   const float *bn_var, int gelu, float *y)
{
	const int OH = (H + 2 * pad - k) / stride + 1,
		  OW = (W + 2 * pad - k) / stride + 1;
#pragma omp parallel for schedule(static)
	for (int64_t p = 0; p < (int64_t)B * OH * OW; p++) {
		int b = (int)(p / ((int64_t)OH * OW)), oy = (int)(p / OW % OH),
		    ox = (int)(p % OW);
		for (int o = 0; o < OC; o++) {
			float acc = 0.0f;
			for (int ky = 0; ky < k; ky++)
				for (int kx = 0; kx < k; kx++) {
					int iy = oy * stride - pad + ky,
					    ix = ox * stride - pad + kx;
					if (iy < 0 || iy >= H || ix < 0 || ix >= W)
						continue;
					const float *wr = w + (((int64_t)o * k + ky) * k + kx) * IC;
					for (int c = 0; c < IC; c++) {
						float v = chw ? x[(((int64_t)b * IC + c) * H + iy) * W + ix]
							      : x[(((int64_t)b * H + iy) * W + ix) * IC + c];
						acc += v * wr[c];
					}
				}
			if (cb)
				acc += cb[o];
			if (bn_mean) {
				float inv = 1.0f / sqrtf(bn_var[o] + 1e-5f);
				acc = (acc - bn_mean[o]) * inv;
				if (bn_w)
					acc *= bn_w[o];
				if (bn_b)
					acc += bn_b[o];
			}
			y[p * OC + o] = gelu ? gelu_tanh(acc) : acc;
		}
	}
}

/* Weights of one TinyViTBlock (image_encoder_tinyvit.h: sam3_tvit_block),
 * F32, linears [out, in]; attn_bias is the expanded [heads, N, N]. */
struct orc_tvit_block {
	const float *attn_norm_w, *attn_norm_b, *qkv_w, *qkv_b, *proj_w,
		*proj_b, *attn_bias;
	const float *lc_w, *lc_b, *lc_bn_w, *lc_bn_b, *lc_bn_mean, *lc_bn_var;
	const float *mlp_norm_w, *mlp_norm_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
};

/* tvit_block_forward (:896-1052) on x [H, W, C] (one image, NHWC), in
 * place: zero-pad to multiples of ws (:916-956), window partition, window
 * attention with its pre-LN (:767-771), unpartition, unpad, residual add;
 * 3x3 depthwise conv + BN; LN -> fc1 -> GELU -> fc2, residual add. */
void orc_tvit_block_forward(const struct orc_tvit_block *bw, float *x, int H,
			    int W, int C, int heads, int ws, int mlp)
{
	const int Hp = (H + ws - 1) / ws * ws, Wp = (W + ws - 1) / ws * ws;
	const int nwy = Hp / ws, nwx = Wp / ws, nw = nwy * nwx, N = ws * ws;
	const int64_t T = (int64_t)nw * N;
	float *win = calloc((size_t)T * C, sizeof(float));
	float *ln = malloc(sizeof(float) * (size_t)T * C);
	float *qkv = malloc(sizeof(float) * (size_t)T * 3 * C);
	float *att = malloc(sizeof(float) * (size_t)T * C);
	float *prj = malloc(sizeof(float) * (size_t)T * C);
	/* pad + partition: window (wy, wx), token (cy, cx) */
	for (int wy = 0; wy < nwy; wy++)
		for (int wx = 0; wx < nwx; wx++)
			for (int t = 0; t < N; t++) {
				int py = wy * ws + t / ws, px = wx * ws + t % ws;
				if (py < H && px < W)
					memcpy(win + ((int64_t)(wy * nwx + wx) * N + t) * C,
					       x + ((int64_t)py * W + px) * C,
					       sizeof(float) * C);
			}
	orc_layernorm(win, bw->attn_norm_w, bw->attn_norm_b, ln, T, C);
	orc_linear(ln, bw->qkv_w, bw->qkv_b, NULL, qkv, T, C, 3 * C, 0);
	orc_tvit_window_attention(qkv, nw, N, heads, C / heads, bw->attn_bias,
				  att);
	orc_linear(att, bw->proj_w, bw->proj_b, NULL, prj, T, C, C, 0);
	/* unpartition + unpad + residual */
	for (int wy = 0; wy < nwy; wy++)
		for (int wx = 0; wx < nwx; wx++)
			for (int t = 0; t < N; t++) {
				int py = wy * ws + t / ws, px = wx * ws + t % ws;
				if (py >= H || px >= W)
					continue;
				const float *s = prj + ((int64_t)(wy * nwx + wx) * N + t) * C;
				float *d = x + ((int64_t)py * W + px) * C;
				for (int c = 0; c < C; c++)
					d[c] = s[c] + d[c];
			}
	free(win);
	free(qkv);
	free(att);
	free(prj);
	/* local conv: 3x3 depthwise + BN (:1015) */
	const int64_t HW = (int64_t)H * W;
	float *lc = malloc(sizeof(float) * (size_t)HW * C);
	orc_dwconv3x3_bn(x, 1, H, W, C, bw->lc_w, bw->lc_b, bw->lc_bn_w,
			 bw->lc_bn_b, bw->lc_bn_mean, bw->lc_bn_var, 0, lc);
	/* MLP with residual (:1027-1046) */
	float *h1 = malloc(sizeof(float) * (size_t)HW * mlp);
	free(ln);
	ln = malloc(sizeof(float) * (size_t)HW * C);
	orc_layernorm(lc, bw->mlp_norm_w, bw->mlp_norm_b, ln, HW, C);
	orc_linear(ln, bw->fc1_w, bw->fc1_b, NULL, h1, HW, C, mlp, 1);
	orc_linear(h1, bw->fc2_w, bw->fc2_b, lc, x, HW, mlp, C, 0);
	free(lc);
	free(h1);
	free(ln);
}

/* 1x1 conv (NHWC, OHWI [O,1,1,I] == linear [O, I]) + optional conv bias +
 * eval BatchNorm + optional GELU: tvit_conv_bn (:655-674) for the MBConv
 * pointwise convs.  x [P, I] -> y [P, O]. */
static void conv1x1_bn(const float *x, int64_t P, int I, int O, const float *w,
		       const float *cb, const float *g, const float *be,
		       const float *mean, const float *var, int gelu, float *y)
{
	orc_linear(x, w, cb, NULL, y, (int)P, I, O, 0);
#pragma omp parallel for schedule(static)
	for (int64_t p = 0; p < P; p++)
		for (int o = 0; o < O; o++) {
			float v = y[p * O + o];
			if (mean) {
				v = (v - mean[o]) * (1.0f / sqrtf(var[o] + 1e-5f));
				if (g)
					v *= g[o];
				if (be)
					v += be[o];
			}
			y[p * O + o] = gelu ? gelu_tanh(v) : v;
		}
}

struct orc_tvit_mbconv {
	const float *conv1_w, *conv1_b, *bn1_w, *bn1_b, *bn1_mean, *bn1_var;
	const float *conv2_w, *conv2_b, *bn2_w, *bn2_b, *bn2_mean, *bn2_var;
	const float *conv3_w, *conv3_b, *bn3_w, *bn3_b, *bn3_mean, *bn3_var;
};

/* tvit_mbconv_forward (:682-720) on x [B, H, W, C] NHWC, in place: conv1
 * 1x1 + BN, GELU; depthwise 3x3 + BN, GELU; conv3 1x1 + BN; + shortcut;
 * GELU. */
void orc_tvit_mbconv_forward(const struct orc_tvit_mbconv *m, float *x, int B,
			     int H, int W, int C, int mid)
{
	const int64_t P = (int64_t)B * H * W;
	float *h = malloc(sizeof(float) * (size_t)P * mid);
	float *h2 = malloc(sizeof(float) * (size_t)P * mid);
	float *o = malloc(sizeof(float) * (size_t)P * C);
	conv1x1_bn(x, P, C, mid, m->conv1_w, m->conv1_b, m->bn1_w, m->bn1_b,
		   m->bn1_mean, m->bn1_var, 1, h);
	orc_dwconv3x3_bn(h, B, H, W, mid, m->conv2_w, m->conv2_b, m->bn2_w,
			 m->bn2_b, m->bn2_mean, m->bn2_var, 1, h2);
	conv1x1_bn(h2, P, mid, C, m->conv3_w, m->conv3_b, m->bn3_w, m->bn3_b,
		   m->bn3_mean, m->bn3_var, 0, o);
	for (int64_t i = 0; i < P * C; i++)
		x[i] = gelu_tanh(o[i] + x[i]);
	free(h);
	free(h2);
	free(o);
}


/* ---- whole TinyViT backbone (sam3_tinyvit_build, :1058-1290) ---------- */

/* These structs have the layouts of the CUDA library's
 * sam3cu_tvit_conv_weights / _block_weights / _mbconv_weights /
 * sam3cu_tinyvit_* (include/sam3cu.h), so one weight tree feeds both. */
struct orc_conv { const float *w, *b, *bn_w, *bn_b, *bn_mean, *bn_var; };
struct orc_tvit_block_c {
	const float *attn_norm_w, *attn_norm_b, *qkv_w, *qkv_b, *proj_w,
		*proj_b, *attn_bias;
	int attn_bias_offsets;
	const float *lc_w, *lc_b, *lc_bn_w, *lc_bn_b, *lc_bn_mean, *lc_bn_var;
	const float *mlp_norm_w, *mlp_norm_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
};
struct orc_tinyvit_cfg {
	int img_size, n_layers, embed_dims[4], depths[4], num_heads[4],
	    window_sizes[4], embed_dim, mlp_ratio;
};
struct orc_tinyvit_layer {
	const struct orc_tvit_mbconv *conv_blocks;
	const struct orc_tvit_block_c *blocks;
	struct orc_conv pm_conv1, pm_conv2, pm_conv3;
};
struct orc_tinyvit_weights {
	struct orc_conv patch_embed_0, patch_embed_1;
	struct orc_tinyvit_layer layers[4];
	struct orc_conv proj_conv1, proj_bn, proj_conv2;
};

/* One image [3, S, S] -> out [grid*grid, embed_dim].  Returns the grid. */
int orc_tinyvit_forward(const struct orc_tinyvit_cfg *c,
			const struct orc_tinyvit_weights *w, const float *img,
			float *out)
{
	const int S = c->img_size, H1 = (S - 1) / 2 + 1, H2 = (H1 - 1) / 2 + 1;
	const int C0 = c->embed_dims[0];
	float *a = malloc(sizeof(float) * (size_t)H1 * H1 * (C0 / 2));
	float *x = malloc(sizeof(float) * (size_t)H2 * H2 * C0);
	const struct orc_conv *p0 = &w->patch_embed_0, *p1 = &w->patch_embed_1;
	orc_conv2d_bn(img, 1, 1, S, S, 3, C0 / 2, 3, 2, 1, p0->w, p0->b, p0->bn_w,
		      p0->bn_b, p0->bn_mean, p0->bn_var, 1, a);
	orc_conv2d_bn(a, 0, 1, H1, H1, C0 / 2, C0, 3, 2, 1, p1->w, p1->b,
		      p1->bn_w, p1->bn_b, p1->bn_mean, p1->bn_var, 0, x);
	free(a);
	int H = H2, C = C0;
	for (int l = 0; l < c->n_layers; l++) {
		for (int b = 0; b < c->depths[l]; b++) {
			if (l == 0) {
				orc_tvit_mbconv_forward(&w->layers[0].conv_blocks[b], x,
							1, H, H, C, C * c->mlp_ratio);
			} else {
				const struct orc_tvit_block_c *bc = &w->layers[l].blocks[b];
				const int ws = c->window_sizes[l], N = ws * ws;
				const int heads = c->num_heads[l];
				float *bias = NULL;
				if (bc->attn_bias) {
					bias = malloc(sizeof(float) * (size_t)heads * N * N);
					orc_tvit_expand_bias(bc->attn_bias, heads,
							     bc->attn_bias_offsets, ws, bias);
				}
				struct orc_tvit_block ob = {
					bc->attn_norm_w, bc->attn_norm_b, bc->qkv_w,
					bc->qkv_b, bc->proj_w, bc->proj_b, bias,
					bc->lc_w, bc->lc_b, bc->lc_bn_w, bc->lc_bn_b,
					bc->lc_bn_mean, bc->lc_bn_var, bc->mlp_norm_w,
					bc->mlp_norm_b, bc->fc1_w, bc->fc1_b, bc->fc2_w,
					bc->fc2_b};
				orc_tvit_block_forward(&ob, x, H, H, C, heads, ws,
						       C * c->mlp_ratio);
				free(bias);
			}
		}
		if (l == c->n_layers - 1)
			break;
		/* PatchMerging (tvit_patch_merging, :726-750) */
		const struct orc_tinyvit_layer *lw = &w->layers[l];
		const int Cn = c->embed_dims[l + 1], Hn = (H - 1) / 2 + 1;
		float *h = malloc(sizeof(float) * (size_t)H * H * Cn);
		float *h2 = malloc(sizeof(float) * (size_t)Hn * Hn * Cn);
		float *xn = malloc(sizeof(float) * (size_t)Hn * Hn * Cn);
		orc_conv2d_bn(x, 0, 1, H, H, C, Cn, 1, 1, 0, lw->pm_conv1.w,
			      lw->pm_conv1.b, lw->pm_conv1.bn_w, lw->pm_conv1.bn_b,
			      lw->pm_conv1.bn_mean, lw->pm_conv1.bn_var, 1, h);
		orc_dwconv3x3_bn_s(h, 1, H, H, Cn, 2, lw->pm_conv2.w,
				   lw->pm_conv2.b, lw->pm_conv2.bn_w,
				   lw->pm_conv2.bn_b, lw->pm_conv2.bn_mean,
				   lw->pm_conv2.bn_var, 1, h2);
		orc_conv2d_bn(h2, 0, 1, Hn, Hn, Cn, Cn, 1, 1, 0, lw->pm_conv3.w,
			      lw->pm_conv3.b, lw->pm_conv3.bn_w, lw->pm_conv3.bn_b,
			      lw->pm_conv3.bn_mean, lw->pm_conv3.bn_var, 0, xn);
		free(x);
		free(h);
		free(h2);
		x = xn;
		H = Hn;
		C = Cn;
	}
	/* head: 1x1 conv (no bias) -> BN -> GELU -> 3x3 conv + bias (:1230-1262) */
	const int E = c->embed_dim;
	float *h = malloc(sizeof(float) * (size_t)H * H * E);
	orc_conv2d_bn(x, 0, 1, H, H, C, E, 1, 1, 0, w->proj_conv1.w, NULL,
		      w->proj_bn.bn_w, w->proj_bn.bn_b, w->proj_bn.bn_mean,
		      w->proj_bn.bn_var, 1, h);
	orc_conv2d_bn(h, 0, 1, H, H, E, E, 3, 1, 1, w->proj_conv2.w,
		      w->proj_conv2.b, NULL, NULL, NULL, NULL, 0, out);
	free(h);
	free(x);
	return H;
}

/* ---- FPN neck (src/model/necks.c) --------------------------------------- */

/* One stage of sam3_neck_build (build_stage, necks.c:327-369), stage plan
 * per scale factor as init_stage_4x / _2x / _1x / _half (:37-148):
 *   >= 3.5: ConvT(dim->dim/2, k2 s2), GELU, ConvT(dim/2->dim/4, k2 s2),
 *           Conv1x1(->d), Conv3x3(d->d, pad 1)
 *   >= 1.5: ConvT(dim->dim/2), Conv1x1(->d), Conv3x3
 *   >= 0.75: Conv1x1(dim->d), Conv3x3
 *   else: MaxPool(2, 2), Conv1x1(dim->d), Conv3x3
 * every conv with bias (a BIAS_ADD node).  x [H, W, dim] NHWC; returns the
 * output size through *oh; out must hold it. */
static void convt_k2s2(const float *x, int H, int W, int C, int OC,
		       const float *w, const float *b, int gelu, float *y)
{
	/* cpu_conv_transpose2d.c with stride 2, pad 0, kernel 2: output
	 * (2h+ky, 2w+kx) = sum_c x[h, w, c] * w[oc, ky, kx, c] */
#pragma omp parallel for schedule(static)
	for (int64_t p = 0; p < (int64_t)H * W; p++) {
		int h = (int)(p / W), ww = (int)(p % W);
		const float *xr = x + p * C;
		for (int ky = 0; ky < 2; ky++)
			for (int kx = 0; kx < 2; kx++) {
				float *yo = y + (((int64_t)(2 * h + ky) * 2 * W) + 2 * ww + kx) * OC;
				for (int o = 0; o < OC; o++) {
					const float *wr = w + (((int64_t)o * 2 + ky) * 2 + kx) * C;
					float acc = 0.0f;
					for (int c = 0; c < C; c++)
						acc += xr[c] * wr[c];
					acc += b ? b[o] : 0.0f;
					yo[o] = gelu ? gelu_tanh(acc) : acc;
				}
			}
	}
}

void orc_neck_forward(int d_model, int dim, int grid, int n_scales,
		      const float *scales, const float *const *w,
		      const float *const *b, const float *feat,
		      float *const *outs)
{
	for (int i = 0; i < n_scales; i++) {
		const float sf = scales[i];
		const float *const *ws = w + i * 4, *const *bs = b + i * 4;
		int H = grid, C = dim;
		float *cur = malloc(sizeof(float) * (size_t)grid * grid * dim);
		memcpy(cur, feat, sizeof(float) * (size_t)grid * grid * dim);
		int j = 0;
		if (sf < 0.75f) {  /* MaxPool(2, 2) (cpu_maxpool2d.c) */
			int Hn = (H - 2) / 2 + 1;
			float *nx = malloc(sizeof(float) * (size_t)Hn * Hn * C);
			for (int y = 0; y < Hn; y++)
				for (int xx = 0; xx < Hn; xx++)
					for (int c = 0; c < C; c++) {
						float m = -FLT_MAX;
						for (int ky = 0; ky < 2; ky++)
							for (int kx = 0; kx < 2; kx++) {
								float v = cur[((int64_t)(2 * y + ky) * H + 2 * xx + kx) * C + c];
								if (v > m)
									m = v;
							}
						nx[((int64_t)y * Hn + xx) * C + c] = m;
					}
			free(cur);
			cur = nx;
			H = Hn;
		}
		int n_t = sf >= 3.5f ? 2 : (sf >= 1.5f ? 1 : 0);
		for (int t = 0; t < n_t; t++, j++) {
			int OC = C / 2;
			float *nx = malloc(sizeof(float) * (size_t)4 * H * H * OC);
			convt_k2s2(cur, H, H, C, OC, ws[j], bs[j], sf >= 3.5f && t == 0, nx);
			free(cur);
			cur = nx;
			H *= 2;
			C = OC;
		}
		float *p1 = malloc(sizeof(float) * (size_t)H * H * d_model);
		orc_conv2d_bn(cur, 0, 1, H, H, C, d_model, 1, 1, 0, ws[j], bs[j], NULL,
			      NULL, NULL, NULL, 0, p1);
		j++;
		orc_conv2d_bn(p1, 0, 1, H, H, d_model, d_model, 3, 1, 1, ws[j], bs[j],
			      NULL, NULL, NULL, NULL, 0, outs[i]);
		free(p1);
		free(cur);
	}
}
