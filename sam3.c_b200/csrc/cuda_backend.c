/*
 * cuda_backend.c - struct sam3_backend_ops for the B200 (C11).
 *
 * The drop-in for sam3.c's backend vtable (src/backend/backend.h:29-56):
 * graph_eval walks the graph in array order, as cpu_graph_eval does
 * (cpu_backend.c:175-202), and lowers each (op, dtype) to the device entry
 * points of include/sam3cu.h.  Three peepholes remove the reference's
 * per-linear glue: TRANSPOSE(W) feeding MATMUL is not materialised (the
 * GEMM reads W [N,K] K-major), an ADD of a [N] bias to a MATMUL output and
 * a following GELU are fused into the GEMM epilogue.
 *
 * Views: RESHAPE, TRANSPOSE/PERMUTE and SLICE produce no data.  Their
 * result is a strided view of the input's device buffer (element strides
 * per dim); ROPE, SDPA and MATMUL's B operand read views directly, every
 * other consumer gets a contiguous copy made on first use.  SDPA writes its
 * output [B,H,S,hd] with head-interleaved strides, so the permute(0,2,1,3)
 * + reshape that gh_multihead_attention_rope puts after it
 * (graph_helpers.c:840-880) are free, and the F32 / 16-bit attention
 * kernels read Q, K and V where the QKV GEMM wrote them.
 *
 * Memory: graph inputs are copied host->device from t->data (non-ephemeral
 * ones once, then cached by header address).  Node outputs come from a
 * device arena owned by the backend: a bump allocator over one buffer that
 * is reset at the end of every graph_eval and regrown (once) to the
 * largest demand seen, so a steady stream of graphs makes no cudaMalloc /
 * cudaFree calls.  Outputs no later node consumes are copied back to
 * t->data; under g->no_readback they get their own device buffer instead
 * and stay cached for the next graph.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "../../include/sam3cu_backend.h"
#include "host_xfer.h"

/* ------------------------------------------------------------------ state */

struct devent {                   /* device copy of a host tensor */
	const struct sam3_tensor *t;
	const void               *data;   /* t->data when copied */
	size_t                    nbytes;
	void                     *dptr;
	int                       kind;   /* 0 empty, 1 cached input, 2 graph-local */
	const void               *aux;    /* derived buffer (f32 bias, q8 repack...) */
	int                       view;   /* dptr + str describe a strided view */
	int                       own;    /* graph-local dptr owned (not arena) */
	int64_t                   str[SAM3_MAX_DIMS];  /* element strides (view) */
};

/* bump allocator for graph-local device buffers */
struct arena {
	char   *base;
	size_t  cap, off, need;
	void  **extra;                    /* overflow allocations of this graph */
	size_t  nextra, capextra;
};

struct hostblk {
	struct hostblk *next;
};

struct impl {
	void            *stream;
	struct devent   *map;             /* open addressing on tensor address */
	size_t           cap, used;
	struct hostblk  *host;            /* alloc_tensor buffers */
	struct arena     ar;              /* graph-local device buffers */
	struct hxfer    *hx;              /* staged host transfers (may be NULL) */
	struct sam3_graph *g;             /* graph being evaluated */
	int              prof;            /* SAM3CU_VTABLE_PROFILE set */
	double           prof_s[SAM3_OP_COUNT + 3];  /* ops, readback, total, uploads */
	long             prof_n[SAM3_OP_COUNT + 3];
	double           prof_b[2];                  /* bytes uploaded / read back */
	/* per-graph scratch tables, sized to n_nodes */
	int             *uses;
	int             *flags;
	int              nflags;
};

enum { F_SKIP = 1, F_LAZY_T = 2, F_BIAS_FUSED = 4, F_GELU_FUSED = 8, F_RES_FUSED = 16 };

static size_t dsize(enum sam3_dtype d)
{
	switch (d) {
	case SAM3_DTYPE_F32: return 4;
	case SAM3_DTYPE_F16: return 2;
	case SAM3_DTYPE_BF16: return 2;
	case SAM3_DTYPE_I32: return 4;
	case SAM3_DTYPE_I8: return 1;
	default: return 0;
	}
}

static int64_t nelems(const struct sam3_tensor *t)
{
	int64_t n = 1;
	for (int i = 0; i < t->n_dims; i++)
		n *= t->dims[i];
	return n;
}

static size_t tbytes(const struct sam3_tensor *t)
{
	if (t->dtype == SAM3_DTYPE_Q8_0)
		return (size_t)((nelems(t) + 31) / 32) * 36;
	return (size_t)nelems(t) * dsize(t->dtype);
}

static struct impl *IM(struct sam3_backend *be)
{
	return (struct impl *)((struct sam3_cuda_backend *)be)->impl;
}

static enum sam3_error st(int rc)
{
	if (rc == 0)
		return SAM3_OK;
	if (rc >= -7)
		return (enum sam3_error)rc;
	if (rc == SAM3CU_EDTYPE2)
		return SAM3_EDTYPE;
	if (rc == SAM3CU_ENOMEM2)
		return SAM3_ENOMEM;
	if (rc == SAM3CU_ESHAPE)
		return SAM3_EINVAL;
	return SAM3_EBACKEND;
}

#define TRY(x) do { enum sam3_error e_ = st(x); if (e_ != SAM3_OK) { \
	fprintf(stderr, "[sam3cu] %s:%d: %s failed: %s\n", __FILE__, __LINE__, #x, \
		sam3cu_strerror(x)); return e_; } } while (0)

static double now_s(void)
{
	struct timespec ts;
	clock_gettime(CLOCK_MONOTONIC, &ts);
	return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* ------------------------------------------------------------------ map */

static size_t hptr(const void *p, size_t cap)
{
	uintptr_t x = (uintptr_t)p;
	x ^= x >> 17;
	x *= 0x9E3779B97F4A7C15ull;
	return (size_t)(x >> 20) & (cap - 1);
}

static struct devent *map_find(struct impl *m, const struct sam3_tensor *t)
{
	if (!m->cap)
		return NULL;
	size_t i = hptr(t, m->cap);
	for (size_t k = 0; k < m->cap; k++, i = (i + 1) & (m->cap - 1)) {
		if (m->map[i].kind == 0)
			return NULL;
		if (m->map[i].t == t && m->map[i].kind > 0)
			return &m->map[i];
	}
	return NULL;
}

static void devent_free(struct devent *e)
{
	if (e->dptr && (e->kind == 1 || e->own))
		sam3cu_dev_free(e->dptr);
	if (e->aux)
		sam3cu_dev_free((void *)e->aux);
	e->dptr = NULL;
	e->aux = NULL;
}

static enum sam3_error map_rehash(struct impl *m, size_t ncap);

static struct devent *map_insert(struct impl *m, const struct sam3_tensor *t)
{
	if ((m->used + 1) * 2 > m->cap &&
	    map_rehash(m, m->cap ? m->cap * 2 : 1024) != SAM3_OK)
		return NULL;
	size_t i = hptr(t, m->cap);
	while (m->map[i].kind != 0 && m->map[i].t != t)
		i = (i + 1) & (m->cap - 1);
	if (m->map[i].kind == 0)
		m->used++;
	else
		devent_free(&m->map[i]);
	memset(&m->map[i], 0, sizeof(m->map[i]));
	m->map[i].t = t;
	return &m->map[i];
}

static enum sam3_error map_rehash(struct impl *m, size_t ncap)
{
	struct devent *old = m->map;
	size_t ocap = m->cap;
	struct devent *nm = calloc(ncap, sizeof(*nm));
	if (!nm)
		return SAM3_ENOMEM;
	m->map = nm;
	m->cap = ncap;
	m->used = 0;
	for (size_t i = 0; i < ocap; i++) {
		if (old[i].kind <= 0)
			continue;
		size_t j = hptr(old[i].t, ncap);
		while (nm[j].kind != 0)
			j = (j + 1) & (ncap - 1);
		nm[j] = old[i];
		m->used++;
	}
	free(old);
	return SAM3_OK;
}

/* remove graph-local entries (kind 2), keep cached inputs */
static void map_drop_local(struct impl *m)
{
	int any = 0;
	for (size_t i = 0; i < m->cap; i++)
		if (m->map[i].kind == 2) {
			if (m->map[i].aux)
				sam3cu_dev_free((void *)m->map[i].aux);
			if (m->map[i].own && m->map[i].dptr)
				sam3cu_dev_free(m->map[i].dptr);
			m->map[i].dptr = NULL;
			m->map[i].aux = NULL;
			m->map[i].own = 0;
			m->map[i].kind = -1; /* tombstone */
			any = 1;
		}
	if (any)
		map_rehash(m, m->cap);
}

static enum sam3_error tmp_alloc(struct impl *m, size_t bytes, void **p)
{
	struct arena *a = &m->ar;
	bytes = (bytes + 255) & ~(size_t)255;
	if (!bytes)
		bytes = 256;
	a->need += bytes;
	if (a->base && a->off + bytes <= a->cap) {
		*p = a->base + a->off;
		a->off += bytes;
		return SAM3_OK;
	}
	/* past the arena: a separate buffer for this graph; the arena grows to
	 * the whole demand when the graph ends */
	if (a->nextra == a->capextra) {
		size_t nc = a->capextra ? a->capextra * 2 : 64;
		void **n = realloc(a->extra, nc * sizeof(void *));
		if (!n)
			return SAM3_ENOMEM;
		a->extra = n;
		a->capextra = nc;
	}
	TRY(sam3cu_dev_alloc(p, bytes));
	a->extra[a->nextra++] = *p;
	return SAM3_OK;
}

/* end of a graph (the stream is idle): release the overflow buffers and
 * regrow the arena to this graph's total demand */
static void tmp_free_all(struct impl *m)
{
	struct arena *a = &m->ar;
	for (size_t i = 0; i < a->nextra; i++)
		sam3cu_dev_free(a->extra[i]);
	if (a->nextra && a->need > a->cap) {
		size_t ncap = (a->need + a->need / 8 + ((size_t)1 << 20) - 1) & ~(((size_t)1 << 20) - 1);
		void *nb = NULL;
		if (a->base)
			sam3cu_dev_free(a->base);
		a->base = NULL;
		a->cap = 0;
		if (sam3cu_dev_alloc(&nb, ncap) == 0) {
			a->base = nb;
			a->cap = ncap;
		}
	}
	a->nextra = 0;
	a->off = 0;
	a->need = 0;
}

static void arena_release(struct impl *m)
{
	tmp_free_all(m);
	if (m->ar.base)
		sam3cu_dev_free(m->ar.base);
	free(m->ar.extra);
	memset(&m->ar, 0, sizeof(m->ar));
}

/* ------------------------------------------------------------------ vtable */

static enum sam3_error cu_init(struct sam3_backend *be)
{
	struct sam3_cuda_backend *cb = (struct sam3_cuda_backend *)be;
	if (sam3cu_init(cb->device) != 0)
		return SAM3_EBACKEND;
	struct impl *m = calloc(1, sizeof(*m));
	if (!m)
		return SAM3_ENOMEM;
	if (sam3cu_stream_create(&m->stream) != 0) {
		free(m);
		return SAM3_EBACKEND;
	}
	m->hx = hxfer_create();  /* NULL: plain cudaMemcpyAsync transfers */
	const char *pv = getenv("SAM3CU_VTABLE_PROFILE");
	m->prof = pv && *pv ? atoi(pv) : 0;
	cb->impl = m;
	return SAM3_OK;
}

static void host_free_all(struct impl *m)
{
	while (m->host) {
		struct hostblk *n = m->host->next;
		free(m->host);
		m->host = n;
	}
}

/* SAM3CU_VTABLE_PROFILE: host time per op kind with a stream sync around
 * every node (so the sum is device + host time, serialised), uploads and
 * read-backs separately; printed to stderr and reset */
static void profile_print(struct impl *m)
{
	static const char *names[SAM3_OP_COUNT + 3] = {
		[SAM3_OP_MATMUL] = "MATMUL", [SAM3_OP_ADD] = "ADD", [SAM3_OP_MUL] = "MUL",
		[SAM3_OP_SOFTMAX] = "SOFTMAX", [SAM3_OP_GELU] = "GELU",
		[SAM3_OP_LAYERNORM] = "LAYERNORM", [SAM3_OP_CONV2D] = "CONV2D",
		[SAM3_OP_RESHAPE] = "RESHAPE", [SAM3_OP_TRANSPOSE] = "TRANSPOSE",
		[SAM3_OP_CAST] = "CAST", [SAM3_OP_CONCAT] = "CONCAT", [SAM3_OP_SLICE] = "SLICE",
		[SAM3_OP_ROPE] = "ROPE", [SAM3_OP_SDPA] = "SDPA",
		[SAM3_OP_COUNT] = "readback", [SAM3_OP_COUNT + 1] = "graph_eval total",
		[SAM3_OP_COUNT + 2] = "(uploads in ops)"};
	for (int i = 0; i < SAM3_OP_COUNT + 3; i++)
		if (m->prof_n[i])
			fprintf(stderr, "[sam3cu profile] %-18s %6ld calls %10.3f ms\n",
				names[i] ? names[i] : "other", m->prof_n[i], 1e3 * m->prof_s[i]);
	fprintf(stderr, "[sam3cu profile] uploaded %.1f MB, read back %.1f MB\n",
		m->prof_b[0] / 1e6, m->prof_b[1] / 1e6);
	memset(m->prof_s, 0, sizeof(m->prof_s));
	memset(m->prof_n, 0, sizeof(m->prof_n));
	memset(m->prof_b, 0, sizeof(m->prof_b));
}

/* measurement hook (no counterpart in the reference): print and reset the
 * SAM3CU_VTABLE_PROFILE counters of a CUDA backend instance */
void sam3cu_backend_profile_dump(struct sam3_backend *be)
{
	struct impl *m = IM(be);
	if (m && m->prof)
		profile_print(m);
}

static void cu_free(struct sam3_backend *be)
{
	struct impl *m = IM(be);
	if (!m)
		return;
	sam3cu_stream_sync(m->stream);
	if (m->prof)
		profile_print(m);
	arena_release(m);
	hxfer_destroy(m->hx);
	for (size_t i = 0; i < m->cap; i++)
		if (m->map[i].kind > 0)
			devent_free(&m->map[i]);
	free(m->map);
	free(m->uses);
	free(m->flags);
	host_free_all(m);
	sam3cu_stream_destroy(m->stream);
	free(m);
	((struct sam3_cuda_backend *)be)->impl = NULL;
}

static enum sam3_error cu_alloc_tensor(struct sam3_backend *be,
				       struct sam3_tensor *t)
{
	struct impl *m = IM(be);
	if (!t || t->n_dims < 1 || t->n_dims > SAM3_MAX_DIMS)
		return SAM3_EINVAL;
	size_t nb = tbytes(t);
	if (!nb)
		return SAM3_EINVAL;
	struct hostblk *b = aligned_alloc(64, (sizeof(*b) + 63) / 64 * 64 + ((nb + 63) / 64 * 64));
	if (!b)
		return SAM3_ENOMEM;
	b->next = m->host;
	m->host = b;
	t->data = (char *)b + (sizeof(*b) + 63) / 64 * 64;
	t->nbytes = nb;
	t->strides[t->n_dims - 1] = 1;
	for (int i = t->n_dims - 2; i >= 0; i--)
		t->strides[i] = t->strides[i + 1] * t->dims[i + 1];
	return SAM3_OK;
}

static void cu_arena_reset(struct sam3_backend *be)
{
	struct impl *m = IM(be);
	sam3cu_stream_sync(m->stream);
	tmp_free_all(m);
	map_drop_local(m);
	host_free_all(m);
}

static void cu_cache_invalidate(struct sam3_backend *be, const void *start,
				size_t len)
{
	struct impl *m = IM(be);
	const char *lo = start, *hi = (const char *)start + len;
	int any = 0;
	sam3cu_stream_sync(m->stream);
	for (size_t i = 0; i < m->cap; i++) {
		struct devent *e = &m->map[i];
		if (e->kind != 1)
			continue;
		const char *a = (const char *)e->t, *d = e->data;
		if ((a >= lo && a < hi) || (d && d >= lo && d < hi)) {
			devent_free(e);
			e->kind = -1;
			any = 1;
		}
	}
	if (any)
		map_rehash(m, m->cap);
}

static void contig_strides(const struct sam3_tensor *t, int64_t *str)
{
	int64_t acc = 1;
	for (int i = t->n_dims - 1; i >= 0; i--) {
		str[i] = acc;
		acc *= t->dims[i];
	}
}

static int is_contig(const struct sam3_tensor *t, const int64_t *str)
{
	int64_t acc = 1;
	for (int i = t->n_dims - 1; i >= 0; i--) {
		if (t->dims[i] != 1 && str[i] != acc)
			return 0;
		acc *= t->dims[i];
	}
	return 1;
}

static int uses_of(struct sam3_graph *g, const struct sam3_tensor *t);
static int res_partner(struct sam3_graph *g, int i, int j);

/* device pointer (and element strides) of a tensor produced in this graph
 * or a graph input; a view is returned as such */
static enum sam3_error dev_view(struct impl *m, const struct sam3_tensor *t,
				int produced, void **p, int64_t *str)
{
	struct devent *e = map_find(m, t);
	if (e && (e->kind == 2 || (e->data == t->data && e->nbytes == tbytes(t)))) {
		*p = e->dptr;
		if (str) {
			if (e->view)
				memcpy(str, e->str, sizeof(e->str));
			else
				contig_strides(t, str);
		}
		return SAM3_OK;
	}
	if (produced) {
		fprintf(stderr, "[sam3cu] tensor %p used before its producer ran\n",
			(const void *)t);
		return SAM3_EINVAL;
	}
	if (!t->data) {
		fprintf(stderr, "[sam3cu] graph input %p has no host data\n",
			(const void *)t);
		return SAM3_EINVAL;
	}
	size_t nb = tbytes(t);
	void *d = NULL;
	if (t->ephemeral) {
		TRY(tmp_alloc(m, nb, &d));
	} else {
		TRY(sam3cu_dev_alloc(&d, nb));
	}
	double tu = 0.0;
	if (m->prof) {
		sam3cu_stream_sync(m->stream);
		tu = now_s();
	}
	if (m->hx)
		TRY(hxfer_h2d(m->hx, d, t->data, nb, m->stream));
	else
		TRY(sam3cu_memcpy_h2d(d, t->data, nb, m->stream));
	if (m->prof) {
		sam3cu_stream_sync(m->stream);
		m->prof_s[SAM3_OP_COUNT + 2] += now_s() - tu;
		m->prof_n[SAM3_OP_COUNT + 2]++;
		m->prof_b[0] += (double)nb;
	}
	e = map_insert(m, t);
	if (!e)
		return SAM3_ENOMEM;
	e->data = t->data;
	e->nbytes = nb;
	e->dptr = d;
	e->kind = t->ephemeral ? 2 : 1;
	*p = d;
	if (str)
		contig_strides(t, str);
	return SAM3_OK;
}

/* contiguous device pointer: a view is gathered into an arena buffer on
 * first use, and the entry then refers to that copy */
static enum sam3_error dev_of(struct impl *m, const struct sam3_tensor *t,
			      int produced, void **p)
{
	TRY(dev_view(m, t, produced, p, NULL));
	struct devent *e = map_find(m, t);
	if (!e || !e->view)
		return SAM3_OK;
	size_t es = dsize(t->dtype);
	void *c;
	if (!es)
		return SAM3_EDTYPE;
	TRY(tmp_alloc(m, tbytes(t), &c));
	TRY(sam3cu_gather_strided(e->dptr, c, (int)es, t->n_dims, t->dims, e->str, m->stream));
	e->dptr = c;
	e->view = 0;
	*p = c;
	return SAM3_OK;
}

/* register `t` as a view of device memory p with element strides str */
static enum sam3_error set_view(struct impl *m, const struct sam3_tensor *t, void *p,
				const int64_t *str)
{
	struct devent *e = map_insert(m, t);
	if (!e)
		return SAM3_ENOMEM;
	e->data = t->data;
	e->nbytes = tbytes(t);
	e->dptr = p;
	e->kind = 2;
	e->view = !is_contig(t, str);
	memcpy(e->str, str, sizeof(int64_t) * (size_t)t->n_dims);
	return SAM3_OK;
}

static enum sam3_error out_buf(struct impl *m, const struct sam3_tensor *t,
			       void **p)
{
	/* a graph output that stays resident (no_readback) gets its own buffer:
	 * it outlives this graph's arena */
	int keep = m->g && m->g->no_readback && uses_of(m->g, t) == 0;
	if (keep)
		TRY(sam3cu_dev_alloc(p, tbytes(t)));
	else
		TRY(tmp_alloc(m, tbytes(t), p));
	struct devent *e = map_insert(m, t);
	if (!e) {
		if (keep)
			sam3cu_dev_free(*p);
		return SAM3_ENOMEM;
	}
	e->data = t->data;
	e->nbytes = tbytes(t);
	e->dptr = *p;
	e->kind = 2;
	e->own = keep;
	return SAM3_OK;
}

/* strides of the tensor `to` (dims) viewing the same elements as one with
 * dims `from` and strides fs, without a copy; 0 if no such strides exist
 * (the grouping of dims into chunks that are contiguous in memory) */
static int reshape_strides(const struct sam3_tensor *from, const int64_t *fs,
			   const struct sam3_tensor *to, int64_t *ts)
{
	int vd = to->n_dims - 1;
	int64_t base = fs[from->n_dims - 1], tn = 1, vn = 1;
	for (int d = from->n_dims - 1; d >= 0; d--) {
		tn *= from->dims[d];
		int chunk_end = d == 0 || (from->dims[d - 1] != 1 && fs[d - 1] != tn * base);
		if (!chunk_end)
			continue;
		while (vd >= 0 && (vn < tn || to->dims[vd] == 1)) {
			ts[vd] = vn * base;
			vn *= to->dims[vd];
			vd--;
		}
		if (vn != tn)
			return 0;
		if (d > 0) {
			base = fs[d - 1];
			tn = 1;
			vn = 1;
		}
	}
	return vd == -1;
}

static int is_16(enum sam3_dtype d)
{
	return d == SAM3_DTYPE_F16 || d == SAM3_DTYPE_BF16;
}

/* f32 copy of a small (bias / gamma / beta) tensor, cached on its entry */
static enum sam3_error f32_view(struct impl *m, const struct sam3_tensor *t,
				int produced, const float **out)
{
	void *d;
	TRY(dev_of(m, t, produced, &d));
	if (t->dtype == SAM3_DTYPE_F32) {
		*out = d;
		return SAM3_OK;
	}
	if (!is_16(t->dtype))
		return SAM3_EDTYPE;
	struct devent *e = map_find(m, t);
	if (e && e->aux) {
		*out = e->aux;
		return SAM3_OK;
	}
	void *f;
	TRY(sam3cu_dev_alloc(&f, (size_t)nelems(t) * 4));
	TRY(sam3cu_cast(d, t->dtype, f, SAM3_DTYPE_F32, nelems(t), m->stream));
	if (e)
		e->aux = f;
	*out = f;
	return SAM3_OK;
}

/* ------------------------------------------------------------------ ops */

/* y broadcasts over x as the reference's check_broadcast allows for these
 * kernels (cpu_elementwise.c:28-62): same size, a scalar, or y's dims equal
 * x's trailing dims (leading size-1 dims of y ignored). */
static int suffix_broadcast(const struct sam3_tensor *x, const struct sam3_tensor *y)
{
	int64_t n = nelems(x), nb = nelems(y);
	if (nb == n || nb == 1)
		return 1;
	if (nb == 0 || n % nb)
		return 0;
	int yd = y->n_dims;
	while (yd > 0 && y->dims[y->n_dims - yd] == 1)
		yd--;  /* skip leading 1s */
	if (yd > x->n_dims)
		return 0;
	for (int d = 0; d < yd; d++)
		if (y->dims[y->n_dims - 1 - d] != x->dims[x->n_dims - 1 - d])
			return 0;
	return 1;
}

static int produced_in(struct sam3_graph *g, int upto, const struct sam3_tensor *t)
{
	for (int i = 0; i < upto; i++)
		if (g->nodes[i].output == t)
			return 1;
	return 0;
}

/* MATMUL (+ fused bias / GELU): cpu_kernel_matmul family, gh_linear */
static enum sam3_error op_matmul(struct impl *m, struct sam3_graph *g, int ni)
{
	struct sam3_node *nd = &g->nodes[ni];
	struct sam3_tensor *a = nd->inputs[0], *b = nd->inputs[1];
	struct sam3_tensor *out = nd->output;
	const struct sam3_tensor *w = NULL;  /* [N,K] K-major */
	int lazy = 0;
	/* B produced by a lazy TRANSPOSE of a 2-D W in this graph? */
	for (int j = 0; j < ni; j++)
		if (g->nodes[j].output == b && (m->flags[j] & F_LAZY_T)) {
			w = g->nodes[j].inputs[0];
			lazy = 1;
		}
	if (!lazy && a->n_dims >= 3 && b->n_dims == a->n_dims) {
		/* batched N-D MATMUL (TinyViT window attention, :836-854): the
		 * leading dims of A and B must agree */
		int nd_ = a->n_dims;
		int64_t batch = 1;
		for (int d = 0; d < nd_ - 2; d++) {
			if (a->dims[d] != b->dims[d])
				return SAM3_EINVAL;
			batch *= a->dims[d];
		}
		int M = a->dims[nd_ - 2], K = a->dims[nd_ - 1], N = b->dims[nd_ - 1];
		if (b->dims[nd_ - 2] != K || a->dtype != b->dtype || batch > 65535)
			return SAM3_EINVAL;
		void *pa, *pb, *py;
		TRY(dev_of(m, a, produced_in(g, ni, a), &pa));
		TRY(dev_of(m, b, produced_in(g, ni, b), &pb));
		TRY(out_buf(m, out, &py));
		TRY(sam3cu_bmm(pa, pb, py, a->dtype, (int)batch, M, K, N, m->stream));
		return SAM3_OK;
	}
	if (!lazy && b->n_dims != 2)
		return SAM3_EINVAL;
	int K = a->dims[a->n_dims - 1];
	int64_t M = nelems(a) / K;
	int N = b->n_dims == 1 ? 1 : b->dims[b->n_dims - 1];
	if (lazy)
		N = w->dims[0];
	if ((lazy ? w->dims[1] : b->dims[b->n_dims - 2]) != K || M > 0x7fffffff)
		return SAM3_EINVAL;
	/* epilogue fusion target: the ADD / GELU output if fused */
	struct sam3_tensor *dst = out;
	const struct sam3_tensor *bias = NULL, *resid = NULL;
	int act = 0;
	if (m->flags[ni] & F_BIAS_FUSED) {
		for (int j = ni + 1; j < g->n_nodes; j++)
			if (g->nodes[j].op == SAM3_OP_ADD && g->nodes[j].inputs[0] == out) {
				bias = g->nodes[j].inputs[1];
				dst = g->nodes[j].output;
				if (m->flags[j] & F_RES_FUSED) {
					int r = res_partner(g, ni, j);
					if (r <= 0)
						return SAM3_EINVAL;
					struct sam3_node *rn = &g->nodes[r];
					resid = rn->inputs[0] == dst ? rn->inputs[1] : rn->inputs[0];
					dst = rn->output;
				}
				if (m->flags[j] & F_GELU_FUSED) {
					for (int k = j + 1; k < g->n_nodes; k++)
						if (g->nodes[k].op == SAM3_OP_GELU &&
						    g->nodes[k].inputs[0] == dst) {
							dst = g->nodes[k].output;
							act = SAM3CU_ACT_GELU_TANH;
							break;
						}
				}
				break;
			}
	}
	void *pa, *pw, *py;
	const float *pb = NULL;
	TRY(dev_of(m, a, produced_in(g, ni, a), &pa));
	if (bias)
		TRY(f32_view(m, bias, produced_in(g, ni, bias), &pb));
	TRY(out_buf(m, dst, &py));
	enum sam3_dtype wt = lazy ? w->dtype : b->dtype;

	if (wt == SAM3_DTYPE_Q8_0 && a->dtype == SAM3_DTYPE_F32) {
		if (lazy) {
			/* F32 x Q8_0 -> F32: activations to BF16, weight dequantised on chip */
			void *abf;
			TRY(tmp_alloc(m, (size_t)M * K * 2, &abf));
			TRY(sam3cu_cast(pa, SAM3_DTYPE_F32, abf, SAM3_DTYPE_BF16, M * K, m->stream));
			/* W [N,K] quantised along K: repack once per weight */
			void *pq;
			TRY(dev_of(m, w, produced_in(g, ni, w), &pq));
			struct devent *e = map_find(m, w);
			if (!e->aux) {
				void *q;
				TRY(sam3cu_dev_alloc(&q, (size_t)N * K + (size_t)(K / 32) * N * 4));
				TRY(sam3cu_q8_repack(pq, N, K, q, (float *)((char *)q + (size_t)N * K),
						     m->stream));
				e->aux = q;
			}
			const int8_t *q = e->aux;
			TRY(sam3cu_linear_q8(abf, SAM3CU_BF16, q, (const float *)(q + (size_t)N * K), pb,
					     NULL, py, SAM3CU_F32, (int)M, K, N, act, m->stream));
			return SAM3_OK;
		}
		/* single-op convention: B [K,N] quantised flat (cpu_matmul_q8.c:28-35) */
		void *pq, *bf, *bt;
		TRY(dev_of(m, b, produced_in(g, ni, b), &pq));
		TRY(tmp_alloc(m, (size_t)K * N * 4, &bf));
		TRY(tmp_alloc(m, (size_t)K * N * 4, &bt));
		TRY(sam3cu_q8_dequantize(pq, bf, (int64_t)K * N, m->stream));
		int dims[2] = {K, N}, perm[2] = {1, 0};
		TRY(sam3cu_permute(bf, bt, 4, 2, dims, perm, m->stream));
		TRY(sam3cu_linear(pa, SAM3CU_F32, bt, pb, NULL, py, SAM3CU_F32, (int)M, K, N, act,
				  m->stream));
		return SAM3_OK;
	}
	if (a->dtype != wt || (a->dtype != SAM3_DTYPE_F32 && !is_16(a->dtype)))
		return SAM3_EDTYPE;
	if (lazy) {
		TRY(dev_of(m, w, produced_in(g, ni, w), &pw));
	} else {
		/* B [K,N]: a transposed view of a contiguous [N,K] is used as it
		 * lies; otherwise B is transposed into [N,K] */
		void *pbk;
		int64_t bs[SAM3_MAX_DIMS];
		TRY(dev_view(m, b, produced_in(g, ni, b), &pbk, bs));
		if (b->n_dims == 2 && bs[0] == 1 && bs[1] == K) {
			pw = pbk;
		} else {
			TRY(dev_of(m, b, produced_in(g, ni, b), &pbk));
			TRY(tmp_alloc(m, (size_t)K * N * dsize(b->dtype), &pw));
			int dims[2] = {K, N}, perm[2] = {1, 0};
			TRY(sam3cu_permute(pbk, pw, (int)dsize(b->dtype), 2, dims, perm, m->stream));
		}
	}
	if (resid) {  /* dst = resid + linear: a copy of resid, then the in-place reduce-add */
		void *pr;
		if (dst->dtype != SAM3_DTYPE_F32 || act)
			return SAM3_EINVAL;
		TRY(dev_of(m, resid, produced_in(g, ni, resid), &pr));
		TRY(sam3cu_memcpy_d2d(py, pr, tbytes(dst), m->stream));
		TRY(sam3cu_linear(pa, a->dtype, pw, pb, py, py, SAM3_DTYPE_F32, (int)M, K, N, 0,
				  m->stream));
		return SAM3_OK;
	}
	TRY(sam3cu_linear(pa, a->dtype, pw, pb, NULL, py, dst->dtype, (int)M, K, N, act,
			  m->stream));
	return SAM3_OK;
}

static enum sam3_error op_node(struct impl *m, struct sam3_graph *g, int ni)
{
	struct sam3_node *nd = &g->nodes[ni];
	struct sam3_tensor *out = nd->output;
	struct sam3_tensor *x = nd->inputs[0];
	void *px = NULL, *py = NULL;
	if (!out || !x)
		return SAM3_EINVAL;

	switch (nd->op) {
	case SAM3_OP_MATMUL:
		return op_matmul(m, g, ni);

	case SAM3_OP_RESHAPE: {  /* a view (cpu_reshape.c:20-38) */
		int64_t xs[SAM3_MAX_DIMS], ys[SAM3_MAX_DIMS];
		if (tbytes(out) != tbytes(x))
			return SAM3_EINVAL;
		TRY(dev_view(m, x, produced_in(g, ni, x), &px, xs));
		if (x->dtype == SAM3_DTYPE_Q8_0 || !reshape_strides(x, xs, out, ys)) {
			TRY(dev_of(m, x, produced_in(g, ni, x), &px));
			contig_strides(out, ys);
		}
		return set_view(m, out, px, ys);
	}

	case SAM3_OP_TRANSPOSE: {  /* a view with permuted strides (cpu_transpose.c:312-387) */
		int64_t xs[SAM3_MAX_DIMS], ys[SAM3_MAX_DIMS];
		if (!dsize(x->dtype))
			return SAM3_EDTYPE;
		int axes[SAM3_MAX_DIMS], has = 0, nd_ = x->n_dims;
		for (int i = 0; i < nd_; i++) {
			axes[i] = nd->params[i];
			if (axes[i])
				has = 1;
		}
		if (!has) {  /* legacy: swap the last two dims (cpu_transpose.c:330-348) */
			for (int i = 0; i < nd_; i++)
				axes[i] = i;
			if (nd_ >= 2) {
				axes[nd_ - 2] = nd_ - 1;
				axes[nd_ - 1] = nd_ - 2;
			}
		}
		if (out->n_dims != nd_)
			return SAM3_EINVAL;
		TRY(dev_view(m, x, produced_in(g, ni, x), &px, xs));
		for (int i = 0; i < nd_; i++) {
			if (axes[i] < 0 || axes[i] >= nd_ || out->dims[i] != x->dims[axes[i]])
				return SAM3_EINVAL;
			ys[i] = xs[axes[i]];
		}
		return set_view(m, out, px, ys);
	}

	case SAM3_OP_SLICE: {  /* a view: [start, end) along params[0] (cpu_slice.c) */
		int64_t xs[SAM3_MAX_DIMS];
		size_t es = dsize(x->dtype);
		int axis = nd->params[0], start = nd->params[1];
		if (!es)
			return SAM3_EDTYPE;
		if (axis < 0 || axis >= x->n_dims || start < 0 || out->n_dims != x->n_dims ||
		    start + out->dims[axis] > x->dims[axis])
			return SAM3_EINVAL;
		TRY(dev_view(m, x, produced_in(g, ni, x), &px, xs));
		return set_view(m, out, (char *)px + (size_t)start * (size_t)xs[axis] * es, xs);
	}

	case SAM3_OP_BIAS_ADD:  /* NHWC x + bias[C] (cpu_bias_add.c) */
	case SAM3_OP_MUL:
	case SAM3_OP_ADD: {
		struct sam3_tensor *y = nd->inputs[1];
		void *pyy;
		if (!y || x->dtype != y->dtype ||
		    (x->dtype != SAM3_DTYPE_F32 && !is_16(x->dtype)))
			return SAM3_EDTYPE;
		int64_t n = nelems(x), nb = nelems(y);
		if (!suffix_broadcast(x, y))
			return SAM3_EINVAL;
		TRY(dev_of(m, x, produced_in(g, ni, x), &px));
		TRY(dev_of(m, y, produced_in(g, ni, y), &pyy));
		TRY(out_buf(m, out, &py));
		if (nd->op == SAM3_OP_MUL)
			TRY(sam3cu_mul(px, pyy, py, x->dtype, n, nb, m->stream));
		else
			TRY(sam3cu_add(px, pyy, py, x->dtype, n, nb, m->stream));
		return SAM3_OK;
	}

	case SAM3_OP_SOFTMAX: {  /* last dim (cpu_softmax.c:29-47) */
		if (x->dtype != SAM3_DTYPE_F32 && !is_16(x->dtype))
			return SAM3_EDTYPE;
		int cols = x->dims[x->n_dims - 1];
		TRY(dev_of(m, x, produced_in(g, ni, x), &px));
		TRY(out_buf(m, out, &py));
		TRY(sam3cu_softmax(px, py, x->dtype, nelems(x) / cols, cols, m->stream));
		return SAM3_OK;
	}

	case SAM3_OP_BATCHNORM: {  /* NHWC, inputs x, gamma, beta, mean, var */
		const float *gm = NULL, *bt = NULL, *mu = NULL, *vr = NULL;
		int C = x->dims[x->n_dims - 1];
		if (nd->n_inputs < 5 || !nd->inputs[3] || !nd->inputs[4])
			return SAM3_EINVAL;
		TRY(dev_of(m, x, produced_in(g, ni, x), &px));
		if (nd->inputs[1])
			TRY(f32_view(m, nd->inputs[1], produced_in(g, ni, nd->inputs[1]), &gm));
		if (nd->inputs[2])
			TRY(f32_view(m, nd->inputs[2], produced_in(g, ni, nd->inputs[2]), &bt));
		TRY(f32_view(m, nd->inputs[3], produced_in(g, ni, nd->inputs[3]), &mu));
		TRY(f32_view(m, nd->inputs[4], produced_in(g, ni, nd->inputs[4]), &vr));
		TRY(out_buf(m, out, &py));
		TRY(sam3cu_batchnorm(px, py, x->dtype, nelems(x), C, gm, bt, mu, vr, m->stream));
		return SAM3_OK;
	}

	case SAM3_OP_CONCAT: {  /* along params[0] (cpu_concat.c) */
		int axis = nd->params[0];
		size_t es = dsize(x->dtype);
		if (!es || axis < 0 || axis >= out->n_dims)
			return SAM3_EINVAL;
		int64_t outer = 1;
		for (int d = 0; d < axis; d++)
			outer *= out->dims[d];
		size_t row_out = (size_t)(nelems(out) / outer) * es, off = 0;
		TRY(out_buf(m, out, &py));
		for (int k = 0; k < nd->n_inputs; k++) {
			struct sam3_tensor *in = nd->inputs[k];
			void *pin;
			if (!in || in->dtype != out->dtype)
				return SAM3_EINVAL;
			size_t row_in = (size_t)(nelems(in) / outer) * es;
			TRY(dev_of(m, in, produced_in(g, ni, in), &pin));
			TRY(sam3cu_memcpy2d_d2d((char *)py + off, row_out, pin, row_in, row_in,
						(size_t)outer, m->stream));
			off += row_in;
		}
		return off == row_out ? SAM3_OK : SAM3_EINVAL;
	}

	case SAM3_OP_GELU:
		if (x->dtype != SAM3_DTYPE_F32 && !is_16(x->dtype))
			return SAM3_EDTYPE;
		TRY(dev_of(m, x, produced_in(g, ni, x), &px));
		TRY(out_buf(m, out, &py));
		TRY(sam3cu_gelu(px, py, x->dtype, nelems(x), m->stream));
		return SAM3_OK;

	case SAM3_OP_CAST:
		TRY(dev_of(m, x, produced_in(g, ni, x), &px));
		TRY(out_buf(m, out, &py));
		TRY(sam3cu_cast(px, x->dtype, py, out->dtype, nelems(x), m->stream));
		return SAM3_OK;

	case SAM3_OP_LAYERNORM: {  /* cpu_layernorm.c:210-254; gamma/beta optional */
		const float *gm = NULL, *bt = NULL;
		int cols = x->dims[x->n_dims - 1];
		TRY(dev_of(m, x, produced_in(g, ni, x), &px));
		if (nd->n_inputs > 1 && nd->inputs[1])
			TRY(f32_view(m, nd->inputs[1], produced_in(g, ni, nd->inputs[1]), &gm));
		if (nd->n_inputs > 2 && nd->inputs[2])
			TRY(f32_view(m, nd->inputs[2], produced_in(g, ni, nd->inputs[2]), &bt));
		TRY(out_buf(m, out, &py));
		TRY(sam3cu_layernorm(px, x->dtype, gm, bt, py, out->dtype, (int)(nelems(x) / cols),
				     cols, m->stream));
		return SAM3_OK;
	}

	case SAM3_OP_ROPE: {  /* [B,S,H,hd]; reads a row-strided view in place */
		struct sam3_tensor *cs = nd->inputs[1], *sn = nd->inputs[2];
		void *pc, *ps;
		int64_t xs[SAM3_MAX_DIMS];
		if (x->n_dims != 4 || !cs || !sn || cs->dtype != SAM3_DTYPE_F32 ||
		    sn->dtype != SAM3_DTYPE_F32)
			return SAM3_EINVAL;
		TRY(dev_view(m, x, produced_in(g, ni, x), &px, xs));
		int hd = x->dims[3], H = x->dims[2], S_ = x->dims[1];
		if (!(xs[3] == 1 && xs[2] == hd && xs[1] >= (int64_t)H * hd &&
		      xs[0] == (int64_t)S_ * xs[1])) {
			TRY(dev_of(m, x, produced_in(g, ni, x), &px));
			xs[1] = (int64_t)H * hd;
		}
		TRY(dev_of(m, cs, produced_in(g, ni, cs), &pc));
		TRY(dev_of(m, sn, produced_in(g, ni, sn), &ps));
		TRY(out_buf(m, out, &py));
		TRY(sam3cu_rope_rows(px, xs[1], pc, ps, py, (int64_t)H * hd, x->dtype, x->dims[0],
				     S_, H, hd, m->stream));
		return SAM3_OK;
	}

	case SAM3_OP_SDPA: {  /* [S,hd] or [B,H,S,hd], optional mask [Sq,Sk] (cpu_sdpa.c:216-288) */
		struct sam3_tensor *k = nd->inputs[1], *v = nd->inputs[2];
		struct sam3_tensor *mk = nd->n_inputs > 3 ? nd->inputs[3] : NULL;
		void *pk, *pv, *pm = NULL;
		int64_t qs[SAM3_MAX_DIMS], ks[SAM3_MAX_DIMS], vs[SAM3_MAX_DIMS];
		int hd = x->dims[x->n_dims - 1];
		int sq = x->dims[x->n_dims - 2], sk = k->dims[k->n_dims - 2];
		int four = x->n_dims == 4 && k->n_dims == 4 && v->n_dims == 4 && out->n_dims == 4;
		int B = four ? x->dims[0] : 1;
		int H = four ? x->dims[1] : (int)(nelems(x) / ((int64_t)sq * hd));
		if (k->dtype != x->dtype || v->dtype != x->dtype || k->dims[k->n_dims - 1] != hd)
			return SAM3_EINVAL;
		if (four) {
			TRY(dev_view(m, x, produced_in(g, ni, x), &px, qs));
			TRY(dev_view(m, k, produced_in(g, ni, k), &pk, ks));
			TRY(dev_view(m, v, produced_in(g, ni, v), &pv, vs));
		} else {  /* leading dims flattened into heads of one batch */
			TRY(dev_of(m, x, produced_in(g, ni, x), &px));
			TRY(dev_of(m, k, produced_in(g, ni, k), &pk));
			TRY(dev_of(m, v, produced_in(g, ni, v), &pv));
			qs[1] = (int64_t)sq * hd, qs[2] = hd, qs[3] = 1;
			ks[1] = vs[1] = (int64_t)sk * hd, ks[2] = vs[2] = hd, ks[3] = vs[3] = 1;
			qs[0] = qs[1] * H, ks[0] = vs[0] = ks[1] * H;
		}
		if (mk)
			TRY(dev_of(m, mk, produced_in(g, ni, mk), &pm));
		/* the output in head-interleaved order [B,S,H,hd]: the permute(0,2,1,3)
		 * that follows in gh_multihead_attention_rope is then contiguous */
		int64_t ld_o = (int64_t)H * hd;
		int64_t os[SAM3_MAX_DIMS] = {(int64_t)sq * ld_o, hd, ld_o, 1};
		void *buf;
		TRY(tmp_alloc(m, tbytes(out), &buf));
		if (four) {
			TRY(set_view(m, out, buf, os));
		} else {
			struct devent *e = map_insert(m, out);
			if (!e)
				return SAM3_ENOMEM;
			e->data = out->data;
			e->nbytes = tbytes(out);
			e->dptr = buf;
			e->kind = 2;
		}
		if (x->dtype == SAM3_DTYPE_F32) {
			int64_t q3[3] = {qs[0], qs[1], qs[2]}, k3[3] = {ks[0], ks[1], ks[2]};
			int64_t v3[3] = {vs[0], vs[1], vs[2]};
			int64_t o3[3] = {(int64_t)sq * ld_o, hd, ld_o};
			if (!four)
				o3[0] = 0, o3[1] = (int64_t)sq * hd, o3[2] = hd;
			if (qs[3] != 1 || ks[3] != 1 || vs[3] != 1)
				return SAM3_EINVAL;
			TRY(sam3cu_sdpa_f32_strided(px, q3, pk, k3, pv, v3, pm, buf, o3, B, H, sq, sk,
						    hd, m->stream));
			return SAM3_OK;
		}
		/* 16-bit: the tcgen05 kernel reads Q/K/V rows (b*S + s) of one
		 * shared pitch with head h at column h*hd, and writes O the same way */
		if (is_16(x->dtype) && !mk && sq == sk && hd == 64) {
			int64_t ld = qs[2];
			int ok = qs[3] == 1 && ks[3] == 1 && vs[3] == 1 && qs[1] == hd && ks[1] == hd &&
				 vs[1] == hd && ks[2] == ld && vs[2] == ld && qs[0] == sq * ld &&
				 ks[0] == sk * ld && vs[0] == sk * ld;
			if (!ok) {
				TRY(dev_of(m, x, produced_in(g, ni, x), &px));
				TRY(dev_of(m, k, produced_in(g, ni, k), &pk));
				TRY(dev_of(m, v, produced_in(g, ni, v), &pv));
				/* contiguous [B,H,S,hd]: one group per (b, h), one head */
				TRY(sam3cu_sdpa(px, pk, pv, 64, buf, 64, x->dtype, B * H, sq, 1, 64,
						m->stream));
				int64_t cs_[SAM3_MAX_DIMS];
				contig_strides(out, cs_);
				return set_view(m, out, buf, cs_);
			}
			TRY(sam3cu_sdpa(px, pk, pv, ld, buf, ld_o, x->dtype, B, sq, H, 64, m->stream));
			return SAM3_OK;
		}
		return SAM3_EDTYPE;
	}

	case SAM3_OP_CONV2D: {  /* NHWC x OHWI, groups 1 (cpu_conv2d.c:296-400) */
		struct sam3_tensor *w = nd->inputs[1];
		int stride = nd->params[0] > 0 ? nd->params[0] : 1, pad = nd->params[1];
		int groups = nd->params[2] > 0 ? nd->params[2] : 1;
		if (groups > 1 && w && x->n_dims == 4 && w->n_dims == 4 && w->dtype == x->dtype &&
		    w->dims[3] * groups == x->dims[3] && !(nd->params[3] && nd->params[3] != pad)) {
			/* grouped / depthwise: direct kernel */
			void *pw;
			TRY(dev_of(m, x, produced_in(g, ni, x), &px));
			TRY(dev_of(m, w, produced_in(g, ni, w), &pw));
			TRY(out_buf(m, out, &py));
			TRY(sam3cu_conv2d_grouped_nhwc(px, pw, py, x->dtype, x->dims[0], x->dims[1],
						       x->dims[2], x->dims[3], w->dims[0], w->dims[1],
						       w->dims[2], stride, pad, groups, m->stream));
			return SAM3_OK;
		}
		if (!w || x->n_dims != 4 || w->n_dims != 4 || groups != 1 ||
		    (nd->params[3] && nd->params[3] != pad) || w->dims[3] != x->dims[3] ||
		    w->dtype != x->dtype)
			return SAM3_EDTYPE;
		int N = x->dims[0], H = x->dims[1], W = x->dims[2], C = x->dims[3];
		int OC = w->dims[0], KH = w->dims[1], KW = w->dims[2];
		int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
		int kk = KH * KW * C, al = x->dtype == SAM3_DTYPE_F32 ? 4 : 8;
		int kpad = (kk + al - 1) / al * al;
		size_t es = dsize(x->dtype);
		void *pw, *col, *wpad;
		TRY(dev_of(m, x, produced_in(g, ni, x), &px));
		TRY(dev_of(m, w, produced_in(g, ni, w), &pw));
		TRY(tmp_alloc(m, (size_t)N * OH * OW * kpad * es, &col));
		TRY(sam3cu_im2col_nhwc(px, col, x->dtype, N, H, W, C, KH, KW, stride, pad, kpad,
				       m->stream));
		if (kpad != kk) {  /* weight rows padded to kpad: im2col of a 1x1 "image" */
			TRY(tmp_alloc(m, (size_t)OC * kpad * es, &wpad));
			TRY(sam3cu_im2col_nhwc(pw, wpad, x->dtype, OC, 1, 1, kk, 1, 1, 1, 0, kpad,
					       m->stream));
		} else {
			wpad = pw;
		}
		TRY(out_buf(m, out, &py));
		TRY(sam3cu_linear(col, x->dtype, wpad, NULL, NULL, py, out->dtype, N * OH * OW, kpad,
				  OC, 0, m->stream));
		return SAM3_OK;
	}

	case SAM3_OP_CONV_TRANSPOSE2D: {  /* NHWC x OHWI (cpu_conv_transpose2d.c) */
		struct sam3_tensor *w = nd->inputs[1];
		int stride = nd->params[0] > 0 ? nd->params[0] : 1, pad = nd->params[1];
		if (!w || x->n_dims != 4 || w->n_dims != 4 || w->dims[3] != x->dims[3] ||
		    w->dtype != x->dtype || (x->dtype != SAM3_DTYPE_F32 && !is_16(x->dtype)))
			return SAM3_EDTYPE;
		int N = x->dims[0], H = x->dims[1], W = x->dims[2], C = x->dims[3];
		int OC = w->dims[0], KH = w->dims[1], KW = w->dims[2];
		size_t es = dsize(x->dtype);
		void *pw;
		TRY(dev_of(m, x, produced_in(g, ni, x), &px));
		TRY(dev_of(m, w, produced_in(g, ni, w), &pw));
		TRY(out_buf(m, out, &py));
		if (KH == stride && KW == stride && pad == 0 && C % (es == 4 ? 4 : 8) == 0) {
			/* non-overlapping (the FPN neck's k2 s2): one GEMM
			 * [N*H*W, C] x [(ky,kx,oc), C]^T, then a pixel shuffle;
			 * the weight re-layout is cached per weight */
			struct devent *e = map_find(m, w);
			void *wg = e ? (void *)e->aux : NULL;
			if (!wg) {
				int dims[4] = {OC, KH, KW, C}, perm[4] = {1, 2, 0, 3};
				TRY(sam3cu_dev_alloc(&wg, (size_t)OC * KH * KW * C * es));
				TRY(sam3cu_permute(pw, wg, (int)es, 4, dims, perm, m->stream));
				if (e)
					e->aux = wg;
			}
			void *tmp;
			int64_t M = (int64_t)N * H * W;
			TRY(tmp_alloc(m, (size_t)M * KH * KW * OC * es, &tmp));
			TRY(sam3cu_linear(px, x->dtype, wg, NULL, NULL, tmp, x->dtype, (int)M, C,
					  KH * KW * OC, 0, m->stream));
			TRY(sam3cu_convt_shuffle(tmp, py, (int)es, N, H, W, KH, OC, m->stream));
			if (!e)
				sam3cu_dev_free(wg);
			return SAM3_OK;
		}
		TRY(sam3cu_conv_transpose2d_nhwc(px, pw, py, x->dtype, N, H, W, C, OC, KH, KW, stride,
						 pad, m->stream));
		return SAM3_OK;
	}

	case SAM3_OP_MAXPOOL2D: {  /* NHWC, params kernel, stride (cpu_maxpool2d.c) */
		int k = nd->params[0], kst = nd->params[1] > 0 ? nd->params[1] : k;
		if (x->n_dims != 4 || k <= 0 || (x->dtype != SAM3_DTYPE_F32 && !is_16(x->dtype)))
			return SAM3_EDTYPE;
		TRY(dev_of(m, x, produced_in(g, ni, x), &px));
		TRY(out_buf(m, out, &py));
		TRY(sam3cu_maxpool2d_nhwc(px, py, x->dtype, x->dims[0], x->dims[1], x->dims[2],
					  x->dims[3], k, kst, m->stream));
		return SAM3_OK;
	}

	default:
		fprintf(stderr, "[sam3cu] op %d (dtype %d) is not supported on CUDA\n",
			(int)nd->op, (int)x->dtype);
		return SAM3_EDTYPE;
	}
}

static int count_uses(struct sam3_graph *g, int from, const struct sam3_tensor *t)
{
	int n = 0;
	for (int i = from; i < g->n_nodes; i++)
		for (int k = 0; k < g->nodes[i].n_inputs; k++)
			if (g->nodes[i].inputs[k] == t)
				n++;
	return n;
}

static int uses_of(struct sam3_graph *g, const struct sam3_tensor *t)
{
	return count_uses(g, 0, t);
}

static int producer_of(struct sam3_graph *g, const struct sam3_tensor *t)
{
	for (int i = 0; i < g->n_nodes; i++)
		if (g->nodes[i].output == t)
			return i;
	return -1;
}

/* The ADD node r that is the only consumer of bias-ADD j's output and adds
 * an F32 tensor of the same shape that exists before MATMUL i runs; 0 if
 * there is none. */
static int res_partner(struct sam3_graph *g, int i, int j)
{
	const struct sam3_tensor *y = g->nodes[j].output;
	if (y->dtype != SAM3_DTYPE_F32 || count_uses(g, j + 1, y) != 1)
		return 0;
	for (int r = j + 1; r < g->n_nodes; r++) {
		struct sam3_node *nd = &g->nodes[r];
		if (nd->op != SAM3_OP_ADD || nd->n_inputs < 2)
			continue;
		if (nd->inputs[0] != y && nd->inputs[1] != y)
			continue;
		const struct sam3_tensor *x = nd->inputs[0] == y ? nd->inputs[1] : nd->inputs[0];
		if (!x || x == y || x->dtype != SAM3_DTYPE_F32 || nelems(x) != nelems(y) ||
		    nd->output->dtype != SAM3_DTYPE_F32)
			return 0;
		return producer_of(g, x) < i ? r : 0;
	}
	return 0;
}

/* mark the peepholes: lazy W transposes, bias / GELU fusion into MATMUL */
static void plan(struct impl *m, struct sam3_graph *g)
{
	memset(m->flags, 0, sizeof(int) * (size_t)g->n_nodes);
	for (int i = 0; i < g->n_nodes; i++) {
		struct sam3_node *nd = &g->nodes[i];
		if (nd->op == SAM3_OP_TRANSPOSE && nd->inputs[0] && nd->inputs[0]->n_dims == 2 &&
		    (nd->params[0] | nd->params[1]) == 0 &&
		    nd->inputs[0]->dtype != SAM3_DTYPE_I32) {
			/* every consumer must be a MATMUL using it as B */
			int ok = 1, any = 0;
			for (int j = i + 1; j < g->n_nodes && ok; j++)
				for (int k = 0; k < g->nodes[j].n_inputs; k++)
					if (g->nodes[j].inputs[k] == nd->output) {
						any = 1;
						if (g->nodes[j].op != SAM3_OP_MATMUL || k != 1)
							ok = 0;
					}
			if (ok && any)
				m->flags[i] |= F_LAZY_T | F_SKIP;
		}
		if (nd->op == SAM3_OP_MATMUL && nd->inputs[1] && nd->inputs[1]->n_dims <= 2 &&
		    count_uses(g, i + 1, nd->output) == 1) {
			for (int j = i + 1; j < g->n_nodes; j++) {
				struct sam3_node *ad = &g->nodes[j];
				if (ad->op != SAM3_OP_ADD || ad->inputs[0] != nd->output)
					continue;
				struct sam3_tensor *b = ad->inputs[1];
				int N = nd->output->dims[nd->output->n_dims - 1];
				if (b && nelems(b) == N && N > 1 && (N % 8) == 0 &&
				    b->dtype == nd->output->dtype) {
					m->flags[i] |= F_BIAS_FUSED;
					m->flags[j] |= F_SKIP;
					if (count_uses(g, j + 1, ad->output) == 1) {
						for (int k = j + 1; k < g->n_nodes; k++)
							if (g->nodes[k].op == SAM3_OP_GELU &&
							    g->nodes[k].inputs[0] == ad->output) {
								m->flags[j] |= F_GELU_FUSED;
								m->flags[k] |= F_SKIP;
								break;
							}
					}
					/* F32 x + linear(...) (the residual ADDs after proj
					 * and fc2, image_encoder.c:793-900): the GEMM adds
					 * into a copy of x in place (reduce-add epilogue) */
					int r = res_partner(g, i, j);
					if (!(m->flags[j] & F_GELU_FUSED) && r > 0) {
						m->flags[j] |= F_RES_FUSED;
						m->flags[r] |= F_SKIP;
					}
				}
				break;
			}
		}
	}
}

static enum sam3_error cu_graph_eval(struct sam3_backend *be,
				     struct sam3_graph *g)
{
	struct impl *m = IM(be);
	enum sam3_error err = SAM3_OK;
	if (!g || g->n_nodes < 0)
		return SAM3_EINVAL;
	if (g->n_nodes > m->nflags) {
		int *f = realloc(m->flags, sizeof(int) * (size_t)g->n_nodes);
		if (!f)
			return SAM3_ENOMEM;
		m->flags = f;
		m->nflags = g->n_nodes;
	}
	plan(m, g);
	m->g = g;
	double t_eval0 = m->prof ? now_s() : 0.0;
	for (int i = 0; i < g->n_nodes; i++) {
		if (m->flags[i] & F_SKIP)
			continue;
		double t0 = 0.0;
		if (m->prof) {
			sam3cu_stream_sync(m->stream);
			t0 = now_s();
		}
		err = op_node(m, g, i);
		if (m->prof) {
			int op = g->nodes[i].op;
			sam3cu_stream_sync(m->stream);
			if (op >= 0 && op < SAM3_OP_COUNT) {
				m->prof_s[op] += now_s() - t0;
				m->prof_n[op]++;
			}
		}
		if (err != SAM3_OK) {
			fprintf(stderr, "[sam3cu] graph_eval: node %d (op=%d) failed (%d)\n", i,
				(int)g->nodes[i].op, (int)err);
			break;
		}
	}
	double t_rb0 = m->prof ? now_s() : 0.0;
	/* outputs nobody in this graph consumes go back to host (or stay
	 * resident); a fused MATMUL's result is its ADD / GELU node's output */
	for (int i = 0; err == SAM3_OK && i < g->n_nodes; i++) {
		struct sam3_tensor *t = g->nodes[i].output;
		if (m->flags[i] & (F_BIAS_FUSED | F_GELU_FUSED))
			continue;  /* the fused chain's last node holds the result */
		if ((m->flags[i] & F_SKIP) && g->nodes[i].op == SAM3_OP_TRANSPOSE)
			continue;
		if (count_uses(g, i + 1, t))
			continue;
		struct devent *e = map_find(m, t);
		if (!e)
			continue;
		void *d;
		if ((err = dev_of(m, t, 1, &d)) != SAM3_OK)  /* views made contiguous */
			break;
		if (g->no_readback) {
			if (!e->own) {  /* an alias of arena memory: copy it out */
				void *keep;
				if (sam3cu_dev_alloc(&keep, e->nbytes) != 0) {
					err = SAM3_ENOMEM;
					break;
				}
				sam3cu_memcpy_d2d(keep, e->dptr, e->nbytes, m->stream);
				e->dptr = keep;
			}
			e->kind = 1;  /* keep resident for the next graph */
			e->own = 0;
			e->data = t->data;
		} else if (t->data) {
			int rc = m->hx ? hxfer_d2h(m->hx, t->data, e->dptr, tbytes(t), m->stream)
				       : sam3cu_memcpy_d2h(t->data, e->dptr, tbytes(t), m->stream);
			if (rc != 0)
				err = SAM3_EBACKEND;
			m->prof_b[1] += (double)tbytes(t);
			if (m->prof > 1)
				fprintf(stderr, "[sam3cu profile] read back node %d op %d dims %d,%d,%d,%d (%zu B)\n",
					i, (int)g->nodes[i].op, t->dims[0], t->n_dims > 1 ? t->dims[1] : 0,
					t->n_dims > 2 ? t->dims[2] : 0, t->n_dims > 3 ? t->dims[3] : 0, tbytes(t));
		}
	}
	if (sam3cu_stream_sync(m->stream) != 0 && err == SAM3_OK)
		err = SAM3_EBACKEND;
	if (err == SAM3_OK && sam3cu_last_device_error() != 0)
		err = SAM3_EBACKEND;
	if (m->prof) {
		double t1 = now_s();
		m->prof_s[SAM3_OP_COUNT] += t1 - t_rb0;
		m->prof_n[SAM3_OP_COUNT]++;
		m->prof_s[SAM3_OP_COUNT + 1] += t1 - t_eval0;
		m->prof_n[SAM3_OP_COUNT + 1]++;
	}
	m->g = NULL;
	tmp_free_all(m);
	map_drop_local(m);
	return err;
}

static const struct sam3_backend_ops cuda_ops = {
	.init             = cu_init,
	.free             = cu_free,
	.alloc_tensor     = cu_alloc_tensor,
	.graph_eval       = cu_graph_eval,
	.arena_reset      = cu_arena_reset,
	.cache_invalidate = cu_cache_invalidate,
};

const struct sam3_backend_ops *sam3_cuda_backend_ops(void)
{
	return &cuda_ops;
}
