/*
 * host_xfer.c - host <-> device copies of the caller's pageable buffers.
 *
 * The reference's encoder hands a non-Metal backend host tensors: the
 * residual stream comes in and goes out through t->data at every graph
 * (image_encoder.c:775-920), 21 MB each way per graph at 1008 px.  A plain
 * cudaMemcpyAsync from pageable memory is staged by the driver through one
 * thread.  Here large copies go through a page-locked staging buffer owned
 * by the backend, in 4 MiB chunks: the pageable side is copied by a small
 * pool of host threads, and the DMA of one chunk overlaps the host copy of
 * the next.  Small copies (< 1 MiB) take the plain path.
 *
 * SAM3CU_XFER_THREADS sets the pool size (default: the online CPUs, at most
 * 8; the variable allows up to 16; 1 = no pool, plain cudaMemcpyAsync for
 * every size).
 */
#include "host_xfer.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "../../include/sam3cu.h"

#define HX_CHUNK   ((size_t)4 << 20)
#define HX_SMALL   ((size_t)1 << 20)
#define HX_MAXEV   64
#define HX_MAXT    16

struct hxjob {
	char       *dst;
	const char *src;
	size_t      n;
};

struct hxfer {
	int              nthreads;       /* workers + the calling thread */
	pthread_t        tid[HX_MAXT];
	pthread_mutex_t  mu;
	pthread_cond_t   cv_go, cv_done;
	unsigned long    gen;            /* job generation */
	int              pending;        /* workers still copying */
	int              quit;
	struct hxjob     job;
	void            *stage;          /* page-locked */
	size_t           cap;
	void            *ev[HX_MAXEV];
	void            *ev_last;        /* last DMA that read / wrote the stage */
	int              stage_busy;
};

static void slice(const struct hxjob *j, int i, int n, char **d, const char **s, size_t *len)
{
	size_t per = (j->n / (size_t)n + 63) & ~(size_t)63;
	size_t lo = per * (size_t)i;
	size_t hi = lo + per;
	if (lo > j->n)
		lo = j->n;
	if (hi > j->n)
		hi = j->n;
	*d = j->dst + lo;
	*s = j->src + lo;
	*len = hi - lo;
}

static void *worker(void *arg)
{
	struct hxfer *x = arg;
	int me;
	unsigned long seen = 0;
	pthread_mutex_lock(&x->mu);
	for (me = 0; me < x->nthreads - 1 && !pthread_equal(x->tid[me], pthread_self()); me++)
		;
	for (;;) {
		while (x->gen == seen && !x->quit)
			pthread_cond_wait(&x->cv_go, &x->mu);
		if (x->quit)
			break;
		seen = x->gen;
		struct hxjob j = x->job;
		pthread_mutex_unlock(&x->mu);
		char *d;
		const char *s;
		size_t len;
		slice(&j, me + 1, x->nthreads, &d, &s, &len);
		if (len)
			memcpy(d, s, len);
		pthread_mutex_lock(&x->mu);
		if (--x->pending == 0)
			pthread_cond_signal(&x->cv_done);
	}
	pthread_mutex_unlock(&x->mu);
	return NULL;
}

/* dst <- src with every thread of the pool (the caller takes slice 0) */
static void par_memcpy(struct hxfer *x, void *dst, const void *src, size_t n)
{
	if (x->nthreads <= 1 || n < HX_SMALL) {
		memcpy(dst, src, n);
		return;
	}
	pthread_mutex_lock(&x->mu);
	x->job.dst = dst;
	x->job.src = src;
	x->job.n = n;
	x->pending = x->nthreads - 1;
	x->gen++;
	pthread_cond_broadcast(&x->cv_go);
	pthread_mutex_unlock(&x->mu);
	char *d;
	const char *s;
	size_t len;
	slice(&x->job, 0, x->nthreads, &d, &s, &len);
	if (len)
		memcpy(d, s, len);
	pthread_mutex_lock(&x->mu);
	while (x->pending)
		pthread_cond_wait(&x->cv_done, &x->mu);
	pthread_mutex_unlock(&x->mu);
}

struct hxfer *hxfer_create(void)
{
	struct hxfer *x = calloc(1, sizeof(*x));
	if (!x)
		return NULL;
	long ncpu = sysconf(_SC_NPROCESSORS_ONLN);
	int nt = ncpu > 0 ? (int)(ncpu < 8 ? ncpu : 8) : 1;
	const char *e = getenv("SAM3CU_XFER_THREADS");
	if (e && atoi(e) > 0)
		nt = atoi(e) < HX_MAXT ? atoi(e) : HX_MAXT;
	x->nthreads = nt;
	pthread_mutex_init(&x->mu, NULL);
	pthread_cond_init(&x->cv_go, NULL);
	pthread_cond_init(&x->cv_done, NULL);
	for (int i = 0; i < HX_MAXEV; i++)
		if (sam3cu_event_create(&x->ev[i]) != 0) {
			hxfer_destroy(x);
			return NULL;
		}
	pthread_mutex_lock(&x->mu);  /* workers find their index once tid[] is filled */
	int started = 0;
	for (int i = 0; i < nt - 1; i++) {
		if (pthread_create(&x->tid[i], NULL, worker, x) != 0)
			break;
		started++;
	}
	x->nthreads = started + 1;
	pthread_mutex_unlock(&x->mu);
	return x;
}

void hxfer_destroy(struct hxfer *x)
{
	if (!x)
		return;
	pthread_mutex_lock(&x->mu);
	x->quit = 1;
	pthread_cond_broadcast(&x->cv_go);
	pthread_mutex_unlock(&x->mu);
	for (int i = 0; i < x->nthreads - 1; i++)
		pthread_join(x->tid[i], NULL);
	if (x->stage_busy)
		sam3cu_event_sync(x->ev_last);
	if (x->stage)
		sam3cu_host_free_pinned(x->stage);
	for (int i = 0; i < HX_MAXEV; i++)
		if (x->ev[i])
			sam3cu_event_destroy(x->ev[i]);
	pthread_mutex_destroy(&x->mu);
	pthread_cond_destroy(&x->cv_go);
	pthread_cond_destroy(&x->cv_done);
	free(x);
}

/* a staging buffer of n bytes that no DMA uses any more */
static int stage_for(struct hxfer *x, size_t n)
{
	if (x->stage_busy) {
		if (sam3cu_event_sync(x->ev_last) != 0)
			return SAM3CU_ECUDA;
		x->stage_busy = 0;
	}
	if (n <= x->cap)
		return 0;
	if (x->stage)
		sam3cu_host_free_pinned(x->stage);
	x->stage = NULL;
	x->cap = 0;
	size_t c = (n + HX_CHUNK - 1) / HX_CHUNK * HX_CHUNK;
	if (sam3cu_host_alloc_pinned(&x->stage, c) != 0) {
		x->stage = NULL;
		return SAM3CU_ENOMEM;
	}
	x->cap = c;
	return 0;
}

static int plain(size_t n, struct hxfer *x)
{
	return x->nthreads <= 1 || n < HX_SMALL || n > HX_CHUNK * HX_MAXEV;
}

int hxfer_h2d(struct hxfer *x, void *dev, const void *host, size_t n, void *stream)
{
	if (plain(n, x))
		return sam3cu_memcpy_h2d(dev, host, n, stream);
	int rc = stage_for(x, n);
	if (rc)
		return sam3cu_memcpy_h2d(dev, host, n, stream);
	for (size_t off = 0; off < n; off += HX_CHUNK) {
		size_t len = n - off < HX_CHUNK ? n - off : HX_CHUNK;
		/* this chunk's host copy overlaps the previous chunk's DMA */
		par_memcpy(x, (char *)x->stage + off, (const char *)host + off, len);
		if ((rc = sam3cu_memcpy_h2d((char *)dev + off, (char *)x->stage + off, len, stream)))
			return rc;
	}
	x->ev_last = x->ev[0];
	x->stage_busy = 1;
	return sam3cu_event_record(x->ev_last, stream);
}

int hxfer_d2h(struct hxfer *x, void *host, const void *dev, size_t n, void *stream)
{
	if (plain(n, x)) {
		int rc = sam3cu_memcpy_d2h(host, dev, n, stream);
		return rc ? rc : sam3cu_stream_sync(stream);
	}
	int rc = stage_for(x, n);
	if (rc) {
		rc = sam3cu_memcpy_d2h(host, dev, n, stream);
		return rc ? rc : sam3cu_stream_sync(stream);
	}
	int k = 0;
	for (size_t off = 0; off < n; off += HX_CHUNK, k++) {
		size_t len = n - off < HX_CHUNK ? n - off : HX_CHUNK;
		if ((rc = sam3cu_memcpy_d2h((char *)x->stage + off, (const char *)dev + off, len, stream)) ||
		    (rc = sam3cu_event_record(x->ev[k], stream)))
			return rc;
	}
	k = 0;
	for (size_t off = 0; off < n; off += HX_CHUNK, k++) {
		size_t len = n - off < HX_CHUNK ? n - off : HX_CHUNK;
		/* this chunk's host copy overlaps the next chunk's DMA */
		if ((rc = sam3cu_event_sync(x->ev[k])))
			return rc;
		par_memcpy(x, (char *)host + off, (const char *)x->stage + off, len);
	}
	return 0;
}
