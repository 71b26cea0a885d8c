/* tgo_mt.c -- CPU oracle, threaded and vectorised (TEST INFRASTRUCTURE ONLY; see tgo.h).
 *
 * The same arithmetic as tgo.c's tgo_matmul_qb and tgo_lm_forward, bit for bit,
 * fast enough to check the decoder at its full Qwen3-0.6B shape (a 1024-token
 * forward is about 1 TFLOP; the scalar restatement needs ~20 minutes a sequence).
 *
 * Why the results are identical: every output of the reference's matmuls is one
 * f32 accumulator that starts at 0 and adds its k products in order p = 0..k-1,
 * each product rounded before the add (runtime/tg_rt.h:81-151; no contraction:
 * this file is compiled with -ffp-contract=off like the reference). Here several
 * such accumulators sit side by side in a vector register and advance together
 * over p -- each lane still rounds the same product and the same sum in the same
 * order, so vectorising across outputs (columns j, or keys, or head_dim) changes
 * nothing. Threads split independent outputs (rows and column blocks), never one
 * sum. Elementwise steps (rmsnorm, softmax, silu, the residual adds, the ordered
 * sum of the heads' outputs) run as in tgo.c, only partitioned by rows.
 *
 * Two shortcuts, both exact: the causal mask's -1e9 entries (import.py:85) are not
 * computed. Each such score is dot*scale - 1e9, whose exp after subtracting the
 * row's maximum (an unmasked score, since every row keeps position 0) is exactly
 * +0 in f32; +0 leaves the softmax sum unchanged, and the P.V sum then adds
 * 0*v = +-0 to a running sum, which leaves it unchanged too. And the LM head is
 * applied to the last position only: take(logits, lastidx) discards the other
 * rows, whose values never reach the output.
 *
 * The vector kernels are compiled for AVX-512, AVX2 and plain x86-64 and the
 * loader picks one per CPU (target_clones); all three compute the same bits. */
#define _GNU_SOURCE /* sysconf */
#include "tgo.h"

#include <math.h>
#include <pthread.h>
#include <unistd.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#define VEC_CLONES __attribute__((target_clones("avx512f", "avx2", "default")))

typedef float v8 __attribute__((vector_size(32)));

/* n floats, 64-byte aligned (every buffer a vector kernel reads through a v8 pointer) */
static float *falloc(size_t n)
{
	return aligned_alloc(64, (n * sizeof(float) + 63) / 64 * 64);
}

/* ---- a minimal thread pool: fn(ctx, item) for items 0..n-1 ------------------------------- */

typedef struct Pool Pool;
typedef void (*item_fn)(void *ctx, long item);

struct Pool {
	int n;
	pthread_t *th;
	pthread_mutex_t mu;
	pthread_cond_t go, done;
	long gen;            /* bumped for every job */
	int quit, busy;      /* busy: workers still inside the current job */
	item_fn fn;
	void *ctx;
	long nitems;
	atomic_long next;
};

static void drain(Pool *p)
{
	for (;;) {
		long i = atomic_fetch_add(&p->next, 1);
		if (i >= p->nitems) return;
		p->fn(p->ctx, i);
	}
}

static void *worker(void *arg)
{
	Pool *p = arg;
	long seen = 0;
	pthread_mutex_lock(&p->mu);
	for (;;) {
		while (!p->quit && p->gen == seen) pthread_cond_wait(&p->go, &p->mu);
		if (p->quit) break;
		seen = p->gen;
		pthread_mutex_unlock(&p->mu);
		drain(p);
		pthread_mutex_lock(&p->mu);
		if (--p->busy == 0) pthread_cond_signal(&p->done);
	}
	pthread_mutex_unlock(&p->mu);
	return NULL;
}

static Pool *pool_new(int threads)
{
	Pool *p = calloc(1, sizeof *p);
	p->n = threads > 1 ? threads - 1 : 0; /* the caller is the last worker */
	pthread_mutex_init(&p->mu, NULL);
	pthread_cond_init(&p->go, NULL);
	pthread_cond_init(&p->done, NULL);
	p->th = calloc((size_t)(p->n ? p->n : 1), sizeof *p->th);
	for (int i = 0; i < p->n; i++) pthread_create(&p->th[i], NULL, worker, p);
	return p;
}

static void pool_for(Pool *p, long nitems, item_fn fn, void *ctx)
{
	if (nitems <= 0) return;
	pthread_mutex_lock(&p->mu);
	p->fn = fn, p->ctx = ctx, p->nitems = nitems;
	atomic_store(&p->next, 0);
	p->busy = p->n;
	p->gen++;
	pthread_cond_broadcast(&p->go);
	pthread_mutex_unlock(&p->mu);
	drain(p);
	pthread_mutex_lock(&p->mu);
	while (p->busy) pthread_cond_wait(&p->done, &p->mu);
	pthread_mutex_unlock(&p->mu);
}

static void pool_free(Pool *p)
{
	pthread_mutex_lock(&p->mu);
	p->quit = 1;
	pthread_cond_broadcast(&p->go);
	pthread_mutex_unlock(&p->mu);
	for (int i = 0; i < p->n; i++) pthread_join(p->th[i], NULL);
	pthread_mutex_destroy(&p->mu);
	pthread_cond_destroy(&p->go);
	pthread_cond_destroy(&p->done);
	free(p->th);
	free(p);
}

static int default_threads(int threads)
{
	if (threads > 0) return threads;
	long n = sysconf(_SC_NPROCESSORS_ONLN);
	return n > 0 ? (int)n : 1;
}

/* ---- the column-block kernel ---------------------------------------------------------------- */

#define JB 32 /* output columns per block: four 8-lane accumulators per row */

/* o[r, c] = sum_p x[r, p] * w[p, c] (p = 0..K-1 in order), for rows r of x (row stride ldx)
 * and the JB columns of the panel w (row stride ldw, 32-byte aligned rows). The sums are
 * returned raw in acc rows of JB floats. */
VEC_CLONES static void panel_dot(float *acc, const float *x, long ldx, int rows, const float *w, long ldw, int K)
{
	int r = 0;
	for (; r + 4 <= rows; r += 4) {
		const float *x0 = x + (long)r * ldx, *x1 = x0 + ldx, *x2 = x1 + ldx, *x3 = x2 + ldx;
		v8 a00 = { 0 }, a01 = { 0 }, a02 = { 0 }, a03 = { 0 }, a10 = { 0 }, a11 = { 0 }, a12 = { 0 }, a13 = { 0 };
		v8 a20 = { 0 }, a21 = { 0 }, a22 = { 0 }, a23 = { 0 }, a30 = { 0 }, a31 = { 0 }, a32 = { 0 }, a33 = { 0 };
		for (int p = 0; p < K; p++) {
			const v8 *wp = (const v8 *)(w + (long)p * ldw);
			const v8 w0 = wp[0], w1 = wp[1], w2 = wp[2], w3 = wp[3];
			const float s0 = x0[p], s1 = x1[p], s2 = x2[p], s3 = x3[p];
			a00 += s0 * w0, a01 += s0 * w1, a02 += s0 * w2, a03 += s0 * w3;
			a10 += s1 * w0, a11 += s1 * w1, a12 += s1 * w2, a13 += s1 * w3;
			a20 += s2 * w0, a21 += s2 * w1, a22 += s2 * w2, a23 += s2 * w3;
			a30 += s3 * w0, a31 += s3 * w1, a32 += s3 * w2, a33 += s3 * w3;
		}
		v8 *o = (v8 *)(acc + (long)r * JB);
		o[0] = a00, o[1] = a01, o[2] = a02, o[3] = a03, o[4] = a10, o[5] = a11, o[6] = a12, o[7] = a13;
		o[8] = a20, o[9] = a21, o[10] = a22, o[11] = a23, o[12] = a30, o[13] = a31, o[14] = a32, o[15] = a33;
	}
	for (; r < rows; r++) {
		const float *x0 = x + (long)r * ldx;
		v8 a0 = { 0 }, a1 = { 0 }, a2 = { 0 }, a3 = { 0 };
		for (int p = 0; p < K; p++) {
			const v8 *wp = (const v8 *)(w + (long)p * ldw);
			const float s0 = x0[p];
			a0 += s0 * wp[0], a1 += s0 * wp[1], a2 += s0 * wp[2], a3 += s0 * wp[3];
		}
		v8 *o = (v8 *)(acc + (long)r * JB);
		o[0] = a0, o[1] = a1, o[2] = a2, o[3] = a3;
	}
}

/* acc[c] += pv[s] * v[s, c] for s = 0..n-1 in order, c over 128 head_dim lanes (one row). */
VEC_CLONES static void pv_row(float *out, const float *pv, const float *v, int n)
{
	v8 a[16];
	for (int c = 0; c < 16; c++) a[c] = (v8){ 0 };
	for (int s = 0; s < n; s++) {
		const v8 *vs = (const v8 *)(v + (long)s * 128);
		const float w = pv[s];
		for (int c = 0; c < 16; c++) a[c] += w * vs[c];
	}
	for (int c = 0; c < 16; c++) memcpy(out + 8 * c, &a[c], 32);
}

/* Code i of a quantized param: int8 one per byte; int4 element i in byte i/2, low nibble
 * first, sign-extended (runtime/tg_rt.h:124-129; tgo_qget inlined). */
static inline int code_at(const signed char *q, int bits, long i)
{
	if (bits == 8) return q[i];
	int byte = q[i >> 1];
	return (i & 1) ? byte >> 4 : (int)(signed char)(unsigned char)((unsigned)byte << 4) >> 4;
}

/* Codes [p0, p0+K) x [j0, j0+nj) of a quantized [*, N] matrix as f32 in a JB-wide panel
 * (columns beyond nj are zero). */
static void fill_panel(float *w, const signed char *q, int bits, long N, long p0, int K, long j0, int nj)
{
	for (int p = 0; p < K; p++) {
		float *row = w + (long)p * JB;
		long base = (p0 + p) * N + j0;
		for (int c = 0; c < nj; c++) row[c] = (float)code_at(q, bits, base + c);
		for (int c = nj; c < JB; c++) row[c] = 0.0f;
	}
}

/* ---- x @ Q with per-column scales, threaded over (column block, row chunk) --------------- */

#define ROWCHUNK 256

typedef struct {
	float *o;
	long ldo;
	const float *x;
	long ldx;
	int m, K;
	const signed char *q;
	int bits;
	long N, p0; /* code rows p0..p0+K-1 of the [*, N] matrix */
	int ncol;   /* columns computed: 0..ncol-1 */
	const float *s;
} QbJob;

static void qb_item(void *ctx, long item)
{
	const QbJob *j = ctx;
	int nchunk = (j->m + ROWCHUNK - 1) / ROWCHUNK;
	long cb = item / nchunk;
	int r0 = (int)(item % nchunk) * ROWCHUNK, rows = j->m - r0 < ROWCHUNK ? j->m - r0 : ROWCHUNK;
	long j0 = cb * JB;
	int nj = j->ncol - j0 < JB ? (int)(j->ncol - j0) : JB;
	float *w = falloc((size_t)j->K * JB), *acc = falloc((size_t)ROWCHUNK * JB);
	fill_panel(w, j->q, j->bits, j->N, j->p0, j->K, j0, nj);
	panel_dot(acc, j->x + (long)r0 * j->ldx, j->ldx, rows, w, JB, j->K);
	for (int r = 0; r < rows; r++)
		for (int c = 0; c < nj; c++) j->o[(long)(r0 + r) * j->ldo + j0 + c] = j->s[j0 + c] * acc[(long)r * JB + c];
	free(w);
	free(acc);
}

static void qb_run(Pool *pool, float *o, long ldo, const float *x, long ldx, int m, int K, const signed char *q, int bits,
		   long N, long p0, int ncol, const float *s)
{
	QbJob j = { o, ldo, x, ldx, m, K, q, bits, N, p0, ncol, s };
	long nitems = (long)((ncol + JB - 1) / JB) * ((m + ROWCHUNK - 1) / ROWCHUNK);
	pool_for(pool, nitems, qb_item, &j);
}

void tgo_matmul_qb_mt(float *o, const float *a, const signed char *q, int bits, const float *s, int m, int k, int n,
		      int threads)
{
	Pool *p = pool_new(default_threads(threads));
	qb_run(p, o, n, a, k, m, k, q, bits, n, 0, n, s);
	pool_free(p);
}

/* ---- the Qwen3 program (import.py:90-132), as tgo_lm_forward ----------------------------- */

typedef struct {
	const tg_cuda_lm_desc *d;
	int T, Tp; /* Tp: T rounded up to JB (the transposed keys' row stride) */
	float *h, *n, *k, *kt, *v, *q, *sv, *oh, *acc, *g, *u, *m, *cosT, *sinT;
	int l;
} Lm;

static void rowmul1(float *x, const float *w, int cols)
{
	for (int i = 0; i < cols; i++) x[i] = x[i] * w[i];
}

static void rotary1(float *v, const float *cs, const float *sn, int HD)
{
	float r[256];
	for (int i = 0; i < HD / 2; i++) {
		r[i] = -v[i + HD / 2];
		r[i + HD / 2] = v[i];
	}
	for (int i = 0; i < HD; i++) {
		float a = v[i] * cs[i], b = r[i] * sn[i];
		v[i] = a + b;
	}
}

/* n = rmsnorm(h) * w, row t */
static void norm_item(void *ctx, long t)
{
	Lm *c = ctx;
	int D = c->d->hidden;
	const float *w = c->l < 0 ? c->d->final_norm : (c->l & 1 ? c->d->ln2[c->l >> 1] : c->d->ln1[c->l >> 1]);
	tgo_rmsnorm(c->n + t * D, c->h + t * D, 1, D);
	rowmul1(c->n + t * D, w, D);
}

/* k rows: rmsnorm * kn, rotary; then the transposed copy kt[head][p][t] */
static void kpost_item(void *ctx, long t)
{
	Lm *c = ctx;
	const tg_cuda_lm_desc *d = c->d;
	int HD = d->head_dim, NKV = d->nkv, L = c->l;
	for (int j = 0; j < NKV; j++) {
		float *x = c->k + ((long)j * c->T + t) * HD;
		tgo_rmsnorm(x, x, 1, HD);
		rowmul1(x, d->kn[L], HD);
		rotary1(x, c->cosT + t * HD, c->sinT + t * HD, HD);
		for (int p = 0; p < HD; p++) c->kt[((long)j * HD + p) * c->Tp + t] = x[p];
	}
}

static void qpost_item(void *ctx, long t)
{
	Lm *c = ctx;
	const tg_cuda_lm_desc *d = c->d;
	int HD = d->head_dim, NQ = d->nq, L = c->l;
	for (int hh = 0; hh < NQ; hh++) {
		float *x = c->q + ((long)hh * c->T + t) * HD;
		tgo_rmsnorm(x, x, 1, HD);
		rowmul1(x, d->qn[L], HD);
		rotary1(x, c->cosT + t * HD, c->sinT + t * HD, HD);
	}
}

/* Attention of query head hh over rows [r0, r0+16): softmax((q k^T) * scale + mask) @ v */
#define ATT_ROWS 16
static void attn_item(void *ctx, long item)
{
	Lm *c = ctx;
	const tg_cuda_lm_desc *d = c->d;
	int HD = d->head_dim, T = c->T, grp = d->nq / d->nkv;
	int nblk = (T + ATT_ROWS - 1) / ATT_ROWS;
	int hh = (int)(item / nblk), r0 = (int)(item % nblk) * ATT_ROWS;
	int rows = T - r0 < ATT_ROWS ? T - r0 : ATT_ROWS;
	int j = hh / grp;
	const float *q = c->q + (long)hh * T * HD, *kt = c->kt + (long)j * HD * c->Tp, *v = c->v + (long)j * T * HD;
	int ncols = r0 + rows; /* keys 0 .. r0+rows-1 cover every row of the block */
	int nkb = (ncols + JB - 1) / JB;
	float *sc = falloc((size_t)ATT_ROWS * nkb * JB), *acc = falloc((size_t)ATT_ROWS * JB);
	for (int kb = 0; kb < nkb; kb++) {
		panel_dot(acc, q + (long)r0 * HD, HD, rows, kt + (long)kb * JB, c->Tp, HD);
		for (int r = 0; r < rows; r++) memcpy(sc + ((long)r * nkb + kb) * JB, acc + (long)r * JB, JB * sizeof(float));
	}
	for (int r = 0; r < rows; r++) {
		int t = r0 + r, n = t + 1;
		float *x = sc + (long)r * nkb * JB;
		for (int s2 = 0; s2 < n; s2++) x[s2] = x[s2] * d->attn_scale + 0.0f;
		/* tg_softmax over the kept keys (runtime/tg_rt.h:154-164) */
		float mx = x[0], sum = 0.0f;
		for (int i = 1; i < n; i++)
			if (x[i] > mx) mx = x[i];
		for (int i = 0; i < n; i++) {
			x[i] = expf(x[i] - mx);
			sum += x[i];
		}
		for (int i = 0; i < n; i++) x[i] /= sum;
		pv_row(c->sv + ((long)hh * T + t) * HD, x, v, n);
	}
	free(sc);
	free(acc);
}

/* acc = o_0 + o_1 + ... (left to right), h += acc, for rows [t, t+1) */
static void headsum_item(void *ctx, long t)
{
	Lm *c = ctx;
	int D = c->d->hidden, NQ = c->d->nq;
	long TD = (long)c->T * D;
	float *h = c->h + t * D;
	for (int i = 0; i < D; i++) {
		float a = c->oh[t * D + i];
		for (int hh = 1; hh < NQ; hh++) a = a + c->oh[hh * TD + t * D + i];
		h[i] = h[i] + a;
	}
}

static void swiglu_item(void *ctx, long t)
{
	Lm *c = ctx;
	int FF = c->d->ffn;
	float *g = c->g + t * FF, *u = c->u + t * FF;
	for (int i = 0; i < FF; i++) g[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

static void resid_item(void *ctx, long t)
{
	Lm *c = ctx;
	int D = c->d->hidden;
	for (int i = 0; i < D; i++) c->h[t * D + i] = c->h[t * D + i] + c->m[t * D + i];
}

int tgo_lm_forward_mt(const tg_cuda_lm_desc *d, const float *ids, int T, float *logits, int threads)
{
	int D = d->hidden, HD = d->head_dim, NQ = d->nq, NKV = d->nkv, FF = d->ffn, V = d->vocab;
	if (HD != 128 || T <= 0) return -1;
	Lm c;
	memset(&c, 0, sizeof c);
	c.d = d, c.T = T, c.Tp = (T + JB - 1) / JB * JB;
	size_t TD = (size_t)T * D;
	c.h = falloc(TD), c.n = falloc(TD), c.m = falloc(TD);
	c.k = falloc((size_t)NKV * T * HD), c.v = falloc((size_t)NKV * T * HD);
	c.kt = falloc((size_t)NKV * HD * c.Tp);
	memset(c.kt, 0, (size_t)NKV * HD * c.Tp * sizeof(float));
	c.q = falloc((size_t)NQ * T * HD), c.sv = falloc((size_t)NQ * T * HD), c.oh = falloc((size_t)NQ * TD);
	c.g = falloc((size_t)T * FF), c.u = falloc((size_t)T * FF);
	c.cosT = falloc((size_t)T * HD), c.sinT = falloc((size_t)T * HD);
	float *qraw = falloc((size_t)T * NQ * HD), *kraw = falloc((size_t)T * NKV * HD), *vraw = falloc((size_t)T * NKV * HD);
	for (int t = 0; t < T; t++) /* RoPE tables as tgo_lm_forward */
		for (int i = 0; i < HD / 2; i++) {
			double inv = pow(d->rope_theta, -((double)(2 * i) / HD)), ang = (double)t * inv;
			c.cosT[(long)t * HD + i] = c.cosT[(long)t * HD + i + HD / 2] = (float)cos(ang);
			c.sinT[(long)t * HD + i] = c.sinT[(long)t * HD + i + HD / 2] = (float)sin(ang);
		}
	for (int t = 0; t < T; t++) { /* h = take(E, ids) */
		float r = floorf(ids[t] + 0.5f);
		int row = r >= 0.0f && r < (float)V ? (int)r : -1;
		for (int i = 0; i < D; i++) c.h[(long)t * D + i] = row >= 0 ? d->embed[(long)row * D + i] : 0.0f;
	}
	Pool *pool = pool_new(default_threads(threads));
	for (int l = 0; l < d->layers; l++) {
		c.l = 2 * l;
		pool_for(pool, T, norm_item, &c);
		/* all kv heads' columns at once: each column is its own sum, as in the per-head params */
		qb_run(pool, kraw, NKV * HD, c.n, D, T, D, d->wk[l].q, d->bits, NKV * HD, 0, NKV * HD, d->wk[l].s);
		qb_run(pool, vraw, NKV * HD, c.n, D, T, D, d->wv[l].q, d->bits, NKV * HD, 0, NKV * HD, d->wv[l].s);
		qb_run(pool, qraw, NQ * HD, c.n, D, T, D, d->wq[l].q, d->bits, NQ * HD, 0, NQ * HD, d->wq[l].s);
		for (int t = 0; t < T; t++) { /* head-major copies */
			for (int j = 0; j < NKV; j++) {
				memcpy(c.k + ((long)j * T + t) * HD, kraw + ((long)t * NKV + j) * HD, HD * sizeof(float));
				memcpy(c.v + ((long)j * T + t) * HD, vraw + ((long)t * NKV + j) * HD, HD * sizeof(float));
			}
			for (int hh = 0; hh < NQ; hh++)
				memcpy(c.q + ((long)hh * T + t) * HD, qraw + ((long)t * NQ + hh) * HD, HD * sizeof(float));
		}
		c.l = l;
		pool_for(pool, T, kpost_item, &c);
		pool_for(pool, T, qpost_item, &c);
		pool_for(pool, (long)NQ * ((T + ATT_ROWS - 1) / ATT_ROWS), attn_item, &c);
		/* o_h = (s @ v) @ Wo_h: rows hh*HD.. of the stacked Wo, per-head column scales */
		for (int hh = 0; hh < NQ; hh++)
			qb_run(pool, c.oh + (long)hh * TD, D, c.sv + (long)hh * T * HD, HD, T, HD, d->wo[l].q, d->bits, D,
			       (long)hh * HD, D, d->wo[l].s + (long)hh * D);
		pool_for(pool, T, headsum_item, &c);
		c.l = 2 * l + 1;
		pool_for(pool, T, norm_item, &c);
		qb_run(pool, c.g, FF, c.n, D, T, D, d->wg[l].q, d->bits, FF, 0, FF, d->wg[l].s);
		qb_run(pool, c.u, FF, c.n, D, T, D, d->wu[l].q, d->bits, FF, 0, FF, d->wu[l].s);
		pool_for(pool, T, swiglu_item, &c);
		qb_run(pool, c.m, D, c.g, FF, T, FF, d->wd[l].q, d->bits, D, 0, D, d->wd[l].s);
		pool_for(pool, T, resid_item, &c);
	}
	/* logits = (rmsnorm(h) * lnf) @ LM; take(logits, lastidx) keeps row T-1 */
	c.l = -1;
	norm_item(&c, T - 1);
	qb_run(pool, logits, V, c.n + (size_t)(T - 1) * D, D, 1, D, d->lm_head.q, d->bits, V, 0, V, d->lm_head.s);
	pool_free(pool);
	free(c.h), free(c.n), free(c.m), free(c.k), free(c.v), free(c.kt), free(c.q), free(c.sv), free(c.oh);
	free(c.g), free(c.u), free(c.cosT), free(c.sinT), free(qraw), free(kraw), free(vraw);
	return 0;
}
