/* ref_harness.c -- TEST INFRASTRUCTURE: exposes the reference's own kernels
 * (runtime/tg_rt.h) and quantizer (src/quant.c, whose helpers are static, so
 * the file is included here) behind plain functions, for the oracle's parity
 * pin. Compiled by oracle/Makefile against the reference sources where they
 * lie; the result, oracle/_ref/libtgref.so, is never part of the product. */
#define _GNU_SOURCE /* dup, dup2 */
#include "quant.c"
#include "tg_rt.h"

#include <fcntl.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

void ref_matmul(float *o, const float *a, const float *b, int m, int k, int n) { tg_matmul(o, a, b, m, k, n); }
void ref_matmul_qa(float *o, const signed char *q, int bits, const float *s, const float *b, int m, int k, int n)
{
	tg_matmul_qa(o, q, bits, s, b, m, k, n);
}
void ref_matmul_qb(float *o, const float *a, const signed char *q, int bits, const float *s, int m, int k, int n)
{
	tg_matmul_qb(o, a, q, bits, s, m, k, n);
}
void ref_rmsnorm(float *o, const float *a, int rows, int cols) { tg_rmsnorm(o, a, rows, cols); }
void ref_softmax(float *o, const float *a, int rows, int cols) { tg_softmax(o, a, rows, cols); }
int ref_qget(const signed char *q, int bits, int i) { return tg_qget(q, bits, i); }

/* quantize_param (src/quant.c:258-316) on a one-param module. H: K x K or NULL (RTN). */
int ref_quantize(const float *w, int rows, int cols, int axis, int bits, const double *H, signed char *q, float *s)
{
	Module *m = mod_new("harness");
	Shape sh = { 2, { rows, cols } };
	int v = mod_value(m, V_PARAM, &sh, "w");
	size_t n = (size_t)rows * (size_t)cols;
	m->val[v].data = xmalloc(n * sizeof(float));
	memcpy(m->val[v].data, w, n * sizeof(float));
	QP qp;
	memset(&qp, 0, sizeof qp);
	qp.v = v;
	qp.axis = axis;
	qp.C = sh.dim[axis];
	qp.K = sh.dim[1 - axis];
	if (H) {
		qp.H = xmalloc((size_t)qp.K * (size_t)qp.K * sizeof(double));
		memcpy(qp.H, H, (size_t)qp.K * (size_t)qp.K * sizeof(double));
		qp.nsamp = 1;
	}
	quantize_param(m, &qp, bits, H != NULL);
	Value *x = &m->val[v];
	memcpy(q, x->q, bits == 8 ? n : (n + 1) / 2);
	memcpy(s, x->qs, (size_t)qp.C * sizeof(float));
	return 0;
}

/* ---- the reference's own VM on a program file, timed (bench.py's reference arm) ----------
 *
 * ref_vm_load loads PATH the way `tgc` does (load_module: the surface program with its
 * file() weights, then plan) and quantizes every eligible param as `tgc quantize --bits
 * BITS --min-size MIN_SIZE [--method gptq]` would (eligible() and quantize_param() of
 * src/quant.c). With gptq, a param of input width K <= 2048 gets the Hessian of NCAL
 * seeded N(0,1) rows of width K -- the synthetic calibration the benchmark configs name,
 * shared by every param of that width -- where calibrate() would collect the program's
 * own activations. BITS 0 leaves the program f32. Returns the module.
 *
 * ref_vm_run runs ROWS rows through vm_run_into REPS times the way `tgc batch -j auto`
 * does: par_init(0) (one worker per online CPU), par_for over the rows with one arena
 * per thread (src/main.c:216-242,421-441). sec[r] gets the wall time of repetition r.
 * Returns the thread count. The row values are seeded uniform numbers in [-1, 1): the
 * kernels' time does not depend on them. */
typedef struct {
	const Module *m;
	const float *all;
	int per, n, nt, afl;
	float *out, *arenas;
	int *steps;
	const float **inptrs;
} HJob;

static void h_rows(void *ctx, int lo, int hi, int tid)
{
	HJob *j = ctx;
	const Module *m = j->m;
	const float **in = j->inptrs + (size_t)tid * (size_t)(m->ninputs ? m->ninputs : 1);
	float *arena = j->arenas + (size_t)tid * (size_t)j->afl;
	for (int r = lo; r < hi; r++) {
		const float *row = j->all + (size_t)r * (size_t)j->per;
		for (int i = 0, o = 0; i < m->ninputs; i++) {
			in[i] = row + o;
			o += shape_numel(&m->val[m->inputs[i]].sh);
		}
		vm_run_into(m, in, j->out + (size_t)r * (size_t)j->n, j->steps + (size_t)r * (size_t)j->nt, arena, NULL);
	}
}

static unsigned h_state;
static double h_uniform(void) /* xorshift32 in (0, 1) */
{
	h_state ^= h_state << 13;
	h_state ^= h_state >> 17;
	h_state ^= h_state << 5;
	return ((h_state >> 8) + 0.5) / 16777216.0;
}
static double h_normal(void) /* Box-Muller */
{
	return sqrt(-2.0 * log(h_uniform())) * cos(6.283185307179586 * h_uniform());
}

/* X^T X of ncal seeded N(0,1) rows of width K (cached per K) */
static const double *h_hessian(int K, int ncal)
{
	static double *cache[8];
	static int ck[8], cn[8], nc;
	for (int i = 0; i < nc; i++)
		if (ck[i] == K && cn[i] == ncal) return cache[i];
	double *H = calloc((size_t)K * (size_t)K, sizeof(double)), *x = xmalloc((size_t)K * sizeof *x);
	h_state = 0x9e3779b9u ^ (unsigned)K;
	for (int r0 = 0; r0 < ncal; r0++) {
		for (int r = 0; r < K; r++) x[r] = h_normal();
		for (int r = 0; r < K; r++)
			for (int c = 0; c < K; c++) H[(size_t)r * K + c] += x[r] * x[c];
	}
	xfree(x);
	if (nc < 8) {
		ck[nc] = K, cn[nc] = ncal, cache[nc] = H;
		nc++;
	}
	return H;
}

typedef struct {
	Module *m;
	QSet *s;
	int bits, gptq, ncal;
} HQuant;

/* quantize_param of params lo..hi-1 (on the calling thread: see ref_vm_load) */
static void h_quant(void *ctx, int lo, int hi, int tid)
{
	(void)tid;
	HQuant *j = ctx;
	for (int i = lo; i < hi; i++) {
		QP *q = &j->s->p[i];
		if (j->gptq && q->K <= 2048) {
			size_t KK = (size_t)q->K * (size_t)q->K;
			q->H = xmalloc(KK * sizeof(double)); /* quantize_param dampens it in place */
			memcpy(q->H, h_hessian(q->K, j->ncal), KK * sizeof(double));
			q->nsamp = j->ncal;
		}
		quantize_param(j->m, q, j->bits, j->gptq);
		xfree(q->H);
		q->H = NULL;
	}
}

void *ref_vm_load(const char *path, int bits, int gptq, int min_size, int ncal)
{
	static int pool;
	if (!pool) {
		par_init(0);
		pool = 1;
	}
	Module *m = load_module(path);
	plan(m);
	if (!bits) return m;
	QSet s = eligible(m, min_size);
	fflush(stderr);
	int keep = dup(2), nul = open("/dev/null", O_WRONLY); /* quantize_param reports each param */
	if (keep >= 0 && nul >= 0) dup2(nul, 2);
	if (gptq) /* the Hessians first, on this thread (the cache is not shared-write safe) */
		for (int i = 0; i < s.n; i++)
			if (s.p[i].K <= 2048) h_hessian(s.p[i].K, ncal);
	HQuant hq = { m, &s, bits, gptq, ncal };
	/* on this thread only: quantize_param allocates through the reference's allocator, whose
	 * block list has no lock (src/util.c:21-75), and par_for workers must not allocate
	 * (src/par.c:11-12); run from workers it corrupted that list now and then, and the
	 * process aborted while stderr pointed at /dev/null */
	h_quant(&hq, 0, s.n, 0);
	fflush(stderr);
	if (keep >= 0 && nul >= 0) dup2(keep, 2);
	if (keep >= 0) close(keep);
	if (nul >= 0) close(nul);
	xfree(s.p);
	return m;
}

int ref_vm_run(void *mod, int rows, int reps, double *sec)
{
	const Module *m = mod;
	int per = 0;
	for (int i = 0; i < m->ninputs; i++) per += shape_numel(&m->val[m->inputs[i]].sh);
	int threads = par_threads(), n = shape_numel(&m->val[m->output].sh), nt = m->nthink ? m->nthink : 1;
	int afl = m->arena ? m->arena : 1;
	HJob j = { m, NULL, per, n, nt, afl, NULL, NULL, NULL, NULL };
	float *all = xmalloc((size_t)rows * (size_t)per * sizeof(float));
	h_state = 0x2545f491u;
	for (size_t i = 0; i < (size_t)rows * (size_t)per; i++) all[i] = (float)(2.0 * h_uniform() - 1.0);
	j.all = all;
	j.out = xmalloc((size_t)rows * (size_t)n * sizeof(float));
	j.steps = xmalloc((size_t)rows * (size_t)nt * sizeof(int));
	j.arenas = xmalloc((size_t)threads * (size_t)afl * sizeof(float));
	j.inptrs = xmalloc((size_t)threads * (size_t)(m->ninputs ? m->ninputs : 1) * sizeof(float *));
	for (int r = 0; r < reps; r++) {
		double t0 = tr_now_ms();
		par_for(rows, 1, h_rows, &j);
		sec[r] = (tr_now_ms() - t0) / 1e3;
	}
	xfree(all);
	xfree(j.out);
	xfree(j.steps);
	xfree(j.arenas);
	xfree(j.inptrs);
	return threads;
}
