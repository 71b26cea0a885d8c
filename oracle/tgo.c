/* tgo.c -- CPU oracle (TEST INFRASTRUCTURE ONLY; see tgo.h).
 *
 * Restates, in this project's own code, the arithmetic of the reference
 * (IlumCI/Technograd) on the batch path. Each function names the reference
 * lines it follows. Build: oracle/Makefile (-O2 -ffp-contract=off). */
#include "tgo.h"

#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---- kernels: runtime/tg_rt.h ------------------------------------------------ */

/* runtime/tg_rt.h:124-129: int8 one per byte; int4 element i in byte i/2, low
 * nibble first, each nibble sign-extended. */
int tgo_qget(const signed char *q, int bits, long i)
{
	if (bits == 8) return q[i];
	int byte = q[i >> 1];
	if (i & 1) return byte >> 4; /* arithmetic shift of the signed byte */
	return (int)(signed char)(unsigned char)((unsigned)byte << 4) >> 4;
}

/* runtime/tg_rt.h:81-116: every output sums its k products in order p = 0..k-1
 * starting from 0 (the narrow-n specialisations keep that order). */
void tgo_matmul(float *o, const float *a, const float *b, int m, int k, int n)
{
	for (int i = 0; i < m; i++)
		for (int j = 0; j < n; j++) {
			float acc = 0.0f;
			for (int p = 0; p < k; p++) acc += a[(long)i * k + p] * b[(long)p * n + j];
			o[(long)i * n + j] = acc;
		}
}

/* runtime/tg_rt.h:132-140: f32 sum of code * b, then one multiply by the row scale. */
void tgo_matmul_qa(float *o, const signed char *q, int bits, const float *s, const float *b, int m, int k, int n)
{
	for (int i = 0; i < m; i++)
		for (int j = 0; j < n; j++) {
			float acc = 0.0f;
			for (int p = 0; p < k; p++) acc += (float)tgo_qget(q, bits, (long)i * k + p) * b[(long)p * n + j];
			o[(long)i * n + j] = s[i] * acc;
		}
}

/* runtime/tg_rt.h:143-151: column scale after the sum. */
void tgo_matmul_qb(float *o, const float *a, const signed char *q, int bits, const float *s, int m, int k, int n)
{
	for (int i = 0; i < m; i++)
		for (int j = 0; j < n; j++) {
			float acc = 0.0f;
			for (int p = 0; p < k; p++) acc += a[(long)i * k + p] * (float)tgo_qget(q, bits, (long)p * n + j);
			o[(long)i * n + j] = s[j] * acc;
		}
}

/* runtime/tg_rt.h:165-175: eps 1e-6f inside the root, reciprocal then multiply. */
void tgo_rmsnorm(float *o, const float *a, int rows, int cols)
{
	for (int r = 0; r < rows; r++) {
		const float *x = a + (long)r * cols;
		float *y = o + (long)r * cols;
		float ss = 0.0f;
		for (int i = 0; i < cols; i++) ss += x[i] * x[i];
		float inv = 1.0f / sqrtf(ss / (float)cols + 1e-6f);
		for (int i = 0; i < cols; i++) y[i] = x[i] * inv;
	}
}

/* runtime/tg_rt.h:154-164: max-subtract, expf, then a division by the sum. */
void tgo_softmax(float *o, const float *a, int rows, int cols)
{
	for (int r = 0; r < rows; r++) {
		const float *x = a + (long)r * cols;
		float *y = o + (long)r * cols;
		float mx = x[0], sum = 0.0f;
		for (int i = 1; i < cols; i++)
			if (x[i] > mx) mx = x[i];
		for (int i = 0; i < cols; i++) {
			y[i] = expf(x[i] - mx);
			sum += y[i];
		}
		for (int i = 0; i < cols; i++) y[i] /= sum;
	}
}

/* runtime/tg_rt.h:39-75 (and :73-75 step): the same float expressions. */
static float un1(int op, float x)
{
	switch (op) {
	case TG_CUDA_OP_NEG: return -x;
	case TG_CUDA_OP_TANH: return tanhf(x);
	case TG_CUDA_OP_RELU: return x > 0.0f ? x : 0.0f;
	case TG_CUDA_OP_SIGMOID: return 1.0f / (1.0f + expf(-x));
	case TG_CUDA_OP_EXP: return expf(x);
	case TG_CUDA_OP_SQRT: return sqrtf(x);
	case TG_CUDA_OP_GELU: return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
	case TG_CUDA_OP_SILU: return x / (1.0f + expf(-x));
	case TG_CUDA_OP_SOFTPLUS: return (x > 0.0f ? x : 0.0f) + log1pf(expf(-fabsf(x)));
	case TG_CUDA_OP_LOG: return logf(x);
	case TG_CUDA_OP_STEP: return x > 0.0f ? 1.0f : 0.0f;
	case TG_CUDA_OP_SIN: return sinf(x);
	case TG_CUDA_OP_COS: return cosf(x);
	case TG_CUDA_OP_FLOOR: return floorf(x);
	}
	return NAN;
}

void tgo_unary(int op, float *o, const float *a, int n)
{
	for (int i = 0; i < n; i++) o[i] = un1(op, a[i]);
}

static float bin1(int op, float x, float y)
{
	switch (op) {
	case TG_CUDA_OP_ADD: return x + y;
	case TG_CUDA_OP_SUB: return x - y;
	case TG_CUDA_OP_MUL: return x * y;
	case TG_CUDA_OP_DIV: return x / y;
	case TG_CUDA_OP_MAX: return x > y ? x : y; /* runtime/tg_rt.h:34-35 */
	case TG_CUDA_OP_MIN: return x < y ? x : y;
	}
	return NAN;
}

/* ---- rand(seed, scale): src/lower.c:661-668, 766-775 ----------------------------- */
void tgo_rand(unsigned seed, float scale, float *out, long n)
{
	uint32_t s = seed ? seed : 0x9e3779b9u;
	for (long i = 0; i < n; i++) {
		s ^= s << 13;
		s ^= s >> 17;
		s ^= s << 5;
		float u = (float)(s >> 8) / 16777216.0f;
		out[i] = (2.0f * u - 1.0f) * scale;
	}
}

/* ---- quantizer: src/quant.c ------------------------------------------------------ */

/* src/quant.c:176-181 */
static int code_of(double w, double s, int lim)
{
	if (s <= 0) return 0;
	double r = nearbyint(w / s);
	return (int)(r > lim ? lim : r < -lim ? -lim : r);
}

/* src/quant.c:183-200: 10-point clipping grid, first minimum wins. */
static double best_scale(const double *w, int K, const double *hd, int lim)
{
	double amax = 0;
	for (int j = 0; j < K; j++)
		if (fabs(w[j]) > amax) amax = fabs(w[j]);
	if (amax == 0) return 1e-8;
	double best = INFINITY, bs = amax / lim;
	for (int g = 0; g < 10; g++) {
		double s = amax * (1.0 - 0.05 * g) / lim, e = 0;
		for (int j = 0; j < K; j++) {
			double d = w[j] - s * code_of(w[j], s, lim);
			e += d * d * (hd ? hd[j] : 1.0);
		}
		if (e < best) {
			best = e;
			bs = s;
		}
	}
	return bs;
}

/* src/quant.c:202-220: in-place lower Cholesky, upper triangle zeroed. */
static int cholesky(double *A, int n)
{
	for (int j = 0; j < n; j++) {
		double d = A[(long)j * n + j];
		for (int k = 0; k < j; k++) d -= A[(long)j * n + k] * A[(long)j * n + k];
		if (d <= 0) return 0;
		d = sqrt(d);
		A[(long)j * n + j] = d;
		for (int i = j + 1; i < n; i++) {
			double s = A[(long)i * n + j];
			for (int k = 0; k < j; k++) s -= A[(long)i * n + k] * A[(long)j * n + k];
			A[(long)i * n + j] = s / d;
		}
		for (int k = j + 1; k < n; k++) A[(long)j * n + k] = 0;
	}
	return 1;
}

/* src/quant.c:222-253: U with H^-1 = U^T U, through L^-1 and a second factorisation. */
static int inv_chol_upper(const double *H, int n, double *U)
{
	size_t nn = (size_t)n * (size_t)n;
	double *L = malloc(nn * sizeof *L), *Li = malloc(nn * sizeof *Li);
	memcpy(L, H, nn * sizeof *L);
	int ok = cholesky(L, n);
	if (ok) {
		for (size_t i = 0; i < nn; i++) Li[i] = 0;
		for (int c = 0; c < n; c++)
			for (int i = c; i < n; i++) {
				double s = i == c ? 1.0 : 0.0;
				for (int k = c; k < i; k++) s -= L[(long)i * n + k] * Li[(long)k * n + c];
				Li[(long)i * n + c] = s / L[(long)i * n + i];
			}
		for (int i = 0; i < n; i++)
			for (int j = i; j < n; j++) {
				double s = 0;
				for (int k = j; k < n; k++) s += Li[(long)k * n + i] * Li[(long)k * n + j];
				U[(long)i * n + j] = U[(long)j * n + i] = s;
			}
		ok = cholesky(U, n);
		if (ok)
			for (int i = 0; i < n; i++)
				for (int j = i + 1; j < n; j++) {
					U[(long)i * n + j] = U[(long)j * n + i];
					U[(long)j * n + i] = 0;
				}
	}
	free(L);
	free(Li);
	return ok;
}

/* src/quant.c:158-174 set_code */
static void set_code(signed char *q, int bits, long i, int code)
{
	if (bits == 8) {
		q[i] = (signed char)code;
		return;
	}
	unsigned char b = (unsigned char)q[i / 2];
	b = i % 2 ? (unsigned char)((b & 0x0f) | (unsigned char)((unsigned)code << 4)) : (unsigned char)((b & 0xf0) | (code & 0x0f));
	q[i / 2] = (signed char)b;
}

/* src/quant.c:92-118: H[r][c] += x_r x_c in double, zero inputs skipped. */
void tgo_hessian_add(double *H, const float *x, int nrows, int K)
{
	for (int r0 = 0; r0 < nrows; r0++) {
		const float *v = x + (long)r0 * K;
		for (int r = 0; r < K; r++) {
			double xr = v[r];
			if (xr == 0) continue;
			for (int c = 0; c < K; c++) H[(long)r * K + c] += xr * v[c];
		}
	}
}

/* src/quant.c:258-302: channels on `axis`, RTN scale per channel, GPTQ error
 * feedback through U when H is given and positive definite. */
int tgo_quantize(const float *w, int rows, int cols, int axis, int bits, double *H, signed char *q, float *s)
{
	int lim = bits == 8 ? 127 : 7;
	int C = axis == 0 ? rows : cols, K = axis == 0 ? cols : rows;
	long n = (long)C * K;
	memset(q, 0, (size_t)(bits == 8 ? n : (n + 1) / 2));
	double *W = malloc((size_t)n * sizeof *W), *hd = NULL, *U = NULL;
	for (int c = 0; c < C; c++)
		for (int j = 0; j < K; j++) W[(long)c * K + j] = axis == 0 ? w[(long)c * K + j] : w[(long)j * C + c];
	if (H) {
		double mean = 0;
		hd = malloc((size_t)K * sizeof *hd);
		for (int j = 0; j < K; j++) mean += H[(long)j * K + j];
		mean /= K;
		for (int j = 0; j < K; j++) {
			if (H[(long)j * K + j] == 0) {
				H[(long)j * K + j] = 1;
				for (int c = 0; c < C; c++) W[(long)c * K + j] = 0;
			}
			H[(long)j * K + j] += 0.01 * mean;
			hd[j] = H[(long)j * K + j];
		}
		U = malloc((size_t)K * (size_t)K * sizeof *U);
		if (!inv_chol_upper(H, K, U)) {
			free(U);
			U = NULL;
		}
	}
	for (int c = 0; c < C; c++) {
		double *wc = W + (long)c * K;
		double sc = best_scale(wc, K, hd, lim);
		s[c] = (float)sc;
		for (int j = 0; j < K; j++) {
			int code = code_of(wc[j], sc, lim);
			set_code(q, bits, axis == 0 ? (long)c * K + j : (long)j * C + c, code);
			if (U) {
				double err = (wc[j] - sc * code) / U[(long)j * K + j];
				for (int jj = j + 1; jj < K; jj++) wc[jj] -= err * U[(long)j * K + jj];
			}
		}
	}
	int used = U != NULL;
	free(W);
	free(hd);
	free(U);
	return used;
}

/* ---- program VM: src/vm.c ----------------------------------------------------- */

typedef struct {
	const tg_cuda_program *p;
	const float *row;
	float *arena;
	long *slot; /* per value: arena offset, or input offset into the row */
	int *steps;
	float *margin; /* per think loop: min over iterations of |delta - eps|, or NULL */
} OVM;

static long numel(const tg_cuda_value *v)
{
	long n = 1;
	for (int i = 0; i < v->rank; i++) n *= v->dim[i];
	return n;
}

static float *optr(OVM *vm, int v)
{
	const tg_cuda_value *x = &vm->p->val[v];
	if (x->kind == TG_CUDA_PARAM || x->kind == TG_CUDA_STATE) return (float *)x->data;
	if (x->kind == TG_CUDA_INPUT) return (float *)vm->row + vm->slot[v];
	return vm->arena + vm->slot[v];
}

static void ocopy(float *o, const float *a, long n)
{
	if (o != a) memmove(o, a, (size_t)n * sizeof *o);
}

/* NumPy broadcasting (src/util.c shape_broadcast): dimensions aligned from the right. */
static void obin(int op, float *o, const tg_cuda_value *vo, const float *a, const tg_cuda_value *va, const float *b,
		 const tg_cuda_value *vb)
{
	int r = vo->rank;
	long n = numel(vo);
	long sa[4] = { 0 }, sb[4] = { 0 };
	long st = 1;
	for (int d = va->rank - 1; d >= 0; d--) {
		int od = r - va->rank + d;
		sa[od] = va->dim[d] == 1 ? 0 : st;
		st *= va->dim[d];
	}
	st = 1;
	for (int d = vb->rank - 1; d >= 0; d--) {
		int od = r - vb->rank + d;
		sb[od] = vb->dim[d] == 1 ? 0 : st;
		st *= vb->dim[d];
	}
	for (long i = 0; i < n; i++) {
		long rem = i, ia = 0, ib = 0;
		for (int d = r - 1; d >= 0; d--) {
			long idx = rem % vo->dim[d];
			rem /= vo->dim[d];
			ia += idx * sa[d];
			ib += idx * sb[d];
		}
		o[i] = bin1(op, a[ia], b[ib]);
	}
}

/* Rounded table index or -1 (runtime/tg_rt.h:200-204, tg_ell_idx). */
static int oell(float v, int d)
{
	float r = floorf(v + 0.5f);
	return r >= 0.0f && r < (float)d ? (int)r : -1;
}

/* spmm / spmm with a quantized table (runtime/tg_rt.h:206-235): rows of ELLPACK (index,
 * value) pairs against a table [d, h], entries in order, padding (value 0) and
 * out-of-range indices skipped; a quantized table multiplies its codes by value * scale
 * of the entry's row. */
static void ospmm(float *o, const float *x, const float *w, const tg_cuda_value *wv, int r, int k, int d, int h)
{
	const int quant = wv->qbits && wv->qaxis == 0;
	for (int i = 0; i < r; i++) {
		float *y = o + (long)i * h;
		for (int j = 0; j < h; j++) y[j] = 0.0f;
		for (int e = 0; e < k; e++) {
			const float *pr = x + ((long)i * k + e) * 2;
			const int t = oell(pr[0], d);
			if (t < 0 || pr[1] == 0.0f) continue;
			if (quant) {
				const float v = pr[1] * wv->qs[t];
				for (int j = 0; j < h; j++) y[j] += v * (float)tgo_qget(wv->q, wv->qbits, (long)t * h + j);
			} else {
				for (int j = 0; j < h; j++) y[j] += pr[1] * w[(long)t * h + j];
			}
		}
	}
}

/* topk (runtime/tg_rt.h:445-483): per row, the indices of the k largest entries, largest
 * first, ties to the lower index, NaN never chosen, -1 past the row's non-NaN entries.
 * Restated as repeated selection of the next entry in the order (value descending,
 * index ascending), which picks the same indices as the reference's insertion buffer. */
static void otopk(float *o, const float *a, int rows, int n, int k)
{
	for (int r = 0; r < rows; r++) {
		const float *x = a + (long)r * n;
		float lv = 0.0f;
		int li = -1; /* the last pick: (value lv, index li); -1 = none yet */
		for (int i = 0; i < k; i++) {
			int bi = -1;
			float bv = 0.0f;
			for (int j = 0; j < n; j++) {
				const float v = x[j];
				if (v != v) continue;
				if (li >= 0 && !(v < lv || (v == lv && j > li))) continue; /* not after the last pick */
				if (bi < 0 || v > bv) bi = j, bv = v;                     /* first index wins a tie */
			}
			o[(long)r * k + i] = (float)bi;
			if (bi < 0) {
				for (int q = i + 1; q < k; q++) o[(long)r * k + q] = -1.0f;
				break;
			}
			lv = bv, li = bi;
		}
	}
}

/* memscan (runtime/tg_rt.h:485-516): a delta-rule memory M (rows, dv), initially m0,
 * read and written by tn steps of k entries (row, read weight a, write weight c[, delta
 * read weight dd]); per step, in entry order: r = sum a M[row], rd = sum dd M[row]
 * (dd = a with 3 fields), then M[row] += c (v - rd) for c != 0. Output: the reads r
 * (tn, dv), the delta reads rd (tn, dv), the final M. */
static void omemscan(float *o, const float *m0, const float *p, const float *v, int tn, int kq, int rows, int dv)
{
	const int k = kq / 2, q = 3 + (kq & 1);
	float *M = o + 2L * tn * dv;
	memmove(M, m0, (size_t)rows * dv * sizeof *M);
	for (long st = 0; st < tn; st++) {
		const float *e = p + st * k * q, *x = v + st * dv;
		float *r = o + st * dv, *rd = o + ((long)tn + st) * dv;
		for (int j = 0; j < dv; j++) r[j] = rd[j] = 0.0f;
		for (int i = 0; i < k; i++) {
			const int t = oell(e[i * q], rows);
			if (t < 0) continue;
			const float a = e[i * q + 1], dd = q == 4 ? e[i * q + 3] : a;
			for (int j = 0; j < dv; j++) {
				r[j] += a * M[(long)t * dv + j];
				rd[j] += dd * M[(long)t * dv + j];
			}
		}
		for (int i = 0; i < k; i++) {
			const int t = oell(e[i * q], rows);
			const float c = e[i * q + 2];
			if (t < 0 || c == 0.0f) continue;
			for (int j = 0; j < dv; j++) M[(long)t * dv + j] += c * (x[j] - rd[j]);
		}
	}
}

/* sufmatch (runtime/tg_rt.h:579-666): per stream, a suffix automaton of the tokens read
 * so far; at step t, the state reached by the longest suffix of x[..t] seen before t, and
 * the token that followed that suffix's first occurrence. The automaton lives in the
 * output's workspace exactly as the reference lays it out (per state: len, link, first
 * end, edge list head; per edge slot of an open-addressing table of H = the first power of
 * two >= max(16, 6T + 6): state, symbol, target, next edge of the state), so the whole
 * output matches, workspace included. */
static long osm_cap(long T)
{
	long h = 16;
	while (h < 6 * T + 6) h *= 2;
	return h;
}
static long osm_slot(const float *E, long H, long st, long c)
{
	unsigned long h = ((unsigned long)st * 2654435761UL ^ (unsigned long)c * 40503UL) & (unsigned long)(H - 1);
	for (;; h = (h + 1) & (unsigned long)(H - 1))
		if (E[h * 4] < 0.0f || ((long)E[h * 4] == st && (long)E[h * 4 + 1] == c)) return (long)h;
}
static long osm_get(const float *E, long H, long st, long c)
{
	const long h = osm_slot(E, H, st, c);
	return E[h * 4] < 0.0f ? -1 : (long)E[h * 4 + 2];
}
static void osm_put(float *E, float *S, long H, long st, long c, long to)
{
	const long h = osm_slot(E, H, st, c);
	if (E[h * 4] < 0.0f) { /* a new edge of st: push it on st's edge list */
		E[h * 4] = (float)st, E[h * 4 + 1] = (float)c, E[h * 4 + 3] = S[st * 4 + 3];
		S[st * 4 + 3] = (float)h;
	}
	E[h * 4 + 2] = (float)to;
}
static void osufmatch(float *o, const float *x, int T, int n)
{
	const long H = osm_cap(T);
	float *S = o + 2L * T * n, *E = S + 4 * (2L * T + 2);
	for (int g = 0; g < n; g++) {
		long nst = 1, last = 0, m = 0, l = 0;
		for (long i = 0; i < H; i++) E[i * 4] = -1.0f;
		S[0] = 0.0f, S[1] = -1.0f, S[2] = -1.0f, S[3] = -1.0f;
		for (long t = 0; t < T; t++) {
			const float xv = x[t * n + g];
			const long c = xv >= 0.0f ? (long)(xv + 0.5f) : -1;
			float *out = o + (t * n + g) * 2;
			if (c < 0) { /* a negative id: no match across it, not added */
				m = 0, l = 0;
				out[0] = -1.0f, out[1] = 0.0f;
				continue;
			}
			/* the longest suffix of x[..t] that occurs before t */
			while (m != 0 && osm_get(E, H, m, c) < 0) {
				m = (long)S[m * 4 + 1];
				l = (long)S[m * 4];
			}
			const long tr = osm_get(E, H, m, c);
			if (tr >= 0) m = tr, l++;
			else m = 0, l = 0;
			const long fe = l > 0 ? (long)S[m * 4 + 2] : -1;
			out[0] = fe >= 0 && fe + 1 <= t ? x[(fe + 1) * n + g] : -1.0f;
			out[1] = (float)l;
			/* extend the automaton by c */
			const long cur = nst++;
			long pp = last;
			S[cur * 4] = S[last * 4] + 1.0f, S[cur * 4 + 2] = (float)t, S[cur * 4 + 3] = -1.0f;
			for (; pp != -1 && osm_get(E, H, pp, c) < 0; pp = (long)S[pp * 4 + 1]) osm_put(E, S, H, pp, c, cur);
			if (pp == -1) {
				S[cur * 4 + 1] = 0.0f;
			} else {
				const long qs = osm_get(E, H, pp, c);
				if (S[pp * 4] + 1.0f == S[qs * 4]) {
					S[cur * 4 + 1] = (float)qs;
				} else { /* split qs: a clone of length len(pp) + 1 */
					const long cl = nst++;
					S[cl * 4] = S[pp * 4] + 1.0f, S[cl * 4 + 1] = S[qs * 4 + 1], S[cl * 4 + 2] = S[qs * 4 + 2], S[cl * 4 + 3] = -1.0f;
					for (long h = (long)S[qs * 4 + 3]; h >= 0; h = (long)E[h * 4 + 3]) osm_put(E, S, H, cl, (long)E[h * 4 + 1], (long)E[h * 4 + 2]);
					for (; pp != -1 && osm_get(E, H, pp, c) == qs; pp = (long)S[pp * 4 + 1]) osm_put(E, S, H, pp, c, cl);
					S[qs * 4 + 1] = (float)cl, S[cur * 4 + 1] = (float)cl;
					if (m == qs && l <= (long)S[cl * 4]) m = cl;
				}
			}
			last = cur;
		}
	}
}

/* The iteration space of an operand broadcast to `out` (src/util.c:172-212, bcast_desc
 * with one operand): size-1 axes of out dropped, adjacent axes merged where the operand's
 * strides allow (both broadcast, or contiguous); d = rank, dims, the operand's strides. */
static void odesc(const tg_cuda_value *out, const tg_cuda_value *a, int *d)
{
	int r = out->rank, dim[4], st[4], nr = 0;
	long acc = 1;
	for (int i = r - 1; i >= 0; i--) {
		const int j = i - (r - a->rank), n = j >= 0 ? a->dim[j] : 1;
		st[i] = n == 1 ? 0 : (int)acc;
		acc *= n;
	}
	int md[4], ms[4];
	for (int i = 0; i < r; i++) {
		if (out->dim[i] == 1) continue;
		if (nr > 0) {
			const int p = nr - 1;
			const long merged = (long)st[i] * out->dim[i];
			if ((ms[p] == 0 && st[i] == 0) || (st[i] != 0 && ms[p] == merged)) {
				md[p] *= out->dim[i];
				ms[p] = st[i];
				continue;
			}
		}
		md[nr] = out->dim[i], ms[nr] = st[i], nr++;
	}
	if (nr == 0) md[0] = 1, ms[0] = 0, nr = 1;
	(void)dim;
	d[0] = nr;
	for (int i = 0; i < nr; i++) d[1 + i] = md[i], d[1 + nr + i] = ms[i];
}

/* sum_to (runtime/tg_rt.h:419-438): o (no elements) = the sum of x over its broadcast
 * axes, in the iteration order of the merged space; a broadcast innermost axis is summed
 * by rows first. */
static void osum_to(float *o, const float *x, long no, const int *d)
{
	const int r = d[0];
	const int *dim = d + 1, *so = d + 1 + r;
	const int w = dim[r - 1];
	int idx[4] = { 0 };
	long n = 1, io = 0;
	for (long i = 0; i < no; i++) o[i] = 0.0f;
	for (int i = 0; i < r - 1; i++) n *= dim[i];
	for (long i = 0; i < n; i++) {
		const float *px = x + i * w;
		if (so[r - 1]) {
			for (int j = 0; j < w; j++) o[io + j] += px[j];
		} else {
			float sacc = 0.0f;
			for (int j = 0; j < w; j++) sacc += px[j];
			o[io] += sacc;
		}
		for (int q = r - 2; q >= 0; q--) {
			io += so[q];
			if (++idx[q] < dim[q]) break;
			io -= (long)so[q] * dim[q];
			idx[q] = 0;
		}
	}
}

/* take_t (runtime/tg_rt.h:324-333): o [d, h] = 0, then the rows of g added at rows r. */
static void otake_t(float *o, const float *r, const float *g, int n, int d, int h)
{
	for (long i = 0; i < (long)d * h; i++) o[i] = 0.0f;
	for (int i = 0; i < n; i++) {
		const int t = oell(r[i], d);
		if (t >= 0)
			for (int j = 0; j < h; j++) o[(long)t * h + j] += g[(long)i * h + j];
	}
}

/* memscan_t (runtime/tg_rt.h:517-578): memscan's derivatives, replaying the steps backwards
 * from the final memory and undoing each write. y is memscan's output, pv (tn, 4k + dv) the
 * entries (row, a, c, d) then the step's value, g the adjoint of y. o: dP (tn k 4) at 0, dM0
 * (rows, dv) at o1, dV (tn, dv) at o2, the working memory at o3, padded to N (the layout's
 * rounding: o1 up to a multiple of dv, N up to a multiple of dv, 2 dv or 4 dv, whichever
 * is a multiple of 4). */
static void omemscan_layout(long tn, int k, int rows, int dv, long *o1, long *o2, long *o3, long *N)
{
	const long np = tn * k * 4, L = dv % 4 == 0 ? dv : dv % 2 == 0 ? 2L * dv : 4L * dv;
	*o1 = (np + dv - 1) / dv * dv;
	*o2 = *o1 + (long)rows * dv;
	*o3 = *o2 + tn * dv;
	*N = (*o3 + (long)rows * dv + L - 1) / L * L;
}
static void omemscan_t(float *o, const float *y, const float *pv, const float *g, int tn, int k, int rows, int dv)
{
	const long w = 4L * k + dv;
	long o1, o2, o3, N;
	omemscan_layout(tn, k, rows, dv, &o1, &o2, &o3, &N);
	float *dP = o, *dM = o + o1, *dV = o + o2, *M = o + o3;
	for (long i = 0; i < N; i++) o[i] = 0.0f;
	for (long i = 0; i < (long)rows * dv; i++) M[i] = y[2L * tn * dv + i], dM[i] = g[2L * tn * dv + i];
	for (long st = (long)tn - 1; st >= 0; st--) {
		const float *e = pv + st * w, *x = e + 4 * k, *rd = y + ((long)tn + st) * dv, *gr = g + st * dv,
			    *grd = g + ((long)tn + st) * dv;
		float *dp = dP + st * k * 4, *dx = dV + st * dv;
		for (int i = k - 1; i >= 0; i--) { /* the memory as this step read it */
			const int t = oell(e[i * 4], rows);
			const float c = e[i * 4 + 2];
			if (t < 0 || c == 0.0f) continue;
			for (int j = 0; j < dv; j++) M[(long)t * dv + j] -= c * (x[j] - rd[j]);
		}
		for (int i = 0; i < k; i++) { /* the writes: dc_i, and the value's gradient */
			const int t = oell(e[i * 4], rows);
			const float c = e[i * 4 + 2];
			float dc = 0.0f;
			if (t < 0) continue;
			for (int j = 0; j < dv; j++) {
				dc += dM[(long)t * dv + j] * (x[j] - rd[j]);
				dx[j] += c * dM[(long)t * dv + j];
			}
			dp[i * 4 + 2] = dc;
		}
		for (int i = 0; i < k; i++) { /* the reads: da_i and dd_i */
			const int t = oell(e[i * 4], rows);
			float da = 0.0f, dd = 0.0f;
			if (t < 0) continue;
			for (int j = 0; j < dv; j++) {
				da += gr[j] * M[(long)t * dv + j];
				dd += (grd[j] - dx[j]) * M[(long)t * dv + j];
			}
			dp[i * 4 + 1] = da, dp[i * 4 + 3] = dd;
		}
		for (int i = 0; i < k; i++) { /* the memory's adjoint before this step */
			const int t = oell(e[i * 4], rows);
			const float a = e[i * 4 + 1], d = e[i * 4 + 3];
			if (t < 0) continue;
			for (int j = 0; j < dv; j++) dM[(long)t * dv + j] += a * gr[j] + d * (grd[j] - dx[j]);
		}
	}
}

static int oexec(OVM *vm, int from, int count);

/* src/ops.c:60-73 matmul_dims / matmul_groups, src/ops.c:310-320 q_axis_for,
 * src/vm.c:262-290 dispatch. */
static void omatmul(OVM *vm, const tg_cuda_ins *in)
{
	const tg_cuda_program *p = vm->p;
	const tg_cuda_value *A = &p->val[in->a[0]], *B = &p->val[in->a[1]];
	int g = A->rank == 3 && B->rank == 3 ? A->dim[0] : 1;
	int m = A->rank == 3 ? (g > 1 || B->rank == 3 ? A->dim[1] : A->dim[0] * A->dim[1]) : A->rank == 2 ? A->dim[0] : 1;
	int k = A->dim[A->rank - 1];
	int n = B->rank >= 2 ? B->dim[B->rank - 1] : 1;
	float *o = optr(vm, in->out);
	const float *a = optr(vm, in->a[0]), *b = optr(vm, in->a[1]);
	if (g > 1) {
		for (int i = 0; i < g; i++)
			tgo_matmul(o + (long)i * m * n, a + (long)i * m * k, b + (long)i * k * n, m, k, n);
		return;
	}
	int qa_axis = A->rank == 2 && in->a[0] != in->a[1] ? 0 : -1;
	int qb_axis = B->rank == 2 && in->a[0] != in->a[1] ? 1 : -1;
	if (A->qbits && qa_axis == A->qaxis) tgo_matmul_qa(o, A->q, A->qbits, A->qs, b, m, k, n);
	else if (B->qbits && qb_axis == B->qaxis) tgo_matmul_qb(o, a, B->q, B->qbits, B->qs, m, k, n);
	else tgo_matmul(o, a, b, m, k, n);
}

static int oone(OVM *vm, const tg_cuda_ins *in)
{
	const tg_cuda_program *p = vm->p;
	const tg_cuda_value *vo = &p->val[in->out];
	long n = numel(vo);
	float *o = optr(vm, in->out);
	const float *a = in->na > 0 ? optr(vm, in->a[0]) : NULL;
	const float *c = in->na > 1 ? optr(vm, in->a[1]) : NULL;
	switch (in->op) {
	case TG_CUDA_OP_CONST:
		o[0] = in->k;
		return 0;
	case TG_CUDA_OP_ADD: case TG_CUDA_OP_SUB: case TG_CUDA_OP_MUL: case TG_CUDA_OP_DIV: case TG_CUDA_OP_MAX: case TG_CUDA_OP_MIN:
		obin(in->op, o, vo, a, &p->val[in->a[0]], c, &p->val[in->a[1]]);
		return 0;
	case TG_CUDA_OP_NEG: case TG_CUDA_OP_TANH: case TG_CUDA_OP_RELU: case TG_CUDA_OP_SIGMOID: case TG_CUDA_OP_EXP:
	case TG_CUDA_OP_SQRT: case TG_CUDA_OP_GELU: case TG_CUDA_OP_SILU: case TG_CUDA_OP_SOFTPLUS: case TG_CUDA_OP_LOG:
	case TG_CUDA_OP_STEP: case TG_CUDA_OP_SIN: case TG_CUDA_OP_COS: case TG_CUDA_OP_FLOOR:
		tgo_unary(in->op, o, a, (int)n);
		return 0;
	case TG_CUDA_OP_MATMUL:
		omatmul(vm, in);
		return 0;
	case TG_CUDA_OP_SOFTMAX: case TG_CUDA_OP_RMSNORM: { /* src/ops.c:75-79 row_dims */
		const tg_cuda_value *x = &p->val[in->a[0]];
		int cols = x->rank ? x->dim[x->rank - 1] : 1, rows = (int)(numel(x) / cols);
		if (in->op == TG_CUDA_OP_SOFTMAX) tgo_softmax(o, a, rows, cols);
		else tgo_rmsnorm(o, a, rows, cols);
		return 0;
	}
	case TG_CUDA_OP_SUM: case TG_CUDA_OP_MEAN: { /* runtime/tg_rt.h:178-181 */
		long k = numel(&p->val[in->a[0]]);
		float s = 0.0f;
		for (long i = 0; i < k; i++) s += a[i];
		o[0] = in->op == TG_CUDA_OP_SUM ? s : s / (float)k;
		return 0;
	}
	case TG_CUDA_OP_TRANSPOSE: { /* runtime/tg_rt.h:183-187, :443-446 */
		const tg_cuda_value *x = &p->val[in->a[0]];
		int g = x->rank == 3 ? x->dim[0] : 1, r = x->dim[x->rank - 2], cc = x->dim[x->rank - 1];
		for (int q = 0; q < g; q++)
			for (int i = 0; i < r; i++)
				for (int j = 0; j < cc; j++) o[(long)q * r * cc + (long)j * r + i] = a[(long)q * r * cc + (long)i * cc + j];
		return 0;
	}
	case TG_CUDA_OP_OUTER: { /* runtime/tg_rt.h:190-194 */
		long m = numel(&p->val[in->a[0]]), nn = numel(&p->val[in->a[1]]);
		for (long i = 0; i < m; i++)
			for (long j = 0; j < nn; j++) o[i * nn + j] = a[i] * c[j];
		return 0;
	}
	case TG_CUDA_OP_TAKE: { /* runtime/tg_rt.h:316-322 with tg_ell_idx :200-204 */
		const tg_cuda_value *w = &p->val[in->a[0]];
		int d = w->dim[0];
		long h = numel(w) / d;
		int cnt = p->val[in->a[1]].dim[0];
		for (int i = 0; i < cnt; i++) {
			float r = floorf(c[i] + 0.5f);
			int t = r >= 0.0f && r < (float)d ? (int)r : -1;
			for (long j = 0; j < h; j++) o[(long)i * h + j] = t >= 0 ? a[(long)t * h + j] : 0.0f;
		}
		return 0;
	}
	case TG_CUDA_OP_RESHAPE:
		ocopy(o, a, n);
		return 0;
	case TG_CUDA_OP_SPMM: { /* src/vm.c:307-313, src/ops.c:82-88 spmm_dims */
		const tg_cuda_value *x = &p->val[in->a[0]], *w = &p->val[in->a[1]];
		ospmm(o, a, c, w, x->rank == 3 ? x->dim[0] : 1, x->dim[x->rank - 2], w->dim[0], w->dim[1]);
		return 0;
	}
	case TG_CUDA_OP_TOPK: { /* src/vm.c:340-345 */
		const tg_cuda_value *x = &p->val[in->a[0]];
		const int cols = x->rank ? x->dim[x->rank - 1] : 1;
		otopk(o, a, (int)(numel(x) / cols), cols, vo->dim[vo->rank - 1]);
		return 0;
	}
	case TG_CUDA_OP_MEMSCAN: { /* src/vm.c:351-357, src/util.c:455-467 memscan_dims */
		const tg_cuda_value *m0 = &p->val[in->a[0]], *pe = &p->val[in->a[1]];
		const float *v = optr(vm, in->a[2]);
		omemscan(o, a, c, v, pe->dim[0] * pe->dim[1], 2 * pe->dim[2] + (pe->dim[3] == 4), m0->dim[0], m0->dim[1]);
		return 0;
	}
	case TG_CUDA_OP_SUM_TO: { /* src/vm.c:358-363 */
		int d[13];
		odesc(&p->val[in->a[0]], &p->val[in->a[1]], d);
		osum_to(o, a, n, d);
		return 0;
	}
	case TG_CUDA_OP_TAKE_T: { /* src/vm.c:320-323 */
		const tg_cuda_value *w = &p->val[in->a[2]];
		otake_t(o, a, c, p->val[in->a[0]].dim[0], w->dim[0], (int)(numel(w) / w->dim[0]));
		return 0;
	}
	case TG_CUDA_OP_MEMSCAN_T: { /* src/vm.c:351-357, src/util.c:455-467 memscan_dims */
		const tg_cuda_value *y = &p->val[in->a[0]], *pv = &p->val[in->a[1]];
		const int dv = y->dim[1], tn = pv->dim[0] * pv->dim[1];
		omemscan_t(o, a, c, optr(vm, in->a[2]), tn, (pv->dim[2] - dv) / 4, y->dim[0] - 2 * tn, dv);
		return 0;
	}
	case TG_CUDA_OP_SUFMATCH: { /* src/vm.c:346-350 */
		const tg_cuda_value *x = &p->val[in->a[0]];
		osufmatch(o, a, x->dim[0], x->rank == 2 ? x->dim[1] : 1);
		return 0;
	}
	case TG_CUDA_OP_THINK: { /* src/vm.c:383-411 */
		ocopy(o, optr(vm, in->init), n);
		int it = 0;
		float survive = 1.0f;
		while (it < in->maxit) {
			if (oexec(vm, in->body, in->nbody)) return -1;
			it++;
			const float *y = optr(vm, in->yield);
			float d = 0.0f; /* runtime/tg_rt.h:361-366 tg_delta */
			for (long i = 0; i < n; i++) {
				float e = fabsf(y[i] - o[i]);
				if (e > d) d = e;
			}
			ocopy(o, y, n);
			if (vm->margin && in->eps >= 0 && fabsf(d - in->eps) < vm->margin[in->tid]) vm->margin[in->tid] = fabsf(d - in->eps);
			if (in->eps >= 0 && d <= in->eps) break;
			if (in->halt >= 0) {
				float pr = *optr(vm, in->halt);
				survive *= 1.0f - (pr < 0.0f ? 0.0f : pr > 1.0f ? 1.0f : pr);
				if (vm->margin && fabsf((1.0f - survive) - in->hthr) < vm->margin[in->tid])
					vm->margin[in->tid] = fabsf((1.0f - survive) - in->hthr);
				if (1.0f - survive > in->hthr) break;
			}
		}
		vm->steps[in->tid] = it;
		return 0;
	}
	case TG_CUDA_OP_SCAN: { /* src/vm.c:364-382 */
		const tg_cuda_scan *s = &p->scans[in->scan];
		for (int k = 0; k < s->nc; k++) ocopy(optr(vm, s->c[k]), optr(vm, s->init[k]), numel(&p->val[s->c[k]]));
		for (int step = 0; step < s->T; step++) {
			int t = s->reverse ? s->T - 1 - step : step;
			for (int j = 0; j < s->nx; j++) {
				long w = numel(&p->val[s->xt[j]]);
				ocopy(optr(vm, s->xt[j]), optr(vm, s->x[j]) + (long)t * w, w);
			}
			if (oexec(vm, in->body, in->nbody)) return -1;
			for (int y = 0; y < s->ny; y++) {
				long w = numel(&p->val[s->y[y]]);
				ocopy(optr(vm, s->ys[y]) + (long)t * w, optr(vm, s->y[y]), w);
			}
			for (int k = 0; k < s->nc; k++) ocopy(optr(vm, s->c[k]), optr(vm, s->next[k]), numel(&p->val[s->c[k]]));
		}
		if (s->tid >= 0) vm->steps[s->tid] = s->T;
		return 0;
	}
	}
	return -1;
}

static int oexec(OVM *vm, int from, int count)
{
	for (int i = from; i < from + count; i++)
		if (oone(vm, &vm->p->ins[i])) return -1;
	return 0;
}

/* One slot per temporary (no sharing): the oracle favours plainness over size. */
static long oplan(const tg_cuda_program *p, long *slot)
{
	long off = 0, in = 0;
	for (int i = 0; i < p->ninputs; i++) {
		slot[p->inputs[i]] = in;
		in += numel(&p->val[p->inputs[i]]);
	}
	for (int v = 0; v < p->nval; v++)
		if (p->val[v].kind == TG_CUDA_TMP) {
			slot[v] = off;
			off += (numel(&p->val[v]) + 3) / 4 * 4;
		}
	return off ? off : 1;
}

long tgo_program_arena(const tg_cuda_program *p)
{
	long *slot = calloc((size_t)p->nval + 1, sizeof *slot);
	long a = oplan(p, slot);
	free(slot);
	return a;
}

int tgo_program_run(const tg_cuda_program *p, const float *row, float *out, int *steps, float *arena, float *margin)
{
	long *slot = calloc((size_t)p->nval + 1, sizeof *slot);
	oplan(p, slot);
	if (margin)
		for (int t = 0; t < p->nthink; t++) margin[t] = INFINITY;
	OVM vm = { p, row, arena, slot, steps, margin };
	int rc = oexec(&vm, 0, p->ntop);
	if (!rc) ocopy(out, optr(&vm, p->output), numel(&p->val[p->output]));
	free(slot);
	return rc;
}

/* ---- the Qwen3 program: examples/qwen3/import.py:90-132 ---------------------------- */

static void rowmul(float *x, const float *w, int rows, int cols) /* x * w, w broadcast over rows */
{
	for (int r = 0; r < rows; r++)
		for (int i = 0; i < cols; i++) x[(long)r * cols + i] = x[(long)r * cols + i] * w[i];
}

/* Column block [c0, c0+nc) of a quantized [K, N] matrix applied as x @ W (tg_matmul_qb on
 * the per-head param the program holds). */
static void qb_block(float *o, const float *x, const tg_cuda_qmat *w, int bits, int T, int K, int N, int c0, int nc,
		     const float *s)
{
	for (int t = 0; t < T; t++)
		for (int j = 0; j < nc; j++) {
			float acc = 0.0f;
			for (int p = 0; p < K; p++) acc += x[(long)t * K + p] * (float)tgo_qget(w->q, bits, (long)p * N + c0 + j);
			o[(long)t * nc + j] = s[j] * acc;
		}
}

/* rotary(x) = x * cosT + (x @ Rot) * sinT with Rot the rotate-half matrix
 * (import.py:79-84,96-97); x @ Rot sums exactly one nonzero product. */
static void rotary(float *x, const float *cosT, const float *sinT, int T, int HD)
{
	float *r = malloc((size_t)HD * sizeof *r);
	for (int t = 0; t < T; t++) {
		float *v = x + (long)t * HD;
		for (int i = 0; i < HD / 2; i++) {
			r[i] = -v[i + HD / 2];
			r[i + HD / 2] = v[i];
		}
		for (int i = 0; i < HD; i++) {
			float a = v[i] * cosT[(long)t * HD + i], b = r[i] * sinT[(long)t * HD + i];
			v[i] = a + b;
		}
	}
	free(r);
}

int tgo_lm_forward(const tg_cuda_lm_desc *d, const float *ids, int T, float *logits)
{
	int D = d->hidden, HD = d->head_dim, NQ = d->nq, NKV = d->nkv, FF = d->ffn, V = d->vocab, grp = NQ / NKV;
	size_t TD = (size_t)T * D;
	float *h = malloc(TD * sizeof *h), *n = malloc(TD * sizeof *n), *acc = malloc(TD * sizeof *acc);
	float *k = malloc((size_t)NKV * T * HD * sizeof *k), *v = malloc((size_t)NKV * T * HD * sizeof *v);
	float *q = malloc((size_t)T * HD * sizeof *q), *sc = malloc((size_t)T * T * sizeof *sc);
	float *sv = malloc((size_t)T * HD * sizeof *sv), *oh = malloc(TD * sizeof *oh);
	float *g = malloc((size_t)T * FF * sizeof *g), *u = malloc((size_t)T * FF * sizeof *u), *m = malloc(TD * sizeof *m);
	float *cosT = malloc((size_t)T * HD * sizeof *cosT), *sinT = malloc((size_t)T * HD * sizeof *sinT);
	/* RoPE tables in double, stored as f32 (import.py:76-78) */
	for (int t = 0; t < T; t++)
		for (int i = 0; i < HD / 2; i++) {
			double inv = pow(d->rope_theta, -((double)(2 * i) / HD)), ang = (double)t * inv;
			cosT[(long)t * HD + i] = cosT[(long)t * HD + i + HD / 2] = (float)cos(ang);
			sinT[(long)t * HD + i] = sinT[(long)t * HD + i + HD / 2] = (float)sin(ang);
		}
	for (int t = 0; t < T; t++) { /* h = take(E, ids) */
		float r = floorf(ids[t] + 0.5f);
		int row = r >= 0.0f && r < (float)V ? (int)r : -1;
		for (int i = 0; i < D; i++) h[(long)t * D + i] = row >= 0 ? d->embed[(long)row * D + i] : 0.0f;
	}
	for (int l = 0; l < d->layers; l++) {
		tgo_rmsnorm(n, h, T, D); /* n = rmsnorm(h) * ln1 */
		rowmul(n, d->ln1[l], T, D);
		for (int j = 0; j < NKV; j++) {
			float *kj = k + (size_t)j * T * HD, *vj = v + (size_t)j * T * HD;
			qb_block(kj, n, &d->wk[l], d->bits, T, D, NKV * HD, j * HD, HD, d->wk[l].s + j * HD);
			tgo_rmsnorm(kj, kj, T, HD);
			rowmul(kj, d->kn[l], T, HD);
			rotary(kj, cosT, sinT, T, HD);
			qb_block(vj, n, &d->wv[l], d->bits, T, D, NKV * HD, j * HD, HD, d->wv[l].s + j * HD);
		}
		for (int hh = 0; hh < NQ; hh++) {
			const float *kj = k + (size_t)(hh / grp) * T * HD, *vj = v + (size_t)(hh / grp) * T * HD;
			qb_block(q, n, &d->wq[l], d->bits, T, D, NQ * HD, hh * HD, HD, d->wq[l].s + hh * HD);
			tgo_rmsnorm(q, q, T, HD);
			rowmul(q, d->qn[l], T, HD);
			rotary(q, cosT, sinT, T, HD);
			/* s = softmax((q @ transpose(k)) * scale + mask), mask 0 / -1e9 (import.py:85) */
			for (int t = 0; t < T; t++)
				for (int s2 = 0; s2 < T; s2++) {
					float dot = 0.0f;
					for (int p = 0; p < HD; p++) dot += q[(long)t * HD + p] * kj[(long)s2 * HD + p];
					sc[(long)t * T + s2] = dot * d->attn_scale + (s2 <= t ? 0.0f : -1e9f);
				}
			tgo_softmax(sc, sc, T, T);
			tgo_matmul(sv, sc, vj, T, T, HD);
			/* o_h = (s @ v) @ Wo_h: rows h*HD.. of the stacked Wo, per-head column scales */
			const tg_cuda_qmat *wo = &d->wo[l];
			for (int t = 0; t < T; t++)
				for (int c = 0; c < D; c++) {
					float a = 0.0f;
					for (int p = 0; p < HD; p++)
						a += sv[(long)t * HD + p] * (float)tgo_qget(wo->q, d->bits, (long)(hh * HD + p) * D + c);
					oh[(long)t * D + c] = wo->s[(long)hh * D + c] * a;
				}
			if (hh == 0) memcpy(acc, oh, TD * sizeof *acc); /* o0 + o1 + ... left to right */
			else
				for (size_t i = 0; i < TD; i++) acc[i] = acc[i] + oh[i];
		}
		for (size_t i = 0; i < TD; i++) h[i] = h[i] + acc[i];
		tgo_rmsnorm(n, h, T, D); /* n = rmsnorm(h) * ln2 */
		rowmul(n, d->ln2[l], T, D);
		qb_block(g, n, &d->wg[l], d->bits, T, D, FF, 0, FF, d->wg[l].s);
		qb_block(u, n, &d->wu[l], d->bits, T, D, FF, 0, FF, d->wu[l].s);
		for (size_t i = 0; i < (size_t)T * FF; i++) g[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
		qb_block(m, g, &d->wd[l], d->bits, T, FF, D, 0, D, d->wd[l].s);
		for (size_t i = 0; i < TD; i++) h[i] = h[i] + m[i];
	}
	/* logits = (rmsnorm(h) * lnf) @ LM; take(logits, lastidx) keeps row T-1 */
	tgo_rmsnorm(n, h + (size_t)(T - 1) * D, 1, D);
	rowmul(n, d->final_norm, 1, D);
	qb_block(logits, n, &d->lm_head, d->bits, 1, D, V, 0, V, d->lm_head.s);
	free(h); free(n); free(acc); free(k); free(v); free(q); free(sc); free(sv); free(oh);
	free(g); free(u); free(m); free(cosT); free(sinT);
	return 0;
}

/* ---- stacked selective-SSM blocks (the program tests/golden/make_golden.py:emit_ssm
 * writes; the scan of src/vm.c:364-382 over the steps of one sequence) ---------------------- */

static float silu1(float x) { return x / (1.0f + expf(-x)); }                      /* runtime/tg_rt.h:59-60 */
static float softplus1(float x) { return (x > 0.0f ? x : 0.0f) + log1pf(expf(-fabsf(x))); } /* :63-64 */

int tgo_ssm_forward(const tg_cuda_ssm_desc *d, const float *u, int T, float *out)
{
	const int DM = d->d_model, DI = d->d_inner, DS = d->d_state, R = d->dt_rank;
	float *cur = malloc((size_t)T * DM * sizeof *cur), *nxt = malloc((size_t)T * DM * sizeof *nxt);
	float *n = malloc(DM * sizeof *n), *x = malloc(DI * sizeof *x), *z = malloc(DI * sizeof *z);
	float *xs = malloc(DI * sizeof *xs), *c1 = malloc(DI * sizeof *c1), *c2 = malloc(DI * sizeof *c2);
	float *c3 = malloc(DI * sizeof *c3), *r = malloc(R * sizeof *r), *bt = malloc(DS * sizeof *bt);
	float *ct = malloc(DS * sizeof *ct), *dt = malloc(DI * sizeof *dt), *g = malloc(DI * sizeof *g);
	float *o = malloc(DM * sizeof *o), *h = malloc((size_t)DI * DS * sizeof *h);
	memcpy(cur, u, (size_t)T * DM * sizeof *cur);
	for (int b = 0; b < d->blocks; b++) {
		const float *cw = d->conv_w[b], *A = d->a[b];
		memset(h, 0, (size_t)DI * DS * sizeof *h);
		memset(c1, 0, DI * sizeof *c1);
		memset(c2, 0, DI * sizeof *c2);
		memset(c3, 0, DI * sizeof *c3);
		for (int t = 0; t < T; t++) {
			const float *ut = cur + (long)t * DM;
			tgo_rmsnorm(n, ut, 1, DM); /* n = rmsnorm(ut) * norm */
			rowmul(n, d->norm[b], 1, DM);
			qb_block(x, n, &d->w_x[b], d->bits, 1, DM, DI, 0, DI, d->w_x[b].s);
			qb_block(z, n, &d->w_z[b], d->bits, 1, DM, DI, 0, DI, d->w_z[b].s);
			for (int i = 0; i < DI; i++) { /* xc, left to right; then the carries shift */
				float xc = (((c3[i] * cw[i] + c2[i] * cw[DI + i]) + c1[i] * cw[2 * DI + i]) + x[i] * cw[3 * DI + i]) +
					   d->conv_b[b][i];
				c3[i] = c2[i];
				c2[i] = c1[i];
				c1[i] = x[i];
				xs[i] = silu1(xc);
			}
			qb_block(r, xs, &d->w_r[b], d->bits, 1, DI, R, 0, R, d->w_r[b].s);
			qb_block(bt, xs, &d->w_b[b], d->bits, 1, DI, DS, 0, DS, d->w_b[b].s);
			qb_block(ct, xs, &d->w_c[b], d->bits, 1, DI, DS, 0, DS, d->w_c[b].s);
			qb_block(dt, r, &d->w_dt[b], d->bits, 1, R, DI, 0, DI, d->w_dt[b].s);
			for (int i = 0; i < DI; i++) dt[i] = softplus1(dt[i] + d->dt_b[b][i]);
			for (int i = 0; i < DI; i++) {
				float m1 = 0.0f;
				for (int s = 0; s < DS; s++) {
					const long k = (long)i * DS + s;
					float e = expf(-(dt[i] * A[k]));
					float t1 = e * h[k], t3 = (1.0f - e) / A[k], t4 = xs[i] * bt[s];
					h[k] = t1 + t3 * t4;
				}
				for (int s = 0; s < DS; s++) m1 += h[(long)i * DS + s] * ct[s]; /* h @ ct */
				float y = m1 + d->d[b][i] * xs[i];
				g[i] = y * silu1(z[i]);
			}
			qb_block(o, g, &d->w_o[b], d->bits, 1, DI, DM, 0, DM, d->w_o[b].s);
			for (int i = 0; i < DM; i++) nxt[(long)t * DM + i] = ut[i] + o[i];
		}
		float *sw = cur;
		cur = nxt;
		nxt = sw;
	}
	tgo_rmsnorm(out, cur, T, DM);
	rowmul(out, d->final_norm, T, DM);
	free(cur); free(nxt); free(n); free(x); free(z); free(xs); free(c1); free(c2); free(c3);
	free(r); free(bt); free(ct); free(dt); free(g); free(o); free(h);
	return 0;
}
