/* ref_harness.c -- TEST INFRASTRUCTURE: exposes the reference's own kernels
 * (runtime/tg_rt.h) and quantizer (src/quant.c, whose helpers are static, so
 * the file is included here) behind plain functions, for the oracle's parity
 * pin. Compiled by oracle/Makefile against the reference sources where they
 * lie; the result, oracle/_ref/libtgref.so, is never part of the product. */
#include "quant.c"
#include "tg_rt.h"

#include <stdlib.h>
#include <string.h>

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
