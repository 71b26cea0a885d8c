/* tgo.h -- CPU oracle for the tests of libtgcuda. TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference arithmetic on the `tgc batch` path
 * (IlumCI/Technograd runtime/tg_rt.h, src/vm.c, src/quant.c, src/lower.c and
 * the program examples/qwen3/import.py emits). Only tests/, the smoke check
 * of __graft_entry__.py and the cpu_baseline leg of bench.py use it; the
 * product library never links or calls it.
 *
 * Parity pin: tests/test_oracle.py checks every function here against the
 * reference itself -- golden vectors the reference produced (tests/golden/,
 * made by tests/golden/make_golden.py from oracle/_ref/tgc and
 * oracle/_ref/libtgref.so, both compiled from the reference's own sources by
 * oracle/Makefile) and, when oracle/_ref is built, live calls on seeded inputs.
 * Compiled with -ffp-contract=off, like the reference (-std=c11 on x86-64
 * contracts nothing), so sums and products round in the reference's order. */
#ifndef TGO_H
#define TGO_H

#include "../include/tg_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* runtime/tg_rt.h kernels */
int tgo_qget(const signed char *q, int bits, long i);
void tgo_matmul(float *o, const float *a, const float *b, int m, int k, int n);
void tgo_matmul_qa(float *o, const signed char *q, int bits, const float *s, const float *b, int m, int k, int n);
void tgo_matmul_qb(float *o, const float *a, const signed char *q, int bits, const float *s, int m, int k, int n);
void tgo_rmsnorm(float *o, const float *a, int rows, int cols);
void tgo_softmax(float *o, const float *a, int rows, int cols);
void tgo_unary(int op, float *o, const float *a, int n);

/* src/lower.c rand(seed, scale) */
void tgo_rand(unsigned seed, float scale, float *out, long n);

/* src/quant.c: quantize one [rows, cols] matrix on axis; H (K x K, K = the
 * non-channel extent) selects GPTQ when non-NULL (it is modified, as in the
 * reference). Returns 1 if GPTQ ran, 0 if RTN. */
int tgo_quantize(const float *w, int rows, int cols, int axis, int bits, double *H, signed char *q, float *s);
/* src/quant.c:92-118 hook: H += x x^T over nrows rows of K values. */
void tgo_hessian_add(double *H, const float *x, int nrows, int K);

/* src/vm.c vm_run_into over a tg_cuda_program: one row. arena is scratch of
 * tgo_program_arena(p) floats; steps gets nthink ints; margin (nthink floats,
 * may be NULL) gets, per think loop, the smallest |delta - eps| over its
 * iterations -- how close the row came to flipping its halting step. Returns 0,
 * or -1 for an op the oracle does not implement. */
long tgo_program_arena(const tg_cuda_program *p);
int tgo_program_run(const tg_cuda_program *p, const float *row, float *out, int *steps, float *arena, float *margin);

/* The Qwen3 program of examples/qwen3/import.py:90-132 over one sequence of
 * T ids, with its quantized linear weights: the logits of the last position.
 * Scratch is allocated inside. */
int tgo_lm_forward(const tg_cuda_lm_desc *d, const float *ids, int T, float *logits);

/* The same results, bit for bit, from vectorised kernels on `threads` threads
 * (0: every online CPU); tgo_mt.c says why the bits cannot differ. */
void tgo_matmul_qb_mt(float *o, const float *a, const signed char *q, int bits, const float *s, int m, int k, int n,
		      int threads);
int tgo_lm_forward_mt(const tg_cuda_lm_desc *d, const float *ids, int T, float *logits, int threads);

/* The stacked selective-SSM program (tg_cuda_ssm_desc) over one sequence of T
 * steps, u and out [T][d_model]. Scratch is allocated inside. */
int tgo_ssm_forward(const tg_cuda_ssm_desc *d, const float *u, int T, float *out);

#ifdef __cplusplus
}
#endif
#endif
