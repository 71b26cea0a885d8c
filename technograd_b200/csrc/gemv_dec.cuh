// gemv_dec.cuh -- the decoder's dequant GEMV for batches of at most 8 rows (decode steps of
// small waves): out[j, i] (+)= s[i] sum_p code(i, p) (hi[j, p] + lo[j, p]), codes [m][k]
// K-major (int4 two per byte, low nibble first), activations as the decoder keeps them (bf16
// hi/lo rows; hi + lo is exact in f32). Grouped scales (o_proj's per-head column scales):
// s[(p / group) * s_ld + i] multiplies the partial sum of each group of K positions.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace tgc {

enum { GD_STORE = 0, GD_ADD = 1 };

struct GemvDecArgs {
	const __nv_bfloat16 *hi, *lo; // activation rows j < nb, row stride lda elements
	// or, with x set: the activations are rmsnorm(x[j]) * nw (f32 rows of stride lda; the
	// arithmetic of the decoder's rmsnorm kernel), and hi / lo are not read
	const float *x, *nw;
	float eps;
	long lda;
	int nb;                       // 1..8
	const signed char *q;         // codes [m][k]
	int m, k, bits;
	const float *s;               // per row (nullptr: 1), or per (group, row) when group > 0
	int group;                    // K positions per scale group (a multiple of 32), 0: per row
	long s_ld;
	float *out;                   // out[j * ldo + i]
	long ldo;
	int epi;                      // GD_STORE / GD_ADD
	int rows;                     // rows per CTA (set by gemv_dec)
};

// Whether gemv_dec takes this shape: k a multiple of 32 codes (one 16-byte int4 chunk, two of
// int8) and at most 3200 (8 rows' activations, as copied and as staged, in shared memory),
// 16-byte aligned code rows and activation rows (lda a multiple of 8 for hi / lo, of 4 for x).
bool gemv_dec_fits(const GemvDecArgs &a);
// Launch on st, with programmatic stream serialization when pdl.
int gemv_dec(GemvDecArgs a, cudaStream_t st, bool pdl);
// Kernel attributes (once per device, outside any stream capture).
int gemv_dec_prepare();

} // namespace tgc
