// gemv_cols.cuh -- the axis-1 dequant GEMV (tg_matmul_qb, runtime/tg_rt.h:143-151) for
// batches of at most 8 rows: split-K partial sums into a caller-provided buffer, then a
// fixed-order reduction. Shared by tg_cuda_matmul_q (gemv.cu, library-owned scratch)
// and tg_cuda_matmul_qb_noalloc (noalloc.cu, a static device array).
#pragma once

#include "common.cuh"

namespace tgc {

// ---- axis 1 --------------------------------------------------------------------------

constexpr int GC_WARPS = 8;

// part[split][i][j] = sum over this CTA's K range of a[i,p] code(p,j); the CTA's 8 warps
// each take a contiguous sub-range and are reduced through shared memory in warp order.
template <int BITS, int MB>
__global__ void __launch_bounds__(GC_WARPS * 32) gemv_cols(float *__restrict__ part, const float *__restrict__ a,
							     const signed char *__restrict__ q, int m, int k, int n,
							     int kper)
{
	constexpr int CPW = BITS == 8 ? 4 : 8; // channels per 32-bit word
	__shared__ float red[GC_WARPS][32 * CPW];
	const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
	const int col0 = (blockIdx.x * 32 + lane) * CPW;
	const int split = blockIdx.y;
	const int kb = split * kper, ke = min(k, kb + kper);
	const int wper = (kper + GC_WARPS - 1) / GC_WARPS;
	const int pb = kb + warp * wper, pe = min(ke, pb + wper);
	const long row_bytes = BITS == 8 ? (long)n : (long)n / 2;
	float acc[MB][CPW];
#pragma unroll
	for (int i = 0; i < MB; i++)
#pragma unroll
		for (int e = 0; e < CPW; e++) acc[i][e] = 0.0f;
	if (col0 < n)
		for (int p = pb; p < pe; p++) {
			uint32_t x = __ldg((const uint32_t *)(q + (long)p * row_bytes + (BITS == 8 ? col0 : col0 / 2)));
			float av[MB];
#pragma unroll
			for (int i = 0; i < MB; i++) av[i] = i < m ? __ldg(a + (long)i * k + p) : 0.0f;
#pragma unroll
			for (int e = 0; e < CPW; e++) {
				float cf = BITS == 8 ? (float)(int)(int8_t)(x >> (8 * e)) : (float)((int32_t)(x << (28 - 4 * e)) >> 28);
#pragma unroll
				for (int i = 0; i < MB; i++) acc[i][e] = fmaf(av[i], cf, acc[i][e]);
			}
		}
#pragma unroll
	for (int i = 0; i < MB; i++) {
		if (i >= m) break;
#pragma unroll
		for (int e = 0; e < CPW; e++) red[warp][lane * CPW + e] = acc[i][e];
		__syncthreads();
		for (int c = threadIdx.x; c < 32 * CPW; c += blockDim.x) {
			int col = blockIdx.x * 32 * CPW + c;
			if (col >= n) continue;
			float v = 0.0f;
			for (int w = 0; w < GC_WARPS; w++) v += red[w][c];
			part[((long)split * m + i) * n + col] = v;
		}
		__syncthreads();
	}
}

static __global__ void reduce_splits(float *__restrict__ o, const float *__restrict__ part, const float *__restrict__ s,
			      int m, int n, int splits)
{
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (t >= (long)m * n) return;
	int j = (int)(t % n);
	float v = 0.0f;
	for (int z = 0; z < splits; z++) v += part[(long)z * m * n + t];
	o[t] = s[j] * v;
}

} // namespace tgc
