// gemv.cu -- weight-only dequant matmuls (W8A32 / W4A32) on CUDA cores: the
// small-batch regime of tg_matmul_qa / tg_matmul_qb (runtime/tg_rt.h:132-151),
// where the op streams codes from HBM once and is bandwidth-bound.
//
//   gemv_rows : axis 0, o[i,j] = s[i] sum_p code(i*k+p) b[p*n+j], n <= 8.
//               One warp owns 4 channel rows; each lane streams 16-byte code
//               chunks of those rows and keeps the matching activations in
//               registers, so one activation load feeds 4 rows.
//   gemv_cols : axis 1, o[i,j] = s[j] sum_p a[i*k+p] code(p*n+j), m <= 8.
//               A code row p is contiguous over channels j: each lane streams
//               4 bytes (8 int4 / 4 int8 channels) of row p; the K axis is split
//               over the 8 warps of a CTA and over CTAs, partial sums reduced in
//               a fixed order (deterministic, no atomics).
//   qmm_exact : any shape; one thread per output, products summed serially in
//               p order without contraction -- the reference's own rounding.
#include "common.cuh"
#include "gemv_cols.cuh"
#include "kernels.cuh"

namespace tgc {

// ---- axis 0 --------------------------------------------------------------------------

constexpr int GR_ROWS = 4;    // channel rows per warp
constexpr int GR_WARPS = 8;   // warps per CTA

template <int BITS, int NB>
__global__ void __launch_bounds__(GR_WARPS * 32) gemv_rows(float *__restrict__ o, const signed char *__restrict__ q,
							     const float *__restrict__ s, const float *__restrict__ b,
							     int m, int k)
{
	constexpr int CPC = BITS == 8 ? 16 : 32;  // codes per 16-byte chunk
	const int lane = threadIdx.x & 31;
	const int warp = blockIdx.x * GR_WARPS + (threadIdx.x >> 5);
	const int nwarps = gridDim.x * GR_WARPS;
	const long row_bytes = BITS == 8 ? (long)k : (long)k / 2;
	const int nchunks = k / CPC;
	for (int r0 = warp * GR_ROWS; r0 < m; r0 += nwarps * GR_ROWS) {
		float acc[GR_ROWS][NB];
#pragma unroll
		for (int r = 0; r < GR_ROWS; r++)
#pragma unroll
			for (int j = 0; j < NB; j++) acc[r][j] = 0.0f;
		for (int c = lane; c < nchunks; c += 32) {
			uint4 w[GR_ROWS];
#pragma unroll
			for (int r = 0; r < GR_ROWS; r++) {
				int row = r0 + r < m ? r0 + r : m - 1;
				w[r] = __ldg((const uint4 *)(q + (long)row * row_bytes + (long)c * 16));
			}
			const float *bp = b + (long)c * CPC * NB;
#pragma unroll
			for (int word = 0; word < 4; word++) {
				constexpr int PER = BITS == 8 ? 4 : 8; // codes per 32-bit word
				float bv[PER][NB];
#pragma unroll
				for (int e = 0; e < PER; e++)
#pragma unroll
					for (int j = 0; j < NB; j++) bv[e][j] = __ldg(bp + (word * PER + e) * NB + j);
#pragma unroll
				for (int r = 0; r < GR_ROWS; r++) {
					uint32_t x = word == 0 ? w[r].x : word == 1 ? w[r].y : word == 2 ? w[r].z : w[r].w;
#pragma unroll
					for (int e = 0; e < PER; e++) {
						float cf = BITS == 8 ? (float)(int)(int8_t)(x >> (8 * e))
								     : (float)((int32_t)(x << (28 - 4 * e)) >> 28);
#pragma unroll
						for (int j = 0; j < NB; j++) acc[r][j] = fmaf(cf, bv[e][j], acc[r][j]);
					}
				}
			}
		}
#pragma unroll
		for (int r = 0; r < GR_ROWS; r++)
#pragma unroll
			for (int j = 0; j < NB; j++) {
				float v = acc[r][j];
#pragma unroll
				for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
				acc[r][j] = v;
			}
		if (lane == 0)
#pragma unroll
			for (int r = 0; r < GR_ROWS; r++)
				if (r0 + r < m) {
					float sc = s[r0 + r];
#pragma unroll
					for (int j = 0; j < NB; j++) o[(long)(r0 + r) * NB + j] = sc * acc[r][j];
				}
	}
}

// axis 1: gemv_cols and reduce_splits live in gemv_cols.cuh

// ---- any shape, reference rounding ---------------------------------------------------------

__global__ void qmm_exact(float *__restrict__ o, const float *__restrict__ act, const signed char *__restrict__ q,
			  int bits, const float *__restrict__ s, int axis, int m, int k, int n)
{
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (t >= (long)m * n) return;
	int i = (int)(t / n), j = (int)(t % n);
	float acc = 0.0f;
	if (axis == 0) {
		for (int p = 0; p < k; p++)
			acc = __fadd_rn(acc, __fmul_rn((float)qcode(q, bits, (long)i * k + p), act[(long)p * n + j]));
		o[t] = __fmul_rn(s[i], acc);
	} else {
		for (int p = 0; p < k; p++)
			acc = __fadd_rn(acc, __fmul_rn(act[(long)i * k + p], (float)qcode(q, bits, (long)p * n + j)));
		o[t] = __fmul_rn(s[j], acc);
	}
}

// ---- dispatch ---------------------------------------------------------------------------------

struct Scratch {
	DevBuf buf;
};
static Scratch g_scratch[64];

static int scratch(size_t bytes, float **p)
{
	int dev;
	cudaGetDevice(&dev);
	if (dev < 0 || dev >= 64) return set_err(TG_CUDA_EINVAL, "device ordinal %d", dev);
	int rc = g_scratch[dev].buf.ensure(bytes, dev);
	if (rc) return rc;
	*p = g_scratch[dev].buf.as<float>();
	return TG_CUDA_OK;
}

static int sm_count()
{
	int dev, n = 148;
	cudaGetDevice(&dev);
	cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
	return n;
}

template <int BITS>
static void launch_rows(int nb, float *o, const signed char *q, const float *s, const float *b, int m, int k,
			cudaStream_t st)
{
	int rows_per_cta = GR_WARPS * GR_ROWS;
	int grid = (m + rows_per_cta - 1) / rows_per_cta;
	switch (nb) {
#define NB_CASE(N) \
	case N: gemv_rows<BITS, N><<<grid, GR_WARPS * 32, 0, st>>>(o, q, s, b, m, k); break;
		NB_CASE(1) NB_CASE(2) NB_CASE(3) NB_CASE(4) NB_CASE(5) NB_CASE(6) NB_CASE(7) NB_CASE(8)
#undef NB_CASE
	}
}

template <int BITS>
static int launch_cols(float *o, const float *a, const signed char *q, const float *s, int m, int k, int n,
		       cudaStream_t st)
{
	constexpr int CPW = BITS == 8 ? 4 : 8;
	int tiles = (n + 32 * CPW - 1) / (32 * CPW);
	int want = (4 * sm_count() + tiles - 1) / tiles; // about four CTAs per SM
	int splits = want < 1 ? 1 : want > k / 64 ? (k / 64 > 0 ? k / 64 : 1) : want;
	int kper = (k + splits - 1) / splits;
	splits = (k + kper - 1) / kper;
	float *part = nullptr;
	int rc = scratch((size_t)splits * m * n * sizeof(float), &part);
	if (rc) return rc;
	dim3 grid(tiles, splits);
	switch (m) {
#define MB_CASE(M) \
	case M: gemv_cols<BITS, M><<<grid, GC_WARPS * 32, 0, st>>>(part, a, q, m, k, n, kper); break;
		MB_CASE(1) MB_CASE(2) MB_CASE(3) MB_CASE(4) MB_CASE(5) MB_CASE(6) MB_CASE(7) MB_CASE(8)
#undef MB_CASE
	}
	long tot = (long)m * n;
	reduce_splits<<<(unsigned)((tot + 255) / 256), 256, 0, st>>>(o, part, s, m, n, splits);
	return TG_CUDA_OK;
}

int matmul_q_exact(int axis, float *o, const float *act, const signed char *q, int bits, const float *s, int m, int k,
		   int n, cudaStream_t st)
{
	long tot = (long)m * n;
	qmm_exact<<<(unsigned)((tot + 255) / 256), 256, 0, st>>>(o, act, q, bits, s, axis, m, k, n);
	TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

int matmul_q_gemv(int axis, float *o, const float *act, const signed char *q, int bits, const float *s, int m, int k,
		  int n, cudaStream_t st, bool *done)
{
	*done = false;
	bool aligned16 = ((uintptr_t)q & 15) == 0;
	if (axis == 0 && n <= 8 && aligned16 && k % (bits == 8 ? 16 : 32) == 0) {
		if (bits == 8) launch_rows<8>(n, o, q, s, act, m, k, st);
		else launch_rows<4>(n, o, q, s, act, m, k, st);
		*done = true;
	} else if (axis == 1 && m <= 8 && ((uintptr_t)q & 3) == 0 && n % (bits == 8 ? 4 : 8) == 0) {
		int rc = bits == 8 ? launch_cols<8>(o, act, q, s, m, k, n, st) : launch_cols<4>(o, act, q, s, m, k, n, st);
		if (rc) return rc;
		*done = true;
	}
	if (*done) TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

} // namespace tgc
