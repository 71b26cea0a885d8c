// gemv.cu -- weight-only dequant matmuls (W8A32 / W4A32) on CUDA cores: the
// small-batch regime of tg_matmul_qa / tg_matmul_qb (runtime/tg_rt.h:132-151),
// where the op streams codes from HBM once and is bandwidth-bound.
//
//   gemv_bulk : axis 0, o[i,j] = s[i] sum_p code(i*k+p) b[p*n+j], n <= 8, when the
//               activations fit in shared memory twice (gemv_bulk.cuh): warps read
//               code rows coalesced into registers, one wave of CTAs over the SMs.
//   gemv_rows : the same op for activations too large for that. A lane owns a
//               channel row and a warp one K slice of 32 rows; the activations of
//               the slice are shared by the 32 lanes.
//   gemv_cols : axis 1, o[i,j] = s[j] sum_p a[i*k+p] code(p*n+j), m <= 8.
//               A code row p is contiguous over channels j: each lane streams
//               4 bytes (8 int4 / 4 int8 channels) of row p; the K axis is split
//               over the 8 warps of a CTA and over CTAs, partial sums reduced in
//               a fixed order (deterministic, no atomics).
//   qmm_exact : any shape; one thread per output, products summed serially in
//               p order without contraction -- the reference's own rounding.
#include "common.cuh"
#include "gemm.cuh"
#include "gemv_bulk.cuh"
#include "gemv_cols.cuh"
#include "kernels.cuh"

namespace tgc {

// ---- axis 0 --------------------------------------------------------------------------
// Lane = channel row: a warp takes 32 rows and one K slice, so every lane needs the same
// activations (broadcast reads of b, staged once per CTA in shared memory when it fits)
// and loads 16-byte code chunks of its own row, U at a time. The KS warps of a CTA take
// the KS slices of the same 32 rows; their partial sums are added in a fixed order.
// Codes become floats without an int-to-float conversion: 2^23 + the unsigned code read as
// an f32, minus 2^23 + the code offset, is exact.

constexpr int GR_U = 4; // 16-byte chunks in flight per lane

template <int BITS, int NB, int KS, bool SMB>
__global__ void __launch_bounds__(32 * KS) gemv_rows(float *__restrict__ o, const signed char *__restrict__ q,
						     const float *__restrict__ s, const float *__restrict__ b, int m, int k)
{
	constexpr int CPC = BITS == 8 ? 16 : 32; // codes per 16-byte chunk
	constexpr int PER = BITS == 8 ? 4 : 8;   // codes per 32-bit word
	__shared__ float part[KS][32][NB];
	extern __shared__ float4 sb4[];          // SMB: b [k][NB]
	const int lane = threadIdx.x & 31, ks = threadIdx.x >> 5;
	const int row = blockIdx.x * 32 + lane;
	const long row_bytes = (long)k * BITS / 8;
	const int nchunks = k / CPC, cper = (nchunks + KS - 1) / KS;
	const int c0 = ks * cper, c1 = min(nchunks, c0 + cper);
	const signed char *qr = q + (long)min(row, m - 1) * row_bytes;
	// this CTA's code rows into L2 while the kernel before it may still run (launched with
	// programmatic serialization), then wait for it: the activations and the output may be its
	const int r0 = blockIdx.x * 32, nr = min(32, m - r0);
	if (threadIdx.x == 0 && nr > 0 && (row_bytes & 15) == 0 && ((uintptr_t)q & 15) == 0)
		prefetch_l2(q + (long)r0 * row_bytes, (uint32_t)(nr * row_bytes));
	pdl_wait();
	pdl_launch();
	if (SMB) {
		for (int i = threadIdx.x; i < k * NB / 4; i += blockDim.x) sb4[i] = ((const float4 *)b)[i];
		__syncthreads();
	}
	float acc[NB];
#pragma unroll
	for (int j = 0; j < NB; j++) acc[j] = 0.0f;
	for (int cb = c0; cb < c1; cb += GR_U) {
		uint4 w[GR_U];
#pragma unroll
		for (int u = 0; u < GR_U; u++) w[u] = cb + u < c1 ? __ldg((const uint4 *)(qr + (long)(cb + u) * 16)) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
		for (int u = 0; u < GR_U; u++) {
			if (cb + u >= c1) break;
			const float4 *bp = SMB ? sb4 + (long)(cb + u) * CPC * NB / 4 : (const float4 *)(b + (long)(cb + u) * CPC * NB);
#pragma unroll
			for (int word = 0; word < 4; word++) {
				const uint32_t x = word == 0 ? w[u].x : word == 1 ? w[u].y : word == 2 ? w[u].z : w[u].w;
				float bv[PER * NB];
#pragma unroll
				for (int i = 0; i < PER * NB / 4; i++) {
					const float4 t = bp[word * PER * NB / 4 + i];
					bv[4 * i] = t.x, bv[4 * i + 1] = t.y, bv[4 * i + 2] = t.z, bv[4 * i + 3] = t.w;
				}
#pragma unroll
				for (int e = 0; e < PER; e++) {
					const float cf = BITS == 8 ? __int_as_float(0x4B000000 | (((x >> (8 * e)) & 0xFF) ^ 0x80)) - 8388736.0f
								   : __int_as_float(0x4B000000 | (((x >> (4 * e)) & 0xF) ^ 0x8)) - 8388616.0f;
#pragma unroll
					for (int j = 0; j < NB; j++) acc[j] = fmaf(cf, bv[e * NB + j], acc[j]);
				}
			}
		}
	}
#pragma unroll
	for (int j = 0; j < NB; j++) part[ks][lane][j] = acc[j];
	__syncthreads();
	if (ks == 0 && row < m)
#pragma unroll
		for (int j = 0; j < NB; j++) {
			float v = part[0][lane][j];
			for (int i = 1; i < KS; i++) v += part[i][lane][j];
			o[(long)row * NB + j] = s[row] * v;
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

template <int BITS, int NB>
static int launch_rows_nb(float *o, const signed char *q, const float *s, const float *b, int m, int k, cudaStream_t st)
{
	constexpr int KS = NB == 1 ? 32 : 16;
	const unsigned grid = (unsigned)((m + 31) / 32);
	const size_t smem = (size_t)k * NB * 4;
	if (smem <= 96 * 1024) {
		static bool attr[64] = {};
		int dev = 0;
		cudaGetDevice(&dev);
		if (!attr[dev]) {
			cudaFuncSetAttribute(gemv_rows<BITS, NB, KS, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
			attr[dev] = true;
		}
		TGC_CUDA(launch_pdl(gemv_rows<BITS, NB, KS, true>, dim3(grid), dim3(32 * KS), smem, st, o, q, s, b, m, k));
	} else {
		TGC_CUDA(launch_pdl(gemv_rows<BITS, NB, KS, false>, dim3(grid), dim3(32 * KS), 0, st, o, q, s, b, m, k));
	}
	return TG_CUDA_OK;
}

// gemv_bulk: rows per CTA so that the grid is one wave over the SMs (a multiple of the rows
// per warp, at most 16 warps); shared memory holds the activations twice.
constexpr size_t GB_SMEM_MAX = 200 * 1024;

static bool bulk_fits(int nb, int k) { return gemv_bulk_smem(nb, k) <= GB_SMEM_MAX; }

template <int BITS, int NB, int NCHL>
static int launch_bulk_nb(float *o, const signed char *q, const float *s, const float *b, int m, int k, cudaStream_t st)
{
	int dev = 0;
	cudaGetDevice(&dev);
	int *status = nullptr;
	int rc = call_status_word(dev, &status);
	if (rc) return rc;
	static bool attr[64] = {};
	if (!attr[dev]) {
		TGC_CUDA(cudaFuncSetAttribute(gemv_bulk<BITS, NB, NCHL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GB_SMEM_MAX));
		attr[dev] = true;
	}
	constexpr int RR = GemvBulkTile<NB>::RR;
	const int sms = sm_count();
	int rows = (m + sms - 1) / sms;
	rows = rows < RR ? RR : rows > RR * GB_MAX_WARPS ? RR * GB_MAX_WARPS : (rows + RR - 1) / RR * RR;
	const unsigned grid = (unsigned)((m + rows - 1) / rows);
	const unsigned threads = (unsigned)(32 * (rows / RR));
	TGC_CUDA(launch_pdl(gemv_bulk<BITS, NB, NCHL>, dim3(grid), dim3(threads), gemv_bulk_smem(NB, k), st, o, q, s, b, m, k, rows,
			    status));
	return TG_CUDA_OK;
}

template <int BITS>
static int launch_bulk(int nb, float *o, const signed char *q, const float *s, const float *b, int m, int k, cudaStream_t st)
{
	// batches of one or two columns whose rows are exactly 32, 64, 96 or 128 chunks (k = 1024 ...
	// 4096 int4, 512 ... 2048 int8) get the unrolled kernel without predicates
	const int per_lane = k / (BITS == 8 ? 16 : 32) % 32 == 0 ? k / (BITS == 8 ? 16 : 32) / 32 : 0;
#define GB_EXACT(NB)                                                                               \
	switch (per_lane) {                                                                         \
	case 1: return launch_bulk_nb<BITS, NB, 1>(o, q, s, b, m, k, st);                           \
	case 2: return launch_bulk_nb<BITS, NB, 2>(o, q, s, b, m, k, st);                           \
	case 3: return launch_bulk_nb<BITS, NB, 3>(o, q, s, b, m, k, st);                           \
	case 4: return launch_bulk_nb<BITS, NB, 4>(o, q, s, b, m, k, st);                           \
	default: return launch_bulk_nb<BITS, NB, 0>(o, q, s, b, m, k, st);                          \
	}
	switch (nb) {
	case 1: GB_EXACT(1)
	case 2: GB_EXACT(2)
	case 3: return launch_bulk_nb<BITS, 3, 0>(o, q, s, b, m, k, st);
	case 4: return launch_bulk_nb<BITS, 4, 0>(o, q, s, b, m, k, st);
	case 5: return launch_bulk_nb<BITS, 5, 0>(o, q, s, b, m, k, st);
	case 6: return launch_bulk_nb<BITS, 6, 0>(o, q, s, b, m, k, st);
	case 7: return launch_bulk_nb<BITS, 7, 0>(o, q, s, b, m, k, st);
	default: return launch_bulk_nb<BITS, 8, 0>(o, q, s, b, m, k, st);
	}
#undef GB_EXACT
}

template <int BITS>
static int launch_rows(int nb, float *o, const signed char *q, const float *s, const float *b, int m, int k, cudaStream_t st)
{
	switch (nb) {
	case 1: return launch_rows_nb<BITS, 1>(o, q, s, b, m, k, st);
	case 2: return launch_rows_nb<BITS, 2>(o, q, s, b, m, k, st);
	case 3: return launch_rows_nb<BITS, 3>(o, q, s, b, m, k, st);
	case 4: return launch_rows_nb<BITS, 4>(o, q, s, b, m, k, st);
	case 5: return launch_rows_nb<BITS, 5>(o, q, s, b, m, k, st);
	case 6: return launch_rows_nb<BITS, 6>(o, q, s, b, m, k, st);
	case 7: return launch_rows_nb<BITS, 7>(o, q, s, b, m, k, st);
	default: return launch_rows_nb<BITS, 8>(o, q, s, b, m, k, st);
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
	bool aligned16 = ((uintptr_t)q & 15) == 0 && ((uintptr_t)act & 15) == 0;
	if (axis == 0 && n <= 8 && aligned16 && k % (bits == 8 ? 16 : 32) == 0) {
		int rc = bulk_fits(n, k) ? (bits == 8 ? launch_bulk<8>(n, o, q, s, act, m, k, st) : launch_bulk<4>(n, o, q, s, act, m, k, st))
					 : (bits == 8 ? launch_rows<8>(n, o, q, s, act, m, k, st) : launch_rows<4>(n, o, q, s, act, m, k, st));
		if (rc) return rc;
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
