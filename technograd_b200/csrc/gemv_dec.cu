// gemv_dec.cu -- the decoder's dequant GEMV (gemv_dec.cuh) on the code decode of gemv_bulk.cuh.
//
// A CTA first stages the activations of every K position once: the live bf16 hi and lo rows
// are copied into shared memory by 16-byte cp.async copies, all in flight at once (with the
// warps' first code loads), then each value hi + lo (exact in f32), divided by the place value
// of its code, is written into the swizzled chunk layout the decode reads. The CTA then takes
// blocks of `rows` consecutive code rows in turn (RR rows per warp): each warp
// streams its rows' 16-byte code chunks (lane j: chunks j, j + 32, ...), the next register
// block (or the next row block's first) in flight while it computes one, and sums over the
// warp with a fixed butterfly (deterministic). Grouped scales: a chunk lies inside one group,
// so each lane's partial sums of a chunk are multiplied by that group's scale before they
// join the row's sum.
//
// The codes are constant weights: a CTA asks L2 to prefetch its first row block before it
// waits for the kernel ahead of it (programmatic launch), and each next block while it
// computes one.
#include <algorithm>

#include "gemv_bulk.cuh"
#include "gemv_dec.cuh"

namespace tgc {

constexpr size_t GD_SMEM_MAX = 200 * 1024;
// Rows per warp and code chunks per lane and row in one register block. More rows than
// gemv_bulk's tile: every staged activation read from shared memory then feeds RR rows, which
// is what bounds a batch of 4 or 8 columns.
template <int NB> struct GemvDecTile {
	static constexpr int RR = NB <= 4 ? 4 : 2, BLK = NB <= 2 ? 2 : 1;
};
constexpr int GD_THREADS = 32 * GB_MAX_WARPS;

__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
	asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// every cp.async of this thread has landed (the hardware completes them; nothing spins)
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Shared memory: the staged activations (k * NB floats), then the copied bf16 rows (hi rows
// then lo rows, NB rows of k each).
__host__ __device__ constexpr size_t gemv_dec_smem(int nb, int k) { return (size_t)k * nb * 8; }

template <int BITS, int NB, int EPI, bool GROUPED>
__global__ void __launch_bounds__(GD_THREADS, 1) gemv_dec_k(const GemvDecArgs a)
{
	using S = GemvBulkShape<BITS, NB>;
	constexpr int RR = GemvDecTile<NB>::RR, BLK = GemvDecTile<NB>::BLK;
	extern __shared__ __align__(128) unsigned char smem[];
	float *sbf = (float *)smem;
	const float4 *sb = (const float4 *)smem;
	__nv_bfloat16 *raw = (__nv_bfloat16 *)(smem + (size_t)a.k * NB * 4);
	const long row_bytes = (long)a.k * BITS / 8;
	const int nch = a.k / S::CPC, k8 = a.k / 8;
	const int nblk = (a.m + a.rows - 1) / a.rows; // blocks of `rows` rows, taken in turn by the CTAs
	const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
	auto block_rows = [&](int rb) { return min(a.rows, a.m - rb * a.rows); };
	auto warp_rows = [&](int rb) { return max(0, min(RR, block_rows(rb) - RR * w)); };
	// chunks c0 + 32 t + lane of this warp's rows of block rb
	auto load_block = [&](uint4 (&dst)[RR][BLK], int rb, int c0) {
		const int rw = warp_rows(rb);
		const uint4 *gq = (const uint4 *)(a.q + ((long)rb * a.rows + RR * w) * row_bytes);
#pragma unroll
		for (int r = 0; r < RR; r++)
#pragma unroll
			for (int t = 0; t < BLK; t++) {
				const int c = c0 + 32 * t + lane;
				dst[r][t] = r < rw && c < nch ? __ldg(gq + (long)r * nch + c) : make_uint4(0u, 0u, 0u, 0u);
			}
	};
	if (threadIdx.x == 0) prefetch_l2(a.q + (long)blockIdx.x * a.rows * row_bytes, (uint32_t)(block_rows(blockIdx.x) * row_bytes));
	pdl_wait(); // the activations come from the kernel ahead of this one
	pdl_launch();
	// the live activation rows into shared memory, 16 bytes per copy, all in flight at once
	const bool norm = a.x != nullptr;
	float *rawf = (float *)raw; // norm: the f32 rows x[j]
	const int k4 = a.k / 4;
	if (norm)
		for (int i = threadIdx.x; i < a.nb * k4; i += blockDim.x) {
			const int j = i / k4, p4 = i - j * k4;
			cp_async16(rawf + (size_t)j * a.k + 4 * p4, a.x + (long)j * a.lda + 4 * p4);
		}
	else
		for (int i = threadIdx.x; i < 2 * a.nb * k8; i += blockDim.x) {
			const int row = i / k8, p8 = i - row * k8, plane = row >= a.nb, j = row - plane * a.nb;
			cp_async16(raw + ((size_t)(plane * NB + j) * a.k + 8 * p8), (plane ? a.lo : a.hi) + (long)j * a.lda + 8 * p8);
		}
	uint4 qa[RR][BLK]; // this warp's first register block, in flight with the copies
	load_block(qa, blockIdx.x, 0);
	cp_async_wait_all();
	__syncthreads();
	if (norm) {
		// 1 / rms of row j by warp j, in the rmsnorm kernel's order (lane-strided FMAs, then a
		// butterfly), so each activation is the value that kernel computes
		__shared__ float rinv[NB];
		if (w < a.nb) {
			const float *xr = rawf + (size_t)w * a.k;
			float ss = 0.0f;
			for (int i = lane; i < a.k; i += 32) ss = fmaf(xr[i], xr[i], ss);
#pragma unroll
			for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
			if (lane == 0) rinv[w] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.k), a.eps)));
		}
		__syncthreads();
		// activation (j, p) = (x * inv) * nw, placed as below (a float4 of positions per item)
		for (int i = threadIdx.x; i < NB * k4; i += blockDim.x) {
			const int j = i / k4, p0 = 4 * (i - j * k4);
			float4 xv = make_float4(0.f, 0.f, 0.f, 0.f), wv = xv;
			float inv = 0.0f;
			if (j < a.nb) {
				xv = *(const float4 *)(rawf + (size_t)j * a.k + p0);
				wv = __ldg((const float4 *)(a.nw + p0));
				inv = rinv[j];
			}
			const float xs[4] = { xv.x, xv.y, xv.z, xv.w }, ws[4] = { wv.x, wv.y, wv.z, wv.w };
#pragma unroll
			for (int e = 0; e < 4; e++) {
				const int p = p0 + e, c = p / S::CPC, pc = p % S::CPC, f = pc * NB + j;
				sbf[4 * (c * S::UPC + S::swz(c, f >> 2)) + (f & 3)] = __fmul_rn(__fmul_rn(xs[e], inv), ws[e]) * S::place(pc);
			}
		}
	} else
	// activation (j, p) = hi + lo (exact) -> chunk c = p / CPC, float f = (p % CPC) * NB + j of
	// the chunk's units, divided by its code's place value; rows j >= nb stage as zeros
	for (int i = threadIdx.x; i < NB * k8; i += blockDim.x) {
		const int j = i / k8, p0 = 8 * (i - j * k8);
		uint4 h = make_uint4(0u, 0u, 0u, 0u), l = h;
		if (j < a.nb) {
			h = *(const uint4 *)(raw + (size_t)j * a.k + p0);
			l = *(const uint4 *)(raw + (size_t)(NB + j) * a.k + p0);
		}
		const uint32_t hw[4] = { h.x, h.y, h.z, h.w }, lw[4] = { l.x, l.y, l.z, l.w };
#pragma unroll
		for (int e = 0; e < 8; e++) {
			const uint32_t hb = e & 1 ? hw[e >> 1] & 0xFFFF0000u : hw[e >> 1] << 16;
			const uint32_t lb = e & 1 ? lw[e >> 1] & 0xFFFF0000u : lw[e >> 1] << 16;
			const int p = p0 + e, c = p / S::CPC, pc = p % S::CPC, f = pc * NB + j;
			sbf[4 * (c * S::UPC + S::swz(c, f >> 2)) + (f & 3)] = __fadd_rn(__uint_as_float(hb), __uint_as_float(lb)) * S::place(pc);
		}
	}
	__syncthreads();
	const CodeConsts<BITS> cc;
	for (int rb = blockIdx.x; rb < nblk; rb += gridDim.x) {
		const int rbn = rb + gridDim.x, r0 = rb * a.rows, rw = warp_rows(rb);
		if (threadIdx.x == 0 && rbn < nblk) // the CTA's next block into L2 meanwhile
			prefetch_l2(a.q + (long)rbn * a.rows * row_bytes, (uint32_t)(block_rows(rbn) * row_bytes));
		float2 acc[RR][S::NP];
#pragma unroll
		for (int r = 0; r < RR; r++)
#pragma unroll
			for (int h = 0; h < S::NP; h++) acc[r][h] = make_float2(0.0f, 0.0f);
		for (int c0 = 0; c0 < nch; c0 += 32 * BLK) {
			// the next register block (of this row block, else the next one's first) in flight
			// while this one is computed
			uint4 qn[RR][BLK];
			const bool more = c0 + 32 * BLK < nch, next = !more && rbn < nblk;
			if (more) load_block(qn, rb, c0 + 32 * BLK);
			else if (next) load_block(qn, rbn, 0);
			if (rw > 0) {
				if (GROUPED) {
#pragma unroll
					for (int t = 0; t < BLK; t++) {
						float2 part[RR][S::NP];
						uint4 q1[RR][1];
#pragma unroll
						for (int r = 0; r < RR; r++) {
							q1[r][0] = qa[r][t];
#pragma unroll
							for (int h = 0; h < S::NP; h++) part[r][h] = make_float2(0.0f, 0.0f);
						}
						gemv_bulk_block<BITS, NB, RR, 1, false>(part, q1, sb, c0 + 32 * t, nch, lane, cc);
						const int c = c0 + 32 * t + lane;
#pragma unroll
						for (int r = 0; r < RR; r++) {
							const float sc =
								r < rw && c < nch ? a.s[(long)(c * S::CPC / a.group) * a.s_ld + r0 + RR * w + r] : 0.0f;
#pragma unroll
							for (int h = 0; h < S::NP; h++) acc[r][h] = __ffma2_rn(make_float2(sc, sc), part[r][h], acc[r][h]);
						}
					}
				} else {
					gemv_bulk_block<BITS, NB, RR, BLK, false>(acc, qa, sb, c0, nch, lane, cc);
				}
			}
			if (more || next)
#pragma unroll
				for (int r = 0; r < RR; r++)
#pragma unroll
					for (int t = 0; t < BLK; t++) qa[r][t] = qn[r][t];
		}
		if (rw == 0) continue;
#pragma unroll
		for (int r = 0; r < RR; r++) {
			float v[NB];
			if (NB == 1) {
				v[0] = acc[r][0].x + acc[r][0].y;
			} else {
#pragma unroll
				for (int jj = 0; jj < NB; jj++) v[jj] = jj & 1 ? acc[r][jj >> 1].y : acc[r][jj >> 1].x;
			}
#pragma unroll
			for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
				for (int jj = 0; jj < NB; jj++) v[jj] += __shfl_xor_sync(0xffffffffu, v[jj], off);
			if (lane == 0 && r < rw) {
				const long row = r0 + RR * w + r;
				const float sc = GROUPED || !a.s ? 1.0f : a.s[row];
#pragma unroll
				for (int jj = 0; jj < NB; jj++) {
					if (jj >= a.nb) break;
					const float y = __fmul_rn(sc, v[jj]);
					float *o = a.out + jj * a.ldo + row;
					*o = EPI == GD_ADD ? __fadd_rn(*o, y) : y;
				}
			}
		}
	}
}

bool gemv_dec_fits(const GemvDecArgs &a)
{
	return a.nb >= 1 && a.nb <= 8 && (a.bits == 4 || a.bits == 8) && a.m >= 1 && a.k >= 32 && a.k % 32 == 0 &&
	       !((uintptr_t)a.q & 15) && gemv_dec_smem(8, a.k) <= GD_SMEM_MAX &&
	       (a.x ? a.nw && a.lda % 4 == 0 && !((uintptr_t)a.x & 15) && !((uintptr_t)a.nw & 15)
		    : a.lda % 8 == 0 && !((uintptr_t)a.hi & 15) && !((uintptr_t)a.lo & 15)) &&
	       (a.group == 0 || (a.s && a.group % 32 == 0));
}

static int sms_of_device()
{
	static int n[64] = {};
	int dev = 0;
	cudaGetDevice(&dev);
	if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
	return n[dev] ? n[dev] : 148;
}

template <int BITS, int NB, int EPI, bool G>
static int launch(GemvDecArgs a, cudaStream_t st, bool pdl)
{
	constexpr int RR = GemvDecTile<NB>::RR;
	const int sms = sms_of_device();
	// rows per block: the rows over the SMs (a multiple of RR, at most 16 warps' worth); one CTA
	// per SM stages the activations once (all 16 warps copy and convert) and takes blocks in turn
	int rows = (a.m + sms - 1) / sms;
	rows = rows < RR ? RR : rows > RR * GB_MAX_WARPS ? RR * GB_MAX_WARPS : (rows + RR - 1) / RR * RR;
	a.rows = rows;
	const long nblk = (a.m + rows - 1) / rows;
	const dim3 grid((unsigned)std::min<long>(nblk, sms)), block(GD_THREADS);
	const size_t smem = gemv_dec_smem(NB, a.k);
	if (pdl) {
		TGC_CUDA(launch_pdl(gemv_dec_k<BITS, NB, EPI, G>, grid, block, smem, st, (const GemvDecArgs)a));
	} else {
		gemv_dec_k<BITS, NB, EPI, G><<<grid, block, smem, st>>>(a);
		TGC_LAUNCH_CHECK();
	}
	return TG_CUDA_OK;
}

template <int BITS, int NB>
static int launch_nb(const GemvDecArgs &a, cudaStream_t st, bool pdl)
{
	if (a.group) return a.epi == GD_ADD ? launch<BITS, NB, GD_ADD, true>(a, st, pdl) : launch<BITS, NB, GD_STORE, true>(a, st, pdl);
	return a.epi == GD_ADD ? launch<BITS, NB, GD_ADD, false>(a, st, pdl) : launch<BITS, NB, GD_STORE, false>(a, st, pdl);
}

template <int BITS>
static int launch_bits(const GemvDecArgs &a, cudaStream_t st, bool pdl)
{
	// batches pad to 1, 2, 4 or 8 columns (the padding stages zeros and is not stored)
	if (a.nb <= 1) return launch_nb<BITS, 1>(a, st, pdl);
	if (a.nb <= 2) return launch_nb<BITS, 2>(a, st, pdl);
	if (a.nb <= 4) return launch_nb<BITS, 4>(a, st, pdl);
	return launch_nb<BITS, 8>(a, st, pdl);
}

int gemv_dec(GemvDecArgs a, cudaStream_t st, bool pdl)
{
	if (!gemv_dec_fits(a)) return set_err(TG_CUDA_EINVAL, "gemv_dec: unsupported shape (nb %d, k %d, bits %d)", a.nb, a.k, a.bits);
	return a.bits == 8 ? launch_bits<8>(a, st, pdl) : launch_bits<4>(a, st, pdl);
}

template <int BITS, int NB>
static int prepare_nb()
{
	TGC_CUDA(cudaFuncSetAttribute(gemv_dec_k<BITS, NB, GD_STORE, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GD_SMEM_MAX));
	TGC_CUDA(cudaFuncSetAttribute(gemv_dec_k<BITS, NB, GD_ADD, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GD_SMEM_MAX));
	TGC_CUDA(cudaFuncSetAttribute(gemv_dec_k<BITS, NB, GD_STORE, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GD_SMEM_MAX));
	TGC_CUDA(cudaFuncSetAttribute(gemv_dec_k<BITS, NB, GD_ADD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GD_SMEM_MAX));
	return TG_CUDA_OK;
}

int gemv_dec_prepare()
{
	static bool done[64] = {};
	int dev = 0;
	cudaGetDevice(&dev);
	if (done[dev]) return TG_CUDA_OK;
	int rc;
	if ((rc = prepare_nb<4, 1>()) || (rc = prepare_nb<4, 2>()) || (rc = prepare_nb<4, 4>()) || (rc = prepare_nb<4, 8>()) ||
	    (rc = prepare_nb<8, 1>()) || (rc = prepare_nb<8, 2>()) || (rc = prepare_nb<8, 4>()) || (rc = prepare_nb<8, 8>()))
		return rc;
	done[dev] = true;
	return TG_CUDA_OK;
}

} // namespace tgc
