// gemv_bulk.cuh -- the axis-0 dequant GEMV (tg_matmul_qa, runtime/tg_rt.h:132-142) for
// batches of at most 8 columns, o[i,j] = s[i] sum_p code(i*k+p) b[p*n+j].
//
// A CTA takes R consecutive channel rows (R chosen so that the grid is one wave over the
// SMs); a warp takes RR of them. Lane j reads the 16-byte code chunks j, j + 32, j + 64, ...
// of the warp's rows straight into registers (a warp instruction reads 512 contiguous bytes
// of a row), a block of 4 chunks per row ahead of the one it computes. The activations are
// brought into shared memory by one bulk copy (cp.async.bulk, completion counted on an
// mbarrier), then scaled and swizzled in place for the decode below; each activation read
// serves RR rows. The rows' partial sums are combined over the warp with a butterfly of
// shuffles, in a fixed order (deterministic).
//
// Decoding without shifts: a nibble (byte) left in place at bits 4e..4e+3 (8e..8e+7) of a
// half-word, XORed with its sign bit and OR'd under the exponent of 2^23, is the float
// 2^23 + 16^e (code + 8) (2^23 + 256^e (code + 128)) exactly: every such value is below
// 2^24. Two codes of a half-word are decoded by one LOP3 each and one packed f32x2
// subtraction, which leaves 16^e code (256^e code) exactly; the activation it multiplies
// was staged divided by 16^e (256^e), a power of two, so each product is the same
// correctly rounded value as code * activation (barring activations below 2^-114, which
// lose low bits to the subnormal range). Products are summed by packed f32x2 FMAs.
//
// The activations of chunk c (CPC codes x NB columns, UPC float4 units) sit at units
// c*UPC + swz(c, u): the eight threads of a quarter-warp read eight consecutive chunks, and
// the XOR by c spreads their reads over the eight 16-byte bank groups.
//
// Launched with programmatic stream serialization: before waiting for the kernel ahead of
// it, a CTA only initialises its barrier and asks L2 to prefetch its code rows (every device
// write lands in L2 first, so a prefetch reads nothing stale); the code loads, the
// activation copy and the stores come after the wait, so in a stream of GEMVs the codes of
// the next call stream into L2 while this one computes.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace tgc {

template <int BITS, int NB>
struct GemvBulkShape {
	static constexpr int CPC = BITS == 8 ? 16 : 32; // codes per 16-byte chunk
	static constexpr int PER = BITS == 8 ? 4 : 8;   // codes per 32-bit word
	static constexpr int UPC = CPC * NB / 4;        // float4 units of activations per chunk
	static constexpr int NP = (NB + 1) / 2;         // column pairs (NB > 1)
	// parts of a word whose activations are read at once (halves for wide batches, to save registers)
	static constexpr int NH = NB > 2 && (PER * NB / 2) % 4 == 0 ? 2 : 1;
	static __host__ __device__ constexpr int swz(int c, int u)
	{
		return (u | 7) < UPC ? ((u & ~7) | ((u ^ c) & 7)) : UPC < 8 ? (u ^ (c & (UPC - 1))) : u;
	}
	// the staging scale of word position e: 2^-(bit offset of the code in its half-word)
	static __device__ __forceinline__ float place(int e)
	{
		return __int_as_float((127 - (BITS == 8 ? 8 * (e & 1) : 4 * (e & 3))) << 23);
	}
};

// Shared memory of one CTA: the staged activations and the activations as copied.
__host__ __device__ constexpr size_t gemv_bulk_smem(int nb, int k) { return 2 * (size_t)k * nb * 4; }

// (a & m) ^ c as one LOP3: with both m and c as immediates the compiler splits it in two.
__device__ __forceinline__ uint32_t and_xor(uint32_t a, uint32_t m, uint32_t c)
{
	uint32_t d;
	asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(m), "r"(c));
	return d;
}

// The masks and offsets of the decode, held in registers for the whole kernel.
template <int BITS>
struct CodeConsts {
	uint32_t m[4], c[4];
	float2 off[2];
	__device__ __forceinline__ CodeConsts()
	{
		if (BITS == 8) {
			m[0] = 0xFFu, m[1] = 0xFF00u, c[0] = 0x4B000080u, c[1] = 0x4B008000u;
			m[2] = m[0], m[3] = m[1], c[2] = c[0], c[3] = c[1];
			off[0] = off[1] = make_float2(-8388736.0f, -8421376.0f); // 2^23 + 128, 2^23 + 128*256
		} else {
			m[0] = 0xFu, m[1] = 0xF0u, m[2] = 0xF00u, m[3] = 0xF000u;
			c[0] = 0x4B000008u, c[1] = 0x4B000080u, c[2] = 0x4B000800u, c[3] = 0x4B008000u;
			off[0] = make_float2(-8388616.0f, -8388736.0f);  // 2^23 + 8, 2^23 + 8*16
			off[1] = make_float2(-8390656.0f, -8421376.0f);  // 2^23 + 8*256, 2^23 + 8*4096
		}
		// opaque to the compiler, so the constants stay in registers
#pragma unroll
		for (int i = 0; i < 4; i++) asm volatile("" : "+r"(m[i]), "+r"(c[i]));
	}
	// Codes 2i and 2i+1 of word x, each times its place value, as a float pair (exact).
	__device__ __forceinline__ float2 pair(uint32_t x, int i) const
	{
		const int j = BITS == 8 ? 0 : 2 * (i & 1); // masks of the pair within its half-word
		const uint32_t h = i < (BITS == 8 ? 1 : 2) ? x : x >> 16;
		const float lo = __int_as_float(and_xor(h, m[j], c[j])), hi = __int_as_float(and_xor(h, m[j + 1], c[j + 1]));
		return __fadd2_rn(make_float2(lo, hi), off[BITS == 8 ? 0 : i & 1]);
	}
};

// Rows per warp and code chunks per lane and row in one register block: fewer of both for
// wider batches, whose activations take the registers.
template <int NB> struct GemvBulkTile {
	static constexpr int RR = NB <= 4 ? 2 : 1, BLK = NB <= 2 ? 4 : 2;
};
constexpr int GB_MAX_WARPS = 16;

// One register block of a warp's rows: chunks c0 + 32 t + lane, t < BLK, of each row.
template <int BITS, int NB, int RR, int BLK, bool EXACT>
__device__ __forceinline__ void gemv_bulk_block(float2 (&acc)[RR][GemvBulkShape<BITS, NB>::NP], const uint4 (&qb)[RR][BLK],
						const float4 *sb, int c0, int nch, int lane, const CodeConsts<BITS> &cc)
{
	using S = GemvBulkShape<BITS, NB>;
#pragma unroll
		for (int t = 0; t < BLK; t++) {
			const int c = c0 + 32 * t + lane;
			if (!EXACT && c >= nch) continue;
			const float4 *bc = sb + c * S::UPC;
#pragma unroll
			for (int word = 0; word < 4; word++) {
#pragma unroll
			for (int half = 0; half < S::NH; half++) { // the word's codes [half * PER / NH, (half + 1) * PER / NH)
				float bv[S::PER * NB / S::NH];
#pragma unroll
				for (int i = 0; i < S::PER * NB / (4 * S::NH); i++) {
					const float4 tv = bc[S::swz(c, (S::NH * word + half) * S::PER * NB / (4 * S::NH) + i)];
					bv[4 * i] = tv.x, bv[4 * i + 1] = tv.y, bv[4 * i + 2] = tv.z, bv[4 * i + 3] = tv.w;
				}
#pragma unroll
				for (int r = 0; r < RR; r++) {
					const uint4 qc = qb[r][t];
					const uint32_t x = word == 0 ? qc.x : word == 1 ? qc.y : word == 2 ? qc.z : qc.w;
#pragma unroll
					for (int ii = 0; ii < S::PER / (2 * S::NH); ii++) {
						const int i = half * S::PER / (2 * S::NH) + ii; // pair of the word; bv holds its part
						const float2 cp = cc.pair(x, i);
						if (NB == 1) {
							acc[r][0] = __ffma2_rn(cp, make_float2(bv[2 * ii], bv[2 * ii + 1]), acc[r][0]);
						} else {
#pragma unroll
							for (int h = 0; h < S::NP; h++) {
								const int j0 = 2 * h, j1 = 2 * h + 1 < NB ? 2 * h + 1 : 2 * h;
								acc[r][h] = __ffma2_rn(make_float2(cp.x, cp.x),
										       make_float2(bv[2 * ii * NB + j0], bv[2 * ii * NB + j1]), acc[r][h]);
								acc[r][h] = __ffma2_rn(make_float2(cp.y, cp.y),
										       make_float2(bv[(2 * ii + 1) * NB + j0], bv[(2 * ii + 1) * NB + j1]),
										       acc[r][h]);
							}
						}
					}
				}
			}
			}
		}
}

// NCHL > 0: the rows hold exactly 32 * NCHL chunks (one register block, no predicates);
// NCHL == 0: any multiple of a chunk, in blocks.
template <int BITS, int NB, int NCHL>
__global__ void __launch_bounds__(32 * GB_MAX_WARPS) gemv_bulk(float *__restrict__ o, const signed char *__restrict__ q,
							       const float *__restrict__ s, const float *__restrict__ b, int m,
							       int k, int rows, int *status)
{
	using S = GemvBulkShape<BITS, NB>;
	constexpr int RR = GemvBulkTile<NB>::RR, BLK = NCHL > 0 ? NCHL : GemvBulkTile<NB>::BLK;
	constexpr bool EXACT = NCHL > 0;
	extern __shared__ __align__(128) unsigned char smem[];
	__shared__ __align__(8) uint64_t bar;
	const long row_bytes = (long)k * BITS / 8;
	const int nch = k / S::CPC;
	const uint32_t bbytes = (uint32_t)k * NB * 4;
	const int r0 = blockIdx.x * rows, nr = min(rows, m - r0);
	float4 *sb = (float4 *)smem;                            // staged activations
	const float4 *raw = (const float4 *)(smem + bbytes);   // the activations as copied
	const signed char *src = q + (long)r0 * row_bytes;
	if (threadIdx.x == 0) {
		mbar_init(&bar, 1);
		fence_barrier_init();
		prefetch_l2(src, (uint32_t)(nr * row_bytes));
	}
	__syncthreads();
	pdl_wait();
	pdl_launch();
	if (threadIdx.x == 0) {
		mbar_expect_tx(&bar, bbytes);
		bulk_load((void *)raw, b, bbytes, &bar);
	}
	const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int rw = max(0, min(RR, nr - RR * w)); // rows of this warp
	const uint4 *gq = (const uint4 *)(src + (long)RR * w * row_bytes);
	uint4 qa[RR][BLK]; // the block being computed
	auto load_block = [&](uint4 (&dst)[RR][BLK], int c0) {
#pragma unroll
		for (int r = 0; r < RR; r++)
#pragma unroll
			for (int t = 0; t < BLK; t++) {
				const int c = c0 + 32 * t + lane;
				dst[r][t] = r < rw && (EXACT || c < nch) ? __ldg(gq + (long)r * nch + c) : make_uint4(0u, 0u, 0u, 0u);
			}
	};
	load_block(qa, 0);
	// activations, each divided by the place value of its code (exact powers of two)
	const bool bok = __all_sync(0xffffffffu, mbar_wait(&bar, 0, status, ST_TIMEOUT_FULL));
	if (bok)
		for (int g = threadIdx.x; g < nch * S::UPC; g += blockDim.x) {
			const int c = g / S::UPC, u = g - c * S::UPC;
			float4 v = raw[g];
			const int f = 4 * u; // first float of the unit within the chunk: position f / NB
			v.x *= S::place((f + 0) / NB), v.y *= S::place((f + 1) / NB), v.z *= S::place((f + 2) / NB),
				v.w *= S::place((f + 3) / NB);
			sb[c * S::UPC + S::swz(c, u)] = v;
		}
	__syncthreads();
	if (!bok || rw == 0) return;
	const CodeConsts<BITS> cc;
	float2 acc[RR][S::NP];
#pragma unroll
	for (int r = 0; r < RR; r++)
#pragma unroll
		for (int h = 0; h < S::NP; h++) acc[r][h] = make_float2(0.0f, 0.0f);
	if (EXACT || nch <= 32 * BLK) { // one block: no loop
		gemv_bulk_block<BITS, NB, RR, BLK, EXACT>(acc, qa, sb, 0, nch, lane, cc);
	} else {
		for (int c0 = 0; c0 < nch; c0 += 32 * BLK) {
			uint4 qn[RR][BLK]; // the next block, in flight while this one is computed
			if (c0 + 32 * BLK < nch) load_block(qn, c0 + 32 * BLK);
			gemv_bulk_block<BITS, NB, RR, BLK, false>(acc, qa, sb, c0, nch, lane, cc);
			if (c0 + 32 * BLK < nch)
#pragma unroll
				for (int r = 0; r < RR; r++)
#pragma unroll
					for (int t = 0; t < BLK; t++) qa[r][t] = qn[r][t];
		}
	}
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
			const float sc = s[row];
#pragma unroll
			for (int jj = 0; jj < NB; jj++) o[row * NB + jj] = sc * v[jj];
		}
	}
}

} // namespace tgc
