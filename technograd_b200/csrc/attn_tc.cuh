// attn_tc.cuh -- causal attention of the prefill on the tcgen05 tensor cores.
//
// The program's per-head attention (examples/qwen3/import.py:110-112):
//   s = softmax((q @ transpose(k)) * scale + mask);  o = s @ v
// with q, k, v f32 [T, 128] per head and the causal mask (-1e9 above the diagonal,
// which the softmax turns into exact zeros). The f32 products are carried on the
// bf16 tensor cores by the hi/lo split x = hi + lo (hi = bf16(x), lo = bf16(x - hi)):
// x.y ~ hi.hi + hi.lo + lo.hi, three MMAs per product with f32 accumulation, which
// keeps about 16 bits of each operand (relative error near 2^-17 per product).
//
// CTA = 128 queries of one head of one sequence; keys in tiles of 64. Warps:
//   0-3  softmax: one query row per thread (TMEM lane = row). Reads the score tile
//        from TMEM, applies scale and mask, keeps the running max and sum, writes the
//        probabilities (split hi/lo) to shared memory as the A operand of P.V, and at
//        the end reads O from TMEM, divides by the sum and stores it split hi/lo (the
//        o_proj GEMM's input).
//   4-7  converters: Q once (from global); then per key tile, from a staging area that
//        bulk copies fill with the tile's rows of the cache (bf16 part and remainder
//        bytes of K and V, kv.cuh), K (rows = keys, K-major over dims) and V^T (rows =
//        dims, K-major over keys) as bf16 hi/lo in the 128-byte-swizzled K-major layout
//        of the UMMA descriptors. The K and V halves of the staging area refill
//        separately: thread 0 issues tile j+1's K copies once K_j is converted, so they
//        land while V_j is converted, and V_{j+1}'s once V_j is.
//   8    TMEM allocation and the MMA issue (one thread): S_j = Q.K_j^T into one of two
//        TMEM score buffers, O += P_j.V_j into the TMEM accumulator, each issued as soon
//        as its operands are ready, so the softmax of tile j+1 overlaps the P.V of tile j
//        and P_j.V_j does not wait for K_{j+1}.
// O stays in TMEM across tiles. The probabilities use a running reference max that is
// raised (and O, l rescaled in place) only when a tile's max exceeds it by more than
// FA_RESCALE, so O is rarely touched between tiles; exp(s - m_ref) <= e^8 keeps the
// sums well inside f32. The quotient O / l is the same as the reference's
// exp(s - max) / sum, up to rounding (the exponentials use the hardware exp2, relative
// error about 2^-21 here).
//
// Every wait is bounded (tc.cuh); a timeout sets the status word and all roles
// leave their loops, waiting for their own MMAs before TMEM is released.
#pragma once

#include <cuda_bf16.h>

#include "kv.cuh"
#include "tc.cuh"

namespace tgc {

constexpr int FA_Q = 128, FA_K = 64, FA_HD = 128;
constexpr float FA_RESCALE = 8.0f;
constexpr int FA_THREADS = 288;
constexpr int FA_LB = 8; // Q items whose global loads a converter issues before converting them

// shared-memory layout (byte offsets from a 1024-aligned base); each operand tile is
// K-major with 128-byte swizzle: rows of 128 bytes, 8-row atoms of 1024 bytes
constexpr int FA_SQ_HI = 0;          // Q hi: [2 k-blocks][128 rows][128 B]
constexpr int FA_SQ_LO = 32768;      // Q lo
constexpr int FA_SK_HI = 65536;      // K hi: [2 k-blocks][64 rows][128 B]
constexpr int FA_SK_LO = 81920;      // K lo
constexpr int FA_SV_HI = 98304;      // V^T hi: [128 rows][128 B]
constexpr int FA_SV_LO = 114688;     // V^T lo
constexpr int FA_SP = 131072;        // P: hi [128 rows][128 B], lo 16384 after it
constexpr int FA_ST_KH = 163840;     // staging, the tile's rows as in the cache: K bf16 [64][128]
constexpr int FA_ST_KQ = 180224;     //   K remainder bytes [64][128]
constexpr int FA_ST_VH = 188416;     //   V bf16
constexpr int FA_ST_VQ = 204800;     //   V remainder bytes
constexpr int FA_SBAR = 212992;      // barriers and the TMEM address
constexpr size_t FA_SMEM = FA_SBAR + 256 + 1024; // + alignment slack

struct FaBars {
	uint64_t q_full, stgk_full, stgk_free, stgv_full, stgv_free, k_full, k_empty, v_full, v_empty;
	uint64_t s_full[2], s_free[2], p_full, p_empty, done;
	uint32_t tmem;
	int abort;
};

__device__ __forceinline__ uint32_t fa_sw(int row, int chunk) { return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4)); }

__device__ __forceinline__ uint32_t fa_pack(float a, float b)
{
	__nv_bfloat162 v = __floats2bfloat162_rn(a, b); // .x = a (low half), .y = b
	return *(uint32_t *)&v;
}

// 8 floats -> one 16-byte chunk of bf16 hi and one of lo. Pairs are rounded by the packed
// conversion (two elements per instruction); the hi values come back as floats by shifts.
__device__ __forceinline__ void fa_split8(const float (&x)[8], uint4 &hi, uint4 &lo)
{
	uint32_t hw[4], lw[4];
#pragma unroll
	for (int i = 0; i < 4; i++) {
		hw[i] = fa_pack(x[2 * i], x[2 * i + 1]);
		const float h0 = __uint_as_float(hw[i] << 16), h1 = __uint_as_float(hw[i] & 0xFFFF0000u);
		lw[i] = fa_pack(x[2 * i] - h0, x[2 * i + 1] - h1);
	}
	hi = make_uint4(hw[0], hw[1], hw[2], hw[3]);
	lo = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

// bf16 bits of the remainders of two cache elements: hw holds their bf16 bits (element 0 in
// the low half), q0 / q1 their remainder bytes (kv.cuh); the remainders are exact in bf16
__device__ __forceinline__ uint32_t kv_lo_pair(uint32_t hw, int q0, int q1)
{
	const uint32_t h0 = hw << 16, h1 = hw & 0xFFFF0000u;
	return fa_pack(__uint_as_float(h0 + (uint32_t)(q0 * 256)) - __uint_as_float(h0),
		       __uint_as_float(h1 + (uint32_t)(q1 * 256)) - __uint_as_float(h1));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16])
{
	asm volatile(
		"tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
		::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
		  "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])),
		  "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
		  "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
		  "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
		: "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// A bounded wait that first checks the CTA's abort flag; false = leave the loop.
// The softmax warps combine the lanes' results (fa_wait_warp) so a warp leaves together.
__device__ __forceinline__ bool fa_wait(FaBars *B, uint64_t *bar, uint32_t parity, int *status)
{
	if (*(volatile int *)&B->abort) return false;
	if (mbar_wait(bar, parity, status, ST_TIMEOUT_FULL)) return true;
	*(volatile int *)&B->abort = 1;
	return false;
}

__device__ __forceinline__ bool fa_wait_warp(FaBars *B, uint64_t *bar, uint32_t parity, int *status)
{
	return __all_sync(0xffffffffu, fa_wait(B, bar, parity, status));
}

// q: [seq][NQ][T][128] f32; kc/vc: the cache [slot][NKV][max_len][128] in the 24-bit
// format of kv.cuh, whose bf16 part is the hi operand and whose remainder is the lo one;
// out hi/lo: [seq * T + t][NQ * 128 + h * 128 + d] bf16.
__global__ void __launch_bounds__(FA_THREADS, 1)
	k_attn_prefill_tc(const float *__restrict__ q, KvPlaneC kc, KvPlaneC vc, int T, int NQ,
			  int NKV, int slot0, int max_len, float scale, __nv_bfloat16 *__restrict__ ohi,
			  __nv_bfloat16 *__restrict__ olo, int *status)
{
	extern __shared__ uint8_t fa_raw[];
	uint8_t *sm = fa_raw + ((1024 - (smem_u32(fa_raw) & 1023)) & 1023);
	FaBars *B = (FaBars *)(sm + FA_SBAR);
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int nqt = (T + FA_Q - 1) / FA_Q;
	const int qt = nqt - 1 - (int)blockIdx.x; // the longest rows of the causal triangle start first
	const int h = blockIdx.y, s = blockIdx.z;
	const int kvh = h / (NQ / NKV);
	const int q0 = qt * FA_Q;
	const int nkt = (min(q0 + FA_Q, T) + FA_K - 1) / FA_K;
	const long cb = ((long)(slot0 + s) * NKV + kvh) * (long)max_len * FA_HD; // this (sequence, kv head)'s cache rows

	if (threadIdx.x == 0) {
		// barriers the 128-thread groups arrive on count warps (mbar_arrive_warp)
		mbar_init(&B->q_full, 4);
		mbar_init(&B->stgk_full, 1);
		mbar_init(&B->stgk_free, 4);
		mbar_init(&B->stgv_full, 1);
		mbar_init(&B->stgv_free, 4);
		mbar_init(&B->k_full, 4);
		mbar_init(&B->k_empty, 1);
		mbar_init(&B->v_full, 4);
		mbar_init(&B->v_empty, 1);
		for (int b = 0; b < 2; b++) {
			mbar_init(&B->s_full[b], 1);
			mbar_init(&B->s_free[b], 4);
		}
		mbar_init(&B->p_full, 4);
		mbar_init(&B->p_empty, 1);
		mbar_init(&B->done, 1);
		B->abort = 0;
		fence_barrier_init();
	}
	if (warp == 8) tmem_alloc(&B->tmem, 256); // S buffers at columns 0 and 64, O at 128
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = B->tmem;

	if (warp >= 4 && warp < 8) {
		// ---------------- converters ----------------
		const int t = threadIdx.x - 128;
		// the bulk copies of key tile j's K rows (and, separately, its V rows) into their halves
		// of the staging area (rows past T are not copied)
		auto stage_k = [&](int j) {
			const int k0 = j * FA_K, rows = min(FA_K, T - k0);
			mbar_expect_tx(&B->stgk_full, (uint32_t)rows * (256 + 128));
			bulk_load(sm + FA_ST_KH, kc.h + cb + (long)k0 * FA_HD, rows * 256, &B->stgk_full);
			bulk_load(sm + FA_ST_KQ, kc.q + cb + (long)k0 * FA_HD, rows * 128, &B->stgk_full);
		};
		auto stage_v = [&](int j) {
			const int k0 = j * FA_K, rows = min(FA_K, T - k0);
			mbar_expect_tx(&B->stgv_full, (uint32_t)rows * (256 + 128));
			bulk_load(sm + FA_ST_VH, vc.h + cb + (long)k0 * FA_HD, rows * 256, &B->stgv_full);
			bulk_load(sm + FA_ST_VQ, vc.q + cb + (long)k0 * FA_HD, rows * 128, &B->stgv_full);
		};
		int pendk = -1, pendv = -1; // thread 0: staged tiles whose copies nobody has waited for yet
		if (t == 0) stage_k(0), stage_v(0), pendk = 0, pendv = 0;
		const float *qb = q + ((long)s * NQ + h) * (long)T * FA_HD;
		for (int i0 = t; i0 < FA_Q * 16; i0 += 128 * FA_LB) { // Q: 128 rows x 16 chunks of 8 dims
			float4 a[FA_LB], b[FA_LB];
#pragma unroll
			for (int u = 0; u < FA_LB; u++) {
				const int i = i0 + u * 128, r = i >> 4, c = i & 15;
				const bool in = i < FA_Q * 16 && q0 + r < T;
				a[u] = in ? *(const float4 *)(qb + (long)(q0 + r) * FA_HD + c * 8) : make_float4(0.f, 0.f, 0.f, 0.f);
				b[u] = in ? *(const float4 *)(qb + (long)(q0 + r) * FA_HD + c * 8 + 4) : make_float4(0.f, 0.f, 0.f, 0.f);
			}
#pragma unroll
			for (int u = 0; u < FA_LB; u++) {
				const int i = i0 + u * 128, r = i >> 4, c = i & 15;
				if (i >= FA_Q * 16) break;
				const float x[8] = { a[u].x, a[u].y, a[u].z, a[u].w, b[u].x, b[u].y, b[u].z, b[u].w };
				uint4 hi, lo;
				fa_split8(x, hi, lo);
				uint32_t off = (uint32_t)((c >> 3) * 16384) + fa_sw(r, c & 7);
				*(uint4 *)(sm + FA_SQ_HI + off) = hi;
				*(uint4 *)(sm + FA_SQ_LO + off) = lo;
			}
		}
		fence_async_smem();
		mbar_arrive_warp(&B->q_full);
		for (int j = 0; j < nkt; j++) {
			const int k0 = j * FA_K;
			if (!fa_wait_warp(B, &B->stgk_full, j & 1, status)) break;
			pendk = -1;
			// K: 64 rows x 16 chunks of 8 dims; the bf16 part as is, the remainder as lo
			if (j > 0 && !fa_wait_warp(B, &B->k_empty, (j - 1) & 1, status)) break;
#pragma unroll 2
			for (int i = t; i < FA_K * 16; i += 128) {
				const int r = i >> 4, c = i & 15;
				uint4 hv = make_uint4(0u, 0u, 0u, 0u);
				uint2 qv = make_uint2(0u, 0u);
				if (k0 + r < T) {
					hv = *(const uint4 *)(sm + FA_ST_KH + r * 256 + c * 16);
					qv = *(const uint2 *)(sm + FA_ST_KQ + r * 128 + c * 8);
				}
				const uint32_t hw[4] = { hv.x, hv.y, hv.z, hv.w }, qw[2] = { qv.x, qv.y };
				uint32_t lw[4];
#pragma unroll
				for (int w = 0; w < 4; w++) {
					const uint32_t qq = qw[w >> 1] >> (16 * (w & 1)); // the two bytes of this word's elements
					lw[w] = kv_lo_bits(hw[w] & 0xFFFF, (int)(int8_t)(qq & 0xFF)) |
						(kv_lo_bits(hw[w] >> 16, (int)(int8_t)((qq >> 8) & 0xFF)) << 16);
				}
				const uint32_t off = (uint32_t)((c >> 3) * 8192) + fa_sw(r, c & 7);
				*(uint4 *)(sm + FA_SK_HI + off) = hv;
				*(uint4 *)(sm + FA_SK_LO + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
			}
			fence_async_smem();
			mbar_arrive_warp(&B->k_full);
			// the K half of the staging area has been read: thread 0 refills it with the next
			// tile's K rows, which then land while V is converted
			mbar_arrive_warp(&B->stgk_free);
			if (j + 1 < nkt) {
				bool ok0 = true;
				if (t == 0) {
					ok0 = fa_wait(B, &B->stgk_free, j & 1, status);
					if (ok0) {
						fence_async_smem();
						stage_k(j + 1);
						pendk = j + 1;
					}
				}
				if (!__shfl_sync(0xffffffffu, ok0, 0)) break; // thread 0's warp leaves together
			}
			// V^T: item = (8 keys, 4 dims) -> one 16-byte chunk in each of 4 rows
			if (!fa_wait_warp(B, &B->stgv_full, j & 1, status)) break;
			pendv = -1;
			if (j > 0 && !fa_wait_warp(B, &B->v_empty, (j - 1) & 1, status)) break;
			for (int i = t; i < 256; i += 128) {
				const int kg = i & 7, dg = i >> 3;
				uint2 hv[8];
				uint32_t qv[8];
#pragma unroll
				for (int e = 0; e < 8; e++) {
					const int key = kg * 8 + e;
					const bool in = k0 + key < T;
					hv[e] = in ? *(const uint2 *)(sm + FA_ST_VH + key * 256 + dg * 8) : make_uint2(0u, 0u);
					qv[e] = in ? *(const uint32_t *)(sm + FA_ST_VQ + key * 128 + dg * 4) : 0u;
				}
#pragma unroll
				for (int dd = 0; dd < 4; dd++) {
					uint32_t hb[8], lb[8]; // dim dg*4+dd of the 8 keys
#pragma unroll
					for (int e = 0; e < 8; e++) {
						const uint32_t hw = dd < 2 ? hv[e].x : hv[e].y;
						hb[e] = (dd & 1) ? hw >> 16 : hw & 0xFFFF;
						lb[e] = kv_lo_bits(hb[e], (int)(int8_t)((qv[e] >> (8 * dd)) & 0xFF));
					}
					const uint4 hi = make_uint4(hb[0] | (hb[1] << 16), hb[2] | (hb[3] << 16), hb[4] | (hb[5] << 16), hb[6] | (hb[7] << 16));
					const uint4 lo = make_uint4(lb[0] | (lb[1] << 16), lb[2] | (lb[3] << 16), lb[4] | (lb[5] << 16), lb[6] | (lb[7] << 16));
					const uint32_t off = fa_sw(dg * 4 + dd, kg);
					*(uint4 *)(sm + FA_SV_HI + off) = hi;
					*(uint4 *)(sm + FA_SV_LO + off) = lo;
				}
			}
			fence_async_smem();
			mbar_arrive_warp(&B->v_full);
			mbar_arrive_warp(&B->stgv_free);
			if (j + 1 < nkt) {
				bool ok0 = true;
				if (t == 0) {
					ok0 = fa_wait(B, &B->stgv_free, j & 1, status);
					if (ok0) {
						fence_async_smem();
						stage_v(j + 1);
						pendv = j + 1;
					}
				}
				if (!__shfl_sync(0xffffffffu, ok0, 0)) break; // thread 0's warp leaves together
			}
		}
		// after an abort: the copies still in flight land before the CTA's shared memory is released
		if (pendk >= 0) mbar_wait(&B->stgk_full, pendk & 1, nullptr, 0);
		if (pendv >= 0) mbar_wait(&B->stgv_full, pendv & 1, nullptr, 0);
	} else if (warp == 8) {
		// ---------------- MMA issue ----------------
		if (lane == 0) {
			const uint32_t idS = idesc_bf16_f32(FA_Q, FA_K), idO = idesc_bf16_f32(FA_Q, FA_HD);
			const uint32_t base = smem_u32(sm);
			bool ok = fa_wait(B, &B->q_full, 0, status);
			auto issue_s = [&](int j) {
				tc_fence_after();
				const uint32_t d = tmem + (uint32_t)((j & 1) * FA_K);
				const uint32_t qa[2] = { base + FA_SQ_HI, base + FA_SQ_LO }, ka[2] = { base + FA_SK_HI, base + FA_SK_LO };
				const int pa[3] = { 0, 0, 1 }, pb[3] = { 0, 1, 0 };
				uint32_t acc = 0;
				for (int kb = 0; kb < 2; kb++)
					for (int kk = 0; kk < 4; kk++)
						for (int pr = 0; pr < 3; pr++) {
							uint32_t a = qa[pa[pr]] + kb * 16384 + kk * 32, b = ka[pb[pr]] + kb * 8192 + kk * 32;
							tc_mma_f16(d, sw128_kmajor_desc(a), sw128_kmajor_desc(b), idS, acc);
							acc = 1;
						}
				tc_commit(&B->s_full[j & 1]);
				tc_commit(&B->k_empty);
			};
			auto issue_pv = [&](int j) {
				tc_fence_after();
				const uint32_t pa2[2] = { base + FA_SP, base + FA_SP + 16384 }, va[2] = { base + FA_SV_HI, base + FA_SV_LO };
				const int pa[3] = { 0, 0, 1 }, pb[3] = { 0, 1, 0 };
				for (int kk = 0; kk < 4; kk++)
					for (int pr = 0; pr < 3; pr++) {
						uint32_t a = pa2[pa[pr]] + kk * 32, b = va[pb[pr]] + kk * 32;
						tc_mma_f16(tmem + 128, sw128_kmajor_desc(a), sw128_kmajor_desc(b), idO,
							   (j > 0 || kk > 0 || pr > 0) ? 1u : 0u);
					}
				tc_commit(&B->p_empty);
				tc_commit(&B->v_empty);
			};
			// S_j and P_j.V_j in the order their operands become ready: S_j once K_j is
			// converted and its score buffer is free (the softmax has read S_{j-2}), P_j.V_j once
			// P_j and V_j are in shared memory. Neither chain waits behind the other; each
			// barrier polled can be at most one phase ahead of the one asked for, because its
			// next phase depends on the MMA not yet issued.
			int ns = 0, npv = 0;
			long long idle0 = clock64();
			for (uint32_t spins = 0; ok && npv < nkt;) {
				bool did = false;
				if (ns < nkt && mbar_try(&B->k_full, ns & 1) && (ns < 2 || mbar_try(&B->s_free[ns & 1], ((ns >> 1) - 1) & 1))) {
					issue_s(ns++);
					did = true;
				}
				if (npv < ns && mbar_try(&B->v_full, npv & 1) && mbar_try(&B->p_full, npv & 1)) {
					issue_pv(npv++);
					did = true;
				}
				if (did) {
					idle0 = clock64();
					spins = 0;
				} else if ((++spins & 63) == 0) {
					if (*(volatile int *)&B->abort) {
						ok = false;
					} else if (clock64() - idle0 > WAIT_CYCLES) {
						if (status) *(volatile int *)status = ST_TIMEOUT_FULL;
						*(volatile int *)&B->abort = 1;
						ok = false;
					}
				}
			}
			// every MMA issued has completed before TMEM is released (also after an abort)
			tc_commit(&B->done);
			mbar_wait(&B->done, 0, status, ST_TIMEOUT_ACC);
		}
		__syncwarp();
	} else {
		// ---------------- softmax / epilogue (warps 0-3) ----------------
		const int row = threadIdx.x; // TMEM lane, query q0 + row
		const int qi = q0 + row;
		const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
		float m_ref = -INFINITY, l = 0.0f;
		bool ok = true;
		for (int j = 0; j < nkt && ok; j++) {
			const int k0 = j * FA_K;
			if (!(ok = fa_wait_warp(B, &B->s_full[j & 1], (j >> 1) & 1, status))) break;
			tc_fence_after();
			float sc[FA_K];
#pragma unroll
			for (int c = 0; c < FA_K / 16; c++) {
				float v[16];
				tmem_ld16(lane_base + (uint32_t)((j & 1) * FA_K + c * 16), v);
#pragma unroll
				for (int e = 0; e < 16; e++) sc[c * 16 + e] = v[e];
			}
			tc_fence_before();
			mbar_arrive_warp(&B->s_free[j & 1]);
			float mt = -INFINITY;
#pragma unroll
			for (int c = 0; c < FA_K; c++) {
				const int kj = k0 + c;
				float v = kj <= qi && kj < T ? __fmul_rn(sc[c], scale) : -INFINITY;
				sc[c] = v;
				mt = fmaxf(mt, v);
			}
			const bool raise = mt > m_ref + FA_RESCALE;
			const float m_new = raise ? mt : m_ref;
			// P's buffer (and O, for a rescale) is free once P_{j-1}.V has completed
			if (j > 0 && !(ok = fa_wait_warp(B, &B->p_empty, (j - 1) & 1, status))) break;
			if (__any_sync(0xffffffffu, raise && m_ref != -INFINITY)) {
				// O holds P.V of tiles < j at the old reference max: rescale it in place
				tc_fence_after();
				const float f = raise && m_ref != -INFINITY ? __expf(m_ref - m_new) : 1.0f;
#pragma unroll 1
				for (int c = 0; c < FA_HD / 16; c++) {
					float v[16];
					tmem_ld16(lane_base + 128 + c * 16, v);
#pragma unroll
					for (int e = 0; e < 16; e++) v[e] *= f;
					tmem_st16(lane_base + 128 + c * 16, v);
				}
				tmem_wait_st();
				l *= f;
			}
			m_ref = m_new;
			float sum = 0.0f;
#pragma unroll
			for (int c = 0; c < FA_K; c++) {
				float p = sc[c] == -INFINITY ? 0.0f : __expf(sc[c] - m_ref);
				sc[c] = p;
				sum += p;
			}
			l += sum;
			uint8_t *pb = sm + FA_SP;
#pragma unroll
			for (int c = 0; c < 8; c++) {
				float x[8];
#pragma unroll
				for (int e = 0; e < 8; e++) x[e] = sc[c * 8 + e];
				uint4 hi, lo;
				fa_split8(x, hi, lo);
				*(uint4 *)(pb + fa_sw(row, c)) = hi;
				*(uint4 *)(pb + 16384 + fa_sw(row, c)) = lo;
			}
			fence_async_smem();
			tc_fence_before();
			mbar_arrive_warp(&B->p_full);
		}
		if (ok) ok = fa_wait_warp(B, &B->p_empty, (nkt - 1) & 1, status);
		if (ok) {
			tc_fence_after();
			const float inv = 1.0f / l;
			const long ob = ((long)s * T + qi) * (long)NQ * FA_HD + (long)h * FA_HD;
#pragma unroll 1
			for (int c = 0; c < FA_HD / 16; c++) {
				float v[16];
				tmem_ld16(lane_base + 128 + c * 16, v);
				if (qi < T) {
#pragma unroll
					for (int half = 0; half < 2; half++) {
						float x[8];
#pragma unroll
						for (int e = 0; e < 8; e++) x[e] = v[half * 8 + e] * inv;
						uint4 hi, lo;
						fa_split8(x, hi, lo);
						*(uint4 *)(ohi + ob + c * 16 + half * 8) = hi;
						*(uint4 *)(olo + ob + c * 16 + half * 8) = lo;
					}
				}
			}
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 8) {
		tc_fence_after();
		tmem_dealloc(tmem, 256);
	}
}

// ---- k_attn_prefill_tma: the cache's bf16 plane loaded by TMA straight into the operands ----
//
// The cache keeps each key and value as its bf16 rounding (the hi operand) and a remainder
// byte (kv.cuh). The bf16 plane's rows are exactly the K operand's rows: a 2D TMA load with
// 128-byte swizzle of a 64-key x 64-dim box lands them in the K-major layout the UMMA
// descriptor reads, and the same load of V is read as an MN-major B operand (keys along K,
// dims along N), so neither needs converting or transposing. Only the lo operands are
// computed, element for element at the same swizzled offsets, from the hi bits and the
// remainder bytes (bulk-copied beside them). The freed staging space double-buffers the hi
// tiles, so tile j+1's rows are in flight while tile j is computed. Warps:
//   0-7  softmax and epilogue: warps w and w + 4 share the 32 query rows of TMEM lanes
//        32 (w % 4) ...; the lower warp takes key columns 0-31 of each score tile and O
//        columns 0-63, the upper one key columns 32-63 and O columns 64-127. They combine
//        their row maxima (every tile) and sums (at the end) through shared memory.
//   8-11 converters: Q (with the softmax warps, before the first scores); per tile the K
//        lo and V lo tiles (and zeros over rows past T, whose cache contents are stale:
//        their probabilities are 0, but 0 * NaN is not);
//   12   TMEM allocation and MMA issue;
//   13-14 producers: warp 13 loads the K tiles, warp 14 the V tiles (one thread each, in
//        warps of their own so that neither spin-waits behind the other), each into the
//        buffer the MMA and the converters released (mbarriers counting one MMA commit and
//        the four converter warps).
constexpr int FB_THREADS = 480;
constexpr int FB_SQ_HI = 0;          // Q hi: [2 k-blocks][128 rows][128 B]
constexpr int FB_SQ_LO = 32768;      // Q lo
constexpr int FB_KH = 65536;         // K hi, two buffers of [2 dim blocks][64 keys][128 B]
constexpr int FB_KL = 98304;         // K lo
constexpr int FB_VH = 114688;        // V hi, two buffers of [2 dim blocks][64 keys][128 B]
constexpr int FB_VL = 147456;        // V lo
constexpr int FB_SP = 163840;        // P: hi [128 rows][128 B], lo 16384 after it
constexpr int FB_KQ = 196608;        // K remainder bytes, two buffers of [64 keys][128]
constexpr int FB_VQ = 212992;        // V remainder bytes, two buffers
constexpr int FB_SBAR = 229376;      // barriers and the TMEM address
constexpr int FB_RED = 229632;       // row maxima and sums of the two softmax halves: [2 tiles][2 halves][128]
constexpr size_t FB_SMEM = FB_RED + 2048; // the base must be 1024-aligned (checked)

struct FbBars {
	uint64_t q_full, kload[2], vload[2], kfree[2], vfree[2], k_full, kl_empty, v_full, vl_empty;
	uint64_t s_full[2], s_free[2], p_full, p_empty, done;
	uint32_t tmem;
	int abort;
};

// Shared-memory matrix descriptor, MN-major, 128-byte swizzle: 64 MN elements (128 bytes)
// per row, 8 rows along K per 1024-byte atom; lbo = bytes to the next 64 MN elements,
// sbo = bytes to the next 8 rows along K.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
	uint64_t d = 0;
	d |= (uint64_t)((saddr >> 4) & 0x3FFF);
	d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
	d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
	d |= (uint64_t)1 << 46;
	d |= (uint64_t)2 << 61;
	return d;
}

// A non-blocking probe of a phase (mbarrier.test_wait), for waiters whose barrier is
// completed by a tcgen05.commit: a suspended try_wait has been seen to resume microseconds
// after such a phase completed.
__device__ __forceinline__ bool fb_test(uint64_t *bar, uint32_t parity)
{
	uint32_t ok;
	asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
		     : "=r"(ok)
		     : "r"(smem_u32(bar)), "r"(parity)
		     : "memory");
	return ok != 0;
}

// Bounded polling wait with test_wait (see fb_test); false after the CTA's abort flag or the
// cycle budget, which then sets the status word and the abort flag.
__device__ __forceinline__ bool fb_poll(FbBars *B, uint64_t *bar, uint32_t parity, int *status)
{
	const long long t0 = clock64();
	for (uint32_t i = 0;; i++) {
		if (fb_test(bar, parity)) return true;
		if ((i & 63) == 63) {
			if (*(volatile int *)&B->abort) return false;
			if (clock64() - t0 > WAIT_CYCLES) {
				if (status) *(volatile int *)status = ST_TIMEOUT_FULL;
				*(volatile int *)&B->abort = 1;
				return false;
			}
		}
	}
}

__device__ __forceinline__ bool fb_wait(FbBars *B, uint64_t *bar, uint32_t parity, int *status)
{
	if (*(volatile int *)&B->abort) return false;
	if (mbar_wait(bar, parity, status, ST_TIMEOUT_FULL)) return true;
	*(volatile int *)&B->abort = 1;
	return false;
}

__device__ __forceinline__ bool fb_wait_warp(FbBars *B, uint64_t *bar, uint32_t parity, int *status)
{
	return __all_sync(0xffffffffu, fb_wait(B, bar, parity, status));
}

// lo tile of one 64-key tile: 16-byte chunks of 8 dims at the swizzled offsets of the hi
// tile; rows at or past `valid` get zeros (and, when zero_hi, so does the hi tile)
__device__ __forceinline__ void fb_lo_tile(uint8_t *hi, uint8_t *lo, const uint8_t *rem, int t, int valid, bool zero_hi)
{
#pragma unroll
	for (int u = 0; u < FA_K * 16 / 128; u++) {
		const int i = t + 128 * u, r = i >> 4, c = i & 15;
		const uint32_t off = (uint32_t)((c >> 3) * 8192) + fa_sw(r, c & 7);
		if (r >= valid) {
			*(uint4 *)(lo + off) = make_uint4(0u, 0u, 0u, 0u);
			if (zero_hi) *(uint4 *)(hi + off) = make_uint4(0u, 0u, 0u, 0u);
			continue;
		}
		const uint4 hv = *(const uint4 *)(hi + off);
		const uint2 qv = *(const uint2 *)(rem + r * 128 + c * 8);
		const uint32_t hw[4] = { hv.x, hv.y, hv.z, hv.w }, qw[2] = { qv.x, qv.y };
		uint32_t lw[4];
#pragma unroll
		for (int w = 0; w < 4; w++) {
			const uint32_t qq = qw[w >> 1] >> (16 * (w & 1)); // the two bytes of this word's elements
			lw[w] = kv_lo_pair(hw[w], (int)(int8_t)(qq & 0xFF), (int)(int8_t)((qq >> 8) & 0xFF));
		}
		*(uint4 *)(lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
	}
}

// q, out hi/lo as in k_attn_prefill_tc; kmap / vmap: TMA maps of this layer's bf16 planes
// as [rows = slot * NKV * max_len + position][128 dims] (boxes of 64 dims x 64 rows);
// kq / vq: the remainder planes.
__global__ void __launch_bounds__(FB_THREADS, 1)
	k_attn_prefill_tma(const float *__restrict__ q, const __grid_constant__ CUtensorMap kmap,
			   const __grid_constant__ CUtensorMap vmap, const signed char *__restrict__ kq,
			   const signed char *__restrict__ vq, int T, int NQ, int NKV, int slot0, int max_len, float scale,
			   __nv_bfloat16 *__restrict__ ohi, __nv_bfloat16 *__restrict__ olo, int *status)
{
	extern __shared__ __align__(1024) uint8_t fb_raw[];
	if (smem_u32(fb_raw) & 1023) { // the operand tiles need 1024-byte alignment
		if (threadIdx.x == 0 && status) *(volatile int *)status = ST_TIMEOUT_FULL;
		return;
	}
	uint8_t *sm = fb_raw;
	FbBars *B = (FbBars *)(sm + FB_SBAR);
	float *red = (float *)(sm + FB_RED);
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int nqt = (T + FA_Q - 1) / FA_Q;
	const int qt = nqt - 1 - (int)blockIdx.x; // the longest rows of the causal triangle start first
	const int h = blockIdx.y, s = blockIdx.z;
	const int kvh = h / (NQ / NKV);
	const int q0 = qt * FA_Q;
	const int nkt = (min(q0 + FA_Q, T) + FA_K - 1) / FA_K;
	const long row0 = ((long)(slot0 + s) * NKV + kvh) * (long)max_len; // this (sequence, kv head)'s first cache row

	if (threadIdx.x == 0) {
		mbar_init(&B->q_full, 12); // the softmax and converter warps
		for (int b = 0; b < 2; b++) {
			mbar_init(&B->kload[b], 1);
			mbar_init(&B->vload[b], 1);
			mbar_init(&B->kfree[b], 5); // the MMA's commit and the four converter warps
			mbar_init(&B->vfree[b], 5);
			mbar_init(&B->s_full[b], 1);
			mbar_init(&B->s_free[b], 8);
		}
		mbar_init(&B->k_full, 4);
		mbar_init(&B->kl_empty, 1);
		mbar_init(&B->v_full, 4);
		mbar_init(&B->vl_empty, 1);
		mbar_init(&B->p_full, 8);
		mbar_init(&B->p_empty, 1);
		mbar_init(&B->done, 1);
		B->abort = 0;
		fence_barrier_init();
	}
	if (warp == 12) tmem_alloc(&B->tmem, 256); // S buffers at columns 0 and 64, O at 128
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = B->tmem;

	if (warp < 12) {
		// Q: 128 rows x 16 chunks of 8 dims, split hi/lo, by the softmax and converter warps
		const float *qb = q + ((long)s * NQ + h) * (long)T * FA_HD;
		for (int i0 = threadIdx.x; i0 < FA_Q * 16; i0 += 384 * 4) {
			float4 a[4], bb[4];
#pragma unroll
			for (int u = 0; u < 4; u++) {
				const int i = i0 + u * 384, r = i >> 4, c = i & 15;
				const bool in = i < FA_Q * 16 && q0 + r < T;
				a[u] = in ? *(const float4 *)(qb + (long)(q0 + r) * FA_HD + c * 8) : make_float4(0.f, 0.f, 0.f, 0.f);
				bb[u] = in ? *(const float4 *)(qb + (long)(q0 + r) * FA_HD + c * 8 + 4) : make_float4(0.f, 0.f, 0.f, 0.f);
			}
#pragma unroll
			for (int u = 0; u < 4; u++) {
				const int i = i0 + u * 384, r = i >> 4, c = i & 15;
				if (i >= FA_Q * 16) break;
				const float x[8] = { a[u].x, a[u].y, a[u].z, a[u].w, bb[u].x, bb[u].y, bb[u].z, bb[u].w };
				uint4 hi, lo;
				fa_split8(x, hi, lo);
				uint32_t off = (uint32_t)((c >> 3) * 16384) + fa_sw(r, c & 7);
				*(uint4 *)(sm + FB_SQ_HI + off) = hi;
				*(uint4 *)(sm + FB_SQ_LO + off) = lo;
			}
		}
		fence_async_smem();
		mbar_arrive_warp(&B->q_full);
	}

	if (warp >= 13) {
		// ---------------- producers: warp 13 the K tiles, warp 14 the V tiles ----------------
		if (lane == 0) {
			const bool isk = warp == 13;
			const CUtensorMap *map = isk ? &kmap : &vmap;
			const signed char *rem = isk ? kq : vq;
			uint64_t *load = isk ? B->kload : B->vload, *freeb = isk ? B->kfree : B->vfree;
			uint8_t *hi0 = sm + (isk ? FB_KH : FB_VH), *q0b = sm + (isk ? FB_KQ : FB_VQ);
			int last[2] = { -1, -1 };
			tma_prefetch_desc(map);
			for (int j = 0; j < nkt; j++) {
				const int b = j & 1, k0 = j * FA_K, rows = min(FA_K, T - k0);
				if (j >= 2 && !fb_poll(B, &freeb[b], ((j >> 1) - 1) & 1, status)) break;
				uint8_t *hi = hi0 + b * 16384;
				mbar_expect_tx(&load[b], 16384u + (uint32_t)rows * 128u);
				tma_load_2d(hi, map, &load[b], 0, (int)(row0 + k0));
				tma_load_2d(hi + 8192, map, &load[b], 64, (int)(row0 + k0));
				bulk_load(q0b + b * 8192, rem + (row0 + k0) * FA_HD, (uint32_t)rows * 128u, &load[b]);
				last[b] = j;
			}
			// the loads still in flight land before the CTA's shared memory is released
			for (int b = 0; b < 2; b++)
				if (last[b] >= 0) mbar_wait(&load[b], (last[b] >> 1) & 1, nullptr, 0);
		}
		__syncwarp();
	} else if (warp >= 8 && warp < 12) {
		// ---------------- converters ----------------
		const int t = threadIdx.x - 256;
		for (int j = 0; j < nkt; j++) {
			const int b = j & 1, valid = min(FA_K, T - j * FA_K);
			if (!fb_wait_warp(B, &B->kload[b], (j >> 1) & 1, status)) break;
			if (j > 0 && !fb_wait_warp(B, &B->kl_empty, (j - 1) & 1, status)) break;
			fb_lo_tile(sm + FB_KH + b * 16384, sm + FB_KL, sm + FB_KQ + b * 8192, t, valid, true);
			fence_async_smem();
			mbar_arrive_warp(&B->k_full);
			mbar_arrive_warp(&B->kfree[b]);
			if (!fb_wait_warp(B, &B->vload[b], (j >> 1) & 1, status)) break;
			if (j > 0 && !fb_wait_warp(B, &B->vl_empty, (j - 1) & 1, status)) break;
			fb_lo_tile(sm + FB_VH + b * 16384, sm + FB_VL, sm + FB_VQ + b * 8192, t, valid, true);
			fence_async_smem();
			mbar_arrive_warp(&B->v_full);
			mbar_arrive_warp(&B->vfree[b]);
		}
	} else if (warp == 12) {
		// ---------------- MMA issue ----------------
		if (lane == 0) {
			const uint32_t idS = idesc_bf16_f32(FA_Q, FA_K);
			const uint32_t idO = idesc_bf16_f32(FA_Q, FA_HD) | (1u << 16); // B (V) MN-major
			const uint32_t base = smem_u32(sm);
			bool ok = fb_wait(B, &B->q_full, 0, status);
			auto issue_s = [&](int j) {
				tc_fence_after();
				const uint32_t d = tmem + (uint32_t)((j & 1) * FA_K);
				const uint32_t qa[2] = { base + FB_SQ_HI, base + FB_SQ_LO };
				const uint32_t ka[2] = { base + FB_KH + (uint32_t)(j & 1) * 16384, base + FB_KL };
				const int pa[3] = { 0, 0, 1 }, pb[3] = { 0, 1, 0 };
				uint32_t acc = 0;
				for (int kb = 0; kb < 2; kb++)
					for (int kk = 0; kk < 4; kk++)
						for (int pr = 0; pr < 3; pr++) {
							uint32_t a = qa[pa[pr]] + kb * 16384 + kk * 32, bb = ka[pb[pr]] + kb * 8192 + kk * 32;
							tc_mma_f16(d, sw128_kmajor_desc(a), sw128_kmajor_desc(bb), idS, acc);
							acc = 1;
						}
				tc_commit(&B->s_full[j & 1]);
				tc_commit(&B->kl_empty);
				tc_commit(&B->kfree[j & 1]);
			};
			auto issue_pv = [&](int j) {
				tc_fence_after();
				const uint32_t pa2[2] = { base + FB_SP, base + FB_SP + 16384 };
				const uint32_t va[2] = { base + FB_VH + (uint32_t)(j & 1) * 16384, base + FB_VL };
				const int pa[3] = { 0, 0, 1 }, pb[3] = { 0, 1, 0 };
				for (int kk = 0; kk < 4; kk++) // 16 keys per MMA: two 8-key atoms of 1024 bytes
					for (int pr = 0; pr < 3; pr++) {
						uint32_t a = pa2[pa[pr]] + kk * 32, bb = va[pb[pr]] + kk * 2048;
						tc_mma_f16(tmem + 128, sw128_kmajor_desc(a), sw128_mnmajor_desc(bb, 8192, 1024), idO,
							   (j > 0 || kk > 0 || pr > 0) ? 1u : 0u);
					}
				tc_commit(&B->p_empty);
				tc_commit(&B->vl_empty);
				tc_commit(&B->vfree[j & 1]);
			};
			// S_j and P_j.V_j in the order their operands become ready (as in k_attn_prefill_tc)
			int ns = 0, npv = 0;
			long long idle0 = clock64();
			for (uint32_t spins = 0; ok && npv < nkt;) {
				bool did = false;
				if (ns < nkt && mbar_try(&B->k_full, ns & 1) && (ns < 2 || mbar_try(&B->s_free[ns & 1], ((ns >> 1) - 1) & 1))) {
					issue_s(ns++);
					did = true;
				}
				if (npv < ns && mbar_try(&B->v_full, npv & 1) && mbar_try(&B->p_full, npv & 1)) {
					issue_pv(npv++);
					did = true;
				}
				if (did) {
					idle0 = clock64();
					spins = 0;
				} else if ((++spins & 63) == 0) {
					if (*(volatile int *)&B->abort) {
						ok = false;
					} else if (clock64() - idle0 > WAIT_CYCLES) {
						if (status) *(volatile int *)status = ST_TIMEOUT_FULL;
						*(volatile int *)&B->abort = 1;
						ok = false;
					}
				}
			}
			// every MMA issued has completed before TMEM is released (also after an abort)
			tc_commit(&B->done);
			mbar_wait(&B->done, 0, status, ST_TIMEOUT_ACC);
		}
		__syncwarp();
	} else {
		// ---------------- softmax / epilogue (warps 0-7) ----------------
		// Every softmax warp takes part in every exchange barrier (bar.sync 2, one per tile
		// and one at the end) whether or not its waits succeeded, so a wait that gives up
		// cannot leave its partner warp at a barrier; after a failed wait a warp only keeps
		// the barrier count.
		const int qw = warp & 3, hf = warp >> 2;  // TMEM lane quarter; key (and O) column half
		const int row = qw * 32 + lane;           // TMEM lane, query q0 + row
		const int qi = q0 + row;
		const uint32_t lane_base = tmem + ((uint32_t)(qw * 32) << 16);
		float m_ref = -INFINITY, l = 0.0f;
		bool ok = true;
		for (int j = 0; j < nkt; j++) {
			const int k0 = j * FA_K + hf * 32;
			float sc[32];
			float *rm = red + (j & 1) * 256;
			if (ok) ok = fb_wait_warp(B, &B->s_full[j & 1], (j >> 1) & 1, status);
			if (ok) {
				tc_fence_after();
#pragma unroll
				for (int c = 0; c < 2; c++) {
					float v[16];
					tmem_ld16(lane_base + (uint32_t)((j & 1) * FA_K + hf * 32 + c * 16), v);
#pragma unroll
					for (int e = 0; e < 16; e++) sc[c * 16 + e] = v[e];
				}
				tc_fence_before();
				mbar_arrive_warp(&B->s_free[j & 1]);
				float mx[8];
#pragma unroll
				for (int c = 0; c < 32; c++) {
					const int kj = k0 + c;
					float v = kj <= qi && kj < T ? __fmul_rn(sc[c], scale) : -INFINITY;
					sc[c] = v;
					mx[c & 7] = c < 8 ? v : fmaxf(mx[c & 7], v); // eight independent chains
				}
				rm[hf * 128 + row] = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
							   fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
			}
			asm volatile("bar.sync 2, 256;" ::: "memory"); // the row's maximum over both halves
			if (!ok) continue;
			const float mt = fmaxf(rm[row], rm[128 + row]);
			const bool raise = mt > m_ref + FA_RESCALE;
			const float m_new = raise ? mt : m_ref;
			if (j > 0 && !(ok = fb_wait_warp(B, &B->p_empty, (j - 1) & 1, status))) continue;
			if (__any_sync(0xffffffffu, raise && m_ref != -INFINITY)) {
				// O holds P.V of tiles < j at the old reference max: rescale this half in place
				tc_fence_after();
				const float f = raise && m_ref != -INFINITY ? __expf(m_ref - m_new) : 1.0f;
#pragma unroll 1
				for (int c = 0; c < 4; c++) {
					float v[16];
					tmem_ld16(lane_base + 128 + hf * 64 + c * 16, v);
#pragma unroll
					for (int e = 0; e < 16; e++) v[e] *= f;
					tmem_st16(lane_base + 128 + hf * 64 + c * 16, v);
				}
				tmem_wait_st();
				l *= f;
			}
			m_ref = m_new;
			float sm8[8];
#pragma unroll
			for (int c = 0; c < 32; c++) {
				float p = sc[c] == -INFINITY ? 0.0f : __expf(sc[c] - m_ref);
				sc[c] = p;
				sm8[c & 7] = c < 8 ? p : sm8[c & 7] + p; // eight independent chains
			}
			l += ((sm8[0] + sm8[1]) + (sm8[2] + sm8[3])) + ((sm8[4] + sm8[5]) + (sm8[6] + sm8[7]));
			uint8_t *pb = sm + FB_SP;
#pragma unroll
			for (int c = 0; c < 4; c++) {
				float x[8];
#pragma unroll
				for (int e = 0; e < 8; e++) x[e] = sc[c * 8 + e];
				uint4 hi, lo;
				fa_split8(x, hi, lo);
				*(uint4 *)(pb + fa_sw(row, hf * 4 + c)) = hi;
				*(uint4 *)(pb + 16384 + fa_sw(row, hf * 4 + c)) = lo;
			}
			fence_async_smem();
			tc_fence_before();
			mbar_arrive_warp(&B->p_full);
		}
		if (ok) ok = fb_wait_warp(B, &B->p_empty, (nkt - 1) & 1, status);
		// the row's sum over both halves, in the exchange buffer no warp reads any more (every
		// warp has passed the last tile's barrier, so all reads of the tile before it are done)
		float *rs = red + (nkt & 1) * 256;
		rs[hf * 128 + row] = l;
		asm volatile("bar.sync 2, 256;" ::: "memory");
		const float lt = rs[row] + rs[128 + row];
		if (ok) {
			tc_fence_after();
			const float inv = 1.0f / lt;
			const long ob = ((long)s * T + qi) * (long)NQ * FA_HD + (long)h * FA_HD + hf * 64;
#pragma unroll 1
			for (int c = 0; c < 4; c++) {
				float v[16];
				tmem_ld16(lane_base + 128 + hf * 64 + c * 16, v);
				if (qi < T) {
#pragma unroll
					for (int half = 0; half < 2; half++) {
						float x[8];
#pragma unroll
						for (int e = 0; e < 8; e++) x[e] = v[half * 8 + e] * inv;
						uint4 hi, lo;
						fa_split8(x, hi, lo);
						*(uint4 *)(ohi + ob + c * 16 + half * 8) = hi;
						*(uint4 *)(olo + ob + c * 16 + half * 8) = lo;
					}
				}
			}
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 12) {
		tc_fence_after();
		tmem_dealloc(tmem, 256);
	}
}

} // namespace tgc
