// gemm_sm100.cu -- the tensor-core dequant GEMM: D[M,N] = sum over operand pairs
// of A_i[M,K] B_j[N,K]^T, bf16 operands, f32 accumulation in TMEM (tcgen05).
//
// Why pairs: weight codes (int8 / int4) are exact in bf16, activations are not.
// An f32 activation is split into hi = bf16(a) and lo = bf16(a - hi); summing
// hi*C + lo*C reproduces the f32 product to ~2^-17 relative, which keeps the
// reference's f32 dequant path (runtime/tg_rt.h:132-151) within 1e-3/1e-4.
// Weights whose scale cannot stay in the epilogue (per-head o_proj scales) are
// pre-scaled and split too, and use hi*hi + hi*lo + lo*hi.
//
// Kernel: 10 warps. Warp 0 lane 0 issues TMA tile loads (128-byte swizzle, K
// blocks of 64) into a STAGES-deep shared-memory ring; warp 1 owns the TMEM
// accumulator (BN f32 columns) and lane 0 issues tcgen05.mma (M=128, N=BN,
// K=16 per instruction), committing each stage back to the producer; warps 2-9
// expand integer codes into the ring (in-kernel dequant only); warps 2-5 drain
// TMEM with tcgen05.ld and run the epilogue (scale, residual add, SwiGLU with a
// bf16 hi/lo split of the result). Every mbarrier wait is bounded and reports
// into a device status word instead of hanging. The persistent variant below
// keeps 6 warps (bf16 operands only).
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace tgc {

constexpr int BM = 128, BK = 64;
constexpr int A_TILE = BM * BK * 2; // 16 KB

struct TmaMaps {
	CUtensorMap a[2], b[2];
	CUtensorMap o[2]; // the output (SwiGLU: the bf16 hi and lo outputs), when p.tma_out
	CUtensorMap c;    // raw codes (p.cside): uint8 [rows, K * bits / 8], unswizzled boxes
	CUtensorMap cpf;  // the same codes in boxes of 256 bytes per row, for L2 prefetches
};

__device__ __forceinline__ uint32_t bf16_bits(float x) { return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x)); }
// two bf16 in one word, a in the low half (the lower K index)
__device__ __forceinline__ uint32_t bf16x2(float a, float b) { return bf16_bits(a) | (bf16_bits(b) << 16); }
// row rr of a 128-byte-swizzled K-major tile: rows of 128 bytes, 8-row atoms of 1024 bytes
__device__ __forceinline__ uint8_t *smem_row(uint8_t *tile, int rr) { return tile + rr * 128; }

// Integer codes -> bf16 without int-to-float conversions. int4: the nibble n of code c
// (n ^ 8 = c + 8, 0..15) below the bf16 pattern of 128.0 reads as 128 + c + 8, exact with
// bf16's 8-bit significand; one packed bf16 subtraction of 136 leaves c, two codes at a
// time. int8: the byte b (b ^ 0x80 = c + 128) below the f32 pattern of 2^23 reads as
// 2^23 + c + 128; subtracting 2^23 + 128 leaves c, whose f32 pattern truncates exactly to
// bf16 (|c| <= 128 needs 8 significant bits).
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b)
{
	uint32_t d;
	asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
	return d;
}
// 8 int4 codes of one word (code 2e in bits 8e..8e+3, 2e+1 in bits 8e+4..8e+7) -> 4 bf16 pairs
__device__ __forceinline__ void int4x8_bf16(uint32_t w, uint32_t h[4])
{
	const uint32_t lo = (w & 0x0F0F0F0Fu) ^ 0x08080808u, hi = ((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
#pragma unroll
	for (int e = 0; e < 4; e++) {
		const uint32_t t = __byte_perm(lo, hi, e | ((4 + e) << 8)) & 0x00FF00FFu; // [lo byte e, -, hi byte e, -]
		h[e] = bf16x2_sub(t | 0x43004300u, 0x43084308u);
	}
}
// 4 int8 codes of one word -> 2 bf16 pairs
__device__ __forceinline__ void int8x4_bf16(uint32_t w, uint32_t h[2])
{
	const uint32_t x = w ^ 0x80808080u;
	float f[4];
#pragma unroll
	for (int e = 0; e < 4; e++) f[e] = __fsub_rn(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540u | e)), 8388736.0f);
	h[0] = __byte_perm(__float_as_uint(f[0]), __float_as_uint(f[1]), 0x7632u);
	h[1] = __byte_perm(__float_as_uint(f[2]), __float_as_uint(f[3]), 0x7632u);
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(320, 1) gemm_tc(const __grid_constant__ TmaMaps maps, const GemmArgs p)
{
	extern __shared__ uint8_t smem_raw[];
	uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
	constexpr int B_TILE = BN * BK * 2;
	const int ops_bytes = p.na * A_TILE + p.nb * B_TILE;
	const int stage_bytes = ops_bytes + p.raw_bytes; // operand tiles, then the raw codes (cside)
	uint64_t *full = (uint64_t *)(smem + STAGES * stage_bytes);
	uint64_t *empty = full + STAGES;
	uint64_t *rawf = empty + STAGES; // raw codes of the stage landed (cside)
	uint64_t *accf = rawf + STAGES;
	uint32_t *tslot = (uint32_t *)(accf + 1);
	float *ssc = (float *)(accf + 2); // BN floats: the tile's scales (SwiGLU: gate then up)
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
	const int kbytes = p.cbits == 8 ? BK : BK / 2; // code bytes per row of a K block
	// split-K (EPI_PARTIAL): this CTA takes K blocks [kb0, kb0 + KB) and stores its raw sums
	const int KBall = (p.K + BK - 1) / BK;
	const int kb0 = p.kb_per_split ? blockIdx.z * p.kb_per_split : 0;
	const int KB = p.kb_per_split ? min(p.kb_per_split, KBall - kb0) : KBall;

	if (threadIdx.x == 0) {
		for (int s = 0; s < STAGES; s++) {
			mbar_init(&full[s], p.cside ? 1 + 8 : 1); // + one arrival per converting warp
			mbar_init(&empty[s], 1);
			mbar_init(&rawf[s], 1);
		}
		mbar_init(accf, 1);
		fence_barrier_init();
		for (int i = 0; i < p.na; i++)
			if (!(i == 0 && p.cside == 1)) tma_prefetch_desc(&maps.a[i]);
		for (int i = 0; i < p.nb; i++)
			if (!(p.cside == 2 && (i == 0 || p.cscale))) tma_prefetch_desc(&maps.b[i]);
		if (p.cside) {
			tma_prefetch_desc(&maps.c);
			tma_prefetch_desc(&maps.cpf);
		}
	}
	if (warp == 1) tmem_alloc(tslot, BN);
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = *tslot;
	pdl_wait(); // the kernel before it (with programmatic launch) has completed: inputs ready
	pdl_launch();

	if (warp == 0 && lane == 0) { // ---- producer
		// the codes of this CTA's whole K range into L2 up front, 256 contiguous bytes per row
		// per request: the stage loads below (one K block of 32 or 64 bytes per row) then hit L2
		if (p.cside)
			for (int x = kb0 * kbytes; x < (kb0 + KB) * kbytes; x += 256)
				tma_prefetch_l2_2d(&maps.cpf, x, p.cside == 1 ? m0 : n0);
		for (int kb = 0; kb < KB; kb++) {
			const int s = kb % STAGES;
			const uint32_t ph = (kb / STAGES) & 1;
			if (!mbar_wait(&empty[s], ph ^ 1, p.status, ST_TIMEOUT_EMPTY)) break;
			uint8_t *st = smem + s * stage_bytes;
			if (p.cside) { // the raw codes first: the converting warps start on them
				mbar_expect_tx(&rawf[s], p.raw_bytes);
				tma_load_2d(st + ops_bytes, &maps.c, &rawf[s], (kb0 + kb) * kbytes, p.cside == 1 ? m0 : n0);
			}
			const int cb = p.cside == 2 ? (p.cscale ? 2 : 1) : 0; // B tiles the converters build
			mbar_expect_tx(&full[s], ops_bytes - (p.cside == 1 ? A_TILE : cb * B_TILE));
			for (int i = p.cside == 1 ? 1 : 0; i < p.na; i++) tma_load_2d(st + i * A_TILE, &maps.a[i], &full[s], (kb0 + kb) * BK, m0);
			for (int j = cb; j < p.nb; j++)
				tma_load_2d(st + p.na * A_TILE + j * B_TILE, &maps.b[j], &full[s], (kb0 + kb) * BK, n0);
		}
	} else if (warp == 1 && lane == 0) { // ---- MMA issuer
		constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
		int issued = 0;
		for (int kb = 0; kb < KB; kb++) {
			const int s = kb % STAGES;
			const uint32_t ph = (kb / STAGES) & 1;
			if (!mbar_wait(&full[s], ph, p.status, ST_TIMEOUT_FULL)) break;
			tc_fence_after();
			const uint32_t base = smem_u32(smem + s * stage_bytes);
			for (int q = 0; q < p.npairs; q++) {
				const uint32_t a = base + p.pa[q] * A_TILE, b = base + p.na * A_TILE + p.pb[q] * B_TILE;
#pragma unroll
				for (int kk = 0; kk < BK / 16; kk++) {
					tc_mma_f16(tmem, sw128_kmajor_desc(a + kk * 32), sw128_kmajor_desc(b + kk * 32), idesc, issued);
					issued = 1;
				}
			}
			tc_commit(&empty[s]);
		}
		tc_commit(accf);
	} else if (warp >= 2) { // ---- warps 2-9 expand codes (cside); 2-5 then run the epilogue
		const int quarter = warp & 3;
		const int r = quarter * 32 + lane; // tile row = TMEM lane
		const int row = m0 + r;
		const int et = threadIdx.x - 64;   // 0..127 over the epilogue warps, 0..255 over the converters
		const bool epi_warp = warp < 6;
		// scales of this tile into shared memory while the main loop runs
		if (!epi_warp) {
		} else if (EPI == EPI_SWIGLU) {
			const int f0 = blockIdx.x * (BN / 2);
			for (int j = et; j < BN / 2; j += 128) {
				ssc[j] = p.scale[f0 + j];
				ssc[BN / 2 + j] = p.scale2[f0 + j];
			}
		} else if (p.scale_mode == 2) {
			for (int j = et; j < BN; j += 128) ssc[j] = n0 + j < p.N ? p.scale[n0 + j] : 0.0f;
		} else if (p.scale_mode == 1) {
			ssc[et] = m0 + et < p.M ? p.scale[m0 + et] : 0.0f;
		}
		if (p.cside) {
			// Expand the raw codes of every K block (TMA'd into the end of its ring stage) into
			// the stage's code operand: exact bf16 in the 128-byte-swizzled K-major layout. Rows
			// past the matrix arrive as zero bytes (TMA's out-of-bounds fill), which expand to
			// code 0. The stage's raw codes landing implies the producer saw the stage free, so
			// the operand slot may be written.
			// Each of the 256 threads owns up to 4 chunks of a block; all are read before any is
			// converted, so the conversions of different chunks overlap.
			const int R = p.cside == 1 ? BM : BN;
			const int cpr = kbytes / 16;                // 16-byte code chunks per row of a K block
			const int chunks = R * cpr;                 // per K block, 128 .. 1024
			for (int kb = 0; kb < KB; kb++) {
				const int s = kb % STAGES;
				const uint32_t ph = (kb / STAGES) & 1;
				if (!__all_sync(0xffffffffu, mbar_wait(&rawf[s], ph, p.status, ST_TIMEOUT_FULL))) break; // the warp leaves together
				uint8_t *stg = smem + s * stage_bytes;
				uint8_t *slot = stg + (p.cside == 1 ? 0 : p.na * A_TILE);
				const uint8_t *raw = stg + ops_bytes;
				uint4 vv[4];
				float sc[4];
#pragma unroll
				for (int i = 0; i < 4; i++) {
					const int it = et + i * 256;
					if (it < chunks) {
						vv[i] = *(const uint4 *)(raw + it * 16);
						if (p.cscale) { // the scale of this chunk's row in this K block's group
							const int n = n0 + it / cpr;
							sc[i] = n < p.N ? p.cscale[(long)((kb0 + kb) * BK / p.cgroup) * p.cscale_ld + n] : 0.0f;
						}
					}
				}
#pragma unroll
				for (int i = 0; i < 4; i++) {
					const int it = et + i * 256;
					if (it >= chunks) break;
					const int rr = it / cpr, c = it % cpr, sw = rr & 7;
					uint8_t *dst = smem_row(slot, rr);
					const uint4 v = vv[i];
					const uint32_t w[4] = { v.x, v.y, v.z, v.w };
					if (p.cscale) {
						// hi and lo of code * scale (f32, rounded once), as the load-time split
						// of the same product: hi into B[0], lo into B[1] at the same offsets
						uint8_t *dlo = dst + B_TILE;
						const int upw = p.cbits == 8 ? 2 : 4;   // bf16 pairs per code word
						const int u0 = p.cbits == 8 ? 2 * c : 4 * c; // first 16-byte unit
#pragma unroll
						for (int j = 0; j < 4; j++) {
							uint32_t h[4];
							if (p.cbits == 8) int8x4_bf16(w[j], h);
							else int4x8_bf16(w[j], h);
							uint32_t hh[4], ll[4];
#pragma unroll
							for (int e = 0; e < 4; e++) {
								if (e >= upw) break;
								const float a = __fmul_rn(__uint_as_float(h[e] << 16), sc[i]);
								const float b = __fmul_rn(__uint_as_float(h[e] & 0xFFFF0000u), sc[i]);
								const uint32_t ah = bf16_bits(a), bh = bf16_bits(b);
								hh[e] = ah | (bh << 16);
								ll[e] = bf16_bits(__fsub_rn(a, __uint_as_float(ah << 16))) |
									(bf16_bits(__fsub_rn(b, __uint_as_float(bh << 16))) << 16);
							}
							if (p.cbits == 8) { // word j = codes 4j..4j+3: half of unit u0 + j / 2
								const int off = (((u0 + (j >> 1)) ^ sw) << 4) + (j & 1) * 8;
								*(uint2 *)(dst + off) = make_uint2(hh[0], hh[1]);
								*(uint2 *)(dlo + off) = make_uint2(ll[0], ll[1]);
							} else {
								const int off = ((u0 + j) ^ sw) << 4;
								*(uint4 *)(dst + off) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
								*(uint4 *)(dlo + off) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
							}
						}
					} else if (p.cbits == 8) { // 16 codes -> swizzle units 2c, 2c + 1
						uint32_t h[8];
#pragma unroll
						for (int j = 0; j < 4; j++) int8x4_bf16(w[j], h + 2 * j);
						*(uint4 *)(dst + (((2 * c) ^ sw) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
						*(uint4 *)(dst + (((2 * c + 1) ^ sw) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
					} else { // 32 codes -> units 4c .. 4c + 3, one 32-bit word (8 codes) each
#pragma unroll
						for (int j = 0; j < 4; j++) {
							uint32_t h[4];
							int4x8_bf16(w[j], h);
							*(uint4 *)(dst + (((4 * c + j) ^ sw) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
						}
					}
				}
				fence_async_smem();
				mbar_arrive_warp(&full[s]);
			}
		}
		if (epi_warp) {
		epilogue_sync();
		const bool ok = mbar_wait(accf, 0, p.status, ST_TIMEOUT_ACC);
		const bool live = ok && row < p.M;
		tc_fence_after();
		const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
		if (EPI == EPI_SWIGLU) {
			// columns come in blocks of 64: 32 gate channels, then the matching 32 up channels.
			// The results (bf16 hi, lo) are staged in the idle ring as 128-byte-swizzled
			// chunks of 64 channels, then written by TMA stores (direct stores when BN = 64).
			const int f0 = blockIdx.x * (BN / 2);
			for (int c = 0; c < BN / 2; c += 32) {
				float g[32], u[32];
				__syncwarp();
				tmem_ld16(trow + 2 * c, *(float(*)[16])g);
				tmem_ld16(trow + 2 * c + 16, *(float(*)[16])(g + 16));
				tmem_ld16(trow + 2 * c + 32, *(float(*)[16])u);
				tmem_ld16(trow + 2 * c + 48, *(float(*)[16])(u + 16));
				uint32_t hi[16], lo[16];
#pragma unroll
				for (int i = 0; i < 32; i++) {
					float gs = g[i] * ssc[c + i], us = u[i] * ssc[BN / 2 + c + i];
					float y = __fmul_rn(__fdiv_rn(gs, __fadd_rn(1.0f, expf(-gs))), us); // silu(g) * u
					uint32_t h = bf16_bits(y);
					uint32_t l = bf16_bits(y - __uint_as_float(h << 16));
					if (i & 1) {
						hi[i >> 1] |= h << 16;
						lo[i >> 1] |= l << 16;
					} else {
						hi[i >> 1] = h;
						lo[i >> 1] = l;
					}
				}
				if (p.tma_out) {
					const int chunk = c / 64, unit0 = (c % 64) / 8; // 32 channels = 64 bytes = 4 units
					uint8_t *rh = smem + chunk * 16384 + r * 128, *rl = smem + (2 + chunk) * 16384 + r * 128;
#pragma unroll
					for (int q = 0; q < 4; q++) {
						const int pu = ((unit0 + q) ^ (r & 7)) * 16;
						*(uint4 *)(rh + pu) = make_uint4(hi[4 * q], hi[4 * q + 1], hi[4 * q + 2], hi[4 * q + 3]);
						*(uint4 *)(rl + pu) = make_uint4(lo[4 * q], lo[4 * q + 1], lo[4 * q + 2], lo[4 * q + 3]);
					}
				} else if (live) {
					const long off = (long)row * p.ldo + f0 + c;
					uint4 *dh = (uint4 *)(p.out_hi + off), *dl = (uint4 *)(p.out_lo + off);
#pragma unroll
					for (int q = 0; q < 4; q++) {
						dh[q] = make_uint4(hi[4 * q], hi[4 * q + 1], hi[4 * q + 2], hi[4 * q + 3]);
						dl[q] = make_uint4(lo[4 * q], lo[4 * q + 1], lo[4 * q + 2], lo[4 * q + 3]);
					}
				}
			}
			if (p.tma_out) {
				fence_async_smem();
				epilogue_sync();
				if (et == 0 && ok) {
					for (int h = 0; h < BN / 128; h++) {
						tma_store_2d(&maps.o[0], smem + h * 16384, f0 + 64 * h, m0);
						tma_store_2d(&maps.o[1], smem + (2 + h) * 16384, f0 + 64 * h, m0);
					}
					tma_store_commit();
					tma_store_wait_read();
				}
			}
		} else if (p.tma_out) {
			// f32 result in 128-byte-swizzled chunks of 32 columns, written (or added into the
			// output, EPI_ADD) by TMA; rows past M and columns past N are clipped by the map
			for (int c = 0; c < BN; c += 32) {
				float v[32];
				__syncwarp();
				tmem_ld16(trow + c, *(float(*)[16])v);
				tmem_ld16(trow + c + 16, *(float(*)[16])(v + 16));
				const float rs = p.scale_mode == 1 ? ssc[r] : 1.0f;
#pragma unroll
				for (int i = 0; i < 32; i++) {
					if (p.scale_mode == 1) v[i] = __fmul_rn(rs, v[i]);
					else if (p.scale_mode == 2) v[i] = __fmul_rn(ssc[c + i], v[i]);
				}
				uint8_t *rp = smem + (c / 32) * 16384 + r * 128;
#pragma unroll
				for (int q = 0; q < 8; q++)
					*(float4 *)(rp + ((q ^ (r & 7)) * 16)) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
			}
			fence_async_smem();
			epilogue_sync();
			if (et == 0 && ok) {
				// EPI_PARTIAL: the split's own padded row block of the partial-sum buffer
				const int y0 = EPI == EPI_PARTIAL ? (int)(blockIdx.z * p.mpad) + m0 : m0;
				for (int c = 0; c < BN; c += 32) {
					if (n0 + c >= p.N) break;
					if (EPI == EPI_ADD) tma_reduce_add_2d(&maps.o[0], smem + (c / 32) * 16384, n0 + c, y0);
					else tma_store_2d(&maps.o[0], smem + (c / 32) * 16384, n0 + c, y0);
				}
				tma_store_commit();
				tma_store_wait_read();
			}
		} else {
			// direct stores, for outputs TMA cannot address (row pitch not a multiple of 16 bytes)
			for (int c = 0; c < BN; c += 16) {
				float v[16];
				__syncwarp();
				tmem_ld16(trow + c, v);
				if (!live) continue;
				const int n = n0 + c;
				float *dst = p.out + (long)row * p.ldo + n;
				const float rs = p.scale_mode == 1 ? ssc[r] : 1.0f;
#pragma unroll
				for (int i = 0; i < 16; i++) {
					float x = v[i];
					if (p.scale_mode == 1) x = __fmul_rn(rs, x);
					else if (p.scale_mode == 2 && n + i < p.N) x = __fmul_rn(ssc[c + i], x);
					v[i] = x;
				}
				for (int i = 0; i < 16 && n + i < p.N; i++) dst[i] = EPI == EPI_ADD ? __fadd_rn(dst[i], v[i]) : v[i];
			}
		}
		tc_fence_before();
		}
	}
	__syncthreads();
	if (warp == 1) {
		tc_fence_after();
		tmem_dealloc(tmem, BN);
	}
}

// ---- persistent variant: one CTA per SM walks many tiles ----------------------------------
// The accumulator is double-buffered in TMEM (2 x BN columns): while the epilogue warps drain
// tile i from one buffer, the MMA warp accumulates tile i + 1 into the other, and the
// producer's ring runs on across tile boundaries. The epilogue stages its output in a
// dedicated 32 KB buffer (two 16 KB halves: f32 chunks of 32 columns alternate between them;
// a SwiGLU chunk of 64 channels uses both, bf16 hi then lo) and writes it by TMA store or
// reduce-add. Tiles go column-block by column-block (m fastest), so the CTAs running at the
// same time share the weight tile. Bf16 operands only, no split-K, outputs through TMA.
constexpr int PSTG = 32768;

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(192, 1) gemm_tc_persistent(const __grid_constant__ TmaMaps maps, const GemmArgs p)
{
	extern __shared__ uint8_t smem_raw[];
	uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
	constexpr int B_TILE = BN * BK * 2;
	const int stage_bytes = p.na * A_TILE + p.nb * B_TILE;
	uint8_t *stg = smem + STAGES * stage_bytes; // 1024-aligned: stage_bytes is a multiple of 1024
	uint8_t *aux = stg + PSTG;
	uint64_t *full = (uint64_t *)aux;
	uint64_t *empty = full + STAGES;
	uint64_t *acc_full = empty + STAGES; // [2]
	uint64_t *acc_empty = acc_full + 2;  // [2]
	uint32_t *tslot = (uint32_t *)(acc_empty + 2);
	float *ssc = (float *)(aux + 256);   // max(BN, BM) scales of the current tile
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int mtiles = (p.M + BM - 1) / BM, ntiles = (p.N + BN - 1) / BN, tiles = mtiles * ntiles;
	const int KB = (p.K + BK - 1) / BK;

	if (threadIdx.x == 0) {
		for (int s = 0; s < STAGES; s++) {
			mbar_init(&full[s], 1);
			mbar_init(&empty[s], 1);
		}
		for (int b = 0; b < 2; b++) {
			mbar_init(&acc_full[b], 1);
			mbar_init(&acc_empty[b], 4); // one arrival per epilogue warp
		}
		fence_barrier_init();
		for (int i = 0; i < p.na; i++) tma_prefetch_desc(&maps.a[i]);
		for (int i = 0; i < p.nb; i++) tma_prefetch_desc(&maps.b[i]);
		tma_prefetch_desc(&maps.o[0]);
	}
	if (warp == 1) tmem_alloc(tslot, 2 * BN);
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = *tslot;

	if (warp == 0 && lane == 0) { // ---- producer
		int it = 0;
		for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
			const int m0 = (t % mtiles) * BM, n0 = (t / mtiles) * BN;
			bool ok = true;
			for (int kb = 0; kb < KB; kb++, it++) {
				const int s = it % STAGES;
				const uint32_t ph = (it / STAGES) & 1;
				if (!(ok = mbar_wait(&empty[s], ph ^ 1, p.status, ST_TIMEOUT_EMPTY))) break;
				uint8_t *st = smem + s * stage_bytes;
				mbar_expect_tx(&full[s], stage_bytes);
				for (int i = 0; i < p.na; i++) tma_load_2d(st + i * A_TILE, &maps.a[i], &full[s], kb * BK, m0);
				for (int j = 0; j < p.nb; j++) tma_load_2d(st + p.na * A_TILE + j * B_TILE, &maps.b[j], &full[s], kb * BK, n0);
			}
			if (!ok) break;
		}
	} else if (warp == 1 && lane == 0) { // ---- MMA issuer
		constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
		int it = 0, i = 0;
		bool ok = true;
		for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, i++) {
			const int b = i & 1;
			if (!(ok = mbar_wait(&acc_empty[b], ((i >> 1) & 1) ^ 1, p.status, ST_TIMEOUT_ACC))) break;
			tc_fence_after();
			const uint32_t d = tmem + (uint32_t)(b * BN);
			int issued = 0;
			for (int kb = 0; kb < KB; kb++, it++) {
				const int s = it % STAGES;
				const uint32_t ph = (it / STAGES) & 1;
				if (!(ok = mbar_wait(&full[s], ph, p.status, ST_TIMEOUT_FULL))) break;
				tc_fence_after();
				const uint32_t base = smem_u32(smem + s * stage_bytes);
				for (int q = 0; q < p.npairs; q++) {
					const uint32_t a = base + p.pa[q] * A_TILE, bb = base + p.na * A_TILE + p.pb[q] * B_TILE;
#pragma unroll
					for (int kk = 0; kk < BK / 16; kk++) {
						tc_mma_f16(d, sw128_kmajor_desc(a + kk * 32), sw128_kmajor_desc(bb + kk * 32), idesc, issued);
						issued = 1;
					}
				}
				tc_commit(&empty[s]);
			}
			tc_commit(&acc_full[b]);
		}
	} else if (warp >= 2) { // ---- epilogue: TMEM lanes of quarter (warp % 4)
		const int quarter = warp & 3;
		const int r = quarter * 32 + lane; // tile row = TMEM lane
		const int et = threadIdx.x - 64;   // 0..127
		int i = 0, chunk = 0;
		bool ok = true;
		for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, i++) {
			const int m0 = (t % mtiles) * BM, n0 = (t / mtiles) * BN, b = i & 1;
			epilogue_sync(); // the previous tile's readers of ssc are done
			if (EPI == EPI_SWIGLU) {
				const int f0 = (t / mtiles) * (BN / 2);
				for (int j = et; j < BN / 2; j += 128) {
					ssc[j] = p.scale[f0 + j];
					ssc[BN / 2 + j] = p.scale2[f0 + j];
				}
			} else if (p.scale_mode == 2) {
				for (int j = et; j < BN; j += 128) ssc[j] = n0 + j < p.N ? p.scale[n0 + j] : 0.0f;
			} else if (p.scale_mode == 1) {
				ssc[et] = m0 + et < p.M ? p.scale[m0 + et] : 0.0f;
			}
			// one thread waits for the accumulator and the barrier hands the outcome to all 128, so
			// they leave the loop together (the named barriers below need every one of them)
			volatile int *flag = (volatile int *)(aux + 192);
			if (et == 0) *flag = mbar_wait(&acc_full[b], (i >> 1) & 1, p.status, ST_TIMEOUT_ACC) ? 1 : 0;
			epilogue_sync();
			if (!(ok = *flag != 0)) break;
			tc_fence_after();
			const uint32_t trow = tmem + (uint32_t)(b * BN) + ((uint32_t)(quarter * 32) << 16);
			if (EPI == EPI_SWIGLU) {
				// 64 output channels per chunk: two blocks of 32 gate + 32 up columns; hi goes to the
				// first half of the staging buffer, lo to the second, each 128-byte swizzled
				const int f0 = (t / mtiles) * (BN / 2);
				for (int c = 0; c < BN / 2; c += 64) {
					if (et == 0) tma_store_wait_read();
					epilogue_sync();
					for (int hf = 0; hf < 2; hf++) {
						const int cc = c + 32 * hf;
						float g[32], u[32];
						__syncwarp();
						tmem_ld16(trow + 2 * cc, *(float(*)[16])g);
						tmem_ld16(trow + 2 * cc + 16, *(float(*)[16])(g + 16));
						tmem_ld16(trow + 2 * cc + 32, *(float(*)[16])u);
						tmem_ld16(trow + 2 * cc + 48, *(float(*)[16])(u + 16));
						uint32_t hi[16], lo[16];
#pragma unroll
						for (int k = 0; k < 32; k++) {
							float gs = g[k] * ssc[cc + k], us = u[k] * ssc[BN / 2 + cc + k];
							float y = __fmul_rn(__fdiv_rn(gs, __fadd_rn(1.0f, expf(-gs))), us); // silu(g) * u
							uint32_t h = bf16_bits(y);
							uint32_t l = bf16_bits(y - __uint_as_float(h << 16));
							if (k & 1) {
								hi[k >> 1] |= h << 16;
								lo[k >> 1] |= l << 16;
							} else {
								hi[k >> 1] = h;
								lo[k >> 1] = l;
							}
						}
						uint8_t *rh = stg + r * 128, *rl = stg + 16384 + r * 128;
#pragma unroll
						for (int q = 0; q < 4; q++) {
							const int pu = ((4 * hf + q) ^ (r & 7)) * 16;
							*(uint4 *)(rh + pu) = make_uint4(hi[4 * q], hi[4 * q + 1], hi[4 * q + 2], hi[4 * q + 3]);
							*(uint4 *)(rl + pu) = make_uint4(lo[4 * q], lo[4 * q + 1], lo[4 * q + 2], lo[4 * q + 3]);
						}
					}
					fence_async_smem();
					epilogue_sync();
					if (et == 0) {
						tma_store_2d(&maps.o[0], stg, f0 + c, m0);
						tma_store_2d(&maps.o[1], stg + 16384, f0 + c, m0);
						tma_store_commit();
					}
				}
			} else {
				for (int c = 0; c < BN; c += 32, chunk++) {
					uint8_t *buf = stg + (chunk & 1) * 16384;
					if (et == 0) tma_store_wait_read1(); // the store that last read this half is done
					epilogue_sync();
					float v[32];
					__syncwarp();
					tmem_ld16(trow + c, *(float(*)[16])v);
					tmem_ld16(trow + c + 16, *(float(*)[16])(v + 16));
					const float rs = p.scale_mode == 1 ? ssc[r] : 1.0f;
#pragma unroll
					for (int k = 0; k < 32; k++) {
						if (p.scale_mode == 1) v[k] = __fmul_rn(rs, v[k]);
						else if (p.scale_mode == 2) v[k] = __fmul_rn(ssc[c + k], v[k]);
					}
					uint8_t *rp = buf + r * 128;
#pragma unroll
					for (int q = 0; q < 8; q++)
						*(float4 *)(rp + ((q ^ (r & 7)) * 16)) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
					fence_async_smem();
					epilogue_sync();
					if (et == 0) {
						if (n0 + c < p.N) {
							if (EPI == EPI_ADD) tma_reduce_add_2d(&maps.o[0], buf, n0 + c, m0);
							else tma_store_2d(&maps.o[0], buf, n0 + c, m0);
						}
						tma_store_commit(); // (an empty group when the chunk is past N)
					}
				}
			}
			tc_fence_before();
			mbar_arrive_warp(&acc_empty[b]); // this warp's TMEM loads of buffer b are complete
		}
		if (et == 0) tma_store_wait_all();
	}
	__syncthreads();
	if (warp == 1) {
		tc_fence_after();
		tmem_dealloc(tmem, 2 * BN);
	}
}

// ---- host ----------------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_encode()
{
	static std::once_flag once;
	static int rc = TG_CUDA_OK;
	std::call_once(once, [] {
		cudaDriverEntryPointQueryResult q;
		void *fn = nullptr;
		cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
		if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) rc = TG_CUDA_ECUDA;
		else g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
	});
	if (rc) return set_err(rc, "cuTensorMapEncodeTiled is not available from the driver");
	return TG_CUDA_OK;
}

// bf16 [rows, K] K-major (row stride ld elements), box of 64 x box_rows, 128-byte swizzle.
static int make_map(CUtensorMap *m, const void *base, long rows, long K, long ld, int box_rows)
{
	if (((uintptr_t)base & 15) || (ld * 2) % 16) return set_err(TG_CUDA_EINVAL, "TMA operand not 16-byte aligned (ld %ld)", ld);
	cuuint64_t dims[2] = { (cuuint64_t)K, (cuuint64_t)rows };
	cuuint64_t strides[1] = { (cuuint64_t)(ld * 2) };
	cuuint32_t box[2] = { (cuuint32_t)BK, (cuuint32_t)box_rows };
	cuuint32_t es[2] = { 1, 1 };
	CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)base, dims, strides, box, es,
			      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
			      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
	if (r != CUDA_SUCCESS) return set_err(TG_CUDA_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
	return TG_CUDA_OK;
}

// f32 or bf16 [rows, cols] output (row pitch ld elements), box of box_x x 128 rows, 128-byte swizzle.
int bf16_tile_map(CUtensorMap *m, const void *base, long rows, long K, long ld, int box_rows)
{
	int rc = get_encode();
	return rc ? rc : make_map(m, base, rows, K, ld, box_rows);
}

static int make_out_map(CUtensorMap *m, CUtensorMapDataType dt, int esize, const void *base, long rows, long cols, long ld,
			int box_x)
{
	cuuint64_t dims[2] = { (cuuint64_t)cols, (cuuint64_t)rows };
	cuuint64_t strides[1] = { (cuuint64_t)(ld * esize) };
	cuuint32_t box[2] = { (cuuint32_t)box_x, 128u };
	cuuint32_t es[2] = { 1, 1 };
	CUresult r = g_encode(m, dt, 2, (void *)base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
			      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
	if (r != CUDA_SUCCESS) return set_err(TG_CUDA_ECUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
	return TG_CUDA_OK;
}

// Raw int8 / int4 codes [rows, K * bits / 8] bytes (row pitch ld bytes), boxes of one K block
// (64 codes) x box_rows rows, unswizzled: a row of the box is 32 or 64 contiguous bytes.
static int make_codes_map(CUtensorMap *m, const void *base, long rows, long row_bytes, long ld, int kbytes, int box_rows)
{
	if (((uintptr_t)base & 15) || ld % 16) return set_err(TG_CUDA_EINVAL, "code rows not 16-byte aligned (ld %ld)", ld);
	cuuint64_t dims[2] = { (cuuint64_t)row_bytes, (cuuint64_t)rows };
	cuuint64_t strides[1] = { (cuuint64_t)ld };
	cuuint32_t box[2] = { (cuuint32_t)kbytes, (cuuint32_t)box_rows };
	cuuint32_t es[2] = { 1, 1 };
	CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
			      CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
	if (r != CUDA_SUCCESS) return set_err(TG_CUDA_ECUDA, "cuTensorMapEncodeTiled (codes) failed (%d)", (int)r);
	return TG_CUDA_OK;
}

template <int BN, int STAGES, int EPI>
static int launch_bn(const TmaMaps &maps, const GemmArgs &p, cudaStream_t st)
{
	int stage = p.na * A_TILE + p.nb * BN * BK * 2 + p.raw_bytes;
	size_t smem = (size_t)STAGES * stage + 1024 + 256 + BN * 4; // ring, alignment, barriers, scales
	static bool attr_set[64] = {};
	int dev;
	cudaGetDevice(&dev);
	if (!attr_set[dev]) {
		cudaFuncSetAttribute(gemm_tc<BN, STAGES, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
		attr_set[dev] = true;
	}
	dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, p.kb_per_split ? (unsigned)(((p.K + BK - 1) / BK + p.kb_per_split - 1) / p.kb_per_split) : 1u);
	if (p.pdl) {
		TGC_CUDA(launch_pdl(gemm_tc<BN, STAGES, EPI>, grid, dim3(320), smem, st, maps, p));
	} else {
		gemm_tc<BN, STAGES, EPI><<<grid, 320, smem, st>>>(maps, p);
		TGC_LAUNCH_CHECK();
	}
	return TG_CUDA_OK;
}

template <int BN, int STAGES, int EPI>
static int launch_persistent(const TmaMaps &maps, const GemmArgs &p, int grid, cudaStream_t st)
{
	const int stage = p.na * A_TILE + p.nb * BN * BK * 2;
	const size_t smem = (size_t)STAGES * stage + PSTG + 1024 + 256 + 1024; // ring, staging, alignment, barriers, scales
	static bool attr_set[64] = {};
	int dev;
	cudaGetDevice(&dev);
	if (!attr_set[dev]) {
		cudaFuncSetAttribute(gemm_tc_persistent<BN, STAGES, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
		attr_set[dev] = true;
	}
	if (smem > 232448) return set_err(TG_CUDA_EINVAL, "gemm: persistent tiles do not fit shared memory");
	gemm_tc_persistent<BN, STAGES, EPI><<<grid, 192, smem, st>>>(maps, p);
	TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

static int launch_split(int BN, int stages, const TmaMaps &maps, const GemmArgs &q, dim3, cudaStream_t st)
{
	if (BN == 32) return stages >= 6 ? launch_bn<32, 6, EPI_PARTIAL>(maps, q, st) : launch_bn<32, 4, EPI_PARTIAL>(maps, q, st);
	if (BN == 64) return launch_bn<64, 4, EPI_PARTIAL>(maps, q, st);
	if (BN == 256)
		return stages >= 4 ? launch_bn<256, 4, EPI_PARTIAL>(maps, q, st)
		       : stages == 3 ? launch_bn<256, 3, EPI_PARTIAL>(maps, q, st) : launch_bn<256, 2, EPI_PARTIAL>(maps, q, st);
	return stages >= 4 ? launch_bn<128, 4, EPI_PARTIAL>(maps, q, st)
	       : stages == 3 ? launch_bn<128, 3, EPI_PARTIAL>(maps, q, st) : launch_bn<128, 2, EPI_PARTIAL>(maps, q, st);
}

// Fixed-order sum of the split-K partials, then the epilogue the split GEMM skipped.
template <int EPI>
__global__ void k_split_reduce(const float *__restrict__ part, int splits, long mpad, int M, int N, GemmArgs p)
{
	pdl_wait();
	pdl_launch();
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	const int outc = EPI == EPI_SWIGLU ? N / 2 : N;
	if (t >= (long)M * outc) return;
	const int m = (int)(t / outc), n = (int)(t % outc);
	if (EPI == EPI_SWIGLU) {
		const int gc = (n / 32) * 64 + n % 32, uc = gc + 32;
		float g = 0.0f, u = 0.0f;
		for (int z = 0; z < splits; z++) {
			g += part[((long)z * mpad + m) * N + gc];
			u += part[((long)z * mpad + m) * N + uc];
		}
		float gs = g * p.scale[n], us = u * p.scale2[n];
		float y = __fmul_rn(__fdiv_rn(gs, __fadd_rn(1.0f, expf(-gs))), us);
		__nv_bfloat16 h = __float2bfloat16_rn(y);
		p.out_hi[(long)m * p.ldo + n] = h;
		p.out_lo[(long)m * p.ldo + n] = __float2bfloat16_rn(y - __bfloat162float(h));
		return;
	}
	float v = 0.0f;
	for (int z = 0; z < splits; z++) v += part[((long)z * mpad + m) * N + n];
	if (p.scale_mode == 2) v = __fmul_rn(p.scale[n], v);
	else if (p.scale_mode == 1) v = __fmul_rn(p.scale[m], v);
	float *o = p.out + (long)m * p.ldo + n;
	*o = EPI == EPI_ADD ? __fadd_rn(*o, v) : v;
}

int gemm(const GemmOperands &ops, GemmArgs p, cudaStream_t st)
{
	int rc = get_encode();
	if (rc) return rc;
	if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.na < 1 || p.na > 2 || p.nb < 1 || p.nb > 2 || p.npairs < 1 || p.npairs > 4)
		return set_err(TG_CUDA_EINVAL, "gemm: bad shape or operand count");
	if (p.K % 8) return set_err(TG_CUDA_EINVAL, "gemm: K %d is not a multiple of 8", p.K);
	if (p.cside && (p.cside > 2 || !p.codes || (p.cbits != 8 && p.cbits != 4) || p.K % BK || p.cld % 16 ||
			((uintptr_t)p.codes & 15) || (p.cside == 1 && p.pa[0] != 0 && p.na < 1)))
		return set_err(TG_CUDA_EINVAL, "gemm: in-kernel dequant needs K %% 64 == 0 and 16-byte aligned code rows");
	if (p.cscale && (p.cside != 2 || p.nb != 2 || p.cgroup <= 0 || p.cgroup % BK || p.cscale_ld < p.N))
		return set_err(TG_CUDA_EINVAL, "gemm: scaled dequant needs the codes as B, two B operands and K groups of 64k");
	int sms = 148, dev = 0;
	cudaGetDevice(&dev);
	cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
	// Small batches (decode): tiles of 64 columns when the wide tiles would leave most SMs idle;
	// each CTA then streams a narrower slab of the weights and no K split may be needed.
	const long mtiles = (p.M + BM - 1) / BM;
	int BN = p.epi == EPI_SWIGLU || p.N >= 256 ? 256 : 128;
	if (((p.N + BN - 1) / BN) * mtiles * 2 <= sms && p.N % 64 == 0 && mtiles <= (p.wide ? 1 : 4)) BN = 64;
	if (p.N <= 32 && p.epi != EPI_SWIGLU) BN = 32; // a batch of up to 32 (drop-in axis 0): one narrow MMA
	// In-kernel dequant adds the raw code block to each stage; keep at least 3 stages of
	// TMA in flight rather than the widest tile
	const int kbytes = p.cbits == 8 ? BK : BK / 2;
	auto stage_of = [&](int bn) { return p.na * A_TILE + p.nb * bn * BK * 2 + (p.cside ? (p.cside == 1 ? BM : bn) * kbytes : 0); };
	if (p.cside && BN == 256 && p.epi != EPI_SWIGLU && (220 * 1024) / stage_of(256) < 3) BN = 128;
	p.raw_bytes = p.cside ? (p.cside == 1 ? BM : BN) * kbytes : 0;
	TmaMaps maps;
	memset(&maps, 0, sizeof maps);
	if (p.cside &&
	    ((rc = make_codes_map(&maps.c, p.codes, p.cside == 1 ? p.M : p.N, (long)p.K * p.cbits / 8, p.cld, kbytes, p.cside == 1 ? BM : BN)) ||
	     (rc = make_codes_map(&maps.cpf, p.codes, p.cside == 1 ? p.M : p.N, (long)p.K * p.cbits / 8, p.cld,
				  (int)std::min<long>(256, (long)p.K * p.cbits / 8), p.cside == 1 ? BM : BN))))
		return rc;
	for (int i = 0; i < p.na; i++)
		if (!(i == 0 && p.cside == 1) && (rc = make_map(&maps.a[i], ops.a[i], p.M, p.K, ops.lda, BM))) return rc;
	for (int j = 0; j < p.nb; j++)
		if (!(p.cside == 2 && (j == 0 || p.cscale)) && (rc = make_map(&maps.b[j], ops.b[j], p.N, p.K, ops.ldb, BN))) return rc;
	// as many ring stages (2..4; 6 for the narrow tile) as fit in 220 KB of shared memory
	const int stage = stage_of(BN);
	const int stages = std::min(BN == 32 ? 6 : 4, std::max(2, (220 * 1024) / stage));
	// Split K when the tiles would leave most SMs idle (small-batch decode): each split stores raw
	// f32 sums into the caller's partial buffer, then k_split_reduce adds them in a fixed order.
	const long tiles = (long)((p.N + BN - 1) / BN) * ((p.M + BM - 1) / BM);
	const int KBall = (p.K + BK - 1) / BK;
	int splits = 1;
	if (p.partial && tiles * 2 <= sms && KBall >= 8 && p.N % 4 == 0) {
		// one wave: the ring takes most of an SM's shared memory, so one CTA per SM
		splits = (int)std::min<long>(sms / tiles, KBall / 4);
		const long mpad = (long)(p.M + BM - 1) / BM * BM;
		while (splits > 1 && (long)splits * mpad * p.N > p.partial_floats) splits--;
	}
	if (splits > 1) {
		const int kper = (KBall + splits - 1) / splits;
		splits = (KBall + kper - 1) / kper;
		GemmArgs q = p;
		q.kb_per_split = kper;
		q.mpad = (long)(p.M + BM - 1) / BM * BM;
		q.epi = EPI_PARTIAL;
		q.scale_mode = 0;
		if (stages * stage < 128 * BN * 4) return set_err(TG_CUDA_EINVAL, "gemm: split tile does not fit the ring");
		if ((rc = make_out_map(&maps.o[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.partial, q.mpad * splits, p.N, p.N, 32)))
			return rc;
		q.tma_out = 1;
		dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, splits);
		if ((rc = launch_split(BN, stages, maps, q, grid, st))) return rc;
		const long outs = (long)p.M * (p.epi == EPI_SWIGLU ? p.N / 2 : p.N);
		const unsigned blocks = (unsigned)((outs + 255) / 256);
		auto reduce = p.epi == EPI_SWIGLU ? k_split_reduce<EPI_SWIGLU> : p.epi == EPI_ADD ? k_split_reduce<EPI_ADD>
											     : k_split_reduce<EPI_STORE>;
		if (p.pdl) {
			TGC_CUDA(launch_pdl(reduce, dim3(blocks), dim3(256), 0, st, (const float *)p.partial, splits, q.mpad, p.M, p.N, p));
		} else {
			reduce<<<blocks, 256, 0, st>>>(p.partial, splits, q.mpad, p.M, p.N, p);
			TGC_LAUNCH_CHECK();
		}
		return TG_CUDA_OK;
	}
	// the output goes through TMA when its pitch and base allow; the tile is staged in the
	// ring once the main loop has drained it (128 rows x BN f32, or 4 bf16 chunks of 16 KB)
	p.tma_out = 0;
	if (p.epi == EPI_SWIGLU) {
		if (BN >= 128 && (p.ldo * 2) % 16 == 0 && !((uintptr_t)p.out_hi & 15) && !((uintptr_t)p.out_lo & 15) &&
		    (p.N / 2) % 64 == 0 && stages * stage >= 4 * 16384) {
			if ((rc = make_out_map(&maps.o[0], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.out_hi, p.M, p.N / 2, p.ldo, 64)) ||
			    (rc = make_out_map(&maps.o[1], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.out_lo, p.M, p.N / 2, p.ldo, 64)))
				return rc;
			p.tma_out = 1;
		}
	} else if ((p.ldo * 4) % 16 == 0 && !((uintptr_t)p.out & 15) && stages * stage >= 128 * BN * 4) {
		if ((rc = make_out_map(&maps.o[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.out, p.M, p.N, p.ldo, 32))) return rc;
		p.tma_out = 1;
	}
	if (stages * stage > 220 * 1024) return set_err(TG_CUDA_EINVAL, "gemm: %d operand tiles do not fit", p.na + p.nb);
	// More tiles than SMs, bf16 operands, a TMA-addressable output: the persistent kernel, whose
	// epilogue overlaps the next tile's main loop
	if (!p.cside && p.tma_out && BN >= 128 && tiles > sms) {
		const int pst = std::min(4, (int)((232448 - 1024 - 256 - 1024 - PSTG) / stage));
		const int grid = (int)std::min<long>(tiles, sms);
		if (pst >= 2) {
#define TGC_GEMM_PERSIST(E)                                                                            \
	if (BN == 256) return pst >= 3 ? launch_persistent<256, 3, E>(maps, p, grid, st) : launch_persistent<256, 2, E>(maps, p, grid, st); \
	return pst >= 4 ? launch_persistent<128, 4, E>(maps, p, grid, st) : launch_persistent<128, 3, E>(maps, p, grid, st);
			if (pst >= 3 || BN == 256) {
				if (p.epi == EPI_SWIGLU) {
					TGC_GEMM_PERSIST(EPI_SWIGLU)
				}
				if (p.epi == EPI_ADD) {
					TGC_GEMM_PERSIST(EPI_ADD)
				}
				TGC_GEMM_PERSIST(EPI_STORE)
			}
#undef TGC_GEMM_PERSIST
		}
	}
#define TGC_GEMM_NARROW(E) \
	if (BN == 32) return stages >= 6 ? launch_bn<32, 6, E>(maps, p, st) : launch_bn<32, 4, E>(maps, p, st);
#define TGC_GEMM_DISPATCH(E)                                                                 \
	if (BN == 64) return launch_bn<64, 4, E>(maps, p, st); /* 40-48 KB stages: always 4 */ \
	if (BN == 256)                                                                      \
		return stages >= 4 ? launch_bn<256, 4, E>(maps, p, st)                      \
		       : stages == 3 ? launch_bn<256, 3, E>(maps, p, st) : launch_bn<256, 2, E>(maps, p, st); \
	return stages >= 4 ? launch_bn<128, 4, E>(maps, p, st)                              \
	       : stages == 3 ? launch_bn<128, 3, E>(maps, p, st) : launch_bn<128, 2, E>(maps, p, st);
	if (p.epi == EPI_SWIGLU) {
		TGC_GEMM_DISPATCH(EPI_SWIGLU)
	}
	if (p.epi == EPI_ADD) {
		TGC_GEMM_NARROW(EPI_ADD)
		TGC_GEMM_DISPATCH(EPI_ADD)
	}
	TGC_GEMM_NARROW(EPI_STORE)
	TGC_GEMM_DISPATCH(EPI_STORE)
#undef TGC_GEMM_NARROW
#undef TGC_GEMM_DISPATCH
}

// ---- conversions feeding the GEMM ------------------------------------------------------------

// f32 [rows, cols] (row stride lds) -> bf16 hi/lo, optionally transposed: dst[c, r] (K-major for B).
__global__ void split_f32(const float *__restrict__ src, long rows, long cols, long lds, int transpose,
			  __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo, long ldd)
{
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (t >= rows * cols) return;
	long r = t / cols, c = t % cols;
	float x = src[r * lds + c];
	__nv_bfloat16 h = __float2bfloat16_rn(x);
	__nv_bfloat16 l = __float2bfloat16_rn(x - __bfloat162float(h));
	long d = transpose ? c * ldd + r : r * ldd + c;
	hi[d] = h;
	if (lo) lo[d] = l;
}

// Codes of a [rows, cols] matrix in the reference packing -> bf16 (exact), optionally transposed.
__global__ void codes_bf16(const signed char *__restrict__ q, int bits, long rows, long cols, int transpose,
			   __nv_bfloat16 *__restrict__ dst, long ldd)
{
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (t >= rows * cols) return;
	long r = t / cols, c = t % cols;
	float v = (float)qcode(q, bits, t);
	dst[transpose ? c * ldd + r : r * ldd + c] = __float2bfloat16_rn(v);
}

// The transposed split through 32 x 32 shared-memory tiles: reads along src rows and
// writes along dst rows are both coalesced.
__global__ void split_f32_t(const float *__restrict__ src, long rows, long cols, long lds, __nv_bfloat16 *__restrict__ hi,
			    __nv_bfloat16 *__restrict__ lo, long ldd)
{
	__shared__ float tile[32][33];
	const long r0 = (long)blockIdx.y * 32, c0 = (long)blockIdx.x * 32;
	for (int i = threadIdx.y; i < 32; i += blockDim.y) {
		long r = r0 + i, c = c0 + threadIdx.x;
		tile[i][threadIdx.x] = r < rows && c < cols ? src[r * lds + c] : 0.0f;
	}
	__syncthreads();
	for (int i = threadIdx.y; i < 32; i += blockDim.y) {
		long c = c0 + i, r = r0 + threadIdx.x; // dst[c, r] = src[r, c]
		if (c >= cols || r >= rows) continue;
		float x = tile[threadIdx.x][i];
		__nv_bfloat16 h = __float2bfloat16_rn(x);
		hi[c * ldd + r] = h;
		if (lo) lo[c * ldd + r] = __float2bfloat16_rn(x - __bfloat162float(h));
	}
}

int split_to_bf16(const float *src, long rows, long cols, long lds, bool transpose, __nv_bfloat16 *hi, __nv_bfloat16 *lo,
		  long ldd, cudaStream_t st)
{
	long n = rows * cols;
	if (transpose && (rows + 31) / 32 <= 65535) {
		dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
		split_f32_t<<<grid, dim3(32, 8), 0, st>>>(src, rows, cols, lds, hi, lo, ldd);
		TGC_LAUNCH_CHECK();
		return TG_CUDA_OK;
	}
	split_f32<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, rows, cols, lds, transpose ? 1 : 0, hi, lo, ldd);
	TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

int codes_to_bf16(const signed char *q, int bits, long rows, long cols, bool transpose, __nv_bfloat16 *dst, long ldd,
		  cudaStream_t st)
{
	long n = rows * cols;
	codes_bf16<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(q, bits, rows, cols, transpose ? 1 : 0, dst, ldd);
	TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

// ---- tg_cuda_matmul_q, large batch -------------------------------------------------------------

// The drop-in call stays asynchronous: the kernels' status word is a pinned, mapped host
// word that a wait which timed out writes directly, and a later call on the device reports
// it (call_status_word; shared with the GEMV of gemv_bulk.cuh).
struct TcScratch {
	DevBuf buf, part;        // part: split-K partial sums of small-batch calls (64 MB)
	int *h_status = nullptr; // pinned, mapped: the kernels' status word (written only by a wait that timed out)
	int *d_status = nullptr; // its device address
};
static TcScratch g_tc[64];

int device_status_check(int *d_status, cudaStream_t st)
{
	int h = 0;
	cudaError_t e = cudaMemcpyAsync(&h, d_status, sizeof h, cudaMemcpyDeviceToHost, st);
	if (e == cudaSuccess) e = cudaStreamSynchronize(st);
	if (e != cudaSuccess) return set_err(TG_CUDA_ECUDA, "status read: %s", cudaGetErrorString(e));
	if (h) return set_err(TG_CUDA_EDEVICE, "a tensor-core kernel gave up waiting (status %d)", h);
	return TG_CUDA_OK;
}

int call_status_word(int dev, int **d_status)
{
	TcScratch &S = g_tc[dev];
	if (!S.h_status) {
		TGC_CUDA(cudaHostAlloc((void **)&S.h_status, sizeof(int), cudaHostAllocMapped));
		*S.h_status = 0;
		TGC_CUDA(cudaHostGetDevicePointer((void **)&S.d_status, S.h_status, 0));
	}
	if (int prev = *(volatile int *)S.h_status) { // an earlier call's kernel gave up waiting
		*S.h_status = 0;
		return set_err(TG_CUDA_EDEVICE, "a kernel of an earlier call on this device gave up waiting (status %d)", prev);
	}
	*d_status = S.d_status;
	return TG_CUDA_OK;
}

int matmul_q_tc(int axis, float *o, const float *act, const signed char *q, int bits, const float *s, int m, int k, int n,
		cudaStream_t st, bool *done)
{
	*done = false;
	// batch = columns of b (axis 0) or rows of a (axis 1); the GEMV covers batches up to 8
	if (k % 8) return TG_CUDA_OK;
	int dev;
	cudaGetDevice(&dev);
	TcScratch &S = g_tc[dev];
	long wrows = axis == 0 ? m : n;   // weight channels
	long brows = axis == 0 ? n : m;   // activation rows (batch)
	size_t wbytes = (size_t)wrows * k * 2, abytes = (size_t)brows * k * 2;
	int *d_status = nullptr;
	int rc = call_status_word(dev, &d_status);
	if (rc) return rc;
	if ((rc = S.buf.ensure(wbytes + 2 * abytes + 256, dev))) return rc;
	__nv_bfloat16 *wq = (__nv_bfloat16 *)S.buf.p;
	__nv_bfloat16 *ahi = (__nv_bfloat16 *)((uint8_t *)S.buf.p + ((wbytes + 127) & ~(size_t)127));
	__nv_bfloat16 *alo = (__nv_bfloat16 *)((uint8_t *)ahi + ((abytes + 127) & ~(size_t)127));
	GemmOperands ops;
	GemmArgs p;
	memset(&p, 0, sizeof p);
	p.K = k;
	p.na = 1;
	p.nb = 2;
	p.npairs = 2;
	p.pa[0] = 0, p.pb[0] = 0, p.pa[1] = 0, p.pb[1] = 1;
	p.epi = EPI_STORE;
	p.out = o;
	p.status = d_status; // no per-call reset or copy: a timeout writes the host word directly
	// small batches leave most SMs idle with one tile per weight slab: let gemm() split K
	if ((rc = S.part.ensure((size_t)64 << 20, dev))) return rc;
	p.partial = S.part.as<float>(), p.partial_floats = (long)((64 << 20) / sizeof(float));
	if (axis == 0) {
		// o[m, n] = diag(s) Q[m, k] b[k, n]: A = codes [m, k], B = b^T [n, k] split. The codes
		// rows are K-major already: the kernel expands them itself when the K blocks are whole.
		if (k % 64 == 0 && !((uintptr_t)q & 15)) {
			p.codes = q, p.cbits = bits, p.cside = 1, p.cld = (long)k * bits / 8;
		} else if ((rc = codes_to_bf16(q, bits, m, k, false, wq, k, st))) {
			return rc;
		}
		if ((rc = split_to_bf16(act, k, n, n, true, ahi, alo, k, st))) return rc;
		ops.a[0] = wq, ops.b[0] = ahi, ops.b[1] = alo;
		p.M = m, p.N = n, p.ldo = n, p.scale = s, p.scale_mode = 1;
	} else {
		// o[m, n] = a[m, k] Q[k, n] diag(s): A = a split, B = codes^T [n, k]
		if ((rc = codes_to_bf16(q, bits, k, n, true, wq, k, st))) return rc;
		if ((rc = split_to_bf16(act, m, k, k, false, ahi, alo, k, st))) return rc;
		ops.a[0] = ahi, ops.a[1] = alo, ops.b[0] = wq;
		p.na = 2, p.nb = 1;
		p.pa[0] = 0, p.pb[0] = 0, p.pa[1] = 1, p.pb[1] = 0;
		p.M = m, p.N = n, p.ldo = n, p.scale = s, p.scale_mode = 2;
	}
	ops.lda = k, ops.ldb = k;
	if ((rc = gemm(ops, p, st))) return rc;
	*done = true;
	return TG_CUDA_OK;
}

} // namespace tgc
