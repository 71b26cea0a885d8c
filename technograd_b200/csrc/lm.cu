// lm.cu -- decoder language models of the Qwen3 import (examples/qwen3/import.py:90-132)
// on the device: batched prefill and greedy decode with a per-sequence KV cache.
//
// The reference runs this program per sequence in the VM: per-head rank-2
// tg_matmul_qb calls (x @ W, axis-1 int8/int4 codes with per-column scales),
// rmsnorm then `* weight`, rotate-half RoPE through cos/sin tables and a
// rotation matrix, softmax((q k^T) * scale + mask), (s v) @ Wo per head summed
// into the residual, a SwiGLU MLP, and the LM head on every row followed by
// take(lastidx). Here the same arithmetic runs for many sequences at once:
//
//   weights  converted once at load: codes -> exact bf16 in [out, in] K-major
//            layout for the tcgen05 GEMM (q/k/v heads concatenated into one
//            matrix; gate/up interleaved in 32-row blocks so every GEMM tile
//            holds matching gate and up channels); o_proj pre-scaled by its
//            per-head column scales and split into bf16 hi/lo.
//   layer    rmsnorm*ln1 (split to bf16 hi/lo) -> QKV GEMM -> q/k rmsnorm*w +
//            RoPE, k/v into the KV cache -> causal attention (prefill) or
//            KV-cache attention (decode), output split hi/lo -> Wo GEMM added
//            into the residual -> rmsnorm*ln2 -> gate/up GEMM with SwiGLU in
//            its epilogue -> down GEMM added into the residual.
//   head     rmsnorm*lnf of the last position only (take(lastidx) discards the
//            other rows), LM-head GEMM, argmax for greedy decode.
//
// KV cache: [layer][slot][kv head][position][head_dim], each f32 key/value kept in 3
// bytes (its bf16 rounding and a byte of remainder, kv.cuh). Sequences run in
// waves of at most max_seqs per device; the prefill of a wave runs in chunks
// of at most PREFILL_ROWS tokens.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <memory>
#include <thread>
#include <vector>

#include "kv.cuh"
#include "attn_tc.cuh"
#include "common.cuh"
#include "gemm.cuh"
#include "gemv_dec.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace tgc {

constexpr long PREFILL_ROWS = 16384;

__device__ __forceinline__ void split_bf16(float y, __nv_bfloat16 &h, __nv_bfloat16 &l)
{
	h = __float2bfloat16_rn(y);
	l = __float2bfloat16_rn(y - __bfloat162float(h));
}

// ---- weight conversion ----------------------------------------------------------------------

// Gate and up [D, FF] codes -> interleaved [2 FF, D]: block b = rows 64b.. holds gate
// channels 32b..32b+31 then the same up channels, so every GEMM tile of 64 or more
// columns holds matching gate and up channels.
__global__ void k_codes_gu(const signed char *__restrict__ qg, const signed char *__restrict__ qu, int bits, int D, int FF,
			   __nv_bfloat16 *__restrict__ dst)
{
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (t >= 2L * D * FF) return;
	int which = (int)(t / ((long)D * FF));
	long e = t % ((long)D * FF); // element of the [D, FF] source
	int p = (int)(e / FF), f = (int)(e % FF);
	float v = (float)qcode(which ? qu : qg, bits, e);
	long row = (long)(f / 32) * 64 + which * 32 + f % 32;
	dst[row * D + p] = __float2bfloat16_rn(v);
}

// [K, N] codes (x @ W layout, int4 two per flat index pair, low nibble first) -> K-major rows
// of codes packed the same way: source column n becomes row row0 + (n / blk) * 2 blk + off +
// n % blk (blk = N: row row0 + n; blk 32 with off 0 / 32: the gate/up interleave of k_codes_gu).
// One thread per output byte. These rows feed the small-batch GEMV and the GEMM's in-kernel
// dequant.
__global__ void k_codes_T(const signed char *__restrict__ q, int bits, long K, long N, long blk, long off, long row0,
			  uint8_t *__restrict__ dst, long ld)
{
	const long kbytes = bits == 8 ? K : K / 2;
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (t >= N * kbytes) return;
	const long n = t / kbytes, j = t % kbytes;
	const long row = row0 + (n / blk) * 2 * blk + off + n % blk;
	uint8_t b;
	if (bits == 8) b = (uint8_t)q[j * N + n];
	else b = (uint8_t)((qcode(q, 4, 2 * j * N + n) & 15) | ((qcode(q, 4, (2 * j + 1) * N + n) & 15) << 4));
	dst[row * ld + j] = b;
}

// o_proj: stacked per-head codes [NQ*HD, D] with scales s[h*D + n] -> B[n][h*HD + p] =
// code * s, split hi/lo (the dequantized value the program's param holds, src/ir.c:503-507).
__global__ void k_wo_prescale(const signed char *__restrict__ q, const float *__restrict__ s, int bits, int KO, int HD,
			      int D, __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo)
{
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (t >= (long)KO * D) return;
	int r = (int)(t / D), n = (int)(t % D), h = r / HD;
	float v = __fmul_rn((float)qcode(q, bits, t), s[(long)h * D + n]);
	__nv_bfloat16 a, b;
	split_bf16(v, a, b);
	hi[(long)n * KO + r] = a;
	lo[(long)n * KO + r] = b;
}

// ---- per-token kernels ----------------------------------------------------------------------

// SwiGLU of the small-batch GEMV's gate/up sums [M][2 FF] (rows in k_codes_gu's interleaved
// order) with the per-channel scales, split to bf16 hi/lo [M][FF]: the arithmetic of the
// GEMM's SwiGLU epilogue on the same sums.
__global__ void k_swiglu_split(const float *__restrict__ gu, long M, int FF, const float *__restrict__ sg,
			       const float *__restrict__ su, __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo)
{
	pdl_wait(); // programmatic dependent launch inside the decode step (no-op otherwise)
	pdl_launch();
	const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (t >= M * FF) return;
	const long j = t / FF;
	const int f = (int)(t % FF);
	const float *r = gu + j * 2 * FF + (f / 32) * 64 + f % 32;
	const float gs = r[0] * sg[f], us = r[32] * su[f];
	split_bf16(__fmul_rn(__fdiv_rn(gs, __fadd_rn(1.0f, expf(-gs))), us), hi[t], lo[t]); // silu(g) * u
}

// h[r] = E[round(ids[r])] or zeros out of range (take, runtime/tg_rt.h:316-322). One warp per row.
__global__ void k_embed(const float *__restrict__ ids, const int *__restrict__ tok, long M, const float *__restrict__ E,
			int V, int D, float *__restrict__ h)
{
	pdl_wait(); // programmatic dependent launch inside the decode step (no-op otherwise)
	pdl_launch();
	long r = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
	int lane = threadIdx.x & 31;
	if (r >= M) return;
	int t;
	if (tok) t = tok[r];
	else {
		float x = floorf(ids[r] + 0.5f);
		t = x >= 0.0f && x < (float)V ? (int)x : -1;
	}
	t = t >= 0 && t < V ? t : -1;
	const float4 *src = (const float4 *)(E + (long)(t < 0 ? 0 : t) * D);
	float4 *dst = (float4 *)(h + r * D);
	for (int i = lane; i < D / 4; i += 32) dst[i] = t >= 0 ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
}

// y = rmsnorm(x) * w (runtime/tg_rt.h:165-175 then the broadcast mul), split to bf16 hi/lo.
// One warp per output row; src row = rowmap ? rowmap(r) : r (the last position of each sequence).
__global__ void k_rmsnorm_split(const float *__restrict__ x, long M, int D, const float *__restrict__ w, float eps,
				int last_T, __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo)
{
	pdl_wait(); // programmatic dependent launch inside the decode step (no-op otherwise)
	pdl_launch();
	long r = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
	int lane = threadIdx.x & 31;
	if (r >= M) return;
	long src = last_T > 0 ? r * last_T + last_T - 1 : r;
	const float *xr = x + src * D;
	float ss = 0.0f;
	for (int i = lane; i < D; i += 32) ss = fmaf(xr[i], xr[i], ss);
#pragma unroll
	for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
	float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
	for (int i = lane; i < D; i += 32) {
		float y = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
		split_bf16(y, hi[r * D + i], lo[r * D + i]);
	}
}

// Per (row, head) of the QKV projection [M, (NQ + 2 NKV) HD]: q and k heads get
// rmsnorm * qn / kn then rotary(x) = x*cos + rotate_half(x)*sin (import.py:96-97);
// q goes to q_out [seq][NQ][T][HD], k and v into the cache (24-bit elements, kv.cuh) at
// position pos0 + t. One warp per head, 4 dims per lane (HD = 128).
__global__ void k_qk_rope(const float *__restrict__ qkv, long M, int T, int pos0, const int *__restrict__ dpos, int NQ,
			  int NKV, float eps, const float *__restrict__ qn, const float *__restrict__ kn,
			  const float *__restrict__ cosT, const float *__restrict__ sinT, float *__restrict__ q_out,
			  KvPlane kc, KvPlane vc, int slot0, int max_len)
{
	pdl_wait(); // programmatic dependent launch inside the decode step (no-op otherwise)
	pdl_launch();
	constexpr int HD = 128;
	long gw = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
	int lane = threadIdx.x & 31;
	const int H = NQ + 2 * NKV;
	if (gw >= M * H) return;
	long r = gw / H;
	int hh = (int)(gw % H);
	if (dpos) pos0 = *dpos; // decode: the position lives on the device (one graph serves every step)
	int s = (int)(r / T), t = (int)(r % T), pos = pos0 + t;
	float4 x = ((const float4 *)(qkv + r * (long)H * HD + (long)hh * HD))[lane];
	if (hh >= NQ + NKV) { // v head: straight into the cache
		int kvh = hh - NQ - NKV;
		const long e = (((long)(slot0 + s) * NKV + kvh) * max_len + pos) * HD + 4 * lane;
		uint2 h;
		uint32_t q;
		kv_encode4(x, h, q);
		*(uint2 *)(vc.h + e) = h;
		*(uint32_t *)(vc.q + e) = q;
		return;
	}
	const float *w = hh < NQ ? qn : kn;
	float ss = fmaf(x.x, x.x, fmaf(x.y, x.y, fmaf(x.z, x.z, x.w * x.w)));
#pragma unroll
	for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
	float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), eps)));
	float v[4] = { x.x, x.y, x.z, x.w };
#pragma unroll
	for (int e = 0; e < 4; e++) v[e] = __fmul_rn(__fmul_rn(v[e], inv), w[lane * 4 + e]);
	// rotate_half: dims i < 64 take -x[i + 64], dims i >= 64 take x[i - 64] (lane +- 16)
	float o4[4];
#pragma unroll
	for (int e = 0; e < 4; e++) {
		float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
		float rot = lane < 16 ? -partner : partner;
		int d = lane * 4 + e, f = d & (HD / 2 - 1);
		float c = cosT[(long)pos * (HD / 2) + f], sn = sinT[(long)pos * (HD / 2) + f];
		o4[e] = __fadd_rn(__fmul_rn(v[e], c), __fmul_rn(rot, sn));
	}
	float4 res = make_float4(o4[0], o4[1], o4[2], o4[3]);
	if (hh < NQ) {
		((float4 *)(q_out + (((long)s * NQ + hh) * T + t) * HD))[lane] = res;
	} else {
		const long e = (((long)(slot0 + s) * NKV + (hh - NQ)) * max_len + pos) * HD + 4 * lane;
		uint2 h;
		uint32_t q;
		kv_encode4(res, h, q);
		*(uint2 *)(kc.h + e) = h;
		*(uint32_t *)(kc.q + e) = q;
	}
}

// causal attention of the prefill: k_attn_prefill_tc (attn_tc.cuh)

// ---- decode attention over the KV cache -------------------------------------------------------
// CTA = (kv head, sequence); the GRP query heads sharing that kv head are done together.
// Scores: each warp takes every 8th position, a lane holds 4 dims; softmax in shared memory;
// values: each warp accumulates its positions, warps are summed through shared memory.
// Grid (NKV, S, splits). With one split a CTA covers every key and writes the normalised
// output. With more (small waves, whose (kv head, sequence) grid leaves most SMs idle), split
// z covers a range of keys (a multiple of 64) and writes, per query head, its maximum score,
// its sum of exp(score - max) and its unnormalised sum of exp(score - max) * v into split_out
// ([S][NQ][splits][HD + 2]: the HD sums, then max and sum); k_attn_combine finishes.
template <int GRP>
__global__ void __launch_bounds__(256) k_attn_decode(const float *__restrict__ q, KvPlaneC kc, KvPlaneC vc, int len,
						     const int *__restrict__ dpos, int NQ,
						     int NKV, int slot0, int max_len, float scale, __nv_bfloat16 *__restrict__ ohi,
						     __nv_bfloat16 *__restrict__ olo, float *__restrict__ split_out)
{
	pdl_wait(); // programmatic dependent launch inside the decode step (no-op otherwise)
	pdl_launch();
	constexpr int HD = 128;
	constexpr int DU = 8; // positions a warp loads per step (8 x 384 bytes in flight)
	static_assert(DU == 8, "the score butterfly reduces exactly 8 positions");
	extern __shared__ float sm[];
	if (dpos) len = *dpos + 1; // keys 0..pos, the new token's own included
	const int nsp = gridDim.z, sp = blockIdx.z;
	const int chunk = nsp == 1 ? len : ((len + nsp - 1) / nsp + 63) & ~63;
	const int k0 = min(len, sp * chunk), k1 = min(len, k0 + chunk); // this CTA's keys [k0, k1)
	float *sc = sm;                               // [GRP][max_len rounded up]
	float *red = sc + GRP * ((max_len + 3) & ~3); // [8][GRP][HD]
	__shared__ float wmax[8][GRP], wsum[8][GRP];
	const int kvh = blockIdx.x, s = blockIdx.y;
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const long base = (((long)(slot0 + s) * NKV + kvh) * max_len) * HD + 4 * lane; // this lane's 4 dims
	const __nv_bfloat16 *kh = kc.h + base, *vh = vc.h + base;
	const signed char *kq = kc.q + base, *vq = vc.q + base;
	float4 qv[GRP];
#pragma unroll
	for (int g = 0; g < GRP; g++) qv[g] = ((const float4 *)(q + ((long)s * NQ + kvh * GRP + g) * HD))[lane];
	float mx[GRP];
#pragma unroll
	for (int g = 0; g < GRP; g++) mx[g] = -INFINITY;
	for (int p0 = k0 + warp * DU; p0 < k1; p0 += 8 * DU) {
		uint2 khv[DU];
		uint32_t kqv[DU];
#pragma unroll
		for (int u = 0; u < DU; u++) {
			const bool in = p0 + u < k1;
			khv[u] = in ? *(const uint2 *)(kh + (long)(p0 + u) * HD) : make_uint2(0u, 0u);
			kqv[u] = in ? *(const uint32_t *)(kq + (long)(p0 + u) * HD) : 0u;
		}
		float4 kv[DU];
#pragma unroll
		for (int u = 0; u < DU; u++) kv[u] = kv_decode4(khv[u], kqv[u]);
		// The 8 dot products are summed over the warp by a halving butterfly: each exchange
		// keeps half of the values and sends the other half, 9 shuffles for 8 positions (not
		// 40). Lane L ends with position ((L >> 4) & 1) * 4 + ((L >> 3) & 1) * 2 + ((L >> 2) & 1).
		const int pu = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
#pragma unroll
		for (int g = 0; g < GRP; g++) {
			float d[DU];
#pragma unroll
			for (int u = 0; u < DU; u++)
				d[u] = fmaf(qv[g].x, kv[u].x, fmaf(qv[g].y, kv[u].y, fmaf(qv[g].z, kv[u].z, qv[g].w * kv[u].w)));
			float v4[4], v2[2];
#pragma unroll
			for (int i = 0; i < 4; i++) {
				const bool up = lane & 16;
				v4[i] = (up ? d[i + 4] : d[i]) + __shfl_xor_sync(0xffffffffu, up ? d[i] : d[i + 4], 16);
			}
#pragma unroll
			for (int i = 0; i < 2; i++) {
				const bool up = lane & 8;
				v2[i] = (up ? v4[i + 2] : v4[i]) + __shfl_xor_sync(0xffffffffu, up ? v4[i] : v4[i + 2], 8);
			}
			const bool up = lane & 4;
			float v = (up ? v2[1] : v2[0]) + __shfl_xor_sync(0xffffffffu, up ? v2[0] : v2[1], 4);
			v += __shfl_xor_sync(0xffffffffu, v, 2);
			v += __shfl_xor_sync(0xffffffffu, v, 1);
			if (p0 + pu < k1) {
				v = __fmul_rn(v, scale);
				if ((lane & 3) == 0) sc[g * ((max_len + 3) & ~3) + p0 + pu] = v;
				mx[g] = fmaxf(mx[g], v);
			}
		}
	}
#pragma unroll
	for (int g = 0; g < GRP; g++)
#pragma unroll
		for (int o = 16; o; o >>= 1) mx[g] = fmaxf(mx[g], __shfl_xor_sync(0xffffffffu, mx[g], o));
	if (lane == 0)
#pragma unroll
		for (int g = 0; g < GRP; g++) wmax[warp][g] = mx[g];
	__syncthreads();
	float gmax[GRP], gsum[GRP];
#pragma unroll
	for (int g = 0; g < GRP; g++) {
		gmax[g] = wmax[0][g];
		for (int w = 1; w < 8; w++) gmax[g] = fmaxf(gmax[g], wmax[w][g]);
	}
	const int stride = (max_len + 3) & ~3;
	float part[GRP];
#pragma unroll
	for (int g = 0; g < GRP; g++) part[g] = 0.0f;
	for (int p = k0 + threadIdx.x; p < k1; p += 256)
#pragma unroll
		for (int g = 0; g < GRP; g++) {
			float e = expf(sc[g * stride + p] - gmax[g]);
			sc[g * stride + p] = e;
			part[g] += e;
		}
#pragma unroll
	for (int g = 0; g < GRP; g++) {
#pragma unroll
		for (int o = 16; o; o >>= 1) part[g] += __shfl_xor_sync(0xffffffffu, part[g], o);
		if (lane == 0) wsum[warp][g] = part[g];
	}
	__syncthreads();
#pragma unroll
	for (int g = 0; g < GRP; g++) {
		gsum[g] = 0.0f;
		for (int w = 0; w < 8; w++) gsum[g] += wsum[w][g];
	}
	float4 acc[GRP];
#pragma unroll
	for (int g = 0; g < GRP; g++) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
	for (int p0 = k0 + warp * DU; p0 < k1; p0 += 8 * DU) {
		uint2 vhv[DU];
		uint32_t vqv[DU];
#pragma unroll
		for (int u = 0; u < DU; u++) {
			const bool in = p0 + u < k1;
			vhv[u] = in ? *(const uint2 *)(vh + (long)(p0 + u) * HD) : make_uint2(0u, 0u);
			vqv[u] = in ? *(const uint32_t *)(vq + (long)(p0 + u) * HD) : 0u;
		}
		float4 vv[DU];
#pragma unroll
		for (int u = 0; u < DU; u++) vv[u] = kv_decode4(vhv[u], vqv[u]);
#pragma unroll
		for (int u = 0; u < DU; u++) {
			if (p0 + u >= k1) break;
#pragma unroll
			for (int g = 0; g < GRP; g++) {
				float e = sc[g * stride + p0 + u];
				acc[g].x = fmaf(e, vv[u].x, acc[g].x);
				acc[g].y = fmaf(e, vv[u].y, acc[g].y);
				acc[g].z = fmaf(e, vv[u].z, acc[g].z);
				acc[g].w = fmaf(e, vv[u].w, acc[g].w);
			}
		}
	}
#pragma unroll
	for (int g = 0; g < GRP; g++) ((float4 *)(red + ((long)warp * GRP + g) * HD))[lane] = acc[g];
	__syncthreads();
	for (int i = threadIdx.x; i < GRP * HD; i += 256) {
		int g = i / HD, d = i % HD;
		float v = 0.0f;
		for (int w = 0; w < 8; w++) v += red[((long)w * GRP + g) * HD + d];
		if (nsp > 1) { // this split's partial sums (an empty range: max -inf, sums 0)
			float *pp = split_out + (((long)s * NQ + kvh * GRP + g) * nsp + sp) * (HD + 2);
			pp[d] = v;
			if (d == 0) pp[HD] = gmax[g], pp[HD + 1] = gsum[g];
			continue;
		}
		v = v / gsum[g];
		long o = (long)s * NQ * HD + (long)(kvh * GRP + g) * HD + d;
		split_bf16(v, ohi[o], olo[o]);
	}
}

// The splits of k_attn_decode for one (query head, sequence) -- grid (NQ, S), 128 threads, a
// dimension each: with M the largest split maximum, out = sum_z acc_z e^(m_z - M) /
// sum_z l_z e^(m_z - M), summed in split order; then split to bf16 hi/lo as the one-split
// kernel writes it.
__global__ void __launch_bounds__(128) k_attn_combine(const float *__restrict__ part, int nsp, int NQ,
						      __nv_bfloat16 *__restrict__ ohi, __nv_bfloat16 *__restrict__ olo)
{
	pdl_wait(); // programmatic dependent launch inside the decode step (no-op otherwise)
	pdl_launch();
	constexpr int HD = 128;
	const int qh = blockIdx.x, s = blockIdx.y, d = threadIdx.x;
	const float *pp = part + ((long)s * NQ + qh) * nsp * (HD + 2);
	float M = -INFINITY;
	for (int z = 0; z < nsp; z++) M = fmaxf(M, pp[z * (HD + 2) + HD]);
	float L = 0.0f, v = 0.0f;
	for (int z = 0; z < nsp; z++) {
		const float *pz = pp + z * (HD + 2);
		if (pz[HD + 1] == 0.0f) continue; // no keys in this split
		const float w = expf(pz[HD] - M);
		L = fmaf(pz[HD + 1], w, L);
		v = fmaf(pz[d], w, v);
	}
	const long o = ((long)s * NQ + qh) * HD + d;
	split_bf16(v / L, ohi[o], olo[o]);
}

// First index of the row maximum (greedy decode).
__global__ void k_argmax(const float *__restrict__ logits, int V, int *__restrict__ tok, int *__restrict__ out, int ld_out,
			 int col, const int *__restrict__ dpos, int T)
{
	pdl_wait(); // programmatic dependent launch inside the decode step (no-op otherwise)
	pdl_launch();
	if (dpos) col = *dpos - T + 1; // decode: the token fed at position pos yields output column pos - T + 1
	const float *x = logits + (long)blockIdx.x * V;
	float best = -INFINITY;
	int bi = 0x7fffffff;
	if ((V & 3) == 0) { // 16-byte loads, several in flight per thread; each thread scans its indices in order
		const float4 *x4 = (const float4 *)x;
		const int n4 = V >> 2;
		int j = threadIdx.x;
		for (; j + 3 * (int)blockDim.x < n4; j += 4 * blockDim.x) {
			float4 v[4];
#pragma unroll
			for (int u = 0; u < 4; u++) v[u] = x4[j + u * blockDim.x];
#pragma unroll
			for (int u = 0; u < 4; u++) {
				const int i = 4 * (j + u * blockDim.x);
				if (v[u].x > best || (v[u].x == best && i < bi)) best = v[u].x, bi = i;
				if (v[u].y > best || (v[u].y == best && i + 1 < bi)) best = v[u].y, bi = i + 1;
				if (v[u].z > best || (v[u].z == best && i + 2 < bi)) best = v[u].z, bi = i + 2;
				if (v[u].w > best || (v[u].w == best && i + 3 < bi)) best = v[u].w, bi = i + 3;
			}
		}
		for (; j < n4; j += blockDim.x) {
			const float4 v = x4[j];
			const int i = 4 * j;
			if (v.x > best || (v.x == best && i < bi)) best = v.x, bi = i;
			if (v.y > best || (v.y == best && i + 1 < bi)) best = v.y, bi = i + 1;
			if (v.z > best || (v.z == best && i + 2 < bi)) best = v.z, bi = i + 2;
			if (v.w > best || (v.w == best && i + 3 < bi)) best = v.w, bi = i + 3;
		}
	} else {
		for (int i = threadIdx.x; i < V; i += blockDim.x) {
			float v = x[i];
			if (v > best || (v == best && i < bi)) best = v, bi = i;
		}
	}
	__shared__ float sv[32];
	__shared__ int si[32];
#pragma unroll
	for (int o = 16; o; o >>= 1) {
		float v2 = __shfl_xor_sync(0xffffffffu, best, o);
		int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
		if (v2 > best || (v2 == best && i2 < bi)) best = v2, bi = i2;
	}
	int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
	if (lane == 0) sv[w] = best, si[w] = bi;
	__syncthreads();
	if (threadIdx.x == 0) {
		for (int i = 1; i < (int)(blockDim.x >> 5); i++)
			if (sv[i] > best || (sv[i] == best && si[i] < bi)) best = sv[i], bi = si[i];
		if (bi == 0x7fffffff) bi = 0; // all NaN
		tok[blockIdx.x] = bi;
		if (out) out[(long)blockIdx.x * ld_out + col] = bi;
	}
}

// ---- the engine --------------------------------------------------------------------------------

struct Layer {
	DevBuf wqkv, sqkv, wo_hi, wo_lo, wgu, sg, su, wd, sd, ln1, ln2, qn, kn;
	// the same weights as packed codes [out][in] (small batches read these: a quarter (int4) or
	// half (int8) of the bf16 bytes), and o_proj's per-head scales [NQ][D]
	DevBuf cqkv, cgu, cd, co, so;
	CUtensorMap kmap, vmap; // the layer's K and V bf16 cache planes as [slot * NKV * max_len][128] (prefill attention)
};

struct Engine {
	int dev = 0;
	cudaStream_t st = nullptr;
	int L, D, NQ, NKV, HD, FF, V, bits, max_seqs, max_len;
	float eps, scale;
	DevBuf E, lnf, lmw, lms, cosT, sinT;
	DevBuf clm; // LM head codes [V][D] packed
	// Batches of at most gemv_rows rows (decode steps of waves of up to 8 sequences) run the
	// layers' products as dequant GEMVs over the packed codes (gemv_dec); batches of at most
	// codes_rows rows run the tensor-core GEMM with the codes expanded in the kernel; the rest
	// read the bf16 copies. TG_CUDA_GEMV_ROWS / TG_CUDA_CODES_ROWS set them at load.
	long gemv_rows = 8, codes_rows = 0;
	bool codes = false; // packed codes built
	DevBuf gus;         // the GEMV's gate/up sums [gemv_rows][2 FF] before SwiGLU
	// decode attention of small waves split over key ranges (k_attn_decode / k_attn_combine):
	// partial sums [seqs][NQ][splits][HD + 2] for up to split_seqs sequences
	DevBuf apart;
	long split_seqs = 0;
	int sms = 148;
	bool use_gemv(long M) const { return codes && M <= gemv_rows; }
	bool use_codes(long M) const { return codes && M <= codes_rows; }
	std::vector<std::unique_ptr<Layer>> layers;
	DevBuf kh, kq, vh, vq; // the KV cache: bf16 and residual-byte planes (kv.cuh)
	// activations
	long rows_cap = 0;
	DevBuf h, xhi, xlo, qkv, q, ahi, alo, ghi, glo, logits, tok, ids, status, out_tok, part;
	int HQKV() const { return (NQ + 2 * NKV) * HD; }
	// measurements of the current call (tg_cuda_lm_stats)
	bool prof = false;
	long launches = 0;
	cudaEvent_t ev_start = nullptr, ev_end = nullptr;
	struct Mark {
		cudaEvent_t a = nullptr, b = nullptr;
		int cls = 0;
		double work = 0, work_len = 0; // decode attention: bytes = work + work_len * keys
	};
	std::vector<Mark> marks, gmarks; // launched directly / recorded inside the decode graph
	size_t nmarks = 0, ngmarks = 0;
	bool capturing = false;
	tg_cuda_lm_stats acc, last;
	const char *ev_fail = nullptr; // first event call that failed in this call (reported by the API)
	// one decode step (every layer, head, argmax, position bump) as a CUDA graph
	DevBuf dpos; // the position of the token being fed, read by the decode kernels
	int pos_host = 0;
	cudaGraphExec_t gexec = nullptr;
	long g_S = -1, g_kernels = 0;
	int g_T = -1, g_nnew = -1;
	bool g_prof = false;
	bool small_gemm = true; // batches of 129-384 rows on gemm_sk (TG_CUDA_SMALL_GEMM=tile: the tile kernels)
	bool wide_tiles = true; // GemmArgs::wide for the tile kernels (TG_CUDA_WIDE_TILES=0: 64-wide tiles up to 4 M tiles)
	bool prefill_tma = true; // k_attn_prefill_tma (TG_CUDA_PREFILL=staged: k_attn_prefill_tc)
	// while the decode step is captured without profiling marks: kernels are launched with
	// programmatic stream serialization, so each one's launch and prologue overlap the tail of
	// the one before it (every kernel of the step waits for its predecessor, pdl_wait, before
	// it touches memory); TG_CUDA_PDL=0 turns it off
	bool pdl = false, pdl_enabled = true;
};

enum { MK_DECODE = 1, MK_PREFILL = 2, MK_GEMM = 3 };

static void ev_check(Engine &g, cudaError_t e, const char *what)
{
	if (e != cudaSuccess && !g.ev_fail) {
		g.ev_fail = what;
		set_err(TG_CUDA_ECUDA, "%s: %s", what, cudaGetErrorString(e));
	}
	if (e != cudaSuccess) cudaGetLastError(); // reported here; do not leave it for the next launch check
}

// Inside a capture a plain cudaEventRecord only orders work; the External flag makes it an
// event-record node that records (with a timestamp) at every replay.
static cudaError_t record(Engine &g, cudaEvent_t ev)
{
	return g.capturing ? cudaEventRecordWithFlags(ev, g.st, cudaEventRecordExternal) : cudaEventRecord(ev, g.st);
}

// A pair of events around one launch of class cls (only while profiling). Inside a graph
// capture the events become event-record nodes of the graph, read after each replay.
static int mark_begin(Engine &g, int cls, double work, double work_len = 0)
{
	g.launches++;
	if (!g.prof) return -1;
	std::vector<Engine::Mark> &v = g.capturing ? g.gmarks : g.marks;
	size_t &n = g.capturing ? g.ngmarks : g.nmarks;
	if (n == v.size()) {
		Engine::Mark m;
		ev_check(g, cudaEventCreate(&m.a), "cudaEventCreate");
		ev_check(g, cudaEventCreate(&m.b), "cudaEventCreate");
		v.push_back(m);
	}
	Engine::Mark &m = v[n];
	m.cls = cls;
	m.work = work;
	m.work_len = work_len;
	ev_check(g, record(g, m.a), "cudaEventRecord(mark begin)");
	return (int)n++;
}

static void mark_end(Engine &g, int i)
{
	if (i >= 0) ev_check(g, record(g, (g.capturing ? g.gmarks : g.marks)[i].b), "cudaEventRecord(mark end)");
}

// A launch on the engine's stream, with programmatic stream serialization while g.pdl.
template <class... KArgs, class... Args>
static cudaError_t launch_k(Engine &g, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args &&...args)
{
	if (g.pdl) return launch_pdl(kernel, grid, block, smem, g.st, std::forward<Args>(args)...);
	kernel<<<grid, block, smem, g.st>>>(std::forward<Args>(args)...);
	return cudaGetLastError();
}

// A layer's GEMM. Batches of 129-384 rows (a decode step of a 256-sequence wave) go to the
// swapped-operand cluster kernel (gemm_sk.cu); measured per decode step of the full model
// (28 layers), it takes 2.62 ms of GEMMs at 256 sequences against 2.88 ms for the tile
// kernels, but 3.97 / 2.22 ms against 3.84 / 2.10 ms at 512 / 128, so other batches, and the
// LM head's 151,936 columns, stay on the tile kernels. TG_CUDA_SMALL_GEMM=tile in the
// environment at load time keeps every GEMM on the tile kernels (for comparisons).
static int gemm_m(Engine &g, const GemmOperands &op, const GemmArgs &p0)
{
	GemmArgs p = p0;
	p.pdl = g.pdl ? 1 : 0;
	p.wide = g.wide_tiles ? 1 : 0;
	p.partial = g.part.as<float>(); // split-K scratch for the tile kernel's small batches
	p.partial_floats = (long)(g.part.bytes / sizeof(float));
	// the weight operand's bytes: codes (+ per-head scales) or bf16 tiles, + the epilogue's scales
	const double wbytes = (p.cside == 2 ? (double)p.N * p.cld + (p.cscale ? 4.0 * p.N * (p.K / p.cgroup) : 0.0)
					    : 2.0 * p.nb * p.N * p.K) + (p.scale ? 4.0 * p.N : 0.0);
	int mk = mark_begin(g, MK_GEMM, 2.0 * p.M * p.N * p.K, wbytes);
	int rc = g.small_gemm && p.M > 128 && p.M <= 384 && p.N <= 16384 && gemm_sk_fits(p) ? gemm_sk(op, p, g.st) : gemm(op, p, g.st);
	mark_end(g, mk);
	return rc;
}

// The times of n marks into t. keys > 0: the marks of one replay of the decode-step graph, whose
// attention reads keys positions per sequence; keys == 0: marks of directly launched kernels.
static void add_marks(Engine &g, tg_cuda_lm_stats &t, const std::vector<Engine::Mark> &v, size_t n, double keys)
{
	for (size_t i = 0; i < n; i++) {
		float e = 0;
		ev_check(g, cudaEventElapsedTime(&e, v[i].a, v[i].b), "cudaEventElapsedTime(mark)");
		switch (v[i].cls) {
		case MK_DECODE:
			t.attn_decode_ms += e, t.attn_decode_bytes += v[i].work + v[i].work_len * keys, t.attn_decode_launches++;
			break;
		case MK_PREFILL: t.attn_prefill_ms += e, t.attn_prefill_flops += v[i].work; break;
		case MK_GEMM:
			t.gemm_ms += e, t.gemm_flops += v[i].work, t.gemm_weight_bytes += v[i].work_len, t.gemm_launches++;
			if (keys > 0) t.decode_gemm_ms += e, t.decode_gemm_weight_bytes += v[i].work_len; // a decode step's
			break;
		}
	}
}

static void call_begin(Engine &g)
{
	g.ev_fail = nullptr;
	if (!g.ev_start) {
		ev_check(g, cudaEventCreate(&g.ev_start), "cudaEventCreate(start)");
		ev_check(g, cudaEventCreate(&g.ev_end), "cudaEventCreate(end)");
	}
	g.launches = 0;
	g.nmarks = 0;
	memset(&g.acc, 0, sizeof g.acc);
	ev_check(g, cudaEventRecord(g.ev_start, g.st), "cudaEventRecord(start)");
}

// After the stream is synchronized: the call's statistics.
static void call_end(Engine &g)
{
	tg_cuda_lm_stats &t = g.acc;
	float ms = 0;
	ev_check(g, cudaEventElapsedTime(&ms, g.ev_start, g.ev_end), "cudaEventElapsedTime(call)");
	t.device_ms = ms;
	t.launches = g.launches;
	add_marks(g, t, g.marks, g.nmarks, 0);
	g.last = t;
}

static size_t decode_smem(const Engine &g)
{
	const int grp = g.NQ / g.NKV;
	return (size_t)(grp * ((g.max_len + 3) & ~3) + 8 * grp * g.HD) * 4;
}

// Host -> device copy ordered on the engine's stream and complete on return. (A plain
// cudaMemcpy from pageable memory may return before its DMA lands, and kernels on a
// non-blocking stream are not ordered after it.)
static int upload(DevBuf &b, const void *src, size_t bytes, int dev, cudaStream_t st)
{
	int rc = b.alloc(bytes, dev);
	if (rc) return rc;
	TGC_CUDA(cudaMemcpyAsync(b.p, src, bytes, cudaMemcpyHostToDevice, st));
	TGC_CUDA(cudaStreamSynchronize(st));
	return TG_CUDA_OK;
}

static size_t qbytes(long n, int bits) { return bits == 8 ? (size_t)n : (size_t)(n + 1) / 2; }

static int load_engine(Engine &g, const tg_cuda_lm_desc *d, int dev, int max_seqs, int max_len)
{
	int rc;
	g.dev = dev;
	TGC_CUDA(cudaSetDevice(dev));
	TGC_CUDA(cudaStreamCreateWithFlags(&g.st, cudaStreamNonBlocking));
	g.L = d->layers, g.D = d->hidden, g.NQ = d->nq, g.NKV = d->nkv, g.HD = d->head_dim, g.FF = d->ffn, g.V = d->vocab;
	g.bits = d->bits, g.eps = d->eps, g.scale = d->attn_scale, g.max_seqs = max_seqs, g.max_len = max_len;
	const int D = g.D, HD = g.HD, NQ = g.NQ, NKV = g.NKV, FF = g.FF, V = g.V, bits = g.bits;
	if ((rc = upload(g.E, d->embed, (size_t)V * D * 4, dev, g.st)) || (rc = upload(g.lnf, d->final_norm, (size_t)D * 4, dev, g.st)))
		return rc;
	// RoPE tables in double, stored f32 (import.py:76-78): [pos][HD/2]
	{
		std::vector<float> c((size_t)max_len * HD / 2), s((size_t)max_len * HD / 2);
		for (int t = 0; t < max_len; t++)
			for (int i = 0; i < HD / 2; i++) {
				double inv = pow(d->rope_theta, -((double)(2 * i) / HD)), ang = (double)t * inv;
				c[(size_t)t * HD / 2 + i] = (float)cos(ang);
				s[(size_t)t * HD / 2 + i] = (float)sin(ang);
			}
		if ((rc = upload(g.cosT, c.data(), c.size() * 4, dev, g.st)) || (rc = upload(g.sinT, s.data(), s.size() * 4, dev, g.st))) return rc;
	}
	{
		const char *e = getenv("TG_CUDA_GEMV_ROWS");
		if (e) g.gemv_rows = std::min(atol(e), 8L);
		e = getenv("TG_CUDA_CODES_ROWS");
		if (e) g.codes_rows = std::min(atol(e), 128L);
		// whole K blocks of 64 (the GEMM's dequant) and per-head scale groups of them
		g.codes = (g.gemv_rows > 0 || g.codes_rows > 0) && (bits == 4 || bits == 8) && D % 64 == 0 &&
			  ((long)NQ * HD) % 64 == 0 && FF % 64 == 0 && HD % 64 == 0;
	}
	const long cpb = bits == 8 ? 1 : 2; // codes per byte
	DevBuf tmpq, tmpq2;
	// the uploaded codes [K, N] (in src) -> packed K-major rows of cdst (when codes are kept)
	auto pack_T = [&](const DevBuf &src, long K, long N, long blk, long off, long row0, DevBuf &cdst) -> int {
		if (!g.codes) return TG_CUDA_OK;
		const long n = N * (K / cpb);
		k_codes_T<<<(unsigned)((n + 255) / 256), 256, 0, g.st>>>(src.as<signed char>(), bits, K, N, blk, off, row0,
									  cdst.as<uint8_t>(), K / cpb);
		TGC_LAUNCH_CHECK();
		return TG_CUDA_OK;
	};
	auto codes_T = [&](const tg_cuda_qmat &m, long rows, long cols, __nv_bfloat16 *dst, long ldd, DevBuf *cdst = nullptr,
			   long row0 = 0) -> int {
		// [rows=in, cols=out] codes -> dst[out][in] (and the packed codes into cdst rows row0..)
		int r;
		if ((r = upload(tmpq, m.q, qbytes(rows * cols, bits), dev, g.st))) return r;
		if ((r = codes_to_bf16(tmpq.as<signed char>(), bits, rows, cols, true, dst, ldd, g.st))) return r;
		if (cdst && (r = pack_T(tmpq, rows, cols, cols, 0, row0, *cdst))) return r;
		TGC_CUDA(cudaStreamSynchronize(g.st));
		return TG_CUDA_OK;
	};
	auto calloc_ = [&](DevBuf &b, long rows, long K) -> int { return g.codes ? b.alloc((size_t)rows * (K / cpb), dev) : TG_CUDA_OK; };
	// LM head [D, V] -> [V][D]
	if ((rc = g.lmw.alloc((size_t)V * D * 2, dev)) || (rc = calloc_(g.clm, V, D)) ||
	    (rc = codes_T(d->lm_head, D, V, g.lmw.as<__nv_bfloat16>(), D, &g.clm)) ||
	    (rc = upload(g.lms, d->lm_head.s, (size_t)V * 4, dev, g.st)))
		return rc;
	for (int l = 0; l < g.L; l++) {
		g.layers.emplace_back(new Layer);
		Layer &Y = *g.layers.back();
		const int HQKV = g.HQKV();
		if ((rc = Y.wqkv.alloc((size_t)HQKV * D * 2, dev)) || (rc = calloc_(Y.cqkv, HQKV, D))) return rc;
		__nv_bfloat16 *w = Y.wqkv.as<__nv_bfloat16>();
		if ((rc = codes_T(d->wq[l], D, NQ * HD, w, D, &Y.cqkv, 0)) ||
		    (rc = codes_T(d->wk[l], D, NKV * HD, w + (size_t)NQ * HD * D, D, &Y.cqkv, (long)NQ * HD)) ||
		    (rc = codes_T(d->wv[l], D, NKV * HD, w + (size_t)(NQ + NKV) * HD * D, D, &Y.cqkv, (long)(NQ + NKV) * HD)))
			return rc;
		{
			std::vector<float> s(HQKV);
			memcpy(s.data(), d->wq[l].s, (size_t)NQ * HD * 4);
			memcpy(s.data() + NQ * HD, d->wk[l].s, (size_t)NKV * HD * 4);
			memcpy(s.data() + (NQ + NKV) * HD, d->wv[l].s, (size_t)NKV * HD * 4);
			if ((rc = upload(Y.sqkv, s.data(), s.size() * 4, dev, g.st))) return rc;
		}
		// o_proj: pre-scaled hi/lo [D][NQ*HD]
		const long KO = (long)NQ * HD;
		if ((rc = Y.wo_hi.alloc((size_t)D * KO * 2, dev)) || (rc = Y.wo_lo.alloc((size_t)D * KO * 2, dev)) ||
		    (rc = calloc_(Y.co, D, KO)) || (rc = upload(tmpq, d->wo[l].q, qbytes(KO * D, bits), dev, g.st)) ||
		    (rc = upload(Y.so, d->wo[l].s, (size_t)NQ * D * 4, dev, g.st)))
			return rc;
		k_wo_prescale<<<(unsigned)((KO * D + 255) / 256), 256, 0, g.st>>>(tmpq.as<signed char>(), Y.so.as<float>(), bits, (int)KO,
										      HD, D, Y.wo_hi.as<__nv_bfloat16>(), Y.wo_lo.as<__nv_bfloat16>());
		TGC_LAUNCH_CHECK();
		if ((rc = pack_T(tmpq, KO, D, D, 0, 0, Y.co))) return rc;
		TGC_CUDA(cudaStreamSynchronize(g.st));
		// gate/up interleaved [2FF][D]
		if ((rc = Y.wgu.alloc((size_t)2 * FF * D * 2, dev)) || (rc = upload(tmpq, d->wg[l].q, qbytes((long)D * FF, bits), dev, g.st)) ||
		    (rc = upload(tmpq2, d->wu[l].q, qbytes((long)D * FF, bits), dev, g.st)))
			return rc;
		k_codes_gu<<<(unsigned)((2L * D * FF + 255) / 256), 256, 0, g.st>>>(tmpq.as<signed char>(), tmpq2.as<signed char>(), bits, D,
										      FF, Y.wgu.as<__nv_bfloat16>());
		TGC_LAUNCH_CHECK();
		if ((rc = calloc_(Y.cgu, 2L * FF, D)) || (rc = pack_T(tmpq, D, FF, 32, 0, 0, Y.cgu)) || (rc = pack_T(tmpq2, D, FF, 32, 32, 0, Y.cgu)))
			return rc;
		TGC_CUDA(cudaStreamSynchronize(g.st));
		if ((rc = upload(Y.sg, d->wg[l].s, (size_t)FF * 4, dev, g.st)) || (rc = upload(Y.su, d->wu[l].s, (size_t)FF * 4, dev, g.st))) return rc;
		// down [FF, D] -> [D][FF]
		if ((rc = Y.wd.alloc((size_t)D * FF * 2, dev)) || (rc = calloc_(Y.cd, D, FF)) ||
		    (rc = codes_T(d->wd[l], FF, D, Y.wd.as<__nv_bfloat16>(), FF, &Y.cd)) ||
		    (rc = upload(Y.sd, d->wd[l].s, (size_t)D * 4, dev, g.st)))
			return rc;
		if ((rc = upload(Y.ln1, d->ln1[l], (size_t)D * 4, dev, g.st)) || (rc = upload(Y.ln2, d->ln2[l], (size_t)D * 4, dev, g.st)) ||
		    (rc = upload(Y.qn, d->qn[l], (size_t)HD * 4, dev, g.st)) || (rc = upload(Y.kn, d->kn[l], (size_t)HD * 4, dev, g.st)))
			return rc;
	}
	const size_t kv = (size_t)g.L * max_seqs * NKV * (size_t)max_len * HD; // elements per plane
	if ((rc = g.kh.alloc(kv * 2, dev)) || (rc = g.kq.alloc(kv, dev)) || (rc = g.vh.alloc(kv * 2, dev)) ||
	    (rc = g.vq.alloc(kv, dev)))
		return rc;
	long R = std::max<long>(PREFILL_ROWS, max_seqs);
	g.rows_cap = R;
	if ((rc = g.h.alloc((size_t)R * D * 4, dev)) || (rc = g.xhi.alloc((size_t)R * D * 2, dev)) ||
	    (rc = g.xlo.alloc((size_t)R * D * 2, dev)) || (rc = g.qkv.alloc((size_t)R * g.HQKV() * 4, dev)) ||
	    (rc = g.q.alloc((size_t)R * NQ * HD * 4, dev)) || (rc = g.ahi.alloc((size_t)R * NQ * HD * 2, dev)) ||
	    (rc = g.alo.alloc((size_t)R * NQ * HD * 2, dev)) || (rc = g.ghi.alloc((size_t)R * FF * 2, dev)) ||
	    (rc = g.glo.alloc((size_t)R * FF * 2, dev)) || (rc = g.logits.alloc((size_t)max_seqs * V * 4, dev)) ||
	    (rc = g.tok.alloc((size_t)max_seqs * 4, dev)) || (rc = g.ids.alloc((size_t)R * 4, dev)) ||
	    (rc = g.status.alloc(64, dev)))
		return rc;
	if ((rc = g.dpos.alloc(16, dev))) return rc;
	if (g.codes && g.gemv_rows > 0 && (rc = g.gus.alloc((size_t)g.gemv_rows * 2 * FF * 4, dev))) return rc;
	cudaDeviceGetAttribute(&g.sms, cudaDevAttrMultiProcessorCount, dev);
	{ // waves whose (kv head, sequence) grid fills at most half the SMs split the decode attention
		const char *e = getenv("TG_CUDA_DECODE_SPLIT");
		g.split_seqs = e && strcmp(e, "0") == 0 ? 0 : std::min<long>(max_seqs, g.sms / (2L * NKV));
		if (g.split_seqs > 0 && HD == 128 &&
		    (rc = g.apart.alloc((size_t)g.split_seqs * NQ * 8 * (HD + 2) * sizeof(float), dev)))
			return rc;
		if (HD != 128) g.split_seqs = 0;
	}
	{ // split-K partial sums of the decode GEMMs: up to 16 splits of a 128-row-padded batch
		long mpad = ((long)max_seqs + 127) / 128 * 128, nmax = std::max<long>(g.HQKV(), std::max<long>(2L * FF, D));
		if ((rc = g.part.alloc((size_t)16 * mpad * nmax * sizeof(float), dev))) return rc;
	}
	// kernel attributes are set here, never inside a graph capture
	if (decode_smem(g) > 220 * 1024) return set_err(TG_CUDA_EINVAL, "max_len %d: decode scores exceed shared memory", max_len);
	{
		const char *e = getenv("TG_CUDA_SMALL_GEMM");
		g.small_gemm = !(e && strcmp(e, "tile") == 0);
	}
	{
		const char *e = getenv("TG_CUDA_PREFILL");
		g.prefill_tma = !(e && strcmp(e, "staged") == 0);
		e = getenv("TG_CUDA_PDL");
		g.pdl_enabled = !(e && strcmp(e, "0") == 0);
		e = getenv("TG_CUDA_WIDE_TILES");
		g.wide_tiles = !(e && strcmp(e, "0") == 0);
	}
	for (int l = 0; l < g.L; l++) { // TMA maps of the cache planes, boxes of 64 dims x 64 positions
		const size_t lo = (size_t)l * max_seqs * NKV * (size_t)max_len * HD;
		const long rows = (long)max_seqs * NKV * max_len;
		if ((rc = bf16_tile_map(&g.layers[l]->kmap, g.kh.as<__nv_bfloat16>() + lo, rows, HD, HD, FA_K)) ||
		    (rc = bf16_tile_map(&g.layers[l]->vmap, g.vh.as<__nv_bfloat16>() + lo, rows, HD, HD, FA_K)))
			return rc;
	}
	if ((rc = gemm_sk_prepare()) || (rc = gemv_dec_prepare())) return rc;
	TGC_CUDA(cudaFuncSetAttribute(k_attn_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FA_SMEM));
	TGC_CUDA(cudaFuncSetAttribute(k_attn_prefill_tma, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FB_SMEM));
	TGC_CUDA(cudaFuncSetAttribute(k_attn_decode<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)decode_smem(g)));
	TGC_CUDA(cudaFuncSetAttribute(k_attn_decode<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)decode_smem(g)));
	TGC_CUDA(cudaMemsetAsync(g.status.p, 0, 64, g.st));
	TGC_CUDA(cudaStreamSynchronize(g.st));
	return TG_CUDA_OK;
}

// B[0] (the weights, [N][K]) from packed codes expanded in the kernel instead of the bf16 copy
static void codes_b(const Engine &g, GemmArgs &p, const DevBuf &c)
{
	p.codes = c.as<signed char>(), p.cbits = g.bits, p.cside = 2, p.cld = (long)p.K * g.bits / 8;
}

// A product of a batch of at most 8 rows: out[j][n] (+)= s * sum_k (hi + lo)[j][k] code(n, k)
// as a dequant GEMV over the packed codes [N][K] (group > 0: per-(K group, n) scales).
// With x set, the activations are rmsnorm(x) * nw, computed in the GEMV (hi / lo unused).
static int gemv_m(Engine &g, const DevBuf &codes, const void *hi, const void *lo, long lda, long M, int N, int K, const float *s,
		  int group, long s_ld, float *out, long ldo, int epi, const float *x = nullptr, const float *nw = nullptr)
{
	GemvDecArgs a;
	memset(&a, 0, sizeof a);
	a.hi = (const __nv_bfloat16 *)hi, a.lo = (const __nv_bfloat16 *)lo, a.lda = lda, a.nb = (int)M;
	a.x = x, a.nw = nw, a.eps = g.eps;
	a.q = codes.as<signed char>(), a.m = N, a.k = K, a.bits = g.bits;
	a.s = s, a.group = group, a.s_ld = s_ld, a.out = out, a.ldo = ldo, a.epi = epi;
	const double wbytes = (double)N * K * g.bits / 8 + (s ? 4.0 * N * (group ? K / group : 1) : 0.0);
	int mk = mark_begin(g, MK_GEMM, 2.0 * M * N * K, wbytes);
	int rc = gemv_dec(a, g.st, g.pdl);
	mark_end(g, mk);
	return rc;
}

static GemmArgs gemm_args(int M, int N, int K, int epi)
{
	GemmArgs p;
	memset(&p, 0, sizeof p);
	p.M = M, p.N = N, p.K = K, p.epi = epi;
	p.na = 2, p.nb = 1, p.npairs = 2;
	p.pa[0] = 0, p.pb[0] = 0, p.pa[1] = 1, p.pb[1] = 0;
	return p;
}

// One pass of every layer over M rows: T tokens per sequence of the chunk (decode: T = 1 at
// position pos0), sequences in KV slots slot0.., attention over len positions (decode).
static int run_layers(Engine &g, long M, int T, int pos0, int slot0, bool decode)
{
	int rc;
	const int D = g.D, HD = g.HD, NQ = g.NQ, NKV = g.NKV, FF = g.FF;
	const long S = M / T;
	int *status = g.status.as<int>();
	const unsigned warps_grid = (unsigned)((M * 32 + 255) / 256);
	// the weights' form: GEMVs over codes (batches of up to 8 rows), the GEMM with the codes
	// expanded in the kernel, or the GEMM on the bf16 copies
	const bool gv = g.use_gemv(M), cw = !gv && g.use_codes(M);
	const long KO = (long)NQ * HD;
	for (int l = 0; l < g.L; l++) {
		Layer &Y = *g.layers[l];
		const size_t lo = (size_t)l * g.max_seqs * NKV * (size_t)g.max_len * HD; // this layer's first element
		const KvPlane kc{ g.kh.as<__nv_bfloat16>() + lo, g.kq.as<signed char>() + lo };
		const KvPlane vc{ g.vh.as<__nv_bfloat16>() + lo, g.vq.as<signed char>() + lo };
		const KvPlaneC kcc{ kc.h, kc.q }, vcc{ vc.h, vc.q };
		g.launches += gv ? 1 : 3; // the q/k rope and (but for the GEMVs, which norm themselves) two norms
		if (!gv)
			TGC_CUDA(launch_k(g, k_rmsnorm_split, dim3(warps_grid), dim3(256), 0, (const float *)g.h.as<float>(), M, D,
					  (const float *)Y.ln1.as<float>(), g.eps, 0, g.xhi.as<__nv_bfloat16>(), g.xlo.as<__nv_bfloat16>()));
		GemmOperands op;
		GemmArgs p;
		if (gv) { // rmsnorm(h) * ln1 in the GEMV
			if ((rc = gemv_m(g, Y.cqkv, nullptr, nullptr, D, M, g.HQKV(), D, Y.sqkv.as<float>(), 0, 0, g.qkv.as<float>(), g.HQKV(),
					 GD_STORE, g.h.as<float>(), Y.ln1.as<float>())))
				return rc;
		} else {
			op.a[0] = g.xhi.p, op.a[1] = g.xlo.p, op.b[0] = Y.wqkv.p, op.lda = D, op.ldb = D;
			p = gemm_args((int)M, g.HQKV(), D, EPI_STORE);
			p.scale = Y.sqkv.as<float>(), p.scale_mode = 2, p.out = g.qkv.as<float>(), p.ldo = g.HQKV(), p.status = status;
			if (cw) codes_b(g, p, Y.cqkv);
			if ((rc = gemm_m(g, op, p))) return rc;
		}
		long heads = M * (NQ + 2 * NKV);
		TGC_CUDA(launch_k(g, k_qk_rope, dim3((unsigned)((heads * 32 + 255) / 256)), dim3(256), 0, (const float *)g.qkv.as<float>(),
				  M, T, pos0, (const int *)(decode ? g.dpos.as<int>() : nullptr), NQ, NKV, g.eps,
				  (const float *)Y.qn.as<float>(), (const float *)Y.kn.as<float>(), (const float *)g.cosT.as<float>(),
				  (const float *)g.sinT.as<float>(), g.q.as<float>(), kc, vc, slot0, g.max_len));
		if (!decode) {
			dim3 grid((T + FA_Q - 1) / FA_Q, NQ, (unsigned)S);
			int mk = mark_begin(g, MK_PREFILL, 4.0 * HD * (double)T * (T + 1) / 2 * NQ * S);
			if (g.prefill_tma)
				k_attn_prefill_tma<<<grid, FB_THREADS, FB_SMEM, g.st>>>(g.q.as<float>(), Y.kmap, Y.vmap, kcc.q, vcc.q, T, NQ,
											NKV, slot0, g.max_len, g.scale,
											g.ahi.as<__nv_bfloat16>(), g.alo.as<__nv_bfloat16>(),
											status);
			else
				k_attn_prefill_tc<<<grid, FA_THREADS, FA_SMEM, g.st>>>(g.q.as<float>(), kcc, vcc, T, NQ, NKV, slot0,
										       g.max_len, g.scale, g.ahi.as<__nv_bfloat16>(),
										       g.alo.as<__nv_bfloat16>(), status);
			mark_end(g, mk);
		} else {
			// the key count (position + 1) is read on the device; bytes = per-key part * len + the rest
			size_t smem = decode_smem(g);
			dim3 grid(NKV, (unsigned)S);
			// per key: K and V rows of 3-byte elements
			int mk = mark_begin(g, MK_DECODE, (double)S * NQ * HD * 4 * 2, (double)S * NKV * HD * 3 * 2);
			// a small wave: key ranges over more CTAs (2 per SM at most), at least 64 keys each
			const int nsp = S <= g.split_seqs
						? (int)std::max<long>(1, std::min<long>({ 8L, 2L * g.sms / (NKV * S), (long)g.max_len / 64 }))
						: 1;
			grid.z = nsp;
			float *part = nsp > 1 ? g.apart.as<float>() : nullptr;
			if (NQ / NKV == 2)
				TGC_CUDA(launch_k(g, k_attn_decode<2>, grid, dim3(256), smem, (const float *)g.q.as<float>(), kcc, vcc, 0,
						  (const int *)g.dpos.as<int>(), NQ, NKV, slot0, g.max_len, g.scale,
						  g.ahi.as<__nv_bfloat16>(), g.alo.as<__nv_bfloat16>(), part));
			else
				TGC_CUDA(launch_k(g, k_attn_decode<1>, grid, dim3(256), smem, (const float *)g.q.as<float>(), kcc, vcc, 0,
						  (const int *)g.dpos.as<int>(), NQ, NKV, slot0, g.max_len, g.scale,
						  g.ahi.as<__nv_bfloat16>(), g.alo.as<__nv_bfloat16>(), part));
			if (nsp > 1) {
				g.launches++;
				TGC_CUDA(launch_k(g, k_attn_combine, dim3(NQ, (unsigned)S), dim3(128), 0, (const float *)part, nsp, NQ,
						  g.ahi.as<__nv_bfloat16>(), g.alo.as<__nv_bfloat16>()));
			}
			mark_end(g, mk);
		}
		TGC_LAUNCH_CHECK();
		// o_proj with the residual: h += attn @ Wo (hi*hi + hi*lo + lo*hi; the GEMV: per-head scales)
		if (gv) {
			if ((rc = gemv_m(g, Y.co, g.ahi.p, g.alo.p, KO, M, D, (int)KO, Y.so.as<float>(), HD, D, g.h.as<float>(), D, GD_ADD)))
				return rc;
		} else {
			op = GemmOperands();
			op.a[0] = g.ahi.p, op.a[1] = g.alo.p, op.b[0] = Y.wo_hi.p, op.b[1] = Y.wo_lo.p, op.lda = KO, op.ldb = KO;
			p = gemm_args((int)M, D, (int)KO, EPI_ADD);
			p.nb = 2, p.npairs = 3;
			p.pa[0] = 0, p.pb[0] = 0, p.pa[1] = 0, p.pb[1] = 1, p.pa[2] = 1, p.pb[2] = 0;
			p.out = g.h.as<float>(), p.ldo = D, p.status = status;
			if (cw) { // hi and lo of code * per-head scale, built in the kernel
				codes_b(g, p, Y.co);
				p.cscale = Y.so.as<float>(), p.cgroup = HD, p.cscale_ld = D;
			}
			if ((rc = gemm_m(g, op, p))) return rc;
		}
		if (!gv)
			TGC_CUDA(launch_k(g, k_rmsnorm_split, dim3(warps_grid), dim3(256), 0, (const float *)g.h.as<float>(), M, D,
					  (const float *)Y.ln2.as<float>(), g.eps, 0, g.xhi.as<__nv_bfloat16>(), g.xlo.as<__nv_bfloat16>()));
		if (gv) { // gate/up sums of rmsnorm(h) * ln2, then SwiGLU with the channel scales
			if ((rc = gemv_m(g, Y.cgu, nullptr, nullptr, D, M, 2 * FF, D, nullptr, 0, 0, g.gus.as<float>(), 2L * FF, GD_STORE,
					 g.h.as<float>(), Y.ln2.as<float>())))
				return rc;
			g.launches++;
			TGC_CUDA(launch_k(g, k_swiglu_split, dim3((unsigned)((M * FF + 255) / 256)), dim3(256), 0, (const float *)g.gus.as<float>(),
					  M, FF, (const float *)Y.sg.as<float>(), (const float *)Y.su.as<float>(), g.ghi.as<__nv_bfloat16>(),
					  g.glo.as<__nv_bfloat16>()));
			if ((rc = gemv_m(g, Y.cd, g.ghi.p, g.glo.p, FF, M, D, FF, Y.sd.as<float>(), 0, 0, g.h.as<float>(), D, GD_ADD))) return rc;
			continue;
		}
		op = GemmOperands();
		op.a[0] = g.xhi.p, op.a[1] = g.xlo.p, op.b[0] = Y.wgu.p, op.lda = D, op.ldb = D;
		p = gemm_args((int)M, 2 * FF, D, EPI_SWIGLU);
		p.scale = Y.sg.as<float>(), p.scale2 = Y.su.as<float>(), p.out_hi = g.ghi.as<__nv_bfloat16>(),
		p.out_lo = g.glo.as<__nv_bfloat16>(), p.ldo = FF, p.status = status;
		if (cw) codes_b(g, p, Y.cgu);
		if ((rc = gemm_m(g, op, p))) return rc;
		op = GemmOperands();
		op.a[0] = g.ghi.p, op.a[1] = g.glo.p, op.b[0] = Y.wd.p, op.lda = FF, op.ldb = FF;
		p = gemm_args((int)M, D, FF, EPI_ADD);
		p.scale = Y.sd.as<float>(), p.scale_mode = 2, p.out = g.h.as<float>(), p.ldo = D, p.status = status;
		if (cw) codes_b(g, p, Y.cd);
		if ((rc = gemm_m(g, op, p))) return rc;
	}
	return TG_CUDA_OK;
}

// Final norm of the last position of each of S sequences (T tokens each), LM head -> logits.
static int head(Engine &g, long S, int T)
{
	int rc;
	g.launches++;
	TGC_CUDA(launch_k(g, k_rmsnorm_split, dim3((unsigned)((S * 32 + 255) / 256)), dim3(256), 0, (const float *)g.h.as<float>(), S,
			  g.D, (const float *)g.lnf.as<float>(), g.eps, T, g.xhi.as<__nv_bfloat16>(), g.xlo.as<__nv_bfloat16>()));
	TGC_LAUNCH_CHECK();
	// the head stays on the tensor cores even for a handful of sequences: a GEMV over its
	// 151,936 rows measured 230 us a step at 8 sequences (FMA and shared-memory bound), the
	// GEMM tens of microseconds
	GemmOperands op;
	op.a[0] = g.xhi.p, op.a[1] = g.xlo.p, op.b[0] = g.lmw.p, op.lda = g.D, op.ldb = g.D;
	GemmArgs p = gemm_args((int)S, g.V, g.D, EPI_STORE);
	p.scale = g.lms.as<float>(), p.scale_mode = 2, p.out = g.logits.as<float>(), p.ldo = g.V, p.status = g.status.as<int>();
	if (g.use_codes(S)) codes_b(g, p, g.clm);
	if ((rc = gemm_m(g, op, p))) return rc;
	return TG_CUDA_OK;
}

// Prefill S sequences (ids on the host, T each) into KV slots slot0..; logits of the last positions.
static int prefill(Engine &g, const float *ids_host, long S, int T, int slot0, float *logits_host, int *tokens_host,
		   int ld_tok)
{
	int rc;
	const long chunk = std::max<long>(1, std::min<long>(S, g.rows_cap / T));
	for (long s0 = 0; s0 < S; s0 += chunk) {
		long n = std::min(chunk, S - s0), M = n * T;
		if (fault("h2d")) return set_err(TG_CUDA_EFAULT, "injected copy failure (TG_CUDA_FAULT=h2d)");
		TGC_CUDA(cudaMemcpyAsync(g.ids.p, ids_host + s0 * T, (size_t)M * 4, cudaMemcpyHostToDevice, g.st));
		g.launches++;
		k_embed<<<(unsigned)((M * 32 + 255) / 256), 256, 0, g.st>>>(g.ids.as<float>(), nullptr, M, g.E.as<float>(), g.V, g.D,
									     g.h.as<float>());
		TGC_LAUNCH_CHECK();
		if ((rc = run_layers(g, M, T, 0, slot0 + (int)s0, false))) return rc;
		if ((rc = head(g, n, T))) return rc;
		if (logits_host)
			TGC_CUDA(cudaMemcpyAsync(logits_host + s0 * g.V, g.logits.p, (size_t)n * g.V * 4, cudaMemcpyDeviceToHost, g.st));
		if (tokens_host) {
			g.launches++;
			k_argmax<<<(unsigned)n, 1024, 0, g.st>>>(g.logits.as<float>(), g.V, g.tok.as<int>() + s0, nullptr, 0, 0, nullptr,
								 0);
			TGC_LAUNCH_CHECK();
		}
	}
	(void)tokens_host;
	(void)ld_tok;
	return TG_CUDA_OK;
}

// One decode step for S sequences whose fed token sits at position *dpos: embed the last
// tokens, every layer against the KV cache, the LM head, argmax into column *dpos - T + 1
// of out_tok, then *dpos += 1. Launch arguments do not depend on the step.
__global__ void k_bump(int *pos)
{
	pdl_wait();
	pdl_launch();
	pos[0] += 1;
}

static int decode_step(Engine &g, long S, int T, int nnew)
{
	int rc;
	g.launches++;
	TGC_CUDA(launch_k(g, k_embed, dim3((unsigned)((S * 32 + 255) / 256)), dim3(256), 0, (const float *)nullptr,
			  (const int *)g.tok.as<int>(), S, (const float *)g.E.as<float>(), g.V, g.D, g.h.as<float>()));
	if ((rc = run_layers(g, S, 1, 0, 0, true))) return rc;
	if ((rc = head(g, S, 1))) return rc;
	g.launches += 2;
	TGC_CUDA(launch_k(g, k_argmax, dim3((unsigned)S), dim3(1024), 0, (const float *)g.logits.as<float>(), g.V, g.tok.as<int>(),
			  g.out_tok.as<int>(), nnew, 0, (const int *)g.dpos.as<int>(), T));
	TGC_CUDA(launch_k(g, k_bump, dim3(1), dim3(1), 0, g.dpos.as<int>()));
	TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

// The decode step captured as a CUDA graph (re-captured when S, T, nnew or profiling change):
// about 9 launches per layer replay without host work per step.
static int decode_graph(Engine &g, long S, int T, int nnew)
{
	if (g.gexec && g.g_S == S && g.g_T == T && g.g_nnew == nnew && g.g_prof == g.prof) return TG_CUDA_OK;
	if (g.gexec) {
		cudaGraphExecDestroy(g.gexec);
		g.gexec = nullptr;
	}
	g.ngmarks = 0;
	const long before = g.launches;
	cudaGraph_t graph = nullptr;
	TGC_CUDA(cudaStreamBeginCapture(g.st, cudaStreamCaptureModeThreadLocal));
	g.capturing = true;
	g.pdl = g.pdl_enabled && !g.prof; // profiling marks between kernels would break the overlap anyway
	int rc = decode_step(g, S, T, nnew);
	g.pdl = false;
	g.capturing = false;
	cudaError_t e = cudaStreamEndCapture(g.st, &graph);
	g.g_kernels = g.launches - before;
	g.launches = before;
	if (rc) {
		if (graph) cudaGraphDestroy(graph);
		return rc;
	}
	if (e != cudaSuccess) return set_err(TG_CUDA_ECUDA, "decode graph capture: %s", cudaGetErrorString(e));
	e = cudaGraphInstantiate(&g.gexec, graph, 0);
	cudaGraphDestroy(graph);
	if (e != cudaSuccess) return set_err(TG_CUDA_ECUDA, "decode graph instantiate: %s", cudaGetErrorString(e));
	g.g_S = S, g.g_T = T, g.g_nnew = nnew, g.g_prof = g.prof;
	return TG_CUDA_OK;
}

static int generate_wave(Engine &g, const float *ids_host, long S, int T, int nnew, int *tokens_host)
{
	int rc;
	if ((rc = prefill(g, ids_host, S, T, 0, nullptr, tokens_host, nnew))) return rc;
	if ((rc = g.out_tok.ensure((size_t)S * nnew * 4, g.dev))) return rc;
	// tokens[:, 0] = the prefill's argmax
	TGC_CUDA(cudaMemcpy2DAsync(g.out_tok.p, (size_t)nnew * 4, g.tok.p, 4, 4, (size_t)S, cudaMemcpyDeviceToDevice, g.st));
	if (nnew > 1) {
		// the first decode step feeds the token at position T; the graph bumps it each step
		g.pos_host = T;
		TGC_CUDA(cudaMemcpyAsync(g.dpos.p, &g.pos_host, sizeof(int), cudaMemcpyHostToDevice, g.st));
		if ((rc = decode_graph(g, S, T, nnew))) return rc;
		for (int step = 1; step < nnew; step++) {
			TGC_CUDA(cudaGraphLaunch(g.gexec, g.st));
			g.launches += g.g_kernels;
			if (g.prof) { // read this replay's event pairs before the next replay re-records them
				TGC_CUDA(cudaStreamSynchronize(g.st));
				add_marks(g, g.acc, g.gmarks, g.ngmarks, (double)(T + step));
			}
		}
	}
	if (fault("gather")) return set_err(TG_CUDA_EFAULT, "injected gather failure (TG_CUDA_FAULT=gather)");
	TGC_CUDA(cudaMemcpyAsync(tokens_host, g.out_tok.p, (size_t)S * nnew * 4, cudaMemcpyDeviceToHost, g.st));
	return TG_CUDA_OK;
}

} // namespace tgc

using namespace tgc;

struct tg_cuda_lm {
	std::vector<std::unique_ptr<Engine>> eng;
};

static int check_desc(const tg_cuda_lm_desc *d)
{
	if (!d) return set_err(TG_CUDA_EINVAL, "NULL descriptor");
	if (d->head_dim != 128) return set_err(TG_CUDA_EUNSUPPORTED, "head_dim %d: the device kernels are built for 128", d->head_dim);
	if (d->nkv <= 0 || d->nq % d->nkv || (d->nq / d->nkv != 1 && d->nq / d->nkv != 2))
		return set_err(TG_CUDA_EUNSUPPORTED, "grouped-query ratio nq/nkv must be 1 or 2");
	if (d->bits != 8 && d->bits != 4) return set_err(TG_CUDA_EINVAL, "bits must be 8 or 4");
	if (d->hidden % 64 || d->ffn % 128 || d->hidden < 64)
		return set_err(TG_CUDA_EUNSUPPORTED, "hidden must be a multiple of 64 and ffn of 128");
	if (!d->embed || !d->final_norm || !d->lm_head.q || !d->ln1 || !d->wq || !d->wo || !d->wd)
		return set_err(TG_CUDA_EINVAL, "descriptor has NULL weights");
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_lm_load(const tg_cuda_lm_desc *d, int max_seqs, int max_len, tg_cuda_lm **out)
{
	clear_err();
	if (!out) return set_err(TG_CUDA_EINVAL, "tg_cuda_lm_load: NULL out");
	*out = nullptr;
	if (!inited()) return set_err(TG_CUDA_ENODEV, "tg_cuda_lm_load: call tg_cuda_init first");
	int rc = check_desc(d);
	if (rc) return rc;
	if (max_seqs <= 0 || max_len <= 0) return set_err(TG_CUDA_EINVAL, "max_seqs and max_len must be positive");
	tg_cuda_lm *g = new tg_cuda_lm;
	for (auto &dv : devices()) {
		g->eng.emplace_back(new Engine);
		if ((rc = load_engine(*g->eng.back(), d, dv.id, max_seqs, max_len))) {
			tg_cuda_lm_free(g);
			return rc;
		}
	}
	cudaSetDevice(devices()[0].id);
	*out = g;
	return TG_CUDA_OK;
}

// Shard nseq sequences over the engines (one host thread each), in waves of max_seqs.
template <class F>
static int shard(tg_cuda_lm *g, long nseq, F &&fn)
{
	size_t G = g->eng.size();
	std::vector<int> rcs(G, 0);
	std::vector<std::string> errs(G);
	auto work = [&](size_t di) {
		Engine &e = *g->eng[di];
		cudaSetDevice(e.dev);
		long lo = nseq * (long)di / (long)G, hi = nseq * (long)(di + 1) / (long)G;
		int rc = TG_CUDA_OK;
		call_begin(e);
		for (long w0 = lo; w0 < hi && !rc; w0 += e.max_seqs) rc = fn(e, w0, std::min<long>(e.max_seqs, hi - w0));
		ev_check(e, cudaEventRecord(e.ev_end, e.st), "cudaEventRecord(end)");
		if (!rc) {
			cudaError_t ce = cudaStreamSynchronize(e.st);
			if (ce != cudaSuccess) rc = set_err(TG_CUDA_ECUDA, "device %d: %s", e.dev, cudaGetErrorString(ce));
		}
		if (!rc) call_end(e);
		if (!rc && e.ev_fail) rc = TG_CUDA_ECUDA; // the text was set by ev_check
		if (!rc) {
			cudaError_t le = cudaGetLastError(); // nothing may be left pending from this call
			if (le != cudaSuccess) rc = set_err(TG_CUDA_ECUDA, "pending error after the call: %s", cudaGetErrorString(le));
		}
		if (!rc) rc = device_status_check(e.status.as<int>(), e.st);
		rcs[di] = rc;
		if (rc) errs[di] = tg_cuda_error();
	};
	if (G == 1) work(0);
	else {
		std::vector<std::thread> th;
		for (size_t di = 0; di < G; di++) th.emplace_back(work, di);
		for (auto &t : th) t.join();
	}
	cudaSetDevice(g->eng[0]->dev);
	for (size_t di = 0; di < G; di++)
		if (rcs[di]) return set_err(rcs[di], "%s", errs[di].c_str());
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_lm_forward(tg_cuda_lm *g, const float *ids, long nseq, int T, float *logits)
{
	clear_err();
	if (!g || !ids || !logits || nseq < 0 || T <= 0) return set_err(TG_CUDA_EINVAL, "tg_cuda_lm_forward: bad arguments");
	if (T > g->eng[0]->max_len) return set_err(TG_CUDA_EINVAL, "T %d exceeds max_len %d", T, g->eng[0]->max_len);
	const int V = g->eng[0]->V;
	return shard(g, nseq, [&](Engine &e, long w0, long n) {
		return prefill(e, ids + w0 * T, n, T, 0, logits + w0 * V, nullptr, 0);
	});
}

extern "C" int tg_cuda_lm_generate(tg_cuda_lm *g, const float *ids, long nseq, int T, int nnew, int *tokens)
{
	clear_err();
	if (!g || !ids || !tokens || nseq < 0 || T <= 0 || nnew <= 0) return set_err(TG_CUDA_EINVAL, "tg_cuda_lm_generate: bad arguments");
	if (T + nnew - 1 > g->eng[0]->max_len)
		return set_err(TG_CUDA_EINVAL, "T + nnew - 1 = %d exceeds max_len %d", T + nnew - 1, g->eng[0]->max_len);
	return shard(g, nseq, [&](Engine &e, long w0, long n) { return generate_wave(e, ids + w0 * T, n, T, nnew, tokens + w0 * nnew); });
}

extern "C" int tg_cuda_lm_profile(tg_cuda_lm *g, int enable)
{
	clear_err();
	if (!g) return set_err(TG_CUDA_EINVAL, "tg_cuda_lm_profile: NULL model");
	for (auto &e : g->eng) e->prof = enable != 0;
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_lm_get_stats(const tg_cuda_lm *g, tg_cuda_lm_stats *out)
{
	clear_err();
	if (!g || !out) return set_err(TG_CUDA_EINVAL, "tg_cuda_lm_get_stats: NULL argument");
	memset(out, 0, sizeof *out);
	for (auto &e : g->eng) {
		const tg_cuda_lm_stats &t = e->last;
		out->device_ms = std::max(out->device_ms, t.device_ms);
		out->launches += t.launches;
		out->attn_decode_ms += t.attn_decode_ms, out->attn_decode_bytes += t.attn_decode_bytes;
		out->attn_decode_launches += t.attn_decode_launches;
		out->attn_prefill_ms += t.attn_prefill_ms, out->attn_prefill_flops += t.attn_prefill_flops;
		out->gemm_ms += t.gemm_ms, out->gemm_flops += t.gemm_flops, out->gemm_launches += t.gemm_launches;
		out->gemm_weight_bytes += t.gemm_weight_bytes;
		out->decode_gemm_ms += t.decode_gemm_ms, out->decode_gemm_weight_bytes += t.decode_gemm_weight_bytes;
	}
	return TG_CUDA_OK;
}

extern "C" void tg_cuda_lm_free(tg_cuda_lm *g)
{
	if (!g) return;
	for (auto &e : g->eng) {
		cudaSetDevice(e->dev);
		if (e->st) {
			cudaStreamSynchronize(e->st);
			cudaStreamDestroy(e->st);
		}
		if (e->gexec) cudaGraphExecDestroy(e->gexec);
		for (auto &m : e->gmarks) {
			cudaEventDestroy(m.a);
			cudaEventDestroy(m.b);
		}
		for (auto &m : e->marks) {
			cudaEventDestroy(m.a);
			cudaEventDestroy(m.b);
		}
		if (e->ev_start) {
			cudaEventDestroy(e->ev_start);
			cudaEventDestroy(e->ev_end);
		}
	}
	delete g;
}
