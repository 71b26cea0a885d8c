// ssm.cu -- stacked selective-SSM blocks (the arithmetic of tg_cuda_ssm_desc in
// include/tg_cuda.h) for many sequences at once.
//
// The reference runs the program one sequence per row: the scan of src/vm.c:364-382
// executes the block body once per step. Here all sequences of a wave advance
// together, a chunk of steps at a time, so every per-step matmul of the body
// becomes one tensor-core GEMM over (sequences x chunk steps) token rows:
//
//   per block:  rmsnorm * w (bf16 hi/lo split)  -> GEMM [x | z] = n @ [Wx | Wz]
//               k_ssm_conv: causal width-4 conv over the chunk (carries across
//               chunks), silu, split -> GEMM [r | bt | ct] = xs @ [Wr | WB | WC]
//               k_ssm_scan: one thread per (sequence, channel) walks the chunk with
//               the state h[d_state] in registers: dt = softplus(r @ Wdt + dt_b)
//               (16 MACs on CUDA cores), the zero-order-hold update, y = h @ ct +
//               d * xs, g = y * silu(z) split -> GEMM u += g @ Wo (residual add)
//   at the end: rmsnorm * final_norm of every row into the output.
//
// Rows of a chunk are sequence-major: row = s * chunk_len + t. The state and the
// conv carries of every block live on the device between chunks.
#include <math.h>
#include <string.h>

#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"
#include "kernels.cuh"

namespace tgc {

__device__ __forceinline__ void ssm_split(float y, __nv_bfloat16 &h, __nv_bfloat16 &l)
{
	h = __float2bfloat16_rn(y);
	l = __float2bfloat16_rn(y - __bfloat162float(h));
}

__device__ __forceinline__ float ssm_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float ssm_softplus(float x) { return __fadd_rn(x > 0.0f ? x : 0.0f, log1pf(expf(-fabsf(x)))); }
// The scan's per-step gate and dt in CUDA's fast intrinsics (absolute error near 2^-21 here);
// the scan is issue-bound and these are most of its work outside the state loop.
__device__ __forceinline__ float ssm_silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float ssm_softplus_fast(float x) { return fmaxf(x, 0.0f) + __logf(1.0f + __expf(-fabsf(x))); }

// Rows of the input chunk (or of the stream) -> n = rmsnorm(x) * w split hi/lo. One warp per row.
// With out != nullptr it is the final norm: the f32 result goes to out row (s, t0 + t) of
// the [nseq][T][D] output instead.
__global__ void k_ssm_norm(const float *__restrict__ x, long M, int D, const float *__restrict__ w, float eps,
			   __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo, float *__restrict__ out, int Tc, int T,
			   int t0)
{
	long r = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
	int lane = threadIdx.x & 31;
	if (r >= M) return;
	const float *xr = x + r * D;
	float ss = 0.0f;
	for (int i = lane; i < D; i += 32) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
#pragma unroll
	for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
	float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
	if (out) {
		long s = r / Tc, t = r % Tc;
		float *o = out + (s * T + t0 + t) * D;
		for (int i = lane; i < D; i += 32) o[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
		return;
	}
	for (int i = lane; i < D; i += 32) ssm_split(__fmul_rn(__fmul_rn(xr[i], inv), w[i]), hi[r * D + i], lo[r * D + i]);
}

// Causal conv + silu. Thread = (sequence, channel); carries c[3][DI] per sequence hold
// x_{t-1}, x_{t-2}, x_{t-3} across chunks. xz rows: [x (DI) | z (DI)]. The inputs of 8
// steps are loaded before any of them is used: one load in flight per thread would leave
// HBM latency-bound at these thread counts.
__global__ void k_ssm_conv(const float *__restrict__ xz, int S, int Tc, int DI, const float *__restrict__ cw,
			   const float *__restrict__ cb, float *__restrict__ carry, float *__restrict__ xs,
			   __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo)
{
	constexpr int U = 8;
	long tid = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (tid >= (long)S * DI) return;
	const int s = (int)(tid / DI), c = (int)(tid % DI);
	float *cr = carry + (long)s * 3 * DI;
	float c1 = cr[c], c2 = cr[DI + c], c3 = cr[2 * DI + c];
	const float w0 = cw[c], w1 = cw[DI + c], w2 = cw[2 * DI + c], w3 = cw[3 * DI + c], b = cb[c];
	auto step = [&](long row, float x) {
		float a = __fadd_rn(__fmul_rn(c3, w0), __fmul_rn(c2, w1));
		a = __fadd_rn(a, __fmul_rn(c1, w2));
		a = __fadd_rn(a, __fmul_rn(x, w3));
		a = __fadd_rn(a, b);
		c3 = c2, c2 = c1, c1 = x;
		const float v = ssm_silu(a);
		xs[row * DI + c] = v;
		ssm_split(v, hi[row * DI + c], lo[row * DI + c]);
	};
	const long row0 = (long)s * Tc;
	int t = 0;
	for (; t + U <= Tc; t += U) {
		float x[U];
#pragma unroll
		for (int u = 0; u < U; u++) x[u] = xz[(row0 + t + u) * 2 * DI + c];
#pragma unroll
		for (int u = 0; u < U; u++) step(row0 + t + u, x[u]);
	}
	for (; t < Tc; t++) step(row0 + t, xz[(row0 + t) * 2 * DI + c]);
	cr[c] = c1, cr[DI + c] = c2, cr[2 * DI + c] = c3;
}

// The selective scan. CTA = (128 channels, one sequence); dbc rows [r (R) | bt (DS) | ct (DS) |
// zero padding] of the chunk are staged in shared memory. Each thread keeps h[DS] of its
// channel in registers for the whole chunk.
template <int DS, int R>
__global__ void __launch_bounds__(128) k_ssm_scan(const float *__restrict__ dbc, int ldd, const float *__restrict__ xs,
						  const float *__restrict__ xz, int Tc, int DI, const float *__restrict__ wdt,
						  const float *__restrict__ sdt, const float *__restrict__ dtb,
						  const float *__restrict__ A, const float *__restrict__ Dv,
						  float *__restrict__ state, __nv_bfloat16 *__restrict__ ghi,
						  __nv_bfloat16 *__restrict__ glo)
{
	extern __shared__ float sd[]; // [Tc][R + 2 DS]
	constexpr int W = R + 2 * DS;
	const int s = blockIdx.y, c = blockIdx.x * 128 + threadIdx.x;
	for (int i = threadIdx.x; i < Tc * W; i += 128) {
		int t = i / W, j = i % W;
		sd[i] = dbc[((long)s * Tc + t) * ldd + j];
	}
	__syncthreads();
	if (c >= DI) return;
	float h[DS], a[DS], ia[DS], w[R];
	float *st = state + ((long)s * DI + c) * DS;
#pragma unroll
	for (int k = 0; k < DS; k++) {
		h[k] = st[k];
		a[k] = A[(long)c * DS + k];
		ia[k] = 1.0f / a[k];
	}
#pragma unroll
	for (int p = 0; p < R; p++) w[p] = wdt[(long)c * R + p]; // codes of column c of Wdt
	const float sc = sdt[c], bias = dtb[c], dd = Dv[c];
	// x and z of step t + 1 are loaded while step t computes (the loop is latency-bound otherwise)
	float xn = xs[(long)s * Tc * DI + c], zn = xz[(long)s * Tc * 2 * DI + DI + c];
	for (int t = 0; t < Tc; t++) {
		const float *row = sd + t * W;
		const long gr = (long)s * Tc + t;
		const float x = xn, zt = zn;
		if (t + 1 < Tc) {
			xn = xs[(gr + 1) * DI + c];
			zn = xz[(gr + 1) * 2 * DI + DI + c];
		}
		// dt = softplus(s * sum_p r[p] code[p] + dt_b), the sum in p order (runtime/tg_rt.h:143-151),
		// each term fused into the running sum (one rounding per term instead of two)
		float acc = 0.0f;
#pragma unroll
		for (int p = 0; p < R; p++) acc = fmaf(row[p], w[p], acc);
		const float dt = ssm_softplus_fast(fmaf(sc, acc, bias));
		float m1 = 0.0f;
		// the state update of the program, h = e*h + (1 - e)/a * (x*bt) with e = exp(-dt*a), in
		// the fast forms: the hardware exp2 approximation (relative error about 2^-21 on this
		// range) and a multiply by 1/a (within an ulp of the division). Written as
		// h = q + e*(h - q) with q = (x*bt)/a, the same value in one instruction fewer per
		// state: the per-state work is the inner loop of the whole SSM
#pragma unroll
		for (int k = 0; k < DS; k++) {
			const float e = __expf(-(dt * a[k]));
			const float q = (x * row[R + k]) * ia[k];
			h[k] = fmaf(e, h[k] - q, q);
		}
#pragma unroll
		for (int k = 0; k < DS; k++) m1 = fmaf(h[k], row[R + DS + k], m1);
		const float y = __fadd_rn(m1, __fmul_rn(dd, x));
		const float g = __fmul_rn(y, ssm_silu_fast(zt));
		ssm_split(g, ghi[gr * DI + c], glo[gr * DI + c]);
	}
#pragma unroll
	for (int k = 0; k < DS; k++) st[k] = h[k];
}

// [rows=in, cols=out] codes -> f32 codes transposed [out][in] (the dt projection's columns)
__global__ void k_codes_f32_t(const signed char *__restrict__ q, int bits, int rows, int cols, float *__restrict__ dst)
{
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (t >= (long)rows * cols) return;
	int r = (int)(t / cols), c = (int)(t % cols);
	dst[(long)c * rows + r] = (float)qcode(q, bits, t);
}

} // namespace tgc

using namespace tgc;

namespace {

constexpr int XP_ROWS = 128; // the x-projection's output rows [r | bt | ct] padded to one GEMM tile

struct Block {
	DevBuf norm, win, swin, conv_w, conv_b, wxp, sxp, wdt, sdt, dtb, a, d, wo, so;
};

struct Engine {
	int dev = -1;
	cudaStream_t st = nullptr;
	int B = 0, DM = 0, DI = 0, DS = 0, R = 0, bits = 0;
	float eps = 1e-6f;
	int max_seqs = 0, chunk = 0;
	std::vector<std::unique_ptr<Block>> blocks;
	DevBuf nf, u, nhi, nlo, xz, xs, xhi, xlo, dbc, ghi, glo, state, carry, status, io;
	cudaEvent_t e0 = nullptr, e1 = nullptr;
	// host rows: a second chunk buffer and copy streams, so that chunk c+1 comes in and
	// chunk c-1 goes out while chunk c computes (created on the first host call)
	DevBuf u2;
	cudaStream_t cp_in = nullptr, cp_out = nullptr;
	cudaEvent_t in_ready[2] = {}, done[2] = {}, wave_start = nullptr, out_done = nullptr;
	long launches = 0;
	// profiling: an event pair around every GEMM / scan launch, reused across calls
	bool prof = false;
	struct Mark {
		cudaEvent_t a, b;
		int scan;
		double flops;
	};
	std::vector<Mark> marks;
	size_t nmarks = 0;
	tg_cuda_ssm_stats last{};
	~Engine()
	{
		if (dev >= 0) cudaSetDevice(dev);
		for (auto &m : marks) {
			cudaEventDestroy(m.a);
			cudaEventDestroy(m.b);
		}
		if (e0) cudaEventDestroy(e0);
		if (e1) cudaEventDestroy(e1);
		for (cudaEvent_t e : { in_ready[0], in_ready[1], done[0], done[1], wave_start, out_done })
			if (e) cudaEventDestroy(e);
		if (cp_in) cudaStreamDestroy(cp_in);
		if (cp_out) cudaStreamDestroy(cp_out);
		if (st) cudaStreamDestroy(st);
	}
};

// Opens a mark (when profiling): returns its index, or -1.
int mark_begin(Engine &g, int scan, double flops)
{
	if (!g.prof) return -1;
	if (g.nmarks == g.marks.size()) {
		Engine::Mark m{};
		if (cudaEventCreate(&m.a) != cudaSuccess || cudaEventCreate(&m.b) != cudaSuccess) return -1;
		g.marks.push_back(m);
	}
	Engine::Mark &m = g.marks[g.nmarks];
	m.scan = scan, m.flops = flops;
	cudaEventRecord(m.a, g.st);
	return (int)g.nmarks++;
}

void mark_end(Engine &g, int i)
{
	if (i >= 0) cudaEventRecord(g.marks[i].b, g.st);
}

int gemm_marked(Engine &g, const GemmOperands &op, const GemmArgs &p, double useful_cols)
{
	int mk = mark_begin(g, 0, 2.0 * p.M * useful_cols * p.K);
	int rc = gemm(op, p, g.st);
	mark_end(g, mk);
	return rc;
}

int upload(DevBuf &b, const void *src, size_t bytes, int dev, cudaStream_t st)
{
	int rc = b.alloc(bytes, dev);
	if (rc) return rc;
	TGC_CUDA(cudaMemcpyAsync(b.p, src, bytes, cudaMemcpyHostToDevice, st));
	TGC_CUDA(cudaStreamSynchronize(st));
	return TG_CUDA_OK;
}

size_t qbytes(long n, int bits) { return bits == 8 ? (size_t)n : (size_t)(n + 1) / 2; }

int load_engine(Engine &g, const tg_cuda_ssm_desc *d, int dev, int max_seqs, int chunk)
{
	int rc;
	g.dev = dev;
	TGC_CUDA(cudaSetDevice(dev));
	TGC_CUDA(cudaStreamCreateWithFlags(&g.st, cudaStreamNonBlocking));
	TGC_CUDA(cudaEventCreate(&g.e0));
	TGC_CUDA(cudaEventCreate(&g.e1));
	g.B = d->blocks, g.DM = d->d_model, g.DI = d->d_inner, g.DS = d->d_state, g.R = d->dt_rank, g.bits = d->bits;
	g.eps = d->eps, g.max_seqs = max_seqs, g.chunk = chunk;
	const int DM = g.DM, DI = g.DI, DS = g.DS, R = g.R, bits = g.bits;
	if ((rc = upload(g.nf, d->final_norm, (size_t)DM * 4, dev, g.st))) return rc;
	DevBuf tq;
	// codes of [rows=in, cols=out] -> rows [row0, row0 + cols) of a [*, ld] bf16 K-major matrix
	auto codes_T = [&](const tg_cuda_qmat &m, long rows, long cols, __nv_bfloat16 *dst, long ld) -> int {
		int r;
		if ((r = upload(tq, m.q, qbytes(rows * cols, bits), dev, g.st))) return r;
		if ((r = codes_to_bf16(tq.as<signed char>(), bits, rows, cols, true, dst, ld, g.st))) return r;
		TGC_CUDA(cudaStreamSynchronize(g.st));
		return TG_CUDA_OK;
	};
	for (int b = 0; b < g.B; b++) {
		auto Y = std::make_unique<Block>();
		if ((rc = upload(Y->norm, d->norm[b], (size_t)DM * 4, dev, g.st)) ||
		    (rc = upload(Y->conv_w, d->conv_w[b], (size_t)4 * DI * 4, dev, g.st)) ||
		    (rc = upload(Y->conv_b, d->conv_b[b], (size_t)DI * 4, dev, g.st)) ||
		    (rc = upload(Y->dtb, d->dt_b[b], (size_t)DI * 4, dev, g.st)) ||
		    (rc = upload(Y->a, d->a[b], (size_t)DI * DS * 4, dev, g.st)) ||
		    (rc = upload(Y->d, d->d[b], (size_t)DI * 4, dev, g.st)))
			return rc;
		// in projection: [Wx | Wz] as one [2 DI, DM] operand, scales concatenated
		if ((rc = Y->win.alloc((size_t)2 * DI * DM * 2, dev)) || (rc = Y->swin.alloc((size_t)2 * DI * 4, dev))) return rc;
		if ((rc = codes_T(d->w_x[b], DM, DI, Y->win.as<__nv_bfloat16>(), DM)) ||
		    (rc = codes_T(d->w_z[b], DM, DI, Y->win.as<__nv_bfloat16>() + (size_t)DI * DM, DM)))
			return rc;
		TGC_CUDA(cudaMemcpy(Y->swin.p, d->w_x[b].s, (size_t)DI * 4, cudaMemcpyHostToDevice));
		TGC_CUDA(cudaMemcpy(Y->swin.as<float>() + DI, d->w_z[b].s, (size_t)DI * 4, cudaMemcpyHostToDevice));
		// x projection: [Wr | WB | WC] as rows 0 .. R + 2 DS of a zero-padded [128, DI] operand
		if ((rc = Y->wxp.alloc((size_t)XP_ROWS * DI * 2, dev)) || (rc = Y->sxp.alloc((size_t)XP_ROWS * 4, dev))) return rc;
		TGC_CUDA(cudaMemset(Y->wxp.p, 0, Y->wxp.bytes));
		TGC_CUDA(cudaMemset(Y->sxp.p, 0, Y->sxp.bytes));
		if ((rc = codes_T(d->w_r[b], DI, R, Y->wxp.as<__nv_bfloat16>(), DI)) ||
		    (rc = codes_T(d->w_b[b], DI, DS, Y->wxp.as<__nv_bfloat16>() + (size_t)R * DI, DI)) ||
		    (rc = codes_T(d->w_c[b], DI, DS, Y->wxp.as<__nv_bfloat16>() + (size_t)(R + DS) * DI, DI)))
			return rc;
		TGC_CUDA(cudaMemcpy(Y->sxp.p, d->w_r[b].s, (size_t)R * 4, cudaMemcpyHostToDevice));
		TGC_CUDA(cudaMemcpy(Y->sxp.as<float>() + R, d->w_b[b].s, (size_t)DS * 4, cudaMemcpyHostToDevice));
		TGC_CUDA(cudaMemcpy(Y->sxp.as<float>() + R + DS, d->w_c[b].s, (size_t)DS * 4, cudaMemcpyHostToDevice));
		// dt projection: f32 codes, column-major ([DI][R]), for the scan's 16 MACs per channel
		if ((rc = upload(tq, d->w_dt[b].q, qbytes((long)R * DI, bits), dev, g.st)) || (rc = Y->wdt.alloc((size_t)DI * R * 4, dev)) ||
		    (rc = upload(Y->sdt, d->w_dt[b].s, (size_t)DI * 4, dev, g.st)))
			return rc;
		k_codes_f32_t<<<(unsigned)((R * DI + 255) / 256), 256, 0, g.st>>>(tq.as<signed char>(), bits, R, DI, Y->wdt.as<float>());
		TGC_LAUNCH_CHECK();
		TGC_CUDA(cudaStreamSynchronize(g.st));
		// out projection [DM, DI]
		if ((rc = Y->wo.alloc((size_t)DM * DI * 2, dev)) || (rc = upload(Y->so, d->w_o[b].s, (size_t)DM * 4, dev, g.st))) return rc;
		if ((rc = codes_T(d->w_o[b], DI, DM, Y->wo.as<__nv_bfloat16>(), DI))) return rc;
		g.blocks.push_back(std::move(Y));
	}
	const size_t M = (size_t)max_seqs * chunk;
	if ((rc = g.u.alloc(M * DM * 4, dev)) || (rc = g.nhi.alloc(M * DM * 2, dev)) || (rc = g.nlo.alloc(M * DM * 2, dev)) ||
	    (rc = g.xz.alloc(M * 2 * DI * 4, dev)) || (rc = g.xs.alloc(M * DI * 4, dev)) || (rc = g.xhi.alloc(M * DI * 2, dev)) ||
	    (rc = g.xlo.alloc(M * DI * 2, dev)) || (rc = g.dbc.alloc(M * XP_ROWS * 4, dev)) || (rc = g.ghi.alloc(M * DI * 2, dev)) ||
	    (rc = g.glo.alloc(M * DI * 2, dev)) || (rc = g.state.alloc((size_t)g.B * max_seqs * DI * DS * 4, dev)) ||
	    (rc = g.carry.alloc((size_t)g.B * max_seqs * 3 * DI * 4, dev)) || (rc = g.status.alloc(64, dev)))
		return rc;
	TGC_CUDA(cudaMemset(g.status.p, 0, 64));
	return TG_CUDA_OK;
}

GemmArgs gemm_args(int M, int N, int K, int *status)
{
	GemmArgs p;
	memset(&p, 0, sizeof p);
	p.M = M, p.N = N, p.K = K, p.epi = EPI_STORE;
	p.na = 2, p.nb = 1, p.npairs = 2;
	p.pa[0] = 0, p.pb[0] = 0, p.pa[1] = 1, p.pb[1] = 0;
	p.scale_mode = 2;
	p.status = status;
	return p;
}

template <int DS, int R>
int launch_scan(Engine &g, Block &Y, int S, int Tc, int b)
{
	const int DI = g.DI;
	dim3 grid((unsigned)((DI + 127) / 128), (unsigned)S);
	size_t smem = (size_t)Tc * (R + 2 * DS) * 4;
	k_ssm_scan<DS, R><<<grid, 128, smem, g.st>>>(g.dbc.as<float>(), XP_ROWS, g.xs.as<float>(), g.xz.as<float>(), Tc, DI,
						     Y.wdt.as<float>(), Y.sdt.as<float>(), Y.dtb.as<float>(), Y.a.as<float>(),
						     Y.d.as<float>(), g.state.as<float>() + (size_t)b * g.max_seqs * DI * DS,
						     g.ghi.as<__nv_bfloat16>(), g.glo.as<__nv_bfloat16>());
	TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

// One chunk of Tc steps of S sequences: u holds the chunk's rows (and is the residual stream the
// blocks add into); the output rows go to out.
int run_chunk(Engine &g, float *u, int S, int Tc, int T, int t0, float *out)
{
	int rc;
	const int DM = g.DM, DI = g.DI;
	const long M = (long)S * Tc;
	int *status = g.status.as<int>();
	const unsigned warps_grid = (unsigned)((M * 32 + 255) / 256);
	for (int b = 0; b < g.B; b++) {
		Block &Y = *g.blocks[b];
		k_ssm_norm<<<warps_grid, 256, 0, g.st>>>(u, M, DM, Y.norm.as<float>(), g.eps, g.nhi.as<__nv_bfloat16>(),
							g.nlo.as<__nv_bfloat16>(), nullptr, Tc, T, t0);
		TGC_LAUNCH_CHECK();
		GemmOperands op;
		op.a[0] = g.nhi.p, op.a[1] = g.nlo.p, op.b[0] = Y.win.p, op.lda = DM, op.ldb = DM;
		GemmArgs p = gemm_args((int)M, 2 * DI, DM, status);
		p.scale = Y.swin.as<float>(), p.out = g.xz.as<float>(), p.ldo = 2 * DI;
		if ((rc = gemm_marked(g, op, p, 2 * DI))) return rc;
		const long thr = (long)S * DI;
		k_ssm_conv<<<(unsigned)((thr + 127) / 128), 128, 0, g.st>>>(
			g.xz.as<float>(), S, Tc, DI, Y.conv_w.as<float>(), Y.conv_b.as<float>(),
			g.carry.as<float>() + (size_t)b * g.max_seqs * 3 * DI, g.xs.as<float>(), g.xhi.as<__nv_bfloat16>(),
			g.xlo.as<__nv_bfloat16>());
		TGC_LAUNCH_CHECK();
		GemmOperands ox;
		ox.a[0] = g.xhi.p, ox.a[1] = g.xlo.p, ox.b[0] = Y.wxp.p, ox.lda = DI, ox.ldb = DI;
		GemmArgs px = gemm_args((int)M, XP_ROWS, DI, status);
		px.scale = Y.sxp.as<float>(), px.out = g.dbc.as<float>(), px.ldo = XP_ROWS;
		if ((rc = gemm_marked(g, ox, px, g.R + 2 * g.DS))) return rc;
		const int mk = mark_begin(g, 1, (double)M * DI * (2.0 * g.R + 10.0 * g.DS + 6.0));
		if (g.DS == 16 && g.R == 16) rc = launch_scan<16, 16>(g, Y, S, Tc, b);
		else if (g.DS == 4 && g.R == 4) rc = launch_scan<4, 4>(g, Y, S, Tc, b);
		else return set_err(TG_CUDA_EUNSUPPORTED, "ssm: d_state %d with dt_rank %d", g.DS, g.R);
		mark_end(g, mk);
		if (rc) return rc;
		GemmOperands oo;
		oo.a[0] = g.ghi.p, oo.a[1] = g.glo.p, oo.b[0] = Y.wo.p, oo.lda = DI, oo.ldb = DI;
		GemmArgs po = gemm_args((int)M, DM, DI, status);
		po.epi = EPI_ADD, po.scale = Y.so.as<float>(), po.out = u, po.ldo = DM;
		if ((rc = gemm_marked(g, oo, po, DM))) return rc;
		g.launches += 6;
	}
	k_ssm_norm<<<warps_grid, 256, 0, g.st>>>(u, M, DM, g.nf.as<float>(), g.eps, nullptr, nullptr, out, Tc, T, t0);
	TGC_LAUNCH_CHECK();
	g.launches += 1;
	return TG_CUDA_OK;
}

// The host path's copy streams and events, made on first use.
int host_pipe(Engine &g)
{
	if (!g.cp_in) TGC_CUDA(cudaStreamCreateWithFlags(&g.cp_in, cudaStreamNonBlocking));
	if (!g.cp_out) TGC_CUDA(cudaStreamCreateWithFlags(&g.cp_out, cudaStreamNonBlocking));
	for (cudaEvent_t *e : { &g.in_ready[0], &g.in_ready[1], &g.done[0], &g.done[1], &g.wave_start, &g.out_done })
		if (!*e) TGC_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
	return TG_CUDA_OK;
}

// Host rows: chunk c computes in buffer c % 2 on the compute stream while chunk c+1's rows
// come into the other buffer on cp_in (once chunk c-1 has finished with it) and chunk c-1's
// output rows go back on cp_out. The compute stream ends the wave waiting for the last copy,
// so a synchronize on it covers the copies, and the next wave reuses the buffers safely.
int run_wave_host(Engine &g, const float *u, int S, int T, float *out)
{
	int rc;
	const int DM = g.DM;
	const size_t pitch = (size_t)T * DM * 4;
	if ((rc = host_pipe(g)) || (rc = g.u2.ensure(g.u.bytes, g.dev)) || (rc = g.io.ensure((size_t)S * pitch, g.dev)))
		return rc;
	float *ub[2] = { g.u.as<float>(), g.u2.as<float>() };
	float *dout = g.io.as<float>();
	const int nch = (T + g.chunk - 1) / g.chunk;
	auto rows = [&](int c) { return std::min(g.chunk, T - c * g.chunk); };
	auto copy_in = [&](int c) -> int { // rows (s, t0 .. t0 + Tc) of every sequence -> the chunk, sequence-major
		const size_t w = (size_t)rows(c) * DM * 4;
		TGC_CUDA(cudaMemcpy2DAsync(ub[c & 1], w, u + (size_t)c * g.chunk * DM, pitch, w, S, cudaMemcpyHostToDevice, g.cp_in));
		TGC_CUDA(cudaEventRecord(g.in_ready[c & 1], g.cp_in));
		return TG_CUDA_OK;
	};
	auto copy_out = [&](int c) -> int {
		const size_t off = (size_t)c * g.chunk * DM;
		TGC_CUDA(cudaStreamWaitEvent(g.cp_out, g.done[c & 1], 0));
		TGC_CUDA(cudaMemcpy2DAsync(out + off, pitch, dout + off, pitch, (size_t)rows(c) * DM * 4, S, cudaMemcpyDeviceToHost,
					   g.cp_out));
		return TG_CUDA_OK;
	};
	auto body = [&]() -> int {
		int rc;
		TGC_CUDA(cudaEventRecord(g.wave_start, g.st)); // the previous wave is done with both buffers
		TGC_CUDA(cudaStreamWaitEvent(g.cp_in, g.wave_start, 0));
		if ((rc = copy_in(0))) return rc;
		for (int c = 0; c < nch; c++) {
			TGC_CUDA(cudaStreamWaitEvent(g.st, g.in_ready[c & 1], 0));
			if ((rc = run_chunk(g, ub[c & 1], S, rows(c), T, c * g.chunk, dout))) return rc;
			TGC_CUDA(cudaEventRecord(g.done[c & 1], g.st));
			if (c + 1 < nch) {
				// the other buffer was chunk c-1's: its done event is that chunk's latest record
				if (c >= 1) TGC_CUDA(cudaStreamWaitEvent(g.cp_in, g.done[(c + 1) & 1], 0));
				if ((rc = copy_in(c + 1))) return rc;
			}
			// chunk c-1's rows leave only now, after chunk c is queued: a pageable destination
			// makes the copy call wait for its chunk, and the GPU has chunk c to run meanwhile
			if (c >= 1 && (rc = copy_out(c - 1))) return rc;
		}
		if ((rc = copy_out(nch - 1))) return rc;
		TGC_CUDA(cudaEventRecord(g.out_done, g.cp_out));
		TGC_CUDA(cudaStreamWaitEvent(g.st, g.out_done, 0));
		return TG_CUDA_OK;
	};
	if ((rc = body())) { // no copy may still use the caller's buffers after an error return
		cudaStreamSynchronize(g.cp_in);
		cudaStreamSynchronize(g.cp_out);
	}
	return rc;
}

// nseq sequences of T steps: u, out [nseq][T][DM], on the device (device == true) or host.
int run_wave(Engine &g, const float *u, int S, int T, float *out, bool device)
{
	int rc;
	const int DM = g.DM, DI = g.DI, DS = g.DS;
	TGC_CUDA(cudaMemsetAsync(g.state.p, 0, (size_t)g.B * g.max_seqs * DI * DS * 4, g.st));
	TGC_CUDA(cudaMemsetAsync(g.carry.p, 0, (size_t)g.B * g.max_seqs * 3 * DI * 4, g.st));
	if (!device) return run_wave_host(g, u, S, T, out);
	for (int t0 = 0; t0 < T; t0 += g.chunk) {
		const int Tc = std::min(g.chunk, T - t0);
		// rows (s, t0 .. t0 + Tc) of every sequence -> the chunk, sequence-major
		TGC_CUDA(cudaMemcpy2DAsync(g.u.p, (size_t)Tc * DM * 4, u + (size_t)t0 * DM, (size_t)T * DM * 4, (size_t)Tc * DM * 4, S,
					   cudaMemcpyDeviceToDevice, g.st));
		if ((rc = run_chunk(g, g.u.as<float>(), S, Tc, T, t0, out))) return rc;
	}
	return TG_CUDA_OK;
}

} // namespace

struct tg_cuda_ssm {
	std::vector<std::unique_ptr<Engine>> eng;
};

extern "C" int tg_cuda_ssm_load(const tg_cuda_ssm_desc *d, int max_seqs, int chunk, tg_cuda_ssm **out)
{
	clear_err();
	if (!out) return set_err(TG_CUDA_EINVAL, "tg_cuda_ssm_load: NULL out");
	*out = nullptr;
	if (!d || max_seqs <= 0 || chunk <= 0 || d->blocks <= 0 || d->d_model <= 0 || d->d_inner <= 0 || d->d_state <= 0 ||
	    d->dt_rank <= 0 || (d->bits != 8 && d->bits != 4) || !d->final_norm || !d->norm || !d->conv_w || !d->conv_b ||
	    !d->dt_b || !d->d || !d->a || !d->w_x || !d->w_z || !d->w_r || !d->w_b || !d->w_c || !d->w_dt || !d->w_o)
		return set_err(TG_CUDA_EINVAL, "tg_cuda_ssm_load: bad descriptor");
	if (!((d->d_state == 16 && d->dt_rank == 16) || (d->d_state == 4 && d->dt_rank == 4)))
		return set_err(TG_CUDA_EUNSUPPORTED, "tg_cuda_ssm_load: d_state %d / dt_rank %d (built: 16/16 and 4/4)", d->d_state,
			       d->dt_rank);
	if (d->d_model % 64 || d->d_inner % 64 || d->dt_rank + 2 * d->d_state > XP_ROWS)
		return set_err(TG_CUDA_EUNSUPPORTED, "tg_cuda_ssm_load: d_model and d_inner must be multiples of 64");
	if (!inited()) return set_err(TG_CUDA_ENODEV, "tg_cuda_ssm_load: call tg_cuda_init first");
	auto *g = new tg_cuda_ssm;
	for (auto &dv : devices()) {
		auto e = std::make_unique<Engine>();
		int rc = load_engine(*e, d, dv.id, max_seqs, chunk);
		if (rc) {
			delete g;
			return rc;
		}
		g->eng.push_back(std::move(e));
	}
	cudaSetDevice(devices()[0].id);
	*out = g;
	return TG_CUDA_OK;
}

static int ssm_forward(tg_cuda_ssm *g, const float *u, long nseq, int T, float *out, bool device)
{
	clear_err();
	if (!g || !u || !out || nseq < 0 || T <= 0) return set_err(TG_CUDA_EINVAL, "tg_cuda_ssm_forward: bad arguments");
	const size_t G = device ? 1 : g->eng.size();
	std::vector<int> rcs(G, 0);
	std::vector<std::string> errs(G);
	auto work = [&](size_t di) {
		Engine &e = *g->eng[di];
		cudaSetDevice(e.dev);
		const long lo = nseq * (long)di / (long)G, hi = nseq * (long)(di + 1) / (long)G;
		const size_t per = (size_t)T * e.DM;
		int rc = TG_CUDA_OK;
		e.launches = 0;
		e.nmarks = 0;
		cudaEventRecord(e.e0, e.st);
		for (long w0 = lo; w0 < hi && !rc; w0 += e.max_seqs) {
			const int S = (int)std::min<long>(e.max_seqs, hi - w0);
			rc = run_wave(e, u + w0 * per, S, T, out + w0 * per, device);
		}
		cudaEventRecord(e.e1, e.st);
		if (!rc) {
			cudaError_t ce = cudaStreamSynchronize(e.st);
			if (ce != cudaSuccess) rc = set_err(TG_CUDA_ECUDA, "device %d: %s", e.dev, cudaGetErrorString(ce));
		}
		if (!rc) {
			tg_cuda_ssm_stats t{};
			float ms = 0;
			cudaEventElapsedTime(&ms, e.e0, e.e1);
			t.device_ms = ms, t.launches = e.launches;
			for (size_t i = 0; i < e.nmarks; i++) {
				float x = 0;
				cudaEventElapsedTime(&x, e.marks[i].a, e.marks[i].b);
				if (e.marks[i].scan) t.scan_ms += x, t.scan_flops += e.marks[i].flops, t.scan_launches++;
				else t.gemm_ms += x, t.gemm_flops += e.marks[i].flops, t.gemm_launches++;
			}
			e.last = t;
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

extern "C" int tg_cuda_ssm_forward(tg_cuda_ssm *g, const float *u, long nseq, int T, float *out)
{
	return ssm_forward(g, u, nseq, T, out, false);
}

extern "C" int tg_cuda_ssm_forward_device(tg_cuda_ssm *g, const float *u, long nseq, int T, float *out)
{
	return ssm_forward(g, u, nseq, T, out, true);
}

extern "C" int tg_cuda_ssm_profile(tg_cuda_ssm *g, int enable)
{
	clear_err();
	if (!g) return set_err(TG_CUDA_EINVAL, "tg_cuda_ssm_profile: NULL model");
	for (auto &e : g->eng) e->prof = enable != 0;
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_ssm_get_stats(const tg_cuda_ssm *g, tg_cuda_ssm_stats *out)
{
	clear_err();
	if (!g || !out) return set_err(TG_CUDA_EINVAL, "tg_cuda_ssm_get_stats: NULL argument");
	memset(out, 0, sizeof *out);
	for (auto &e : g->eng) {
		const tg_cuda_ssm_stats &t = e->last;
		out->device_ms = std::max(out->device_ms, t.device_ms);
		out->launches += t.launches;
		out->gemm_ms += t.gemm_ms, out->gemm_flops += t.gemm_flops, out->gemm_launches += t.gemm_launches;
		out->scan_ms += t.scan_ms, out->scan_flops += t.scan_flops, out->scan_launches += t.scan_launches;
	}
	return TG_CUDA_OK;
}

extern "C" void tg_cuda_ssm_free(tg_cuda_ssm *g)
{
	if (!g) return;
	for (auto &e : g->eng) {
		cudaSetDevice(e->dev);
		if (e->st) cudaStreamSynchronize(e->st);
	}
	delete g;
}
