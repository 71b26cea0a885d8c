// rowvm.cu -- the batch executor: a planned TGIR program run over many rows at
// once (tg_cuda_load / tg_cuda_batch). Replaces the par_for(batch_rows) loop of
// the batch branch (src/main.c:421-441) and vm_run_into per row (src/vm.c:475-481).
//
// Layout. The host compiles the program into a tape of device ops. Each thread
// executes the tape for one row. Its arena (the temporaries, planned with
// liveness sharing like src/plan.c) lives in shared memory in SoA form,
// arena[slot * ROWS_PER_CTA + thread], so the 32 lanes of a warp touch 32
// consecutive words: conflict-free. Params live once per CTA in shared memory
// (quantized params as their exact codes in f32 plus the channel scales), or in
// global memory when they do not fit. Think loops run on the device: at the end
// of a body each lane applies the halting test of src/vm.c:383-411 to its own
// row, the warp repeats the body while any lane is still iterating, and a lane
// that halted is masked off until the loop ends for the whole warp.
//
// Arithmetic follows the reference kernels (runtime/tg_rt.h) operation by
// operation: products and sums in the same order with explicit rounding
// (__fmul_rn/__fadd_rn, no contraction), scale after the sum for quantized
// matmuls, division by the sum in softmax. Transcendentals are CUDA's libm,
// which differs from glibc by a few ulp.
#include <limits.h>
#include <string.h>

#include <algorithm>
#include <condition_variable>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"
#include "jit.cuh"
#include "kernels.cuh"

namespace tgc {

// ---- device tape ----------------------------------------------------------------------

enum : int {
	D_CONST = 1, D_BIN, D_UN, D_MATMUL, D_ROW, D_RED, D_TRANS, D_OUTER, D_TAKE, D_COPY,
	D_THINK_BEGIN, D_THINK_END, D_SCAN_BEGIN, D_SCAN_SLICE, D_SCAN_END, D_SPMM, D_TOPK, D_MEMSCAN, D_SUFMATCH, D_SUMTO, D_TAKE_T, D_MEMSCAN_T,
};

// An operand: >= 0 an arena slot (per row), < 0 a param offset -(loc + 1) in the param blob.
struct DOp {
	int code, sub;        // tape opcode; TG op (bin/un/row/red) or variant
	int out, a, b, c;     // operand locations
	int n;                // element count of out (elementwise), etc.
	int dims[4], sa[4], sb[4]; // broadcast: out dims (rank in sub2), operand strides
	int rank;
	int m, k, nn, g;      // matmul dims, groups
	int scale;            // matmul: 0 none, 1 per row (qa), 2 per column (qb); c = scale location
	int depth, target;    // loops: depth, jump target
	int tid, maxit, yield, halt;
	float f, eps, hthr;
	int cnt, len;         // copies / scans: count and lengths
};

struct Prog {
	std::vector<DOp> tape;
	std::vector<float> blob; // params
	int arena = 0;           // floats per row
	int per = 0, nout = 0, nthink = 0, out_loc = 0;
	std::vector<int> in_off, in_len; // input i: arena location, length
	int max_depth = 0;
};

constexpr int VM_ROWS = 128; // rows (threads) per CTA
constexpr int VM_MAXDEPTH = 4;

struct Loc {
	float *p;
	int st;
};

__device__ __forceinline__ Loc loc(int l, float *ar, const float *pb)
{
	if (l >= 0) return { ar + (long)l * VM_ROWS, VM_ROWS };
	return { (float *)pb + (-(l + 1)), 1 };
}

// The element functions. They are compiled here for the interpreter and handed as source
// text to the run-time compiler for the specialised kernels, so both paths share one
// definition.
#define TGC_ROW_MATH(...) \
	__VA_ARGS__       \
	static const char kRowMathSrc[] = #__VA_ARGS__;
TGC_ROW_MATH(
__device__ __forceinline__ float un_op(int op, float x)
{
	switch (op) {
	case TG_CUDA_OP_NEG: return -x;
	case TG_CUDA_OP_TANH: return tanhf(x);
	case TG_CUDA_OP_RELU: return x > 0.0f ? x : 0.0f;
	case TG_CUDA_OP_SIGMOID: return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
	case TG_CUDA_OP_EXP: return expf(x);
	case TG_CUDA_OP_SQRT: return __fsqrt_rn(x);
	case TG_CUDA_OP_GELU: {
		float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
		float t = tanhf(__fmul_rn(0.7978845608f, __fadd_rn(x, x3)));
		return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
	}
	case TG_CUDA_OP_SILU: return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
	case TG_CUDA_OP_SOFTPLUS: return __fadd_rn(x > 0.0f ? x : 0.0f, log1pf(expf(-fabsf(x))));
	case TG_CUDA_OP_LOG: return logf(x);
	case TG_CUDA_OP_STEP: return x > 0.0f ? 1.0f : 0.0f;
	case TG_CUDA_OP_SIN: return sinf(x);
	case TG_CUDA_OP_COS: return cosf(x);
	case TG_CUDA_OP_FLOOR: return floorf(x);
	}
	return 0.0f;
}

__device__ __forceinline__ float bin_op(int op, float x, float y)
{
	switch (op) {
	case TG_CUDA_OP_ADD: return __fadd_rn(x, y);
	case TG_CUDA_OP_SUB: return __fsub_rn(x, y);
	case TG_CUDA_OP_MUL: return __fmul_rn(x, y);
	case TG_CUDA_OP_DIV: return __fdiv_rn(x, y);
	case TG_CUDA_OP_MAX: return x > y ? x : y;
	case TG_CUDA_OP_MIN: return x < y ? x : y;
	}
	return 0.0f;
}
)

// o[i,j] (+ per-group offsets) = sum_p a[i,p] b[p,j], in p order, scale after the sum.
__device__ void vm_matmul(const DOp &op, float *ar, const float *pb)
{
	Loc o = loc(op.out, ar, pb), a = loc(op.a, ar, pb), b = loc(op.b, ar, pb);
	const float *sc = op.scale ? loc(op.c, ar, pb).p : nullptr;
	const int m = op.m, k = op.k, n = op.nn;
	for (int g = 0; g < op.g; g++) {
		long oo = (long)g * m * n, ao = (long)g * m * k, bo = (long)g * k * n;
		for (int i = 0; i < m; i++)
			for (int j = 0; j < n; j++) {
				float acc = 0.0f;
				for (int p = 0; p < k; p++)
					acc = __fadd_rn(acc, __fmul_rn(a.p[(ao + (long)i * k + p) * a.st], b.p[(bo + (long)p * n + j) * b.st]));
				if (op.scale == 1) acc = __fmul_rn(sc[i], acc);
				else if (op.scale == 2) acc = __fmul_rn(sc[j], acc);
				o.p[(oo + (long)i * n + j) * o.st] = acc;
			}
	}
}

// Rounded table index or -1 (runtime/tg_rt.h:200-204).
__device__ __forceinline__ int ell_idx(float v, int d)
{
	const float r = floorf(__fadd_rn(v, 0.5f));
	return r >= 0.0f && r < (float)d ? (int)r : -1;
}

// spmm (runtime/tg_rt.h:206-235): ELLPACK rows of (index, value) pairs against a table
// [d, h], entries in order; a quantized table (sc != nullptr) holds exact codes and
// multiplies them by value * scale of the entry's row.
__device__ void vm_spmm(const DOp &op, float *ar, const float *pb)
{
	Loc o = loc(op.out, ar, pb), x = loc(op.a, ar, pb), w = loc(op.b, ar, pb);
	const float *sc = op.scale ? loc(op.c, ar, pb).p : nullptr;
	const int h = op.nn;
	for (int i = 0; i < op.m; i++) {
		for (int j = 0; j < h; j++) o.p[((long)i * h + j) * o.st] = 0.0f;
		for (int e = 0; e < op.k; e++) {
			const long xe = ((long)i * op.k + e) * 2;
			const float val = x.p[(xe + 1) * x.st];
			const int t = ell_idx(x.p[xe * x.st], op.g);
			if (t < 0 || val == 0.0f) continue;
			const float v = sc ? __fmul_rn(val, sc[t]) : val;
			for (int j = 0; j < h; j++) {
				float &y = o.p[((long)i * h + j) * o.st];
				y = __fadd_rn(y, __fmul_rn(v, w.p[((long)t * h + j) * w.st]));
			}
		}
	}
}

// topk (runtime/tg_rt.h:445-483): per row, the indices of the k largest entries, largest
// first, ties to the lower index, NaN never chosen, -1 past the row's other entries; by
// repeated selection of the next entry in the order (value descending, index ascending).
__device__ void vm_topk(const DOp &op, float *ar, const float *pb)
{
	Loc o = loc(op.out, ar, pb), x = loc(op.a, ar, pb);
	const int n = op.k, k = op.nn;
	for (int r = 0; r < op.m; r++) {
		float lv = 0.0f;
		int li = -1;
		for (int i = 0; i < k; i++) {
			int bi = -1;
			float bv = 0.0f;
			for (int j = 0; j < n; j++) {
				const float v = x.p[((long)r * n + j) * x.st];
				if (v != v) continue;
				if (li >= 0 && !(v < lv || (v == lv && j > li))) continue;
				if (bi < 0 || v > bv) bi = j, bv = v;
			}
			o.p[((long)r * k + i) * o.st] = (float)bi;
			if (bi >= 0) lv = bv, li = bi;
		}
	}
}

// memscan (runtime/tg_rt.h:485-516): the delta-rule memory, initially m0 (rows, dv), read
// and written by tn steps of k entries (row, a, c[, dd]); per step in entry order the reads
// r = sum a M[row] and rd = sum dd M[row], then M[row] += c (v - rd). Output: r, rd, final M.
__device__ void vm_memscan(const DOp &op, float *ar, const float *pb)
{
	Loc o = loc(op.out, ar, pb), m0 = loc(op.a, ar, pb), p = loc(op.b, ar, pb), v = loc(op.c, ar, pb);
	const int tn = op.m, k = op.k / 2, q = 3 + (op.k & 1), rows = op.nn, dv = op.g;
	const long mo = 2L * tn * dv; // M's offset in the output
	for (long i = 0; i < (long)rows * dv; i++) o.p[(mo + i) * o.st] = m0.p[i * m0.st];
	for (long st = 0; st < tn; st++) {
		const long e0 = st * k * q, ro = st * dv, rdo = ((long)tn + st) * dv;
		for (int j = 0; j < dv; j++) o.p[(ro + j) * o.st] = o.p[(rdo + j) * o.st] = 0.0f;
		for (int i = 0; i < k; i++) {
			const int t = ell_idx(p.p[(e0 + (long)i * q) * p.st], rows);
			if (t < 0) continue;
			const float a = p.p[(e0 + (long)i * q + 1) * p.st], dd = q == 4 ? p.p[(e0 + (long)i * q + 3) * p.st] : a;
			for (int j = 0; j < dv; j++) {
				const float mv = o.p[(mo + (long)t * dv + j) * o.st];
				o.p[(ro + j) * o.st] = __fadd_rn(o.p[(ro + j) * o.st], __fmul_rn(a, mv));
				o.p[(rdo + j) * o.st] = __fadd_rn(o.p[(rdo + j) * o.st], __fmul_rn(dd, mv));
			}
		}
		for (int i = 0; i < k; i++) {
			const int t = ell_idx(p.p[(e0 + (long)i * q) * p.st], rows);
			const float c = p.p[(e0 + (long)i * q + 2) * p.st];
			if (t < 0 || c == 0.0f) continue;
			for (int j = 0; j < dv; j++) {
				float &mv = o.p[(mo + (long)t * dv + j) * o.st];
				mv = __fadd_rn(mv, __fmul_rn(c, __fsub_rn(v.p[(st * dv + j) * v.st], o.p[(rdo + j) * o.st])));
			}
		}
	}
}

// sum_to (runtime/tg_rt.h:419-438): out (n elements) = the sum of x over its broadcast axes,
// walking the merged iteration space the compiler describes (rank, dims, out's strides); a
// broadcast innermost axis is summed by rows first, as the reference does.
__device__ void vm_sum_to(const DOp &op, float *ar, const float *pb)
{
	Loc o = loc(op.out, ar, pb), x = loc(op.a, ar, pb);
	const int r = op.rank, w = op.dims[r - 1];
	for (int i = 0; i < op.n; i++) o.p[(long)i * o.st] = 0.0f;
	long outer = 1, io = 0;
	for (int i = 0; i < r - 1; i++) outer *= op.dims[i];
	int idx[4] = { 0, 0, 0, 0 };
	for (long i = 0; i < outer; i++) {
		const long xo = i * w;
		if (op.sa[r - 1]) {
			for (int j = 0; j < w; j++) o.p[(io + j) * o.st] = __fadd_rn(o.p[(io + j) * o.st], x.p[(xo + j) * x.st]);
		} else {
			float acc = 0.0f;
			for (int j = 0; j < w; j++) acc = __fadd_rn(acc, x.p[(xo + j) * x.st]);
			o.p[io * o.st] = __fadd_rn(o.p[io * o.st], acc);
		}
		for (int q = r - 2; q >= 0; q--) {
			io += op.sa[q];
			if (++idx[q] < op.dims[q]) break;
			io -= (long)op.sa[q] * op.dims[q];
			idx[q] = 0;
		}
	}
}

// take_t (runtime/tg_rt.h:324-333): out [d, h] = 0, then g's rows added at the rows r names.
__device__ void vm_take_t(const DOp &op, float *ar, const float *pb)
{
	Loc o = loc(op.out, ar, pb), r = loc(op.a, ar, pb), g = loc(op.b, ar, pb);
	const int h = op.nn;
	for (long i = 0; i < (long)op.k * h; i++) o.p[i * o.st] = 0.0f;
	for (int i = 0; i < op.m; i++) {
		const int t = ell_idx(r.p[(long)i * r.st], op.k);
		if (t < 0) continue;
		for (int j = 0; j < h; j++) {
			float &y = o.p[((long)t * h + j) * o.st];
			y = __fadd_rn(y, g.p[((long)i * h + j) * g.st]);
		}
	}
}

// memscan_t (runtime/tg_rt.h:517-578): memscan's derivatives by replaying the steps backwards
// from the final memory, undoing each write. y is memscan's output, pv (tn, 4k + dv) the
// entries (row, a, c, d) then the step's value, g y's adjoint. Out: dP (tn k 4) at 0, dM0 at
// o1, dV at o2, the working memory at o3, zero-padded to n.
__device__ void vm_memscan_t(const DOp &op, float *ar, const float *pb)
{
	Loc o = loc(op.out, ar, pb), y = loc(op.a, ar, pb), pv = loc(op.b, ar, pb), g = loc(op.c, ar, pb);
	const long tn = op.m, k = op.k, rows = op.nn, dv = op.g, w = 4 * k + dv;
	const long o1 = (tn * k * 4 + dv - 1) / dv * dv, o2 = o1 + rows * dv, o3 = o2 + tn * dv;
	auto O = [&](long i) -> float & { return o.p[i * o.st]; };
	for (long i = 0; i < op.n; i++) O(i) = 0.0f;
	for (long i = 0; i < rows * dv; i++) O(o3 + i) = y.p[(2 * tn * dv + i) * y.st], O(o1 + i) = g.p[(2 * tn * dv + i) * g.st];
	for (long st = tn - 1; st >= 0; st--) {
		const long e = st * w, xo = e + 4 * k, rdo = (tn + st) * dv, gro = st * dv, grdo = (tn + st) * dv, dpo = st * k * 4,
			   dxo = o2 + st * dv;
		auto E = [&](long i) { return pv.p[(e + i) * pv.st]; };
		auto X = [&](long j) { return pv.p[(xo + j) * pv.st]; };
		auto RD = [&](long j) { return y.p[(rdo + j) * y.st]; };
		auto GR = [&](long j) { return g.p[(gro + j) * g.st]; };
		auto GRD = [&](long j) { return g.p[(grdo + j) * g.st]; };
		for (long i = k - 1; i >= 0; i--) { // the memory as this step read it
			const int t = ell_idx(E(i * 4), (int)rows);
			const float c = E(i * 4 + 2);
			if (t < 0 || c == 0.0f) continue;
			for (long j = 0; j < dv; j++) O(o3 + t * dv + j) = __fsub_rn(O(o3 + t * dv + j), __fmul_rn(c, __fsub_rn(X(j), RD(j))));
		}
		for (long i = 0; i < k; i++) { // the writes: dc_i and the value's gradient
			const int t = ell_idx(E(i * 4), (int)rows);
			const float c = E(i * 4 + 2);
			float dc = 0.0f;
			if (t < 0) continue;
			for (long j = 0; j < dv; j++) {
				const float dm = O(o1 + t * dv + j);
				dc = __fadd_rn(dc, __fmul_rn(dm, __fsub_rn(X(j), RD(j))));
				O(dxo + j) = __fadd_rn(O(dxo + j), __fmul_rn(c, dm));
			}
			O(dpo + i * 4 + 2) = dc;
		}
		for (long i = 0; i < k; i++) { // the reads: da_i and dd_i
			const int t = ell_idx(E(i * 4), (int)rows);
			float da = 0.0f, dd = 0.0f;
			if (t < 0) continue;
			for (long j = 0; j < dv; j++) {
				const float m = O(o3 + t * dv + j);
				da = __fadd_rn(da, __fmul_rn(GR(j), m));
				dd = __fadd_rn(dd, __fmul_rn(__fsub_rn(GRD(j), O(dxo + j)), m));
			}
			O(dpo + i * 4 + 1) = da, O(dpo + i * 4 + 3) = dd;
		}
		for (long i = 0; i < k; i++) { // the memory's adjoint before this step
			const int t = ell_idx(E(i * 4), (int)rows);
			const float a = E(i * 4 + 1), d = E(i * 4 + 3);
			if (t < 0) continue;
			for (long j = 0; j < dv; j++)
				O(o1 + t * dv + j) = __fadd_rn(O(o1 + t * dv + j),
							      __fadd_rn(__fmul_rn(a, GR(j)), __fmul_rn(d, __fsub_rn(GRD(j), O(dxo + j)))));
		}
	}
}

// sufmatch (runtime/tg_rt.h:579-666): per stream, a suffix automaton of the tokens so far;
// at step t the token that followed the first occurrence of the longest suffix of x[..t]
// seen before t (or -1) and that suffix's length. The automaton lives in the output's
// workspace as the reference lays it out -- per state (len, link, first end, edge list),
// per slot of an open-addressing edge table of H slots (state, symbol, target, next edge)
// -- so the whole output matches, workspace included.
struct SufWs {
	float *base;
	int st;
	long S0, E0, H;
	__device__ float &s(long i) const { return base[(S0 + i) * st]; }
	__device__ float &e(long i) const { return base[(E0 + i) * st]; }
	__device__ long slot(long state, long c) const
	{
		unsigned long h = ((unsigned long)state * 2654435761UL ^ (unsigned long)c * 40503UL) & (unsigned long)(H - 1);
		for (long probe = 0; probe < H; probe++, h = (h + 1) & (unsigned long)(H - 1))
			if (e(h * 4) < 0.0f || ((long)e(h * 4) == state && (long)e(h * 4 + 1) == c)) break;
		return (long)h; // the table holds fewer edges than slots, so an empty slot is reached
	}
	__device__ long get(long state, long c) const
	{
		const long h = slot(state, c);
		return e(h * 4) < 0.0f ? -1 : (long)e(h * 4 + 2);
	}
	__device__ void put(long state, long c, long to) const
	{
		const long h = slot(state, c);
		if (e(h * 4) < 0.0f) {
			e(h * 4) = (float)state, e(h * 4 + 1) = (float)c, e(h * 4 + 3) = s(state * 4 + 3);
			s(state * 4 + 3) = (float)h;
		}
		e(h * 4 + 2) = (float)to;
	}
};

__device__ void vm_sufmatch(const DOp &op, float *ar, const float *pb)
{
	Loc o = loc(op.out, ar, pb), x = loc(op.a, ar, pb);
	const long T = op.m, n = op.k;
	long H = 16;
	while (H < 6 * T + 6) H *= 2;
	const SufWs W{ o.p, o.st, 2 * T * n, 2 * T * n + 4 * (2 * T + 2), H };
	for (long g = 0; g < n; g++) {
		long nst = 1, last = 0, m = 0, l = 0;
		for (long i = 0; i < H; i++) W.e(i * 4) = -1.0f;
		W.s(0) = 0.0f, W.s(1) = -1.0f, W.s(2) = -1.0f, W.s(3) = -1.0f;
		for (long t = 0; t < T; t++) {
			const float xv = x.p[(t * n + g) * x.st];
			const long c = xv >= 0.0f ? (long)__fadd_rn(xv, 0.5f) : -1;
			float &o0 = o.p[((t * n + g) * 2) * o.st], &o1 = o.p[((t * n + g) * 2 + 1) * o.st];
			if (c < 0) {
				m = 0, l = 0;
				o0 = -1.0f, o1 = 0.0f;
				continue;
			}
			while (m != 0 && W.get(m, c) < 0) {
				m = (long)W.s(m * 4 + 1);
				l = (long)W.s(m * 4);
			}
			const long tr = W.get(m, c);
			if (tr >= 0) m = tr, l++;
			else m = 0, l = 0;
			const long fe = l > 0 ? (long)W.s(m * 4 + 2) : -1;
			o0 = fe >= 0 && fe + 1 <= t ? x.p[((fe + 1) * n + g) * x.st] : -1.0f;
			o1 = (float)l;
			const long cur = nst++;
			long pp = last;
			W.s(cur * 4) = __fadd_rn(W.s(last * 4), 1.0f), W.s(cur * 4 + 2) = (float)t, W.s(cur * 4 + 3) = -1.0f;
			for (; pp != -1 && W.get(pp, c) < 0; pp = (long)W.s(pp * 4 + 1)) W.put(pp, c, cur);
			if (pp == -1) {
				W.s(cur * 4 + 1) = 0.0f;
			} else {
				const long qs = W.get(pp, c);
				if (__fadd_rn(W.s(pp * 4), 1.0f) == W.s(qs * 4)) {
					W.s(cur * 4 + 1) = (float)qs;
				} else {
					const long cl = nst++;
					W.s(cl * 4) = __fadd_rn(W.s(pp * 4), 1.0f), W.s(cl * 4 + 1) = W.s(qs * 4 + 1), W.s(cl * 4 + 2) = W.s(qs * 4 + 2),
						 W.s(cl * 4 + 3) = -1.0f;
					for (long h = (long)W.s(qs * 4 + 3); h >= 0; h = (long)W.e(h * 4 + 3)) W.put(cl, (long)W.e(h * 4 + 1), (long)W.e(h * 4 + 2));
					for (; pp != -1 && W.get(pp, c) == qs; pp = (long)W.s(pp * 4 + 1)) W.put(pp, c, cl);
					W.s(qs * 4 + 1) = (float)cl, W.s(cur * 4 + 1) = (float)cl;
					if (m == qs && l <= (long)W.s(cl * 4)) m = cl;
				}
			}
			last = cur;
		}
	}
}

__global__ void __launch_bounds__(VM_ROWS) vm_kernel(const DOp *__restrict__ tape, int ntape,
						    const float *__restrict__ gblob, int nblob, int blob_in_smem, int arena,
						    const float *__restrict__ in, int per, long rows, float *__restrict__ out,
						    int nout, int out_loc, int *__restrict__ steps, int nt,
						    const int *__restrict__ in_loc, const int *__restrict__ in_len, int ninputs,
						    float *__restrict__ gar)
{
	extern __shared__ float sm[];
	float *blob = blob_in_smem ? sm : (float *)gblob;
	float *arsm = sm + (blob_in_smem ? (nblob + 3) / 4 * 4 : 0);
	if (blob_in_smem)
		for (int i = threadIdx.x; i < nblob; i += blockDim.x) sm[i] = gblob[i];
	// per-thread arena base: column threadIdx.x of a [arena][VM_ROWS] table
	float *ar = gar ? gar + (long)blockIdx.x * arena * VM_ROWS + threadIdx.x : arsm + threadIdx.x;
	__syncthreads();
	const long row = (long)blockIdx.x * VM_ROWS + threadIdx.x;
	const bool live = row < rows;
	// inputs -> arena
	if (live)
		for (int i = 0, o = 0; i < ninputs; i++) {
			const float *src = in + row * per + o;
			float *dst = ar + (long)in_loc[i] * VM_ROWS;
			for (int e = 0; e < in_len[i]; e++) dst[(long)e * VM_ROWS] = src[e];
			o += in_len[i];
		}
	unsigned done = live ? 0u : 1u << VM_MAXDEPTH; // bit d: halted in the loop at depth d
	int it[VM_MAXDEPTH];
	float surv[VM_MAXDEPTH];
	for (int pc = 0; pc < ntape;) {
		const DOp &op = tape[pc];
		const bool act = done == 0;
		switch (op.code) {
		case D_CONST:
			if (act) ar[(long)op.out * VM_ROWS] = op.f;
			break;
		case D_BIN:
			if (act) {
				Loc o = loc(op.out, ar, blob), a = loc(op.a, ar, blob), b = loc(op.b, ar, blob);
				if (op.rank == 0) { // equal shapes or scalars: sa/sb[0] are 1 or 0
					for (int e = 0; e < op.n; e++)
						o.p[(long)e * o.st] = bin_op(op.sub, a.p[(long)e * op.sa[0] * a.st], b.p[(long)e * op.sb[0] * b.st]);
				} else {
					for (int e = 0; e < op.n; e++) {
						int rem = e, ia = 0, ib = 0;
						for (int d = op.rank - 1; d >= 0; d--) {
							int idx = rem % op.dims[d];
							rem /= op.dims[d];
							ia += idx * op.sa[d];
							ib += idx * op.sb[d];
						}
						o.p[(long)e * o.st] = bin_op(op.sub, a.p[(long)ia * a.st], b.p[(long)ib * b.st]);
					}
				}
			}
			break;
		case D_UN:
			if (act) {
				Loc o = loc(op.out, ar, blob), a = loc(op.a, ar, blob);
				for (int e = 0; e < op.n; e++) o.p[(long)e * o.st] = un_op(op.sub, a.p[(long)e * a.st]);
			}
			break;
		case D_MATMUL:
			if (act) vm_matmul(op, ar, blob);
			break;
		case D_ROW:
			if (act) {
				Loc o = loc(op.out, ar, blob), a = loc(op.a, ar, blob);
				for (int r = 0; r < op.m; r++) {
					const long base = (long)r * op.k;
					if (op.sub == TG_CUDA_OP_SOFTMAX) { // runtime/tg_rt.h:154-164
						float mx = a.p[base * a.st], s = 0.0f;
						for (int i = 1; i < op.k; i++) {
							float v = a.p[(base + i) * a.st];
							if (v > mx) mx = v;
						}
						for (int i = 0; i < op.k; i++) {
							float y = expf(__fsub_rn(a.p[(base + i) * a.st], mx));
							o.p[(base + i) * o.st] = y;
							s = __fadd_rn(s, y);
						}
						for (int i = 0; i < op.k; i++) o.p[(base + i) * o.st] = __fdiv_rn(o.p[(base + i) * o.st], s);
					} else { // rmsnorm, runtime/tg_rt.h:165-175
						float s = 0.0f;
						for (int i = 0; i < op.k; i++) {
							float x = a.p[(base + i) * a.st];
							s = __fadd_rn(s, __fmul_rn(x, x));
						}
						float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)op.k), 1e-6f)));
						for (int i = 0; i < op.k; i++) o.p[(base + i) * o.st] = __fmul_rn(a.p[(base + i) * a.st], inv);
					}
				}
			}
			break;
		case D_RED:
			if (act) {
				Loc o = loc(op.out, ar, blob), a = loc(op.a, ar, blob);
				float s = 0.0f;
				for (int e = 0; e < op.n; e++) s = __fadd_rn(s, a.p[(long)e * a.st]);
				o.p[0] = op.sub == TG_CUDA_OP_MEAN ? __fdiv_rn(s, (float)op.n) : s;
			}
			break;
		case D_TRANS:
			if (act) {
				Loc o = loc(op.out, ar, blob), a = loc(op.a, ar, blob);
				for (int g = 0; g < op.g; g++)
					for (int i = 0; i < op.m; i++)
						for (int j = 0; j < op.k; j++)
							o.p[((long)g * op.m * op.k + (long)j * op.m + i) * o.st] = a.p[((long)g * op.m * op.k + (long)i * op.k + j) * a.st];
			}
			break;
		case D_OUTER:
			if (act) {
				Loc o = loc(op.out, ar, blob), a = loc(op.a, ar, blob), b = loc(op.b, ar, blob);
				for (int i = 0; i < op.m; i++)
					for (int j = 0; j < op.k; j++) o.p[((long)i * op.k + j) * o.st] = __fmul_rn(a.p[(long)i * a.st], b.p[(long)j * b.st]);
			}
			break;
		case D_TAKE: // runtime/tg_rt.h:316-322, rows of a [d, h] by rounded index
			if (act) {
				Loc o = loc(op.out, ar, blob), a = loc(op.a, ar, blob), b = loc(op.b, ar, blob);
				for (int i = 0; i < op.m; i++) {
					float r = floorf(__fadd_rn(b.p[(long)i * b.st], 0.5f));
					int t = r >= 0.0f && r < (float)op.k ? (int)r : -1;
					for (int j = 0; j < op.nn; j++)
						o.p[((long)i * op.nn + j) * o.st] = t >= 0 ? a.p[((long)t * op.nn + j) * a.st] : 0.0f;
				}
			}
			break;
		case D_SPMM:
			if (act) vm_spmm(op, ar, blob);
			break;
		case D_TOPK:
			if (act) vm_topk(op, ar, blob);
			break;
		case D_MEMSCAN:
			if (act) vm_memscan(op, ar, blob);
			break;
		case D_SUFMATCH:
			if (act) vm_sufmatch(op, ar, blob);
			break;
		case D_SUMTO:
			if (act) vm_sum_to(op, ar, blob);
			break;
		case D_TAKE_T:
			if (act) vm_take_t(op, ar, blob);
			break;
		case D_MEMSCAN_T:
			if (act) vm_memscan_t(op, ar, blob);
			break;
		case D_COPY:
			if (act && op.out != op.a) {
				Loc o = loc(op.out, ar, blob), a = loc(op.a, ar, blob);
				for (int e = 0; e < op.n; e++) o.p[(long)e * o.st] = a.p[(long)e * a.st];
			}
			break;
		case D_THINK_BEGIN: // copy init into the state, reset this depth's counters
			if (act) {
				Loc o = loc(op.out, ar, blob), a = loc(op.a, ar, blob);
				if (op.out != op.a)
					for (int e = 0; e < op.n; e++) o.p[(long)e * o.st] = a.p[(long)e * a.st];
				it[op.depth] = 0;
				surv[op.depth] = 1.0f;
			}
			break;
		case D_THINK_END: { // src/vm.c:389-409
			if (act) {
				Loc o = loc(op.out, ar, blob), y = loc(op.yield, ar, blob);
				it[op.depth]++;
				float d = 0.0f;
				for (int e = 0; e < op.n; e++) {
					float v = fabsf(__fsub_rn(y.p[(long)e * y.st], o.p[(long)e * o.st]));
					if (v > d) d = v;
				}
				for (int e = 0; e < op.n; e++) o.p[(long)e * o.st] = y.p[(long)e * y.st];
				bool stop = it[op.depth] >= op.maxit;
				if (op.eps >= 0 && d <= op.eps) stop = true;
				if (op.halt != INT_MIN) {
					float p = loc(op.halt, ar, blob).p[0];
					surv[op.depth] = __fmul_rn(surv[op.depth], __fsub_rn(1.0f, p < 0.0f ? 0.0f : p > 1.0f ? 1.0f : p));
					if (__fsub_rn(1.0f, surv[op.depth]) > op.hthr) stop = true;
				}
				if (stop) {
					done |= 1u << op.depth;
					if (live && op.tid < nt) steps[row * nt + op.tid] = it[op.depth];
				}
			}
			if (__any_sync(0xffffffffu, done == 0)) {
				pc = op.target;
				continue;
			}
			done &= ~(1u << op.depth);
			break;
		}
		case D_SCAN_BEGIN: // carries <- init (cnt copies listed in the following D_COPY ops)
			it[op.depth] = 0;
			break;
		case D_SCAN_SLICE: // sub bit 0: reverse; bit 1 clear: xt <- row t of x, set: row t of ys <- y
			if (act) {
				int t = (op.sub & 1) ? op.len - 1 - it[op.depth] : it[op.depth];
				Loc o = loc(op.out, ar, blob), a = loc(op.a, ar, blob);
				if (op.sub & 2)
					for (int e = 0; e < op.n; e++) o.p[((long)t * op.n + e) * o.st] = a.p[(long)e * a.st];
				else
					for (int e = 0; e < op.n; e++) o.p[(long)e * o.st] = a.p[((long)t * op.n + e) * a.st];
			}
			break;
		case D_SCAN_END: // ys[t] <- y (sub-ops follow as D_COPY with a per-step offset)
			it[op.depth]++;
			if (it[op.depth] < op.len) {
				pc = op.target;
				continue;
			}
			if (act && op.tid >= 0 && op.tid < nt && live) steps[row * nt + op.tid] = op.len;
			break;
		}
		pc++;
	}
	if (live) {
		Loc o = loc(out_loc, ar, blob);
		for (int e = 0; e < nout; e++) out[row * nout + e] = o.p[(long)e * o.st];
	}
}

// ---- host: program -> tape -------------------------------------------------------------------

// Pinned host memory, grown on demand.
struct HostBuf {
	void *p = nullptr;
	size_t bytes = 0;
	HostBuf() = default;
	HostBuf(const HostBuf &) = delete;
	HostBuf &operator=(const HostBuf &) = delete;
	~HostBuf()
	{
		if (p) cudaFreeHost(p);
	}
	int ensure(size_t n)
	{
		if (n <= bytes) return TG_CUDA_OK;
		if (p) cudaFreeHost(p);
		p = nullptr;
		bytes = 0;
		if (cudaHostAlloc(&p, n, cudaHostAllocDefault) != cudaSuccess) {
			cudaGetLastError();
			return set_err(TG_CUDA_ENOMEM, "cudaHostAlloc(%zu) failed", n);
		}
		bytes = n;
		return TG_CUDA_OK;
	}
};

// One stage of the host-buffer pipeline of tg_cuda_batch: pinned staging, the device
// buffers of one chunk of rows and the stream that carries it.
struct Slot {
	HostBuf hin, hout, hsteps;
	DevBuf din, dout, dsteps;
	cudaStream_t st = nullptr;
	cudaEvent_t done = nullptr;
	long lo = 0, cnt = 0; // rows of the chunk in flight (offset within the device's shard)
	bool busy = false;
	Slot() = default;
	Slot(const Slot &) = delete;
	Slot &operator=(const Slot &) = delete;
	~Slot()
	{
		if (done) cudaEventDestroy(done);
		if (st) cudaStreamDestroy(st);
	}
};

struct Model {
	Prog prog;
	struct PerDev {
		DevBuf tape, blob, inloc, inlen, gar;
		long gar_rows = 0;
		JitModule jit; // the program's specialised kernel on this device
		Slot slot[3];  // tg_cuda_batch pipeline: two with staging, three straight from the caller's buffers
		std::mutex mu; // one tg_cuda_batch at a time on this device's slots
	};
	std::vector<std::unique_ptr<PerDev>> dev;
	bool blob_in_smem = true;
	size_t smem = 0;
	bool global_arena = false;
	bool jit = false;    // rows run on the specialised kernel (else on vm_kernel)
	std::string jit_why; // why not, when not
};

static long numel(const tg_cuda_value &v)
{
	long n = 1;
	for (int i = 0; i < v.rank; i++) n *= v.dim[i];
	return n;
}

struct Compiler {
	const tg_cuda_program *p;
	Prog *out;
	std::vector<int> slot;     // arena slot of each temporary
	std::vector<int> pslot;    // blob offset of each param (f32 values or exact codes)
	std::vector<int> sslot;    // blob offset of each quantized param's scales
	std::vector<int> inloc;    // arena slot of each input value
	std::string err;
	int status = TG_CUDA_OK;

	int fail(int st, const char *msg, int v = -1)
	{
		if (status == TG_CUDA_OK) {
			status = st;
			char b[256];
			snprintf(b, sizeof b, "%s%s%d", msg, v >= 0 ? " (instruction " : "", v);
			err = b;
			if (v >= 0) err += ")";
		}
		return st;
	}

	int L(int v) // location of a value
	{
		const tg_cuda_value &x = p->val[v];
		if (x.kind == TG_CUDA_PARAM || x.kind == TG_CUDA_STATE) return -(pslot[v] + 1);
		if (x.kind == TG_CUDA_INPUT) return inloc[v];
		return slot[v];
	}
};

// Liveness over a linear numbering of instructions, a loop body's reads of outer values
// extended to the loop end (the algorithm of src/plan.c: lifetimes, then greedy by size).
struct Life {
	int def = -1, last = -1;
};

static void number_ins(const tg_cuda_program *p, int from, int cnt, int &pos, std::vector<int> &beg, std::vector<int> &end)
{
	for (int i = from; i < from + cnt; i++) {
		const tg_cuda_ins &in = p->ins[i];
		beg[i] = pos++;
		bool loop = in.op == TG_CUDA_OP_THINK || in.op == TG_CUDA_OP_SCAN;
		if (loop) number_ins(p, in.body, in.nbody, pos, beg, end);
		end[i] = loop ? pos++ : beg[i];
	}
}

static void lives(const tg_cuda_program *p, int from, int cnt, const std::vector<int> &beg, const std::vector<int> &end,
		  std::vector<int> &loops, std::vector<Life> &life)
{
	auto use = [&](int v, int at) {
		if (v < 0 || p->val[v].kind != TG_CUDA_TMP) return;
		int last = at;
		for (int li : loops)
			if (life[v].def < beg[li] && end[li] > last) last = end[li];
		if (last > life[v].last) life[v].last = last;
	};
	auto def = [&](int v, int at) {
		if (v < 0 || p->val[v].kind != TG_CUDA_TMP) return;
		if (life[v].def < 0 || at < life[v].def) life[v].def = at;
		if (life[v].last < at) life[v].last = at;
	};
	for (int i = from; i < from + cnt; i++) {
		const tg_cuda_ins &in = p->ins[i];
		if (in.op == TG_CUDA_OP_THINK) {
			use(in.init, beg[i]);
			def(in.out, beg[i]);
			loops.push_back(i);
			lives(p, in.body, in.nbody, beg, end, loops, life);
			use(in.yield, end[i]);
			if (in.halt >= 0) use(in.halt, end[i]);
			loops.pop_back();
			use(in.out, end[i]);
		} else if (in.op == TG_CUDA_OP_SCAN) {
			const tg_cuda_scan &s = p->scans[in.scan];
			for (int k = 0; k < s.nc; k++) {
				use(s.init[k], beg[i]);
				def(s.c[k], beg[i]);
			}
			for (int j = 0; j < s.nx; j++) {
				use(s.x[j], end[i]);
				def(s.xt[j], beg[i]);
			}
			for (int y = 0; y < s.ny; y++) def(s.ys[y], beg[i]);
			loops.push_back(i);
			lives(p, in.body, in.nbody, beg, end, loops, life);
			for (int k = 0; k < s.nc; k++) use(s.next[k], end[i]);
			for (int y = 0; y < s.ny; y++) use(s.y[y], end[i]);
			loops.pop_back();
			for (int k = 0; k < s.nc; k++) use(s.c[k], end[i]);
			for (int j = 0; j < s.nx; j++) use(s.xt[j], end[i]);
			for (int y = 0; y < s.ny; y++) use(s.ys[y], end[i]);
		} else {
			for (int j = 0; j < in.na; j++) use(in.a[j], beg[i]);
			def(in.out, beg[i]);
		}
	}
}

static int plan_arena(Compiler &C)
{
	const tg_cuda_program *p = C.p;
	std::vector<int> beg(p->nins, 0), end(p->nins, 0);
	int pos = 0;
	number_ins(p, 0, p->ntop, pos, beg, end);
	std::vector<Life> life(p->nval);
	std::vector<int> loops;
	lives(p, 0, p->ntop, beg, end, loops, life);
	if (p->val[p->output].kind == TG_CUDA_TMP) life[p->output].last = pos;
	// inputs occupy their own slots for the whole run
	int top = 0;
	C.inloc.assign(p->nval, -1);
	for (int i = 0; i < p->ninputs; i++) {
		int v = p->inputs[i];
		C.inloc[v] = top;
		top += (int)((numel(p->val[v]) + 3) / 4 * 4);
	}
	std::vector<int> order;
	for (int v = 0; v < p->nval; v++)
		if (p->val[v].kind == TG_CUDA_TMP && life[v].def >= 0) order.push_back(v);
	auto asz = [&](int v) { return (int)((numel(p->val[v]) + 3) / 4 * 4); };
	std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
		if (asz(a) != asz(b)) return asz(a) > asz(b);
		return life[a].def < life[b].def;
	});
	C.slot.assign(p->nval, -1);
	std::vector<int> placed;
	int arena = top;
	for (int v : order) {
		std::vector<std::pair<int, int>> busy; // [off, off+size) of overlapping placed values
		for (int w : placed)
			if (life[w].def <= life[v].last && life[v].def <= life[w].last) busy.push_back({ C.slot[w], C.slot[w] + asz(w) });
		std::sort(busy.begin(), busy.end());
		int off = top, sz = asz(v);
		for (auto &b : busy) {
			if (off + sz <= b.first) break;
			if (b.second > off) off = b.second;
		}
		C.slot[v] = off;
		arena = std::max(arena, off + sz);
		placed.push_back(v);
	}
	C.out->arena = arena ? arena : 4;
	return TG_CUDA_OK;
}

static int emit_block(Compiler &C, int from, int cnt, int depth);

// The iteration space of sum_to (src/util.c:172-212, bcast_desc with one operand): x's
// shape with its size-1 axes dropped and adjacent axes merged where the target's strides
// allow (both broadcast, or contiguous); rank, dims and the target's strides into d.
static void sumto_desc(const tg_cuda_value &x, const tg_cuda_value &tgt, DOp &d)
{
	const int r = x.rank;
	int st[4];
	long acc = 1;
	for (int i = r - 1; i >= 0; i--) {
		const int j = i - (r - tgt.rank), n = j >= 0 ? tgt.dim[j] : 1;
		st[i] = n == 1 ? 0 : (int)acc;
		acc *= n;
	}
	int nr = 0;
	for (int i = 0; i < r; i++) {
		if (x.dim[i] == 1) continue;
		if (nr > 0) {
			const int p = nr - 1;
			if ((d.sa[p] == 0 && st[i] == 0) || (st[i] != 0 && (long)d.sa[p] == (long)st[i] * x.dim[i])) {
				d.dims[p] *= x.dim[i];
				d.sa[p] = st[i];
				continue;
			}
		}
		d.dims[nr] = x.dim[i], d.sa[nr] = st[i], nr++;
	}
	if (nr == 0) d.dims[0] = 1, d.sa[0] = 0, nr = 1;
	d.rank = nr;
}

static void bcast(const tg_cuda_value &o, const tg_cuda_value &a, const tg_cuda_value &b, DOp &d)
{
	long n = numel(o), na = numel(a), nb = numel(b);
	d.n = (int)n;
	if ((na == n || na == 1) && (nb == n || nb == 1)) {
		d.rank = 0;
		d.sa[0] = na == n ? 1 : 0;
		d.sb[0] = nb == n ? 1 : 0;
		return;
	}
	d.rank = o.rank;
	for (int i = 0; i < 4; i++) d.dims[i] = i < o.rank ? o.dim[i] : 1;
	long st = 1;
	for (int x = 0; x < 4; x++) d.sa[x] = d.sb[x] = 0;
	for (int i = a.rank - 1; i >= 0; i--) {
		int od = o.rank - a.rank + i;
		d.sa[od] = a.dim[i] == 1 ? 0 : (int)st;
		st *= a.dim[i];
	}
	st = 1;
	for (int i = b.rank - 1; i >= 0; i--) {
		int od = o.rank - b.rank + i;
		d.sb[od] = b.dim[i] == 1 ? 0 : (int)st;
		st *= b.dim[i];
	}
}

static int emit_ins(Compiler &C, int idx, int depth)
{
	const tg_cuda_program *p = C.p;
	const tg_cuda_ins &in = p->ins[idx];
	std::vector<DOp> &T = C.out->tape;
	DOp d;
	memset(&d, 0, sizeof d);
	d.out = in.out >= 0 ? C.L(in.out) : 0;
	d.a = in.na > 0 ? C.L(in.a[0]) : 0;
	d.b = in.na > 1 ? C.L(in.a[1]) : 0;
	const tg_cuda_value &vo = p->val[in.out];
	switch (in.op) {
	case TG_CUDA_OP_CONST:
		d.code = D_CONST;
		d.f = in.k;
		T.push_back(d);
		return 0;
	case TG_CUDA_OP_ADD: case TG_CUDA_OP_SUB: case TG_CUDA_OP_MUL: case TG_CUDA_OP_DIV: case TG_CUDA_OP_MAX: case TG_CUDA_OP_MIN:
		d.code = D_BIN;
		d.sub = in.op;
		bcast(vo, p->val[in.a[0]], p->val[in.a[1]], d);
		T.push_back(d);
		return 0;
	case TG_CUDA_OP_NEG: case TG_CUDA_OP_TANH: case TG_CUDA_OP_RELU: case TG_CUDA_OP_SIGMOID: case TG_CUDA_OP_EXP:
	case TG_CUDA_OP_SQRT: case TG_CUDA_OP_GELU: case TG_CUDA_OP_SILU: case TG_CUDA_OP_SOFTPLUS: case TG_CUDA_OP_LOG:
	case TG_CUDA_OP_STEP: case TG_CUDA_OP_SIN: case TG_CUDA_OP_COS: case TG_CUDA_OP_FLOOR:
		d.code = D_UN;
		d.sub = in.op;
		d.n = (int)numel(vo);
		T.push_back(d);
		return 0;
	case TG_CUDA_OP_MATMUL: { // src/ops.c:60-73 dims, src/vm.c:262-290 dispatch, src/ops.c:310-320 axes
		const tg_cuda_value &A = p->val[in.a[0]], &B = p->val[in.a[1]];
		int g = A.rank == 3 && B.rank == 3 ? A.dim[0] : 1;
		d.code = D_MATMUL;
		d.m = A.rank == 3 ? (g > 1 || B.rank == 3 ? A.dim[1] : A.dim[0] * A.dim[1]) : A.rank == 2 ? A.dim[0] : 1;
		d.k = A.dim[A.rank - 1];
		d.nn = B.rank >= 2 ? B.dim[B.rank - 1] : 1;
		d.g = g;
		if (g == 1) {
			bool distinct = in.a[0] != in.a[1];
			if (A.qbits && A.rank == 2 && distinct && A.qaxis == 0) {
				d.scale = 1;
				d.c = -(C.sslot[in.a[0]] + 1);
			} else if (B.qbits && B.rank == 2 && distinct && B.qaxis == 1) {
				d.scale = 2;
				d.c = -(C.sslot[in.a[1]] + 1);
			}
			// a quantized param used on another axis reads its dequantized values
			if (A.qbits && d.scale != 1) d.a = -(C.pslot[in.a[0]] + 1 + (int)numel(A) + A.dim[A.qaxis]);
			if (B.qbits && d.scale != 2) d.b = -(C.pslot[in.a[1]] + 1 + (int)numel(B) + B.dim[B.qaxis]);
		}
		T.push_back(d);
		return 0;
	}
	case TG_CUDA_OP_SOFTMAX: case TG_CUDA_OP_RMSNORM: {
		const tg_cuda_value &x = p->val[in.a[0]];
		d.code = D_ROW;
		d.sub = in.op;
		d.k = x.rank ? x.dim[x.rank - 1] : 1;
		d.m = (int)(numel(x) / d.k);
		T.push_back(d);
		return 0;
	}
	case TG_CUDA_OP_SUM: case TG_CUDA_OP_MEAN:
		d.code = D_RED;
		d.sub = in.op;
		d.n = (int)numel(p->val[in.a[0]]);
		T.push_back(d);
		return 0;
	case TG_CUDA_OP_TRANSPOSE: {
		const tg_cuda_value &x = p->val[in.a[0]];
		d.code = D_TRANS;
		d.g = x.rank == 3 ? x.dim[0] : 1;
		d.m = x.dim[x.rank - 2];
		d.k = x.dim[x.rank - 1];
		T.push_back(d);
		return 0;
	}
	case TG_CUDA_OP_OUTER:
		d.code = D_OUTER;
		d.m = (int)numel(p->val[in.a[0]]);
		d.k = (int)numel(p->val[in.a[1]]);
		T.push_back(d);
		return 0;
	case TG_CUDA_OP_TAKE: {
		const tg_cuda_value &w = p->val[in.a[0]];
		d.code = D_TAKE;
		d.k = w.dim[0];
		d.nn = (int)(numel(w) / w.dim[0]);
		d.m = p->val[in.a[1]].dim[0];
		if (w.qbits) d.a = -(C.pslot[in.a[0]] + 1 + (int)numel(w) + w.dim[w.qaxis]);
		T.push_back(d);
		return 0;
	}
	case TG_CUDA_OP_SPMM: { // src/vm.c:307-313, src/ops.c:82-88 spmm_dims
		const tg_cuda_value &X = p->val[in.a[0]], &W = p->val[in.a[1]];
		d.code = D_SPMM;
		d.m = X.rank == 3 ? X.dim[0] : 1;
		d.k = X.dim[X.rank - 2];
		d.g = W.dim[0];
		d.nn = W.dim[1];
		if (W.qbits && W.qaxis == 0) { // the table's exact codes, times value * scale of the row
			d.scale = 1;
			d.b = -(C.pslot[in.a[1]] + 1);
			d.c = -(C.sslot[in.a[1]] + 1);
		} else if (W.qbits) { // quantized on the other axis: its dequantized values
			d.b = -(C.pslot[in.a[1]] + 1 + (int)numel(W) + W.dim[W.qaxis]);
		}
		T.push_back(d);
		return 0;
	}
	case TG_CUDA_OP_TOPK: { // src/vm.c:340-345 with row_dims, src/ops.c:90-94
		const tg_cuda_value &X = p->val[in.a[0]];
		d.code = D_TOPK;
		d.k = X.rank ? X.dim[X.rank - 1] : 1;
		d.m = (int)(numel(X) / d.k);
		d.nn = vo.dim[vo.rank - 1];
		T.push_back(d);
		return 0;
	}
	case TG_CUDA_OP_MEMSCAN: { // src/vm.c:351-357, src/util.c:455-467 memscan_dims
		const tg_cuda_value &M0 = p->val[in.a[0]], &P = p->val[in.a[1]];
		d.code = D_MEMSCAN;
		d.c = C.L(in.a[2]);
		d.m = P.dim[0] * P.dim[1];
		d.k = 2 * P.dim[2] + (P.dim[3] == 4);
		d.nn = M0.dim[0];
		d.g = M0.dim[1];
		T.push_back(d);
		return 0;
	}
	case TG_CUDA_OP_SUM_TO: // src/vm.c:358-363
		d.code = D_SUMTO;
		d.n = (int)numel(vo);
		sumto_desc(p->val[in.a[0]], p->val[in.a[1]], d);
		T.push_back(d);
		return 0;
	case TG_CUDA_OP_TAKE_T: { // src/vm.c:320-323: take_t(r, g, w) -> the shape of w
		const tg_cuda_value &W = p->val[in.a[2]];
		d.code = D_TAKE_T;
		d.m = p->val[in.a[0]].dim[0];
		d.k = W.dim[0];
		d.nn = (int)(numel(W) / W.dim[0]);
		T.push_back(d);
		return 0;
	}
	case TG_CUDA_OP_MEMSCAN_T: { // src/vm.c:351-357, src/util.c:455-467 memscan_dims
		const tg_cuda_value &Y = p->val[in.a[0]], &PV = p->val[in.a[1]];
		d.code = D_MEMSCAN_T;
		d.c = C.L(in.a[2]);
		d.g = Y.dim[1];
		d.m = PV.dim[0] * PV.dim[1];
		d.k = (PV.dim[2] - d.g) / 4;
		d.nn = Y.dim[0] - 2 * d.m;
		d.n = (int)numel(vo);
		T.push_back(d);
		return 0;
	}
	case TG_CUDA_OP_SUFMATCH: { // src/vm.c:346-350
		const tg_cuda_value &X = p->val[in.a[0]];
		d.code = D_SUFMATCH;
		d.m = X.dim[0];
		d.k = X.rank == 2 ? X.dim[1] : 1;
		T.push_back(d);
		return 0;
	}
	case TG_CUDA_OP_RESHAPE:
		d.code = D_COPY;
		d.n = (int)numel(vo);
		if (p->val[in.a[0]].qbits) d.a = -(C.pslot[in.a[0]] + 1 + (int)numel(p->val[in.a[0]]) + p->val[in.a[0]].dim[p->val[in.a[0]].qaxis]);
		T.push_back(d);
		return 0;
	case TG_CUDA_OP_THINK: {
		if (depth >= VM_MAXDEPTH) return C.fail(TG_CUDA_EUNSUPPORTED, "think/scan nesting deeper than 4", idx);
		C.out->max_depth = std::max(C.out->max_depth, depth + 1);
		d.code = D_THINK_BEGIN;
		d.a = C.L(in.init);
		d.n = (int)numel(vo);
		d.depth = depth;
		T.push_back(d);
		int body = (int)T.size();
		if (emit_block(C, in.body, in.nbody, depth + 1)) return C.status;
		DOp e;
		memset(&e, 0, sizeof e);
		e.code = D_THINK_END;
		e.out = C.L(in.out);
		e.yield = C.L(in.yield);
		e.n = (int)numel(vo);
		e.depth = depth;
		e.target = body;
		e.maxit = in.maxit;
		e.eps = in.eps;
		e.tid = in.tid;
		e.halt = in.halt >= 0 ? C.L(in.halt) : INT_MIN;
		e.hthr = in.hthr;
		T.push_back(e);
		return 0;
	}
	case TG_CUDA_OP_SCAN: {
		if (depth >= VM_MAXDEPTH) return C.fail(TG_CUDA_EUNSUPPORTED, "think/scan nesting deeper than 4", idx);
		C.out->max_depth = std::max(C.out->max_depth, depth + 1);
		const tg_cuda_scan &s = p->scans[in.scan];
		for (int k = 0; k < s.nc; k++) { // carries <- init
			DOp c;
			memset(&c, 0, sizeof c);
			c.code = D_COPY;
			c.out = C.L(s.c[k]);
			c.a = C.L(s.init[k]);
			c.n = (int)numel(p->val[s.c[k]]);
			T.push_back(c);
		}
		DOp b0;
		memset(&b0, 0, sizeof b0);
		b0.code = D_SCAN_BEGIN;
		b0.depth = depth;
		T.push_back(b0);
		int body = (int)T.size();
		for (int j = 0; j < s.nx; j++) {
			DOp c;
			memset(&c, 0, sizeof c);
			c.code = D_SCAN_SLICE;
			c.sub = s.reverse;
			c.len = s.T;
			c.out = C.L(s.xt[j]);
			c.a = C.L(s.x[j]);
			c.n = (int)numel(p->val[s.xt[j]]);
			c.depth = depth;
			T.push_back(c);
		}
		if (emit_block(C, in.body, in.nbody, depth + 1)) return C.status;
		// ys[t] <- y: a slice op in reverse (out is the stack): encode as a strided copy
		for (int y = 0; y < s.ny; y++) {
			DOp c;
			memset(&c, 0, sizeof c);
			c.code = D_SCAN_SLICE;
			c.sub = s.reverse | 2; // bit 1: write into the stack
			c.len = s.T;
			c.out = C.L(s.ys[y]);
			c.a = C.L(s.y[y]);
			c.n = (int)numel(p->val[s.y[y]]);
			c.depth = depth;
			T.push_back(c);
		}
		for (int k = 0; k < s.nc; k++) {
			DOp c;
			memset(&c, 0, sizeof c);
			c.code = D_COPY;
			c.out = C.L(s.c[k]);
			c.a = C.L(s.next[k]);
			c.n = (int)numel(p->val[s.c[k]]);
			T.push_back(c);
		}
		DOp e;
		memset(&e, 0, sizeof e);
		e.code = D_SCAN_END;
		e.depth = depth;
		e.target = body;
		e.len = s.T;
		e.tid = s.tid;
		T.push_back(e);
		return 0;
	}
	}
	return C.fail(TG_CUDA_EUNSUPPORTED, "op not implemented by the device executor", idx);
}

static int emit_block(Compiler &C, int from, int cnt, int depth)
{
	for (int i = from; i < from + cnt; i++)
		if (emit_ins(C, i, depth)) return C.status;
	return 0;
}

// ---- program verification -------------------------------------------------------------------
//
// tg_cuda_load trusts nothing about the program it is handed. Every index is in range, every
// instruction belongs to exactly one block, and every declared shape is the one its operands
// give by the reference's own rules: op_infer (src/ops.c:96-295) and the instruction, think
// and scan checks of its TGIR reader (src/ir.c:258-447). So no kernel indexes past a value,
// whatever the caller passes.

struct VShape {
	int rank = 0, dim[4] = { 1, 1, 1, 1 };
};

static VShape vshape(const tg_cuda_value &v)
{
	VShape s;
	s.rank = v.rank;
	for (int d = 0; d < v.rank && d < 4; d++) s.dim[d] = v.dim[d];
	return s;
}

static bool veq(const VShape &a, const VShape &b)
{
	if (a.rank != b.rank) return false;
	for (int d = 0; d < a.rank; d++)
		if (a.dim[d] != b.dim[d]) return false;
	return true;
}

static long vnumel(const VShape &s)
{
	long n = 1;
	for (int d = 0; d < s.rank; d++) n *= s.dim[d];
	return n;
}

static std::string vstr(const VShape &s)
{
	std::string r = "(f32";
	for (int d = 0; d < s.rank; d++) r += " " + std::to_string(s.dim[d]);
	return r + ")";
}

// src/util.c:154-165: dimensions compared from the right, each pair equal or one of them 1
static bool vbroadcast(const VShape &a, const VShape &b, VShape &o)
{
	o = VShape();
	o.rank = std::max(a.rank, b.rank);
	for (int i = 1; i <= o.rank; i++) {
		int x = i <= a.rank ? a.dim[a.rank - i] : 1, y = i <= b.rank ? b.dim[b.rank - i] : 1;
		if (x != y && x != 1 && y != 1) return false;
		o.dim[o.rank - i] = x == 1 ? y : x;
	}
	return true;
}

// operand counts of the reference's op table (src/ops.c:7-50), in TG_CUDA_OP_* order
static const signed char kArity[TG_CUDA_OP_COUNT] = {
	0, 2, 2, 2, 2, 2, 2, // const add sub mul div max min
	1, 1, 1, 1, 1, 1, 1, // neg tanh relu sigmoid exp sqrt gelu
	1, 1, 1, 2, 1, 1,    // silu softplus log matmul softmax rmsnorm
	1, 1, 1, 2, 1, 2,    // sum mean transpose outer step spmm
	3, 3, 2, 2, 3, 3,    // spmm_t spmm_dx active take take_t spmm_tc
	1, 1, 1, 1, 2, 1,    // sin cos reshape floor sum_to topk
	3, 3, 1, 0, 0        // memscan memscan_t sufmatch think scan
};

// sufmatch's output length (src/util.c:469-474): 2 T n results, then the automaton's workspace
static long vsufmatch_size(long T, long n)
{
	long h = 16;
	while (h < 6 * T + 6) h *= 2;
	return 2 * T * n + 4 * (2 * T + 2) + 4 * h;
}

// memscan_t's output length (runtime/tg_rt.h:524-532, tg_memscan_layout)
static long vmemscan_t_size(long tn, long k, long rows, long dv)
{
	long np = tn * k * 4, L = dv % 4 == 0 ? dv : dv % 2 == 0 ? 2 * dv : 4 * dv;
	long o1 = (np + dv - 1) / dv * dv, o2 = o1 + rows * dv, o3 = o2 + tn * dv, end = o3 + rows * dv;
	return (end + L - 1) / L * L;
}

// The shape a value op yields from its operands' shapes (src/ops.c:96-295), or false with err.
static bool vinfer(int op, const VShape *a, VShape &o, std::string &err)
{
	o = VShape();
	switch (op) {
	case TG_CUDA_OP_ADD: case TG_CUDA_OP_SUB: case TG_CUDA_OP_MUL: case TG_CUDA_OP_DIV: case TG_CUDA_OP_MAX:
	case TG_CUDA_OP_MIN:
		if (vbroadcast(a[0], a[1], o)) return true;
		err = "shape mismatch " + vstr(a[0]) + " vs " + vstr(a[1]);
		return false;
	case TG_CUDA_OP_SUM_TO: {
		VShape b;
		if (!vbroadcast(a[0], a[1], b) || !veq(b, a[0])) {
			err = "'sum_to' cannot reduce " + vstr(a[0]) + " to " + vstr(a[1]);
			return false;
		}
		o = a[1];
		return true;
	}
	case TG_CUDA_OP_NEG: case TG_CUDA_OP_TANH: case TG_CUDA_OP_RELU: case TG_CUDA_OP_SIGMOID: case TG_CUDA_OP_EXP:
	case TG_CUDA_OP_SQRT: case TG_CUDA_OP_GELU: case TG_CUDA_OP_SILU: case TG_CUDA_OP_SOFTPLUS: case TG_CUDA_OP_LOG:
	case TG_CUDA_OP_STEP: case TG_CUDA_OP_SIN: case TG_CUDA_OP_COS: case TG_CUDA_OP_FLOOR:
		o = a[0];
		return true;
	case TG_CUDA_OP_MATMUL: {
		int ra = a[0].rank, rb = a[1].rank;
		int ka = ra >= 1 ? a[0].dim[ra - 1] : -1, kb = rb == 3 ? a[1].dim[1] : rb >= 1 ? a[1].dim[0] : -1;
		if (ra < 1 || ra > 3 || rb < 1 || rb > 3 || ka != kb || (rb == 3 && (ra != 3 || a[0].dim[0] != a[1].dim[0]))) {
			err = "'matmul' incompatible operands " + vstr(a[0]) + " @ " + vstr(a[1]);
			return false;
		}
		for (int i = 0; i < ra - 1; i++) o.dim[o.rank++] = a[0].dim[i];
		if (rb >= 2) o.dim[o.rank++] = a[1].dim[rb - 1];
		return true;
	}
	case TG_CUDA_OP_SOFTMAX: case TG_CUDA_OP_RMSNORM:
		if (a[0].rank == 0) {
			err = "row op needs rank >= 1";
			return false;
		}
		o = a[0];
		return true;
	case TG_CUDA_OP_SUM: case TG_CUDA_OP_MEAN:
		return true; // a scalar
	case TG_CUDA_OP_TRANSPOSE:
		if (a[0].rank != 2 && a[0].rank != 3) {
			err = "'transpose' needs rank 2 or 3";
			return false;
		}
		o = a[0];
		o.dim[o.rank - 2] = a[0].dim[a[0].rank - 1];
		o.dim[o.rank - 1] = a[0].dim[a[0].rank - 2];
		return true;
	case TG_CUDA_OP_OUTER:
		if (a[0].rank != 1 || a[1].rank != 1) {
			err = "'outer' needs two vectors, got " + vstr(a[0]) + " and " + vstr(a[1]);
			return false;
		}
		o.rank = 2, o.dim[0] = a[0].dim[0], o.dim[1] = a[1].dim[0];
		return true;
	case TG_CUDA_OP_SPMM: case TG_CUDA_OP_SPMM_T: case TG_CUDA_OP_SPMM_DX: {
		const VShape &x = a[0], &w = a[op == TG_CUDA_OP_SPMM_T ? 2 : 1];
		if ((x.rank != 2 && x.rank != 3) || x.dim[x.rank - 1] != 2 || w.rank != 2) {
			err = "spmm needs sparse rows (K, 2) or (B, K, 2) and a matrix (D, H), got " + vstr(x) + " and " + vstr(w);
			return false;
		}
		VShape y;
		if (x.rank == 3) y.dim[y.rank++] = x.dim[0];
		y.dim[y.rank++] = w.dim[1];
		if (op == TG_CUDA_OP_SPMM) {
			o = y;
			return true;
		}
		if (!veq(a[op == TG_CUDA_OP_SPMM_T ? 1 : 2], y)) {
			err = "spmm gradient does not match the product shape " + vstr(y);
			return false;
		}
		o = op == TG_CUDA_OP_SPMM_T ? w : x;
		return true;
	}
	case TG_CUDA_OP_TAKE_T: {
		VShape want = a[2];
		bool ok = a[0].rank == 1 && want.rank >= 1;
		if (ok) want.dim[0] = a[0].dim[0];
		if (!ok || !veq(a[1], want)) {
			err = "'take_t' needs rows (n), a gradient (n, ...) and the table it scatters into";
			return false;
		}
		o = a[2];
		return true;
	}
	case TG_CUDA_OP_TAKE:
		if (a[0].rank < 1 || a[1].rank != 1) {
			err = "'take' needs a tensor (D, ...) and row indices (n), got " + vstr(a[0]) + " and " + vstr(a[1]);
			return false;
		}
		o = a[0];
		o.dim[0] = a[1].dim[0];
		return true;
	case TG_CUDA_OP_ACTIVE: case TG_CUDA_OP_SPMM_TC: {
		const VShape &x = a[0];
		if ((x.rank != 2 && x.rank != 3) || x.dim[x.rank - 1] != 2) {
			err = "sparse rows (K, 2) or (B, K, 2) expected, got " + vstr(x);
			return false;
		}
		int n = x.rank == 3 ? x.dim[0] * x.dim[1] : x.dim[0];
		if (op == TG_CUDA_OP_ACTIVE) {
			if (a[1].rank < 1) {
				err = "'active' needs the table the rows index";
				return false;
			}
			o.rank = 1, o.dim[0] = n;
			return true;
		}
		const VShape &g = a[1], &r = a[2];
		int gr = x.rank == 3 ? 2 : 1;
		if (g.rank != gr || (gr == 2 && g.dim[0] != x.dim[0]) || r.rank != 1 || r.dim[0] != n) {
			err = "'spmm_tc' operand shapes do not fit";
			return false;
		}
		o.rank = 2, o.dim[0] = n, o.dim[1] = g.dim[g.rank - 1];
		return true;
	}
	case TG_CUDA_OP_MEMSCAN: {
		const VShape &m0 = a[0], &pp = a[1], &v = a[2];
		if (m0.rank != 2 || pp.rank != 4 || (pp.dim[3] != 3 && pp.dim[3] != 4) || v.rank != 3 || v.dim[0] != pp.dim[0] ||
		    v.dim[1] != pp.dim[1] || v.dim[2] != m0.dim[1]) {
			err = "'memscan' needs a memory (rows, dv), entries (T, n, k, 3 or 4) and values (T, n, dv)";
			return false;
		}
		o.rank = 2, o.dim[0] = 2 * pp.dim[0] * pp.dim[1] + m0.dim[0], o.dim[1] = m0.dim[1];
		return true;
	}
	case TG_CUDA_OP_MEMSCAN_T: {
		const VShape &y = a[0], &pv = a[1], &g = a[2];
		long dv = y.rank == 2 ? y.dim[1] : 0, tn = pv.rank == 3 ? (long)pv.dim[0] * pv.dim[1] : 0;
		if (!dv || !tn || !veq(y, g) || y.dim[0] <= 2 * tn || pv.dim[2] <= dv || (pv.dim[2] - dv) % 4) {
			err = "'memscan_t' needs memscan's output, the packed entries and values, and the output's adjoint";
			return false;
		}
		long N = vmemscan_t_size(tn, (pv.dim[2] - dv) / 4, y.dim[0] - 2 * tn, dv);
		if (N > INT32_MAX) {
			err = "'memscan_t' output too large";
			return false;
		}
		o.rank = 1, o.dim[0] = (int)N;
		return true;
	}
	case TG_CUDA_OP_SUFMATCH: {
		const VShape &x = a[0];
		if (x.rank != 1 && x.rank != 2) {
			err = "'sufmatch' needs token ids (T) or (T, n), got " + vstr(x);
			return false;
		}
		long N = vsufmatch_size(x.dim[0], x.rank == 2 ? x.dim[1] : 1);
		if (N > INT32_MAX) {
			err = "'sufmatch' output too large";
			return false;
		}
		o.rank = 1, o.dim[0] = (int)N;
		return true;
	}
	default:
		err = "not a value operation";
		return false;
	}
}

struct Verifier {
	const tg_cuda_program *p;
	std::vector<char> seen;
	std::string err;
	int status = TG_CUDA_OK;

	bool fail(int st, int i, const std::string &why)
	{
		status = st;
		err = "instruction " + std::to_string(i) + ": " + why;
		return false;
	}
	bool val(int v) const { return v >= 0 && v < p->nval; }
	VShape sh(int v) const { return vshape(p->val[v]); }

	bool block(int from, int cnt, int depth)
	{
		if (from < 0 || cnt < 0 || from > p->nins || cnt > p->nins - from) return fail(TG_CUDA_EINVAL, from, "block out of range");
		if (depth > VM_MAXDEPTH) return fail(TG_CUDA_EUNSUPPORTED, from, "think/scan nesting deeper than 4");
		for (int i = from; i < from + cnt; i++)
			if (!ins(i, depth)) return false;
		return true;
	}

	bool ins(int i, int depth)
	{
		const tg_cuda_ins &in = p->ins[i];
		if (seen[i]) return fail(TG_CUDA_EINVAL, i, "belongs to two blocks");
		seen[i] = 1;
		if (in.op < 0 || in.op >= TG_CUDA_OP_COUNT) return fail(TG_CUDA_EINVAL, i, "unknown op");
		if (!val(in.out)) return fail(TG_CUDA_EINVAL, i, "result out of range");
		const VShape decl = sh(in.out);
		if (in.op == TG_CUDA_OP_THINK) {
			if (!val(in.init) || !val(in.yield) || (in.halt != -1 && !val(in.halt)) || in.maxit < 1 || in.tid < 0 ||
			    in.tid >= p->nthink)
				return fail(TG_CUDA_EINVAL, i, "malformed think");
			if (!veq(sh(in.init), decl) || !veq(sh(in.yield), decl))
				return fail(TG_CUDA_EINVAL, i, "think state, initial value and yield differ in shape");
			if (in.halt >= 0 && sh(in.halt).rank != 0) return fail(TG_CUDA_EINVAL, i, "halting value must be a scalar");
			return block(in.body, in.nbody, depth + 1);
		}
		if (in.op == TG_CUDA_OP_SCAN) {
			if (in.scan < 0 || in.scan >= p->nscan || !p->scans) return fail(TG_CUDA_EINVAL, i, "scan out of range");
			const tg_cuda_scan &s = p->scans[in.scan];
			if (s.T < 1 || s.nc < 1 || s.nx < 0 || s.ny < 0 || !s.c || !s.init || !s.next || (s.nx && (!s.x || !s.xt)) ||
			    (s.ny && (!s.y || !s.ys)) || (s.tid != -1 && (s.tid < 0 || s.tid >= p->nthink)))
				return fail(TG_CUDA_EINVAL, i, "malformed scan");
			for (int k = 0; k < s.nc; k++) {
				if (!val(s.c[k]) || !val(s.init[k]) || !val(s.next[k])) return fail(TG_CUDA_EINVAL, i, "scan carry out of range");
				if (!veq(sh(s.c[k]), sh(s.init[k])) || !veq(sh(s.c[k]), sh(s.next[k])))
					return fail(TG_CUDA_EINVAL, i, "scan carry, initial and next values differ in shape");
			}
			for (int j = 0; j < s.nx; j++) {
				if (!val(s.x[j]) || !val(s.xt[j])) return fail(TG_CUDA_EINVAL, i, "scan sequence out of range");
				VShape want = sh(s.x[j]);
				if (want.rank < 1 || want.dim[0] != s.T)
					return fail(TG_CUDA_EINVAL, i, "sequence does not have T steps along its first axis");
				for (int d = 1; d < want.rank; d++) want.dim[d - 1] = want.dim[d];
				want.rank--;
				if (!veq(sh(s.xt[j]), want)) return fail(TG_CUDA_EINVAL, i, "slice type differs from a row of its sequence");
			}
			for (int y = 0; y < s.ny; y++) {
				if (!val(s.y[y]) || !val(s.ys[y])) return fail(TG_CUDA_EINVAL, i, "scan stack out of range");
				VShape want = sh(s.y[y]);
				if (want.rank >= 4) return fail(TG_CUDA_EINVAL, i, "stack rank exceeds 4");
				for (int d = want.rank; d > 0; d--) want.dim[d] = want.dim[d - 1];
				want.dim[0] = s.T;
				want.rank++;
				if (!veq(sh(s.ys[y]), want)) return fail(TG_CUDA_EINVAL, i, "emit stack differs from T rows of its value");
			}
			return block(in.body, in.nbody, depth + 1);
		}
		if (in.na != kArity[in.op])
			return fail(TG_CUDA_EINVAL, i,
				    "op takes " + std::to_string(kArity[in.op]) + " operand(s), got " + std::to_string(in.na));
		VShape a[3], got;
		for (int j = 0; j < in.na; j++) a[j] = sh(in.a[j]); // operand indices were range-checked
		switch (in.op) {
		case TG_CUDA_OP_CONST:
			return true;
		case TG_CUDA_OP_TOPK: { // the declared type carries k in its last dimension (src/ir.c:389-399)
			bool ok = a[0].rank >= 1 && decl.rank == a[0].rank && decl.dim[decl.rank - 1] >= 1 &&
				  decl.dim[decl.rank - 1] <= 256;
			for (int d = 0; ok && d < a[0].rank - 1; d++) ok = decl.dim[d] == a[0].dim[d];
			return ok || fail(TG_CUDA_EINVAL, i, "topk: the declared type must keep the leading dimensions and set the last to k (1 to 256)");
		}
		case TG_CUDA_OP_RESHAPE: // only the element count is checked (src/ir.c:400-407)
			return vnumel(a[0]) == vnumel(decl) || fail(TG_CUDA_EINVAL, i, "reshape changes the element count");
		default:
			if (!vinfer(in.op, a, got, err)) return fail(TG_CUDA_EINVAL, i, err);
			if (!veq(got, decl)) return fail(TG_CUDA_EINVAL, i, "declared " + vstr(decl) + " but operation yields " + vstr(got));
			return true;
		}
	}
};

static int verify_program(const tg_cuda_program *p, std::string &err)
{
	for (int v = 0; v < p->nval; v++) {
		const tg_cuda_value &x = p->val[v];
		long n = 1;
		bool ok = x.rank >= 0 && x.rank <= 4;
		for (int d = 0; ok && d < x.rank; d++) {
			ok = x.dim[d] >= 1;
			n *= ok ? x.dim[d] : 1;
			ok = ok && n <= INT32_MAX;
		}
		if (!ok) {
			err = "value " + std::to_string(v) + ": bad rank or dimension";
			return TG_CUDA_EINVAL;
		}
		if (x.qbits && (x.rank != 2 || x.qaxis < 0 || x.qaxis > 1)) {
			err = "value " + std::to_string(v) + ": quantized params are rank 2 with axis 0 or 1";
			return TG_CUDA_EINVAL;
		}
	}
	if (p->ninputs < 0 || (p->ninputs && !p->inputs) || p->nthink < 0 || p->nscan < 0 || (p->nins && !p->ins)) {
		err = "malformed program";
		return TG_CUDA_EINVAL;
	}
	for (int i = 0; i < p->ninputs; i++)
		if (p->inputs[i] < 0 || p->inputs[i] >= p->nval || p->val[p->inputs[i]].kind != TG_CUDA_INPUT) {
			err = "entry input " + std::to_string(i) + " is not an input value";
			return TG_CUDA_EINVAL;
		}
	Verifier V{ p, std::vector<char>(p->nins, 0), "", TG_CUDA_OK };
	if (!V.block(0, p->ntop, 0)) {
		err = V.err;
		return V.status;
	}
	return TG_CUDA_OK;
}

static int compile_program(const tg_cuda_program *p, Prog &out, std::string &err)
{
	Compiler C;
	C.p = p;
	C.out = &out;
	if (p->nupd > 0) {
		err = "stateful model (update statements): rows are not independent, the GPU batch path rejects it";
		return TG_CUDA_EUNSUPPORTED;
	}
	if (p->nval <= 0 || !p->val || p->nins < 0 || p->ntop < 0 || p->ntop > p->nins || p->output < 0 || p->output >= p->nval) {
		err = "malformed program";
		return TG_CUDA_EINVAL;
	}
	for (int i = 0; i < p->nins; i++) {
		const tg_cuda_ins &in = p->ins[i];
		if (in.out < -1 || in.out >= p->nval || in.na < 0 || in.na > 3) {
			err = "malformed instruction";
			return TG_CUDA_EINVAL;
		}
		for (int j = 0; j < in.na; j++)
			if (in.a[j] < 0 || in.a[j] >= p->nval) {
				err = "operand out of range";
				return TG_CUDA_EINVAL;
			}
	}
	if (int rc = verify_program(p, err)) return rc;
	// params: f32 values; quantized params additionally keep codes (exact, in f32) and scales
	C.pslot.assign(p->nval, -1);
	C.sslot.assign(p->nval, -1);
	for (int v = 0; v < p->nval; v++) {
		const tg_cuda_value &x = p->val[v];
		if (x.kind == TG_CUDA_STATE) {
			err = "state values are not supported on the GPU batch path";
			return TG_CUDA_EUNSUPPORTED;
		}
		if (x.kind != TG_CUDA_PARAM) continue;
		long n = numel(x);
		C.pslot[v] = (int)out.blob.size();
		if (x.qbits) {
			if (!x.q || !x.qs || (x.qbits != 8 && x.qbits != 4) || x.rank != 2) {
				err = "malformed quantized param";
				return TG_CUDA_EINVAL;
			}
			int nch = x.dim[x.qaxis];
			for (long e = 0; e < n; e++) {
				int c;
				if (x.qbits == 8) c = x.q[e];
				else {
					int b = x.q[e >> 1];
					c = (e & 1) ? (b >> 4) : ((int)(signed char)(b << 4) >> 4);
				}
				out.blob.push_back((float)c);
			}
			C.sslot[v] = (int)out.blob.size();
			for (int c = 0; c < nch; c++) out.blob.push_back(x.qs[c]);
			// dequantized values for uses on another axis: data = code * scale (src/ir.c:503-507)
			for (long e = 0; e < n; e++) {
				int ch = x.qaxis == 0 ? (int)(e / x.dim[1]) : (int)(e % x.dim[1]);
				out.blob.push_back(x.data ? x.data[e] : out.blob[C.pslot[v] + e] * x.qs[ch]);
			}
		} else {
			if (!x.data) {
				err = "param without data";
				return TG_CUDA_EINVAL;
			}
			for (long e = 0; e < n; e++) out.blob.push_back(x.data[e]);
		}
		while (out.blob.size() % 4) out.blob.push_back(0.0f);
	}
	if (plan_arena(C)) {
		err = C.err;
		return C.status;
	}
	if (emit_block(C, 0, p->ntop, 0)) {
		err = C.err;
		return C.status;
	}
	out.nout = (int)numel(p->val[p->output]);
	out.out_loc = C.L(p->output);
	out.nthink = p->nthink;
	out.per = 0;
	for (int i = 0; i < p->ninputs; i++) {
		int v = p->inputs[i];
		out.in_off.push_back(C.inloc[v]);
		out.in_len.push_back((int)numel(p->val[v]));
		out.per += (int)numel(p->val[v]);
	}
	return TG_CUDA_OK;
}

// ---- run-time specialisation of the tape --------------------------------------------------
//
// The tape above is also turned into CUDA source for one kernel per program: every op
// becomes straight-line code with its element indices resolved, so the arena is an
// array of the thread's own registers (all indices are constants), params small enough
// for the 64 KB constant bank are read from it as instruction operands, and op
// dispatch, operand decoding and loop bookkeeping disappear. Control flow, rounding
// and operation order are those of vm_kernel, op for op (the same element functions,
// the same accumulation chains), with think loops as warp-uniform backward jumps.
// Programs whose arena is indexed at run time (scan slices, take from a computed value)
// run on vm_kernel: such a kernel would keep its arena in local memory, and one of them
// (the nested_grad test program, every index checked in range) stopped with an illegal
// address on the B200 for a cause not found; jit_build also refuses any generated kernel
// that needs local memory.

static const struct {
	const char *name;
	int v;
} kOpNames[] = {
#define TGC_OPNAME(x) { #x, x }
	TGC_OPNAME(TG_CUDA_OP_ADD), TGC_OPNAME(TG_CUDA_OP_SUB), TGC_OPNAME(TG_CUDA_OP_MUL), TGC_OPNAME(TG_CUDA_OP_DIV),
	TGC_OPNAME(TG_CUDA_OP_MAX), TGC_OPNAME(TG_CUDA_OP_MIN), TGC_OPNAME(TG_CUDA_OP_NEG), TGC_OPNAME(TG_CUDA_OP_TANH),
	TGC_OPNAME(TG_CUDA_OP_RELU), TGC_OPNAME(TG_CUDA_OP_SIGMOID), TGC_OPNAME(TG_CUDA_OP_EXP), TGC_OPNAME(TG_CUDA_OP_SQRT),
	TGC_OPNAME(TG_CUDA_OP_GELU), TGC_OPNAME(TG_CUDA_OP_SILU), TGC_OPNAME(TG_CUDA_OP_SOFTPLUS), TGC_OPNAME(TG_CUDA_OP_LOG),
	TGC_OPNAME(TG_CUDA_OP_STEP), TGC_OPNAME(TG_CUDA_OP_SIN), TGC_OPNAME(TG_CUDA_OP_COS), TGC_OPNAME(TG_CUDA_OP_FLOOR),
#undef TGC_OPNAME
};

constexpr long JIT_MAX_STMTS = 20000;   // larger programs stay on the interpreter (compile time)
constexpr int JIT_MAX_ARENA = 192;      // floats per row: beyond this the arena no longer fits the registers
constexpr size_t JIT_MAX_CPARAMS = 16000; // floats of params in the constant bank

struct Gen {
	const Prog &P;
	bool cparams;
	std::string s;
	long stmts = 0;
	std::vector<char> label;

	explicit Gen(const Prog &p) : P(p), cparams(p.blob.size() <= JIT_MAX_CPARAMS), label(p.tape.size() + 1, 0) {}

	static std::string num(long v) { return std::to_string(v); }
	static std::string flt(float f)
	{
		uint32_t u;
		memcpy(&u, &f, 4);
		char b[32];
		snprintf(b, sizeof b, "__uint_as_float(0x%08xu)", u);
		return b;
	}
	// element e of a location, e a constant
	std::string at(int l, long e) const
	{
		if (l >= 0) return "ar[" + num(l + e) + "]";
		long i = -(long)(l + 1) + e;
		return cparams ? "CP(" + num(i) + ")" : "__ldg(GP + " + num(i) + ")";
	}
	// element `e` (a run-time expression) of a param location
	std::string atd(int l, const std::string &e) const { return "__ldg(GP + " + num(-(long)(l + 1)) + " + (" + e + "))"; }
	void line(const std::string &x)
	{
		s += x;
		s += '\n';
		stmts++;
	}
	int op(int pc);
};

int Gen::op(int pc)
{
	const DOp &o = P.tape[pc];
	const std::string D = num(o.depth);
	if (label[pc]) line("L" + num(pc) + ":;");
	switch (o.code) {
	case D_CONST:
		line("if (done == 0u) " + at(o.out, 0) + " = " + flt(o.f) + ";");
		return 0;
	case D_BIN:
		line("if (done == 0u) {");
		for (int e = 0; e < o.n; e++) {
			long ia, ib;
			if (o.rank == 0) {
				ia = (long)e * o.sa[0];
				ib = (long)e * o.sb[0];
			} else {
				int rem = e;
				ia = ib = 0;
				for (int d = o.rank - 1; d >= 0; d--) {
					int idx = rem % o.dims[d];
					rem /= o.dims[d];
					ia += (long)idx * o.sa[d];
					ib += (long)idx * o.sb[d];
				}
			}
			line(at(o.out, e) + " = bin_op(" + num(o.sub) + ", " + at(o.a, ia) + ", " + at(o.b, ib) + ");");
		}
		line("}");
		return 0;
	case D_UN:
		line("if (done == 0u) {");
		for (int e = 0; e < o.n; e++) line(at(o.out, e) + " = un_op(" + num(o.sub) + ", " + at(o.a, e) + ");");
		line("}");
		return 0;
	case D_MATMUL: {
		line("if (done == 0u) {");
		const int m = o.m, k = o.k, n = o.nn;
		for (int g = 0; g < o.g; g++) {
			long oo = (long)g * m * n, ao = (long)g * m * k, bo = (long)g * k * n;
			for (int i = 0; i < m; i++)
				for (int j = 0; j < n; j++) {
					std::string x = "{ float acc = 0.0f;";
					for (int p = 0; p < k; p++)
						x += " acc = __fadd_rn(acc, __fmul_rn(" + at(o.a, ao + (long)i * k + p) + ", " + at(o.b, bo + (long)p * n + j) + "));";
					if (o.scale == 1) x += " acc = __fmul_rn(" + at(o.c, i) + ", acc);";
					else if (o.scale == 2) x += " acc = __fmul_rn(" + at(o.c, j) + ", acc);";
					x += " " + at(o.out, oo + (long)i * n + j) + " = acc; }";
					line(x);
					stmts += k;
				}
		}
		line("}");
		return 0;
	}
	case D_ROW:
		line("if (done == 0u) {");
		for (int r = 0; r < o.m; r++) {
			const long base = (long)r * o.k;
			if (o.sub == TG_CUDA_OP_SOFTMAX) {
				line("{ float mx = " + at(o.a, base) + ", s = 0.0f, v, y;");
				for (int i = 1; i < o.k; i++) line("v = " + at(o.a, base + i) + "; if (v > mx) mx = v;");
				for (int i = 0; i < o.k; i++)
					line("y = expf(__fsub_rn(" + at(o.a, base + i) + ", mx)); " + at(o.out, base + i) + " = y; s = __fadd_rn(s, y);");
				for (int i = 0; i < o.k; i++) line(at(o.out, base + i) + " = __fdiv_rn(" + at(o.out, base + i) + ", s);");
				line("}");
			} else {
				line("{ float s = 0.0f, x;");
				for (int i = 0; i < o.k; i++) line("x = " + at(o.a, base + i) + "; s = __fadd_rn(s, __fmul_rn(x, x));");
				line("const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, " + flt((float)o.k) + "), 1e-6f)));");
				for (int i = 0; i < o.k; i++) line(at(o.out, base + i) + " = __fmul_rn(" + at(o.a, base + i) + ", inv);");
				line("}");
			}
		}
		line("}");
		return 0;
	case D_RED: {
		line("if (done == 0u) { float s = 0.0f;");
		for (int e = 0; e < o.n; e++) line("s = __fadd_rn(s, " + at(o.a, e) + ");");
		line(at(o.out, 0) + " = " + (o.sub == TG_CUDA_OP_MEAN ? "__fdiv_rn(s, " + flt((float)o.n) + ")" : std::string("s")) + "; }");
		return 0;
	}
	case D_TRANS:
		line("if (done == 0u) {");
		for (int g = 0; g < o.g; g++)
			for (int i = 0; i < o.m; i++)
				for (int j = 0; j < o.k; j++)
					line(at(o.out, (long)g * o.m * o.k + (long)j * o.m + i) + " = " + at(o.a, (long)g * o.m * o.k + (long)i * o.k + j) + ";");
		line("}");
		return 0;
	case D_OUTER:
		line("if (done == 0u) {");
		for (int i = 0; i < o.m; i++)
			for (int j = 0; j < o.k; j++)
				line(at(o.out, (long)i * o.k + j) + " = __fmul_rn(" + at(o.a, i) + ", " + at(o.b, j) + ");");
		line("}");
		return 0;
	case D_TAKE: // from a param table only (gen_source), in global memory
		line("if (done == 0u) {");
		for (int i = 0; i < o.m; i++) {
			line("{ const float r = floorf(__fadd_rn(" + at(o.b, i) + ", 0.5f)); const int t = r >= 0.0f && r < " +
			     flt((float)o.k) + " ? (int)r : -1;");
			for (int j = 0; j < o.nn; j++)
				line(at(o.out, (long)i * o.nn + j) + " = t >= 0 ? " + atd(o.a, "t * " + num(o.nn) + " + " + num(j)) + " : 0.0f;");
			line("}");
		}
		line("}");
		return 0;
	case D_SPMM: // from a param table only (gen_source): run-time rows of it in global memory
		line("if (done == 0u) {");
		for (int i = 0; i < o.m; i++) {
			for (int j = 0; j < o.nn; j++) line(at(o.out, (long)i * o.nn + j) + " = 0.0f;");
			for (int e = 0; e < o.k; e++) {
				const long xe = ((long)i * o.k + e) * 2;
				line("{ const float val = " + at(o.a, xe + 1) + ", rr = floorf(__fadd_rn(" + at(o.a, xe) + ", 0.5f)); const int t = rr >= 0.0f && rr < " +
				     flt((float)o.g) + " ? (int)rr : -1;");
				line("if (t >= 0 && val != 0.0f) { const float v = " + (o.scale ? "__fmul_rn(val, " + atd(o.c, "t") + ")" : std::string("val")) + ";");
				for (int j = 0; j < o.nn; j++)
					line(at(o.out, (long)i * o.nn + j) + " = __fadd_rn(" + at(o.out, (long)i * o.nn + j) + ", __fmul_rn(v, " +
					     atd(o.b, "t * " + num(o.nn) + " + " + num(j)) + "));");
				line("} }");
				stmts += o.nn;
			}
		}
		line("}");
		return 0;
	case D_SUMTO: { // the merged iteration space walked at generation time: constant indices
		line("if (done == 0u) {");
		for (int i = 0; i < o.n; i++) line(at(o.out, i) + " = 0.0f;");
		const int r = o.rank, w = o.dims[r - 1];
		long outer = 1, io = 0;
		for (int i = 0; i < r - 1; i++) outer *= o.dims[i];
		int idx[4] = { 0, 0, 0, 0 };
		for (long i = 0; i < outer; i++) {
			if (o.sa[r - 1]) {
				for (int j = 0; j < w; j++) line(at(o.out, io + j) + " = __fadd_rn(" + at(o.out, io + j) + ", " + at(o.a, i * w + j) + ");");
			} else {
				std::string x = "{ float acc = 0.0f;";
				for (int j = 0; j < w; j++) x += " acc = __fadd_rn(acc, " + at(o.a, i * w + j) + ");";
				line(x + " " + at(o.out, io) + " = __fadd_rn(" + at(o.out, io) + ", acc); }");
				stmts += w;
			}
			for (int q = r - 2; q >= 0; q--) {
				io += o.sa[q];
				if (++idx[q] < o.dims[q]) break;
				io -= (long)o.sa[q] * o.dims[q];
				idx[q] = 0;
			}
		}
		line("}");
		return 0;
	}
	case D_TOPK: // repeated selection in the order (value descending, index ascending)
		line("if (done == 0u) {");
		for (int r = 0; r < o.m; r++) {
			line("{ float lv = 0.0f; int li = -1;");
			for (int i = 0; i < o.nn; i++) {
				line("{ int bi = -1; float bv = 0.0f, v;");
				for (int j = 0; j < o.k; j++)
					line("v = " + at(o.a, (long)r * o.k + j) + "; if (v == v && (li < 0 || v < lv || (v == lv && " + num(j) +
					     " > li)) && (bi < 0 || v > bv)) bi = " + num(j) + ", bv = v;");
				line(at(o.out, (long)r * o.nn + i) + " = (float)bi; if (bi >= 0) lv = bv, li = bi; }");
			}
			line("}");
		}
		line("}");
		return 0;
	case D_COPY:
		if (o.out == o.a) return 0;
		line("if (done == 0u) {");
		for (int e = 0; e < o.n; e++) line(at(o.out, e) + " = " + at(o.a, e) + ";");
		line("}");
		return 0;
	case D_THINK_BEGIN:
		line("if (done == 0u) {");
		if (o.out != o.a)
			for (int e = 0; e < o.n; e++) line(at(o.out, e) + " = " + at(o.a, e) + ";");
		line("it" + D + " = 0; surv" + D + " = 1.0f; }");
		return 0;
	case D_THINK_END: {
		const std::string bit = num(1u << o.depth) + "u";
		line("if (done == 0u) { it" + D + "++; float dd = 0.0f, v;");
		for (int e = 0; e < o.n; e++)
			line("v = fabsf(__fsub_rn(" + at(o.yield, e) + ", " + at(o.out, e) + ")); if (v > dd) dd = v;");
		for (int e = 0; e < o.n; e++) line(at(o.out, e) + " = " + at(o.yield, e) + ";");
		line("bool stop = it" + D + " >= " + num(o.maxit) + ";");
		if (o.eps >= 0) line("if (dd <= " + flt(o.eps) + ") stop = true;");
		if (o.halt != INT_MIN) {
			line("{ const float p = " + at(o.halt, 0) + "; surv" + D + " = __fmul_rn(surv" + D +
			     ", __fsub_rn(1.0f, p < 0.0f ? 0.0f : p > 1.0f ? 1.0f : p)); if (__fsub_rn(1.0f, surv" + D + ") > " + flt(o.hthr) +
			     ") stop = true; }");
		}
		line("if (stop) { done |= " + bit + "; if (live && " + num(o.tid) + " < nt) steps[row * nt + " + num(o.tid) + "] = it" + D + "; }");
		line("}");
		line("if (__any_sync(0xffffffffu, done == 0u)) goto L" + num(o.target) + ";");
		line("done &= ~" + bit + ";");
		return 0;
	}
	}
	return -1;
}

// CUDA source of the specialised kernel `tg_rowvm`, or an empty string when the program
// is beyond the limits above (it then runs on vm_kernel).
static std::string gen_source(const Prog &P, std::string &why)
{
	if (P.arena > JIT_MAX_ARENA) {
		why = "arena larger than " + std::to_string(JIT_MAX_ARENA) + " floats per row";
		return "";
	}
	// Every arena index must be a constant, so that the arena stays in registers: scans
	// (a slice per step) and take from a computed value index it at run time and keep
	// their programs on vm_kernel.
	for (const DOp &o : P.tape)
		if (o.code == D_SCAN_BEGIN || o.code == D_SCAN_SLICE || o.code == D_SCAN_END || o.code == D_MEMSCAN ||
		    o.code == D_MEMSCAN_T || o.code == D_SUFMATCH || o.code == D_TAKE_T || (o.code == D_TAKE && o.a >= 0) ||
		    (o.code == D_SPMM && o.b >= 0)) {
			why = "run-time arena index (scan, memscan, sufmatch, take_t, or take / spmm from a computed table)";
			return "";
		}
	Gen G(P);
	for (const DOp &o : P.tape)
		if (o.code == D_THINK_END) G.label[o.target] = 1;
	std::string h;
	for (auto &e : kOpNames) h += "#define " + std::string(e.name) + " " + std::to_string(e.v) + "\n";
	h += kRowMathSrc;
	h += "\n";
	if (G.cparams) {
		h += "__constant__ unsigned CPU_[" + std::to_string(std::max<size_t>(P.blob.size(), 1)) + "] = {";
		for (size_t i = 0; i < P.blob.size(); i++) {
			uint32_t u;
			memcpy(&u, &P.blob[i], 4);
			char b[16];
			snprintf(b, sizeof b, "%s0x%xu", i ? "," : "", u);
			h += b;
			if (i % 16 == 15) h += "\n";
		}
		if (P.blob.empty()) h += "0u";
		h += "};\n#define CP(i) __uint_as_float(CPU_[i])\n";
	}
	h += "extern \"C\" __global__ void __launch_bounds__(" + std::to_string(VM_ROWS) +
	     ") tg_rowvm(const float *__restrict__ in, long rows, float *__restrict__ out, int *__restrict__ steps, int nt, "
	     "const float *__restrict__ GP)\n{\n";
	h += "const long row = (long)blockIdx.x * " + std::to_string(VM_ROWS) + " + threadIdx.x;\nconst bool live = row < rows;\n";
	h += "float ar[" + std::to_string(std::max(P.arena, 1)) + "];\n#pragma unroll\nfor (int i = 0; i < " +
	     std::to_string(std::max(P.arena, 1)) + "; i++) ar[i] = 0.0f;\n";
	h += "unsigned done = live ? 0u : " + std::to_string(1u << VM_MAXDEPTH) + "u;\n";
	for (int d = 0; d < VM_MAXDEPTH; d++) h += "int it" + std::to_string(d) + " = 0; float surv" + std::to_string(d) + " = 1.0f;\n";
	h += "if (live) {\nconst float *src = in + row * " + std::to_string(P.per) + ";\n";
	for (size_t i = 0, o = 0; i < P.in_off.size(); i++) {
		for (int e = 0; e < P.in_len[i]; e++)
			h += "ar[" + std::to_string(P.in_off[i] + e) + "] = src[" + std::to_string(o + e) + "];\n";
		o += P.in_len[i];
	}
	h += "}\n";
	G.s = h;
	for (int pc = 0; pc < (int)P.tape.size(); pc++) {
		if (G.op(pc)) {
			why = "tape op without a generator";
			return "";
		}
		if (G.stmts > JIT_MAX_STMTS) {
			why = "program larger than " + std::to_string(JIT_MAX_STMTS) + " statements";
			return "";
		}
	}
	G.line("if (live) {");
	for (int e = 0; e < P.nout; e++) G.line("out[row * " + std::to_string(P.nout) + " + " + std::to_string(e) + "] = " + G.at(P.out_loc, e) + ";");
	G.line("}\n}");
	return G.s;
}

} // namespace tgc

using namespace tgc;

struct tg_cuda_model {
	Model m;
};

extern "C" int tg_cuda_load(const tg_cuda_program *p, tg_cuda_model **out)
{
	clear_err();
	if (!p || !out) return set_err(TG_CUDA_EINVAL, "tg_cuda_load: NULL argument");
	*out = nullptr;
	if (!inited()) return set_err(TG_CUDA_ENODEV, "tg_cuda_load: call tg_cuda_init first");
	tg_cuda_model *g = new tg_cuda_model;
	std::string err;
	int rc = compile_program(p, g->m.prog, err);
	if (rc) {
		delete g;
		return set_err(rc, "tg_cuda_load: %s", err.c_str());
	}
	Prog &P = g->m.prog;
	size_t blob_bytes = (P.blob.size() + 3) / 4 * 4 * sizeof(float);
	size_t arena_bytes = (size_t)P.arena * VM_ROWS * sizeof(float);
	g->m.blob_in_smem = blob_bytes <= 96 * 1024;
	g->m.global_arena = arena_bytes + (g->m.blob_in_smem ? blob_bytes : 0) > 200 * 1024;
	g->m.smem = (g->m.blob_in_smem ? blob_bytes : 0) + (g->m.global_arena ? 0 : arena_bytes);
	for (size_t i = 0; i < devices().size(); i++) g->m.dev.emplace_back(new Model::PerDev);
	for (size_t i = 0; i < devices().size(); i++) {
		auto &D = *g->m.dev[i];
		int id = devices()[i].id;
		if ((rc = D.tape.alloc(P.tape.size() * sizeof(DOp), id)) || (rc = D.blob.alloc(blob_bytes, id)) ||
		    (rc = D.inloc.alloc(P.in_off.size() * sizeof(int) + 4, id)) || (rc = D.inlen.alloc(P.in_len.size() * sizeof(int) + 4, id))) {
			delete g;
			return rc;
		}
		cudaSetDevice(id);
		if (fault("h2d")) {
			delete g;
			return set_err(TG_CUDA_EFAULT, "injected copy failure (TG_CUDA_FAULT=h2d)");
		}
		TGC_CUDA(cudaMemcpy(D.tape.p, P.tape.data(), P.tape.size() * sizeof(DOp), cudaMemcpyHostToDevice));
		TGC_CUDA(cudaMemcpy(D.blob.p, P.blob.data(), P.blob.size() * sizeof(float), cudaMemcpyHostToDevice));
		TGC_CUDA(cudaMemcpy(D.inloc.p, P.in_off.data(), P.in_off.size() * sizeof(int), cudaMemcpyHostToDevice));
		TGC_CUDA(cudaMemcpy(D.inlen.p, P.in_len.data(), P.in_len.size() * sizeof(int), cudaMemcpyHostToDevice));
		// copies from pageable memory may still be in flight on return; later kernels run on
		// non-blocking streams, so wait for them here
		TGC_CUDA(cudaDeviceSynchronize());
		TGC_CUDA(cudaFuncSetAttribute(vm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
	}
	// the specialised kernel, on every device or on none
	const char *mode = getenv("TG_CUDA_ROWVM");
	std::string src;
	if (mode && !strcmp(mode, "interp")) g->m.jit_why = "TG_CUDA_ROWVM=interp";
	else src = gen_source(P, g->m.jit_why);
	if (!src.empty()) {
		g->m.jit = true;
		for (size_t i = 0; i < devices().size() && g->m.jit; i++) {
			std::string log;
			if (jit_build(src, "tg_rowvm", devices()[i].id, 0, g->m.dev[i]->jit, log)) {
				g->m.jit = false;
				g->m.jit_why = tg_cuda_error();
				clear_err();
			}
		}
	}
	cudaSetDevice(devices()[0].id);
	*out = g;
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_program_kernel(const tg_cuda_program *p, char *src, long n, long *len, int compile)
{
	clear_err();
	if (!p) return set_err(TG_CUDA_EINVAL, "tg_cuda_program_kernel: NULL program");
	Prog P;
	std::string err, why;
	int rc = compile_program(p, P, err);
	if (rc) return set_err(rc, "tg_cuda_program_kernel: %s", err.c_str());
	std::string s = gen_source(P, why);
	if (s.empty()) return set_err(TG_CUDA_EUNSUPPORTED, "tg_cuda_program_kernel: %s", why.c_str());
	if (len) *len = (long)s.size();
	if (src && n > 0) snprintf(src, (size_t)n, "%s", s.c_str());
	if (compile) {
		std::vector<char> cubin;
		std::string log;
		if ((rc = jit_compile(s, cubin, log))) return rc;
	}
	return TG_CUDA_OK;
}

// Row sizes of a loaded model, for the micro-batcher (batcher.cu).
int tgc::model_shape(const tg_cuda_model *g, int *per, int *nout, int *nthink)
{
	*per = g->m.prog.per, *nout = g->m.prog.nout, *nthink = g->m.prog.nthink;
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_model_jit(const tg_cuda_model *g, char *why, int n)
{
	if (!g) return set_err(TG_CUDA_EINVAL, "tg_cuda_model_jit: NULL model");
	if (why && n > 0) snprintf(why, (size_t)n, "%s", g->m.jit ? "" : g->m.jit_why.c_str());
	return g->m.jit ? 1 : 0;
}

static int run_rows(Model &M, size_t di, const float *d_in, long rows, float *d_out, int *d_steps, int nt, cudaStream_t st)
{
	Prog &P = M.prog;
	auto &D = *M.dev[di];
	if (rows <= 0) return TG_CUDA_OK;
	long ctas = (rows + VM_ROWS - 1) / VM_ROWS;
	float *gar = nullptr;
	if (M.global_arena && !M.jit) {
		size_t need = (size_t)ctas * P.arena * VM_ROWS * sizeof(float);
		int rc = D.gar.ensure(need, devices()[di].id);
		if (rc) return rc;
		gar = D.gar.as<float>();
	}
	if (fault("launch")) return set_err(TG_CUDA_EFAULT, "injected launch failure (TG_CUDA_FAULT=launch)");
	if (M.jit) {
		const float *gp = D.blob.as<float>();
		int ntv = nt;
		void *args[] = { (void *)&d_in, (void *)&rows, (void *)&d_out, (void *)&d_steps, (void *)&ntv, (void *)&gp };
		return jit_launch(D.jit, (unsigned)ctas, VM_ROWS, 0, st, args);
	}
	vm_kernel<<<(unsigned)ctas, VM_ROWS, M.smem, st>>>(D.tape.as<DOp>(), (int)P.tape.size(), D.blob.as<float>(),
							   (int)P.blob.size(), M.blob_in_smem ? 1 : 0, P.arena, d_in, P.per,
							   rows, d_out, P.nout, P.out_loc, d_steps, nt, D.inloc.as<int>(),
							   D.inlen.as<int>(), (int)P.in_off.size(), gar);
	TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_batch_device(tg_cuda_model *g, const float *all, long rows, float *out, int *steps, void *stream)
{
	clear_err();
	if (!g || (rows > 0 && (!all || !out))) return set_err(TG_CUDA_EINVAL, "tg_cuda_batch_device: NULL argument");
	if (g->m.prog.nthink > 0 && rows > 0 && !steps) return set_err(TG_CUDA_EINVAL, "tg_cuda_batch_device: steps is NULL");
	cudaSetDevice(devices()[0].id);
	return run_rows(g->m, 0, all, rows, out, steps, g->m.prog.nthink, (cudaStream_t)stream);
}

// Host copies of a few MB and more split over up to 4 threads: the caller and up to three
// workers (fewer on hosts with fewer hardware threads) that live as long as the process
// (thread start-up would cost more than the copy of a 4 MB chunk). More threads measured
// no faster: four saturate the host's copy bandwidth.
class CopyPool {
	std::mutex mu;
	std::condition_variable cv, idle;
	struct Job {
		void *dst;
		const void *src;
		size_t n;
	};
	std::vector<Job> jobs;
	int running = 0;
	std::vector<std::thread> th;
	bool stop = false;

public:
	const int workers;
	CopyPool() : workers((int)std::min(3u, std::max(2u, std::thread::hardware_concurrency()) - 1))
	{
		for (int i = 0; i < workers; i++)
			th.emplace_back([this] {
				std::unique_lock<std::mutex> lk(mu);
				for (;;) {
					cv.wait(lk, [this] { return stop || !jobs.empty(); });
					if (stop) return;
					Job j = jobs.back();
					jobs.pop_back();
					running++;
					lk.unlock();
					memcpy(j.dst, j.src, j.n);
					lk.lock();
					running--;
					if (jobs.empty() && running == 0) idle.notify_all();
				}
			});
	}
	~CopyPool()
	{
		{
			std::lock_guard<std::mutex> lk(mu);
			stop = true;
		}
		cv.notify_all();
		for (auto &t : th) t.join();
	}
	// copies [0, first) on the calling thread, the rest as `parts - 1` jobs, then waits
	void copy(void *dst, const void *src, size_t n, int parts)
	{
		const size_t each = (n / parts + 63) / 64 * 64;
		{
			std::lock_guard<std::mutex> lk(mu);
			for (int i = 1; i < parts; i++) {
				size_t off = each * i;
				if (off >= n) break;
				jobs.push_back({ (char *)dst + off, (const char *)src + off, std::min(each, n - off) });
			}
		}
		cv.notify_all();
		memcpy(dst, src, std::min(each, n));
		std::unique_lock<std::mutex> lk(mu);
		idle.wait(lk, [this] { return jobs.empty() && running == 0; });
	}
};

static void par_copy(void *dst, const void *src, size_t n)
{
	static CopyPool pool;
	static std::mutex one; // one split copy at a time (several GPUs' host threads share the pool)
	const int parts = (int)std::min<size_t>((size_t)pool.workers + 1, n / (1 << 20));
	if (parts <= 1) {
		memcpy(dst, src, n);
		return;
	}
	std::lock_guard<std::mutex> lk(one);
	pool.copy(dst, src, n, parts);
}

constexpr size_t BATCH_CHUNK_BYTES = 4 << 20;  // input bytes per pipeline chunk through staging
constexpr size_t DIRECT_CHUNK_BYTES = 2 << 20; // ... and straight from page-locked caller buffers

// One host thread per GPU over its contiguous shard of rows. The shard goes through the
// device in chunks of ~4 MB of input on two alternating slots: while the GPU copies in,
// runs and copies out chunk k on one slot's stream, the host copies chunk k-1's results
// out of the other slot's pinned buffers and chunk k+1's rows into them. Output rows
// land at their own offsets, so the gather keeps input order. When the caller's buffers
// are page-locked (tg_cuda_host_register) the staging copies drop out: each chunk is
// copied in, run and copied out on its slot's stream straight from and to the caller's
// memory, and the host thread only queues work and waits at the end.
extern "C" int tg_cuda_batch(tg_cuda_model *g, const float *all, long rows, int per, float *out, int n, int *steps, int nt)
{
	clear_err();
	if (!g || rows < 0 || (rows > 0 && (!all || !out))) return set_err(TG_CUDA_EINVAL, "tg_cuda_batch: NULL argument");
	Prog &P = g->m.prog;
	if (per != P.per) return set_err(TG_CUDA_EINVAL, "tg_cuda_batch: %d values per row, the model needs %d", per, P.per);
	if (n != P.nout) return set_err(TG_CUDA_EINVAL, "tg_cuda_batch: %d outputs per row, the model has %d", n, P.nout);
	if (P.nthink > 0 && (!steps || nt < P.nthink))
		return set_err(TG_CUDA_EINVAL, "tg_cuda_batch: steps needs %d slots per row", P.nthink);
	if (rows == 0) return TG_CUDA_OK;
	const bool want_steps = nt > 0 && steps;
	const bool direct = host_registered(all, (size_t)rows * per * sizeof(float)) &&
			    host_registered(out, (size_t)rows * n * sizeof(float)) &&
			    (!want_steps || host_registered(steps, (size_t)rows * nt * sizeof(int)));
	size_t G = devices().size();
	std::vector<int> rcs(G, 0);
	std::vector<std::string> errs(G);
	auto work = [&](size_t di) {
		long lo = rows * (long)di / (long)G, hi = rows * (long)(di + 1) / (long)G, cnt = hi - lo;
		if (cnt <= 0) return;
		Device &dv = devices()[di];
		cudaSetDevice(dv.id);
		auto &D = *g->m.dev[di];
		std::lock_guard<std::mutex> lk(D.mu);
		// direct: three slots keep the copy-in engine busy (a slot's next chunk waits for its
		// previous copy-out), smaller chunks shorten the pipeline's fill and drain
		const int nslot = direct ? 3 : 2;
		const long chunk = std::max<long>(
			VM_ROWS, (long)((direct ? DIRECT_CHUNK_BYTES : BATCH_CHUNK_BYTES) / ((size_t)per * sizeof(float))) / VM_ROWS * VM_ROWS);
		auto drain = [&] {
			for (Slot &S : D.slot) {
				if (S.st) cudaStreamSynchronize(S.st);
				S.busy = false;
			}
		};
		auto done = [&](int r) {
			rcs[di] = r;
			if (r) {
				errs[di] = tg_cuda_error();
				drain();
			}
		};
		auto finish = [&](Slot &S) -> int {
			cudaError_t e = cudaEventSynchronize(S.done);
			if (e != cudaSuccess) return set_err(TG_CUDA_ECUDA, "device %d: %s", dv.id, cudaGetErrorString(e));
			par_copy(out + (size_t)(lo + S.lo) * n, S.hout.p, (size_t)S.cnt * n * sizeof(float));
			if (want_steps) par_copy(steps + (size_t)(lo + S.lo) * nt, S.hsteps.p, (size_t)S.cnt * nt * sizeof(int));
			S.busy = false;
			return TG_CUDA_OK;
		};
		int rc;
		for (int si = 0; si < nslot; si++) {
			Slot &S = D.slot[si];
			if (!S.st && cudaStreamCreateWithFlags(&S.st, cudaStreamNonBlocking) != cudaSuccess)
				return done(set_err(TG_CUDA_ECUDA, "cudaStreamCreate failed"));
			if (!S.done && cudaEventCreateWithFlags(&S.done, cudaEventDisableTiming) != cudaSuccess)
				return done(set_err(TG_CUDA_ECUDA, "cudaEventCreate failed"));
			const long m = std::min(chunk, cnt);
			if (!direct && ((rc = S.hin.ensure((size_t)m * per * sizeof(float))) || (rc = S.hout.ensure((size_t)m * n * sizeof(float))) ||
					(rc = S.hsteps.ensure((size_t)m * std::max(nt, 1) * sizeof(int)))))
				return done(rc);
			if ((rc = S.din.ensure((size_t)m * per * sizeof(float), dv.id)) || (rc = S.dout.ensure((size_t)m * n * sizeof(float), dv.id)) ||
			    (rc = S.dsteps.ensure((size_t)m * std::max(nt, 1) * sizeof(int), dv.id)))
				return done(rc);
		}
		if (fault("h2d")) return done(set_err(TG_CUDA_EFAULT, "injected copy failure (TG_CUDA_FAULT=h2d)"));
		if (direct) {
			for (long c0 = 0, k = 0; c0 < cnt; c0 += chunk, k++) {
				Slot &S = D.slot[k % nslot];
				const long m = std::min(chunk, cnt - c0);
				const size_t r0 = (size_t)(lo + c0);
				cudaError_t e = cudaMemcpyAsync(S.din.p, all + r0 * per, (size_t)m * per * sizeof(float), cudaMemcpyHostToDevice, S.st);
				if (e == cudaSuccess && nt > 0) e = cudaMemsetAsync(S.dsteps.p, 0, (size_t)m * nt * sizeof(int), S.st);
				if (e != cudaSuccess) return done(set_err(TG_CUDA_ECUDA, "H2D: %s", cudaGetErrorString(e)));
				if ((rc = run_rows(g->m, di, S.din.as<float>(), m, S.dout.as<float>(), nt > 0 ? S.dsteps.as<int>() : nullptr, nt,
						   S.st)))
					return done(rc);
				if (fault("gather")) return done(set_err(TG_CUDA_EFAULT, "injected gather failure (TG_CUDA_FAULT=gather)"));
				e = cudaMemcpyAsync(out + r0 * n, S.dout.p, (size_t)m * n * sizeof(float), cudaMemcpyDeviceToHost, S.st);
				if (e == cudaSuccess && want_steps)
					e = cudaMemcpyAsync(steps + r0 * nt, S.dsteps.p, (size_t)m * nt * sizeof(int), cudaMemcpyDeviceToHost, S.st);
				if (e != cudaSuccess) return done(set_err(TG_CUDA_ECUDA, "device %d: %s", dv.id, cudaGetErrorString(e)));
			}
			for (int si = 0; si < nslot; si++) {
				cudaError_t e = cudaStreamSynchronize(D.slot[si].st);
				if (e != cudaSuccess) return done(set_err(TG_CUDA_ECUDA, "device %d: %s", dv.id, cudaGetErrorString(e)));
			}
			return done(TG_CUDA_OK);
		}
		for (long c0 = 0, k = 0; c0 < cnt; c0 += chunk, k++) {
			Slot &S = D.slot[k & 1];
			if (S.busy && (rc = finish(S))) return done(rc);
			const long m = std::min(chunk, cnt - c0);
			par_copy(S.hin.p, all + (size_t)(lo + c0) * per, (size_t)m * per * sizeof(float));
			cudaError_t e = cudaMemcpyAsync(S.din.p, S.hin.p, (size_t)m * per * sizeof(float), cudaMemcpyHostToDevice, S.st);
			if (e == cudaSuccess && nt > 0) e = cudaMemsetAsync(S.dsteps.p, 0, (size_t)m * nt * sizeof(int), S.st);
			if (e != cudaSuccess) return done(set_err(TG_CUDA_ECUDA, "H2D: %s", cudaGetErrorString(e)));
			if ((rc = run_rows(g->m, di, S.din.as<float>(), m, S.dout.as<float>(), nt > 0 ? S.dsteps.as<int>() : nullptr, nt, S.st)))
				return done(rc);
			if (fault("gather")) return done(set_err(TG_CUDA_EFAULT, "injected gather failure (TG_CUDA_FAULT=gather)"));
			e = cudaMemcpyAsync(S.hout.p, S.dout.p, (size_t)m * n * sizeof(float), cudaMemcpyDeviceToHost, S.st);
			if (e == cudaSuccess && want_steps)
				e = cudaMemcpyAsync(S.hsteps.p, S.dsteps.p, (size_t)m * nt * sizeof(int), cudaMemcpyDeviceToHost, S.st);
			if (e == cudaSuccess) e = cudaEventRecord(S.done, S.st);
			if (e != cudaSuccess) return done(set_err(TG_CUDA_ECUDA, "device %d: %s", dv.id, cudaGetErrorString(e)));
			S.lo = c0;
			S.cnt = m;
			S.busy = true;
		}
		for (Slot &S : D.slot)
			if (S.busy && (rc = finish(S))) return done(rc);
		done(TG_CUDA_OK);
	};
	if (G == 1) work(0);
	else {
		std::vector<std::thread> th;
		for (size_t di = 0; di < G; di++) th.emplace_back(work, di);
		for (auto &t : th) t.join();
	}
	cudaSetDevice(devices()[0].id);
	for (size_t di = 0; di < G; di++)
		if (rcs[di]) return set_err(rcs[di], "%s", errs[di].c_str());
	return TG_CUDA_OK;
}

extern "C" void tg_cuda_free(tg_cuda_model *g) { delete g; }
