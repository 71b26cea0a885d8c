// quant.cu -- per-channel RTN quantization on the device, bit-exact with the
// reference quantizer (src/quant.c:176-200 best_scale/code_of, :258-310 packing).
//
// Pass 1, one thread per channel: the 10-point clipping grid over the channel's
// absmax; the squared error of each candidate is summed serially in element
// order in double with explicitly rounded operations (no contraction), so the
// arg-min and the chosen scale are the reference's. Pass 2, one thread per
// output byte: each code is code_of(w, s) of its own element with its channel's
// double scale, and int4 nibbles are packed low-first like set_code.
#include "common.cuh"
#include "kernels.cuh"

namespace tgc {

__device__ __forceinline__ int code_of_d(double w, double s, int lim)
{
	if (s <= 0) return 0;
	double r = rint(__ddiv_rn(w, s)); // nearbyint in round-to-nearest-even
	return (int)(r > lim ? lim : r < -lim ? -lim : r);
}

__global__ void rtn_scales(const float *__restrict__ w, int C, int K, int axis, int lim, double *__restrict__ sd,
			   float *__restrict__ sf)
{
	int c = blockIdx.x * blockDim.x + threadIdx.x;
	if (c >= C) return;
	// element j of channel c: axis 0 -> row c (w[c*K + j]); axis 1 -> column c (w[j*C + c])
	long base = axis == 0 ? (long)c * K : c;
	long step = axis == 0 ? 1 : C;
	double amax = 0;
	for (int j = 0; j < K; j++) {
		double v = fabs((double)w[base + j * step]);
		if (v > amax) amax = v;
	}
	double bs;
	if (amax == 0) {
		bs = 1e-8;
	} else {
		double best = INFINITY;
		bs = __ddiv_rn(amax, (double)lim);
		for (int g = 0; g < 10; g++) {
			double s = __ddiv_rn(__dmul_rn(amax, __dsub_rn(1.0, __dmul_rn(0.05, (double)g))), (double)lim);
			double e = 0;
			for (int j = 0; j < K; j++) {
				double x = (double)w[base + j * step];
				double d = __dsub_rn(x, __dmul_rn(s, (double)code_of_d(x, s, lim)));
				e = __dadd_rn(e, __dmul_rn(__dmul_rn(d, d), 1.0));
			}
			if (e < best) {
				best = e;
				bs = s;
			}
		}
	}
	sd[c] = bs;
	sf[c] = (float)bs;
}

__global__ void rtn_codes(const float *__restrict__ w, int C, int K, int axis, int bits, int lim,
			  const double *__restrict__ sd, signed char *__restrict__ q, long nbytes)
{
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	if (t >= nbytes) return;
	long n = (long)C * K;
	auto code = [&](long e) -> int {
		// element e of the row-major [rows, cols] matrix belongs to channel e/K (axis 0) or e%C (axis 1)
		int c = axis == 0 ? (int)(e / K) : (int)(e % C);
		return code_of_d((double)w[e], sd[c], lim);
	};
	if (bits == 8) {
		q[t] = (signed char)code(t);
		return;
	}
	int lo = code(2 * t), hi = 2 * t + 1 < n ? code(2 * t + 1) : 0;
	q[t] = (signed char)(unsigned char)((lo & 0x0f) | ((unsigned)hi << 4));
}

static DevBuf g_sd[64];

int quantize_rtn(const float *w, int rows, int cols, int axis, int bits, signed char *q, float *s, cudaStream_t st)
{
	int C = axis == 0 ? rows : cols, K = axis == 0 ? cols : rows, dev;
	cudaGetDevice(&dev);
	int rc = g_sd[dev].ensure((size_t)C * sizeof(double), dev);
	if (rc) return rc;
	int lim = bits == 8 ? 127 : 7;
	rtn_scales<<<(C + 127) / 128, 128, 0, st>>>(w, C, K, axis, lim, g_sd[dev].as<double>(), s);
	TGC_LAUNCH_CHECK();
	long n = (long)C * K, nbytes = bits == 8 ? n : (n + 1) / 2;
	rtn_codes<<<(unsigned)((nbytes + 255) / 256), 256, 0, st>>>(w, C, K, axis, bits, lim, g_sd[dev].as<double>(), q,
								  nbytes);
	TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

} // namespace tgc

extern "C" int tg_cuda_quantize_rtn(const float *w, int rows, int cols, int axis, int bits, signed char *q, float *s,
				    void *stream)
{
	tgc::clear_err();
	if (!w || !q || !s || rows <= 0 || cols <= 0 || (axis != 0 && axis != 1) || (bits != 8 && bits != 4))
		return tgc::set_err(TG_CUDA_EINVAL, "tg_cuda_quantize_rtn: bad arguments (rows %d cols %d axis %d bits %d)", rows,
				    cols, axis, bits);
	return tgc::quantize_rtn(w, rows, cols, axis, bits, q, s, (cudaStream_t)stream);
}
