// gptq.cu -- GPTQ quantization (src/quant.c:92-316) with the per-channel sweep on
// the device, bit-exact with the reference.
//
// Host: H = sum over calibration rows of x x^T in double (src/quant.c:100-116, zero
// inputs skipped), an unused input's diagonal set to 1 with its weights zeroed, 1%
// dampening, and U with H^-1 = U^T U through two Cholesky factorisations
// (src/quant.c:202-253), every loop in the reference's order.
// Device: one thread per output channel runs best_scale with the Hessian diagonal
// as weights (src/quant.c:183-200) and the error feedback w[jj] -= err * U[j][jj]
// (src/quant.c:290-302) in double with explicitly rounded operations; the
// channel's working weights live in a [K][C] scratch so a warp's accesses are
// contiguous, and U's rows are shared by every thread. Codes are written as
// signed bytes into a second scratch and packed afterwards (int4 channels of a
// byte can belong to different threads).
#include <math.h>
#include <string.h>

#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace tgc {

__device__ __forceinline__ int code_of_g(double w, double s, int lim)
{
	if (s <= 0) return 0;
	double r = rint(__ddiv_rn(w, s));
	return (int)(r > lim ? lim : r < -lim ? -lim : r);
}

__global__ void gptq_sweep(const float *__restrict__ w, int C, int K, int axis, int lim, int feedback, const double *__restrict__ U,
			   const double *__restrict__ hd, const unsigned char *__restrict__ dead, double *__restrict__ work,
			   signed char *__restrict__ code8, float *__restrict__ sf)
{
	int c = blockIdx.x * blockDim.x + threadIdx.x;
	if (c >= C) return;
	// element j of channel c: axis 0 -> w[c*K + j]; axis 1 -> w[j*C + c]
	auto col = [&](int j) -> double & { return work[(long)j * C + c]; };
	for (int j = 0; j < K; j++) col(j) = dead[j] ? 0.0 : (double)w[axis == 0 ? (long)c * K + j : (long)j * C + c];
	double amax = 0;
	for (int j = 0; j < K; j++) {
		double v = fabs(col(j));
		if (v > amax) amax = v;
	}
	double s;
	if (amax == 0) {
		s = 1e-8;
	} else {
		double best = INFINITY;
		s = __ddiv_rn(amax, (double)lim);
		for (int g = 0; g < 10; g++) {
			double sc = __ddiv_rn(__dmul_rn(amax, __dsub_rn(1.0, __dmul_rn(0.05, (double)g))), (double)lim), e = 0;
			for (int j = 0; j < K; j++) {
				double x = col(j);
				double d = __dsub_rn(x, __dmul_rn(sc, (double)code_of_g(x, sc, lim)));
				e = __dadd_rn(e, __dmul_rn(__dmul_rn(d, d), hd[j]));
			}
			if (e < best) {
				best = e;
				s = sc;
			}
		}
	}
	sf[c] = (float)s;
	for (int j = 0; j < K; j++) {
		double x = col(j);
		int code = code_of_g(x, s, lim);
		code8[axis == 0 ? (long)c * K + j : (long)j * C + c] = (signed char)code;
		if (!feedback) continue;
		double err = __ddiv_rn(__dsub_rn(x, __dmul_rn(s, (double)code)), U[(long)j * K + j]);
		const double *Uj = U + (long)j * K;
		for (int jj = j + 1; jj < K; jj++) col(jj) = __dsub_rn(col(jj), __dmul_rn(err, Uj[jj]));
	}
}

__global__ void pack_codes(const signed char *__restrict__ code8, long n, int bits, signed char *__restrict__ q)
{
	long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
	long nb = bits == 8 ? n : (n + 1) / 2;
	if (t >= nb) return;
	if (bits == 8) {
		q[t] = code8[t];
		return;
	}
	int lo = code8[2 * t], hi = 2 * t + 1 < n ? code8[2 * t + 1] : 0;
	q[t] = (signed char)(unsigned char)((lo & 0x0f) | ((unsigned)hi << 4));
}

// ---- host: Hessian and its inverse factor, in the reference's loop order ------------------------

static int cholesky(double *A, int n)
{
	for (int j = 0; j < n; j++) {
		double d = A[(long)j * n + j];
		for (int k = 0; k < j; k++) d -= A[(long)j * n + k] * A[(long)j * n + k];
		if (d <= 0) return 0;
		d = sqrt(d);
		A[(long)j * n + j] = d;
		for (int i = j + 1; i < n; i++) {
			double s = A[(long)i * n + j];
			for (int k = 0; k < j; k++) s -= A[(long)i * n + k] * A[(long)j * n + k];
			A[(long)i * n + j] = s / d;
		}
		for (int k = j + 1; k < n; k++) A[(long)j * n + k] = 0;
	}
	return 1;
}

static int inv_chol_upper(const double *H, int n, double *U)
{
	size_t nn = (size_t)n * n;
	std::vector<double> L(H, H + nn), Li(nn, 0.0);
	if (!cholesky(L.data(), n)) return 0;
	for (int c = 0; c < n; c++)
		for (int i = c; i < n; i++) {
			double s = i == c ? 1.0 : 0.0;
			for (int k = c; k < i; k++) s -= L[(long)i * n + k] * Li[(long)k * n + c];
			Li[(long)i * n + c] = s / L[(long)i * n + i];
		}
	for (int i = 0; i < n; i++)
		for (int j = i; j < n; j++) {
			double s = 0;
			for (int k = j; k < n; k++) s += Li[(long)k * n + i] * Li[(long)k * n + j];
			U[(long)i * n + j] = U[(long)j * n + i] = s;
		}
	if (!cholesky(U, n)) return 0;
	for (int i = 0; i < n; i++)
		for (int j = i + 1; j < n; j++) {
			U[(long)i * n + j] = U[(long)j * n + i];
			U[(long)j * n + i] = 0;
		}
	return 1;
}

} // namespace tgc

using namespace tgc;

struct tg_cuda_gptq {
	int K = 0, dev = -1;
	bool ok = false; // U exists (H positive definite); otherwise quantization is RTN
	DevBuf U, hd, dead;
};

extern "C" int tg_cuda_gptq_prepare(const float *calib, int nrows, int K, tg_cuda_gptq **out)
{
	clear_err();
	if (!out || !calib || nrows <= 0 || K <= 0) return set_err(TG_CUDA_EINVAL, "tg_cuda_gptq_prepare: bad arguments");
	*out = nullptr;
	if (!inited()) return set_err(TG_CUDA_ENODEV, "tg_cuda_gptq_prepare: call tg_cuda_init first");
	std::vector<double> H((size_t)K * K, 0.0), U((size_t)K * K, 0.0), hd(K);
	std::vector<unsigned char> dead(K, 0);
	for (int r0 = 0; r0 < nrows; r0++) { // src/quant.c:108-115
		const float *x = calib + (long)r0 * K;
		for (int r = 0; r < K; r++) {
			double xr = x[r];
			if (xr == 0) continue;
			for (int c = 0; c < K; c++) H[(long)r * K + c] += xr * x[c];
		}
	}
	double mean = 0; // src/quant.c:270-282
	for (int j = 0; j < K; j++) mean += H[(long)j * K + j];
	mean /= K;
	for (int j = 0; j < K; j++) {
		if (H[(long)j * K + j] == 0) {
			H[(long)j * K + j] = 1;
			dead[j] = 1;
		}
		H[(long)j * K + j] += 0.01 * mean;
		hd[j] = H[(long)j * K + j];
	}
	tg_cuda_gptq *g = new tg_cuda_gptq;
	g->K = K;
	g->ok = inv_chol_upper(H.data(), K, U.data()) != 0;
	int dev;
	cudaGetDevice(&dev);
	g->dev = dev;
	int rc;
	if ((rc = g->U.alloc((size_t)K * K * 8, dev)) || (rc = g->hd.alloc((size_t)K * 8, dev)) || (rc = g->dead.alloc((size_t)K, dev))) {
		delete g;
		return rc;
	}
	TGC_CUDA(cudaMemcpy(g->U.p, U.data(), (size_t)K * K * 8, cudaMemcpyHostToDevice));
	TGC_CUDA(cudaMemcpy(g->hd.p, hd.data(), (size_t)K * 8, cudaMemcpyHostToDevice));
	TGC_CUDA(cudaMemcpy(g->dead.p, dead.data(), (size_t)K, cudaMemcpyHostToDevice));
	TGC_CUDA(cudaDeviceSynchronize());
	*out = g;
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_quantize_gptq(tg_cuda_gptq *g, const float *w, int rows, int cols, int axis, int bits, signed char *q,
				     float *s, void *stream)
{
	clear_err();
	if (!g || !w || !q || !s || rows <= 0 || cols <= 0 || (axis != 0 && axis != 1) || (bits != 8 && bits != 4))
		return set_err(TG_CUDA_EINVAL, "tg_cuda_quantize_gptq: bad arguments");
	const int C = axis == 0 ? rows : cols, K = axis == 0 ? cols : rows;
	if (K != g->K) return set_err(TG_CUDA_EINVAL, "tg_cuda_quantize_gptq: %d inputs per channel, calibration has %d", K, g->K);
	cudaStream_t st = (cudaStream_t)stream;
	static DevBuf work[64], code8[64];
	int dev;
	cudaGetDevice(&dev);
	long n = (long)C * K;
	int rc;
	if ((rc = work[dev].ensure((size_t)n * 8, dev)) || (rc = code8[dev].ensure((size_t)n, dev))) return rc;
	const int lim = bits == 8 ? 127 : 7;
	// H not positive definite: the reference keeps the Hessian-weighted scale search and
	// drops the error feedback (src/quant.c:284-289)
	gptq_sweep<<<(C + 63) / 64, 64, 0, st>>>(w, C, K, axis, lim, g->ok ? 1 : 0, g->U.as<double>(), g->hd.as<double>(), g->dead.as<unsigned char>(),
						 work[dev].as<double>(), code8[dev].as<signed char>(), s);
	TGC_LAUNCH_CHECK();
	long nb = bits == 8 ? n : (n + 1) / 2;
	pack_codes<<<(unsigned)((nb + 255) / 256), 256, 0, st>>>(code8[dev].as<signed char>(), n, bits, q);
	TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

extern "C" void tg_cuda_gptq_free(tg_cuda_gptq *g) { delete g; }
