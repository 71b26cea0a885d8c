// selftest.cu -- tg_cuda_selftest_wait: the bounded-wait path of the tcgen05 kernels, run on
// purpose. One thread initialises an mbarrier that nothing arrives on and waits for it
// with a limit of `cycles` SM clock cycles; the wait gives up, writes ST_TIMEOUT_FULL into
// the status word and the kernel returns. Nothing faults or hangs: the host reads the
// status, and the context stays usable for the next call.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"
#include "tc.cuh"

namespace tgc {

__global__ void k_selftest_wait(long long cycles, int *status, int *outcome)
{
	__shared__ uint64_t bar;
	if (threadIdx.x == 0) {
		mbar_init(&bar, 1);
		fence_barrier_init();
	}
	__syncthreads();
	if (threadIdx.x == 0) *outcome = mbar_wait_for(&bar, 0, status, ST_TIMEOUT_FULL, cycles) ? 1 : 2;
}

} // namespace tgc

using namespace tgc;

extern "C" int tg_cuda_selftest_wait(long long cycles, int *status)
{
	clear_err();
	if (!inited()) return set_err(TG_CUDA_ENODEV, "tg_cuda_selftest_wait: call tg_cuda_init first");
	if (cycles <= 0 || cycles > 4000000000ll) return set_err(TG_CUDA_EINVAL, "tg_cuda_selftest_wait: cycles out of range");
	cudaSetDevice(devices()[0].id);
	DevBuf buf;
	int rc = buf.alloc(2 * sizeof(int), devices()[0].id);
	if (rc) return rc;
	TGC_CUDA(cudaMemset(buf.p, 0, 2 * sizeof(int)));
	k_selftest_wait<<<1, 32>>>(cycles, buf.as<int>(), buf.as<int>() + 1);
	TGC_LAUNCH_CHECK();
	int h[2];
	TGC_CUDA(cudaMemcpy(h, buf.p, sizeof h, cudaMemcpyDeviceToHost));
	if (status) *status = h[0];
	if (h[1] != 2) return set_err(TG_CUDA_ECUDA, "tg_cuda_selftest_wait: the wait did not give up (outcome %d)", h[1]);
	return set_err(TG_CUDA_EDEVICE, "a wait gave up as asked (status %d)", h[0]);
}

// The decode GEMM on the caller's device buffers, through either kernel, for the tests:
// the tile kernel (path 0, gemm_sm100.cu, with its split-K scratch) or the swapped-operand
// cluster kernel (path 1, gemm_sk.cu). Synchronous; the status word is checked.
extern "C" int tg_cuda_selftest_gemm(int path, const void *const *a, int na, const void *const *b, int nb, int npairs,
				     const int *pa, const int *pb, int m, int n, int k, int epi, const float *scale,
				     const float *scale2, float *out, long ldo, void *out_hi, void *out_lo, void *stream)
{
	clear_err();
	if (!inited()) return set_err(TG_CUDA_ENODEV, "tg_cuda_selftest_gemm: call tg_cuda_init first");
	if ((path != 0 && path != 1) || !a || !b || na < 1 || na > 2 || nb < 1 || nb > 2 || npairs < 1 || npairs > 4 || !pa ||
	    !pb || m <= 0 || n <= 0 || k <= 0 || epi < EPI_STORE || epi > EPI_SWIGLU)
		return set_err(TG_CUDA_EINVAL, "tg_cuda_selftest_gemm: bad arguments");
	int dev;
	TGC_CUDA(cudaGetDevice(&dev));
	cudaStream_t st = (cudaStream_t)stream;
	GemmOperands ops;
	for (int i = 0; i < na; i++) ops.a[i] = a[i];
	for (int j = 0; j < nb; j++) ops.b[j] = b[j];
	ops.lda = k, ops.ldb = k;
	GemmArgs p;
	memset(&p, 0, sizeof p);
	p.M = m, p.N = n, p.K = k, p.na = na, p.nb = nb, p.npairs = npairs;
	for (int q = 0; q < npairs; q++) {
		if (pa[q] < 0 || pa[q] >= na || pb[q] < 0 || pb[q] >= nb) return set_err(TG_CUDA_EINVAL, "pair %d out of range", q);
		p.pa[q] = pa[q], p.pb[q] = pb[q];
	}
	p.epi = epi;
	p.scale = scale, p.scale2 = scale2, p.scale_mode = epi != EPI_SWIGLU && scale ? 2 : 0;
	p.out = out, p.ldo = ldo, p.out_hi = (__nv_bfloat16 *)out_hi, p.out_lo = (__nv_bfloat16 *)out_lo;
	DevBuf status, part;
	int rc;
	if ((rc = status.alloc(64, dev))) return rc;
	TGC_CUDA(cudaMemsetAsync(status.p, 0, 64, st));
	p.status = status.as<int>();
	{ // the tile kernel's split-K sums (up to 16 splits of a 128-row-padded batch), or the cluster
	  // kernel's partials (up to 4 ranks of 128-channel x 256-row tiles)
		const long mpad = ((long)m + 255) / 256 * 256, npad = ((long)n + 127) / 128 * 128;
		const long floats = std::max(16 * mpad * n, 4 * mpad * npad);
		if ((rc = part.alloc((size_t)floats * sizeof(float), dev))) return rc;
		p.partial = part.as<float>(), p.partial_floats = floats;
	}
	if (path == 0) {
		rc = gemm(ops, p, st);
	} else {
		if ((rc = gemm_sk_prepare())) return rc;
		rc = gemm_sk(ops, p, st);
	}
	if (rc) return rc;
	TGC_CUDA(cudaStreamSynchronize(st));
	return device_status_check(status.as<int>(), st);
}
