// selftest.cu -- tg_cuda_selftest_wait: the bounded-wait path of the tcgen05 kernels, run on
// purpose. One thread initialises an mbarrier that nothing arrives on and waits for it
// with a limit of `cycles` SM clock cycles; the wait gives up, writes ST_TIMEOUT_FULL into
// the status word and the kernel returns. Nothing faults or hangs: the host reads the
// status, and the context stays usable for the next call.
#include "common.cuh"
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
