// matmul.cu -- tg_cuda_matmul_q: the kernel-level drop-in for tg_matmul_qa (axis 0)
// and tg_matmul_qb (axis 1), runtime/tg_rt.h:132-151, on device pointers.
//
// Dispatch: a batch of at most 8 (n for axis 0, m for axis 1) streams the codes
// through the CUDA-core GEMV of gemv.cu; larger batches go to the tensor-core
// dequant GEMM (gemm_sm100.cu); shapes neither supports (unaligned code rows)
// run the one-thread-per-output kernel that reproduces the reference rounding.
#include "common.cuh"
#include "kernels.cuh"

using namespace tgc;

extern "C" int tg_cuda_matmul_q(int axis, float *o, const float *act, const signed char *q, int bits, const float *s, int m,
				int k, int n, void *stream)
{
	clear_err();
	if (!o || !act || !q || !s) return set_err(TG_CUDA_EINVAL, "tg_cuda_matmul_q: NULL pointer");
	if ((axis != 0 && axis != 1) || (bits != 8 && bits != 4) || m <= 0 || k <= 0 || n <= 0)
		return set_err(TG_CUDA_EINVAL, "tg_cuda_matmul_q: bad arguments (axis %d bits %d m %d k %d n %d)", axis, bits, m, k, n);
	cudaStream_t st = (cudaStream_t)stream;
	bool done = false;
	int rc = matmul_q_gemv(axis, o, act, q, bits, s, m, k, n, st, &done);
	if (rc || done) return rc;
	rc = matmul_q_tc(axis, o, act, q, bits, s, m, k, n, st, &done);
	if (rc || done) return rc;
	return matmul_q_exact(axis, o, act, q, bits, s, m, k, n, st);
}
