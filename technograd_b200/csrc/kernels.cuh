// kernels.cuh -- internal entry points shared between the library's .cu files.
#pragma once

#include "common.cuh"

namespace tgc {

// gemv.cu
int matmul_q_exact(int axis, float *o, const float *act, const signed char *q, int bits, const float *s, int m, int k,
		   int n, cudaStream_t st);
int matmul_q_gemv(int axis, float *o, const float *act, const signed char *q, int bits, const float *s, int m, int k,
		  int n, cudaStream_t st, bool *done);

// gemm_sm100.cu: tensor-core path for large batches; *done = false when the shape is not taken
int matmul_q_tc(int axis, float *o, const float *act, const signed char *q, int bits, const float *s, int m, int k, int n,
		cudaStream_t st, bool *done);

// quant.cu
int quantize_rtn(const float *w, int rows, int cols, int axis, int bits, signed char *q, float *s, cudaStream_t st);

} // namespace tgc
