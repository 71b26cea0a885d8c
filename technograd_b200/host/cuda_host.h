/* cuda_host.h -- the reference-side binding of libtgcuda (cuda.c, tgc_cuda.c): a planned
 * Module flattened for the C ABI, and the loaded model. Needs src/tg.h and tg_cuda.h. */
#ifndef TG_CUDA_HOST_H
#define TG_CUDA_HOST_H

typedef struct {
	tg_cuda_program p; /* points into the arrays below and into the Module */
	tg_cuda_value *val;
	tg_cuda_ins *ins;
	tg_cuda_scan *scans;
} CudaFlat;

void cuda_flatten(const Module *m, CudaFlat *cf);
void cuda_flat_free(CudaFlat *cf);
/* tg_cuda_init on every visible GPU + tg_cuda_load; die()s with the library's text on failure */
tg_cuda_model *cuda_load(const Module *m);

#endif
