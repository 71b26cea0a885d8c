// lm.cu -- decoder language models (the Qwen3 import) on the device.
#include "common.cuh"
#include "kernels.cuh"

using namespace tgc;

struct tg_cuda_lm {
	int unused;
};

extern "C" int tg_cuda_lm_load(const tg_cuda_lm_desc *d, int max_seqs, int max_len, tg_cuda_lm **out)
{
	(void)d; (void)max_seqs; (void)max_len;
	if (out) *out = nullptr;
	return set_err(TG_CUDA_EUNSUPPORTED, "tg_cuda_lm_load: not built yet");
}
extern "C" int tg_cuda_lm_forward(tg_cuda_lm *g, const float *ids, long nseq, int T, float *logits)
{
	(void)g; (void)ids; (void)nseq; (void)T; (void)logits;
	return set_err(TG_CUDA_EUNSUPPORTED, "tg_cuda_lm_forward: not built yet");
}
extern "C" int tg_cuda_lm_generate(tg_cuda_lm *g, const float *ids, long nseq, int T, int nnew, int *tokens)
{
	(void)g; (void)ids; (void)nseq; (void)T; (void)nnew; (void)tokens;
	return set_err(TG_CUDA_EUNSUPPORTED, "tg_cuda_lm_generate: not built yet");
}
extern "C" void tg_cuda_lm_free(tg_cuda_lm *g) { delete g; }
