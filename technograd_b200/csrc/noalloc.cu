// noalloc.cu -- tg_cuda_matmul_qb_noalloc: the small-batch x @ W dequant GEMV
// without any allocation.
//
// Who needs it: callers that must not allocate device memory while they run.
// The reference's own batch workers are one example -- functions run by
// par_for must not allocate, trace or die (src/par.c:11-12), because its
// allocator is single-threaded -- and so are hosts that budget all device
// memory up front, or that call from a context where a cudaMalloc could block
// or fail mid-run. tg_cuda_matmul_q allocates (and caches) its split-K scratch
// on first use; this variant never does. Its partial sums live in the
// file-scope array below, which every GPU that loads the library holds for the
// life of the process.
//
// Set-up: the array's name in host code is only a host-side stand-in, not a
// device address. The first call on each device, with that device current,
// looks the address up with cudaGetSymbolAddress and caches it; make that first
// call before any stream capture. Every call then passes the cached pointer to
// the kernels.
//
// Sharing: all calls on a device use the same array. Each call writes every
// partial sum it later reads, so nothing has to be cleared first. A call holds a
// per-device lock while it enqueues its two kernels, so calls from several host
// threads on the SAME stream (the reference's par_for workers sharing the NULL
// stream, say) run one after the other on the GPU. Calls on DIFFERENT streams
// can still overlap on the GPU and race on the array, corrupting each other's
// results: such callers must order them (one stream per device, or events).
//
// The cached address is per device ordinal for the life of the process, so
// cudaDeviceReset is not supported while the library is loaded.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemv_cols.cuh"

namespace tgc {

// 4 MiB of f32 partial sums per device.
constexpr long NOALLOC_SCRATCH_FLOATS = 1L << 20;
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_SCRATCH_FLOATS];

constexpr int NOALLOC_MAX_DEVICES = 64;
static float *g_scratch_addr[NOALLOC_MAX_DEVICES];
static int g_scratch_sms[NOALLOC_MAX_DEVICES];
static std::mutex g_scratch_mu;                           // guards the two tables above
static std::mutex g_dev_mu[NOALLOC_MAX_DEVICES];          // held while a call enqueues its kernels

// The current device, the device address of g_noalloc_scratch on it and its SM count
// (looked up once per device, with that device current).
static int scratch_address(int *dev_out, float **out, int *sms_out)
{
	int dev = -1;
	cudaError_t e = cudaGetDevice(&dev);
	if (e != cudaSuccess) return set_err(TG_CUDA_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
	if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return set_err(TG_CUDA_EINVAL, "device ordinal %d", dev);
	std::lock_guard<std::mutex> lk(g_scratch_mu);
	if (!g_scratch_addr[dev]) {
		int sms = 0;
		e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
		if (e != cudaSuccess || sms <= 0)
			return set_err(TG_CUDA_ECUDA, "cudaDeviceGetAttribute(SM count) on device %d: %s", dev, cudaGetErrorString(e));
		g_scratch_sms[dev] = sms;
		void *p = nullptr;
		e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
		if (e != cudaSuccess || !p)
			return set_err(TG_CUDA_ECUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev, cudaGetErrorString(e));
		g_scratch_addr[dev] = (float *)p;
	}
	*dev_out = dev;
	*out = g_scratch_addr[dev];
	*sms_out = g_scratch_sms[dev];
	return TG_CUDA_OK;
}

template <int BITS>
static int run(float *o, const float *a, const signed char *q, const float *s, int m, int k, int n, float *part,
	       int sms, cudaStream_t st)
{
	constexpr int CPW = BITS == 8 ? 4 : 8;
	int tiles = (n + 32 * CPW - 1) / (32 * CPW);
	int want = (4 * sms + tiles - 1) / tiles; // about four CTAs per SM, as tg_cuda_matmul_q
	int cap = k / 64 > 0 ? k / 64 : 1;
	int fit = (int)(NOALLOC_SCRATCH_FLOATS / ((long)m * n)); // splits the array can hold
	int splits = std::max(1, std::min(std::min(want, cap), fit));
	int kper = (k + splits - 1) / splits;
	splits = (k + kper - 1) / kper;
	dim3 grid(tiles, splits);
	switch (m) {
#define MB_CASE(M) \
	case M: gemv_cols<BITS, M><<<grid, GC_WARPS * 32, 0, st>>>(part, a, q, m, k, n, kper); break;
		MB_CASE(1) MB_CASE(2) MB_CASE(3) MB_CASE(4) MB_CASE(5) MB_CASE(6) MB_CASE(7) MB_CASE(8)
#undef MB_CASE
	}
	TGC_LAUNCH_CHECK();
	long tot = (long)m * n;
	reduce_splits<<<(unsigned)((tot + 255) / 256), 256, 0, st>>>(o, part, s, m, n, splits);
	TGC_LAUNCH_CHECK();
	return TG_CUDA_OK;
}

} // namespace tgc

using namespace tgc;

extern "C" int tg_cuda_matmul_qb_noalloc(float *o, const float *act, const signed char *q, int bits, const float *s, int m,
					 int k, int n, void *stream)
{
	clear_err();
	if (!o || !act || !q || !s) return set_err(TG_CUDA_EINVAL, "tg_cuda_matmul_qb_noalloc: NULL pointer");
	if ((bits != 8 && bits != 4) || m <= 0 || k <= 0 || n <= 0)
		return set_err(TG_CUDA_EINVAL, "tg_cuda_matmul_qb_noalloc: bad arguments (bits %d m %d k %d n %d)", bits, m, k, n);
	if (m > 8)
		return set_err(TG_CUDA_EINVAL, "tg_cuda_matmul_qb_noalloc: batch m = %d exceeds the maximum of 8 rows", m);
	if ((long)m * n > NOALLOC_SCRATCH_FLOATS)
		return set_err(TG_CUDA_EINVAL,
			       "tg_cuda_matmul_qb_noalloc: m * n = %ld exceeds the %ld partial sums its fixed scratch holds",
			       (long)m * n, NOALLOC_SCRATCH_FLOATS);
	if (n % (bits == 8 ? 4 : 8) || ((uintptr_t)q & 3))
		return set_err(TG_CUDA_EINVAL,
			       "tg_cuda_matmul_qb_noalloc: n must be a multiple of %d and the codes 4-byte aligned", bits == 8 ? 4 : 8);
	float *part = nullptr;
	int dev = -1, sms = 0;
	int rc = scratch_address(&dev, &part, &sms);
	if (rc) return rc;
	cudaStream_t st = (cudaStream_t)stream;
	// both kernels of this call enqueue before any other call's on this device
	std::lock_guard<std::mutex> lk(g_dev_mu[dev]);
	return bits == 8 ? run<8>(o, act, q, s, m, k, n, part, sms, st) : run<4>(o, act, q, s, m, k, n, part, sms, st);
}
