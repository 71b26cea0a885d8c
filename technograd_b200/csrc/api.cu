// api.cu -- device selection, errors and fault injection of libtgcuda.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <mutex>

#include "common.cuh"

namespace tgc {

static thread_local char g_err[1024];
static std::vector<Device> g_devs;
static std::mutex g_mu;

int set_err(int status, const char *fmt, ...)
{
	va_list ap;
	va_start(ap, fmt);
	vsnprintf(g_err, sizeof g_err, fmt, ap);
	va_end(ap);
	return status;
}

void clear_err() { g_err[0] = 0; }

bool fault(const char *step)
{
	const char *f = getenv("TG_CUDA_FAULT");
	return f && strcmp(f, step) == 0;
}

std::vector<Device> &devices() { return g_devs; }
bool inited() { return !g_devs.empty(); }

// Caller ranges page-locked through tg_cuda_host_register: start -> bytes.
static std::map<uintptr_t, size_t> g_host;
static std::mutex g_host_mu;

bool host_registered(const void *p, size_t n)
{
	if (n == 0) return true;
	const uintptr_t a = (uintptr_t)p;
	std::lock_guard<std::mutex> lk(g_host_mu);
	auto it = g_host.upper_bound(a);
	if (it == g_host.begin()) return false;
	--it;
	const size_t off = a - it->first;
	return off < it->second && n <= it->second - off;
}

int DevBuf::alloc(size_t n, int device)
{
	release();
	if (fault("alloc")) return set_err(TG_CUDA_EFAULT, "injected allocation failure (TG_CUDA_FAULT=alloc)");
	int prev;
	cudaGetDevice(&prev);
	cudaSetDevice(device);
	cudaError_t e = cudaMalloc(&p, n ? n : 16);
	cudaSetDevice(prev);
	if (e != cudaSuccess) {
		p = nullptr;
		return set_err(TG_CUDA_ENOMEM, "cudaMalloc(%zu) on device %d: %s", n, device, cudaGetErrorString(e));
	}
	bytes = n;
	dev = device;
	return TG_CUDA_OK;
}

void DevBuf::release()
{
	if (p) {
		int prev;
		cudaGetDevice(&prev);
		cudaSetDevice(dev);
		cudaFree(p);
		cudaSetDevice(prev);
	}
	p = nullptr;
	bytes = 0;
	dev = -1;
}

} // namespace tgc

using namespace tgc;

extern "C" const char *tg_cuda_error(void) { return g_err; }

extern "C" int tg_cuda_init(int ngpus, const int *devs)
{
	std::lock_guard<std::mutex> lk(g_mu);
	clear_err();
	int count = 0;
	cudaError_t e = cudaGetDeviceCount(&count);
	if (e != cudaSuccess || count == 0)
		return set_err(TG_CUDA_ENODEV, "no CUDA device: %s", e != cudaSuccess ? cudaGetErrorString(e) : "count 0");
	std::vector<int> want;
	if (devs && ngpus > 0) {
		for (int i = 0; i < ngpus; i++) {
			if (devs[i] < 0 || devs[i] >= count) return set_err(TG_CUDA_EINVAL, "device %d not visible (%d devices)", devs[i], count);
			want.push_back(devs[i]);
		}
	} else {
		int n = ngpus > 0 && ngpus < count ? ngpus : count;
		for (int i = 0; i < n; i++) want.push_back(i);
	}
	if (!g_devs.empty()) {
		bool same = g_devs.size() == want.size();
		for (size_t i = 0; same && i < want.size(); i++) same = g_devs[i].id == want[i];
		if (same) return TG_CUDA_OK;
		return set_err(TG_CUDA_EINVAL, "tg_cuda_init: already initialised with another device set; call tg_cuda_shutdown first");
	}
	for (int id : want) {
		cudaDeviceProp prop;
		TGC_CUDA(cudaGetDeviceProperties(&prop, id));
		if (prop.major != 10)
			return set_err(TG_CUDA_ENODEV, "device %d is sm_%d%d; this library is built for sm_100a only", id, prop.major, prop.minor);
		Device d;
		d.id = id;
		d.sms = prop.multiProcessorCount;
		TGC_CUDA(cudaSetDevice(id));
		TGC_CUDA(cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking));
		g_devs.push_back(d);
	}
	TGC_CUDA(cudaSetDevice(g_devs[0].id));
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_ngpus(void) { return (int)g_devs.size(); }

extern "C" int tg_cuda_host_register(void *p, size_t bytes)
{
	clear_err();
	if (!p || bytes == 0) return set_err(TG_CUDA_EINVAL, "tg_cuda_host_register: NULL or empty range");
	if (!inited()) return set_err(TG_CUDA_ENODEV, "tg_cuda_host_register: call tg_cuda_init first");
	std::lock_guard<std::mutex> lk(g_host_mu);
	cudaError_t e = cudaHostRegister(p, bytes, cudaHostRegisterPortable);
	if (e != cudaSuccess) {
		cudaGetLastError();
		return set_err(e == cudaErrorHostMemoryAlreadyRegistered ? TG_CUDA_EINVAL : TG_CUDA_ECUDA,
			       "tg_cuda_host_register(%zu bytes): %s", bytes, cudaGetErrorString(e));
	}
	g_host[(uintptr_t)p] = bytes;
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_host_unregister(void *p)
{
	clear_err();
	std::lock_guard<std::mutex> lk(g_host_mu);
	auto it = g_host.find((uintptr_t)p);
	if (it == g_host.end()) return set_err(TG_CUDA_EINVAL, "tg_cuda_host_unregister: %p is not the start of a registered range", p);
	g_host.erase(it);
	cudaError_t e = cudaHostUnregister(p);
	if (e != cudaSuccess) {
		cudaGetLastError();
		return set_err(TG_CUDA_ECUDA, "cudaHostUnregister: %s", cudaGetErrorString(e));
	}
	return TG_CUDA_OK;
}

extern "C" void tg_cuda_shutdown(void)
{
	{
		std::lock_guard<std::mutex> lk(g_host_mu);
		for (auto &r : g_host) cudaHostUnregister((void *)r.first);
		g_host.clear();
	}
	std::lock_guard<std::mutex> lk(g_mu);
	for (auto &d : g_devs) {
		cudaSetDevice(d.id);
		cudaStreamSynchronize(d.stream);
		cudaStreamDestroy(d.stream);
	}
	g_devs.clear();
}
