// jit.cu -- NVRTC compilation and driver-API launch of generated kernels (jit.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <map>
#include <mutex>
#include <vector>

#include "jit.cuh"

namespace tgc {

namespace {

struct Nvrtc {
	bool ok = false;
	decltype(&nvrtcCreateProgram) create = nullptr;
	decltype(&nvrtcCompileProgram) compile = nullptr;
	decltype(&nvrtcGetProgramLogSize) logsize = nullptr;
	decltype(&nvrtcGetProgramLog) getlog = nullptr;
	decltype(&nvrtcGetCUBINSize) cubinsize = nullptr;
	decltype(&nvrtcGetCUBIN) getcubin = nullptr;
	decltype(&nvrtcDestroyProgram) destroy = nullptr;
};

struct Driver {
	bool ok = false;
	PFN_cuModuleLoadData_v2000 load = nullptr;
	PFN_cuModuleUnload_v2000 unload = nullptr;
	PFN_cuModuleGetFunction_v2000 getfn = nullptr;
	PFN_cuFuncSetAttribute_v9000 setattr = nullptr;
	PFN_cuFuncGetAttribute_v2020 getattr = nullptr;
	PFN_cuLaunchKernel_v4000 launch = nullptr;
};

Nvrtc &nvrtc()
{
	static Nvrtc N;
	static std::once_flag once;
	std::call_once(once, [] {
		const char *names[] = { "/usr/local/cuda/lib64/libnvrtc.so.12", "libnvrtc.so.12", "libnvrtc.so" };
		void *h = nullptr;
		for (const char *n : names)
			if ((h = dlopen(n, RTLD_NOW | RTLD_LOCAL))) break;
		if (!h) return;
		N.create = (decltype(N.create))dlsym(h, "nvrtcCreateProgram");
		N.compile = (decltype(N.compile))dlsym(h, "nvrtcCompileProgram");
		N.logsize = (decltype(N.logsize))dlsym(h, "nvrtcGetProgramLogSize");
		N.getlog = (decltype(N.getlog))dlsym(h, "nvrtcGetProgramLog");
		N.cubinsize = (decltype(N.cubinsize))dlsym(h, "nvrtcGetCUBINSize");
		N.getcubin = (decltype(N.getcubin))dlsym(h, "nvrtcGetCUBIN");
		N.destroy = (decltype(N.destroy))dlsym(h, "nvrtcDestroyProgram");
		N.ok = N.create && N.compile && N.logsize && N.getlog && N.cubinsize && N.getcubin && N.destroy;
	});
	return N;
}

Driver &driver()
{
	static Driver D;
	static std::once_flag once;
	std::call_once(once, [] {
		auto get = [](const char *name, int ver) -> void * {
			void *fn = nullptr;
			cudaDriverEntryPointQueryResult q;
			if (cudaGetDriverEntryPointByVersion(name, &fn, ver, cudaEnableDefault, &q) != cudaSuccess ||
			    q != cudaDriverEntryPointSuccess)
				return nullptr;
			return fn;
		};
		D.load = (PFN_cuModuleLoadData_v2000)get("cuModuleLoadData", 2000);
		D.unload = (PFN_cuModuleUnload_v2000)get("cuModuleUnload", 2000);
		D.getfn = (PFN_cuModuleGetFunction_v2000)get("cuModuleGetFunction", 2000);
		D.setattr = (PFN_cuFuncSetAttribute_v9000)get("cuFuncSetAttribute", 9000);
		D.getattr = (PFN_cuFuncGetAttribute_v2020)get("cuFuncGetAttribute", 2020);
		D.launch = (PFN_cuLaunchKernel_v4000)get("cuLaunchKernel", 4000);
		D.ok = D.load && D.unload && D.getfn && D.setattr && D.getattr && D.launch;
	});
	return D;
}

} // namespace

JitModule::~JitModule()
{
	if (mod && driver().ok) {
		int cur = -1;
		cudaGetDevice(&cur);
		cudaSetDevice(dev); // the module belongs to this device's primary context
		driver().unload((CUmodule)mod);
		if (cur >= 0) cudaSetDevice(cur);
	}
}

// Compiled cubins by source text: a program loaded again, or on another device, is not
// compiled twice.
static std::mutex cache_mu;
static std::map<std::string, std::vector<char>> cache;

int jit_compile(const std::string &src, std::vector<char> &cubin, std::string &log)
{
	{
		std::lock_guard<std::mutex> lk(cache_mu);
		auto it = cache.find(src);
		if (it != cache.end()) {
			cubin = it->second;
			return TG_CUDA_OK;
		}
	}
	Nvrtc &N = nvrtc();
	if (!N.ok) return set_err(TG_CUDA_EUNSUPPORTED, "NVRTC is not available");
	nvrtcProgram prog;
	if (N.create(&prog, src.c_str(), "tgjit.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
		return set_err(TG_CUDA_ECUDA, "nvrtcCreateProgram failed");
	const char *opts[] = { "-arch=sm_100a", "--std=c++17", "-default-device", "-lineinfo" };
	nvrtcResult r = N.compile(prog, (int)(sizeof opts / sizeof *opts), opts);
	size_t ls = 0;
	N.logsize(prog, &ls);
	log.assign(ls, '\0');
	if (ls) N.getlog(prog, &log[0]);
	if (r != NVRTC_SUCCESS) {
		N.destroy(&prog);
		return set_err(TG_CUDA_ECUDA, "the generated kernel did not compile: %.300s", log.c_str());
	}
	size_t cs = 0;
	N.cubinsize(prog, &cs);
	cubin.resize(cs);
	N.getcubin(prog, cubin.data());
	N.destroy(&prog);
	std::lock_guard<std::mutex> lk(cache_mu);
	cache[src] = cubin;
	return TG_CUDA_OK;
}

int jit_build(const std::string &src, const char *entry, int dev, size_t max_dyn_smem, JitModule &out, std::string &log)
{
	Driver &D = driver();
	if (!D.ok) return set_err(TG_CUDA_EUNSUPPORTED, "driver module entry points are not available");
	std::vector<char> cubin;
	int rc = jit_compile(src, cubin, log);
	if (rc) return rc;
	TGC_CUDA(cudaSetDevice(dev));
	TGC_CUDA(cudaFree(nullptr)); // the device's primary context is current from here on
	CUmodule mod;
	CUfunction fn;
	if (D.load(&mod, cubin.data()) != CUDA_SUCCESS) return set_err(TG_CUDA_ECUDA, "cuModuleLoadData failed");
	if (D.getfn(&fn, mod, entry) != CUDA_SUCCESS) {
		D.unload(mod);
		return set_err(TG_CUDA_ECUDA, "cuModuleGetFunction(%s) failed", entry);
	}
	// generated kernels run from registers only: one that needs local memory (an arena
	// indexed at run time, spills, a library slow path with a local array) is not used
	int lmem = -1;
	if (D.getattr(&lmem, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, fn) != CUDA_SUCCESS || lmem != 0) {
		D.unload(mod);
		return set_err(TG_CUDA_EUNSUPPORTED, "the generated kernel needs %d bytes of local memory per thread", lmem);
	}
	if (max_dyn_smem > 48 * 1024 &&
	    D.setattr(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)max_dyn_smem) != CUDA_SUCCESS) {
		D.unload(mod);
		return set_err(TG_CUDA_ECUDA, "cuFuncSetAttribute failed");
	}
	out.mod = mod;
	out.func = fn;
	out.dev = dev;
	return TG_CUDA_OK;
}

int jit_launch(const JitModule &m, unsigned grid, unsigned block, size_t smem, cudaStream_t st, void **args)
{
	if (driver().launch((CUfunction)m.func, grid, 1, 1, block, 1, 1, (unsigned)smem, (CUstream)st, args, nullptr) != CUDA_SUCCESS)
		return set_err(TG_CUDA_ECUDA, "cuLaunchKernel failed");
	return TG_CUDA_OK;
}

} // namespace tgc
