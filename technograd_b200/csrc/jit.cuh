// jit.cuh -- run-time compilation of generated CUDA source for sm_100a (NVRTC, loaded
// on first use) and launching of the resulting kernel through the driver API (entry
// points obtained from the runtime, no link-time dependency on libcuda).
#pragma once

#include <string>
#include <vector>

#include "common.cuh"

namespace tgc {

struct JitModule {
	void *mod = nullptr;  // CUmodule
	void *func = nullptr; // CUfunction
	int dev = -1;
	JitModule() = default;
	JitModule(const JitModule &) = delete; // owns the module: unloaded once, by the destructor
	JitModule &operator=(const JitModule &) = delete;
	~JitModule();
};

// Compiles `src` to a cubin for sm_100a (cached in-process by source text). Needs no GPU.
int jit_compile(const std::string &src, std::vector<char> &cubin, std::string &log);

// Compiles `src` (one extern "C" __global__ function named `entry`) to a cubin for
// sm_100a and loads it on device `dev`. Returns TG_CUDA_OK, or an error status with the
// compiler log in `log` (TG_CUDA_EUNSUPPORTED when NVRTC is not available).
int jit_build(const std::string &src, const char *entry, int dev, size_t max_dyn_smem, JitModule &out, std::string &log);

// Launches a loaded kernel with an argument array (pointers to the argument values).
int jit_launch(const JitModule &m, unsigned grid, unsigned block, size_t smem, cudaStream_t st, void **args);

} // namespace tgc
