// common.cuh -- shared internals of libtgcuda: status handling, device
// selection, fault injection and small device helpers.
#pragma once

#include <utility>

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <string>
#include <vector>

#include "../../include/tg_cuda.h"

namespace tgc {

// Thread-local last error; set_err returns the status so `return set_err(...)` reads naturally.
int set_err(int status, const char *fmt, ...);
void clear_err();

// Fault injection for host-side failure tests: TG_CUDA_FAULT=alloc|h2d|launch|gather makes
// the named step report TG_CUDA_EFAULT instead of running (no GPU fault is ever produced).
bool fault(const char *step);

struct Device {
	int id;
	int sms;
	cudaStream_t stream;
};

// Row sizes of a loaded model (values per row, outputs per row, think-step slots).
int model_shape(const tg_cuda_model *g, int *per, int *nout, int *nthink);

// Devices chosen by tg_cuda_init, in shard order.
std::vector<Device> &devices();
bool inited();

// True when [p, p + n) lies inside one range registered with tg_cuda_host_register.
bool host_registered(const void *p, size_t n);

#define TGC_CUDA(call)                                                                                    \
	do {                                                                                              \
		cudaError_t e_ = (call);                                                                  \
		if (e_ != cudaSuccess)                                                                    \
			return ::tgc::set_err(TG_CUDA_ECUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
					      __FILE__, __LINE__);                                        \
	} while (0)

#define TGC_LAUNCH_CHECK()                                                                                   \
	do {                                                                                                 \
		cudaError_t e_ = cudaGetLastError();                                                         \
		if (e_ != cudaSuccess)                                                                       \
			return ::tgc::set_err(TG_CUDA_ECUDA, "kernel launch: %s (%s:%d)", cudaGetErrorString(e_), \
					      __FILE__, __LINE__);                                           \
	} while (0)

// A device buffer owned by the library.
struct DevBuf {
	void *p = nullptr;
	size_t bytes = 0;
	int dev = -1;
	DevBuf() = default;
	DevBuf(const DevBuf &) = delete;
	DevBuf &operator=(const DevBuf &) = delete;
	~DevBuf() { release(); }
	int alloc(size_t n, int device);
	int ensure(size_t n, int device) { return n <= bytes && device == dev ? TG_CUDA_OK : alloc(n, device); }
	void release();
	template <class T> T *as() const { return (T *)p; }
};

// Programmatic dependent launch. A kernel launched with the programmatic-serialization
// attribute (launch_pdl) may start while the kernel before it on the stream is finishing;
// pdl_wait() blocks the calling thread until that kernel has completed and its writes are
// visible, so every thread calls it before it reads data a previous kernel may write or
// writes data one may read. pdl_launch() lets the next such kernel start early. Both are
// no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// L2 prefetch of a contiguous global range (16-byte aligned, bytes a multiple of 16). L2 is
// where every device write lands first, so prefetching before pdl_wait reads no stale data.
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes)
{
	asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((uint64_t)p), "r"(bytes) : "memory");
}

template <class... KArgs, class... Args>
static inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
				     Args &&...args)
{
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = grid, cfg.blockDim = block, cfg.dynamicSmemBytes = smem, cfg.stream = st;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = attr, cfg.numAttrs = 1;
	return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Decoding of the reference's int4 packing: element e in byte e/2, low nibble first,
// sign-extended (runtime/tg_rt.h:124-129).
__device__ __forceinline__ int qcode(const signed char *q, int bits, long e)
{
	if (bits == 8) return q[e];
	int b = q[e >> 1];
	return (e & 1) ? (b >> 4) : ((int)(signed char)(b << 4) >> 4);
}

// The two nibbles of a byte, as signed ints.
__device__ __forceinline__ int lo4(uint32_t b) { return (int)((int32_t)(b << 28) >> 28); }
__device__ __forceinline__ int hi4(uint32_t b) { return (int)((int32_t)(b << 24) >> 28); }

} // namespace tgc
