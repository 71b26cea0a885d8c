// common.cuh -- shared internals of libtgcuda: status handling, device
// selection, fault injection and small device helpers.
#pragma once

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
