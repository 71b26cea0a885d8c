// tc.cuh -- Blackwell (sm_100a) building blocks in inline PTX: mbarriers with
// bounded waits, TMA tile loads (no multicast), tcgen05 TMEM allocation, MMA,
// commit and loads, and the shared-memory matrix descriptors of UMMA.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace tgc {

// Device status word values (set by a kernel that gave up waiting).
enum : int { ST_OK = 0, ST_TIMEOUT_FULL = 1, ST_TIMEOUT_EMPTY = 2, ST_TIMEOUT_ACC = 3 };

// A wait gives up (and reports ST_TIMEOUT_*) after this many SM clock cycles: about
// 2 s at the B200's 1.965 GHz maximum, longer at lower clocks. The per-SM cycle
// counter is cheap to read, unlike the global timer, so the check costs nothing on
// the waits of the main loop.
constexpr long long WAIT_CYCLES = 4000000000ll;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
	asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
	asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
	asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One arrival for a whole warp (the barrier counts warps): __syncwarp orders every lane's
// preceding shared-memory writes, proxy fences and TMEM loads before lane 0's arrive. 32
// threads arriving one by one serialize on the barrier word and delay every other barrier
// operation of the CTA. All 32 lanes must call it at the same point.
__device__ __forceinline__ void mbar_arrive_warp(uint64_t *bar)
{
	__syncwarp();
	if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity)
{
	uint32_t ok;
	asm volatile(
		"{\n\t.reg .pred p;\n\t"
		"mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
		"selp.u32 %0, 1, 0, p;\n\t}"
		: "=r"(ok)
		: "r"(smem_u32(bar)), "r"(parity)
		: "memory");
	return ok != 0;
}

// Bounded wait: false (and *status set to code; any nonzero code reports the failure) if the
// phase did not complete within `limit` SM clock cycles.
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity, int *status, int code, long long limit)
{
	if (mbar_try(bar, parity)) return true;
	const long long t0 = clock64();
	for (uint32_t i = 1;; i++) {
		if (mbar_try(bar, parity)) return true;
		if ((i & 63) == 0 && clock64() - t0 > limit) break;
	}
	if (status) *(volatile int *)status = code; // a plain store: the word may be mapped host memory
	return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *status, int code)
{
	return mbar_wait_for(bar, parity, status, code, WAIT_CYCLES);
}

__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2D TMA tile load into shared memory, completion counted on bar (bytes).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y)
{
	asm volatile(
		"cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
		::"r"(smem_u32(dst)), "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y)
		: "memory");
}

// Bulk copy of a contiguous global range into shared memory (no tensor map), completion
// counted on bar. Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
	asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
		     ::"r"(smem_u32(dst)), "l"((uint64_t)src), "r"(bytes), "r"(smem_u32(bar))
		     : "memory");
}

// 2D TMA tile store / reduce-add from shared memory (bulk-group completion; no multicast).
// The x coordinate must be 16-byte aligned and neither coordinate negative.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y)
{
	asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
		     ::"l"((uint64_t)map), "r"(smem_u32(src)), "r"(x), "r"(y)
		     : "memory");
}

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *src, int x, int y)
{
	asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];"
		     ::"l"((uint64_t)map), "r"(smem_u32(src)), "r"(x), "r"(y)
		     : "memory");
}

__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void tma_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// ... until at most the most recent committed group may still be reading shared memory
__device__ __forceinline__ void tma_store_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// Wait until the committed bulk stores have completed (their writes performed).
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Barrier among the 128 threads of the four epilogue warps (barrier 0 is __syncthreads).
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map)
{
	asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// Prefetch of a 2D tile into L2 (no shared memory, no completion); x 16-byte aligned.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap *map, int x, int y)
{
	asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"((uint64_t)map), "r"(x), "r"(y)
		     : "memory");
}

// ---- TMEM -------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols)
{
	asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols));
	asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
	asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, f32 accumulate), issued by one thread.
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate)
{
	asm volatile(
		"{\n\t.reg .pred p;\n\t"
		"setp.ne.b32 p, %4, 0;\n\t"
		"tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
		::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
		: "memory");
}

// Arrive on bar once every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar)
{
	asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16])
{
	uint32_t r[16];
	asm volatile(
		"tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
		: "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
		  "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
		: "r"(taddr));
	asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
	for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 bytes
// (64 bf16), 8-row atoms 1024 bytes apart; the tile base is 1024-byte aligned.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr)
{
	uint64_t d = 0;
	d |= (uint64_t)((saddr >> 4) & 0x3FFF);        // start address
	d |= (uint64_t)1 << 16;                         // leading byte offset (unused with swizzle)
	d |= (uint64_t)(1024 >> 4) << 32;               // stride byte offset: next 8-row atom
	d |= (uint64_t)1 << 46;                         // descriptor version (sm_100)
	d |= (uint64_t)2 << 61;                         // SWIZZLE_128B
	return d;
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N)
{
	return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

} // namespace tgc
