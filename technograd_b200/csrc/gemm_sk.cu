// gemm_sk.cu -- the decode-step GEMMs: a small batch of rows (a wave of at most a few
// hundred sequences) against a layer's weights, on tcgen05 with the operands swapped and
// K split across a thread-block cluster.
//
// Why swapped: the tile kernel (gemm_sm100.cu) puts the batch in the MMA's 128-row slot and
// the weights in its N slot; at a few hundred rows that leaves narrow N = 64 tiles, whose
// 128x64x16 MMAs run at about a third of the tensor pipe's rate. Here the weights fill the
// 128-row slot (128 output channels per tile) and the batch is the MMA's N (up to 256 rows
// at once), so every MMA is 128 x 256 x 16. The batch then makes few tiles, so K is split:
// the S CTAs of a cluster (S = 1, 2 or 4) each take a contiguous range of K blocks into
// their own TMEM accumulator and stage it, as f32, in their shared memory. After a cluster
// barrier each CTA pushes the rows of the tile that another rank owns into that rank's shared
// memory with bulk copies (the TMA engine, through distributed shared memory), and each rank
// sums its slice of the tile's channels over all S partials in rank order 0..S-1 -- so the
// result does not depend on timing -- and writes the epilogue (per-channel scale, residual
// add, or SwiGLU with the bf16 hi/lo split). No scratch memory, no atomics, no second
// kernel. (Measured alternatives: scalar remote loads through distributed shared memory took
// ~40 us per tile and a round trip of the partials through L2 ~15 us, against ~6 us for the
// main loop.)
//
// Warps: 0 lane 0 issues TMA loads (weights [N, K] and the batch's bf16 hi/lo [M, K], both
// K-major with 128-byte swizzle, no multicast) into a 2-6 stage ring; 1 owns TMEM (NB f32
// columns) and lane 0 issues the MMAs; 2-5 write the partial and reduce. Every mbarrier
// wait is bounded and reports into the status word; every path reaches the cluster
// barrier, so a CTA that gave up never strands its cluster.
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "gemm.cuh"
#include "tc.cuh"

namespace tgc {

constexpr int SK_W = 128;               // weight rows (output channels) per tile: the UMMA M
constexpr int SK_K = 64;                // K block
constexpr int SK_WT = SK_W * SK_K * 2;  // 16 KB bf16 weight tile
constexpr int SK_SMEM = 232448;         // dynamic shared memory per CTA

struct SkMaps {
	CUtensorMap w[2], x[2];
};

struct SkArgs {
	int M, N, K;                   // batch rows, output channels (weight rows), reduction length
	int nw, nx, npairs, pw[4], px[4];
	int epi;                       // EPI_STORE, EPI_ADD, EPI_SWIGLU
	const float *scale, *scale2;   // per output channel or NULL (SwiGLU: gate, up)
	float *out;                    // out[m * ldo + n]
	long ldo;
	__nv_bfloat16 *out_hi, *out_lo;
	int kper;                      // K blocks per cluster rank
	int *status;
	int pdl;                       // launched with programmatic stream serialization
};

__device__ __forceinline__ uint32_t cluster_rank()
{
	uint32_t r;
	asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
	return r;
}
__device__ __forceinline__ uint32_t cluster_nranks()
{
	uint32_t r;
	asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
	return r;
}
// All threads of every CTA of the cluster; release/acquire orders each rank's scratch writes
// before it with the other ranks' reads after it.
__device__ __forceinline__ void cluster_sync()
{
	asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank)
{
	uint32_t r;
	asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
	return r;
}
// Bulk copy of `bytes` from this CTA's shared memory into another cluster rank's, completing
// on that rank's mbarrier (both given as shared::cluster addresses); 16-byte aligned sizes.
__device__ __forceinline__ void bulk_to_rank(uint32_t dst_cluster, const void *src, uint32_t bytes, uint32_t bar_cluster)
{
	asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
		     ::"r"(dst_cluster), "r"(smem_u32(src)), "r"(bytes), "r"(bar_cluster)
		     : "memory");
}

// Shared memory after the main loop: this rank's partial [128][NB] f32 (float4 chunks of a
// row XOR-swizzled by row & 7), then S - 1 receive slots of 128 / S rows each, then the
// slice's channel scales (at most 256 floats).
__host__ __device__ constexpr int sk_red_bytes(int NB, int S) { return 512 * NB + (S - 1) * (128 / S) * NB * 4 + 1024; }

template <int NB, int STAGES, int EPI>
__global__ void __launch_bounds__(192, 1) gemm_sk(const __grid_constant__ SkMaps maps, const __grid_constant__ SkArgs p)
{
	extern __shared__ uint8_t smem_raw[];
	uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
	constexpr int XT = NB * SK_K * 2; // one batch tile: NB rows of a K block, bf16
	const int stage_bytes = p.nw * SK_WT + p.nx * XT;
	const uint32_t S = cluster_nranks(), rank = cluster_rank();
	uint64_t *full = (uint64_t *)(smem + max(STAGES * stage_bytes, sk_red_bytes(NB, (int)S)));
	uint64_t *empty = full + STAGES;
	uint64_t *accf = empty + STAGES;
	uint64_t *recv = accf + 1; // the other ranks' rows of this rank's slice have landed
	uint32_t *tslot = (uint32_t *)(recv + 1);
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int n0 = blockIdx.x * SK_W, m0 = blockIdx.y * NB;

	const int KB = (p.K + SK_K - 1) / SK_K;
	const int kb0 = (int)rank * p.kper;
	const int nkb = max(0, min(p.kper, KB - kb0));

	if (threadIdx.x == 0) {
		for (int s = 0; s < STAGES; s++) {
			mbar_init(&full[s], 1);
			mbar_init(&empty[s], 1);
		}
		mbar_init(accf, 1);
		mbar_init(recv, 1);
		fence_barrier_init();
		for (int i = 0; i < p.nw; i++) tma_prefetch_desc(&maps.w[i]);
		for (int i = 0; i < p.nx; i++) tma_prefetch_desc(&maps.x[i]);
	}
	if (warp == 1) tmem_alloc(tslot, NB);
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = *tslot;
	pdl_wait(); // the kernel before it (with programmatic launch) has completed: inputs ready
	pdl_launch();

	if (warp == 0) { // ---- producer
		if (lane == 0)
			for (int i = 0; i < nkb; i++) {
				const int s = i % STAGES;
				const uint32_t ph = (i / STAGES) & 1;
				if (!mbar_wait(&empty[s], ph ^ 1, p.status, ST_TIMEOUT_EMPTY)) break;
				uint8_t *st = smem + s * stage_bytes;
				const int kx = (kb0 + i) * SK_K;
				mbar_expect_tx(&full[s], stage_bytes); // out-of-range rows arrive as zeros and count
				for (int w = 0; w < p.nw; w++) tma_load_2d(st + w * SK_WT, &maps.w[w], &full[s], kx, n0);
				for (int x = 0; x < p.nx; x++) tma_load_2d(st + p.nw * SK_WT + x * XT, &maps.x[x], &full[s], kx, m0);
			}
		__syncwarp();
	} else if (warp == 1) { // ---- MMA issuer
		if (lane == 0) {
			constexpr uint32_t idesc = idesc_bf16_f32(SK_W, NB);
			uint32_t issued = 0;
			for (int i = 0; i < nkb; i++) {
				const int s = i % STAGES;
				const uint32_t ph = (i / STAGES) & 1;
				if (!mbar_wait(&full[s], ph, p.status, ST_TIMEOUT_FULL)) break;
				tc_fence_after();
				const uint32_t base = smem_u32(smem + s * stage_bytes);
				for (int q = 0; q < p.npairs; q++) {
					const uint32_t a = base + p.pw[q] * SK_WT, b = base + p.nw * SK_WT + p.px[q] * XT;
#pragma unroll
					for (int kk = 0; kk < SK_K / 16; kk++) {
						tc_mma_f16(tmem, sw128_kmajor_desc(a + kk * 32), sw128_kmajor_desc(b + kk * 32), idesc, issued);
						issued = 1;
					}
				}
				tc_commit(&empty[s]);
			}
			tc_commit(accf);
		}
		__syncwarp();
	} else { // ---- warps 2-5: the accumulator (TMEM lanes 32q..32q+31 for warp quarter q) into P
		const int quarter = warp & 3;
		const int r = quarter * 32 + lane;
		const bool ok = mbar_wait(accf, 0, p.status, ST_TIMEOUT_ACC) && nkb > 0;
		tc_fence_after();
		float4 *row = (float4 *)smem + r * (NB / 4); // the ring is idle: every load fed a finished MMA
		const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
		for (int c = 0; c < NB; c += 16) {
			float v[16];
			__syncwarp();
			tmem_ld16(trow + c, v);
#pragma unroll
			for (int i = 0; i < 4; i++)
				row[(c / 4 + i) ^ (r & 7)] = ok ? make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3])
							      : make_float4(0.f, 0.f, 0.f, 0.f);
		}
		fence_async_smem(); // the bulk copies read P through the async proxy
	}
	tc_fence_before();
	cluster_sync(); // every rank's P is written and every ring idle: the receive slots are free
	if (warp == 1) {
		tc_fence_after();
		tmem_dealloc(tmem, NB);
	}

	// ---- this rank's slice of the tile's rows. Slices: R = 128 / S rows (rank y: rows
	// [y R, y R + R)); SwiGLU: 64 / S channels, i.e. a run of gate rows and the run of up rows
	// 32 below it. Each rank pushes its own rows of every other rank's slice into that rank's
	// receive slot (slot of source z at rank y: z if z < y, else z - 1).
	const float4 *P = (const float4 *)smem;
	const int R = SK_W / (int)S, RC = 64 / (int)S;
	const int wq = warp - 2, rr = lane & 7, cc = lane >> 3;
	auto run_start = [&](int y, int half) { // first row of rank y's slice (SwiGLU: gate or up run)
		if (EPI != EPI_SWIGLU) return y * R;
		const int c = y * RC;
		return (c / 32) * 64 + c % 32 + 32 * half;
	};
	if (warp >= 2) {
	if (S > 1 && threadIdx.x == 64) {
		mbar_expect_tx(recv, (uint32_t)((S - 1) * R * NB * 4));
		const uint32_t recv_l = smem_u32(recv), slot0 = smem_u32(smem + 512 * NB);
		for (int y = 0; y < (int)S; y++) {
			if (y == (int)rank) continue;
			const int slot = (int)rank < y ? (int)rank : (int)rank - 1;
			const uint32_t dst = cluster_map(slot0 + (uint32_t)(slot * R * NB * 4), (uint32_t)y), bar = cluster_map(recv_l, (uint32_t)y);
			if (EPI == EPI_SWIGLU) {
				bulk_to_rank(dst, P + run_start(y, 0) * (NB / 4), (uint32_t)(RC * NB * 4), bar);
				bulk_to_rank(dst + (uint32_t)(RC * NB * 4), P + run_start(y, 1) * (NB / 4), (uint32_t)(RC * NB * 4), bar);
			} else {
				bulk_to_rank(dst, P + run_start(y, 0) * (NB / 4), (uint32_t)(R * NB * 4), bar);
			}
		}
	}
	// the slice's scales into shared memory while the copies are in flight
	float *ssc = (float *)(smem + 512 * NB + (S - 1) * R * NB * 4);
	const int et = threadIdx.x - 64;
	if (EPI == EPI_SWIGLU) {
		for (int i = et; i < RC; i += 128) {
			const int f = n0 / 2 + (int)rank * RC + i;
			ssc[i] = 2 * f < p.N ? p.scale[f] : 0.0f;
			ssc[RC + i] = 2 * f < p.N ? p.scale2[f] : 0.0f;
		}
	} else if (p.scale) {
		for (int i = et; i < R; i += 128) {
			const int n = n0 + (int)rank * R + i;
			ssc[i] = n < p.N ? p.scale[n] : 0.0f;
		}
	}
	const bool landed = S == 1 || __all_sync(0xffffffffu, mbar_wait(recv, 0, p.status, ST_TIMEOUT_FULL));
	epilogue_sync(); // the scales are in place
	const float4 *slots = (const float4 *)(smem + 512 * NB);
	// partial z's float4 chunk j of tile row `row` (at slot row `srow` when z is another rank)
	auto chunk = [&](int z, int row, int srow, int j) -> float4 {
		const int jj = j ^ (row & 7);
		if (z == (int)rank) return P[row * (NB / 4) + jj];
		const int slot = z < (int)rank ? z : z - 1;
		return slots[(slot * R + srow) * (NB / 4) + jj];
	};
	if (EPI == EPI_SWIGLU) {
		const int c_lo = (int)rank * RC, f0 = n0 / 2;
		const int nblk = (RC / 8) * (NB / 16);
		for (int b = wq; b < nblk && landed; b += 4) {
			const int ci = (b % (RC / 8)) * 8 + rr, c = c_lo + ci, col = (b / (RC / 8)) * 16 + cc * 4;
			const int gr = (c / 32) * 64 + c % 32, ur = gr + 32;
			float gs[4], us[4];
#pragma unroll
			for (int z = 0; z < 8; z++)
				if (z < (int)S) {
					const float4 g = chunk(z, gr, ci, col / 4), u = chunk(z, ur, RC + ci, col / 4);
					if (z == 0) {
						gs[0] = g.x, gs[1] = g.y, gs[2] = g.z, gs[3] = g.w;
						us[0] = u.x, us[1] = u.y, us[2] = u.z, us[3] = u.w;
					} else {
						gs[0] = __fadd_rn(gs[0], g.x), gs[1] = __fadd_rn(gs[1], g.y), gs[2] = __fadd_rn(gs[2], g.z), gs[3] = __fadd_rn(gs[3], g.w);
						us[0] = __fadd_rn(us[0], u.x), us[1] = __fadd_rn(us[1], u.y), us[2] = __fadd_rn(us[2], u.z), us[3] = __fadd_rn(us[3], u.w);
					}
				}
			const int f = f0 + c;
			if (2 * f >= p.N) continue;
			const float sg = ssc[ci], su = ssc[RC + ci];
#pragma unroll
			for (int i = 0; i < 4; i++) {
				const int m = m0 + col + i;
				if (m >= p.M) break;
				const float gv = __fmul_rn(gs[i], sg), uv = __fmul_rn(us[i], su);
				const float y = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv); // silu(g) * u
				const __nv_bfloat16 h = __float2bfloat16_rn(y);
				p.out_hi[(long)m * p.ldo + f] = h;
				p.out_lo[(long)m * p.ldo + f] = __float2bfloat16_rn(y - __bfloat162float(h));
			}
		}
	} else {
		const int r_lo = (int)rank * R;
		const int nblk = (R / 8) * (NB / 16);
		for (int b = wq; b < nblk && landed; b += 4) {
			const int ri = (b % (R / 8)) * 8 + rr, r = r_lo + ri, col = (b / (R / 8)) * 16 + cc * 4, n = n0 + r;
			float a[4];
#pragma unroll
			for (int z = 0; z < 8; z++)
				if (z < (int)S) {
					const float4 v = chunk(z, r, ri, col / 4);
					if (z == 0) a[0] = v.x, a[1] = v.y, a[2] = v.z, a[3] = v.w;
					else a[0] = __fadd_rn(a[0], v.x), a[1] = __fadd_rn(a[1], v.y), a[2] = __fadd_rn(a[2], v.z), a[3] = __fadd_rn(a[3], v.w);
				}
			if (n >= p.N) continue;
			const float sc = ssc[ri];
#pragma unroll
			for (int i = 0; i < 4; i++) {
				const int m = m0 + col + i;
				if (m >= p.M) break;
				const float x = p.scale ? __fmul_rn(sc, a[i]) : a[i];
				float *o = p.out + (long)m * p.ldo + n;
				// the residual add: the one add this element receives, as a reduction that
				// needs no read (f32 atomics flush subnormals, which these sums never are)
				if (EPI == EPI_ADD) asm volatile("red.global.add.f32 [%0], %1;" ::"l"(o), "f"(x) : "memory");
				else *o = x;
			}
		}
	}
	}
	__syncwarp();
	// no rank leaves while a bulk copy may still read its P: every copy has landed once every
	// rank has passed its wait above
	asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---- host side -------------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 g_sk_encode = nullptr;

static int sk_encode_fn()
{
	if (g_sk_encode) return TG_CUDA_OK;
	cudaDriverEntryPointQueryResult q;
	void *fn = nullptr;
	cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
	if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
		return set_err(TG_CUDA_ECUDA, "cuTensorMapEncodeTiled is unavailable");
	g_sk_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
	return TG_CUDA_OK;
}

// bf16 [rows, K] (row stride ld elements), boxes of box_rows x 64 with 128-byte swizzle
static int sk_map(CUtensorMap *m, const void *base, long rows, long K, long ld, int box_rows)
{
	if (((uintptr_t)base & 15) || (ld * 2) % 16) return set_err(TG_CUDA_EINVAL, "gemm: operand base or row pitch not 16-byte aligned");
	cuuint64_t dims[2] = { (cuuint64_t)K, (cuuint64_t)rows };
	cuuint64_t strides[1] = { (cuuint64_t)ld * 2 };
	cuuint32_t box[2] = { (cuuint32_t)SK_K, (cuuint32_t)box_rows };
	cuuint32_t es[2] = { 1, 1 };
	CUresult r = g_sk_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
				 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
				 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
	if (r != CUDA_SUCCESS) return set_err(TG_CUDA_ECUDA, "cuTensorMapEncodeTiled(gemm_sk): error %d", (int)r);
	return TG_CUDA_OK;
}

constexpr int SK_RING = SK_SMEM - 1024 - 256; // alignment slack and the barriers

static int sk_body(int NB, int stages, int nw, int nx, int S)
{
	return std::max(stages * (nw * SK_WT + nx * NB * SK_K * 2), sk_red_bytes(NB, S));
}

template <int NB, int STAGES, int EPI>
static cudaLaunchConfig_t sk_config(const SkArgs &p, int S, int body, cudaStream_t st, cudaLaunchAttribute *attr)
{
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3((unsigned)((p.N + SK_W - 1) / SK_W), (unsigned)((p.M + NB - 1) / NB), (unsigned)S);
	cfg.blockDim = dim3(192);
	cfg.dynamicSmemBytes = (size_t)body + 1024 + 256;
	cfg.stream = st;
	attr[0].id = cudaLaunchAttributeClusterDimension;
	attr[0].val.clusterDim.x = 1;
	attr[0].val.clusterDim.y = 1;
	attr[0].val.clusterDim.z = (unsigned)S;
	cfg.attrs = attr;
	cfg.numAttrs = 1;
	if (p.pdl) {
		attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
		attr[1].val.programmaticStreamSerializationAllowed = 1;
		cfg.numAttrs = 2;
	}
	return cfg;
}

template <int NB, int STAGES, int EPI>
static int sk_launch(const SkMaps &maps, const SkArgs &p, int S, cudaStream_t st)
{
	const int body = sk_body(NB, STAGES, p.nw, p.nx, S);
	if (body > SK_RING) return set_err(TG_CUDA_EINVAL, "gemm_sk: %d bytes of shared memory", body);
	cudaLaunchAttribute attr[2];
	cudaLaunchConfig_t cfg = sk_config<NB, STAGES, EPI>(p, S, body, st, attr);
	TGC_CUDA(cudaLaunchKernelEx(&cfg, gemm_sk<NB, STAGES, EPI>, maps, p));
	return TG_CUDA_OK;
}

// Clusters of S CTAs that can run at once, per device, kernel shape (NB, stages), weight
// operands (1 or 2) and S (1, 2, 4): measured once with the occupancy API at set-up.
struct SkOcc {
	bool done = false;
	int clusters[3][2][4] = {}; // [NB 256/128/64][nw - 1][log2 S]; 0: does not fit
};
static SkOcc g_sk_occ[64];

static int sk_nb_index(int NB) { return NB == 256 ? 0 : NB == 128 ? 1 : 2; }
static int sk_stages(int NB, int nw)
{
	const int stage = nw * SK_WT + 2 * NB * SK_K * 2;
	if (NB == 256) return 2;
	if (NB == 128) return 4 * stage <= SK_RING ? 4 : 3;
	return 6 * stage <= SK_RING ? 6 : 4;
}

template <int NB, int STAGES>
static int sk_occ_one(SkOcc &o, int nw)
{
	SkArgs p;
	memset(&p, 0, sizeof p);
	p.N = 128 * 64, p.M = NB, p.nw = nw, p.nx = 2;
	for (int ls = 0; ls < 4; ls++) {
		const int S = 1 << ls, body = sk_body(NB, STAGES, nw, 2, S);
		int n = 0;
		if (body <= SK_RING) {
			cudaLaunchAttribute attr[2];
			cudaLaunchConfig_t cfg = sk_config<NB, STAGES, EPI_STORE>(p, S, body, nullptr, attr);
			TGC_CUDA(cudaOccupancyMaxActiveClusters(&n, gemm_sk<NB, STAGES, EPI_STORE>, &cfg));
		}
		o.clusters[sk_nb_index(NB)][nw - 1][ls] = n;
	}
	return TG_CUDA_OK;
}

// The kernels' shared-memory limit, set once per device outside any stream capture.
template <int NB, int STAGES>
static int sk_attrs()
{
	TGC_CUDA(cudaFuncSetAttribute(gemm_sk<NB, STAGES, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM));
	TGC_CUDA(cudaFuncSetAttribute(gemm_sk<NB, STAGES, EPI_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM));
	TGC_CUDA(cudaFuncSetAttribute(gemm_sk<NB, STAGES, EPI_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM));
	return TG_CUDA_OK;
}

int gemm_sk_prepare()
{
	int rc, dev = 0;
	if ((rc = sk_encode_fn())) return rc;
	TGC_CUDA(cudaGetDevice(&dev));
	if (dev < 0 || dev >= 64) return set_err(TG_CUDA_EINVAL, "device ordinal %d", dev);
	SkOcc &o = g_sk_occ[dev];
	if (o.done) return TG_CUDA_OK;
	if ((rc = sk_attrs<256, 2>()) || (rc = sk_attrs<128, 4>()) || (rc = sk_attrs<128, 3>()) || (rc = sk_attrs<64, 6>()) ||
	    (rc = sk_attrs<64, 4>()))
		return rc;
	for (int nw = 1; nw <= 2; nw++) {
		if ((rc = sk_occ_one<256, 2>(o, nw))) return rc;
		if ((rc = sk_stages(128, nw) == 4 ? sk_occ_one<128, 4>(o, nw) : sk_occ_one<128, 3>(o, nw))) return rc;
		if ((rc = sk_stages(64, nw) == 6 ? sk_occ_one<64, 6>(o, nw) : sk_occ_one<64, 4>(o, nw))) return rc;
	}
	o.done = true;
	return TG_CUDA_OK;
}

bool gemm_sk_fits(const GemmArgs &p)
{
	return p.M >= 1 && p.M <= 1024 && p.N >= 1 && p.K >= SK_K && p.K % 8 == 0 && !p.cside && p.nb >= 1 && p.nb <= 2 &&
	       p.na == 2 && (p.epi == EPI_STORE || p.epi == EPI_ADD || p.epi == EPI_SWIGLU) &&
	       (p.scale_mode == 0 || p.scale_mode == 2) && (p.epi != EPI_SWIGLU || (p.N % 128 == 0 && p.scale && p.scale2));
}

// Tile width NB (batch rows per MMA: 256, 128 or 64) and split count S (cluster size 1, 2, 4
// or 8): the shape with the least estimated time, from a model fitted to traced launches
// (microseconds): rounds of co-resident clusters x (pipeline fill 1.5 + per K block and
// operand pair 0.30 / 0.20 / 0.15 at NB 256 / 128 / 64 + staging the accumulator + pushing
// the other ranks' rows + the reduction of this rank's slice). Every rank gets K blocks.
struct SkShape {
	int NB, S, kper;
};
static SkShape sk_shape(int M, int N, int KB, int npairs, const int (*clusters)[2][4], int nw)
{
	SkShape best = { 0, 1, KB };
	double best_t = 1e30;
	for (int nbi = 0; nbi < 3; nbi++) {
		const int NB = 256 >> nbi;
		if (NB < 64 || (NB > 64 && (NB >> 1) >= M)) continue; // no wider than the batch needs
		const double c = nbi == 0 ? 0.30 : nbi == 1 ? 0.20 : 0.15, f = NB / 256.0;
		const long tiles = (long)((N + SK_W - 1) / SK_W) * ((M + NB - 1) / NB);
		for (int ls = 0; ls < 4; ls++) {
			const int S = 1 << ls, resident = clusters[nbi][nw - 1][ls];
			if (S > KB || resident <= 0) continue;
			const int kp = (KB + S - 1) / S;
			if ((KB + kp - 1) / kp != S) continue;
			const double per = 1.5 + kp * npairs * c + 1.2 * f + (S > 1 ? 0.5 + 3.0 * (S - 1) / S * f : 0.0) +
					   (128.0 / S) * NB / 8192.0;
			const double t = (double)((tiles + resident - 1) / resident) * per;
			if (t < best_t - 1e-9) best_t = t, best = { NB, S, kp };
		}
	}
	return best;
}

// D[M, N] = sum over pairs of A[pa] (the batch, [M, K] bf16) times B[pb]^T (the weights,
// [N, K] bf16), with the tile kernel's epilogues; the caller's GemmOperands / GemmArgs.
int gemm_sk(const GemmOperands &ops, const GemmArgs &p, cudaStream_t st)
{
	int rc;
	if (!gemm_sk_fits(p)) return set_err(TG_CUDA_EINVAL, "gemm_sk: shape or epilogue not supported");
	int dev = 0;
	TGC_CUDA(cudaGetDevice(&dev));
	if (dev < 0 || dev >= 64 || !g_sk_occ[dev].done) return set_err(TG_CUDA_EINVAL, "gemm_sk: gemm_sk_prepare was not called on device %d", dev);
	const SkShape sh = sk_shape(p.M, p.N, (p.K + SK_K - 1) / SK_K, p.npairs, g_sk_occ[dev].clusters, p.nb);
	if (!sh.NB) return set_err(TG_CUDA_EINVAL, "gemm_sk: no tile shape fits");
	const int NB = sh.NB, S = sh.S;
	SkMaps maps;
	memset(&maps, 0, sizeof maps);
	SkArgs a;
	memset(&a, 0, sizeof a);
	a.M = p.M, a.N = p.N, a.K = p.K;
	a.nw = p.nb, a.nx = p.na, a.npairs = p.npairs;
	for (int q = 0; q < p.npairs; q++) a.pw[q] = p.pb[q], a.px[q] = p.pa[q];
	a.epi = p.epi;
	a.scale = p.scale_mode == 2 || p.epi == EPI_SWIGLU ? p.scale : nullptr;
	a.scale2 = p.scale2;
	a.out = p.out, a.ldo = p.ldo, a.out_hi = p.out_hi, a.out_lo = p.out_lo, a.status = p.status;
	a.kper = sh.kper;
	a.pdl = p.pdl;
	for (int j = 0; j < p.nb; j++)
		if ((rc = sk_map(&maps.w[j], ops.b[j], p.N, p.K, ops.ldb, SK_W))) return rc;
	for (int i = 0; i < p.na; i++)
		if ((rc = sk_map(&maps.x[i], ops.a[i], p.M, p.K, ops.lda, NB))) return rc;
#define SK_GO(NB_, ST_)                                                                                   \
	do {                                                                                              \
		if (p.epi == EPI_SWIGLU) return sk_launch<NB_, ST_, EPI_SWIGLU>(maps, a, S, st);          \
		if (p.epi == EPI_ADD) return sk_launch<NB_, ST_, EPI_ADD>(maps, a, S, st);                \
		return sk_launch<NB_, ST_, EPI_STORE>(maps, a, S, st);                                    \
	} while (0)
	const int stages = sk_stages(NB, a.nw);
	if (NB == 256) SK_GO(256, 2);
	if (NB == 128) {
		if (stages == 4) SK_GO(128, 4);
		SK_GO(128, 3);
	}
	if (stages == 6) SK_GO(64, 6);
	SK_GO(64, 4);
#undef SK_GO
}

} // namespace tgc
