// gemm.cuh -- the tensor-core GEMM interface used inside the library.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace tgc {

enum { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_PARTIAL = 3 };

// Operands: up to two A matrices [M, K] and two B matrices [N, K], bf16, K-major.
struct GemmOperands {
	const void *a[2] = { nullptr, nullptr };
	const void *b[2] = { nullptr, nullptr };
	long lda = 0, ldb = 0; // row strides in elements
};

struct GemmArgs {
	int M, N, K;
	int na, nb, npairs;
	int pa[4], pb[4];        // pair q multiplies A[pa[q]] by B[pb[q]]
	int epi;                 // EPI_*
	int scale_mode;          // 0 none, 1 per row of D, 2 per column of D
	const float *scale;      // per row / column; SwiGLU: gate scales (per channel)
	const float *scale2;     // SwiGLU: up scales
	float *out;              // f32 D (STORE: written; ADD: D += result)
	__nv_bfloat16 *out_hi, *out_lo; // SwiGLU: bf16 hi/lo of silu(g) * u
	long ldo;                // row stride of the output, elements
	int *status;             // device status word (ST_*), may not be NULL
	int tma_out;             // set by gemm(): the output is written through a TMA map
	float *partial;          // optional scratch for split-K (small batches); NULL: never split
	long partial_floats;     // its size in floats
	int kb_per_split;        // set by gemm() for the split launch: K blocks per split
	long mpad;               // set by gemm(): rows per split block of the partial buffer
	// Dequant in the kernel: with cside 1 (A[0]) or 2 (B[0]) that operand is built in shared
	// memory from integer codes (K-major rows of cld bytes; int8 one code per byte, int4 two
	// per byte low nibble first), which are exact in bf16: TMA brings each K block of raw
	// codes into its ring stage, four warps expand them in place. K must be a multiple of
	// 64, cld and the base 16-byte aligned.
	const signed char *codes;
	int cbits, cside;
	long cld;
	int raw_bytes; // set by gemm(): bytes of one K block of codes (TMA-loaded into each ring stage)
	// Scaled dequant (cside 2 with nb 2): B[0] and B[1] are both built from the codes, as the
	// bf16 hi and lo parts of code * cscale[(k / cgroup) * cscale_ld + n] (weights whose scale
	// changes along K, such as per-head o_proj scales); cgroup a multiple of 64
	const float *cscale;
	int cgroup;
	long cscale_ld;
	// the decoder's batches of 2-4 M tiles (waves of up to 512 sequences): tiles as wide as
	// the output allows, the K range split over the SMs, instead of 64-wide tiles
	int wide;
	// launch with programmatic stream serialization (the kernels wait for the one before them
	// with griddepcontrol.wait before touching memory; only the decoder's captured step sets it)
	int pdl;
};

// Launch on stream. SwiGLU: B rows come in blocks of 64 (32 gate rows then the
// 32 matching up rows), N = 2 * channels, output channels = N / 2.
int gemm(const GemmOperands &ops, GemmArgs p, cudaStream_t st);

// Small batches (gemm_sk.cu): the same product with the weights in the MMA's 128-row slot
// and K split over a thread-block cluster, summed in a fixed order. bf16 operands, epilogues
// STORE / ADD / SWIGLU with scale_mode 0 or 2. gemm_sk_prepare sets the kernels' attributes
// (once per device, outside any stream capture).
bool gemm_sk_fits(const GemmArgs &p);
int gemm_sk(const GemmOperands &ops, const GemmArgs &p, cudaStream_t st);
int gemm_sk_prepare();

int split_to_bf16(const float *src, long rows, long cols, long lds, bool transpose, __nv_bfloat16 *hi, __nv_bfloat16 *lo,
		  long ldd, cudaStream_t st);
int codes_to_bf16(const signed char *q, int bits, long rows, long cols, bool transpose, __nv_bfloat16 *dst, long ldd,
		  cudaStream_t st);
int device_status_check(int *d_status, cudaStream_t st);
// The per-device status word of the drop-in matmul calls (pinned, mapped; written only by a
// kernel wait that timed out): an earlier call's timeout is reported, then cleared.
int call_status_word(int dev, int **d_status);
// A TMA map of a bf16 [rows, K] matrix (row stride ld elements): boxes of 64 columns x
// box_rows rows, 128-byte swizzle (the K-major operand layout of the UMMA descriptors).
int bf16_tile_map(CUtensorMap *m, const void *base, long rows, long K, long ld, int box_rows);

} // namespace tgc
