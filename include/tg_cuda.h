/* tg_cuda.h -- C ABI of libtgcuda, the B200 (sm_100a) batch backend for Technograd.
 *
 * Plain C: pointers, sizes and status codes only. Every entry point returns
 * TG_CUDA_OK (0) or a negative status; the text of the last error on the
 * calling thread is tg_cuda_error(). The library never exits the process and
 * never prints; the caller (the `tgc batch --device cuda` branch) turns a
 * status into its own die() before it creates any output file, which keeps
 * the reference's atomic-failure rule (src/main.c:414-419, docs/SPEC.md:282-285).
 *
 * Reference interfaces replaced (paths inside IlumCI/Technograd):
 *   tg_cuda_batch      <- the par_for(batch_rows) loop of the batch branch,
 *                         src/main.c:421-441, and vm_run_into per row, src/vm.c:475-481
 *   tg_cuda_matmul_q   <- tg_matmul_qa / tg_matmul_qb, runtime/tg_rt.h:132-151
 *   tg_cuda_load       <- the planned Module handed to the VM, src/tg.h:177-200, src/plan.c:154
 *   tg_cuda_lm_*       <- `tgc batch` over the Qwen3 program that examples/qwen3/import.py:51-131
 *                         emits (per-head tg_matmul_qb, rmsnorm, softmax, take), run per sequence
 *   tg_cuda_quantize_rtn <- the RTN branch of quantize_param, src/quant.c:176-200,258-316
 *   tg_cuda_batcher_*  <- vm_run_into per request line in run_line, src/serve.c:129-149
 *   tg_cuda_host_register <- no counterpart: pins the batch branch's sample array (load_samples,
 *                         src/main.c:175-214) and output block for direct DMA
 */
#ifndef TG_CUDA_H
#define TG_CUDA_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status ------------------------------------------------------------- */
#define TG_CUDA_OK            0
#define TG_CUDA_EINVAL       -1 /* bad argument (shape, pointer, size) */
#define TG_CUDA_ENODEV       -2 /* no usable CUDA device, or not initialised */
#define TG_CUDA_ECUDA        -3 /* a CUDA runtime call failed */
#define TG_CUDA_EUNSUPPORTED -4 /* op or model form the GPU path does not run (no CPU fallback) */
#define TG_CUDA_ENOMEM       -5 /* device or pinned host allocation failed */
#define TG_CUDA_EFAULT       -6 /* failure injected through TG_CUDA_FAULT (host-side tests) */
#define TG_CUDA_EDEVICE      -7 /* a kernel reported an error in its device status word */

/* Last error text of the calling thread ("" if none). */
const char *tg_cuda_error(void);

/* ---- devices -------------------------------------------------------------- */
/* Select the GPUs rows are sharded over. ngpus <= 0 or devices == NULL: every
 * visible device (or the first ngpus). Idempotent for the same set. */
int tg_cuda_init(int ngpus, const int *devices);
/* Number of devices selected by tg_cuda_init (0 before it). */
int tg_cuda_ngpus(void);
/* Failure-path self-test on device 0 of the selection: a kernel waits on an mbarrier
 * that nothing arrives on, with a limit of `cycles` SM clock cycles (the same bounded
 * wait every tcgen05 kernel uses, whose default limit is about 2 s). The wait gives
 * up, the kernel writes its status word and returns: TG_CUDA_EDEVICE with *status =
 * the kernel's status code (1, a timed-out full-barrier wait). Any other return means
 * the mechanism failed. The context stays usable. No reference counterpart. */
int tg_cuda_selftest_wait(long long cycles, int *status);
/* Test hook, no reference counterpart: the decoder's bf16 GEMM on device buffers,
 * out = epilogue(sum over pairs q of a[pa[q]] [m, k] times b[pb[q]] [n, k] transposed),
 * through the tile kernel (path 0) or the swapped-operand cluster kernel that the decode
 * steps use (path 1). epi 0 stores (times scale[n] when scale is not NULL), 1 adds into
 * out, 2 is SwiGLU: b's rows interleave blocks of 32 gate and 32 up channels, and
 * out_hi/out_lo receive the bf16 hi/lo of silu(gate * scale) * (up * scale2), [m, n/2]
 * with row stride ldo. Synchronous. */
int tg_cuda_selftest_gemm(int path, const void *const *a, int na, const void *const *b, int nb, int npairs,
			  const int *pa, const int *pb, int m, int n, int k, int epi, const float *scale,
			  const float *scale2, float *out, long ldo, void *out_hi, void *out_lo, void *stream);
/* Release every device resource the library holds. */
void tg_cuda_shutdown(void);

/* ---- kernel-level drop-in --------------------------------------------------
 * axis 0 (tg_matmul_qa, runtime/tg_rt.h:132-140): o[m,n] = s[i] * sum_p code(q, i*k+p) * act[p*n+j]
 * axis 1 (tg_matmul_qb, runtime/tg_rt.h:143-151): o[m,n] = s[j] * sum_p act[i*k+p] * code(q, p*n+j)
 * Codes: bits 8 = one signed byte per element; bits 4 = two per byte, element
 * e in byte e/2, low nibble first, sign-extended (runtime/tg_rt.h:124-129).
 * All pointers are DEVICE pointers on the current device; the call is
 * asynchronous on `stream` (NULL = the legacy default stream). Scratch for the
 * tensor-core path (m*k or k*n large) is cached per device by the library. A
 * tensor-core kernel that gave up waiting (TG_CUDA_EDEVICE) is reported by a
 * later call on the same device, like CUDA's own asynchronous errors. */
int tg_cuda_matmul_q(int axis, float *o, const float *act, const signed char *q, int bits, const float *s, int m,
		     int k, int n, void *stream);

/* The x @ W case of tg_cuda_matmul_q (axis 1) for a batch m <= 8, without any
 * allocation. No counterpart in the reference: it exists for callers that must
 * not allocate device memory while they run (the reference's par_for workers
 * may not allocate at all, src/par.c:11-12; hosts with a fixed memory budget).
 * Its split-K partial sums use a 4 MiB static device array that every GPU
 * loading the library keeps until exit, so m * n may be at most 1,048,576; n a
 * multiple of 8 (int4) or 4 (int8), q 4-byte aligned. The first call on a
 * device looks the array's address up (make it before any stream capture) and
 * caches it for the life of the process, so cudaDeviceReset is not supported
 * while the library is loaded. Every call on a device shares the array: calls
 * from several host threads on the same stream are serialised (a per-device
 * lock covers the enqueue of both kernels), calls on different streams that
 * overlap on the GPU race. Device pointers, asynchronous on stream; larger
 * shapes are rejected with TG_CUDA_EINVAL. */
int tg_cuda_matmul_qb_noalloc(float *o, const float *act, const signed char *q, int bits, const float *s, int m, int k,
			      int n, void *stream);

/* Per-channel RTN quantization on the device, bit-exact with quant.c: w is the
 * f32 matrix [rows, cols] (device), axis 0 = one scale per row, 1 = per column;
 * q receives (bits 8) rows*cols bytes or (bits 4) (rows*cols+1)/2 bytes, s one
 * f32 scale per channel. */
int tg_cuda_quantize_rtn(const float *w, int rows, int cols, int axis, int bits, signed char *q, float *s, void *stream);

/* GPTQ, bit-exact with quant.c (src/quant.c:92-316, the GPTQ branch of
 * quantize_param). prepare: the Hessian of nrows calibration rows of K inputs
 * (HOST memory), dampened 1%, and the upper Cholesky factor of its inverse,
 * kept on the current device. quantize: like tg_cuda_quantize_rtn (device
 * pointers) with K = the non-channel extent; a Hessian that is not positive
 * definite keeps the Hessian-weighted scale search without error feedback, as
 * the reference does. The reference only calibrates inputs of at most 2048
 * (src/quant.c:346); wider layers are the caller's RTN. */
typedef struct tg_cuda_gptq tg_cuda_gptq;
int tg_cuda_gptq_prepare(const float *calib, int nrows, int K, tg_cuda_gptq **out);
int tg_cuda_quantize_gptq(tg_cuda_gptq *g, const float *w, int rows, int cols, int axis, int bits, signed char *q, float *s,
			  void *stream);
void tg_cuda_gptq_free(tg_cuda_gptq *g);

/* ---- programs ------------------------------------------------------------- */
/* A planned TGIR program, flattened. The host builds it from its Module
 * (src/tg.h:112-200); the numbering of ops is the reference's enum Op. */
enum {
	TG_CUDA_OP_CONST, TG_CUDA_OP_ADD, TG_CUDA_OP_SUB, TG_CUDA_OP_MUL, TG_CUDA_OP_DIV, TG_CUDA_OP_MAX, TG_CUDA_OP_MIN,
	TG_CUDA_OP_NEG, TG_CUDA_OP_TANH, TG_CUDA_OP_RELU, TG_CUDA_OP_SIGMOID, TG_CUDA_OP_EXP, TG_CUDA_OP_SQRT, TG_CUDA_OP_GELU,
	TG_CUDA_OP_SILU, TG_CUDA_OP_SOFTPLUS, TG_CUDA_OP_LOG, TG_CUDA_OP_MATMUL, TG_CUDA_OP_SOFTMAX, TG_CUDA_OP_RMSNORM,
	TG_CUDA_OP_SUM, TG_CUDA_OP_MEAN, TG_CUDA_OP_TRANSPOSE, TG_CUDA_OP_OUTER, TG_CUDA_OP_STEP, TG_CUDA_OP_SPMM,
	TG_CUDA_OP_SPMM_T, TG_CUDA_OP_SPMM_DX, TG_CUDA_OP_ACTIVE, TG_CUDA_OP_TAKE, TG_CUDA_OP_TAKE_T, TG_CUDA_OP_SPMM_TC,
	TG_CUDA_OP_SIN, TG_CUDA_OP_COS, TG_CUDA_OP_RESHAPE, TG_CUDA_OP_FLOOR, TG_CUDA_OP_SUM_TO, TG_CUDA_OP_TOPK,
	TG_CUDA_OP_MEMSCAN, TG_CUDA_OP_MEMSCAN_T, TG_CUDA_OP_SUFMATCH, TG_CUDA_OP_THINK, TG_CUDA_OP_SCAN, TG_CUDA_OP_COUNT
};

enum { TG_CUDA_PARAM, TG_CUDA_INPUT, TG_CUDA_TMP, TG_CUDA_STATE }; /* VKind, src/tg.h:114 */

typedef struct {
	int kind;                /* TG_CUDA_PARAM / INPUT / TMP / STATE */
	int rank, dim[4];        /* Shape, src/tg.h:36-39 */
	const float *data;       /* params: f32 values (host memory, copied at load) */
	int qbits, qaxis;        /* quantized params: 8 or 4, axis 0 (rows) or 1 (columns); qbits 0 = f32 */
	const signed char *q;    /* codes in the reference packing (host memory) */
	const float *qs;         /* one scale per channel (host memory) */
	int index;               /* inputs: position in the entry signature */
} tg_cuda_value;

typedef struct {
	int T, reverse, tid;     /* Scan, src/tg.h:140-147 */
	int nc; const int *c, *init, *next;
	int nx; const int *x, *xt;
	int ny; const int *y, *ys;
} tg_cuda_scan;

typedef struct {
	int op;                  /* TG_CUDA_OP_* */
	int out, a[3], na;       /* value indices */
	float k;                 /* const */
	int init, maxit;         /* think: initial state, budget */
	float eps;               /* think: delta threshold, < 0 = none */
	int yield, tid, halt;    /* think: next state, steps slot, halting scalar or -1 */
	float hthr;              /* think: learned-halt threshold */
	int body, nbody;         /* think/scan: body = ins[body .. body + nbody) */
	int scan;                /* scan: index into tg_cuda_program.scans, else -1 */
} tg_cuda_ins;

typedef struct {
	int nval; const tg_cuda_value *val;
	int nins; const tg_cuda_ins *ins;
	int ntop;                /* the top-level block is ins[0 .. ntop) */
	int nscan; const tg_cuda_scan *scans;
	int ninputs; const int *inputs; /* value index of each entry input, in order */
	int output;
	int nthink;              /* steps slots per row */
	int nupd;                /* state updates; > 0 is rejected (rows would not be independent) */
} tg_cuda_program;

typedef struct tg_cuda_model tg_cuda_model;

/* Validate a program, plan its device arena and upload its params to every
 * selected GPU. TG_CUDA_EUNSUPPORTED for stateful models (nupd > 0) and ops the
 * device executor does not implement. */
int tg_cuda_load(const tg_cuda_program *p, tg_cuda_model **out);
/* Run rows independent samples. all: rows * per floats (host), each row the
 * concatenated inputs; out: rows * n floats; steps: rows * nt ints (nt >= the
 * program's nthink, may be NULL when nthink == 0). Rows keep input order; the
 * call blocks until out and steps are written. Rows are sharded across the
 * selected GPUs in contiguous blocks. */
int tg_cuda_batch(tg_cuda_model *g, const float *all, long rows, int per, float *out, int n, int *steps, int nt);
/* Page-lock [p, p + bytes) of the caller's host memory for every selected GPU
 * (after tg_cuda_init). A tg_cuda_batch whose input rows, output rows and steps
 * each lie inside one registered range copies straight between those buffers and
 * the GPUs; otherwise it goes through the library's own page-locked staging
 * buffers. For long-lived buffers such as the batch branch's sample array and
 * output block (src/main.c:400-444); registration costs far more than one copy.
 * Unregister (by the same p) before the memory is freed, and not while a call
 * uses it; tg_cuda_shutdown unregisters what is left. EINVAL for a range that
 * overlaps one already registered. */
int tg_cuda_host_register(void *p, size_t bytes);
int tg_cuda_host_unregister(void *p);
/* Same, with every buffer already on device 0 of the selection (device pointers,
 * asynchronous on stream). Used for measurements with inputs resident in HBM. */
int tg_cuda_batch_device(tg_cuda_model *g, const float *all, long rows, float *out, int *steps, void *stream);
void tg_cuda_free(tg_cuda_model *g);
/* 1 when the model's rows run on a kernel generated for this program (compiled
 * at load time with NVRTC for sm_100a), 0 when they run on the general tape
 * interpreter kernel; then `why` (n bytes, may be NULL) receives the reason.
 * TG_CUDA_ROWVM=interp in the environment at load time selects the interpreter.
 * Both are GPU kernels with the same arithmetic. No reference counterpart: the
 * reference's VM is the interpreter (src/vm.c:475-481). */
int tg_cuda_model_jit(const tg_cuda_model *g, char *why, int n);

/* Micro-batching for servers (`tgc serve` / `tgc stream`, src/serve.c:129-149): many
 * threads each submit one row (tg_cuda_batcher_run blocks until that row's output and
 * think steps are written); one dispatcher thread gathers the waiting rows -- up to
 * max_rows, or those that arrive within max_wait_us of the first -- into one
 * tg_cuda_batch call. Host buffers; rows sized as the model's (per values in, n out,
 * nthink steps; steps may be NULL when nthink == 0). A failed batch returns its status
 * to every row in it. tg_cuda_batcher_free answers the rows already queued, then stops;
 * the model must outlive the batcher. */
typedef struct tg_cuda_batcher tg_cuda_batcher;
int tg_cuda_batcher_new(tg_cuda_model *g, int max_rows, int max_wait_us, tg_cuda_batcher **out);
int tg_cuda_batcher_run(tg_cuda_batcher *b, const float *row, float *out, int *steps);
int tg_cuda_batcher_stats(tg_cuda_batcher *b, long *rows, long *batches);
void tg_cuda_batcher_free(tg_cuda_batcher *b);
/* The CUDA source generated for a program (written to src, n bytes, NUL-terminated,
 * may be NULL; *len = its full length), and with compile != 0 its compilation for
 * sm_100a. Needs neither tg_cuda_init nor a GPU. TG_CUDA_EUNSUPPORTED when the
 * program is beyond the generator's limits (such a model runs on the interpreter). */
int tg_cuda_program_kernel(const tg_cuda_program *p, char *src, long n, long *len, int compile);

/* ---- decoder language models (the Qwen3 import) ---------------------------
 * Weights follow examples/qwen3/import.py:37-60: every linear weight is stored
 * as W^T [in, out] and used as x @ W, so it is quantized on axis 1 (one scale
 * per output column, src/ops.c:310-320). Per-head projections are separate
 * params in the program; here they arrive concatenated along the output axis
 * (q: head h at columns h*HD..), which keeps each head's own column scales.
 * Wo arrives as the per-head params stacked along the input axis ([NQ*HD, D]);
 * its scales are per head and column: wo_s[h*D + n]. */
typedef struct {
	const signed char *q;    /* codes, reference packing over the [in, out] matrix */
	const float *s;          /* scales, one per output column (wo: per head and column) */
} tg_cuda_qmat;

typedef struct {
	int layers, hidden, nq, nkv, head_dim, ffn, vocab;
	int bits;                /* 8 or 4 */
	float eps;               /* rmsnorm epsilon of the program (1e-6, runtime/tg_rt.h:172) */
	float attn_scale;        /* the f32 constant the program multiplies scores by */
	double rope_theta;
	const float *embed;      /* E [vocab, hidden] f32 (take operand, never quantized) */
	const float *final_norm; /* lnf [hidden] */
	tg_cuda_qmat lm_head;    /* LM [hidden, vocab] */
	const float *const *ln1, *const *ln2, *const *qn, *const *kn; /* per layer */
	const tg_cuda_qmat *wq, *wk, *wv, *wo, *wg, *wu, *wd;          /* per layer */
} tg_cuda_lm_desc;

typedef struct tg_cuda_lm tg_cuda_lm;

int tg_cuda_lm_load(const tg_cuda_lm_desc *d, int max_seqs, int max_len, tg_cuda_lm **out);
/* Prefill nseq sequences of T token ids each (ids as f32, the program's input
 * type) and return the logits of the last position, [nseq, vocab]. */
int tg_cuda_lm_forward(tg_cuda_lm *g, const float *ids, long nseq, int T, float *logits);
/* Greedy decode: prefill, then nnew argmax tokens per sequence (tokens [nseq, nnew]),
 * each step feeding the previous token back through a per-sequence KV cache. */
int tg_cuda_lm_generate(tg_cuda_lm *g, const float *ids, long nseq, int T, int nnew, int *tokens);
void tg_cuda_lm_free(tg_cuda_lm *g);

/* Measurements of the last tg_cuda_lm_forward / _generate call (no reference
 * counterpart: the reference's --profile times VM instructions, src/vm.c:100-193).
 * Times are CUDA-event device times on the engine streams; with several devices,
 * device_ms is the maximum and the rest are sums. Per-kernel-class times are
 * collected only after tg_cuda_lm_profile(g, 1). */
typedef struct {
	double device_ms;          /* first to last launch of the call */
	long launches;             /* kernels the call launched */
	double attn_decode_ms;     /* KV-cache attention launches */
	double attn_decode_bytes;  /* their algorithmic bytes: K and V rows read, q read, output written */
	long attn_decode_launches;
	double attn_prefill_ms;    /* causal attention of the prefill */
	double attn_prefill_flops; /* 4 * head_dim per (query, key) pair kept by the causal mask */
	double gemm_ms;            /* tensor-core GEMMs */
	double gemm_flops;         /* 2 M N K per GEMM (the useful work, not the bf16 hi/lo passes) */
	long gemm_launches;
	double gemm_weight_bytes;  /* the weight operands the GEMMs read: bf16 tiles, or packed codes
	                              (+ scales) for the batches that dequantize in the kernel */
	double decode_gemm_ms;     /* the part of gemm_ms spent in the decode steps */
	double decode_gemm_weight_bytes; /* the part of gemm_weight_bytes read by the decode steps */
} tg_cuda_lm_stats;
int tg_cuda_lm_profile(tg_cuda_lm *g, int enable);
int tg_cuda_lm_get_stats(const tg_cuda_lm *g, tg_cuda_lm_stats *out);

/* ---- stacked selective-SSM blocks -------------------------------------------------
 * `tgc batch` over a program of Mamba-style blocks written with the reference's
 * ops (scan with carries, outer, broadcasting, softplus, exp, silu, rmsnorm,
 * x @ W matmuls; src/vm.c:364-382 for the scan), one sequence per row. Per block
 * b and step t, with u_t the residual stream [d_model] and the carries h
 * [d_inner, d_state] and c1..c3 [d_inner] (the last three x, zero at t = 0):
 *   n  = rmsnorm(u_t) * norm[b];      x = n @ w_x;   z = n @ w_z
 *   xc = c3*conv_w[0] + c2*conv_w[1] + c1*conv_w[2] + x*conv_w[3] + conv_b
 *   xs = silu(xc);  r = xs @ w_r;  bt = xs @ w_b;  ct = xs @ w_c
 *   dt = softplus(r @ w_dt + dt_b)
 *   e  = exp(-(reshape(dt, d_inner, 1) * a));  h = e * h + (1 - e) / a * outer(xs, bt)
 *   u_t = u_t + ((h @ ct + d * xs) * silu(z)) @ w_o
 * and the output row t is rmsnorm(u_t) * final_norm. The matrices are x @ W
 * (axis 1) int8/int4 codes with one scale per output column, as `tgc quantize`
 * writes them; a [d_inner, d_state] must be positive. */
typedef struct {
	int blocks, d_model, d_inner, d_state, dt_rank;
	int bits;
	float eps;
	const float *final_norm;                          /* [d_model] */
	const float *const *norm;                         /* per block [d_model] */
	const float *const *conv_w;                       /* per block [4][d_inner] */
	const float *const *conv_b, *const *dt_b, *const *d; /* per block [d_inner] */
	const float *const *a;                            /* per block [d_inner, d_state] */
	const tg_cuda_qmat *w_x, *w_z, *w_r, *w_b, *w_c, *w_dt, *w_o; /* per block */
} tg_cuda_ssm_desc;

typedef struct tg_cuda_ssm tg_cuda_ssm;

/* max_seqs sequences run at once per device; chunk steps of each are in flight
 * per pass (the token block of every GEMM is max_seqs * chunk rows). */
int tg_cuda_ssm_load(const tg_cuda_ssm_desc *d, int max_seqs, int chunk, tg_cuda_ssm **out);
/* u, out: host [nseq][T][d_model] f32 (out may not alias u). */
int tg_cuda_ssm_forward(tg_cuda_ssm *g, const float *u, long nseq, int T, float *out);
/* The same on device buffers of the first device, on its stream (no copies). */
int tg_cuda_ssm_forward_device(tg_cuda_ssm *g, const float *u, long nseq, int T, float *out);
void tg_cuda_ssm_free(tg_cuda_ssm *g);

/* Measurements of the last forward (no reference counterpart). Times are CUDA-event
 * device times; with several devices device_ms is the maximum and the rest are sums.
 * The per-kernel-class times are collected only after tg_cuda_ssm_profile(g, 1). */
typedef struct {
	double device_ms;   /* first to last launch of the call */
	long launches;      /* kernels the call launched */
	double gemm_ms;     /* the three projections of every block (tensor cores) */
	double gemm_flops;  /* 2 M N K of the useful columns (not the bf16 hi/lo passes or padding) */
	long gemm_launches;
	double scan_ms;     /* the selective scan (dt projection, state update, readout, gate) */
	double scan_flops;  /* per (token, channel): 2 dt_rank + 7 d_state + 2 d_state + 4, plus
	                       the d_state exps, softplus and silu counted as one flop each */
	long scan_launches;
} tg_cuda_ssm_stats;
int tg_cuda_ssm_profile(tg_cuda_ssm *g, int enable);
int tg_cuda_ssm_get_stats(const tg_cuda_ssm *g, tg_cuda_ssm_stats *out);

#ifdef __cplusplus
}
#endif
#endif
