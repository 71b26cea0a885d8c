/* tgc_cuda.c -- the reference's tgc driver with `tgc batch ... --device cuda`.
 *
 * The reference's own main() (src/main.c, compiled with -Dmain=tgc_ref_main) handles
 * every command. This file adds what a maintainer adds to its batch branch
 * (src/main.c:400-444): with `--device cuda` the rows of each block run on the GPUs
 * through libtgcuda (tg_cuda_batch) instead of par_for(batch_rows) over the VM.
 * Everything around that call follows the reference's branch step for step: the model is
 * loaded and planned, the whole input is read and validated (load_samples' rules and
 * messages), the program is handed to the library, and only then is the output file
 * opened, so every error -- a bad row, an unsupported program, no GPU -- ends the run
 * before the output exists (src/main.c:414-419). Rows come back in input order and are
 * written with io_write_row, so text output is byte-compatible with the CPU path's format.
 *
 *   tgc_cuda [flags] batch MODEL DATA [-o OUT] --device cuda
 *   tgc_cuda [flags] stream MODEL [SRC] [-o DST] --device cuda
 *                                            row in, row out, flushed (src/serve.c:251-285):
 *                                            each row runs through the micro-batcher
 *                                            (tg_cuda_batcher_run), the compute of run_line
 *                                            (src/serve.c:129-149); SRC/DST '-' or a file
 *   tgc_cuda cuda-kernel MODEL [-o OUT.cu]   the CUDA source generated for MODEL, compiled
 *                                            for sm_100a without a GPU (a build-time check)
 *   tgc_cuda <anything else>                 the reference's tgc, unchanged
 *
 * Built with the reference's sources (oracle/Makefile, target tgc_cuda). */
#define _GNU_SOURCE /* getline */
#include "tg.h"
#include "tg_cuda.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "cuda_host.h"

int tgc_ref_main(int argc, char **argv); /* src/main.c's main */

static void usage_cuda(void)
{
	fputs("usage: tgc batch <file> <data> [-o out] --device cuda\n"
	      "       tgc stream <file> [src] [-o dst] --device cuda\n"
	      "       tgc cuda-kernel <file> [-o out.cu]\n", stderr);
	exit(2);
}

/* The batch input as one row-major array of `per` floats per sample, validated completely
 * first: the rules and messages of the reference's load_samples (src/main.c:177-214). */
static float *samples(const char *data, int per, const char *model, int *rows)
{
	if (io_is_binary(data)) {
		int cnt;
		float *all = io_load(data, &cnt);
		if (cnt % per) die(NULL, 0, "'%s': %d values is not a multiple of the %d per sample", data, cnt, per);
		*rows = cnt / per;
		return all;
	}
	char *raw = read_file(data, NULL);
	int nrows = 0;
	float *all = NULL;
	for (int fill = 0; fill < 2; fill++) { /* count and check every row, then parse */
		if (fill) all = xmalloc((size_t)(nrows ? nrows : 1) * (size_t)per * sizeof *all);
		int r = 0, line = 1;
		for (char *s = raw; *s; line++) {
			char *nl = strchr(s, '\n');
			if (nl) *nl = 0;
			const char *bad;
			int k = io_parse_row(s, NULL, 0, &bad);
			if (k < 0) die(data, line, "bad number near '%.20s'", bad);
			if (k > 0 && k != per) die(data, line, "row has %d values, model %s needs %d per sample", k, model, per);
			if (k > 0) {
				if (fill) io_parse_row(s, all + (size_t)r * (size_t)per, per, &bad);
				r++;
			}
			if (nl) *nl = '\n';
			if (!nl) break;
			s = nl + 1;
		}
		nrows = r;
	}
	xfree(raw);
	*rows = nrows;
	return all;
}

static FILE *open_out(const char *path)
{
	FILE *f = fopen(path, io_is_binary(path) ? "wb" : "w");
	if (!f) die(NULL, 0, "cannot write '%s'", path);
	return f;
}

static void close_out(FILE *f, const char *path)
{
	if (ferror(f) | fclose(f)) die(NULL, 0, "write failed '%s'", path);
}

static int batch_cuda(int argc, char **argv)
{
	const char *opath = NULL;
	if (argc >= 5 && strcmp(argv[argc - 2], "-o") == 0) { /* a trailing -o PATH pair */
		opath = argv[argc - 1];
		argc -= 2;
	}
	if (argc != 4) usage_cuda();
	const char *data = argv[3];
	Module *m = load_module(argv[2]);
	double tp = tr_now_ms();
	plan(m);
	if (tr_on(1)) {
		tr_begin(1, "plan");
		tr_num("arena_bytes", m->arena * 4);
		tr_num("ms", tr_now_ms() - tp);
		tr_end("arena %d bytes in %.2f ms", m->arena * 4, tr_now_ms() - tp);
	}
	int per = 0;
	for (int i = 0; i < m->ninputs; i++) per += shape_numel(&m->val[m->inputs[i]].sh);
	int n = shape_numel(&m->val[m->output].sh), nt = m->nthink ? m->nthink : 1;
	int obin = opath && io_is_binary(opath);

	/* 1. load and validate everything, and hand the program to the GPUs, before the output exists */
	int rows;
	float *all = samples(data, per, m->name, &rows);
	tg_signals(); /* a stop request ends the batch after the current block */
	double tb = tr_now_ms();
	tg_cuda_model *gpu = cuda_load(m);
	if (tr_on(1)) {
		char why[256];
		int jit = tg_cuda_model_jit(gpu, why, sizeof why);
		tr_begin(1, "device");
		tr_str("kernel", jit ? "generated" : "interpreter");
		tr_end("--device cuda: %s%s%s", jit ? "kernel generated for the program" : "tape interpreter (", jit ? "" : why,
		       jit ? "" : ")");
	}
	FILE *f = opath ? open_out(opath) : stdout;

	/* 2. blocks of up to 2^20 rows on every GPU; rows come back in input order */
	int block = rows < (1 << 20) ? (rows > 0 ? rows : 1) : 1 << 20;
	float *out = xmalloc((size_t)block * (size_t)n * sizeof *out);
	int *steps = xmalloc((size_t)block * (size_t)nt * sizeof *steps);
	/* page-locked once, so each chunk moves by DMA straight from these buffers */
	int reg = rows > 0 && !tg_cuda_host_register(all, (size_t)rows * (size_t)per * sizeof(float)) &&
		  !tg_cuda_host_register(out, (size_t)block * (size_t)n * sizeof(float)) &&
		  !tg_cuda_host_register(steps, (size_t)block * (size_t)nt * sizeof(int));
	long sum[64] = { 0 };
	int mn[64], mx[64], done = 0;
	for (int b0 = 0; b0 < rows && !tg_stopping(); b0 += block) {
		int cnt = rows - b0 < block ? rows - b0 : block;
		if (tg_cuda_batch(gpu, all + (size_t)b0 * (size_t)per, cnt, per, out, n, steps, nt))
			die(NULL, 0, "--device cuda: %s", tg_cuda_error());
		for (int r = 0; r < cnt; r++, done++) {
			const int *st = steps + (size_t)r * (size_t)nt;
			for (int t = 0; t < m->nthink && t < 64; t++) {
				sum[t] += st[t];
				if (!done || st[t] < mn[t]) mn[t] = st[t];
				if (!done || st[t] > mx[t]) mx[t] = st[t];
			}
			io_write_row(f, obin, out + (size_t)r * (size_t)n, n, st, obin ? 0 : m->nthink);
		}
	}
	if (opath) close_out(f, opath);
	else fflush(stdout);
	if (reg) {
		tg_cuda_host_unregister(all);
		tg_cuda_host_unregister(out);
		tg_cuda_host_unregister(steps);
	}
	double ms = tr_now_ms() - tb;
	if (tr_on(1)) {
		tr_begin(1, "batch");
		tr_num("rows", done);
		tr_str("device", "cuda");
		tr_num("ms", ms);
		tr_num("us_per_row", done ? 1e3 * ms / done : 0);
		tr_end("%d row(s) in %.2f ms (%.1f us/row) on --device cuda", done, ms, done ? 1e3 * ms / done : 0.0);
		for (int t = 0; t < m->nthink && t < 64 && done; t++) {
			tr_begin(1, "think");
			tr_num("loop", t);
			tr_num("steps_min", mn[t]);
			tr_num("steps_mean", (double)sum[t] / done);
			tr_num("steps_max", mx[t]);
			tr_end("think[%d] over batch: steps min %d mean %.2f max %d", t, mn[t], (double)sum[t] / done, mx[t]);
		}
	}
	tg_cuda_free(gpu);
	tg_cuda_shutdown();
	xfree(out);
	xfree(steps);
	xfree(all);
	return tg_exit_status();
}

/* tgc stream on the GPUs: the loop of stream_main (src/serve.c:251-285) with run_line's
 * compute (src/serve.c:129-149) handed to the micro-batcher. A row with a bad number or the
 * wrong count gets the reference's `error:` line and the stream goes on; a row the device
 * could not run gets `error: <the library's text>`. One reader thread submits one row at a
 * time, so the batcher runs each row at once (max_wait 0); a server with many connections
 * would let rows of different connections share batches. tcp:// endpoints stay with the
 * reference's path. */
static int stream_cuda(int argc, char **argv)
{
	const char *opath = NULL;
	if (argc >= 5 && strcmp(argv[argc - 2], "-o") == 0) {
		opath = argv[argc - 1];
		argc -= 2;
	}
	if (argc != 3 && argc != 4) usage_cuda();
	const char *src = argc == 4 ? argv[3] : "-";
	if (strncmp(src, "tcp://", 6) == 0 || (opath && strncmp(opath, "tcp://", 6) == 0))
		die(NULL, 0, "--device cuda: stream reads and writes '-' or files; tcp:// runs on the CPU path");
	Module *m = load_module(argv[2]);
	plan(m);
	int per = 0;
	for (int i = 0; i < m->ninputs; i++) per += shape_numel(&m->val[m->inputs[i]].sh);
	const int n = shape_numel(&m->val[m->output].sh), nt = m->nthink ? m->nthink : 1;
	tg_cuda_model *gpu = cuda_load(m);
	tg_cuda_batcher *bt = NULL;
	if (tg_cuda_batcher_new(gpu, 8192, 0, &bt)) die(NULL, 0, "--device cuda: %s", tg_cuda_error());
	FILE *in = strcmp(src, "-") ? fopen(src, "r") : stdin;
	if (!in) die(NULL, 0, "cannot open '%s'", src);
	FILE *out = opath ? fopen(opath, "w") : stdout;
	if (!out) die(NULL, 0, "cannot write '%s'", opath);
	tg_signals();
	float *row = xmalloc((size_t)(per ? per : 1) * sizeof *row), *o = xmalloc((size_t)n * sizeof *o);
	int *steps = xmalloc((size_t)nt * sizeof *steps);
	char *line = NULL;
	size_t cap = 0;
	long rows = 0;
	double t0 = tr_now_ms();
	ssize_t len;
	while (!tg_stopping() && (len = getline(&line, &cap, in)) >= 0) {
		while (len > 0 && (line[len - 1] == '\n' || line[len - 1] == '\r')) line[--len] = 0; /* as serve.c's read_line */
		const char *bad;
		const int k = io_parse_row(line, NULL, 0, &bad);
		if (k == 0) continue;
		rows++;
		if (k < 0) fprintf(out, "error: bad number near '%.20s'\n", bad);
		else if (k != per) fprintf(out, "error: row has %d values, model %s needs %d\n", k, m->name, per);
		else {
			io_parse_row(line, row, per, &bad);
			if (tg_cuda_batcher_run(bt, row, o, steps)) fprintf(out, "error: %s\n", tg_cuda_error());
			else io_write_row(out, 0, o, n, steps, m->nthink);
		}
		if (fflush(out)) break; /* peer gone */
	}
	free(line);
	if (in != stdin) fclose(in);
	if (out != stdout && fclose(out)) die(NULL, 0, "write failed '%s'", opath);
	if (tr_on(1)) {
		tr_begin(1, "stream");
		tr_num("rows", (double)rows);
		tr_num("ms", tr_now_ms() - t0);
		tr_end("%ld row(s) streamed on --device cuda", rows);
	}
	tg_cuda_batcher_free(bt);
	tg_cuda_free(gpu);
	tg_cuda_shutdown();
	xfree(row);
	xfree(o);
	xfree(steps);
	return tg_exit_status();
}

/* The kernel the library generates for MODEL, compiled for sm_100a: no GPU needed. */
static int cuda_kernel(int argc, char **argv)
{
	const char *opath = NULL;
	if (argc == 5 && strcmp(argv[3], "-o") == 0) opath = argv[4];
	else if (argc != 3) usage_cuda();
	Module *m = load_module(argv[2]);
	plan(m);
	CudaFlat cf;
	cuda_flatten(m, &cf);
	long len = 0;
	int rc = tg_cuda_program_kernel(&cf.p, NULL, 0, &len, 0);
	if (rc == TG_CUDA_EUNSUPPORTED) {
		printf("interpreter: %s\n", tg_cuda_error());
		cuda_flat_free(&cf);
		return 0;
	}
	if (rc) die(NULL, 0, "--device cuda: %s", tg_cuda_error());
	char *src = xmalloc((size_t)len + 1);
	if (tg_cuda_program_kernel(&cf.p, src, len + 1, &len, 1)) die(NULL, 0, "--device cuda: %s", tg_cuda_error());
	FILE *f = opath ? fopen(opath, "w") : stdout;
	if (!f) die(NULL, 0, "cannot write '%s'", opath);
	fputs(src, f);
	if (opath && fclose(f)) die(NULL, 0, "write failed '%s'", opath);
	fprintf(stderr, "cuda-kernel: %ld bytes of CUDA source, compiled for sm_100a\n", len);
	xfree(src);
	cuda_flat_free(&cf);
	return 0;
}

int main(int argc, char **argv)
{
	/* `--device cuda` and the global flags the batch path honours, as src/main.c:291-327 parses them */
	int cuda = 0, k = 1;
	const char *cmd = NULL, *log = NULL;
	char **orig = xmalloc((size_t)(argc + 1) * sizeof *orig);
	memcpy(orig, argv, (size_t)(argc + 1) * sizeof *orig);
	for (int i = 1; i < argc; i++) {
		if (strcmp(argv[i], "--device") == 0) {
			if (++i == argc) die(NULL, 0, "--device expects 'cuda'");
			if (strcmp(argv[i], "cuda") != 0) die(NULL, 0, "--device: only 'cuda' is available, got '%s'", argv[i]);
			cuda = 1;
		} else if (strcmp(argv[i], "-v") == 0 || strcmp(argv[i], "--verbose") == 0) tg_verbose = tg_verbose > 1 ? tg_verbose : 1;
		else if (strcmp(argv[i], "-vv") == 0) tg_verbose = 2;
		else if (strcmp(argv[i], "--log") == 0) {
			if (++i == argc) usage_cuda();
			log = argv[i];
			argv[k++] = argv[i - 1], argv[k++] = argv[i];
		} else if (strcmp(argv[i], "-j") == 0 || strcmp(argv[i], "--threads") == 0) {
			if (++i == argc) usage_cuda();
			argv[k++] = argv[i - 1], argv[k++] = argv[i];
		} else {
			if (!cmd && argv[i][0] != '-') cmd = argv[i];
			argv[k++] = argv[i];
		}
	}
	argv[k] = NULL;
	int ours = cuda || (cmd && strcmp(cmd, "cuda-kernel") == 0);
	if (ours && log) {
		tr_open_log(log);
		atexit(tr_close_log);
	}
	if (cmd && strcmp(cmd, "cuda-kernel") == 0) {
		int n = 1;
		for (int i = 1; i < k; i++) {
			if (strcmp(argv[i], "--log") == 0 || strcmp(argv[i], "-j") == 0 || strcmp(argv[i], "--threads") == 0) {
				i++;
				continue;
			}
			if (argv[i][0] == '-' && strcmp(argv[i], "-o") != 0) die(NULL, 0, "cuda-kernel: unexpected flag '%s'", argv[i]);
			argv[n++] = argv[i];
		}
		argv[n] = NULL;
		return cuda_kernel(n, argv);
	}
	if (!cuda) return tgc_ref_main(argc, orig); /* not ours: the reference, with its arguments untouched */
	if (!cmd || (strcmp(cmd, "batch") != 0 && strcmp(cmd, "stream") != 0))
		die(NULL, 0, "--device cuda applies to `tgc batch` and `tgc stream`");
	/* drop the -j/--log pairs the reference would have consumed: the GPU path has no CPU threads */
	int n = 1;
	for (int i = 1; i < k; i++) {
		if (strcmp(argv[i], "-j") == 0 || strcmp(argv[i], "--threads") == 0 || strcmp(argv[i], "--log") == 0) {
			i++;
			continue;
		}
		if (argv[i][0] == '-' && strcmp(argv[i], "-o") != 0 && strcmp(argv[i], "-") != 0)
			die(NULL, 0, "--device cuda: option '%s' is not available on the GPU path", argv[i]);
		argv[n++] = argv[i];
	}
	argv[n] = NULL;
	return strcmp(cmd, "stream") == 0 ? stream_cuda(n, argv) : batch_cuda(n, argv);
}
