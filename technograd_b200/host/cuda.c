/* cuda.c -- the adapter a maintainer adds to the reference as src/cuda.c: it hands a
 * planned Module (src/tg.h:112-200) to libtgcuda through the C ABI of include/tg_cuda.h.
 *
 * cuda_flatten turns the Module's nested blocks into tg_cuda_program's flat instruction
 * array: a block occupies a contiguous range and the bodies of its think and scan loops
 * are appended after it. Values, instructions and scans keep the reference's own numbering
 * (the op codes are its enum Op), so nothing is renamed on the way. cuda_load flattens,
 * initialises the library on every visible GPU and loads the program; the library copies
 * what it needs, so the flat arrays are freed before it returns.
 *
 * Built with the reference's sources (oracle/Makefile, target tgc_cuda), never into the
 * library itself. */
#include "tg.h"
#include "tg_cuda.h"

#include <stdlib.h>
#include <string.h>

#include "cuda_host.h"

typedef struct {
	tg_cuda_ins *ins;
	int n, cap;
	tg_cuda_scan *scans;
	int nscan, capscan;
} Flat;

static int flat_block(Flat *f, const Block *b)
{
	int start = f->n;
	if (f->n + b->len > f->cap) {
		f->cap = 2 * (f->n + b->len) + 8;
		f->ins = xrealloc(f->ins, (size_t)f->cap * sizeof *f->ins);
	}
	f->n += b->len;
	for (int i = 0; i < b->len; i++) {
		const Ins *in = &b->v[i];
		tg_cuda_ins *o = &f->ins[start + i];
		memset(o, 0, sizeof *o);
		o->op = (int)in->op;
		o->out = in->out;
		o->na = in->na;
		for (int j = 0; j < 3; j++) o->a[j] = j < in->na ? in->a[j] : -1;
		o->k = in->k;
		o->init = in->init, o->maxit = in->maxit, o->eps = in->eps;
		o->yield = in->yield, o->tid = in->tid, o->halt = in->halt, o->hthr = in->hthr;
		o->body = -1, o->nbody = 0, o->scan = -1;
		if (in->op == OP_SCAN) {
			const Scan *s = in->sc;
			if (f->nscan == f->capscan) {
				f->capscan = f->capscan ? 2 * f->capscan : 4;
				f->scans = xrealloc(f->scans, (size_t)f->capscan * sizeof *f->scans);
			}
			tg_cuda_scan *c = &f->scans[f->nscan];
			c->T = s->T, c->reverse = s->reverse, c->tid = s->tid;
			c->nc = s->nc, c->c = s->c, c->init = s->init, c->next = s->next;
			c->nx = s->nx, c->x = s->x, c->xt = s->xt;
			c->ny = s->ny, c->y = s->y, c->ys = s->ys;
			o->scan = f->nscan++;
		}
	}
	for (int i = 0; i < b->len; i++) { /* bodies after the block, so its range stays contiguous */
		const Ins *in = &b->v[i];
		if (in->op != OP_THINK && in->op != OP_SCAN) continue;
		int body = flat_block(f, in->body); /* may move f->ins */
		f->ins[start + i].body = body;
		f->ins[start + i].nbody = in->body->len;
	}
	return start;
}

void cuda_flatten(const Module *m, CudaFlat *cf)
{
	tg_cuda_value *val = xmalloc((size_t)(m->nval ? m->nval : 1) * sizeof *val);
	for (int v = 0; v < m->nval; v++) {
		const Value *x = &m->val[v];
		tg_cuda_value *o = &val[v];
		memset(o, 0, sizeof *o);
		o->kind = (int)x->kind; /* VKind order: PARAM, INPUT, TMP, STATE */
		o->rank = x->sh.rank;
		for (int d = 0; d < 4; d++) o->dim[d] = d < x->sh.rank ? x->sh.dim[d] : 1;
		o->data = x->data;
		o->qbits = x->qbits, o->qaxis = x->qaxis, o->q = x->q, o->qs = x->qs;
		o->index = x->index;
	}
	Flat f;
	memset(&f, 0, sizeof f);
	flat_block(&f, &m->top);
	cf->val = val, cf->ins = f.ins, cf->scans = f.scans;
	tg_cuda_program p = { m->nval, val, f.n, f.ins, m->top.len, f.nscan, f.scans,
			      m->ninputs, m->inputs, m->output, m->nthink, m->nupd };
	cf->p = p;
}

void cuda_flat_free(CudaFlat *cf)
{
	xfree(cf->val);
	xfree(cf->ins);
	xfree(cf->scans);
	memset(cf, 0, sizeof *cf);
}

tg_cuda_model *cuda_load(const Module *m)
{
	CudaFlat cf;
	cuda_flatten(m, &cf);
	tg_cuda_model *g = NULL;
	if (tg_cuda_init(0, NULL) || tg_cuda_load(&cf.p, &g)) /* copies everything it needs */
		die(NULL, 0, "--device cuda: %s", tg_cuda_error());
	cuda_flat_free(&cf);
	return g;
}
