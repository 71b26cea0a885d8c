// batcher.cu -- micro-batching of single-row requests (tg_cuda_batcher_*): the device side
// of `tgc serve` / `tgc stream`. The reference runs each request line on its connection's
// thread with vm_run_into (src/serve.c:129-149, run_line); here connection threads hand
// their rows to one dispatcher thread, which gathers whatever is waiting -- up to max_rows,
// or what has arrived within max_wait_us of the first row -- into one tg_cuda_batch call
// and hands every thread its own output row. Rows keep no order across threads (each
// request gets its own result); a thread's own rows are answered in submission order
// because it waits for each.
#include <string.h>

#include <chrono>
#include <condition_variable>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

namespace {

struct Request {
	const float *in;
	float *out;
	int *steps;
	int rc = 1;          // 1 pending, else the batch's status
	std::string err;     // the batch's error text when rc != 0
	bool done = false;
};

} // namespace

struct tg_cuda_batcher {
	tg_cuda_model *g = nullptr;
	int per = 0, nout = 0, nthink = 0, max_rows = 0;
	std::chrono::microseconds max_wait{ 0 };
	std::mutex mu;
	std::condition_variable cv_work, cv_done;
	std::deque<Request *> q;
	bool stop = false;
	long rows = 0, batches = 0;
	std::thread th;

	void loop()
	{
		std::vector<float> in, out;
		std::vector<int> st;
		std::vector<Request *> take;
		std::unique_lock<std::mutex> lk(mu);
		for (;;) {
			cv_work.wait(lk, [&] { return stop || !q.empty(); });
			if (q.empty() && stop) return;
			// the first row waits at most max_wait for company, or until max_rows are queued
			const auto deadline = std::chrono::steady_clock::now() + max_wait;
			while (!stop && (int)q.size() < max_rows && std::chrono::steady_clock::now() < deadline)
				cv_work.wait_until(lk, deadline);
			take.clear();
			while (!q.empty() && (int)take.size() < max_rows) {
				take.push_back(q.front());
				q.pop_front();
			}
			lk.unlock();
			const long n = (long)take.size();
			const int nt = nthink > 0 ? nthink : 1;
			in.resize((size_t)n * per);
			out.resize((size_t)n * nout);
			st.assign((size_t)n * nt, 0);
			for (long i = 0; i < n; i++) memcpy(in.data() + (size_t)i * per, take[i]->in, (size_t)per * sizeof(float));
			int rc = tg_cuda_batch(g, in.data(), n, per, out.data(), nout, st.data(), nt);
			std::string err = rc ? tg_cuda_error() : "";
			lk.lock();
			for (long i = 0; i < n; i++) {
				Request *r = take[i];
				if (!rc) {
					memcpy(r->out, out.data() + (size_t)i * nout, (size_t)nout * sizeof(float));
					if (r->steps && nthink > 0) memcpy(r->steps, st.data() + (size_t)i * nt, (size_t)nthink * sizeof(int));
				}
				r->rc = rc;
				r->err = err;
				r->done = true;
			}
			rows += n;
			batches++;
			cv_done.notify_all();
		}
	}
};

using namespace tgc;

extern "C" int tg_cuda_batcher_new(tg_cuda_model *g, int max_rows, int max_wait_us, tg_cuda_batcher **out)
{
	clear_err();
	if (!g || !out) return set_err(TG_CUDA_EINVAL, "tg_cuda_batcher_new: NULL argument");
	*out = nullptr;
	if (max_rows <= 0 || max_wait_us < 0)
		return set_err(TG_CUDA_EINVAL, "tg_cuda_batcher_new: bad limits (max_rows %d, max_wait_us %d)", max_rows, max_wait_us);
	tg_cuda_batcher *b = new tg_cuda_batcher;
	b->g = g;
	model_shape(g, &b->per, &b->nout, &b->nthink);
	b->max_rows = max_rows;
	b->max_wait = std::chrono::microseconds(max_wait_us);
	b->th = std::thread([b] { b->loop(); });
	*out = b;
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_batcher_run(tg_cuda_batcher *b, const float *row, float *out, int *steps)
{
	clear_err();
	if (!b || !row || !out) return set_err(TG_CUDA_EINVAL, "tg_cuda_batcher_run: NULL argument");
	if (b->nthink > 0 && !steps) return set_err(TG_CUDA_EINVAL, "tg_cuda_batcher_run: steps is NULL");
	Request r;
	r.in = row, r.out = out, r.steps = steps;
	std::unique_lock<std::mutex> lk(b->mu);
	if (b->stop) return set_err(TG_CUDA_EINVAL, "tg_cuda_batcher_run: the batcher is stopping");
	b->q.push_back(&r);
	b->cv_work.notify_one();
	b->cv_done.wait(lk, [&] { return r.done; });
	if (r.rc) return set_err(r.rc, "%s", r.err.c_str());
	return TG_CUDA_OK;
}

extern "C" int tg_cuda_batcher_stats(tg_cuda_batcher *b, long *rows, long *batches)
{
	if (!b) return set_err(TG_CUDA_EINVAL, "tg_cuda_batcher_stats: NULL batcher");
	std::lock_guard<std::mutex> lk(b->mu);
	if (rows) *rows = b->rows;
	if (batches) *batches = b->batches;
	return TG_CUDA_OK;
}

extern "C" void tg_cuda_batcher_free(tg_cuda_batcher *b)
{
	if (!b) return;
	{
		std::lock_guard<std::mutex> lk(b->mu);
		b->stop = true;
	}
	b->cv_work.notify_all();
	b->th.join(); // requests already queued are answered first
	delete b;
}
