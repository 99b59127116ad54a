// cpu_executor.cu — routed experts on the host CPU and the asynchronous hand-off of their results.
//
// Reference: the CPU expert path CpuExperts::forward (src/moe/expert.rs:59-117) and the fused decode
// the miss stage calls (src/moe/stages/cpu_miss.rs:21-54, mistralrs_quant::fused_moe_decode: gate +
// up + SiLU per distinct (expert, row), then down and the router-weighted sum), and the executor
// that runs such a job on a worker thread and publishes its rows through the result doorbell
// (src/executor.rs:116-166, Pending::upload :220-231, SetFlag :330-378).
//
// moe_cpu_experts owns a host copy of the GGML stacks (Q8_0 or BF16) and computes any subset of a
// call's routed pairs in two passes over a pool of std::threads: pass 1 gives h = silu(gate x) *
// (up x) per selected pair (f32 accumulation, Q8_0 blocks dequantised on the fly), pass 2 gives
// y[t] = sum over the token's selected pairs, in slot order, of w * (down h). moe_executor runs
// those jobs FIFO on one worker thread and publishes each [T, H] f32 result into a host -> device
// moe_ring; the device takes it with moe_ring_device_take (bounded wait) and folds it into the
// GPU's output with moe_add_f32_into_bf16. A job that fails publishes zeros (so the device never
// waits for it) and latches its error, which the next submit returns (executor.rs:124).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "cpu_kernels.h"
#include "moe_internal.cuh"

using namespace moe;

namespace {

inline float bf16_bits_to_f32(uint16_t h) {
  const uint32_t b = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

// Worker threads reused by every call (starting threads per call cost ~0.4 ms of a 1.3 ms decode
// call). run(n, f) runs f(i) for i in [0, n) on the workers and the calling thread and returns when
// every worker has finished its share. One run at a time per pool: concurrent callers take turns.
class ThreadPool {
 public:
  explicit ThreadPool(int threads) {
    for (int i = 1; i < threads; ++i) workers_.emplace_back([this] { loop(); });
  }
  ~ThreadPool() {
    {
      std::lock_guard<std::mutex> l(m_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  void run(int n, const std::function<void(int)>& f) {
    if (n <= 0) return;
    std::lock_guard<std::mutex> call(call_m_);
    {
      std::lock_guard<std::mutex> l(m_);
      f_ = &f;
      n_ = n;
      next_.store(0);
      pending_ = (int)workers_.size();
      ++gen_;
    }
    cv_.notify_all();
    body();
    std::unique_lock<std::mutex> l(m_);
    done_cv_.wait(l, [&] { return pending_ == 0; });  // every worker has left body() for this run
    f_ = nullptr;
  }

 private:
  void body() {
    for (int i; (i = next_.fetch_add(1)) < n_;) (*f_)(i);
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> l(m_);
      cv_.wait(l, [&] { return stop_ || gen_ != seen; });
      if (stop_) return;
      seen = gen_;
      l.unlock();
      body();
      l.lock();
      if (--pending_ == 0) done_cv_.notify_one();
    }
  }
  std::vector<std::thread> workers_;
  std::mutex m_, call_m_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int)>* f_ = nullptr;
  int n_ = 0, pending_ = 0;
  std::atomic<int> next_{0};
  uint64_t gen_ = 0;
  bool stop_ = false;
};

// One pool per thread count, shared by every CPU-experts object of the process (a model has one per
// layer and runs them one at a time). The pools are created on first use and kept until the
// process exits: idle workers only wait on a condition variable.
ThreadPool* shared_pool(int threads) {
  static std::mutex m;
  static std::map<int, ThreadPool*>* pools = new std::map<int, ThreadPool*>();
  std::lock_guard<std::mutex> l(m);
  ThreadPool*& pool = (*pools)[threads];
  if (!pool) pool = new ThreadPool(threads);
  return pool;
}

}  // namespace

struct moe_cpu_experts {
  int E = 0, k = 0, H = 0, I = 0, wdtype = 0, threads = 1;
  std::vector<uint8_t> gate, up, down;  // GGML bytes, [E, N, K] stacked
  ThreadPool* pool = nullptr;           // shared: threads - 1 workers plus the calling thread

  int64_t row_bytes(int K) const { return wdtype == MOE_DTYPE_Q8_0 ? (int64_t)K / 32 * 34 : (int64_t)K * 2; }
};

struct moe_executor {
  moe_cpu_experts* cpu = nullptr;
  moe_ring* ring = nullptr;
  int64_t publish_timeout_us = 10'000'000;
  struct Job {
    std::vector<uint16_t> x;
    std::vector<uint32_t> ids;
    std::vector<float> w;
    std::vector<uint8_t> select;
    int T = 0, width = 0;
  };
  std::thread worker;
  std::mutex m;
  std::condition_variable cv, idle_cv;
  std::deque<Job> jobs;
  bool stop = false, busy = false;
  uint32_t next_target = 0;
  std::string error;  // latched worker error, returned by the next submit
  moe_status error_status = MOE_OK;
};

// Row r of expert e's [N, K] projection (GGML bytes) times nx f32 vectors: out[j] = row . xs[j].
static void row_dots(const moe_cpu_experts* c, const std::vector<uint8_t>& stack, int N, int K, int e, int r,
                     const float* const* xs, int nx, float* out) {
  const uint8_t* row = stack.data() + ((int64_t)e * N + r) * c->row_bytes(K);
  if (c->wdtype == MOE_DTYPE_Q8_0) cpu_dot_q8_0(row, xs, nx, K, out);
  else cpu_dot_bf16(reinterpret_cast<const uint16_t*>(row), xs, nx, K, out);
}

// Two passes over the selected pairs grouped by expert, so every weight row is read once per call
// however many of the call's tokens use the expert (the row dots take the expert's vectors
// together): pass 1 h = silu(gate x) * (up x) per pair, pass 2 ypair = w * (down h) per pair; then
// y[t] sums the token's pairs in slot order.
static moe_status cpu_forward_impl(const moe_cpu_experts* c, const uint16_t* x_bf16, const uint32_t* ids,
                                   const float* w, int T, int width, const uint8_t* select, float* y) {
  const int H = c->H, I = c->I, E = c->E;
  for (int64_t p = 0; p < (int64_t)T * width; ++p)
    if (ids[p] != MOE_ID_NONE && ids[p] >= (uint32_t)E)
      return fail(MOE_ERR_BAD_IDS, "moe_cpu_forward: routed expert id >= num_experts");
  std::vector<float> xf((size_t)T * H);
  for (size_t i = 0; i < xf.size(); ++i) xf[i] = bf16_bits_to_f32(x_bf16[i]);
  // selected pairs (weight-0 slots skipped, as the reference's fused decode does), grouped by expert
  std::vector<int> pairs;
  for (int p = 0; p < T * width; ++p)
    if ((!select || select[p]) && ids[p] != MOE_ID_NONE && w[p] != 0.0f) pairs.push_back(p);
  std::stable_sort(pairs.begin(), pairs.end(), [&](int a, int b) { return ids[a] < ids[b]; });
  std::vector<int> seg_start;  // experts' ranges in `pairs`
  for (size_t i = 0; i < pairs.size(); ++i)
    if (i == 0 || ids[pairs[i]] != ids[pairs[i - 1]]) seg_start.push_back((int)i);
  seg_start.push_back((int)pairs.size());
  const int n_seg = (int)seg_start.size() - 1;
  std::vector<float> h((size_t)pairs.size() * I), ypair((size_t)pairs.size() * H);
  constexpr int RB = 32;  // rows per task
  const int gu_blocks = (I + RB - 1) / RB, dn_blocks = (H + RB - 1) / RB;
  // pass 1
  c->pool->run(n_seg * gu_blocks, [&](int task) {
    const int sg = task / gu_blocks, r0 = (task % gu_blocks) * RB, r1 = std::min(I, r0 + RB);
    const int e = (int)ids[pairs[seg_start[sg]]];
    const int i0 = seg_start[sg], n = seg_start[sg + 1] - i0;
    std::vector<const float*> xs(n);
    for (int j = 0; j < n; ++j) xs[j] = xf.data() + (size_t)(pairs[i0 + j] / width) * H;
    std::vector<float> g(n), u(n);
    for (int r = r0; r < r1; ++r) {
      row_dots(c, c->gate, I, H, e, r, xs.data(), n, g.data());
      row_dots(c, c->up, I, H, e, r, xs.data(), n, u.data());
      for (int j = 0; j < n; ++j) h[(size_t)(i0 + j) * I + r] = g[j] / (1.0f + std::exp(-g[j])) * u[j];
    }
  });
  // pass 2
  c->pool->run(n_seg * dn_blocks, [&](int task) {
    const int sg = task / dn_blocks, r0 = (task % dn_blocks) * RB, r1 = std::min(H, r0 + RB);
    const int e = (int)ids[pairs[seg_start[sg]]];
    const int i0 = seg_start[sg], n = seg_start[sg + 1] - i0;
    std::vector<const float*> hs(n);
    for (int j = 0; j < n; ++j) hs[j] = h.data() + (size_t)(i0 + j) * I;
    std::vector<float> v(n);
    for (int r = r0; r < r1; ++r) {
      row_dots(c, c->down, H, I, e, r, hs.data(), n, v.data());
      for (int j = 0; j < n; ++j) ypair[(size_t)(i0 + j) * H + r] = w[pairs[i0 + j]] * v[j];
    }
  });
  // y[t]: the token's pairs in slot order
  std::vector<int> pos((size_t)T * width, -1);
  for (size_t i = 0; i < pairs.size(); ++i) pos[pairs[i]] = (int)i;
  c->pool->run(T, [&](int t) {
    float* yt = y + (size_t)t * H;
    for (int n = 0; n < H; ++n) yt[n] = 0.0f;
    for (int j = 0; j < width; ++j) {
      const int i = pos[(size_t)t * width + j];
      if (i < 0) continue;
      const float* yp = ypair.data() + (size_t)i * H;
      for (int n = 0; n < H; ++n) yt[n] += yp[n];
    }
  });
  return MOE_OK;
}

static void executor_loop(moe_executor* ex) {
  for (;;) {
    moe_executor::Job job;
    {
      std::unique_lock<std::mutex> lk(ex->m);
      ex->cv.wait(lk, [&] { return ex->stop || !ex->jobs.empty(); });
      if (ex->jobs.empty()) return;  // stop requested and nothing left
      job = std::move(ex->jobs.front());
      ex->jobs.pop_front();
      ex->busy = true;
    }
    std::vector<float> y((size_t)job.T * ex->cpu->H, 0.0f);
    moe_status st = cpu_forward_impl(ex->cpu, job.x.data(), job.ids.data(), job.w.data(), job.T, job.width,
                                     job.select.empty() ? nullptr : job.select.data(), y.data());
    std::string msg = st == MOE_OK ? std::string() : last_error_message();
    if (st != MOE_OK) std::fill(y.begin(), y.end(), 0.0f);  // publish zeros: the device never waits in vain
    uint32_t seq = 0;
    const moe_status ps = moe_ring_host_publish(ex->ring, y.data(), y.size() * sizeof(float), ex->publish_timeout_us, &seq);
    std::lock_guard<std::mutex> lk(ex->m);
    if (st != MOE_OK && ex->error_status == MOE_OK) {
      ex->error_status = MOE_ERR_WORKER;
      ex->error = "cpu executor job failed: " + msg;
    }
    if (ps != MOE_OK && ex->error_status == MOE_OK) {
      ex->error_status = MOE_ERR_WORKER;
      ex->error = "cpu executor could not publish its result: " + last_error_message();
    }
    ex->busy = false;
    ex->idle_cv.notify_all();
  }
}

extern "C" {

moe_status moe_cpu_experts_create(const moe_layer_desc* d, int n_threads, moe_cpu_experts** out) {
  if (!out) return fail(MOE_ERR_INVALID, "moe_cpu_experts_create: null out");
  *out = nullptr;
  if (!d) return fail(MOE_ERR_INVALID, "moe_cpu_experts_create: null desc");
  if (d->wdtype != MOE_DTYPE_Q8_0 && d->wdtype != MOE_DTYPE_BF16)
    return fail(MOE_ERR_UNSUPPORTED, "moe_cpu_experts_create: the CPU path serves Q8_0 and BF16 stacks");
  if (d->weights_on_device) return fail(MOE_ERR_INVALID, "moe_cpu_experts_create: stacks must be host memory");
  if (d->num_experts <= 0 || d->hidden <= 0 || d->inter <= 0 || d->hidden % 32 || d->inter % 32)
    return fail(MOE_ERR_INVALID, "moe_cpu_experts_create: bad shape");
  if (!d->gate || !d->up || !d->down) return fail(MOE_ERR_INVALID, "moe_cpu_experts_create: null stack");
  moe_cpu_experts* c = new moe_cpu_experts();
  c->E = d->num_experts;
  c->k = d->top_k;
  c->H = d->hidden;
  c->I = d->inter;
  c->wdtype = d->wdtype;
  c->threads = n_threads > 0 ? n_threads : (int)std::max(1u, std::thread::hardware_concurrency());
  c->pool = shared_pool(c->threads);
  const int64_t gu = c->row_bytes(c->H) * c->I * c->E, dn = c->row_bytes(c->I) * c->H * c->E;
  c->gate.assign(static_cast<const uint8_t*>(d->gate), static_cast<const uint8_t*>(d->gate) + gu);
  c->up.assign(static_cast<const uint8_t*>(d->up), static_cast<const uint8_t*>(d->up) + gu);
  c->down.assign(static_cast<const uint8_t*>(d->down), static_cast<const uint8_t*>(d->down) + dn);
  *out = c;
  return MOE_OK;
}

void moe_cpu_experts_destroy(moe_cpu_experts* c) { delete c; }

const char* moe_cpu_isa(void) { return cpu_dot_isa(); }

moe_status moe_cpu_forward(const moe_cpu_experts* c, const uint16_t* x, const uint32_t* ids, const float* weights,
                           int T, int width, const uint8_t* select, float* y) {
  if (!c) return fail(MOE_ERR_INVALID, "moe_cpu_forward: null experts");
  if (T < 0 || width <= 0) return fail(MOE_ERR_INVALID, "moe_cpu_forward: need T >= 0 and width > 0");
  if (T == 0) return MOE_OK;
  if (!x || !ids || !weights || !y) return fail(MOE_ERR_INVALID, "moe_cpu_forward: null pointer");
  return cpu_forward_impl(c, x, ids, weights, T, width, select, y);
}

moe_status moe_executor_create(moe_cpu_experts* cpu, moe_ring* result_ring, moe_executor** out) {
  if (!out) return fail(MOE_ERR_INVALID, "moe_executor_create: null out");
  *out = nullptr;
  if (!cpu || !result_ring) return fail(MOE_ERR_INVALID, "moe_executor_create: null experts or ring");
  moe_executor* ex = new moe_executor();
  ex->cpu = cpu;
  ex->ring = result_ring;
  ex->worker = std::thread(executor_loop, ex);
  *out = ex;
  return MOE_OK;
}

moe_status moe_executor_submit(moe_executor* ex, const uint16_t* x, const uint32_t* ids, const float* weights, int T,
                               int width, const uint8_t* select, uint32_t* target) {
  if (!ex) return fail(MOE_ERR_INVALID, "moe_executor_submit: null executor");
  if (T <= 0 || width <= 0 || !x || !ids || !weights || !target)
    return fail(MOE_ERR_INVALID, "moe_executor_submit: bad arguments");
  if ((size_t)T * ex->cpu->H * sizeof(float) > moe_ring_slot_bytes(ex->ring))
    return fail(MOE_ERR_INVALID, "moe_executor_submit: T * hidden f32 exceeds the result ring's slot");
  std::lock_guard<std::mutex> lk(ex->m);
  if (ex->error_status != MOE_OK) {  // a failed earlier job surfaces here (executor.rs:124)
    const moe_status st = ex->error_status;
    const std::string msg = ex->error;
    ex->error_status = MOE_OK;
    ex->error.clear();
    return fail(st, msg);
  }
  moe_executor::Job job;
  job.T = T;
  job.width = width;
  job.x.assign(x, x + (size_t)T * ex->cpu->H);
  job.ids.assign(ids, ids + (size_t)T * width);
  job.w.assign(weights, weights + (size_t)T * width);
  if (select) job.select.assign(select, select + (size_t)T * width);
  ex->jobs.push_back(std::move(job));
  *target = ++ex->next_target;  // jobs publish in FIFO order: the n-th job is the ring's n-th slot
  ex->cv.notify_one();
  return MOE_OK;
}

moe_status moe_executor_drain(moe_executor* ex) {
  if (!ex) return fail(MOE_ERR_INVALID, "moe_executor_drain: null executor");
  std::unique_lock<std::mutex> lk(ex->m);
  ex->idle_cv.wait(lk, [&] { return ex->jobs.empty() && !ex->busy; });
  if (ex->error_status != MOE_OK) {
    const moe_status st = ex->error_status;
    const std::string msg = ex->error;
    ex->error_status = MOE_OK;
    ex->error.clear();
    return fail(st, msg);
  }
  return MOE_OK;
}

void moe_executor_destroy(moe_executor* ex) {
  if (!ex) return;
  {
    std::lock_guard<std::mutex> lk(ex->m);
    ex->stop = true;
  }
  ex->cv.notify_all();
  if (ex->worker.joinable()) ex->worker.join();
  delete ex;
}

}  // extern "C"
