// paged.cu — decode and prefill through an expert cache: the reference's CachedLayer call path in C++.
//
// One moe_paged object per cached MoE layer (a moe_layer created with cache_slots > 0). It replaces
// the reference's per-layer decode split (src/moe/decode.rs:224-378 with stages/route.rs:19-158,
// stages/dma_miss.rs:80-160, stages/cpu_miss.rs:21-54), its lookahead prefetch
// (stages/preload.rs:18-195, cached_layer.rs:1236-1300) and its ring-batched prefill
// (rings.rs:68-156, prefill_stream.rs:1066, :1362-1694):
//
//   decode call (moe_paged_forward), on the caller's stream, token thread:
//     1. the router's top-k and the activation go to the host through mapped doorbell rings (no
//        stream synchronisation; the host waits only for the router);
//     2. under the layer's cache lock: the route split (published cache slots are hits), then
//        streamed_misses picks the missed experts worth copying now; they go to the layer's staging
//        slots (past the cache slots, so the cache is never evicted for a one-shot miss) on the copy
//        stream, after the slots' previous readers (last_read), with their own completion event;
//     3. the remaining misses go to the CPU executor (the activation's host copy and a pair mask);
//     4. the resident pairs run first (the copies of earlier lookahead passes are waited for, the
//        staging copies are not), then the stream waits for the staging event and the staged pairs
//        run; both passes leave per-pair outputs and one combine sums them, so the GPU part is
//        bit-identical to an all-resident layer wherever each expert came from; the CPU rows come
//        back through the result ring and are added in f32;
//     5. the activation is handed to the lookahead thread for the next layer.
//   lookahead (one thread for the process): the next layer's router on the CPU (f32 logits of the
//     activation), each row's top-k (top_k_ids), their union by votes (union_by_votes); the
//     predicted experts that are not resident are admitted into free slots or replace the least
//     recently used slot outside the prediction (at most lookahead_swaps per row), copied on that
//     layer's copy stream after its last readers; the pass ends with the layer's copies_done event,
//     which every later forward of the layer waits on, and only then are the slots published.
//   prefill (moe_paged_prefill): per chunk, the resident experts run first while the copy stream
//     fills half of the staging slots with the first wave of missing experts; waves are balanced by
//     routed-pair count and alternate between the two halves, so each wave's upload overlaps the
//     previous wave's compute; the waves leave per-pair outputs and one combine per chunk sums them
//     (the bits of an all-resident layer).
//
// Staging slots are per layer here, not one ring shared by every layer as in the reference
// (staging.rs:23-33, there to fit 12 GB cards): 16 slots per layer of config 4 are 3.9 GB of a
// B200's 180 GB, and per-layer slots keep the kernels' one bank per projection.
#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <string>
#include <thread>

#include "layer_internal.cuh"

namespace moe {

static float bf16_bits_to_f32(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

}  // namespace moe

using namespace moe;

struct moe_paged {
  moe_layer* L = nullptr;
  moe_cpu_experts* cpu = nullptr;
  moe_executor* ex = nullptr;
  moe_ring *topk_ring = nullptr, *act_ring = nullptr, *result_ring = nullptr;
  moe_paged* next = nullptr;
  moe_paged_opts o{};
  int E = 0, H = 0, k = 0;
  std::vector<float> router;  // [E, H] f32: this layer's router on the host, for its predictions
  uint32_t* ids_sel = nullptr;  // device [3][max_tokens * 2k]: resident / staged / union pair masks
  float* rows = nullptr;          // device [max_tokens * H] f32: the CPU rows
  cudaEvent_t staging_done = nullptr;
  cudaEvent_t half_read[2] = {nullptr, nullptr};  // prefill: last reader of each staging half
  cudaEvent_t up_done[2] = {nullptr, nullptr};    // prefill: the latest copies into each half
  moe_paged_stats st{};
  std::mutex stats_mu;
};

// ---- the lookahead thread ----------------------------------------------------------------------

namespace {

constexpr size_t LOOKAHEAD_DEPTH = 64;  // queued jobs; more are dropped (reference preload.rs:127)

struct LookJob {
  moe_paged* target;
  int rows;
  std::vector<uint16_t> x;  // [rows, H] bf16
};

struct Lookahead {
  std::mutex m;
  std::condition_variable cv, idle_cv;
  std::deque<LookJob> jobs;
  moe_paged* running = nullptr;
  std::vector<moe_paged*> live;  // every paged runtime not yet destroyed
  std::thread worker;
  bool started = false;

  void start() {
    if (!started) {
      started = true;
      worker = std::thread([this] { loop(); });
      worker.detach();  // lives until the process exits
    }
  }
  void loop();
  void push(LookJob&& j, moe_paged* p) {
    std::lock_guard<std::mutex> l(m);
    if (std::find(live.begin(), live.end(), p) == live.end() || !p->L) return;  // target gone or detached
    start();
    if (jobs.size() >= LOOKAHEAD_DEPTH) {
      std::lock_guard<std::mutex> s(p->stats_mu);
      ++p->st.lookahead_dropped;
      return;
    }
    jobs.push_back(std::move(j));
    cv.notify_one();
  }
  // Drops the queued jobs of `p` and waits until none of them runs; with `remove`, p also leaves
  // the live set and every other runtime's link to it is cut.
  void forget(moe_paged* p, bool remove, bool detach = false) {
    std::unique_lock<std::mutex> l(m);
    for (auto it = jobs.begin(); it != jobs.end();) it = it->target == p ? jobs.erase(it) : it + 1;
    idle_cv.wait(l, [&] { return running != p; });
    if (detach) p->L = nullptr;  // under the lock: push() refuses p from now on
    if (remove) {
      live.erase(std::remove(live.begin(), live.end(), p), live.end());
      for (moe_paged* q : live)
        if (q->next == p) q->next = nullptr;
    }
  }
  void add(moe_paged* p) {
    std::lock_guard<std::mutex> l(m);
    live.push_back(p);
  }
  // Waits until the queue is empty and no job runs.
  void drain() {
    std::unique_lock<std::mutex> l(m);
    idle_cv.wait(l, [&] { return jobs.empty() && running == nullptr; });
  }
};

Lookahead& lookahead() {
  static Lookahead* la = new Lookahead();  // never destroyed: the detached worker may still use it
  return *la;
}

// The reference's predict (cached_layer.rs:1236-1249): f32 logits of each row against this layer's
// router, each row's top-k, their union by votes.
std::vector<int> predict(const moe_paged* p, const uint16_t* x, int rows) {
  std::vector<float> xf((size_t)p->H), logits((size_t)p->E);
  std::vector<std::vector<int32_t>> ranks((size_t)rows, std::vector<int32_t>((size_t)p->k));
  for (int r = 0; r < rows; ++r) {
    for (int h = 0; h < p->H; ++h) xf[(size_t)h] = bf16_bits_to_f32(x[(size_t)r * p->H + h]);
    for (int e = 0; e < p->E; ++e) {
      const float* w = p->router.data() + (size_t)e * p->H;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int h = 0;
      for (; h + 8 <= p->H; h += 8)
        for (int l = 0; l < 8; ++l) acc[l] += xf[(size_t)(h + l)] * w[h + l];
      float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
      for (; h < p->H; ++h) s += xf[(size_t)h] * w[h];
      logits[(size_t)e] = s;
    }
    moe_policy_top_k_ids(logits.data(), p->E, p->k, ranks[(size_t)r].data());
  }
  std::vector<const int32_t*> ptrs((size_t)rows);
  std::vector<int32_t> lens((size_t)rows, p->k), out((size_t)rows * p->k);
  for (int r = 0; r < rows; ++r) ptrs[(size_t)r] = ranks[(size_t)r].data();
  const int n = moe_policy_union_by_votes(ptrs.data(), lens.data(), rows, out.data());
  return std::vector<int>(out.begin(), out.begin() + (n > 0 ? n : 0));
}

// The reference's prefetch_predicted (cached_layer.rs:1251-1300): admit / replace the predicted
// experts, copies on the layer's copy stream, then the claim (copies_done + publish).
void prefetch(moe_paged* p, const std::vector<int>& predicted, int rows) {
  moe_layer* L = p->L;
  std::lock_guard<std::recursive_mutex> lock(L->cache_mu);
  DeviceGuard guard(L->dev);
  std::vector<int32_t> protect(predicted.begin(), predicted.end());
  const int max_swaps = p->o.lookahead_swaps * rows;
  int swaps = 0, loads = 0;
  bool waited = false;
  SlotEdits ed{};
  std::vector<int> loading;
  moe_status status = MOE_OK;
  for (int e : predicted) {
    if (e < 0 || e >= p->E || L->slot_of_host[(size_t)e] >= 0) continue;  // resident already
    int slot = -1;
    for (int s = 0; s < L->slots; ++s)
      if (L->slot_state[(size_t)s] == SLOT_EMPTY) {
        slot = s;
        break;
      }
    if (slot < 0) {
      if (swaps >= max_swaps) continue;
      std::vector<int32_t> published((size_t)L->slots);
      for (int s = 0; s < L->slots; ++s) published[(size_t)s] = L->slot_state[(size_t)s] == SLOT_PUBLISHED;
      int32_t victim = -1;
      slot = moe_policy_lru_victim(L->slot_expert.data(), published.data(), L->last_use.data(), L->slots,
                                   protect.data(), (int)protect.size(), &victim);
      if (slot < 0) break;
      L->slot_of_host[(size_t)victim] = -1;
      if (ed.n == 64) {
        launch_slot_edits(L->slot_of, ed, L->copy_stream);
        ed.n = 0;
      }
      ed.expert[ed.n] = victim;
      ed.slot[ed.n++] = -1;
      ++swaps;
    }
    if (!waited) {  // every reader of the slots so far has finished before one is overwritten
      if (cudaStreamWaitEvent(L->copy_stream, L->last_read, 0) != cudaSuccess) {
        status = MOE_ERR_CUDA;
        break;
      }
      waited = true;
    }
    if ((status = cache_copy_expert(L, e, slot)) != MOE_OK) break;
    L->slot_expert[(size_t)slot] = e;
    L->slot_state[(size_t)slot] = SLOT_LOADING;
    L->last_use[(size_t)slot] = L->tick;
    L->slot_of_host[(size_t)e] = slot;
    loading.push_back(slot);
    if (ed.n == 64) {
      launch_slot_edits(L->slot_of, ed, L->copy_stream);
      ed.n = 0;
    }
    ed.expert[ed.n] = e;
    ed.slot[ed.n++] = slot;
    ++loads;
  }
  if (ed.n) launch_slot_edits(L->slot_of, ed, L->copy_stream);
  if (loads || ed.n) {
    // the claim: the completion event first, then the slots become visible to the split
    if (cudaEventRecord(L->copies_done, L->copy_stream) == cudaSuccess) L->copies_pending = true;
    else status = MOE_ERR_CUDA;
  }
  for (int s : loading) L->slot_state[(size_t)s] = SLOT_PUBLISHED;
  std::lock_guard<std::mutex> sl(p->stats_mu);
  ++p->st.lookahead_passes;
  p->st.lookahead_loads += loads;
  p->st.lookahead_swaps += swaps;
  p->st.predicted += (int64_t)predicted.size();
  if (status != MOE_OK) ++p->st.lookahead_errors;
}

void Lookahead::loop() {
  for (;;) {
    LookJob job;
    {
      std::unique_lock<std::mutex> l(m);
      cv.wait(l, [&] { return !jobs.empty(); });
      job = std::move(jobs.front());
      jobs.pop_front();
      if (!job.target->L) continue;  // its layer was destroyed
      running = job.target;
    }
    const std::vector<int> predicted = predict(job.target, job.x.data(), job.rows);
    prefetch(job.target, predicted, job.rows);
    {
      std::lock_guard<std::mutex> l(m);
      running = nullptr;
    }
    idle_cv.notify_all();
  }
}

}  // namespace

// ---- create / destroy ------------------------------------------------------------------------------

extern "C" {

void moe_paged_default_opts(moe_paged_opts* o) {
  if (!o) return;
  std::memset(o, 0, sizeof(*o));
  o->staging_slots = 16;
  o->pcie_frac = 1.0f;
  o->stream_cap = 16;
  o->lookahead = 1;
  o->lookahead_swaps = 1;
  o->max_tokens = 256;
  o->host_timeout_us = 5000000;
}

void moe_paged_destroy(moe_paged* p) {
  if (!p) return;
  lookahead().forget(p, true);
  if (p->L) {
    std::lock_guard<std::recursive_mutex> lock(p->L->cache_mu);
    auto& v = p->L->paged;
    v.erase(std::remove(v.begin(), v.end(), p), v.end());
  }
  if (p->ex) moe_executor_destroy(p->ex);
  moe_ring_destroy(p->topk_ring);
  moe_ring_destroy(p->act_ring);
  moe_ring_destroy(p->result_ring);
  {
    DeviceGuard guard(p->L ? p->L->dev : 0);
    cudaFree(p->ids_sel);
    cudaFree(p->rows);
    if (p->staging_done) cudaEventDestroy(p->staging_done);
    for (auto& e : p->half_read)
      if (e) cudaEventDestroy(e);
    for (auto& e : p->up_done)
      if (e) cudaEventDestroy(e);
  }
  delete p;
}

moe_status moe_paged_create(moe_layer* L, moe_cpu_experts* cpu, const moe_paged_opts* opts, moe_paged** out) {
  if (!out) return fail(MOE_ERR_INVALID, "moe_paged_create: null out");
  *out = nullptr;
  if (!L) return fail(MOE_ERR_INVALID, "moe_paged_create: null layer");
  if (!L->slots) return fail(MOE_ERR_INVALID, "moe_paged_create: the layer has no expert cache (cache_slots = 0)");
  moe_paged_opts o;
  if (opts) o = *opts;
  else moe_paged_default_opts(&o);
  const int E = L->d.num_experts;
  if (o.max_tokens <= 0 || o.max_tokens > L->cap_tokens)
    return fail(MOE_ERR_INVALID, "moe_paged_create: max_tokens must be in 1..the layer's max_tokens");
  if (o.staging_slots < 0 || o.stream_cap < 0 || o.lookahead_swaps < 0 || o.pcie_frac < 0.0f)
    return fail(MOE_ERR_INVALID, "moe_paged_create: negative option");
  if (o.staging_slots > E - L->slots) o.staging_slots = E - L->slots;
  if (o.stream_cap > o.staging_slots) o.stream_cap = o.staging_slots;
  DeviceGuard guard(L->dev);
  moe_paged* p = new moe_paged();
  p->L = L;
  p->cpu = cpu;
  p->o = o;
  p->E = E;
  p->H = L->d.hidden;
  p->k = L->d.top_k;
  auto bad = [&](moe_status s) {
    moe_paged_destroy(p);
    return s;
  };
  moe_status s;
  if (o.staging_slots > 0 && (s = cache_reserve_staging(L, o.staging_slots)) != MOE_OK) return bad(s);
  const int T = o.max_tokens;
  // the widest row a caller may pass is 2 * top_k (weight-0 padding); ids and weights share a slot
  const size_t topk_bytes = (size_t)T * 2 * p->k * 8;
  if ((s = moe_ring_create(L->dev, 4, topk_bytes, &p->topk_ring)) != MOE_OK) return bad(s);
  if ((s = moe_ring_create(L->dev, 4, (size_t)T * p->H * 2, &p->act_ring)) != MOE_OK) return bad(s);
  if (cpu) {
    if ((s = moe_ring_create(L->dev, 4, (size_t)T * p->H * 4, &p->result_ring)) != MOE_OK) return bad(s);
    if ((s = moe_executor_create(cpu, p->result_ring, &p->ex)) != MOE_OK) return bad(s);
  }
  // pair masks sized for the prefill chunks too (up to the layer's scratch)
  const size_t mask = (size_t)L->cap_pairs > (size_t)T * 2 * p->k ? (size_t)L->cap_pairs : (size_t)T * 2 * p->k;
  cudaError_t e = cudaMalloc(&p->ids_sel, sizeof(uint32_t) * 3 * mask);
  if (e == cudaSuccess) e = cudaMalloc(&p->rows, sizeof(float) * (size_t)T * p->H);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->staging_done, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->half_read[0], cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->half_read[1], cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->up_done[0], cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->up_done[1], cudaEventDisableTiming);
  if (e != cudaSuccess) return bad(cuda_fail(e, "moe_paged_create"));
  if (L->router_w) {  // the router on the host in f32 (the reference keeps it there, provider.rs:618-629)
    std::vector<uint16_t> bf((size_t)E * p->H);
    e = cudaMemcpy(bf.data(), L->router_w, bf.size() * 2, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return bad(cuda_fail(e, "moe_paged_create: router copy"));
    p->router.resize(bf.size());
    for (size_t i = 0; i < bf.size(); ++i) p->router[i] = bf16_bits_to_f32(bf[i]);
  }
  {
    std::lock_guard<std::recursive_mutex> lock(L->cache_mu);
    L->paged.push_back(p);
  }
  lookahead().add(p);
  *out = p;
  return MOE_OK;
}

}  // extern "C"

void moe::paged_detach_all(moe_layer* L) {
  std::vector<moe_paged*> ps;
  {
    std::lock_guard<std::recursive_mutex> lock(L->cache_mu);
    ps.swap(L->paged);
  }
  for (moe_paged* p : ps) lookahead().forget(p, false, true);  // no job of p runs on L; later calls fail
}

extern "C" {

moe_status moe_paged_set_next(moe_paged* p, moe_paged* next) {
  if (!p || !p->L) return fail(MOE_ERR_INVALID, "moe_paged_set_next: null paged layer or its layer was destroyed");
  if (next && next->router.empty())
    return fail(MOE_ERR_INVALID, "moe_paged_set_next: the next layer has no router to predict with");
  if (next && next->H != p->H) return fail(MOE_ERR_INVALID, "moe_paged_set_next: hidden sizes differ");
  p->next = next;
  return MOE_OK;
}

// ---- decode ---------------------------------------------------------------------------------------

moe_status moe_paged_forward(moe_paged* p, const void* x, int T, const uint32_t* ids, const float* weights, int width,
                             void* y, void* stream) {
  if (!p || !p->L) return fail(MOE_ERR_INVALID, "moe_paged_forward: null paged layer or its layer was destroyed");
  if (T < 0 || width <= 0 || width > 2 * p->k) return fail(MOE_ERR_INVALID, "moe_paged_forward: bad T or width");
  if (T == 0) return MOE_OK;
  if (T > p->o.max_tokens) return fail(MOE_ERR_INVALID, "moe_paged_forward: T exceeds the paged max_tokens");
  if (!x || !ids || !weights || !y) return fail(MOE_ERR_INVALID, "moe_paged_forward: null pointer");
  moe_layer* L = p->L;
  DeviceGuard guard(L->dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n = T * width;
  // 1. the top-k and the activation reach the host behind the router, not behind the stream
  uint32_t seq = 0, aseq = 0;
  MOE_TRY(moe_ring_publish_from_device(p->topk_ring, ids, (size_t)n * 4, weights, (size_t)n * 4, stream, &seq));
  const bool need_x = p->ex != nullptr || (p->next != nullptr && p->o.lookahead);
  if (need_x) MOE_TRY(moe_ring_publish_from_device(p->act_ring, x, (size_t)T * p->H * 2, nullptr, 0, stream, &aseq));
  std::vector<uint32_t> buf((size_t)n * 2);
  MOE_TRY(moe_ring_host_take(p->topk_ring, seq, buf.data(), (size_t)n * 8, p->o.host_timeout_us));
  const uint32_t* ids_h = buf.data();
  const float* w_h = reinterpret_cast<const float*>(buf.data() + n);
  std::vector<uint16_t> x_h;
  if (need_x) {
    x_h.resize((size_t)T * p->H);
    MOE_TRY(moe_ring_host_take(p->act_ring, aseq, x_h.data(), x_h.size() * 2, p->o.host_timeout_us));
  }
  int64_t pairs = 0, hits = 0, staged_pairs = 0, cpu_pairs = 0;
  int staged_experts = 0;
  {
    std::lock_guard<std::recursive_mutex> lock(L->cache_mu);
    // 2. the route split (stages/route.rs:19-158) and the streamed misses (cached_layer.rs:385-398)
    std::vector<uint8_t> hit((size_t)n);
    const moe_status split = moe_cache_split(L, ids_h, n, hit.data());
    if (split != MOE_OK) {  // name the ring state with the bad id, so a malformed hand-off is visible
      uint32_t rseq = 0, rcons = 0;
      moe_ring_counters(p->topk_ring, &rseq, &rcons);
      std::string msg;
      for (int i = 0; i < n && i < 8; ++i) msg += " " + std::to_string(ids_h[i]);
      return fail(split, "moe_paged_forward: " + last_error_message() + " (top-k slot " + std::to_string(seq) +
                             ", ring seq " + std::to_string(rseq) + ", consumed " + std::to_string(rcons) +
                             ", T " + std::to_string(T) + ", width " + std::to_string(width) + "; first ids" + msg +
                             ")");
    }
    std::vector<uint32_t> miss_ids;
    std::vector<float> miss_w;
    std::vector<int32_t> row_lens((size_t)T, 0);
    for (int t = 0; t < T; ++t)
      for (int j = 0; j < width; ++j) {
        const int i = t * width + j;
        if (hit[(size_t)i] == 0) {
          miss_ids.push_back(ids_h[i]);
          miss_w.push_back(w_h[i]);
          ++row_lens[(size_t)t];
        }
        pairs += hit[(size_t)i] != 2;
        hits += hit[(size_t)i] == 1;
      }
    std::vector<uint32_t> streamed((size_t)p->o.stream_cap + 1);
    int n_stream = 0;
    if (!miss_ids.empty() && p->o.stream_cap > 0 && p->o.pcie_frac > 0.0f)
      n_stream = moe_policy_streamed_misses(miss_ids.data(), miss_w.data(), row_lens.data(), T, p->o.pcie_frac,
                                            p->o.stream_cap, streamed.data());
    streamed.resize((size_t)(n_stream > 0 ? n_stream : 0));
    // staging copies (stages/dma_miss.rs:80-160): into staging slots, after the slots' last readers
    if (!streamed.empty()) {
      MOE_CUDA_TRY(cudaStreamWaitEvent(L->copy_stream, L->last_read, 0));
      SlotEdits ed{};
      for (size_t j = 0; j < streamed.size(); ++j) {
        MOE_TRY(cache_copy_expert(L, (int)streamed[j], L->slots + (int)j));
        ed.expert[ed.n] = (int)streamed[j];
        ed.slot[ed.n++] = L->slots + (int)j;
      }
      MOE_TRY(launch_slot_edits(L->slot_of, ed, L->copy_stream));
      MOE_CUDA_TRY(cudaEventRecord(p->staging_done, L->copy_stream));
      staged_experts = (int)streamed.size();
    }
    // 3. the rest of the misses on the CPU (stages/cpu_miss.rs:21-54)
    std::vector<uint8_t> cpu_sel((size_t)n, 0);
    bool any_cpu = false;
    for (int i = 0; i < n; ++i) {
      if (hit[(size_t)i] != 0) continue;
      bool is_staged = false;
      for (uint32_t s : streamed) is_staged |= s == ids_h[i];
      if (is_staged) {
        ++staged_pairs;
      } else {
        cpu_sel[(size_t)i] = 1;
        any_cpu = true;
        ++cpu_pairs;
      }
    }
    uint32_t target = 0;
    if (any_cpu) {
      if (!p->ex)
        return fail(MOE_ERR_INVALID, "moe_paged_forward: missed experts with no CPU path and no staging slot left");
      MOE_TRY(moe_executor_submit(p->ex, x_h.data(), ids_h, w_h, T, width, cpu_sel.data(), &target));
    }
    // 4. resident pairs first, then the staged ones behind their copies (decode.rs:224-330)
    std::vector<uint32_t> resident;
    for (int s = 0; s < L->slots; ++s)
      if (L->slot_state[(size_t)s] == SLOT_PUBLISHED && L->slot_expert[(size_t)s] >= 0)
        resident.push_back((uint32_t)L->slot_expert[(size_t)s]);
    // Both passes leave their pairs' outputs in the layer's per-pair rows; one combine over the union
    // then gives the bits of a single forward over all of them (layer_experts), so where an expert
    // came from (cache, lookahead, staging) never changes the output.
    const size_t stride = (size_t)p->o.max_tokens * 2 * p->k;
    uint32_t* ids_r = p->ids_sel;
    uint32_t* ids_s = p->ids_sel + stride;
    uint32_t* ids_u = p->ids_sel + 2 * stride;
    MOE_TRY(moe_select_ids(ids, n, p->E, resident.data(), (int)resident.size(), ids_r, stream));
    MOE_TRY(layer_experts(L, x, T, ids_r, weights, width, st));
    std::vector<uint32_t> both(resident);
    if (!streamed.empty()) {
      MOE_CUDA_TRY(cudaStreamWaitEvent(st, p->staging_done, 0));
      MOE_TRY(moe_select_ids(ids, n, p->E, streamed.data(), (int)streamed.size(), ids_s, stream));
      MOE_TRY(layer_experts(L, x, T, ids_s, weights, width, st));
      both.insert(both.end(), streamed.begin(), streamed.end());
    }
    MOE_TRY(moe_select_ids(ids, n, p->E, both.data(), (int)both.size(), ids_u, stream));
    MOE_TRY(layer_combine(L, T, ids_u, width, y, st));
    if (target) {
      MOE_TRY(moe_ring_device_take(p->result_ring, target, p->rows, (size_t)T * p->H * 4, stream));
      MOE_TRY(moe_add_f32_into_bf16(y, p->rows, (int64_t)T * p->H, stream));
    }
    MOE_CUDA_TRY(cudaEventRecord(L->last_read, st));  // every slot this call read
    if (!streamed.empty()) {  // the staged experts leave the slot map: plain forwards must not see them
      SlotEdits ed{};
      for (uint32_t e : streamed) {
        ed.expert[ed.n] = (int)e;
        ed.slot[ed.n++] = -1;
      }
      MOE_TRY(launch_slot_edits(L->slot_of, ed, st));
    }
  }
  // 5. the next layer's prediction from this activation (stages/preload.rs:18-112)
  if (p->next && p->o.lookahead) lookahead().push(LookJob{p->next, T, std::move(x_h)}, p->next);
  std::lock_guard<std::mutex> sl(p->stats_mu);
  ++p->st.calls;
  p->st.pairs += pairs;
  p->st.hits += hits;
  p->st.staged_experts += staged_experts;
  p->st.staged_pairs += staged_pairs;
  p->st.cpu_pairs += cpu_pairs;
  return MOE_OK;
}

// ---- prefill --------------------------------------------------------------------------------------

moe_status moe_paged_prefill(moe_paged* p, const void* x, int T, const uint32_t* ids, const float* weights, int width,
                             void* y, void* stream) {
  if (!p || !p->L) return fail(MOE_ERR_INVALID, "moe_paged_prefill: null paged layer or its layer was destroyed");
  if (T < 0 || width <= 0) return fail(MOE_ERR_INVALID, "moe_paged_prefill: bad T or width");
  if (T == 0) return MOE_OK;
  if (!x || !ids || !weights || !y) return fail(MOE_ERR_INVALID, "moe_paged_prefill: null pointer");
  moe_layer* L = p->L;
  const int half = L->staging / 2;
  if (half < 1) return fail(MOE_ERR_INVALID, "moe_paged_prefill: needs at least two staging slots");
  DeviceGuard guard(L->dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int chunk = L->cap_pairs / width < L->cap_tokens ? L->cap_pairs / width : L->cap_tokens;
  if (chunk <= 0) return fail(MOE_ERR_INVALID, "moe_paged_prefill: width exceeds the layer's scratch");
  // the routing of the whole prompt on the host (prefill is not on the token path)
  std::vector<uint32_t> ids_h((size_t)T * width);
  MOE_CUDA_TRY(cudaMemcpyAsync(ids_h.data(), ids, ids_h.size() * 4, cudaMemcpyDeviceToHost, st));
  MOE_CUDA_TRY(cudaStreamSynchronize(st));
  std::lock_guard<std::recursive_mutex> lock(L->cache_mu);  // the lookahead stays out of this layer
  const int H = p->H;
  int64_t waves_total = 0, uploads = 0;
  bool half_used[2] = {false, false};
  for (int t0 = 0; t0 < T; t0 += chunk) {
    const int nt = T - t0 < chunk ? T - t0 : chunk;
    const int nn = nt * width;
    const uint32_t* cid = ids_h.data() + (size_t)t0 * width;
    std::vector<int64_t> count((size_t)p->E, 0);
    for (int i = 0; i < nn; ++i)
      if (cid[i] < (uint32_t)p->E) ++count[cid[i]];
      else if (cid[i] != MOE_ID_NONE) return fail(MOE_ERR_BAD_IDS, "moe_paged_prefill: routed expert id >= num_experts");
    // wave 0: the resident experts, no upload
    std::vector<uint32_t> resident, missing;
    for (int e = 0; e < p->E; ++e) {
      if (!count[(size_t)e]) continue;
      const int s = L->slot_of_host[(size_t)e];
      if (s >= 0 && L->slot_state[(size_t)s] == SLOT_PUBLISHED) resident.push_back((uint32_t)e);
      else missing.push_back((uint32_t)e);
    }
    // the missing experts in waves of at most `half`, balanced by routed pairs (rings.rs:68-156):
    // largest first, each to the wave with the fewest pairs that still has room
    const int n_waves = (int)((missing.size() + half - 1) / half);
    std::sort(missing.begin(), missing.end(), [&](uint32_t a, uint32_t b) {
      return count[a] != count[b] ? count[a] > count[b] : a < b;
    });
    std::vector<std::vector<uint32_t>> waves((size_t)n_waves);
    std::vector<int64_t> load((size_t)n_waves, 0);
    for (uint32_t e : missing) {
      int best = -1;
      for (int w = 0; w < n_waves; ++w)
        if ((int)waves[(size_t)w].size() < half && (best < 0 || load[(size_t)w] < load[(size_t)best])) best = w;
      waves[(size_t)best].push_back(e);
      load[(size_t)best] += count[e];
    }
    const void* xc = static_cast<const __nv_bfloat16*>(x) + (int64_t)t0 * H;
    const uint32_t* idc = ids + (int64_t)t0 * width;
    const float* wc = weights + (int64_t)t0 * width;
    uint32_t* sel = p->ids_sel;
    // every wave leaves its pairs' outputs in the layer's per-pair rows; one combine over the chunk
    // then gives the bits of a resident layer's forward (layer_experts)
    auto run = [&](const std::vector<uint32_t>& set) -> moe_status {
      MOE_TRY(moe_select_ids(idc, nn, p->E, set.data(), (int)set.size(), sel, stream));
      MOE_TRY(layer_experts(L, xc, nt, sel, wc, width, st));
      ++waves_total;
      return MOE_OK;
    };
    // wave w's copies into staging half w % 2, after that half's last reader; up_done[half] marks them
    auto upload = [&](int w) -> moe_status {
      const int h = w % 2;
      MOE_CUDA_TRY(cudaStreamWaitEvent(L->copy_stream, half_used[h] ? p->half_read[h] : L->last_read, 0));
      SlotEdits ed{};
      for (size_t j = 0; j < waves[(size_t)w].size(); ++j) {
        const int slot = L->slots + h * half + (int)j;
        MOE_TRY(cache_copy_expert(L, (int)waves[(size_t)w][j], slot));
        ed.expert[ed.n] = (int)waves[(size_t)w][j];
        ed.slot[ed.n++] = slot;
        ++uploads;
      }
      MOE_TRY(launch_slot_edits(L->slot_of, ed, L->copy_stream));
      MOE_CUDA_TRY(cudaEventRecord(p->up_done[h], L->copy_stream));
      return MOE_OK;
    };
    // The copy stream runs one wave ahead of the compute stream (prefill_stream.rs:1066 load,
    // :1362-1694): wave 0's copies go out before the resident experts run, and wave w + 1's before
    // wave w runs, so every upload overlaps the compute before it.
    if (n_waves > 0) MOE_TRY(upload(0));
    if (!resident.empty()) MOE_TRY(run(resident));
    for (int w = 0; w < n_waves; ++w) {
      if (w + 1 < n_waves) MOE_TRY(upload(w + 1));
      MOE_CUDA_TRY(cudaStreamWaitEvent(st, p->up_done[w % 2], 0));
      MOE_TRY(run(waves[(size_t)w]));
      MOE_CUDA_TRY(cudaEventRecord(p->half_read[w % 2], st));
      half_used[w % 2] = true;
    }
    // the combine reads only the per-pair rows; a staged expert's (stale) map entry still marks its
    // pairs live, so the chunk's own ids serve as the union
    MOE_TRY(layer_combine(L, nt, idc, width, static_cast<__nv_bfloat16*>(y) + (int64_t)t0 * H, st));
    SlotEdits ed{};
    for (uint32_t e : missing) {  // the staged experts leave the slot map
      if (ed.n == 64) {
        MOE_TRY(launch_slot_edits(L->slot_of, ed, st));
        ed.n = 0;
      }
      ed.expert[ed.n] = (int)e;
      ed.slot[ed.n++] = -1;
    }
    MOE_TRY(launch_slot_edits(L->slot_of, ed, st));
  }
  MOE_CUDA_TRY(cudaEventRecord(L->last_read, st));
  std::lock_guard<std::mutex> sl(p->stats_mu);
  ++p->st.prefill_calls;
  p->st.prefill_waves += waves_total;
  p->st.prefill_uploads += uploads;
  return MOE_OK;
}

// ---- stats / fill / check -------------------------------------------------------------------------

moe_status moe_paged_get_stats(moe_paged* p, moe_paged_stats* out) {
  if (!p || !out) return fail(MOE_ERR_INVALID, "moe_paged_get_stats: null argument");
  std::lock_guard<std::mutex> sl(p->stats_mu);
  *out = p->st;
  return MOE_OK;
}

moe_status moe_paged_fill(moe_paged* p, void* stream) {
  if (!p || !p->L) return fail(MOE_ERR_INVALID, "moe_paged_fill: null paged layer or its layer was destroyed");
  moe_layer* L = p->L;
  std::lock_guard<std::recursive_mutex> lock(L->cache_mu);
  for (;;) {  // the reference's spawn_fill loop (cached_layer.rs:1303-1337), synchronous here
    const int c = moe_policy_fill_candidate(L->slot_expert.data(), L->slots, L->hit_counts.data(), p->E);
    if (c < 0) return MOE_OK;
    const uint32_t e = (uint32_t)c;
    int loaded = 0;
    MOE_TRY(moe_cache_upload(L, &e, 1, nullptr, 0, stream, &loaded));
    if (!loaded) return MOE_OK;
  }
}

moe_status moe_paged_drain_lookahead(void) {
  lookahead().drain();
  return MOE_OK;
}

moe_status moe_paged_check(moe_paged* p, void* stream) {
  if (!p || !p->L) return fail(MOE_ERR_INVALID, "moe_paged_check: null paged layer or its layer was destroyed");
  MOE_TRY(moe_layer_check(p->L, stream));
  MOE_TRY(moe_ring_check(p->topk_ring, stream));
  MOE_TRY(moe_ring_check(p->act_ring, stream));
  if (p->ex) {
    MOE_TRY(moe_ring_check(p->result_ring, stream));
    MOE_TRY(moe_executor_drain(p->ex));
  }
  std::lock_guard<std::mutex> sl(p->stats_mu);
  if (p->st.lookahead_errors) {
    p->st.lookahead_errors = 0;
    return fail(MOE_ERR_CUDA, "moe_paged: a lookahead pass failed to enqueue its copies");
  }
  return MOE_OK;
}

}  // extern "C"
