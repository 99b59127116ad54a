// layer.cu — the moe_layer object and the C ABI (include/moe_b200.h).
//
// moe_layer plays the role of the reference's per-MoE-block operator: GpuCacheMoeProvider::build
// (src/moe/provider.rs:316-615) creates it from the block's expert stacks, and its forward is
// RoutedExperts::forward (src/moe/cached_layer.rs:524-664 / src/moe/expert.rs:59-117). Here every
// expert is resident in HBM (180 GB holds every config of this path), so the per-call work is:
// plan (histogram + stable permute) -> gate/up+SwiGLU -> down*weight -> combine, all on the
// caller's stream with no host synchronisation, so a sequence of calls captures into one CUDA graph.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include <vector>

#include "layer_internal.cuh"
#include <cmath>
#include <sys/mman.h>

namespace moe {

// ---- errors ----------------------------------------------------------------------------------

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }
const std::string& last_error_message() { return g_last_error; }

moe_status fail(moe_status st, const std::string& msg) {
  g_last_error = msg;
  return st;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MOE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

moe_status cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return e == cudaErrorMemoryAllocation ? MOE_ERR_OOM : MOE_ERR_CUDA;
}

}  // namespace moe

using namespace moe;

static void free_scratch(moe_layer* L) {
  cudaFree(L->counts);
  cudaFree(L->offsets);
  cudaFree(L->perm);
  cudaFree(L->active);
  cudaFree(L->act_rec);
  L->act_rec = nullptr;
  cudaFree(L->n_active);
  cudaFree(L->err);
  cudaFree(L->plan_ws);
  cudaFree(L->h);
  cudaFree(L->ypair);
  cudaFree(L->xq);
  cudaFree(L->xq_scale);
  L->xq = nullptr;
  L->xq_scale = nullptr;
  cudaFree(L->route_ws);
  L->route_ws = nullptr;
  L->route_ws_bytes = 0;
  cudaFree(L->x16);
  cudaFree(L->xscale);
  cudaFree(L->h16);
  cudaFree(L->hscale);
  cudaFree(L->tile_list);
  cudaFree(L->n_tiles);
  L->x16 = L->h16 = nullptr;
  L->xscale = L->hscale = nullptr;
  L->tile_list = L->n_tiles = nullptr;
  L->counts = L->offsets = L->perm = L->active = L->n_active = L->err = nullptr;
  L->plan_ws = nullptr;
  L->h = L->ypair = nullptr;
  L->cap_pairs = 0;
  L->cap_tokens = 0;
  L->scratch_bytes = 0;
}

template <class T>
static moe_status dalloc(T** p, size_t bytes, int64_t* acct) {
  void* v = nullptr;
  cudaError_t e = cudaMalloc(&v, bytes ? bytes : 16);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  *p = static_cast<T*>(v);
  if (acct) *acct += (int64_t)(bytes ? bytes : 16);
  return MOE_OK;
}

static moe_status alloc_scratch(moe_layer* L, int max_tokens) {
  const int64_t cap64 = (int64_t)max_tokens * L->d.top_k;
  if (cap64 > (1 << 28)) return fail(MOE_ERR_INVALID, "max_tokens * top_k too large");
  const int cap = (int)cap64;
  if (cap <= L->cap_pairs && max_tokens <= L->cap_tokens && L->counts) return MOE_OK;
  free_scratch(L);
  const int E = L->d.num_experts, H = L->d.hidden, I = L->d.inter;
  int64_t acc = 0;
  MOE_TRY(dalloc(&L->counts, sizeof(int32_t) * E, &acc));
  MOE_TRY(dalloc(&L->offsets, sizeof(int32_t) * (E + 1), &acc));
  MOE_TRY(dalloc(&L->perm, sizeof(int32_t) * cap, &acc));
  MOE_TRY(dalloc(&L->active, sizeof(int32_t) * E, &acc));
  MOE_TRY(dalloc(&L->act_rec, sizeof(int4) * E, &acc));
  MOE_TRY(dalloc(&L->n_active, sizeof(int32_t), &acc));
  MOE_TRY(dalloc(&L->err, sizeof(int32_t), &acc));
  MOE_CUDA_TRY(cudaMemset(L->err, 0, sizeof(int32_t)));
  L->plan_ws_bytes = plan_workspace_bytes(cap, E);
  MOE_TRY(dalloc(&L->plan_ws, L->plan_ws_bytes, &acc));
  MOE_TRY(dalloc(&L->h, sizeof(float) * (size_t)cap * I, &acc));
  MOE_TRY(dalloc(&L->ypair, sizeof(float) * (size_t)cap * H, &acc));
  if (L->q8_tiles) {  // a call has at most cap rows (width >= 1)
    MOE_TRY(dalloc(&L->xq, (size_t)cap * H * 2, &acc));
    MOE_TRY(dalloc(&L->xq_scale, sizeof(float) * cap, &acc));
  }
  L->route_ws_bytes = route_workspace_bytes(max_tokens, E);
  MOE_TRY(dalloc(&L->route_ws, L->route_ws_bytes, &acc));
  MOE_CUDA_TRY(cudaMemset(L->route_ws, 0, L->route_ws_bytes));  // arrival counters start at zero
  if (L->tc) {
    MOE_TRY(dalloc(&L->x16, (size_t)cap * H * 2, &acc));
    MOE_TRY(dalloc(&L->xscale, sizeof(float) * cap, &acc));
    MOE_TRY(dalloc(&L->h16, (size_t)cap * I * 2, &acc));
    MOE_TRY(dalloc(&L->hscale, sizeof(float) * cap, &acc));
    MOE_TRY(dalloc(&L->tile_list, sizeof(int32_t) * ((size_t)cap / TC_BN_MIN + E + 1), &acc));
    // [0] the tile-list length, [1] / [2] the work-item counters of the gate/up and down GEMM launches
    MOE_TRY(dalloc(&L->n_tiles, 4 * sizeof(int32_t), &acc));
    MOE_TRY(make_row_tmap(L->tmap_x, L->x16, cap, H));
    MOE_TRY(make_row_tmap(L->tmap_h, L->h16, cap, I));
  }
  L->cap_pairs = cap;
  L->cap_tokens = max_tokens;
  L->scratch_bytes = acc;
  return MOE_OK;
}

__global__ void slot_edit_kernel(int32_t* __restrict__ slot_of, SlotEdits ed) {
  if ((int)threadIdx.x < ed.n) slot_of[ed.expert[threadIdx.x]] = ed.slot[threadIdx.x];
}

moe_status moe::launch_slot_edits(int32_t* slot_of, const SlotEdits& ed, cudaStream_t st) {
  if (ed.n <= 0) return MOE_OK;
  slot_edit_kernel<<<1, 64, 0, st>>>(slot_of, ed);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

// Pinned host memory for the expert store. The reference advises the kernel to back its pinned
// expert stacks with transparent huge pages before pinning them (host_memory.rs:30-55): the DMA
// engine then walks a 2 MiB page per 2 MiB of experts instead of 512 small ones, and pinning is
// faster. Here: an anonymous mapping rounded up to 2 MiB, madvise(MADV_HUGEPAGE) (advice only; a
// kernel without transparent huge pages ignores it), then cudaHostRegister. If the mapping or the
// registration fails, cudaHostAlloc as before. The block's length is recorded so that free_cache
// undoes whichever was done.
static moe_status host_pin_alloc(moe_layer* L, size_t bytes, void** out) {
  constexpr size_t kHugePage = 2u << 20;
  const size_t len = (bytes + kHugePage - 1) / kHugePage * kHugePage;
  void* p = mmap(nullptr, len, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (p != MAP_FAILED) {
#ifdef MADV_HUGEPAGE
    madvise(p, len, MADV_HUGEPAGE);
#endif
    if (cudaHostRegister(p, len, cudaHostRegisterPortable) == cudaSuccess) {
      L->hs_blocks.emplace_back(p, len);
      *out = p;
      return MOE_OK;
    }
    cudaGetLastError();  // clear the failed registration
    munmap(p, len);
  }
  MOE_CUDA_TRY(cudaHostAlloc(out, bytes, cudaHostAllocPortable));
  L->hs_blocks.emplace_back(*out, 0);
  return MOE_OK;
}

static void free_cache(moe_layer* L) {
  for (auto& b : L->hs_blocks) {
    if (b.second) {
      cudaHostUnregister(b.first);
      munmap(b.first, b.second);
    } else {
      cudaFreeHost(b.first);
    }
  }
  L->hs_blocks.clear();
  L->hs_gu_q = L->hs_gu_s = L->hs_dn_q = L->hs_dn_s = nullptr;
  L->hs_gu_scale = L->hs_dn_scale = nullptr;
  cudaFree(L->slot_of);
  L->slot_of = nullptr;
  if (L->copy_stream) cudaStreamDestroy(L->copy_stream);
  if (L->last_read) cudaEventDestroy(L->last_read);
  if (L->copies_done) cudaEventDestroy(L->copies_done);
  L->copy_stream = nullptr;
  L->last_read = L->copies_done = nullptr;
}

// Moves a projection's E-expert device buffer into pinned host memory and replaces it by a bank of
// `slots` experts. stride: bytes per expert.
static moe_status to_host_store(moe_layer* L, uint8_t** dev_buf, uint8_t** host_buf, int64_t stride, int E, int slots,
                                int64_t* acct) {
  if (!*dev_buf || stride == 0) return MOE_OK;
  void* h = nullptr;
  MOE_TRY(host_pin_alloc(L, (size_t)(stride * E), &h));
  *host_buf = static_cast<uint8_t*>(h);
  MOE_CUDA_TRY(cudaMemcpy(h, *dev_buf, (size_t)(stride * E), cudaMemcpyDeviceToHost));
  cudaFree(*dev_buf);
  *dev_buf = nullptr;
  *acct -= stride * E;
  return dalloc(dev_buf, (size_t)(stride * slots), acct);
}

static moe_status setup_cache(moe_layer* L, int64_t* acct) {
  const int E = L->d.num_experts, S = L->slots;
  MOE_TRY(to_host_store(L, &L->gu_q, &L->hs_gu_q, L->gu_q_stride, E, S, acct));
  MOE_TRY(to_host_store(L, &L->gu_s, &L->hs_gu_s, L->gu_s_stride, E, S, acct));
  MOE_TRY(to_host_store(L, &L->dn_q, &L->hs_dn_q, L->dn_q_stride, E, S, acct));
  MOE_TRY(to_host_store(L, &L->dn_s, &L->hs_dn_s, L->dn_s_stride, E, S, acct));
  if (L->gu_scale) {
    uint8_t* g = reinterpret_cast<uint8_t*>(L->gu_scale);
    uint8_t* hg = nullptr;
    MOE_TRY(to_host_store(L, &g, &hg, L->gu_scale_stride * 4, E, S, acct));
    L->gu_scale = reinterpret_cast<float*>(g);
    L->hs_gu_scale = reinterpret_cast<float*>(hg);
    uint8_t* d = reinterpret_cast<uint8_t*>(L->dn_scale);
    uint8_t* hd = nullptr;
    MOE_TRY(to_host_store(L, &d, &hd, L->dn_scale_stride * 4, E, S, acct));
    L->dn_scale = reinterpret_cast<float*>(d);
    L->hs_dn_scale = reinterpret_cast<float*>(hd);
  }
  MOE_TRY(dalloc(&L->slot_of, sizeof(int32_t) * E, acct));
  MOE_CUDA_TRY(cudaMemset(L->slot_of, 0xFF, sizeof(int32_t) * E));  // nothing resident
  MOE_CUDA_TRY(cudaStreamCreateWithFlags(&L->copy_stream, cudaStreamNonBlocking));
  MOE_CUDA_TRY(cudaEventCreateWithFlags(&L->last_read, cudaEventDisableTiming));
  MOE_CUDA_TRY(cudaEventCreateWithFlags(&L->copies_done, cudaEventDisableTiming));
  L->slot_expert.assign(S, -1);
  L->slot_state.assign(S, SLOT_EMPTY);
  L->last_use.assign(S, 0);
  L->slot_of_host.assign(E, -1);
  L->hit_counts.assign(E, 0);
  return MOE_OK;
}

static void free_weights(moe_layer* L) {
  cudaFree(L->gu_q);
  cudaFree(L->gu_s);
  cudaFree(L->dn_q);
  cudaFree(L->dn_s);
  cudaFree(L->router_w);
  cudaFree(L->router_b);
  cudaFree(L->gu_scale);
  cudaFree(L->dn_scale);
  L->gu_scale = L->dn_scale = nullptr;
  L->gu_q = L->gu_s = L->dn_q = L->dn_s = nullptr;
  L->router_w = nullptr;
  L->router_b = nullptr;
}

static int64_t ggml_bytes(int wdtype, int64_t n) {
  switch (wdtype) {
    case MOE_DTYPE_BF16: return n * 2;
    case MOE_DTYPE_Q8_0: return n / 32 * 34;
    case MOE_DTYPE_Q4_K: return n / 256 * 144;
    case MOE_DTYPE_FP8_E4M3_B128: return n;
    case MOE_DTYPE_Q2_0: return n / 64 * 18;
  }
  return -1;
}

// Source bytes on the device: either the caller's device pointer or a temporary upload.
static moe_status stage_source(const void* src, int64_t bytes, bool on_device, uint8_t** out, bool* owned) {
  if (on_device) {
    *out = (uint8_t*)src;
    *owned = false;
    return MOE_OK;
  }
  MOE_TRY(dalloc(out, (size_t)bytes, nullptr));
  *owned = true;
  cudaError_t e = cudaMemcpy(*out, src, (size_t)bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(*out);
    *out = nullptr;
    return cuda_fail(e, "cudaMemcpy(weights)");
  }
  return MOE_OK;
}

static moe_status validate_desc(const moe_layer_desc* d) {
  if (!d) return fail(MOE_ERR_INVALID, "moe_layer_create: null desc");
  if (d->num_experts <= 0 || d->num_experts > 1024) return fail(MOE_ERR_INVALID, "num_experts must be in 1..1024");
  if (d->top_k <= 0 || d->top_k > d->num_experts || d->top_k > 32)
    return fail(MOE_ERR_INVALID, "top_k must be in 1..min(num_experts, 32)");
  if (d->hidden <= 0 || d->inter <= 0) return fail(MOE_ERR_INVALID, "hidden and inter must be positive");
  if (d->hidden % 32 || d->inter % 32)
    return fail(MOE_ERR_INVALID, "hidden and inter must be multiples of 32 (one Q8_0 block / two k16 MMA steps)");
  if (d->wdtype == MOE_DTYPE_Q4_K && (d->hidden % 256 || d->inter % 256))
    return fail(MOE_ERR_INVALID, "Q4_K needs hidden and inter multiples of 256 (one super-block)");
  if (d->wdtype == MOE_DTYPE_FP8_E4M3_B128 && (d->hidden % 128 || d->inter % 128))
    return fail(MOE_ERR_INVALID, "FP8 128x128-block weights need hidden and inter multiples of 128");
  if (d->wdtype == MOE_DTYPE_FP8_E4M3_B128 && (!d->gate_scale || !d->up_scale || !d->down_scale))
    return fail(MOE_ERR_INVALID, "FP8 weights need gate_scale, up_scale and down_scale");
  if (d->wdtype == MOE_DTYPE_Q2_0 && (d->hidden % 128 || d->inter % 128))
    return fail(MOE_ERR_INVALID, "Q2_0 weights need hidden and inter multiples of 128 (two blocks per group)");
  if (d->wdtype < MOE_DTYPE_BF16 || d->wdtype > MOE_DTYPE_Q2_0) return fail(MOE_ERR_UNSUPPORTED, "unknown weight format");
  if (!d->gate || !d->up || !d->down) return fail(MOE_ERR_INVALID, "null expert stack");
  if (d->max_tokens <= 0) return fail(MOE_ERR_INVALID, "max_tokens must be positive");
  if (d->cache_slots < 0) return fail(MOE_ERR_INVALID, "cache_slots must be >= 0");
  return MOE_OK;
}

extern "C" {

// The per-thread stack (local memory: register spills of some kernel variants) is reserved once
// per device, before any forward runs. Left to the driver, the local-memory pool grows the first
// time a kernel needs a larger frame; the test order decides when that happens, and when it fell
// inside a chain of programmatically overlapped launches the forward ended in an illegal memory
// access (five runs of the GPU test files in non-default orders ended that way; the two runs made
// in those orders with the pool reserved up front passed). The limit is a per-process setting of this device's context:
// MOE_STACK_RESERVE (bytes)
// changes the reserve, 0 leaves the limit to the driver. 16 KB per thread reserves about 5 GB on a
// 148-SM B200 (16 KB x 2,048 threads x 148 SMs).
static moe_status reserve_local_memory(int dev) {
  static std::mutex mu;
  static bool done[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64 || done[dev]) return MOE_OK;
  static const size_t want = [] {
    const char* v = std::getenv("MOE_STACK_RESERVE");
    return v ? (size_t)std::strtoull(v, nullptr, 10) : (size_t)16384;
  }();
  if (want) {
    size_t cur = 0;
    MOE_CUDA_TRY(cudaDeviceGetLimit(&cur, cudaLimitStackSize));
    if (cur < want) MOE_CUDA_TRY(cudaDeviceSetLimit(cudaLimitStackSize, want));
  }
  done[dev] = true;
  return MOE_OK;
}

moe_status moe_layer_create(const moe_layer_desc* desc, moe_layer** out) {
  if (!out) return fail(MOE_ERR_INVALID, "moe_layer_create: null out");
  *out = nullptr;
  MOE_TRY(validate_desc(desc));
  DeviceGuard guard(desc->device);
  if (!guard.ok) return fail(MOE_ERR_CUDA, "moe_layer_create: cannot select device");
  MOE_TRY(reserve_local_memory(desc->device));
  moe_layer* L = new moe_layer();
  L->d = *desc;
  L->dev = desc->device;
  cudaDeviceGetAttribute(&L->sms, cudaDevAttrMultiProcessorCount, L->dev);
  const int E = desc->num_experts, H = desc->hidden, I = desc->inter, w = desc->wdtype;
  const bool on_dev = desc->weights_on_device != 0;
  auto cleanup = [&](moe_status st) {
    free_weights(L);
    free_scratch(L);
    free_cache(L);
    delete L;
    return st;
  };
  L->tc = (w == MOE_DTYPE_Q4_K || w == MOE_DTYPE_FP8_E4M3_B128);
  // Q8_0 with 128-multiple shapes: one copy of the weights in 17 KB units (repack_q8_units), read by
  // the decode GEMV (few tokens per expert) and by the tcgen05 GEMM (more)
  L->q8_tiles = w == MOE_DTYPE_Q8_0 && H % 128 == 0 && I % 128 == 0;
  if (L->q8_tiles) L->tc = true;
  L->gu_q_stride = L->tc ? tc_weight_bytes(w, 2 * I, H) : device_q_bytes(w, 2 * I, H);
  L->gu_s_stride = L->tc ? 0 : device_s_bytes(w, 2 * I, H);
  L->dn_q_stride = L->tc ? tc_weight_bytes(w, H, I) : device_q_bytes(w, H, I);
  L->dn_s_stride = L->tc ? 0 : device_s_bytes(w, H, I);
  int64_t acct = 0;
  moe_status st;
  if ((st = dalloc(&L->gu_q, (size_t)(L->gu_q_stride * E), &acct)) != MOE_OK) return cleanup(st);
  if ((st = dalloc(&L->dn_q, (size_t)(L->dn_q_stride * E), &acct)) != MOE_OK) return cleanup(st);
  if (L->gu_s_stride && (st = dalloc(&L->gu_s, (size_t)(L->gu_s_stride * E), &acct)) != MOE_OK) return cleanup(st);
  if (L->dn_s_stride && (st = dalloc(&L->dn_s, (size_t)(L->dn_s_stride * E), &acct)) != MOE_OK) return cleanup(st);
  {
    const int64_t gb = ggml_bytes(w, (int64_t)E * I * H);
    uint8_t *g = nullptr, *u = nullptr, *dn = nullptr;
    bool og = false, ou = false, od = false;
    st = stage_source(desc->gate, gb, on_dev, &g, &og);
    if (st == MOE_OK) st = stage_source(desc->up, gb, on_dev, &u, &ou);
    if (st == MOE_OK) st = stage_source(desc->down, gb, on_dev, &dn, &od);
    uint8_t *gs = nullptr, *us = nullptr, *ds = nullptr;
    bool ogs = false, ous = false, ods = false;
    if (L->tc) {
      if (st == MOE_OK && w == MOE_DTYPE_FP8_E4M3_B128) {
        const int64_t gsb = (int64_t)E * (I / 128) * (H / 128) * 4;
        st = stage_source(desc->gate_scale, gsb, on_dev, &gs, &ogs);
        if (st == MOE_OK) st = stage_source(desc->up_scale, gsb, on_dev, &us, &ous);
        if (st == MOE_OK) st = stage_source(desc->down_scale, gsb, on_dev, &ds, &ods);
        if (st == MOE_OK) st = dalloc(&L->gu_scale, sizeof(float) * tc_scale_count(w, 2 * I, H) * E, &acct);
        if (st == MOE_OK) st = dalloc(&L->dn_scale, sizeof(float) * tc_scale_count(w, H, I) * E, &acct);
      }
      if (st == MOE_OK)
        st = tc_repack(w, g, u, (const float*)gs, (const float*)us, E, I, H, L->gu_q, L->gu_scale, 0);
      if (st == MOE_OK)
        st = tc_repack(w, dn, nullptr, (const float*)ds, (const float*)ds, E, H, I, L->dn_q, L->dn_scale, 0);
    } else {
      if (st == MOE_OK) st = repack_projection(w, g, u, E, I, H, L->gu_q, L->gu_s, 0);
      if (st == MOE_OK) st = repack_projection(w, dn, nullptr, E, H, I, L->dn_q, L->dn_s, 0);
    }
    cudaError_t se = cudaDeviceSynchronize();
    if (og) cudaFree(g);
    if (ou) cudaFree(u);
    if (od) cudaFree(dn);
    if (ogs) cudaFree(gs);
    if (ous) cudaFree(us);
    if (ods) cudaFree(ds);
    if (st != MOE_OK) return cleanup(st);
    if (se != cudaSuccess) return cleanup(cuda_fail(se, "repack"));
  }
  if (desc->router_weight) {
    const size_t rb = (size_t)E * H * 2;
    if ((st = dalloc(&L->router_w, rb, &acct)) != MOE_OK) return cleanup(st);
    cudaError_t e = cudaMemcpy(L->router_w, desc->router_weight, rb, on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMemcpy(router)"));
  }
  if (desc->router_bias) {
    if ((st = dalloc(&L->router_b, sizeof(float) * E, &acct)) != MOE_OK) return cleanup(st);
    cudaError_t e = cudaMemcpy(L->router_b, desc->router_bias, sizeof(float) * E,
                               on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMemcpy(router bias)"));
  }
  if (desc->cache_slots > 0 && desc->cache_slots < E) {
    L->slots = desc->cache_slots;
    L->gu_scale_stride = L->gu_scale ? tc_scale_count(w, 2 * I, H) : 0;
    L->dn_scale_stride = L->dn_scale ? tc_scale_count(w, H, I) : 0;
    if ((st = setup_cache(L, &acct)) != MOE_OK) return cleanup(st);
  }
  L->weight_bytes = acct;
  // the desc keeps no caller pointers beyond create
  L->d.gate = L->d.up = L->d.down = nullptr;
  L->d.gate_scale = L->d.up_scale = L->d.down_scale = nullptr;
  L->d.router_weight = nullptr;
  L->d.router_bias = nullptr;
  if ((st = alloc_scratch(L, desc->max_tokens)) != MOE_OK) return cleanup(st);
  *out = L;
  return MOE_OK;
}

moe_status moe_layer_warmup(moe_layer* L, int max_tokens) {
  if (!L) return fail(MOE_ERR_INVALID, "moe_layer_warmup: null layer");
  if (max_tokens <= 0) return fail(MOE_ERR_INVALID, "moe_layer_warmup: max_tokens must be positive");
  DeviceGuard guard(L->dev);
  MOE_CUDA_TRY(cudaDeviceSynchronize());
  MOE_TRY(alloc_scratch(L, max_tokens));
  L->d.max_tokens = max_tokens > L->d.max_tokens ? max_tokens : L->d.max_tokens;
  return MOE_OK;
}

moe_status moe_route(moe_layer* L, const void* x, int T, uint32_t* ids, float* weights, void* stream) {
  if (!L) return fail(MOE_ERR_INVALID, "moe_route: null layer");
  if (!L->router_w) return fail(MOE_ERR_INVALID, "moe_route: layer was created without router weights");
  if (T > L->cap_tokens)
    return fail(MOE_ERR_INVALID, "moe_route: T exceeds the max_tokens sized at create/warmup");
  DeviceGuard guard(L->dev);
  RouteParams p{static_cast<const __nv_bfloat16*>(x), L->router_w, L->router_b, ids, weights, T, L->d.hidden,
                L->d.num_experts, L->d.top_k, L->d.router_mode, L->d.n_group, L->d.topk_group,
                L->d.routed_scale};
  return route_tokens(p, L->route_ws, L->route_ws_bytes, static_cast<cudaStream_t>(stream));
}

// Row tiles per CTA for the expected number of distinct experts (uniform routing:
// E (1 - (1 - 1/E)^pairs)). Large passes (>= 24 tokens, shared memory for one CTA per SM) take
// 16-warp CTAs with one full-K row tile per warp; otherwise the largest of 8/4/2/1 tiles per 8-warp
// CTA that still gives a CTA per SM (fewer tiles per CTA split K across more warps). Asking for no
// more than one CTA per SM keeps small batches in one wave (measured: T = 1 and 2 of config 2 run
// 15% faster than with two per SM, larger batches are unchanged).
static int pick_rowt(int tiles, int tpp, double est_active, int sms) {
  if (tpp >= 24 && tiles >= 16 && est_active * ceil_div(tiles, 16) >= 2.0 * sms) return 16;
  for (int r = 8; r >= 1; r >>= 1) {
    if (r > tiles) continue;
    if (est_active * ceil_div(tiles, r) >= sms) return r;
  }
  return 1;
}

static moe_status forward_impl(moe_layer* L, const void* x, int T, const uint32_t* ids, const float* weights,
                               int width, void* y, void* stream, void* const* events, bool combine = true);

// A Q8_0 unit-layout layer runs the tcgen05 GEMM once the batch averages 4 or more tokens per
// expert (below that the GEMV streams the weights faster: it splits K across warps, so few experts
// still fill the GPU, and its MMA work is still small; measured on config 2, T = 32 is a tie and
// T = 64 is 4% faster on the GEMM). When the GEMM's gate/up work items (one per expert and 128-row
// tile) cannot fill the CTA slots (an expert-parallel rank's 16 experts: 192 items for 296 slots),
// the GEMV keeps batches up to 16 tokens per expert (measured at 8 ranks: 8 tokens per expert 28%
// faster on the GEMV, 16 tokens per expert 7% faster on the GEMM). MOE_Q8_PATH=gemv|gemm pins the
// choice.
static bool q8_uses_gemm(int n_pairs, int E, int gate_up_tiles, int sms) {
  static const int forced = [] {
    const char* v = std::getenv("MOE_Q8_PATH");
    if (!v) return 0;
    return std::string(v) == "gemm" ? 1 : std::string(v) == "gemv" ? -1 : 0;
  }();
  if (forced) return forced > 0;
  const bool fills = (int64_t)E * gate_up_tiles >= 2ll * sms;
  return (int64_t)n_pairs >= (fills ? 4ll : 16ll) * E;
}

// Below the tcgen05 threshold a Q8_0 unit layer streams its weights through registers (the decode
// GEMV, expert_decode.cu) or through one shared-memory ring per CTA (expert_stream.cu; measured
// slower at every decode size on config 2, kept selectable). MOE_DECODE=gemv|stream pins the choice.
enum DecodeKernel { DECODE_GEMV = 0, DECODE_STREAM = 1 };
static DecodeKernel decode_kernel(int n_pairs, int E) {
  static const int forced = [] {
    const char* v = std::getenv("MOE_DECODE");
    if (!v) return -1;
    const std::string s(v);
    return s == "stream" ? (int)DECODE_STREAM : s == "gemv" ? (int)DECODE_GEMV : -1;
  }();
  if (forced >= 0) return (DecodeKernel)forced;
  (void)n_pairs;
  (void)E;
  return DECODE_GEMV;
}

moe_status moe_forward(moe_layer* L, const void* x, int T, const uint32_t* ids, const float* weights, int width,
                       void* y, void* stream) {
  return forward_impl(L, x, T, ids, weights, width, y, stream, nullptr);
}

moe_status moe_forward_marked(moe_layer* L, const void* x, int T, const uint32_t* ids, const float* weights,
                              int width, void* y, void* stream, void* const* events) {
  if (!events) return fail(MOE_ERR_INVALID, "moe_forward_marked: null events");
  for (int i = 0; i < 5; ++i)
    if (!events[i]) return fail(MOE_ERR_INVALID, "moe_forward_marked: null event");
  return forward_impl(L, x, T, ids, weights, width, y, stream, events);
}

}  // extern "C"

// Stage marker: under stream capture the event becomes an external event-record node of the graph;
// outside capture it is a plain record.
static moe_status mark(void* const* events, int i, cudaStream_t st) {
  if (!events) return MOE_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  MOE_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
  cudaEvent_t ev = static_cast<cudaEvent_t>(events[i]);
  if (cs == cudaStreamCaptureStatusActive) MOE_CUDA_TRY(cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal));
  else MOE_CUDA_TRY(cudaEventRecord(ev, st));
  return MOE_OK;
}

static moe_status forward_impl(moe_layer* L, const void* x, int T, const uint32_t* ids, const float* weights,
                               int width, void* y, void* stream, void* const* events, bool combine) {
  if (!L) return fail(MOE_ERR_INVALID, "moe_forward: null layer");
  if (T < 0 || width <= 0) return fail(MOE_ERR_INVALID, "moe_forward: need T >= 0 and width > 0");
  if (T == 0) return MOE_OK;
  if (!x || !ids || !weights || (combine && !y)) return fail(MOE_ERR_INVALID, "moe_forward: null pointer");
  if ((uintptr_t)x & 15) return fail(MOE_ERR_INVALID, "moe_forward: x must be 16-byte aligned");
  if (((uintptr_t)ids | (uintptr_t)weights) & 3)
    return fail(MOE_ERR_INVALID, "moe_forward: ids and weights must be 4-byte aligned");
  if ((uintptr_t)y & 7) return fail(MOE_ERR_INVALID, "moe_forward: y must be 8-byte aligned");
  const int64_t n64 = (int64_t)T * width;
  if (n64 > L->cap_pairs)
    return fail(MOE_ERR_INVALID, "moe_forward: T * width exceeds the scratch sized at create/warmup (call "
                                 "moe_layer_warmup with a larger max_tokens)");
  DeviceGuard guard(L->dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n_pairs = (int)n64;
  const int E = L->d.num_experts, H = L->d.hidden, I = L->d.inter;
  const int32_t* slot_of = L->slots ? L->slot_of : nullptr;
  if (L->slots) {  // uploads issued since the last forward land first
    std::lock_guard<std::recursive_mutex> lock(L->cache_mu);
    if (L->copies_pending) {
      MOE_CUDA_TRY(cudaStreamWaitEvent(st, L->copies_done, 0));
      L->copies_pending = false;
    }
  }
  const int max_active = n_pairs < E ? n_pairs : E;
  // the kernel-path choices below follow the pairs expected to be live (moe_layer_set_live_hint);
  // grid bounds keep using every slot
  const int n_live = L->live_hint < 1.0f ? std::max(1, (int)((double)n_pairs * L->live_hint)) : n_pairs;
  const double est = (double)E * (1.0 - std::pow(1.0 - 1.0 / E, (double)n_live));
  const bool use_tc = L->tc && (!L->q8_tiles || q8_uses_gemm(n_live, E, 2 * I / 128, L->sms));
  const DecodeKernel dk = L->q8_tiles ? decode_kernel(n_live, E) : DECODE_GEMV;
  // the decode GEMV on Q8_0 units stages tokens converted once by the plan launch
  const bool prep = !use_tc && L->q8_tiles && dk == DECODE_GEMV && L->xq && plan_preps_tokens(n_pairs);
  const TokenPrep tp{static_cast<const __nv_bfloat16*>(x), T, H, L->xq, L->xq_scale};
  PlanOut po{L->counts, L->offsets, L->perm, L->active, L->n_active, L->err, slot_of, L->act_rec};
  MOE_TRY(mark(events, 0, st));
  MOE_TRY(plan_pairs(ids, n_pairs, E, po, L->plan_ws, L->plan_ws_bytes, st, prep ? &tp : nullptr));
  MOE_TRY(mark(events, 1, st));
  if (use_tc) {
    const int w = L->d.wdtype;
    const int bn = tc_token_tile(n_live, E);
    MOE_TRY(tc_tile_list(L->counts, L->active, L->n_active, bn, L->tile_list, L->n_tiles, st));
    MOE_TRY(tc_gather(x, nullptr, H, width, L->perm, n_pairs, L->offsets + E, L->x16, L->xscale, st, bn < 128));
    TcArgs ga{};
    ga.w = L->gu_q;
    ga.wscale = L->gu_scale;
    ga.w_stride = L->gu_q_stride;
    ga.N_rows = 2 * I;
    ga.K = H;
    ga.phase = 0;
    ga.tile_list = L->tile_list;
    ga.n_tiles = L->n_tiles;
    ga.work = L->n_tiles + 1;
    ga.offsets = L->offsets;
    ga.active = L->active;
    ga.perm = L->perm;
    ga.tscale = L->xscale;
    ga.route_w = weights;
    ga.out = L->h;
    ga.err = L->err;
    ga.tmap = L->tmap_x;
    ga.n_pairs = n_pairs;
    ga.max_active = max_active;
    ga.bn = bn;
    ga.slot_of = slot_of;
    MOE_TRY(tc_gemm(w, ga, st));
    MOE_TRY(mark(events, 2, st));
    MOE_TRY(tc_gather(nullptr, L->h, I, width, L->perm, n_pairs, L->offsets + E, L->h16, L->hscale, st, bn < 128));
    TcArgs da = ga;
    da.w = L->dn_q;
    da.wscale = L->dn_scale;
    da.w_stride = L->dn_q_stride;
    da.N_rows = H;
    da.K = I;
    da.phase = 1;
    da.tscale = L->hscale;
    da.out = L->ypair;
    da.tmap = L->tmap_h;
    da.work = L->n_tiles + 2;
    MOE_TRY(tc_gemm(w, da, st));
    MOE_TRY(mark(events, 3, st));
    if (combine) MOE_TRY(launch_combine(L->ypair, ids, T, width, H, E, y, st, slot_of));
    if (L->slots) MOE_CUDA_TRY(cudaEventRecord(L->last_read, st));  // the slots' readers
    return mark(events, 4, st);
  }

  ExpertParams gp{};
  gp.wq = L->gu_q;
  gp.wsc = L->gu_s;
  gp.q_stride = L->gu_q_stride;
  gp.s_stride = L->gu_s_stride;
  gp.N = 2 * I;
  gp.K = H;
  gp.tiles = 2 * I / 16;
  gp.kb_count = H / 32;
  gp.phase = 0;
  gp.tpp = choose_tpp(H, n_live / (est > 1.0 ? est : 1.0));
  gp.width = width;
  gp.n_pairs = n_pairs;
  gp.x = static_cast<const __nv_bfloat16*>(x);
  gp.out = L->h;
  gp.offsets = L->offsets;
  gp.perm = L->perm;
  gp.active = L->active;
  gp.n_active = L->n_active;
  gp.act_rec = L->act_rec;
  gp.n_wslots = L->slots ? L->slots + L->staging : E;
  gp.slot_of = slot_of;
  gp.tile_major = L->q8_tiles ? 1 : 0;
  if (prep) {
    gp.xq = L->xq;
    gp.xq_scale = L->xq_scale;
  }
  gp.err = L->err;
  auto rowt_of = [&](const ExpertParams& q) { return pick_rowt(q.tiles, q.tpp, est, L->sms); };
  auto launch_pass = [&](const ExpertParams& q) -> moe_status {
    if (dk == DECODE_STREAM) return launch_expert_stream(q, max_active, L->sms, st);
    return launch_expert_gemv(L->d.wdtype, q, max_active, rowt_of(q), st);
  };
  MOE_TRY(launch_pass(gp));
  MOE_TRY(mark(events, 2, st));

  ExpertParams dp = gp;
  dp.wq = L->dn_q;
  dp.wsc = L->dn_s;
  dp.q_stride = L->dn_q_stride;
  dp.s_stride = L->dn_s_stride;
  dp.N = H;
  dp.K = I;
  dp.tiles = H / 16;
  dp.kb_count = I / 32;
  dp.phase = 1;
  dp.tpp = choose_tpp(I, n_live / (est > 1.0 ? est : 1.0));
  dp.x = nullptr;
  dp.xq = nullptr;
  dp.xq_scale = nullptr;
  dp.h_in = L->h;
  dp.route_w = weights;
  dp.out = L->ypair;
  MOE_TRY(launch_pass(dp));
  MOE_TRY(mark(events, 3, st));
  if (combine) MOE_TRY(launch_combine(L->ypair, ids, T, width, H, E, y, st, slot_of));
  if (L->slots) MOE_CUDA_TRY(cudaEventRecord(L->last_read, st));  // the slots' readers
  return mark(events, 4, st);
}

extern "C" {

void moe_layer_destroy(moe_layer* L) {
  if (!L) return;
  paged_detach_all(L);
  DeviceGuard guard(L->dev);
  cudaDeviceSynchronize();
  free_weights(L);
  free_scratch(L);
  free_cache(L);
  delete L;
}

int64_t moe_layer_device_bytes(const moe_layer* L) { return L ? L->weight_bytes + L->scratch_bytes : 0; }

moe_status moe_layer_set_live_hint(moe_layer* L, float live_fraction) {
  if (!L) return fail(MOE_ERR_INVALID, "moe_layer_set_live_hint: null layer");
  if (!(live_fraction > 0.0f && live_fraction <= 1.0f))
    return fail(MOE_ERR_INVALID, "moe_layer_set_live_hint: the fraction must be in (0, 1]");
  L->live_hint = live_fraction;
  return MOE_OK;
}

moe_status moe_layer_check(moe_layer* L, void* stream) {
  if (!L) return fail(MOE_ERR_INVALID, "moe_layer_check: null layer");
  DeviceGuard guard(L->dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  MOE_CUDA_TRY(cudaMemcpyAsync(&v, L->err, sizeof(v), cudaMemcpyDeviceToHost, st));
  MOE_CUDA_TRY(cudaMemsetAsync(L->err, 0, sizeof(int32_t), st));
  MOE_CUDA_TRY(cudaStreamSynchronize(st));
  if (v == MOE_ERR_BAD_IDS) return fail(MOE_ERR_BAD_IDS, "routed expert id >= num_experts");
  if (v != 0) return fail((moe_status)v, "device error word set");
  return MOE_OK;
}

size_t moe_last_error(char* buf, size_t n) {
  if (buf && n) {
    size_t m = g_last_error.size() < n - 1 ? g_last_error.size() : n - 1;
    memcpy(buf, g_last_error.data(), m);
    buf[m] = 0;
  }
  return g_last_error.size();
}

moe_status moe_route_tokens(const void* x, const void* w_router, const float* bias, int T, int H, int E, int k,
                            int mode, int n_group, int topk_group, float routed_scale, uint32_t* ids,
                            float* weights, void* workspace, size_t workspace_bytes, void* stream) {
  RouteParams p{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w_router), bias, ids,
                weights, T, H, E, k, mode, n_group, topk_group, routed_scale};
  return route_tokens(p, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t moe_route_workspace_bytes(int T, int E) { return route_workspace_bytes(T, E); }

moe_status moe_plan_pairs(const uint32_t* ids, int n_pairs, int E, int32_t* counts, int32_t* offsets,
                          int32_t* perm, int32_t* active, int32_t* n_active, void* workspace,
                          size_t workspace_bytes, int32_t* error_word, void* stream) {
  PlanOut o{counts, offsets, perm, active, n_active, error_word};
  return plan_pairs(ids, n_pairs, E, o, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t moe_plan_workspace_bytes(int n_pairs, int E) { return plan_workspace_bytes(n_pairs, E); }

const char* moe_version(void) { return "moe_b200 0.1 (sm_100a)"; }

}  // extern "C"

// ---- expert cache: route split (a2) and paging (a8) ----------------------------------------------

extern "C" {

moe_status moe_cache_split(moe_layer* L, const uint32_t* ids, int n_pairs, uint8_t* hit) {
  if (!L) return fail(MOE_ERR_INVALID, "moe_cache_split: null layer");
  if (!L->slots) return fail(MOE_ERR_INVALID, "moe_cache_split: the layer has no expert cache (cache_slots = 0)");
  if (n_pairs < 0 || (n_pairs && (!ids || !hit))) return fail(MOE_ERR_INVALID, "moe_cache_split: bad arguments");
  const int E = L->d.num_experts;
  for (int p = 0; p < n_pairs; ++p)
    if (ids[p] != MOE_ID_NONE && ids[p] >= (uint32_t)E)
      return fail(MOE_ERR_BAD_IDS, "moe_cache_split: routed expert id " + std::to_string(ids[p]) + " >= num_experts");
  std::lock_guard<std::recursive_mutex> lock(L->cache_mu);
  const uint64_t tick = ++L->tick;
  for (int p = 0; p < n_pairs; ++p) {
    const uint32_t id = ids[p];
    if (id == MOE_ID_NONE) {
      hit[p] = 2;
      continue;
    }
    L->hit_counts[id] += 1;
    const int s = L->slot_of_host[id];
    if (s >= 0 && L->slot_state[s] == SLOT_PUBLISHED) {  // a slot still loading is a miss
      L->last_use[s] = tick;
      hit[p] = 1;
      ++L->stat_hits;
    } else {
      hit[p] = 0;
      ++L->stat_misses;
    }
  }
  return MOE_OK;
}

moe_status moe_cache_upload(moe_layer* L, const uint32_t* experts, int n, const uint32_t* protect, int n_protect,
                            void* stream, int* n_loaded) {
  if (n_loaded) *n_loaded = 0;
  if (!L) return fail(MOE_ERR_INVALID, "moe_cache_upload: null layer");
  if (!L->slots) return fail(MOE_ERR_INVALID, "moe_cache_upload: the layer has no expert cache (cache_slots = 0)");
  if (n < 0 || n_protect < 0 || (n && !experts) || (n_protect && !protect))
    return fail(MOE_ERR_INVALID, "moe_cache_upload: bad arguments");
  const int E = L->d.num_experts;
  for (int i = 0; i < n; ++i)
    if (experts[i] >= (uint32_t)E) return fail(MOE_ERR_BAD_IDS, "moe_cache_upload: expert id >= num_experts");
  DeviceGuard guard(L->dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::recursive_mutex> lock(L->cache_mu);
  // experts to keep: the caller's protect list and everything this call brings in
  std::vector<int> keep;
  keep.reserve((size_t)(n + n_protect));
  for (int i = 0; i < n_protect; ++i)
    if (protect[i] < (uint32_t)E) keep.push_back((int)protect[i]);
  for (int i = 0; i < n; ++i) keep.push_back((int)experts[i]);
  std::vector<int> published(L->slots);  // a slot still loading (lookahead pass) is never a victim
  for (int s = 0; s < L->slots; ++s) published[s] = L->slot_state[s] == SLOT_PUBLISHED;
  SlotEdits ed{};
  bool waited = false;
  int loaded = 0;
  auto flush = [&]() -> moe_status {
    MOE_TRY(launch_slot_edits(L->slot_of, ed, st));
    ed.n = 0;
    return MOE_OK;
  };
  for (int i = 0; i < n; ++i) {
    const int e = (int)experts[i];
    if (L->slot_of_host[e] >= 0) continue;  // already resident
    int slot = -1;
    for (int s = 0; s < L->slots; ++s)
      if (L->slot_expert[s] < 0) {
        slot = s;
        break;
      }
    if (slot < 0) {
      int victim = -1;
      slot = moe_policy_lru_victim(L->slot_expert.data(), published.data(), L->last_use.data(), L->slots, keep.data(),
                                   (int)keep.size(), &victim);
      if (slot < 0) break;  // every slot holds an expert this call needs
      L->slot_of_host[victim] = -1;
      published[slot] = 0;
      if (ed.n == 64) MOE_TRY(flush());
      ed.expert[ed.n] = victim;
      ed.slot[ed.n++] = -1;
    }
    if (!waited) {  // the previous forward's reads of any slot finish before a slot is overwritten
      MOE_CUDA_TRY(cudaStreamWaitEvent(L->copy_stream, L->last_read, 0));
      waited = true;
    }
    MOE_TRY(cache_copy_expert(L, e, slot));
    L->slot_expert[slot] = e;
    L->slot_state[slot] = SLOT_PUBLISHED;  // copies_done covers it: the next forward waits on it
    L->last_use[slot] = L->tick;
    L->slot_of_host[e] = slot;
    if (ed.n == 64) MOE_TRY(flush());
    ed.expert[ed.n] = e;
    ed.slot[ed.n++] = slot;
    ++loaded;
  }
  if (loaded) {
    MOE_CUDA_TRY(cudaEventRecord(L->copies_done, L->copy_stream));
    L->copies_pending = true;
  }
  MOE_TRY(flush());
  if (n_loaded) *n_loaded = loaded;
  return MOE_OK;
}

int moe_cache_slots(const moe_layer* L, int32_t* slot_expert) {
  if (!L || !L->slots) return 0;
  std::lock_guard<std::recursive_mutex> lock(const_cast<moe_layer*>(L)->cache_mu);
  if (slot_expert)
    for (int s = 0; s < L->slots; ++s) slot_expert[s] = L->slot_expert[s];
  return L->slots;
}

moe_status moe_cache_stats(const moe_layer* L, int64_t* hits, int64_t* misses, int64_t* uploads,
                           int64_t* upload_bytes, uint64_t* hit_counts) {
  if (!L) return fail(MOE_ERR_INVALID, "moe_cache_stats: null layer");
  std::lock_guard<std::recursive_mutex> lock(const_cast<moe_layer*>(L)->cache_mu);
  if (hits) *hits = L->stat_hits;
  if (misses) *misses = L->stat_misses;
  if (uploads) *uploads = L->stat_uploads;
  if (upload_bytes) *upload_bytes = L->stat_upload_bytes;
  if (hit_counts)
    for (size_t e = 0; e < L->hit_counts.size(); ++e) hit_counts[e] = L->hit_counts[e];
  return MOE_OK;
}

}  // extern "C"

extern "C" moe_status moe_forward_chunked(moe_layer* L, const void* x, int T, const uint32_t* ids, const float* weights,
                                          int width, void* y, void* stream) {
  if (!L) return fail(MOE_ERR_INVALID, "moe_forward_chunked: null layer");
  if (T < 0 || width <= 0) return fail(MOE_ERR_INVALID, "moe_forward_chunked: need T >= 0 and width > 0");
  const int chunk = L->cap_pairs / width;  // the most tokens one forward's scratch holds at this width
  if (chunk <= 0) return fail(MOE_ERR_INVALID, "moe_forward_chunked: width exceeds the layer's scratch");
  const int H = L->d.hidden;
  for (int t0 = 0; t0 < T; t0 += chunk) {
    const int n = T - t0 < chunk ? T - t0 : chunk;
    MOE_TRY(forward_impl(L, static_cast<const __nv_bfloat16*>(x) + (int64_t)t0 * H, n, ids + (int64_t)t0 * width,
                         weights + (int64_t)t0 * width, width, static_cast<__nv_bfloat16*>(y) + (int64_t)t0 * H,
                         stream, nullptr));
  }
  return MOE_OK;
}

// ---- cache internals shared with the paged runtime -------------------------------------------------

moe_status moe::cache_copy_expert(moe_layer* L, int e, int slot) {
  auto copy = [&](void* bank, const void* store, int64_t stride) -> moe_status {
    if (!bank || !stride) return MOE_OK;
    MOE_CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(bank) + (int64_t)slot * stride,
                                 static_cast<const uint8_t*>(store) + (int64_t)e * stride, (size_t)stride,
                                 cudaMemcpyHostToDevice, L->copy_stream));
    L->stat_upload_bytes += stride;
    return MOE_OK;
  };
  MOE_TRY(copy(L->gu_q, L->hs_gu_q, L->gu_q_stride));
  MOE_TRY(copy(L->gu_s, L->hs_gu_s, L->gu_s_stride));
  MOE_TRY(copy(L->dn_q, L->hs_dn_q, L->dn_q_stride));
  MOE_TRY(copy(L->dn_s, L->hs_dn_s, L->dn_s_stride));
  MOE_TRY(copy(L->gu_scale, L->hs_gu_scale, L->gu_scale_stride * 4));
  MOE_TRY(copy(L->dn_scale, L->hs_dn_scale, L->dn_scale_stride * 4));
  ++L->stat_uploads;
  return MOE_OK;
}

moe_status moe::cache_reserve_staging(moe_layer* L, int n) {
  if (!L->slots) return fail(MOE_ERR_INVALID, "staging slots need a layer with an expert cache");
  if (n <= L->staging) return MOE_OK;
  DeviceGuard guard(L->dev);
  MOE_CUDA_TRY(cudaDeviceSynchronize());
  const int old_total = L->slots + L->staging, total = L->slots + n;
  int64_t acct = L->weight_bytes;
  auto grow = [&](uint8_t** bank, int64_t stride) -> moe_status {
    if (!*bank || !stride) return MOE_OK;
    uint8_t* nb = nullptr;
    cudaError_t e = cudaMalloc(&nb, (size_t)(stride * total));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(staging slots)");
    e = cudaMemcpy(nb, *bank, (size_t)(stride * old_total), cudaMemcpyDeviceToDevice);
    if (e != cudaSuccess) {
      cudaFree(nb);
      return cuda_fail(e, "cudaMemcpy(staging slots)");
    }
    cudaFree(*bank);
    *bank = nb;
    acct += stride * (total - old_total);
    return MOE_OK;
  };
  MOE_TRY(grow(&L->gu_q, L->gu_q_stride));
  MOE_TRY(grow(&L->gu_s, L->gu_s_stride));
  MOE_TRY(grow(&L->dn_q, L->dn_q_stride));
  MOE_TRY(grow(&L->dn_s, L->dn_s_stride));
  uint8_t* gs = reinterpret_cast<uint8_t*>(L->gu_scale);
  uint8_t* ds = reinterpret_cast<uint8_t*>(L->dn_scale);
  MOE_TRY(grow(&gs, L->gu_scale_stride * 4));
  MOE_TRY(grow(&ds, L->dn_scale_stride * 4));
  L->gu_scale = reinterpret_cast<float*>(gs);
  L->dn_scale = reinterpret_cast<float*>(ds);
  L->staging = n;
  L->weight_bytes = acct;
  return MOE_OK;
}

moe_status moe::layer_forward(moe_layer* L, const void* x, int T, const uint32_t* ids, const float* weights, int width,
                              void* y, cudaStream_t st) {
  return forward_impl(L, x, T, ids, weights, width, y, st, nullptr);
}

moe_status moe::layer_experts(moe_layer* L, const void* x, int T, const uint32_t* ids, const float* weights, int width,
                              cudaStream_t st) {
  return forward_impl(L, x, T, ids, weights, width, nullptr, st, nullptr, false);
}

moe_status moe::layer_combine(moe_layer* L, int T, const uint32_t* ids, int width, void* y, cudaStream_t st) {
  if ((int64_t)T * width > L->cap_pairs) return fail(MOE_ERR_INVALID, "layer_combine: T * width exceeds the scratch");
  DeviceGuard guard(L->dev);
  return launch_combine(L->ypair, ids, T, width, L->d.hidden, L->d.num_experts, y, st, L->slots ? L->slot_of : nullptr);
}
