// layer_internal.cuh — the moe_layer object (include/moe_b200.h) shared by layer.cu and paged.cu.
//
// moe_layer plays the role of the reference's per-MoE-block operator (GpuCacheMoeProvider::build,
// src/moe/provider.rs:316-615; RoutedExperts::forward, src/moe/cached_layer.rs:524-664). With an
// expert cache (cache_slots > 0) it also holds the reference's CachedLayer state
// (cached_layer.rs:1056-1228): every expert in pinned host memory in the device layout, `slots`
// device slots, and optionally `staging` more slots past them that the paged runtime (paged.cu)
// streams one call's misses into (the reference's staging ring, staging.rs:23-183).
#pragma once
#include <cuda.h>

#include <mutex>
#include <vector>

#include "moe_internal.cuh"

// Cache slot states. A slot admitted by the lookahead thread is LOADING until its pass has recorded
// the completion event the next forward waits on; only PUBLISHED slots count as hits (the
// reference's published flag, cached_layer.rs:401-410).
enum : int { SLOT_EMPTY = 0, SLOT_LOADING = 1, SLOT_PUBLISHED = 2 };

struct moe_layer {
  moe_layer_desc d{};
  int dev = 0;
  int sms = 148;
  // weights (device layout)
  uint8_t* gu_q = nullptr;
  uint8_t* gu_s = nullptr;
  uint8_t* dn_q = nullptr;
  uint8_t* dn_s = nullptr;
  int64_t gu_q_stride = 0, gu_s_stride = 0, dn_q_stride = 0, dn_s_stride = 0;
  __nv_bfloat16* router_w = nullptr;
  float* router_b = nullptr;
  // scratch
  int cap_pairs = 0;
  int cap_tokens = 0;
  int32_t* counts = nullptr;
  int32_t* offsets = nullptr;
  int32_t* perm = nullptr;
  int32_t* active = nullptr;
  int4* act_rec = nullptr;  // [E] per-active-index {expert, slot, offset, count} records of the plan
  int32_t* n_active = nullptr;
  int32_t* err = nullptr;
  void* plan_ws = nullptr;
  size_t plan_ws_bytes = 0;
  float* h = nullptr;
  float* ypair = nullptr;
  uint32_t* xq = nullptr;     // Q8_0 units: token rows converted by the plan launch for the decode GEMV
  float* xq_scale = nullptr;
  void* route_ws = nullptr;
  size_t route_ws_bytes = 0;
  // tensor-core path (Q4_K / FP8 / Q8_0 at 128-multiples): tile-major weights, f16 staging, TMA maps
  bool tc = false;
  bool q8_tiles = false;  // Q8_0 in units: GEMV or tcgen05 per call (q8_uses_gemm)
  float* gu_scale = nullptr;
  float* dn_scale = nullptr;
  void* x16 = nullptr;
  float* xscale = nullptr;
  void* h16 = nullptr;
  float* hscale = nullptr;
  int32_t* tile_list = nullptr;
  int32_t* n_tiles = nullptr;
  alignas(128) unsigned char tmap_x[128];
  alignas(128) unsigned char tmap_h[128];
  int64_t weight_bytes = 0;
  int64_t scratch_bytes = 0;
  float live_hint = 1.0f;  // expected share of a forward's id slots that are live (kernel-path choice only)
  // expert cache (cache_slots > 0): every expert in pinned host memory in the device layout, `slots`
  // of them (plus `staging` streamed ones) in the device banks above; slot_of maps expert -> slot
  // (-1: not resident)
  int slots = 0;
  int staging = 0;  // staging slots past the cache slots (paged runtime), 0 until reserved
  uint8_t* hs_gu_q = nullptr;
  uint8_t* hs_gu_s = nullptr;
  uint8_t* hs_dn_q = nullptr;
  uint8_t* hs_dn_s = nullptr;
  float* hs_gu_scale = nullptr;
  float* hs_dn_scale = nullptr;
  // how each host-store buffer was pinned: mapped + registered (length > 0) or cudaHostAlloc (0)
  std::vector<std::pair<void*, size_t>> hs_blocks;
  int64_t gu_scale_stride = 0, dn_scale_stride = 0;  // floats per expert (tensor-core FP8 scales)
  int32_t* slot_of = nullptr;                         // device [E]
  std::vector<int> slot_expert;                       // [slots], -1 empty
  std::vector<int> slot_state;                        // [slots] SLOT_*
  std::vector<uint64_t> last_use;                     // [slots]
  std::vector<int> slot_of_host;                      // [E] cache slot (any state), -1 none
  std::vector<uint64_t> hit_counts;                   // [E] routed pairs seen per expert
  uint64_t tick = 0;
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t last_read = nullptr;    // recorded after every forward: the slots' readers
  cudaEvent_t copies_done = nullptr;  // recorded after the latest uploads
  bool copies_pending = false;
  int64_t stat_hits = 0, stat_misses = 0, stat_uploads = 0, stat_upload_bytes = 0;
  // Serialises the cache state above between the thread that calls the layer and the paged
  // runtime's lookahead thread (the reference's per-layer Mutex, cached_layer.rs:494); recursive so
  // the paged runtime can call the layer's own entry points while it holds it.
  std::recursive_mutex cache_mu;
  // Paged runtimes built on this layer (paged.cu); destroying the layer detaches them first, so no
  // lookahead job can reach a freed layer.
  std::vector<struct moe_paged*> paged;
};

namespace moe {

// Device slot-map edits carried in the launch arguments (no host buffer to race with).
struct SlotEdits {
  int n;
  int expert[64];
  int slot[64];
};
moe_status launch_slot_edits(int32_t* slot_of, const SlotEdits& ed, cudaStream_t st);

// Enqueues on L's copy stream the host -> device copies of expert e's stored bytes into device slot
// `slot` (a cache slot or a staging slot); counts them in the upload stats. Call with cache_mu held.
moe_status cache_copy_expert(moe_layer* L, int e, int slot);

// Grows the device banks by n staging slots past the cache slots (synchronises the device; the
// existing slots keep their contents). No-op when the layer already has at least n.
moe_status cache_reserve_staging(moe_layer* L, int n);

// Detaches every paged runtime of L before L is destroyed: their queued lookahead jobs are dropped,
// a running one is waited for, and their later calls fail instead of touching the freed layer.
void paged_detach_all(moe_layer* L);

// moe_forward on an explicit stream, for the paged runtime.
moe_status layer_forward(moe_layer* L, const void* x, int T, const uint32_t* ids, const float* weights, int width,
                         void* y, cudaStream_t st);
// moe_forward without its combine: the per-pair outputs of the live pairs of `ids` land in the
// layer's ypair rows (indexed by pair, t * width + j) and stay there. Several such passes over
// disjoint pair sets followed by one layer_combine over their union give the same bits as one
// forward over the union: every pass sees the same T * width, so it takes the same kernel path.
moe_status layer_experts(moe_layer* L, const void* x, int T, const uint32_t* ids, const float* weights, int width,
                         cudaStream_t st);
// The combine of the live pairs of `ids` from the ypair rows the passes above left: y [T, H] bf16.
moe_status layer_combine(moe_layer* L, int T, const uint32_t* ids, int width, void* y, cudaStream_t st);

}  // namespace moe
