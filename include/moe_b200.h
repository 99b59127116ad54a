/*
 * moe_b200.h — C ABI of the B200 (sm_100a) MoE-layer library, libmoe_b200.so.
 *
 * The reference (flaneur2020/naiwa-rs) installs a routed-experts operator into its model through
 * a Rust trait pair in its mistral.rs fork:
 *
 *   RoutedExpertsProvider::build(&self, ctx: ExpertLoadContext)
 *       -> Result<Option<Arc<dyn RoutedExperts>>>              src/moe/provider.rs:316-615
 *   RoutedExperts::forward(&self, xs: &Tensor, topk_weights: Tensor, topk_ids: &Tensor)
 *       -> Result<Tensor>                                        src/moe/cached_layer.rs:524-664,
 *                                                                src/moe/expert.rs:59-117
 *
 * Each entry point below names the reference interface it replaces. The ABI carries plain
 * pointers, sizes and status codes only: no Rust, candle or torch types. Device pointers are
 * CUDA device addresses on the layer's device; `stream` is a cudaStream_t (NULL = legacy stream).
 *
 * Ownership: the library owns expert weights (device copies, repacked for the kernels), routers,
 * scratch and cache slots. The caller owns x, ids, weights and y of every call. Errors never
 * abort: every call returns a moe_status, and moe_last_error() gives the message of the last
 * failing call on the calling thread (the reference bails with messages, e.g. route.rs:52-68).
 */
#ifndef MOE_B200_H
#define MOE_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  MOE_OK = 0,
  MOE_ERR_INVALID = 1,     /* bad argument, shape or unsupported combination */
  MOE_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  MOE_ERR_OOM = 3,         /* device or pinned allocation failed */
  MOE_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up (doorbells, paging fences) */
  MOE_ERR_BAD_IDS = 5,     /* a routed expert id >= num_experts (reference route.rs:52-68) */
  MOE_ERR_UNSUPPORTED = 6, /* feature not built for this configuration */
  MOE_ERR_WORKER = 7       /* a latched host-worker error (reference executor.rs:242-253) */
} moe_status;

/* Expert weight formats. Host/device inputs are GGML stacks [E, N, K] (gate/up N=I,K=H;
 * down N=H,K=I), the byte layout src/moe/expert.rs:123-145 slices. */
typedef enum {
  MOE_DTYPE_BF16 = 0,          /* 2 B / weight, row-major */
  MOE_DTYPE_Q8_0 = 1,          /* 34 B / 32 weights: f16 d, int8 qs[32] */
  MOE_DTYPE_Q4_K = 2,          /* 144 B / 256 weights: f16 d, f16 dmin, u8 scales[12], u8 qs[128] */
  MOE_DTYPE_FP8_E4M3_B128 = 3, /* 1 B / weight e4m3 + one f32 scale per 128x128 block ([E, N/128, K/128]) */
  MOE_DTYPE_Q2_0 = 4           /* 18 B / 64 weights: f16 d, 2-bit codes (weight j at bits 2*(j%4) of byte
                                * j/4), weight = (code - 1) * d: the reference's resident-pool format
                                * (src/moe/resident.rs:29-45); hidden and inter multiples of 128 */
} moe_wdtype;

typedef enum {
  MOE_ROUTER_SOFTMAX = 0,        /* softmax over all experts, top-k of it, no renormalisation */
  MOE_ROUTER_SOFTMAX_RENORM = 1, /* softmax, top-k, renormalised over the k (Qwen3-MoE) */
  MOE_ROUTER_SIGMOID_GROUP = 2   /* sigmoid scores + bias, group-limited top-k (DeepSeek-V3) */
} moe_router_mode;

/* Routed-id sentinel: an empty top-k slot. moe_forward and moe_plan_pairs skip it without error
 * (the reference pads with weight 0 and a real id, gpu.rs:100-131; the sentinel also skips the work). */
#define MOE_ID_NONE 0xFFFFFFFFu

typedef struct moe_layer moe_layer;

typedef struct {
  int num_experts;      /* E   (reference: ctx.config.num_experts) */
  int top_k;            /* k   (config.num_experts_per_tok) */
  int hidden;           /* H   (config.hidden_size), multiple of 32 */
  int inter;            /* I   (config.moe_intermediate_size), multiple of 32 */
  int wdtype;           /* moe_wdtype */
  /* Stacked projections in GGML layout; host or device memory per `weights_on_device`.
   * For MOE_DTYPE_FP8_E4M3_B128 the *_scale arrays give the [E, N/128, K/128] f32 block scales. */
  const void* gate;
  const void* up;
  const void* down;
  const float* gate_scale;
  const float* up_scale;
  const float* down_scale;
  int weights_on_device; /* 0: host pointers, 1: device pointers on `device` */
  /* Router (the fork's gate linear; kept on the CPU for prediction at provider.rs:618-629). */
  const uint16_t* router_weight; /* [E, H] bf16, same memory kind as the weights; may be NULL */
  const float* router_bias;      /* [E] f32 selection bias for MOE_ROUTER_SIGMOID_GROUP; may be NULL */
  int router_mode;               /* moe_router_mode */
  int n_group;                   /* groups for MOE_ROUTER_SIGMOID_GROUP */
  int topk_group;                /* groups kept */
  float routed_scale;            /* multiplier on routed weights (1.0 when unused) */
  int device;                    /* CUDA ordinal (reference: ctx.layer_device) */
  int max_tokens;                /* largest T of one forward call; sizes scratch at create */
  /* Expert cache (the reference's CachedLayer slots, cached_layer.rs:1056-1228): 0 keeps every
   * expert in device memory; 0 < cache_slots < num_experts keeps all experts in pinned host memory
   * (already in the device layout) and cache_slots of them in device slots, managed with
   * moe_cache_split / moe_cache_upload. A forward then runs only the resident experts' pairs. */
  int cache_slots;
} moe_layer_desc;

/* Replaces RoutedExpertsProvider::build (src/moe/provider.rs:316-615): validates the shape,
 * copies and repacks the expert stacks into device memory, allocates scratch for max_tokens.
 * The first layer created on a device raises that device's cudaLimitStackSize to 16 KB per thread
 * (MOE_STACK_RESERVE=<bytes> changes it, 0 leaves the limit alone) for the rest of the process, so
 * the driver never grows its local-memory pool in the middle of the forward's overlapped launches. */
moe_status moe_layer_create(const moe_layer_desc* desc, moe_layer** out);

/* Replaces the provider's warmup (src/moe/provider.rs:192-303): grows scratch to max_tokens. */
moe_status moe_layer_warmup(moe_layer* layer, int max_tokens);

/* Router + top-k for T tokens, upstream of RoutedExperts::forward in the reference's fork model
 * (its CPU restatement is CachedLayer::predict, cached_layer.rs:1236-1249 with top_k_ids
 * :358-363). x: [T, H] bf16 device; ids: [T, k] u32 device; weights: [T, k] f32 device. ids are
 * ordered by score, largest first, ties to the lowest expert id. */
moe_status moe_route(moe_layer* layer, const void* x, int T, uint32_t* ids, float* weights, void* stream);

/* Replaces RoutedExperts::forward(xs, topk_weights, topk_ids) (cached_layer.rs:524-664,
 * expert.rs:59-117): y[t] = sum_j weights[t,j] * down(silu(gate x_t) * up x_t) of expert ids[t,j].
 * x, y: [T, H] bf16 device; ids [T, width] u32; weights [T, width] f32. `width` may differ from
 * top_k (weight-0 padded rows, gpu.rs:100-131). An id of MOE_ID_NONE marks an empty slot that is
 * skipped (no expert runs for it); other ids >= num_experts fail with MOE_ERR_BAD_IDS (reported by
 * the next call that synchronises; checked on device, no host read). */
moe_status moe_forward(moe_layer* layer, const void* x, int T, const uint32_t* ids, const float* weights,
                       int width, void* y, void* stream);

/* moe_forward with five caller-created CUDA events recorded on `stream` around its stages:
 * events[0] before the plan, [1] after the plan, [2] after gate/up, [3] after down, [4] after the
 * combine (recorded as external events, so they also become event nodes of a captured graph).
 * The per-stage timing probe the reference keeps behind NAIWA_STEP_BUDGET (src/stats/budget.rs). */
moe_status moe_forward_marked(moe_layer* layer, const void* x, int T, const uint32_t* ids, const float* weights,
                              int width, void* y, void* stream, void* const* events);

/* Releases everything the layer owns (the provider's Drop). Safe on NULL. */
void moe_layer_destroy(moe_layer* layer);

/* Number of device bytes the layer holds (weights + scratch); the slot pricing of
 * src/moe/slot.rs:76-111 extended to scratch. */
int64_t moe_layer_device_bytes(const moe_layer* layer);

/* The share of a forward's id slots expected to be live (not MOE_ID_NONE), default 1. The layer picks
 * its kernels (decode GEMV or tcgen05 GEMM, token tile sizes) from the live pairs it expects; a caller
 * whose ids are mostly empty slots says so here (an expert-parallel rank runs world * T received rows
 * of which about 1 / world of the slots are its own). Results do not depend on it. No counterpart in
 * the reference. */
moe_status moe_layer_set_live_hint(moe_layer* layer, float live_fraction);

/* Reads and clears the device-side error word of the layer (bad ids seen by a forward).
 * Synchronises `stream`. Returns MOE_OK or the latched status. */
moe_status moe_layer_check(moe_layer* layer, void* stream);

/* Message of the last failing call on this thread; returns its length. */
size_t moe_last_error(char* buf, size_t n);

/* ---- stateless kernels (the layer calls the same code) ----------------------------------- */

/* Router logits + top-k without a layer. w_router: [E, H] bf16; bias: [E] f32 or NULL.
 * workspace: 16-byte aligned device scratch of moe_route_workspace_bytes(T, E) bytes, zero-filled
 * before its first use; every call leaves it ready for the next call on the same stream. */
moe_status moe_route_tokens(const void* x, const void* w_router, const float* bias, int T, int H, int E, int k,
                            int mode, int n_group, int topk_group, float routed_scale, uint32_t* ids,
                            float* weights, void* workspace, size_t workspace_bytes, void* stream);
size_t moe_route_workspace_bytes(int T, int E);

/* Expert histogram + stable token->expert permutation of n_pairs routed pairs (the grouping the
 * reference does in Gpu::submit, gpu.rs:103-132, and rings::group_rows, rings.rs:68-156).
 * counts [E], offsets [E+1] (exclusive prefix), perm [n_pairs] (sorted position -> pair index,
 * stable), active [E] (experts with count > 0, ascending) and n_active [1], all int32 device.
 * workspace: device scratch of moe_plan_workspace_bytes(n_pairs, E) bytes. */
moe_status moe_plan_pairs(const uint32_t* ids, int n_pairs, int E, int32_t* counts, int32_t* offsets,
                          int32_t* perm, int32_t* active, int32_t* n_active, void* workspace,
                          size_t workspace_bytes, int32_t* error_word, void* stream);
size_t moe_plan_workspace_bytes(int n_pairs, int E);

/* Router logits + top-k for callers that cannot allocate device memory. No counterpart in the
 * reference: its router runs inside the model it links against. Some callers of this library have
 * no allocator to give moe_route_tokens its workspace: a host binding that owns no CUDA allocator
 * and only forwards pointers it was handed, code running while a stream capture is active (a
 * cudaMalloc there breaks the capture), or an embedding that fixes the library's device memory up
 * front. This call runs the same router kernel with its workspace in a file-scope device array of
 * MOE_ROUTE_NOALLOC_MAX_BYTES, which every GPU that loads the library holds until the process exits.
 * It never allocates or frees. Calls needing more than the array (moe_route_workspace_bytes(T, E)
 * above the maximum) fail with MOE_ERR_INVALID. The first call on a device looks up the array's
 * device address; make that first call before any stream capture. All calls on a device share the
 * array: calls that overlap on the GPU (different streams without ordering) race and give wrong
 * results. Arguments and results are those of moe_route_tokens without the workspace. */
#define MOE_ROUTE_NOALLOC_MAX_BYTES (1u << 20)
moe_status moe_route_tokens_noalloc(const void* x, const void* w_router, const float* bias, int T, int H, int E,
                                    int k, int mode, int n_group, int topk_group, float routed_scale, uint32_t* ids,
                                    float* weights, void* stream);

/* ---- expert parallelism (one process per GPU, experts sharded by rank) ---------------------
 * No counterpart in the reference, which runs one GPU plus CPU offload. Rank r owns the experts
 * [r * experts_per_rank, (r + 1) * experts_per_rank). Each rank routes its own T tokens; a token is
 * sent once to every rank that owns at least one of its experts (with group-limited routing and one
 * group per rank, at most topk_group ranks), carrying its k (id, weight) slots with the ids local to
 * the destination and the other slots set to MOE_ID_NONE / 0. The receiving rank runs moe_forward on
 * the rows it received; the per-rank outputs travel back and moe_ep_combine sums them per token. */

/* Dispatch plan. ids, weights: [T, k] (global expert ids; MOE_ID_NONE slots are ignored; other ids
 * >= experts_per_rank * world latch MOE_ERR_BAD_IDS in error_word and are ignored). Outputs (int32
 * unless noted, device): rank_counts [world] rows per destination; n_send [1] their sum;
 * token_rows [T, world] the send row of (token, rank) or -1; send rows ordered by rank, then token:
 * send_token [cap], send_ids [cap, k] u32, send_weights [cap, k] f32, cap = T * min(world, k).
 * One CTA; world <= 64. */
moe_status moe_ep_dispatch_plan(const uint32_t* ids, const float* weights, int T, int k, int experts_per_rank,
                                int world, int32_t* rank_counts, int32_t* n_send, int32_t* token_rows,
                                int32_t* send_token, uint32_t* send_ids, float* send_weights, int32_t* error_word,
                                void* stream);

/* send_x[row] = x[send_token[row]] for row < *n_send. x [T, H] bf16, send_x [cap, H] bf16. */
moe_status moe_ep_pack_rows(const void* x, int T, int H, const int32_t* send_token, const int32_t* n_send, int cap,
                            void* send_x, void* stream);

/* y[t] = y_add[t] + sum over ranks r (in rank order) of y_back[token_rows[t, r]] (rows < 0 skipped),
 * accumulated in f32 and rounded once to bf16. y_back [*, H] bf16 in send-row order; y_add [T, H]
 * bf16 or NULL (e.g. the shared expert's output); y [T, H] bf16. */
moe_status moe_ep_combine(const void* y_back, const int32_t* token_rows, int T, int world, int H, const void* y_add,
                          void* y, void* stream);

/* ---- expert cache (layers created with cache_slots > 0) ------------------------------------
 * One layer, one compute stream: the calls below and the layer's forwards must be issued from one
 * host thread onto the same stream. */

/* Route split (src/moe/stages/route.rs:19-158): for each routed pair (host ids, n_pairs), hit[p] = 1
 * when its expert is resident, 0 when it is a miss, 2 for MOE_ID_NONE. Resident experts that are hit
 * get this call's LRU tick; every routed pair counts toward its expert's hit count. Ids >= E other
 * than MOE_ID_NONE fail with MOE_ERR_BAD_IDS (route.rs:52-68). Host only: no stream work. */
moe_status moe_cache_split(moe_layer* layer, const uint32_t* ids, int n_pairs, uint8_t* hit);

/* Paging (CachedLayer::admit / replace, cached_layer.rs:1056-1228; CopyStream upload with its read
 * fence, copy_stream.rs:22-26, 66-102, 291-410): makes `experts` resident in order, each into a free
 * slot, else into the least-recently-used slot whose expert is in neither `experts` nor `protect`;
 * stops when no slot can be freed. Copies run on the layer's copy stream from the pinned host store,
 * after the last forward that may read the slot; the next forward on `stream` waits for them, and the
 * slot map is updated on `stream`. *n_loaded = experts brought in by this call. */
moe_status moe_cache_upload(moe_layer* layer, const uint32_t* experts, int n, const uint32_t* protect, int n_protect,
                            void* stream, int* n_loaded);

/* Number of slots (0 without a cache); slot_expert [slots] receives each slot's expert or -1. */
int moe_cache_slots(const moe_layer* layer, int32_t* slot_expert);

/* Counters since create: pair hits and misses of moe_cache_split, experts uploaded and their bytes;
 * hit_counts [E] (optional) receives each expert's routed-pair count. */
moe_status moe_cache_stats(const moe_layer* layer, int64_t* hits, int64_t* misses, int64_t* uploads,
                           int64_t* upload_bytes, uint64_t* hit_counts);

/* ---- the cache's decision functions (host only, no CUDA) ----------------------------------- */
/* top_k_ids (cached_layer.rs:358-363): the k largest logits, largest first, ties to the lowest
 * index, f32 total order. Returns the count written (min(k, n)). */
int moe_policy_top_k_ids(const float* logits, int n, int k, int32_t* out);
/* union_by_votes (:367-379): every listed expert once, by votes, then best rank, then id. */
int moe_policy_union_by_votes(const int32_t* const* rankings, const int32_t* lens, int n_rankings, int32_t* out);
/* streamed_misses (:385-398): the distinct missed experts ranked by total routed weight (ties to the
 * lower id), the first min(ceil(frac * distinct), cap). Rows of (id, weight) pairs, row_lens[rows]. */
int moe_policy_streamed_misses(const uint32_t* ids, const float* weights, const int32_t* row_lens, int rows,
                               float frac, int cap, uint32_t* out);
/* lru_victim (:401-410): the slot of the least-recently-used published expert not in `protect`
 * (ties to the lower expert id), its expert in *expert_out; -1 when there is none. */
int moe_policy_lru_victim(const int32_t* slot_expert, const int32_t* slot_published, const uint64_t* last_use,
                          int n_slots, const int32_t* protect, int n_protect, int32_t* expert_out);
/* fill_candidate (:344-355): the most-routed expert not in a slot (ties to the lowest id); -1 when
 * every slot is taken. */
int moe_policy_fill_candidate(const int32_t* slot_expert, int n_slots, const uint64_t* hit_counts, int n_experts);

/* ---- doorbells: host <-> device hand-off rings over mapped pinned memory ------------------
 * Replace src/doorbell (doorbell.cu:15-149, mapped.rs:18-141, payload_ring.rs:14-81): the top-k
 * doorbell that brings a layer's routing to the host thread without a stream sync
 * (d2h/topk.rs:20-125) and the result doorbell that brings CPU-computed expert outputs back to the
 * device (h2d/result.rs:27-123). A ring is `depth` slots of slot_bytes (rounded up to 16) behind a
 * {seq, consumed, status} header in cudaHostAllocMapped memory. Publishing slot n (1-based) stores
 * the payload, fences, then sets seq = n; the consumer waits for seq >= n, reads the slot and sets
 * consumed = n; a producer waits while seq - consumed == depth. Device-side waits are bounded
 * (about one second): one that runs out records MOE_ERR_TIMEOUT in the ring (see moe_ring_check)
 * and its kernel returns without writing its destination. Host waits take timeout_us (< 0: none).
 * One producer and one consumer per ring; the producer's calls must be made from one thread. */
typedef struct moe_ring moe_ring;
moe_status moe_ring_create(int device, int depth, size_t slot_bytes, moe_ring** out);
void moe_ring_destroy(moe_ring* ring);
size_t moe_ring_slot_bytes(const moe_ring* ring);
/* Device -> host. Enqueues on `stream` a copy of src0[0:n0] followed by src1[0:n1] (device memory;
 * src1 may be NULL with n1 = 0) into the next slot; *seq_out = the slot's number, the target the
 * host waits for. */
moe_status moe_ring_publish_from_device(moe_ring* ring, const void* src0, size_t n0, const void* src1, size_t n1,
                                        void* stream, uint32_t* seq_out);
/* Waits on the calling host thread until slot `target` is published, copies n bytes of it to dst
 * (host memory) and releases the slot. MOE_ERR_TIMEOUT when it does not arrive in time. */
moe_status moe_ring_host_take(moe_ring* ring, uint32_t target, void* dst, size_t n, int64_t timeout_us);
/* Host -> device. Copies src[0:n] (host memory) into the next slot once one is free and publishes
 * it; *seq_out = its number. */
moe_status moe_ring_host_publish(moe_ring* ring, const void* src, size_t n, int64_t timeout_us, uint32_t* seq_out);
/* Enqueues on `stream` a wait for slot `target` and a copy of n bytes of it to dst (device
 * memory); later work on the stream sees dst filled. */
moe_status moe_ring_device_take(moe_ring* ring, uint32_t target, void* dst, size_t n, void* stream);
/* Synchronises `stream`, then reads and clears the ring's status: MOE_OK or MOE_ERR_TIMEOUT. */
moe_status moe_ring_check(moe_ring* ring, void* stream);
/* Current header counters (host view). */
void moe_ring_counters(const moe_ring* ring, uint32_t* seq, uint32_t* consumed);

/* ---- the CPU expert path and its executor --------------------------------------------------
 * Replace CpuExperts::forward (src/moe/expert.rs:59-117), the miss stage's fused decode
 * (src/moe/stages/cpu_miss.rs:21-54) and the result executor (src/executor.rs:116-166, 220-231,
 * 330-378). The CPU experts keep a host copy of Q8_0 or BF16 GGML stacks (desc with host pointers). */
typedef struct moe_cpu_experts moe_cpu_experts;
typedef struct moe_executor moe_executor;
/* n_threads (0: all hardware threads) includes the calling thread; the other n_threads - 1 belong to
 * a worker pool shared by every CPU-experts object with the same n_threads, started by the first
 * such create and kept until the process exits. Calls that share a pool take turns. */
moe_status moe_cpu_experts_create(const moe_layer_desc* desc, int n_threads, moe_cpu_experts** out);
void moe_cpu_experts_destroy(moe_cpu_experts* cpu);
/* Synchronous: y [T, H] f32 (host) = sum over the routed pairs with select[p] != 0 (select NULL: all),
 * skipping MOE_ID_NONE and weight-0 slots, of w * down(silu(gate x) * up x); x [T, H] bf16 host. */
moe_status moe_cpu_forward(const moe_cpu_experts* cpu, const uint16_t* x, const uint32_t* ids, const float* weights,
                           int T, int width, const uint8_t* select, float* y);
/* The instruction set moe_cpu_forward's row dot products use on this host: "avx512", "avx2" or
 * "scalar" (the widest the host reports, chosen at the first call; the environment variable
 * MOE_CPU_ISA=scalar|avx2 caps it, for testing each build). */
const char* moe_cpu_isa(void);
/* An executor runs moe_cpu_forward jobs FIFO on a worker thread and publishes each result ([T, H]
 * f32) into `result_ring` (a host -> device ring whose slots hold max T * H * 4 bytes, used by this
 * executor alone). submit copies its inputs, returns at once, and gives the ring slot the result
 * will occupy in *target (take it with moe_ring_device_take). A failed job publishes zeros and its
 * error is returned by the next submit or drain as MOE_ERR_WORKER. */
moe_status moe_executor_create(moe_cpu_experts* cpu, moe_ring* result_ring, moe_executor** out);
moe_status moe_executor_submit(moe_executor* ex, const uint16_t* x, const uint32_t* ids, const float* weights, int T,
                               int width, const uint8_t* select, uint32_t* target);
/* Waits until every submitted job has published; returns a latched job error if any. */
moe_status moe_executor_drain(moe_executor* ex);
void moe_executor_destroy(moe_executor* ex);
/* y = bf16(y + add) over n elements (device): folds a CPU result into the GPU's output. */
moe_status moe_add_f32_into_bf16(void* y, const float* add, int64_t n, void* stream);

/* ---- prefill chunking (src/moe/prefill_stream.rs:1362-1694) -------------------------------- */
/* moe_forward over T tokens in consecutive chunks of as many tokens as the layer's scratch holds at
 * this width (max_tokens * top_k / width), so a long prompt needs no scratch beyond create/warmup. */
moe_status moe_forward_chunked(moe_layer* layer, const void* x, int T, const uint32_t* ids, const float* weights,
                               int width, void* y, void* stream);
/* out[i] = ids[i] when ids[i] is one of `experts` (host list, E <= 1024), else MOE_ID_NONE (device
 * arrays of n ids): one wave of a paged prefill runs only the experts uploaded for it. */
moe_status moe_select_ids(const uint32_t* ids, int64_t n, int E, const uint32_t* experts, int n_experts,
                          uint32_t* out, void* stream);

/* ---- expert parallelism over NVLink peer memory (one process per GPU, >= 2 GPUs) ----------
 * No counterpart in the reference. Replaces the NCCL all-to-alls around the per-rank layer with
 * kernels that store rows straight into the peers' memory (CUDA IPC mappings, plain loads/stores,
 * no multicast). Each rank creates one peer object (cap_rows = the most tokens one rank sends per
 * call), exports its handle, gathers every rank's handle by any host channel and connects. Per call
 * (epoch = 1, 2, ... identical on every rank; or epoch = 0 in every call, which takes the epoch after
 * the last one whose combine completed on this rank from device memory, so that a captured CUDA
 * graph of whole steps can be replayed), on one stream, either
 *   moe_ep_peer_dispatch_routed -> moe_forward of the local layer on moe_ep_peer_recv_rows /
 *   moe_ep_peer_recv_ids / moe_ep_peer_recv_weights (world * cap_rows rows) -> moe_ep_peer_return ->
 *   moe_ep_peer_combine                                   (three launches besides the forward), or
 *   moe_ep_dispatch_plan (above) -> moe_ep_peer_dispatch -> moe_ep_peer_receive -> moe_forward of the
 *   local layer on moe_ep_peer_recv_rows and the received ids/weights -> moe_ep_peer_return ->
 *   moe_ep_peer_combine.
 * No host synchronisation: the counts travel with the rows. Waits for other ranks are bounded (about
 * five seconds); one that runs out records MOE_ERR_TIMEOUT (moe_ep_peer_check) and its kernel reads no
 * peer data. The local layer needs max_tokens * top_k >= world * cap_rows * top_k. */
typedef struct moe_ep_peer moe_ep_peer;
moe_status moe_ep_peer_create(int device, int rank, int world, int cap_rows, int hidden, int top_k, moe_ep_peer** out);
size_t moe_ep_peer_handle_bytes(void);
moe_status moe_ep_peer_export(moe_ep_peer* peer, void* handle);
/* handles: world * moe_ep_peer_handle_bytes() bytes, rank r's at r * moe_ep_peer_handle_bytes(). */
moe_status moe_ep_peer_connect(moe_ep_peer* peer, const void* handles);
void moe_ep_peer_destroy(moe_ep_peer* peer);
/* This rank's receive rows: [world * cap_rows, hidden] bf16, region s holding source s's rows. */
void* moe_ep_peer_recv_rows(moe_ep_peer* peer);
/* Source and destination in one launch: the plan of moe_ep_dispatch_plan (same rank_counts and
 * token_rows, bit for bit; error_word as there) built from ids [T, top_k] (global expert ids; rank r
 * owns [r * experts_per_rank, (r + 1) * experts_per_rank)), the rows of x [T, hidden] bf16 and their
 * local ids/weights stored into the destinations' receive regions, every flag of this epoch published,
 * then a bounded wait for every source's rows of this epoch. The local forward then reads the regions
 * as they lie: ids of rows past a source's count are MOE_ID_NONE. */
moe_status moe_ep_peer_dispatch_routed(moe_ep_peer* peer, const void* x, int T, const uint32_t* ids,
                                       const float* weights, int experts_per_rank, uint32_t epoch,
                                       int32_t* rank_counts, int32_t* token_rows, int32_t* error_word,
                                       void* stream);
/* This rank's received slots after moe_ep_peer_dispatch_routed: [world * cap_rows, top_k] local ids
 * (uint32) and routing weights (float), the layout moe_forward takes. */
void* moe_ep_peer_recv_ids(moe_ep_peer* peer);
void* moe_ep_peer_recv_weights(moe_ep_peer* peer);
/* Source: the plan's rows (rank_counts, send_token, send_ids, send_weights of moe_ep_dispatch_plan)
 * from x [T, hidden] bf16 into the destinations' receive regions, then this epoch's flags. */
moe_status moe_ep_peer_dispatch(moe_ep_peer* peer, const void* x, int T, const int32_t* rank_counts,
                                const int32_t* send_token, const uint32_t* send_ids, const float* send_weights,
                                uint32_t epoch, void* stream);
/* Destination: waits for every source's rows of this epoch; ids/weights [world * cap_rows, top_k]
 * (device) receive the local slots, MOE_ID_NONE past each source's count. */
moe_status moe_ep_peer_receive(moe_ep_peer* peer, uint32_t epoch, uint32_t* ids, float* weights, void* stream);
/* Destination: y_local [world * cap_rows, hidden] bf16 (the local forward's output) back to the sources. */
moe_status moe_ep_peer_return(moe_ep_peer* peer, const void* y_local, uint32_t epoch, void* stream);
/* Source: waits for every destination's return of this epoch; y [T, hidden] = y_add (or 0) + the
 * token's returned rows in rank order, f32, rounded once (rank_counts / token_rows of the plan). One
 * launch; it completes the epoch (T = 0 only waits). */
moe_status moe_ep_peer_combine(moe_ep_peer* peer, uint32_t epoch, int T, const int32_t* rank_counts,
                               const int32_t* token_rows, const void* y_add, void* y, void* stream);
/* Synchronises `stream`, then reads and clears the peer status: MOE_OK, MOE_ERR_TIMEOUT (a wait for
 * another rank ran out on this rank, or a destination this rank's rows went to reported that its own
 * receive ran out; that epoch's combine then added no returned row) or MOE_ERR_INVALID (a dispatch
 * plan sent more than cap_rows rows to one rank; the extra rows were dropped). */
moe_status moe_ep_peer_check(moe_ep_peer* peer, void* stream);
/* Sets how long the peer's device-side waits for other ranks last (default five seconds), for the
 * launches issued after this call. No counterpart in the reference. */
moe_status moe_ep_peer_set_wait_limit(moe_ep_peer* peer, int64_t timeout_us);

/* ---- paged decode and prefill through an expert cache ---------------------------------------
 * Replaces the reference's CachedLayer call path: the decode split of one layer call between resident
 * slots, streamed misses and the CPU (src/moe/decode.rs:224-378, stages/route.rs:19-158,
 * stages/dma_miss.rs:80-160, stages/cpu_miss.rs:21-54, staging.rs:23-183), the lookahead prefetch of
 * the next layer's predicted experts (stages/preload.rs:18-195, cached_layer.rs:1236-1337) and the
 * ring-batched, upload-overlapped prefill (rings.rs:68-156, prefill_stream.rs:1066, :1362-1694).
 * One moe_paged per cached layer (cache_slots > 0); calls on one layer come from one host thread, on
 * one stream. A process-wide lookahead thread runs the predictions: it reads a layer's router on the
 * host and enqueues copies on that layer's copy stream; every forward of the layer waits for them. */
typedef struct moe_paged moe_paged;
typedef struct {
  int staging_slots;       /* device slots past the cache slots for streamed misses and prefill waves (16) */
  float pcie_frac;         /* streamed_misses fraction of the missed experts copied per call (1.0) */
  int stream_cap;          /* at most this many experts streamed per call, <= staging_slots (16) */
  int lookahead;           /* 1: predict and prefetch the next layer (moe_paged_set_next) from each call's activation */
  int lookahead_swaps;     /* slots a prediction may take from other experts, per activation row (1) */
  int max_tokens;          /* largest T of one moe_paged_forward (<= the layer's max_tokens) (256) */
  int64_t host_timeout_us; /* how long the host waits for the router's top-k and the CPU rows (5 s) */
} moe_paged_opts;
typedef struct {
  int64_t calls, pairs, hits, staged_experts, staged_pairs, cpu_pairs;
  int64_t lookahead_passes, lookahead_loads, lookahead_swaps, lookahead_dropped, lookahead_errors, predicted;
  int64_t prefill_calls, prefill_waves, prefill_uploads;
} moe_paged_stats;
void moe_paged_default_opts(moe_paged_opts* opts);
/* cpu: the CPU expert path for misses that are not streamed (NULL: every miss must fit the staging
 * slots). opts NULL: the defaults. Reserves the staging slots in the layer (synchronises the device). */
moe_status moe_paged_create(moe_layer* layer, moe_cpu_experts* cpu, const moe_paged_opts* opts, moe_paged** out);
void moe_paged_destroy(moe_paged* paged);
/* The layer whose experts this layer's calls predict (the next MoE layer of the model), or NULL. */
moe_status moe_paged_set_next(moe_paged* paged, moe_paged* next);
/* RoutedExperts::forward through the cache: x, y [T, H] bf16 device, ids/weights [T, width] device,
 * width <= 2 * top_k. Waits on the host for this call's top-k (behind the router only). */
moe_status moe_paged_forward(moe_paged* paged, const void* x, int T, const uint32_t* ids, const float* weights,
                             int width, void* y, void* stream);
/* A prompt through the cache: chunks of the layer's scratch; per chunk the resident experts first,
 * then the missing ones in waves of staging_slots / 2, balanced by routed pairs, each wave's upload
 * overlapping the previous wave's compute; the waves' outputs summed in f32, rounded once. */
moe_status moe_paged_prefill(moe_paged* paged, const void* x, int T, const uint32_t* ids, const float* weights,
                             int width, void* y, void* stream);
/* Fills empty cache slots with the most-routed experts not resident (fill_candidate), now. */
moe_status moe_paged_fill(moe_paged* paged, void* stream);
moe_status moe_paged_get_stats(moe_paged* paged, moe_paged_stats* out);
/* Waits until the lookahead thread has no queued or running prediction. */
moe_status moe_paged_drain_lookahead(void);
/* Synchronises `stream`; reports latched errors of the layer, its rings, its CPU jobs and its lookahead. */
moe_status moe_paged_check(moe_paged* paged, void* stream);

/* ---- GGUF expert stacks (on-disk model files) ---------------------------------------------
 * The reference reads its weights from GGUF shards through candle (src/load.rs:414-450) and hands
 * the provider each MoE block's blk.{L}.ffn_{gate,up,down}_exps.weight as stacked [E, N, K] GGML
 * tensors (provider.rs:367), sliced per expert by byte range (expert.rs:123-145). moe_gguf_open maps
 * a GGUF v2/v3 file read-only and parses its header, metadata and tensor table (every read bounds-
 * checked; a malformed file fails with MOE_ERR_INVALID and a message). Pointers it returns point
 * into the mapping and stay valid until moe_gguf_close. */
typedef struct moe_gguf moe_gguf;
moe_status moe_gguf_open(const char* path, moe_gguf** out);
void moe_gguf_close(moe_gguf* file);
int moe_gguf_tensor_count(const moe_gguf* file);
const char* moe_gguf_tensor_name(const moe_gguf* file, int i);
/* A tensor by name: GGML type id, dims[4] (dims[0] fastest; unused dims 1), n_dims, its bytes in the
 * mapping and their count (-1 for a type whose block size this library does not know). */
moe_status moe_gguf_tensor(const moe_gguf* file, const char* name, int* ggml_type, int64_t* dims, int* n_dims,
                           const void** data, int64_t* nbytes);
/* Integer (or bool) metadata value; MOE_ERR_INVALID when absent or not an integer. */
moe_status moe_gguf_get_int(const moe_gguf* file, const char* key, int64_t* value);
/* String metadata value copied into buf (n bytes with the terminator); returns its length, 0 if absent. */
size_t moe_gguf_get_str(const moe_gguf* file, const char* key, char* buf, size_t n);
/* Fills desc from MoE layer `layer` of the file: num_experts, hidden, inter and wdtype from the
 * expert stacks (Q8_0, Q4_K or BF16, one type for all three projections), gate/up/down as host
 * pointers into the mapping (weights_on_device = 0), top_k from {general.architecture}.expert_used_count
 * when present, and router_weight from blk.{L}.ffn_gate_inp.weight (bf16 as stored; f32 / f16
 * converted to bf16 into memory the file object owns), NULL when the file has none. Other fields
 * (device, max_tokens, router mode, cache_slots, ...) are left as the caller set them. */
moe_status moe_gguf_layer_desc(moe_gguf* file, int layer, moe_layer_desc* desc);

/* ---- the resident Q2_0 pool --------------------------------------------------------------------
 * The reference keeps a model's always-needed expert block resident by requantising its stacks to
 * Q2_0 and running them through the ordinary expert kernels (resident.rs:92-182, quantize_q2_0
 * :46-88). Requantises a stacked [E, N, K] projection held on the device in src_dtype (BF16, Q8_0 or
 * Q4_K; K a multiple of 256 for Q4_K, of 64 otherwise) into Q2_0 bytes on the device
 * (E * N * K / 64 * 18 of them): each 64-weight block's f16 scale is searched over
 * amax / {1, 1.25, 1.5, 1.75, 2} for the smallest squared error, codes = clamp(round(x / d) + 1, 0, 3),
 * an all-zero block decodes to zeros. The result is a moe_layer_desc stack with wdtype
 * MOE_DTYPE_Q2_0 (the decode GEMV streams it: 0.28 B per weight). */
moe_status moe_requantize_q2_0(int src_dtype, const void* src, int E, int N, int K, void* dst, void* stream);

/* Library version string. */
const char* moe_version(void);

#ifdef __cplusplus
}
#endif
#endif
