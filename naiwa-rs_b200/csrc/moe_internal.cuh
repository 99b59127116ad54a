// moe_internal.cuh — kernel parameter blocks and launchers shared between translation units.
#pragma once
#include "moe_common.cuh"

namespace moe {

struct RouteParams {
  const __nv_bfloat16* x;  // [T, H]
  const __nv_bfloat16* w;  // [E, H]
  const float* bias;       // [E] or null
  uint32_t* ids;           // [T, k]
  float* weights;          // [T, k]
  int T, H, E, k, mode, n_group, topk_group;
  float routed_scale;
};
// Argument checks of route_tokens alone (shape, mode, pointers, alignment); enqueues nothing.
moe_status route_validate(const RouteParams& p);
moe_status route_tokens(const RouteParams& p, void* ws, size_t ws_bytes, cudaStream_t st);
size_t route_workspace_bytes(int T, int E);

struct PlanOut {
  int32_t* counts;    // [E]
  int32_t* offsets;   // [E+1]
  int32_t* perm;      // [n_pairs]
  int32_t* active;    // [E]
  int32_t* n_active;  // [1]
  int32_t* err;       // [1] or null
  const int32_t* slot_of = nullptr;  // [E] cache slot of each expert (-1: not resident) or null (all resident)
  // [E] or null: per active index a < n_active {expert, weight slot, offset, count}, {-1, 0, 0, 0}
  // past it, so a decode CTA learns its expert with one 16-byte load instead of a dependent chain
  int4* act_rec = nullptr;
};
// Token rows converted once per call for the decode GEMV's gate/up pass: each row's values scaled by
// a power of two into f16 (the scale that stage_row picks) and laid out in B-fragment block order,
// per 32-column block kb 64 bytes whose 16-byte piece c holds the (k, k+1) pairs
// k = 32 kb + 16 s + 8 h + 2 c at word 2 s + h. A CTA then stages a token with 16-byte copies.
struct TokenPrep {
  const __nv_bfloat16* x;  // [T, K]
  int T, K;
  uint32_t* xq;            // [T, K / 2] words
  float* scale;            // [T]
};
// prep (optional): the single-CTA plan launch also converts the token rows, in extra CTAs.
moe_status plan_pairs(const uint32_t* ids, int n_pairs, int E, const PlanOut& o, void* ws, size_t ws_bytes,
                      cudaStream_t st, const TokenPrep* prep = nullptr);
// Whether plan_pairs converts the rows for a call of n_pairs pairs (its single-CTA path).
bool plan_preps_tokens(int n_pairs);
size_t plan_workspace_bytes(int n_pairs, int E);

struct ExpertParams {
  const uint8_t* wq;   // fragment-native weights, expert-major (or Q8_0 tile-major, tile_major = 1)
  const uint8_t* wsc;  // Q8_0 scales (null for BF16)
  int64_t q_stride;    // bytes per expert
  int64_t s_stride;
  int N;               // device rows (gate/up: 2I with 8+8 interleave; down: H)
  int K;               // columns (gate/up: H; down: I)
  int tiles;           // N / 16
  int kb_count;        // K / 32
  int phase;           // 0: gate/up (+SwiGLU) -> h ; 1: down (* w) -> ypair
  int tpp;             // tokens per pass, multiple of 8, <= 32
  int width;           // pairs per token
  int n_pairs;
  const __nv_bfloat16* x;     // phase 0: [T, K] bf16 activations
  const float* h_in;          // phase 1: [n_pairs (sorted), K] f32
  const float* route_w;       // phase 1: [n_pairs] routing weights (pair order)
  float* out;                 // phase 0: h [n_pairs (sorted), N/2]; phase 1: ypair [n_pairs, N]
  const int32_t* offsets;     // [E+1]
  const int32_t* perm;        // [n_pairs] sorted position -> pair
  const int32_t* active;      // [E]
  const int32_t* n_active;    // [1]
  int units_per_expert;
  const int32_t* slot_of;     // [E] cache slot of each expert, or null: weights indexed by expert id
  int tile_major;             // Q8_0 only: weights in 128 x 128 units (repack_q8_units)
  int32_t* err;               // [1] error word (a bounded wait that ran out), or null
  const int4* act_rec = nullptr;    // the plan's per-active-index records (PlanOut::act_rec), or null
  int n_wslots = 0;                 // weight slots the kernel may index (0: not checked)
  const uint32_t* xq = nullptr;     // phase 0, Q8_0 units: the TokenPrep rows (null: stage from x)
  const float* xq_scale = nullptr;  // their scales
};
moe_status launch_expert_gemv(int wdtype, ExpertParams p, int max_active, int rowt, cudaStream_t st);
// The Q8_0 unit-layout pass through a shared-memory weight stream (expert_stream.cu): same results
// as launch_expert_gemv, one persistent CTA per SM.
moe_status launch_expert_stream(ExpertParams p, int max_active, int sms, cudaStream_t st);
int stream_stages(int K, int tpp);
moe_status launch_combine(const float* ypair, const uint32_t* ids, int T, int width, int H, int E, void* y,
                          cudaStream_t st, const int32_t* slot_of = nullptr);
int choose_tpp(int K, double mean_tokens_per_expert);
size_t expert_smem_bytes(int K, int tpp, int rowt, int warps);

int64_t device_q_bytes(int wdtype, int N, int K);
int64_t device_s_bytes(int wdtype, int N, int K);
moe_status repack_projection(int wdtype, const uint8_t* a, const uint8_t* b, int E, int N_src, int K, uint8_t* dq,
                             uint8_t* ds, cudaStream_t st);
// Q8_0 units: per (expert, 128-row tile, 128-column chunk) 16 KB of fragments + 1 KB of scales,
// read by the decode GEMV (tile_major) and the tcgen05 GEMM.
constexpr int Q8_UNIT_BYTES = 128 * 128 + 1024;
moe_status repack_q8_units(const uint8_t* a, const uint8_t* b, int E, int N_src, int K, uint8_t* dst,
                           cudaStream_t st);

// tensor-core (tcgen05) grouped GEMM path for Q4_K and FP8 layers
struct TcArgs {
  const uint8_t* w;
  const float* wscale;
  int64_t w_stride;
  int N_rows, K, phase;
  const int32_t *tile_list, *n_tiles, *offsets, *active, *perm;
  const float *tscale, *route_w;
  float* out;
  int32_t* err;
  const void* tmap;
  int n_pairs, max_active;            // grid bound: token tiles <= n_pairs / bn + max_active
  int bn = 128;                       // tokens per work item: 32 / 64 (decode shapes) or 128 (prefill)
  const int32_t* slot_of = nullptr;  // [E] cache slot of each expert, or null
  int32_t* work = nullptr;            // the launch's work-item counter: zero when the launch starts
};
constexpr int TC_BN_MIN = 32;  // smallest token tile (sizes the tile list)
// Token tile for a forward of n_pairs pairs over E experts: 32 or 64 for decode batches (mean tokens
// per expert <= 16 or <= 24), else 128.
int tc_token_tile(int n_pairs, int E);
moe_status make_row_tmap(void* map_out, const void* base, int64_t rows, int cols);
size_t tensor_map_bytes();
int64_t tc_weight_bytes(int wdtype, int N, int K);
int64_t tc_scale_count(int wdtype, int N, int K);
moe_status tc_repack(int wdtype, const uint8_t* a, const uint8_t* b, const float* sa, const float* sb, int E, int N_src,
                     int K, uint8_t* dst, float* dscale, cudaStream_t st);
// n_valid: device count of sorted positions the plan filled (offsets[E]); positions past it are skipped.
// pdl: programmatic launch (the decode shapes' pipeline)
moe_status tc_gather(const void* x_bf16, const float* x_f32, int K, int width, const int32_t* perm, int n_pairs,
                     const int32_t* n_valid, void* out_f16, float* scale, cudaStream_t st, bool pdl);
// n_list[0]: the list length; n_list[1] and n_list[2] (the work-item counters of the two GEMM launches
// that follow, gate/up and down) are zeroed.
moe_status tc_tile_list(const int32_t* counts, const int32_t* active, const int32_t* n_active, int bn, int32_t* list,
                        int32_t* n_list, cudaStream_t st);
moe_status tc_gemm(int wdtype, const TcArgs& a, cudaStream_t st);

// Makes `dev` current for the guard's lifetime and restores the previous device afterwards.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace moe
