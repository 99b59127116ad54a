// plan.cu — expert histogram + stable token->expert permutation of the routed pairs.
//
// The reference groups routed pairs per expert on the host: per bank in pair order in Gpu::submit
// (src/moe/stages/gpu.rs:103-132), per row in input order in rings::group_rows
// (src/moe/rings.rs:146-156); the grouped kernels of its fork sort again on the device. Here the
// grouping is one stable counting sort on the device: pair p = t*width + j goes to position
// offsets[id_p] + (number of earlier pairs with the same id). The result is a pure function of the
// ids, so it is bit-exact against the oracle's orc_permute.
//
// Ranks inside a chunk of 1024 pairs come from __match_any_sync (lanes with the same id) plus an
// exclusive prefix of per-warp counts over the warps in order; chunks are laid end to end in
// order. Small calls (decode) run the whole plan in one CTA; large ones (prefill, EP dispatch) use
// a histogram / scan / scatter kernel triple over chunk-private counts.
#include "moe_internal.cuh"

namespace moe {

constexpr int PLAN_THREADS = 1024;
constexpr int PLAN_WARPS = PLAN_THREADS / 32;
constexpr int PLAN_CHUNK = PLAN_THREADS;
constexpr int PLAN_MAX_E = 1024;
constexpr int PLAN_SINGLE_MAX = 8 * PLAN_CHUNK;

// Ranks the pairs of one chunk [c0, c0 + 1024) stably and scatters them to perm.
// base[e]: first free position of expert e before this chunk (advanced by the chunk's counts).
// whist: [PLAN_WARPS][E] shared scratch.
__device__ __forceinline__ void rank_chunk(const uint32_t* __restrict__ ids, int n_pairs, int E, int c0,
                                           int* base, int* whist, int32_t* __restrict__ perm,
                                           const int32_t* __restrict__ slot_of) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < PLAN_WARPS * E; i += PLAN_THREADS) whist[i] = 0;
  __syncthreads();
  const int p = c0 + threadIdx.x;
  const bool valid = p < n_pairs;
  uint32_t id = valid ? ids[p] : 0xffffffffu;
  const bool good = valid && pair_live(id, E, slot_of);
  unsigned grp = __match_any_sync(FULL, good ? id : 0xfffffffeu);
  const int lrank = __popc(grp & ((1u << lane) - 1u));
  if (good && lrank == 0) whist[warp * E + id] = __popc(grp);
  __syncthreads();
  // exclusive prefix over warps for every expert; the chunk total advances base
  for (int e = threadIdx.x; e < E; e += PLAN_THREADS) {
    int run = 0;
    for (int w = 0; w < PLAN_WARPS; ++w) {
      int c = whist[w * E + e];
      whist[w * E + e] = run;
      run += c;
    }
    whist[PLAN_WARPS * E + e] = run;  // chunk count of e (one extra row of scratch)
  }
  __syncthreads();
  if (good) {  // a position outside the call's pairs (ids that changed under the plan) is never written
    const int pos = base[id] + whist[warp * E + id] + lrank;
    if (pos >= 0 && pos < n_pairs) perm[pos] = p;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += PLAN_THREADS) base[e] += whist[PLAN_WARPS * E + e];
  __syncthreads();
}


// One warp converts token row t of a TokenPrep: the row's largest magnitude gives the power-of-two
// scale that puts it in [2^13, 2^14) (stage_row's rule, so the f16 values are the same bits), then
// every (k, k+1) pair goes to its word in the block-ordered row. Rows of up to 2048 values are
// loaded once, every load in flight together; longer rows are read twice.
__device__ void prep_row(const TokenPrep& q, int t, int lane) {
  constexpr int MAXC = 8;
  const int chunks = q.K >> 3;
  const __nv_bfloat16* row = q.x + (size_t)t * q.K;
  uint32_t* out = q.xq + (size_t)t * (q.K >> 1);
  uint4 raw[MAXC];
  float m = 0.0f;
  for (int c0 = 0; c0 < chunks; c0 += 32 * MAXC) {
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = c0 + lane + 32 * i;
      if (c < chunks) raw[i] = ldg_nc(row + c * 8);
    }
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      if (c0 + lane + 32 * i >= chunks) continue;
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b2[j]);
        m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
  m = warp_max(m);
  float inv = 1.0f, sc = 1.0f;
  if (m > 0.0f && m < __int_as_float(0x7f800000)) {
    int ex;
    frexpf(m, &ex);  // m < 2^ex
    const int sh = max(-100, min(100, ex - 14));
    sc = ldexpf(1.0f, sh);
    inv = ldexpf(1.0f, -sh);
  }
  if (lane == 0) q.scale[t] = sc;
  for (int c0 = 0; c0 < chunks; c0 += 32 * MAXC) {
    if (chunks > 32 * MAXC) {  // the row did not fit the registers: read this round again
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = c0 + lane + 32 * i;
        if (c < chunks) raw[i] = ldg_nc(row + c * 8);
      }
    }
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = c0 + lane + 32 * i;
      if (c >= chunks) continue;
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
      const int kb = c >> 2, s = (c >> 1) & 1, h = c & 1;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b2[j]);
        out[(kb * 4 + j) * 4 + s * 2 + h] = pack_f16x2(f.x * inv, f.y * inv);
      }
    }
  }
}

// The per-active-index record of expert e (called once per e < E): active index a when it has pairs,
// else one of the E - total trailing {-1, 0, 0, 0} records (e - a experts without pairs precede it).
__device__ __forceinline__ void write_act_rec(const PlanOut& o, int e, int a, int total, int off, int count) {
  if (count > 0) o.act_rec[a] = make_int4(e, o.slot_of ? o.slot_of[e] : e, off, count);
  else o.act_rec[total + (e - a)] = make_int4(-1, 0, 0, 0);
}

// Whole plan in one CTA (n_pairs <= PLAN_SINGLE_MAX); CTAs 1.. convert the token rows of `prep`
// (one warp per row) when it is given.
__global__ void __launch_bounds__(PLAN_THREADS) plan_single_kernel(const uint32_t* __restrict__ ids, int n_pairs,
                                                                    int E, PlanOut o, TokenPrep prep) {
  pdl_wait();  // ids and x (and, for the later passes, the earlier passes' output)
  pdl_trigger();
  if (blockIdx.x > 0) {
    const int t = (blockIdx.x - 1) * PLAN_WARPS + (threadIdx.x >> 5);
    if (t < prep.T) prep_row(prep, t, threadIdx.x & 31);
    return;
  }
  extern __shared__ int psm[];
  int* cnt = psm;                      // [E]
  int* base = cnt + PLAN_MAX_E;        // [E]
  int* wsum = base + PLAN_MAX_E;       // [33]
  int* whist = wsum + 64;              // [(PLAN_WARPS + 1) * E]
  for (int e = threadIdx.x; e < E; e += PLAN_THREADS) cnt[e] = 0;
  __syncthreads();
  int bad = 0;
  for (int p = threadIdx.x; p < n_pairs; p += PLAN_THREADS) {
    uint32_t id = ids[p];
    if (pair_live(id, E, o.slot_of)) atomicAdd(&cnt[id], 1);
    else if (id >= (uint32_t)E && id != MOE_ID_NONE) bad = 1;  // the sentinel is an empty slot
  }
  if (bad && o.err) atomicExch(o.err, (int)MOE_ERR_BAD_IDS);
  __syncthreads();
  // offsets (exclusive scan of counts) and the active list (scan of count > 0), E <= 1024
  int c = threadIdx.x < E ? cnt[threadIdx.x] : 0;
  int total;
  int off = block_exclusive_scan(c, wsum, &total);
  int a = block_exclusive_scan(c > 0 ? 1 : 0, wsum, &total);
  if (threadIdx.x < E) {
    o.counts[threadIdx.x] = c;
    o.offsets[threadIdx.x] = off;
    base[threadIdx.x] = off;
    if (c > 0) o.active[a] = threadIdx.x;
    if (o.act_rec) write_act_rec(o, threadIdx.x, a, total, off, c);
  }
  if (threadIdx.x == E - 1) o.offsets[E] = off + c;
  if (threadIdx.x == 0) *o.n_active = total;
  __syncthreads();
  for (int c0 = 0; c0 < n_pairs; c0 += PLAN_CHUNK) rank_chunk(ids, n_pairs, E, c0, base, whist, o.perm, o.slot_of);
}

// Large plans: per-chunk histograms -> scan -> per-chunk stable scatter.
__global__ void __launch_bounds__(PLAN_THREADS) plan_hist_kernel(const uint32_t* __restrict__ ids, int n_pairs, int E,
                                                                  int32_t* __restrict__ chunk_counts, int32_t* err,
                                                                  const int32_t* __restrict__ slot_of) {
  pdl_wait();  // ids (and, for the later passes, the earlier passes' output)
  pdl_trigger();
  extern __shared__ int psm[];
  for (int e = threadIdx.x; e < E; e += PLAN_THREADS) psm[e] = 0;
  __syncthreads();
  const int p = blockIdx.x * PLAN_CHUNK + threadIdx.x;
  if (p < n_pairs) {
    uint32_t id = ids[p];
    if (pair_live(id, E, slot_of)) atomicAdd(&psm[id], 1);
    else if (id >= (uint32_t)E && id != MOE_ID_NONE && err) atomicExch(err, (int)MOE_ERR_BAD_IDS);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += PLAN_THREADS) chunk_counts[(size_t)blockIdx.x * E + e] = psm[e];
}

__global__ void __launch_bounds__(PLAN_THREADS) plan_scan_kernel(int n_chunks, int E, int32_t* __restrict__ chunk_counts,
                                                                  PlanOut o) {
  pdl_wait();  // ids (and, for the later passes, the earlier passes' output)
  pdl_trigger();
  __shared__ int wsum[64];
  const int e = threadIdx.x;
  int total_e = 0;
  if (e < E)
    for (int c = 0; c < n_chunks; ++c) total_e += chunk_counts[(size_t)c * E + e];
  int total;
  int off = block_exclusive_scan(total_e, wsum, &total);
  int a = block_exclusive_scan(total_e > 0 ? 1 : 0, wsum, &total);
  if (e < E) {
    o.counts[e] = total_e;
    o.offsets[e] = off;
    if (total_e > 0) o.active[a] = e;
    if (o.act_rec) write_act_rec(o, e, a, total, off, total_e);
    int run = off;  // chunk bases in place
    for (int c = 0; c < n_chunks; ++c) {
      int v = chunk_counts[(size_t)c * E + e];
      chunk_counts[(size_t)c * E + e] = run;
      run += v;
    }
  }
  if (e == E - 1) o.offsets[E] = off + total_e;
  if (e == 0) *o.n_active = total;
}

__global__ void __launch_bounds__(PLAN_THREADS) plan_scatter_kernel(const uint32_t* __restrict__ ids, int n_pairs, int E,
                                                                     const int32_t* __restrict__ chunk_base,
                                                                     int32_t* __restrict__ perm,
                                                                     const int32_t* __restrict__ slot_of) {
  pdl_wait();  // ids (and, for the later passes, the earlier passes' output)
  pdl_trigger();
  extern __shared__ int psm[];
  int* base = psm;                 // [E]
  int* whist = psm + PLAN_MAX_E;   // [(PLAN_WARPS + 1) * E]
  for (int e = threadIdx.x; e < E; e += PLAN_THREADS) base[e] = chunk_base[(size_t)blockIdx.x * E + e];
  __syncthreads();
  rank_chunk(ids, n_pairs, E, blockIdx.x * PLAN_CHUNK, base, whist, perm, slot_of);
}

size_t plan_workspace_bytes(int n_pairs, int E) {
  if (n_pairs <= PLAN_SINGLE_MAX) return 0;
  return (size_t)ceil_div(n_pairs, PLAN_CHUNK) * E * sizeof(int32_t);
}

static size_t single_smem(int E) { return (size_t)(2 * PLAN_MAX_E + 64 + (PLAN_WARPS + 1) * E) * sizeof(int); }
static size_t scatter_smem(int E) { return (size_t)(PLAN_MAX_E + (PLAN_WARPS + 1) * E) * sizeof(int); }

bool plan_preps_tokens(int n_pairs) { return n_pairs <= PLAN_SINGLE_MAX; }

moe_status plan_pairs(const uint32_t* ids, int n_pairs, int E, const PlanOut& o, void* ws, size_t ws_bytes,
                      cudaStream_t st, const TokenPrep* prep) {
  if (E <= 0 || E > PLAN_MAX_E) return fail(MOE_ERR_INVALID, "moe_plan_pairs: need 0 < E <= 1024");
  if (n_pairs < 0) return fail(MOE_ERR_INVALID, "moe_plan_pairs: n_pairs < 0");
  if (!o.counts || !o.offsets || !o.perm || !o.active || !o.n_active)
    return fail(MOE_ERR_INVALID, "moe_plan_pairs: null output");
  if (n_pairs > 0 && !ids) return fail(MOE_ERR_INVALID, "moe_plan_pairs: null ids");
  if (((uintptr_t)ids | (uintptr_t)o.counts | (uintptr_t)o.offsets | (uintptr_t)o.perm | (uintptr_t)o.active |
       (uintptr_t)o.n_active | (uintptr_t)o.err) & 3)
    return fail(MOE_ERR_INVALID, "moe_plan_pairs: arrays must be 4-byte aligned");
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(plan_single_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)single_smem(PLAN_MAX_E)));
    MOE_CUDA_TRY(cudaFuncSetAttribute(plan_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)scatter_smem(PLAN_MAX_E)));
    attr_done[dev & 63] = true;
  }
  if (n_pairs <= PLAN_SINGLE_MAX) {
    TokenPrep tp{};
    int grid = 1;
    if (prep && prep->T > 0) {
      if (!prep->x || !prep->xq || !prep->scale || prep->K % 32 || ((uintptr_t)prep->x & 15))
        return fail(MOE_ERR_INVALID, "plan_pairs: bad token rows to convert");
      tp = *prep;
      grid += ceil_div(prep->T, PLAN_WARPS);
    }
    MOE_CUDA_TRY(launch_pdl(plan_single_kernel, dim3(grid), dim3(PLAN_THREADS), single_smem(E), st, ids, n_pairs, E, o,
                            tp));
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
  }
  const int n_chunks = ceil_div(n_pairs, PLAN_CHUNK);
  if (!ws || ws_bytes < plan_workspace_bytes(n_pairs, E))
    return fail(MOE_ERR_INVALID, "moe_plan_pairs: workspace too small");
  int32_t* chunk = static_cast<int32_t*>(ws);
  MOE_CUDA_TRY(launch_pdl(plan_hist_kernel, dim3(n_chunks), dim3(PLAN_THREADS), E * sizeof(int), st, ids, n_pairs, E,
                          chunk, o.err, o.slot_of));
  MOE_CUDA_TRY(cudaGetLastError());
  MOE_CUDA_TRY(launch_pdl(plan_scan_kernel, dim3(1), dim3(PLAN_THREADS), 0, st, n_chunks, E, chunk, o));
  MOE_CUDA_TRY(cudaGetLastError());
  MOE_CUDA_TRY(launch_pdl(plan_scatter_kernel, dim3(n_chunks), dim3(PLAN_THREADS), scatter_smem(E), st, ids, n_pairs,
                          E, chunk, o.perm, o.slot_of));
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

}  // namespace moe
