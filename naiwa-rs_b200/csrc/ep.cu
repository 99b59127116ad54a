// ep.cu — expert-parallel dispatch plan, row packing and combine around the per-rank MoE layer.
//
// No counterpart in the reference (one GPU plus CPU offload). The exchange itself runs over NCCL
// (ragged all-to-all of the packed rows and their (id, weight) slots, then of the per-rank
// outputs); these kernels build what it sends and fold what comes back:
//   * the dispatch plan sends each token once to every rank that owns one of its experts. Rows are
//     ordered by destination rank, then token, so a receiver sees each source's tokens in order and
//     the plan is a pure function of the ids (checked bit-exactly against the oracle's
//     ep_dispatch_plan). The slots of a row keep their positions j: ids local to the destination,
//     MOE_ID_NONE elsewhere, so the receiver's moe_forward combines the row's experts in the same j
//     order as a single-GPU forward would;
//   * the combine sums a token's per-rank outputs in rank order in f32 and rounds once to bf16.
#include "moe_internal.cuh"

namespace moe {

constexpr int EP_THREADS = 1024;
constexpr int EP_MAX_WORLD = 64;

// One CTA of 1024 threads. Pass 1 counts rows per destination rank; pass 2 walks the tokens in
// chunks of 1024 and, rank by rank, places each chunk's rows after the earlier chunks' rows by a
// block-wide exclusive scan of "token t has a row for rank r".
__global__ void __launch_bounds__(EP_THREADS) ep_plan_kernel(const uint32_t* __restrict__ ids,
                                                             const float* __restrict__ w, int T, int k, int epr,
                                                             int world, int32_t* __restrict__ rank_counts,
                                                             int32_t* __restrict__ n_send,
                                                             int32_t* __restrict__ token_rows,
                                                             int32_t* __restrict__ send_token,
                                                             uint32_t* __restrict__ send_ids,
                                                             float* __restrict__ send_w, int32_t* err) {
  __shared__ int s_cnt[EP_MAX_WORLD];
  __shared__ int s_next[EP_MAX_WORLD];  // next free row of each rank's section
  __shared__ int wsum[64];
  int bad = 0;
  for (int r = threadIdx.x; r < world; r += EP_THREADS) s_cnt[r] = 0;
  __syncthreads();
  for (int t = threadIdx.x; t < T; t += EP_THREADS) {
    uint64_t m = token_rank_mask(ids, t, k, epr, world, &bad);
    while (m) {
      const int r = __ffsll((long long)m) - 1;
      m &= m - 1;
      atomicAdd(&s_cnt[r], 1);
    }
  }
  if (bad && err) atomicExch(err, (int)MOE_ERR_BAD_IDS);
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int r = 0; r < world; ++r) {
      rank_counts[r] = s_cnt[r];
      s_next[r] = run;
      run += s_cnt[r];
    }
    *n_send = run;
  }
  __syncthreads();
  for (int c0 = 0; c0 < T; c0 += EP_THREADS) {
    const int t = c0 + threadIdx.x;
    int dummy = 0;
    const uint64_t m = t < T ? token_rank_mask(ids, t, k, epr, world, &dummy) : 0ull;
    for (int r = 0; r < world; ++r) {
      const int has = (int)((m >> r) & 1ull);
      int total;
      const int pos = block_exclusive_scan(has, wsum, &total);  // synchronises the block
      const int row = s_next[r] + pos;
      if (t < T) token_rows[(int64_t)t * world + r] = has ? row : -1;
      if (has) {
        send_token[row] = t;
        for (int j = 0; j < k; ++j) {
          const uint32_t id = ids[(int64_t)t * k + j];
          const bool mine = id != MOE_ID_NONE && id < (uint32_t)epr * (uint32_t)world && id / (uint32_t)epr == (uint32_t)r;
          send_ids[(int64_t)row * k + j] = mine ? id - (uint32_t)r * (uint32_t)epr : MOE_ID_NONE;
          send_w[(int64_t)row * k + j] = mine ? w[(int64_t)t * k + j] : 0.0f;
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) s_next[r] += total;
      __syncthreads();
    }
  }
}

// One warp per send row, 16-byte copies.
__global__ void ep_pack_kernel(const uint4* __restrict__ x, int H16, const int32_t* __restrict__ send_token,
                               const int32_t* __restrict__ n_send, uint4* __restrict__ out) {
  const int n = *n_send;
  const int lane = threadIdx.x & 31;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n; row += (gridDim.x * blockDim.x) >> 5) {
    const uint4* src = x + (int64_t)send_token[row] * H16;
    uint4* dst = out + (int64_t)row * H16;
    for (int c = lane; c < H16; c += 32) dst[c] = ldg_nc(src + c);
  }
}

// One warp per token; 8 bf16 per lane step.
__global__ void ep_combine_kernel(const uint4* __restrict__ y_back, const int32_t* __restrict__ token_rows, int T,
                                  int world, int H8, const uint4* __restrict__ y_add, uint4* __restrict__ y) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (t >= T) return;
  for (int c = lane; c < H8; c += 32) {
    float acc[8];
    if (y_add) {
      const uint4 v = ldg_nc(y_add + (int64_t)t * H8 + c);
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(b[i]);
        acc[2 * i] = f.x;
        acc[2 * i + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    }
    for (int r = 0; r < world; ++r) {
      const int row = token_rows[(int64_t)t * world + r];
      if (row < 0) continue;
      const uint4 v = ldg_nc(y_back + (int64_t)row * H8 + c);
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(b[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    y[(int64_t)t * H8 + c] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                        pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
}

// out[i] = ids[i] when its expert is in the bitmap `keep` (bit e of word e / 32), else MOE_ID_NONE.
struct ExpertSet {
  uint32_t words[32];  // E <= 1024
};

__global__ void select_ids_kernel(const uint32_t* __restrict__ ids, int64_t n, int E, ExpertSet keep,
                                  uint32_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t id = ids[i];
  out[i] = (id < (uint32_t)E && ((keep.words[id >> 5] >> (id & 31)) & 1u)) ? id : MOE_ID_NONE;
}

// y = bf16(float(y) + add), n elements.
__global__ void add_f32_into_bf16_kernel(__nv_bfloat16* __restrict__ y, const float* __restrict__ add, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2bfloat16_rn(__bfloat162float(y[i]) + add[i]);
}

}  // namespace moe

using namespace moe;

extern "C" {

moe_status moe_ep_dispatch_plan(const uint32_t* ids, const float* weights, int T, int k, int experts_per_rank,
                                int world, int32_t* rank_counts, int32_t* n_send, int32_t* token_rows,
                                int32_t* send_token, uint32_t* send_ids, float* send_weights, int32_t* error_word,
                                void* stream) {
  if (T < 0 || k <= 0 || experts_per_rank <= 0 || world <= 0 || world > EP_MAX_WORLD)
    return fail(MOE_ERR_INVALID, "moe_ep_dispatch_plan: need T >= 0, k > 0, experts_per_rank > 0, 0 < world <= 64");
  if ((int64_t)experts_per_rank * world > 0xFFFFFFF0ll) return fail(MOE_ERR_INVALID, "moe_ep_dispatch_plan: too many experts");
  if (!rank_counts || !n_send || (T > 0 && (!ids || !weights || !token_rows || !send_token || !send_ids || !send_weights)))
    return fail(MOE_ERR_INVALID, "moe_ep_dispatch_plan: null pointer");
  if (((uintptr_t)ids | (uintptr_t)weights | (uintptr_t)rank_counts | (uintptr_t)n_send | (uintptr_t)token_rows |
       (uintptr_t)send_token | (uintptr_t)send_ids | (uintptr_t)send_weights | (uintptr_t)error_word) & 3)
    return fail(MOE_ERR_INVALID, "moe_ep_dispatch_plan: arrays must be 4-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ep_plan_kernel<<<1, EP_THREADS, 0, st>>>(ids, weights, T, k, experts_per_rank, world, rank_counts, n_send,
                                           token_rows, send_token, send_ids, send_weights, error_word);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status moe_ep_pack_rows(const void* x, int T, int H, const int32_t* send_token, const int32_t* n_send, int cap,
                            void* send_x, void* stream) {
  if (T < 0 || H <= 0 || H % 8 || cap < 0) return fail(MOE_ERR_INVALID, "moe_ep_pack_rows: need H % 8 == 0");
  if (cap == 0) return MOE_OK;
  if (!x || !send_token || !n_send || !send_x) return fail(MOE_ERR_INVALID, "moe_ep_pack_rows: null pointer");
  if (((uintptr_t)x | (uintptr_t)send_x) & 15) return fail(MOE_ERR_INVALID, "moe_ep_pack_rows: rows must be 16-byte aligned");
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>(((int64_t)cap * 32 + threads - 1) / threads, 4096);
  ep_pack_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(x), H / 8, send_token, n_send, static_cast<uint4*>(send_x));
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status moe_ep_combine(const void* y_back, const int32_t* token_rows, int T, int world, int H, const void* y_add,
                          void* y, void* stream) {
  if (T < 0 || world <= 0 || H <= 0 || H % 8) return fail(MOE_ERR_INVALID, "moe_ep_combine: need H % 8 == 0");
  if (T == 0) return MOE_OK;
  if (!y_back || !token_rows || !y) return fail(MOE_ERR_INVALID, "moe_ep_combine: null pointer");
  if (((uintptr_t)y_back | (uintptr_t)y_add | (uintptr_t)y) & 15)
    return fail(MOE_ERR_INVALID, "moe_ep_combine: rows must be 16-byte aligned");
  const int threads = 256;
  const int blocks = (int)(((int64_t)T * 32 + threads - 1) / threads);
  ep_combine_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(y_back), token_rows, T, world, H / 8, static_cast<const uint4*>(y_add),
      static_cast<uint4*>(y));
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status moe_select_ids(const uint32_t* ids, int64_t n, int E, const uint32_t* experts, int n_experts,
                          uint32_t* out, void* stream) {
  if (n < 0 || E <= 0 || E > 1024 || n_experts < 0) return fail(MOE_ERR_INVALID, "moe_select_ids: need 0 < E <= 1024");
  if (n == 0) return MOE_OK;
  if (!ids || !out || (n_experts && !experts)) return fail(MOE_ERR_INVALID, "moe_select_ids: null pointer");
  ExpertSet keep{};
  for (int i = 0; i < n_experts; ++i)
    if (experts[i] < (uint32_t)E) keep.words[experts[i] >> 5] |= 1u << (experts[i] & 31);
  const int threads = 256;
  select_ids_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      ids, n, E, keep, out);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status moe_add_f32_into_bf16(void* y, const float* add, int64_t n, void* stream) {
  if (n < 0) return fail(MOE_ERR_INVALID, "moe_add_f32_into_bf16: n < 0");
  if (n == 0) return MOE_OK;
  if (!y || !add) return fail(MOE_ERR_INVALID, "moe_add_f32_into_bf16: null pointer");
  const int threads = 256;
  add_f32_into_bf16_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(y), add, n);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

}  // extern "C"
