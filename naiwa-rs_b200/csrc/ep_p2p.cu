// ep_p2p.cu — expert-parallel dispatch and return over NVLink peer memory (one process per GPU).
//
// No counterpart in the reference (one GPU plus CPU offload). This replaces the NCCL all-to-alls of
// moe_b200/ep.py with kernels that store rows straight into the peers' memory:
//
//   every rank owns one device allocation, shared with the other ranks by CUDA IPC handles:
//     recv_x    [W][cap][H] bf16    rows sent to me, region s written by source rank s
//     recv_ids  [W][cap][k] u32     their slots' ids, local to me (MOE_ID_NONE: not mine / no row)
//     recv_w    [W][cap][k] f32     their slots' routing weights
//     ret_y     [W][cap][H] bf16    my rows' outputs, region d written back by destination rank d
//     disp_flag [W] u64             (epoch << 32 | row count) from source s, written by s
//     ret_flag  [W] u64             (epoch << 32 | failed) from destination d, written by d
//   and, local only: recv_count [W], three last-block counters, a status word, the last epoch whose
//   receive completed and the last epoch whose combine completed.
//
//   moe_ep_peer_dispatch_routed (source, one launch): every CTA scans the routed ids [T, k] for the
//     ranks each token goes to and places (token, rank) at its position in rank r's section (tokens
//     in order: the dispatch plan of ep.cu, bit for bit); each warp then copies its tokens' rows to
//     every destination with 16-byte stores over NVLink, with the slots' local ids and weights, and
//     the CTAs fill the destinations' unused rows' ids with MOE_ID_NONE, so the destination's forward
//     reads its receive regions as they lie. Each CTA fences at system scope and counts itself done;
//     the last one publishes every destination's flag (count 0 included) with a system-scope release
//     store, then waits, bounded, for the W flags addressed to this rank and records the counts.
//   moe_ep_peer_dispatch + moe_ep_peer_receive: the same exchange from a plan built beforehand by
//     moe_ep_dispatch_plan, with the receive expanding the regions into caller arrays.
//   moe_ep_peer_return (destination): each source's rows of the local output go back into that
//     source's ret_y region [my rank]; last block publishes the return flags, with the failed bit
//     set when this epoch's receive did not complete (its rows were never computed).
//   moe_ep_peer_combine (source, one launch): every CTA waits, bounded, for all W return flags of
//     this epoch, then y[t] = y_add[t] + sum over ranks of ret_y[r][position of (t, r)], f32, rounded
//     once. A CTA whose wait ran out, or that saw a destination flag a failure, records
//     MOE_ERR_TIMEOUT in the status word and adds no returned row (y = y_add or 0). The last CTA to
//     finish marks the epoch complete.
//
// Reuse is safe without resets: a source issues epoch n + 1's dispatch only after its combine of
// epoch n, which waited for every destination's return, which each destination issued after its
// forward had read its regions; a destination's return of epoch n + 1 follows its receive of that
// epoch, which follows the source's combine of epoch n.
//
// Epochs are either given by the host (1, 2, ... identical on every rank) or, with epoch 0, held on
// the device: each call then uses the epoch after the last one whose combine completed on this
// rank, so a captured CUDA graph of a whole step can be replayed any number of times. Every wait is
// bounded (%globaltimer limit, five seconds unless moe_ep_peer_set_wait_limit changes it): one that
// runs out records MOE_ERR_TIMEOUT in the status word (moe_ep_peer_check) and the kernel returns
// without reading the regions. A failure travels with the return flag, so every rank whose rows went
// through the failed destination sees it too. No multicast: peers are reached by plain stores and
// loads through IPC mappings only.
#include <algorithm>
#include <cstring>

#include "moe_internal.cuh"

namespace moe {

constexpr int P2P_THREADS = 256;
constexpr uint64_t P2P_WAIT_NS_DEFAULT = 5ull * 1000ull * 1000ull * 1000ull;  // 5 s
constexpr int P2P_MAX_WORLD = 64;
constexpr uint64_t P2P_FLAG_FAILED = 1;  // low word of a return flag: the destination's receive failed

struct PeerLayout {
  size_t recv_x, recv_ids, recv_w, ret_y, disp_flag, ret_flag, recv_count, counters, status, recv_ok_epoch,
      done_epoch, total;
};

static PeerLayout peer_layout(int W, int cap, int H, int k) {
  PeerLayout l{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o += (bytes + 255) & ~(size_t)255;
    return at;
  };
  l.recv_x = take((size_t)W * cap * H * 2);
  l.recv_ids = take((size_t)W * cap * k * 4);
  l.recv_w = take((size_t)W * cap * k * 4);
  l.ret_y = take((size_t)W * cap * H * 2);
  l.disp_flag = take((size_t)W * 8);
  l.ret_flag = take((size_t)W * 8);
  l.recv_count = take((size_t)W * 4);
  l.counters = take(3 * 4);  // dispatch, return, combine
  l.status = take(4);
  l.recv_ok_epoch = take(4);
  l.done_epoch = take(4);
  l.total = o;
  return l;
}

struct PeerPtrs {
  unsigned char* base[P2P_MAX_WORLD];  // every rank's allocation as this rank sees it (own included)
};

__device__ __forceinline__ uint64_t p2p_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint64_t ld_acquire_sys64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// The epoch of a call: the host's, or (epoch_arg 0) the one after this rank's last completed combine,
// which every kernel of a call reads before that call's own combine advances it (same stream,
// launched in order).
__device__ __forceinline__ uint32_t call_epoch(const unsigned char* mine, const PeerLayout& L, uint32_t epoch_arg) {
  return epoch_arg ? epoch_arg : *reinterpret_cast<const volatile uint32_t*>(mine + L.done_epoch) + 1;
}

// Rank r's section of the send rows: [start[r], start[r] + counts[r]).
__device__ __forceinline__ int rank_of_row(const int* start, int W, int row) {
  int r = 0;
  while (r + 1 < W && start[r + 1] <= row) ++r;
  return r;
}

// Source: rows -> peers' recv regions; last block publishes the flags.
__global__ void __launch_bounds__(P2P_THREADS) peer_dispatch_kernel(PeerPtrs peers, PeerLayout L, int me, int W, int cap,
                                                                    int H, int k, uint32_t epoch_arg,
                                                                    const uint4* __restrict__ x,
                                                                    const int32_t* __restrict__ rank_counts,
                                                                    const int32_t* __restrict__ send_token,
                                                                    const uint32_t* __restrict__ send_ids,
                                                                    const float* __restrict__ send_w) {
  __shared__ int start[P2P_MAX_WORLD + 1];
  __shared__ int s_last;
  const uint32_t epoch = call_epoch(peers.base[me], L, epoch_arg);
  if (threadIdx.x == 0) {
    int run = 0;
    for (int r = 0; r < W; ++r) {
      start[r] = run;
      run += rank_counts[r];
    }
    start[W] = run;
  }
  __syncthreads();
  const int n = start[W];
  const int H16 = H / 8, lane = threadIdx.x & 31;
  const int warps = gridDim.x * (P2P_THREADS / 32);
  for (int row = blockIdx.x * (P2P_THREADS / 32) + (threadIdx.x >> 5); row < n; row += warps) {
    const int r = rank_of_row(start, W, row), pos = row - start[r];
    if (pos >= cap) continue;  // past the destination's region: dropped, the flag says cap, status latched
    unsigned char* dst = peers.base[r];
    uint4* dx = reinterpret_cast<uint4*>(dst + L.recv_x) + ((size_t)me * cap + pos) * H16;
    const uint4* sx = x + (size_t)send_token[row] * H16;
    for (int c = lane; c < H16; c += 32) dx[c] = ldg_nc(sx + c);
    uint32_t* di = reinterpret_cast<uint32_t*>(dst + L.recv_ids) + ((size_t)me * cap + pos) * k;
    float* dw = reinterpret_cast<float*>(dst + L.recv_w) + ((size_t)me * cap + pos) * k;
    for (int j = lane; j < k; j += 32) {
      di[j] = send_ids[(size_t)row * k + j];
      dw[j] = send_w[(size_t)row * k + j];
    }
  }
  __threadfence_system();  // this block's peer stores are visible before it counts itself done
  __syncthreads();
  uint32_t* done = reinterpret_cast<uint32_t*>(peers.base[me] + L.counters);
  if (threadIdx.x == 0) s_last = atomicAdd(&done[0], 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last) {
    __threadfence_system();
    for (int r = threadIdx.x; r < W; r += P2P_THREADS) {
      int n_r = start[r + 1] - start[r];
      if (n_r > cap) {  // a malformed plan: never publish more rows than the region holds
        n_r = cap;
        atomicExch(reinterpret_cast<int32_t*>(peers.base[me] + L.status), (int32_t)MOE_ERR_INVALID);
      }
      uint64_t* f = reinterpret_cast<uint64_t*>(peers.base[r] + L.disp_flag) + me;
      st_release_sys64(f, ((uint64_t)epoch << 32) | (uint32_t)n_r);
    }
    if (threadIdx.x == 0) done[0] = 0;  // every block has counted: ready for the next epoch
  }
}

// Waits (thread 0, bounded by wait_ns) until flags[0..W) all carry `epoch`; false after the time
// limit or, for return flags (whose low word is the failed bit; a dispatch flag's low word is its row
// count), when a flag of this epoch reports a failed receive.
__device__ bool wait_flags(const uint64_t* flags, int W, uint32_t epoch, int32_t* status, uint64_t wait_ns,
                           bool return_flags) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const uint64_t t0 = p2p_now();
    int ok = 0;
    for (;;) {
      int all = 1, failed = 0;
      for (int r = 0; r < W && all; ++r) {
        const uint64_t f = ld_acquire_sys64(flags + r);
        all = (uint32_t)(f >> 32) == epoch;
        failed |= return_flags && all && (f & P2P_FLAG_FAILED);
      }
      if (all) {
        ok = !failed;
        break;
      }
      if (p2p_now() - t0 > wait_ns) break;
      __nanosleep(128);
    }
    if (!ok) atomicExch(status, (int32_t)MOE_ERR_TIMEOUT);
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Destination: wait for every source of this epoch, then ids/weights for the local forward.
__global__ void __launch_bounds__(P2P_THREADS) peer_receive_kernel(PeerPtrs peers, PeerLayout L, int me, int W, int cap,
                                                                   int k, uint32_t epoch_arg, uint64_t wait_ns,
                                                                   uint32_t* __restrict__ ids, float* __restrict__ w) {
  unsigned char* mine = peers.base[me];
  const uint32_t epoch = call_epoch(mine, L, epoch_arg);
  const uint64_t* flags = reinterpret_cast<const uint64_t*>(mine + L.disp_flag);
  int32_t* counts = reinterpret_cast<int32_t*>(mine + L.recv_count);
  int32_t* status = reinterpret_cast<int32_t*>(mine + L.status);
  uint32_t* recv_ok = reinterpret_cast<uint32_t*>(mine + L.recv_ok_epoch);
  __shared__ int cnt[P2P_MAX_WORLD];
  if (!wait_flags(flags, W, epoch, status, wait_ns, false)) {
    // sources that did not arrive: run nothing (all slots empty), so the forward reads no region
    for (size_t i = threadIdx.x; i < (size_t)W * cap * k; i += P2P_THREADS) ids[i] = MOE_ID_NONE;
    for (int r = threadIdx.x; r < W; r += P2P_THREADS) counts[r] = 0;
    return;
  }
  for (int r = threadIdx.x; r < W; r += P2P_THREADS) {
    const int c = (int)(uint32_t)(ld_acquire_sys64(flags + r) & 0xffffffffu);
    cnt[r] = c < cap ? c : cap;  // a flag never names more rows than the region holds
    counts[r] = cnt[r];
  }
  if (threadIdx.x == 0) *recv_ok = epoch;  // read by this epoch's return (same stream, later launch)
  __syncthreads();
  const uint32_t* rid = reinterpret_cast<const uint32_t*>(mine + L.recv_ids);
  const float* rw = reinterpret_cast<const float*>(mine + L.recv_w);
  for (size_t i = threadIdx.x; i < (size_t)W * cap * k; i += P2P_THREADS) {
    const size_t row = i / k;
    const int s = (int)(row / cap), pos = (int)(row % cap);
    if (pos < cnt[s]) {  // peer-written: L2-coherent loads, no stale L1 line from an earlier epoch
      ids[i] = __ldcg(rid + i);
      w[i] = __ldcg(rw + i);
    } else {
      ids[i] = MOE_ID_NONE;
      w[i] = 0.0f;
    }
  }
}

// Tokens one CTA of the routed dispatch copies: its table of positions is [P2P_SPAN][W] in shared memory.
constexpr int P2P_SPAN = 32;

// Source, one launch for the whole exchange of a call: plan + rows + ids/weights + flags, then (last
// CTA) the receive. Every CTA scans all T tokens in chunks of P2P_THREADS with warp ballots, so each
// knows every rank's running row count; it keeps the positions of its own span of tokens
// [t0, t0 + span) and copies their rows, one warp per token (the row is read once and stored to every
// rank it goes to). Positions follow ep_plan_kernel exactly: rank r's rows are its tokens in order.
__global__ void __launch_bounds__(P2P_THREADS) peer_dispatch_routed_kernel(
    PeerPtrs peers, PeerLayout L, int me, int W, int cap, int H, int k, int epr, uint32_t epoch_arg,
    uint64_t wait_ns, const uint4* __restrict__ x, int T, const uint32_t* __restrict__ ids,
    const float* __restrict__ w, int32_t* __restrict__ rank_counts, int32_t* __restrict__ token_rows,
    int32_t* __restrict__ err) {
  constexpr int WARPS = P2P_THREADS / 32;
  __shared__ int s_total[P2P_MAX_WORLD];  // rows per destination in the chunks scanned so far
  __shared__ int s_start[P2P_MAX_WORLD];
  __shared__ int s_wcnt[WARPS][P2P_MAX_WORLD];
  __shared__ int s_pos[P2P_SPAN][P2P_MAX_WORLD];  // (token t0 + i, rank r) -> position in r's section, -1: none
  __shared__ int s_last;
  unsigned char* mine = peers.base[me];
  int32_t* status = reinterpret_cast<int32_t*>(mine + L.status);
  const uint32_t epoch = call_epoch(mine, L, epoch_arg);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int span = (T + (int)gridDim.x - 1) / (int)gridDim.x;  // the launcher keeps span <= P2P_SPAN
  const int t0 = min(T, (int)blockIdx.x * span), t1 = min(T, t0 + span);
  for (int i = threadIdx.x; i < P2P_MAX_WORLD; i += P2P_THREADS) s_total[i] = 0;
  for (int i = threadIdx.x; i < P2P_SPAN * P2P_MAX_WORLD; i += P2P_THREADS) (&s_pos[0][0])[i] = -1;
  __syncthreads();
  int bad = 0;
  const unsigned lt = (1u << lane) - 1u;
  for (int c0 = 0; c0 < T; c0 += P2P_THREADS) {
    const int t = c0 + threadIdx.x;
    const uint64_t m = t < T ? token_rank_mask(ids, t, k, epr, W, &bad) : 0ull;
    for (int r = 0; r < W; ++r) {
      const unsigned b = __ballot_sync(FULL, (m >> r) & 1ull);
      if (lane == 0) s_wcnt[warp][r] = __popc(b);
    }
    __syncthreads();
    for (int r = 0; r < W; ++r) {
      const bool has = (m >> r) & 1ull;
      const unsigned b = __ballot_sync(FULL, has);
      if (has && t >= t0 && t < t1) {
        int pos = s_total[r] + __popc(b & lt);
        for (int v = 0; v < warp; ++v) pos += s_wcnt[v][r];
        s_pos[t - t0][r] = pos;
      }
    }
    __syncthreads();
    if (threadIdx.x < W) {
      int add = 0;
      for (int v = 0; v < WARPS; ++v) add += s_wcnt[v][threadIdx.x];
      s_total[threadIdx.x] += add;
    }
    __syncthreads();
  }
  if (bad && err && blockIdx.x == 0) atomicExch(err, (int)MOE_ERR_BAD_IDS);
  if (threadIdx.x == 0) {
    int run = 0;
    for (int r = 0; r < W; ++r) {
      s_start[r] = run;
      run += s_total[r];
    }
  }
  __syncthreads();
  if (blockIdx.x == 0)
    for (int r = threadIdx.x; r < W; r += P2P_THREADS) rank_counts[r] = s_total[r];
  for (int i = threadIdx.x; i < (t1 - t0) * W; i += P2P_THREADS) {
    const int ti = i / W, r = i - ti * W;
    const int pos = s_pos[ti][r];
    token_rows[(size_t)(t0 + ti) * W + r] = pos < 0 ? -1 : s_start[r] + pos;
  }
  const int H16 = H / 8;
  for (int ti = warp; ti < t1 - t0; ti += WARPS) {
    const int t = t0 + ti;
    const uint4* sx = x + (size_t)t * H16;
    for (int c = lane; c < H16; c += 32) {
      const uint4 v = ldg_nc(sx + c);
      for (int r = 0; r < W; ++r) {
        const int pos = s_pos[ti][r];
        if (pos < 0 || pos >= cap) continue;  // past the region: dropped, the flag says cap, status latched
        reinterpret_cast<uint4*>(peers.base[r] + L.recv_x)[((size_t)me * cap + pos) * H16 + c] = v;
      }
    }
    for (int r = 0; r < W; ++r) {
      const int pos = s_pos[ti][r];
      if (pos < 0 || pos >= cap) continue;
      uint32_t* di = reinterpret_cast<uint32_t*>(peers.base[r] + L.recv_ids) + ((size_t)me * cap + pos) * k;
      float* dw = reinterpret_cast<float*>(peers.base[r] + L.recv_w) + ((size_t)me * cap + pos) * k;
      for (int j = lane; j < k; j += 32) {
        const uint32_t id = ids[(size_t)t * k + j];
        const bool here = id != MOE_ID_NONE && id < (uint32_t)epr * (uint32_t)W && id / (uint32_t)epr == (uint32_t)r;
        di[j] = here ? id - (uint32_t)r * (uint32_t)epr : MOE_ID_NONE;
        dw[j] = here ? w[(size_t)t * k + j] : 0.0f;
      }
    }
  }
  // rows past this epoch's count: no slot, so the destination's forward skips them as they lie
  for (int r = 0; r < W; ++r) {
    const int from = min(s_total[r], cap);
    uint32_t* di = reinterpret_cast<uint32_t*>(peers.base[r] + L.recv_ids) + ((size_t)me * cap + from) * k;
    const size_t n = (size_t)(cap - from) * k;
    for (size_t i = (size_t)blockIdx.x * P2P_THREADS + threadIdx.x; i < n; i += (size_t)gridDim.x * P2P_THREADS)
      di[i] = MOE_ID_NONE;
  }
  __threadfence_system();  // this block's peer stores are visible before it counts itself done
  __syncthreads();
  uint32_t* done = reinterpret_cast<uint32_t*>(mine + L.counters);
  if (threadIdx.x == 0) s_last = atomicAdd(&done[0], 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  for (int r = threadIdx.x; r < W; r += P2P_THREADS) {
    int n_r = s_total[r];
    if (n_r > cap) {  // more rows for one rank than its region holds: never publish past the region
      n_r = cap;
      atomicExch(status, (int32_t)MOE_ERR_INVALID);
    }
    st_release_sys64(reinterpret_cast<uint64_t*>(peers.base[r] + L.disp_flag) + me, ((uint64_t)epoch << 32) | (uint32_t)n_r);
  }
  if (threadIdx.x == 0) done[0] = 0;  // every block has counted: ready for the next epoch
  // the receive: every source's rows of this epoch
  const uint64_t* flags = reinterpret_cast<const uint64_t*>(mine + L.disp_flag);
  int32_t* counts = reinterpret_cast<int32_t*>(mine + L.recv_count);
  if (!wait_flags(flags, W, epoch, status, wait_ns, false)) {
    // sources that did not arrive: run nothing (every slot empty), so the forward reads no stale row
    uint32_t* rid = reinterpret_cast<uint32_t*>(mine + L.recv_ids);
    for (size_t i = threadIdx.x; i < (size_t)W * cap * k; i += P2P_THREADS) rid[i] = MOE_ID_NONE;
    for (int r = threadIdx.x; r < W; r += P2P_THREADS) counts[r] = 0;
    return;
  }
  for (int r = threadIdx.x; r < W; r += P2P_THREADS) {
    const int c = (int)(uint32_t)(ld_acquire_sys64(flags + r) & 0xffffffffu);
    counts[r] = c < cap ? c : cap;
  }
  if (threadIdx.x == 0) *reinterpret_cast<uint32_t*>(mine + L.recv_ok_epoch) = epoch;  // read by this epoch's return
}

// Destination: each source's output rows back into its ret_y region; last block publishes.
__global__ void __launch_bounds__(P2P_THREADS) peer_return_kernel(PeerPtrs peers, PeerLayout L, int me, int W, int cap,
                                                                  int H, uint32_t epoch_arg, const uint4* __restrict__ y) {
  __shared__ int s_last;
  unsigned char* mine = peers.base[me];
  const uint32_t epoch = call_epoch(mine, L, epoch_arg);
  const int32_t* counts = reinterpret_cast<const int32_t*>(mine + L.recv_count);
  const int H16 = H / 8, lane = threadIdx.x & 31;
  const int warps = gridDim.x * (P2P_THREADS / 32);
  for (int row = blockIdx.x * (P2P_THREADS / 32) + (threadIdx.x >> 5); row < W * cap; row += warps) {
    const int s = row / cap, pos = row % cap;
    if (pos >= counts[s]) continue;
    uint4* d = reinterpret_cast<uint4*>(peers.base[s] + L.ret_y) + ((size_t)me * cap + pos) * H16;
    const uint4* src = y + (size_t)row * H16;
    for (int c = lane; c < H16; c += 32) d[c] = ldg_nc(src + c);
  }
  __threadfence_system();
  __syncthreads();
  uint32_t* done = reinterpret_cast<uint32_t*>(mine + L.counters) + 1;
  if (threadIdx.x == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last) {
    __threadfence_system();
    // a receive that did not complete this epoch computed none of the sources' rows: say so
    const uint64_t failed =
        *reinterpret_cast<const volatile uint32_t*>(mine + L.recv_ok_epoch) == epoch ? 0 : P2P_FLAG_FAILED;
    for (int s = threadIdx.x; s < W; s += P2P_THREADS) {
      uint64_t* f = reinterpret_cast<uint64_t*>(peers.base[s] + L.ret_flag) + me;
      st_release_sys64(f, ((uint64_t)epoch << 32) | failed);
    }
    if (threadIdx.x == 0) *done = 0;
  }
}

// Source: y[t] = y_add[t] + sum_r ret_y[r][token_rows[t, r] - start[r]] (rows < 0 skipped); one warp
// per token. Every CTA first waits, bounded, for all W return flags of this epoch; the last CTA to
// finish advances the device-held epoch (every CTA has read it by then).
__global__ void __launch_bounds__(P2P_THREADS) peer_combine_kernel(PeerPtrs peers, PeerLayout L, int me, int W, int cap,
                                                                   int T, int H, uint32_t epoch_arg, uint64_t wait_ns,
                                                                   const int32_t* __restrict__ rank_counts,
                                                                   const int32_t* __restrict__ token_rows,
                                                                   const uint4* __restrict__ y_add,
                                                                   uint4* __restrict__ y) {
  __shared__ int start[P2P_MAX_WORLD];
  __shared__ int s_last;
  unsigned char* mine = peers.base[me];
  const uint32_t epoch = call_epoch(mine, L, epoch_arg);
  if (threadIdx.x == 0) {
    int run = 0;
    for (int r = 0; r < W; ++r) {
      start[r] = run;
      run += rank_counts[r];
    }
  }
  const bool ok = wait_flags(reinterpret_cast<const uint64_t*>(mine + L.ret_flag), W, epoch,
                             reinterpret_cast<int32_t*>(mine + L.status), wait_ns, true);  // synchronises the block
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int H8 = H / 8;
  const uint4* ret = reinterpret_cast<const uint4*>(mine + L.ret_y);
  for (int c = lane; t < T && c < H8; c += 32) {
    float acc[8];
    if (y_add) {
      const uint4 v = ldg_nc(y_add + (size_t)t * H8 + c);
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
    for (int r = 0; r < W && ok; ++r) {
      const int row = token_rows[(size_t)t * W + r];
      if (row < 0 || row - start[r] >= cap) continue;  // rows past the region were never sent
      const uint4 v = __ldcg(ret + ((size_t)r * cap + (row - start[r])) * H8 + c);  // peer-written
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(b[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    y[(size_t)t * H8 + c] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                       pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
  __syncthreads();
  uint32_t* done = reinterpret_cast<uint32_t*>(mine + L.counters) + 2;
  if (threadIdx.x == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    *done = 0;
    *reinterpret_cast<volatile uint32_t*>(mine + L.done_epoch) = epoch;  // the next device-held epoch follows it
  }
}

}  // namespace moe

using namespace moe;

struct moe_ep_peer {
  int dev = 0, rank = 0, world = 0, cap = 0, H = 0, k = 0;
  PeerLayout L{};
  unsigned char* local = nullptr;
  PeerPtrs peers{};
  bool opened[P2P_MAX_WORLD] = {};
  int grid = 0;
  uint64_t wait_ns = P2P_WAIT_NS_DEFAULT;
};

extern "C" {

moe_status moe_ep_peer_create(int device, int rank, int world, int cap_rows, int hidden, int top_k, moe_ep_peer** out) {
  if (!out) return fail(MOE_ERR_INVALID, "moe_ep_peer_create: null out");
  *out = nullptr;
  if (world < 2 || world > P2P_MAX_WORLD || rank < 0 || rank >= world || cap_rows <= 0 || hidden <= 0 ||
      hidden % 8 || top_k <= 0)
    return fail(MOE_ERR_INVALID, "moe_ep_peer_create: need 2 <= world <= 64, 0 <= rank < world, H % 8 == 0");
  DeviceGuard guard(device);
  if (!guard.ok) return fail(MOE_ERR_CUDA, "moe_ep_peer_create: cannot select device");
  moe_ep_peer* p = new moe_ep_peer();
  p->dev = device;
  p->rank = rank;
  p->world = world;
  p->cap = cap_rows;
  p->H = hidden;
  p->k = top_k;
  p->L = peer_layout(world, cap_rows, hidden, top_k);
  void* base = nullptr;
  cudaError_t e = cudaMalloc(&base, p->L.total);
  if (e != cudaSuccess) {
    delete p;
    return cuda_fail(e, "cudaMalloc(ep peer buffers)");
  }
  e = cudaMemset(base, 0, p->L.total);  // flags start at epoch 0, counters at 0
  if (e != cudaSuccess) {
    cudaFree(base);
    delete p;
    return cuda_fail(e, "cudaMemset(ep peer buffers)");
  }
  p->local = static_cast<unsigned char*>(base);
  p->peers.base[rank] = p->local;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  p->grid = sms;
  *out = p;
  return MOE_OK;
}

size_t moe_ep_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

moe_status moe_ep_peer_export(moe_ep_peer* p, void* handle) {
  if (!p || !handle) return fail(MOE_ERR_INVALID, "moe_ep_peer_export: null argument");
  DeviceGuard guard(p->dev);
  cudaIpcMemHandle_t h;
  MOE_CUDA_TRY(cudaIpcGetMemHandle(&h, p->local));
  std::memcpy(handle, &h, sizeof(h));
  return MOE_OK;
}

moe_status moe_ep_peer_connect(moe_ep_peer* p, const void* handles) {
  if (!p || !handles) return fail(MOE_ERR_INVALID, "moe_ep_peer_connect: null argument");
  DeviceGuard guard(p->dev);
  for (int r = 0; r < p->world; ++r) {
    if (r == p->rank || p->opened[r]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const unsigned char*>(handles) + (size_t)r * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    MOE_CUDA_TRY(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
    p->peers.base[r] = static_cast<unsigned char*>(ptr);
    p->opened[r] = true;
  }
  return MOE_OK;
}

void moe_ep_peer_destroy(moe_ep_peer* p) {
  if (!p) return;
  DeviceGuard guard(p->dev);
  cudaDeviceSynchronize();
  for (int r = 0; r < p->world; ++r)
    if (p->opened[r]) cudaIpcCloseMemHandle(p->peers.base[r]);
  cudaFree(p->local);
  delete p;
}

void* moe_ep_peer_recv_rows(moe_ep_peer* p) { return p ? p->local + p->L.recv_x : nullptr; }

static moe_status peer_ready(moe_ep_peer* p, const char* who) {
  if (!p) return fail(MOE_ERR_INVALID, std::string(who) + ": null peer");
  for (int r = 0; r < p->world; ++r)
    if (!p->peers.base[r]) return fail(MOE_ERR_INVALID, std::string(who) + ": call moe_ep_peer_connect first");
  return MOE_OK;
}

moe_status moe_ep_peer_dispatch(moe_ep_peer* p, const void* x, int T, const int32_t* rank_counts,
                                const int32_t* send_token, const uint32_t* send_ids, const float* send_w,
                                uint32_t epoch, void* stream) {
  MOE_TRY(peer_ready(p, "moe_ep_peer_dispatch"));
  if (T > p->cap) return fail(MOE_ERR_INVALID, "moe_ep_peer_dispatch: T exceeds cap_rows");
  DeviceGuard guard(p->dev);
  peer_dispatch_kernel<<<p->grid, P2P_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      p->peers, p->L, p->rank, p->world, p->cap, p->H, p->k, epoch, static_cast<const uint4*>(x), rank_counts,
      send_token, send_ids, send_w);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status moe_ep_peer_dispatch_routed(moe_ep_peer* p, const void* x, int T, const uint32_t* ids, const float* weights,
                                       int experts_per_rank, uint32_t epoch, int32_t* rank_counts, int32_t* token_rows,
                                       int32_t* error_word, void* stream) {
  MOE_TRY(peer_ready(p, "moe_ep_peer_dispatch_routed"));
  if (T < 0 || T > p->cap) return fail(MOE_ERR_INVALID, "moe_ep_peer_dispatch_routed: need 0 <= T <= cap_rows");
  if (experts_per_rank <= 0 || (int64_t)experts_per_rank * p->world > 0xFFFFFFF0ll)
    return fail(MOE_ERR_INVALID, "moe_ep_peer_dispatch_routed: bad experts_per_rank");
  if (!rank_counts || (T && (!x || !ids || !weights || !token_rows)))
    return fail(MOE_ERR_INVALID, "moe_ep_peer_dispatch_routed: null pointer");
  if (((uintptr_t)x & 15) ||
      (((uintptr_t)ids | (uintptr_t)weights | (uintptr_t)rank_counts | (uintptr_t)token_rows | (uintptr_t)error_word) & 3))
    return fail(MOE_ERR_INVALID, "moe_ep_peer_dispatch_routed: x must be 16-byte and the arrays 4-byte aligned");
  DeviceGuard guard(p->dev);
  // one warp per token while that fits the SMs, else at most P2P_SPAN tokens per CTA
  int grid = T ? ceil_div(T, P2P_THREADS / 32) : 1;
  if (grid > p->grid) grid = std::max(p->grid, ceil_div(T, P2P_SPAN));
  peer_dispatch_routed_kernel<<<grid, P2P_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      p->peers, p->L, p->rank, p->world, p->cap, p->H, p->k, experts_per_rank, epoch, p->wait_ns,
      static_cast<const uint4*>(x), T, ids, weights, rank_counts, token_rows, error_word);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

void* moe_ep_peer_recv_ids(moe_ep_peer* p) { return p ? p->local + p->L.recv_ids : nullptr; }
void* moe_ep_peer_recv_weights(moe_ep_peer* p) { return p ? p->local + p->L.recv_w : nullptr; }

moe_status moe_ep_peer_receive(moe_ep_peer* p, uint32_t epoch, uint32_t* ids, float* weights, void* stream) {
  MOE_TRY(peer_ready(p, "moe_ep_peer_receive"));
  if (!ids || !weights) return fail(MOE_ERR_INVALID, "moe_ep_peer_receive: null output");
  DeviceGuard guard(p->dev);
  peer_receive_kernel<<<1, P2P_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      p->peers, p->L, p->rank, p->world, p->cap, p->k, epoch, p->wait_ns, ids, weights);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status moe_ep_peer_return(moe_ep_peer* p, const void* y_local, uint32_t epoch, void* stream) {
  MOE_TRY(peer_ready(p, "moe_ep_peer_return"));
  if (!y_local) return fail(MOE_ERR_INVALID, "moe_ep_peer_return: null rows");
  DeviceGuard guard(p->dev);
  const int grid = std::min(p->grid, ceil_div(p->world * p->cap, P2P_THREADS / 32));  // one warp per row
  peer_return_kernel<<<grid, P2P_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      p->peers, p->L, p->rank, p->world, p->cap, p->H, epoch, static_cast<const uint4*>(y_local));
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status moe_ep_peer_combine(moe_ep_peer* p, uint32_t epoch, int T, const int32_t* rank_counts,
                               const int32_t* token_rows, const void* y_add, void* y, void* stream) {
  MOE_TRY(peer_ready(p, "moe_ep_peer_combine"));
  if (T < 0 || !rank_counts || (T && (!token_rows || !y))) return fail(MOE_ERR_INVALID, "moe_ep_peer_combine: bad arguments");
  DeviceGuard guard(p->dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = T ? ceil_div(T, P2P_THREADS / 32) : 1;  // one warp per token; T == 0 only waits
  peer_combine_kernel<<<grid, P2P_THREADS, 0, st>>>(p->peers, p->L, p->rank, p->world, p->cap, T, p->H, epoch,
                                                    p->wait_ns, rank_counts, token_rows,
                                                    static_cast<const uint4*>(y_add), static_cast<uint4*>(y));
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status moe_ep_peer_check(moe_ep_peer* p, void* stream) {
  if (!p) return fail(MOE_ERR_INVALID, "moe_ep_peer_check: null peer");
  DeviceGuard guard(p->dev);
  MOE_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int32_t st = 0;
  MOE_CUDA_TRY(cudaMemcpy(&st, p->local + p->L.status, 4, cudaMemcpyDeviceToHost));
  if (st != 0) {
    MOE_CUDA_TRY(cudaMemset(p->local + p->L.status, 0, 4));
    if (st == MOE_ERR_INVALID)
      return fail(MOE_ERR_INVALID, "moe_ep_peer: a dispatch plan sent more rows to one rank than cap_rows");
    return fail((moe_status)st, "moe_ep_peer: a wait for another rank ran out, or a destination reported that its "
                                "receive did (a peer stopped or fell behind)");
  }
  return MOE_OK;
}

moe_status moe_ep_peer_set_wait_limit(moe_ep_peer* p, int64_t timeout_us) {
  if (!p) return fail(MOE_ERR_INVALID, "moe_ep_peer_set_wait_limit: null peer");
  if (timeout_us <= 0) return fail(MOE_ERR_INVALID, "moe_ep_peer_set_wait_limit: the limit must be positive");
  p->wait_ns = (uint64_t)timeout_us * 1000ull;
  return MOE_OK;
}

}  // extern "C"
