// router.cu — router logits + softmax / sigmoid-group top-k.
//
// The reference computes the router in its fork's model, upstream of RoutedExperts::forward; its
// CPU copy for prediction is CachedLayer::predict (src/moe/cached_layer.rs:1236-1249) with the
// ranking rule of top_k_ids (:358-363): largest first, ties to the lowest index, f32::total_cmp.
//
// Layout of the work: a 2-D grid of (block of TB tokens) x (block of EB experts) CTAs computes the
// logits into a workspace; the CTA that finishes a token block last (threadfence + arrival
// counter, no waiting) runs the selection for those tokens. One SM never walks the whole router
// matrix alone, so the decode case (T = 1) is a handful of parallel 16-byte streams instead of a
// serial loop over 128 expert rows.
//
// Bit-exactness: every logit is a warp dot product in a fixed order (lane l owns the 8-element
// chunks l, l+32, ... and accumulates them in order with fused multiply-adds; the 32 partial sums
// meet in an xor butterfly 16,8,4,2,1), which the oracle restates operation for operation.
// Selection is a warp argmax over 64-bit keys (total-order value, then lowest index), so ids are
// exact; weights use det_exp and IEEE-rounded division and are exact as well.
#include <cstdlib>

#include "moe_internal.cuh"

namespace moe {

constexpr int ROUTER_THREADS = 256;
constexpr int ROUTER_WARPS = ROUTER_THREADS / 32;
constexpr int ROUTER_EB = 8;  // experts per CTA (one per warp: twice the CTAs of two per warp, and each
                               // warp's row loads are one HBM round trip at decode sizes)
constexpr int ROUTER_LOADS = 8;  // 16-byte router-row loads in flight per lane (a whole H = 2048 row)
constexpr int ROUTER_MAX_E = 1024;

// Warp argmax over candidates not yet taken: the winning index (largest total-order key, ties to
// the lowest index) or -1 when no candidate is left.
__device__ __forceinline__ int warp_argmax(const float* vals, int n, const uint32_t* taken_bits, int lane) {
  unsigned long long best = 0ull;
  for (int i = lane; i < n; i += 32) {
    if (taken_bits[i >> 5] & (1u << (i & 31))) continue;
    unsigned long long key = ((unsigned long long)total_key_u(vals[i]) << 32) | (uint32_t)(~(uint32_t)i);
    best = key > best ? key : best;
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    unsigned long long other = __shfl_xor_sync(FULL, best, o);
    best = other > best ? other : best;
  }
  if (best == 0ull) return -1;
  return (int)(~(uint32_t)(best & 0xffffffffull));
}

// Selection for one token by one warp. l: the token's E logits (shared, overwritten in sigmoid
// mode), a: E floats of shared scratch, tk: E bits of shared scratch.
__device__ void select_token(const RouteParams& p, float* l, float* a, uint32_t* tk, int t, int lane) {
  const int E = p.E;
  for (int i = lane; i < (E + 31) / 32; i += 32) tk[i] = 0u;
  __syncwarp();
  uint32_t* out_ids = p.ids + (size_t)t * p.k;
  float* out_w = p.weights + (size_t)t * p.k;
  if (p.mode == MOE_ROUTER_SOFTMAX || p.mode == MOE_ROUTER_SOFTMAX_RENORM) {
    int first = -1;
    for (int j = 0; j < p.k; ++j) {
      int id = warp_argmax(l, E, tk, lane);
      if (lane == 0) {
        tk[id >> 5] |= 1u << (id & 31);
        out_ids[j] = (uint32_t)id;
        a[j] = __int_as_float(id);  // ids kept in shared for the weight pass
      }
      __syncwarp();
      if (j == 0) first = id;
    }
    __syncwarp();
    const float m = l[first];
    if (p.mode == MOE_ROUTER_SOFTMAX) {
      float s = 0.0f;
      for (int e = lane; e < E; e += 32) s = __fadd_rn(s, det_exp(__fsub_rn(l[e], m)));
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(FULL, s, o));
      if (lane == 0)
        for (int j = 0; j < p.k; ++j) out_w[j] = __fdiv_rn(det_exp(__fsub_rn(l[__float_as_int(a[j])], m)), s);
    } else if (lane == 0) {
      float z = 0.0f;
      for (int j = 0; j < p.k; ++j) {
        const float ex = det_exp(__fsub_rn(l[__float_as_int(a[j])], m));
        a[32 + j] = ex;
        z = __fadd_rn(z, ex);
      }
      for (int j = 0; j < p.k; ++j) out_w[j] = __fdiv_rn(a[32 + j], z);
    }
  } else {  // MOE_ROUTER_SIGMOID_GROUP
    float* s = a;    // sigmoid scores
    float* sel = l;  // selection scores overwrite the logits
    for (int e = lane; e < E; e += 32) s[e] = det_sigmoid(l[e]);
    __syncwarp();
    for (int e = lane; e < E; e += 32) sel[e] = p.bias ? __fadd_rn(s[e], p.bias[e]) : s[e];
    __syncwarp();
    const int gs = E / p.n_group;
    // group score = top-1 + top-2 selection score of the group (lane g owns group g)
    float gscore = 0.0f;
    if (lane < p.n_group) {
      uint32_t b1 = 0, b2 = 0;
      float v1 = 0.0f, v2 = 0.0f;
      int have = 0;
      for (int i = 0; i < gs; ++i) {
        float v = sel[lane * gs + i];
        uint32_t kv = total_key_u(v);
        if (have == 0 || kv > b1) {
          if (have) { b2 = b1; v2 = v1; }
          b1 = kv; v1 = v;
          have = have < 2 ? have + 1 : 2;
        } else if (have == 1 || kv > b2) {
          b2 = kv; v2 = v;
          have = 2;
        }
      }
      gscore = have == 2 ? __fadd_rn(v1, v2) : v1;
    }
    uint32_t group_kept = 0u;
    for (int r = 0; r < p.topk_group; ++r) {
      unsigned long long key = 0ull;
      if (lane < p.n_group && !(group_kept & (1u << lane)))
        key = ((unsigned long long)total_key_u(gscore) << 32) | (uint32_t)(~(uint32_t)lane);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(FULL, key, o);
        key = other > key ? other : key;
      }
      group_kept |= 1u << (int)(~(uint32_t)(key & 0xffffffffull));
    }
    // experts outside the kept groups are marked taken so the argmax skips them
    for (int e = lane; e < E; e += 32)
      if (!(group_kept & (1u << (e / gs)))) atomicOr(&tk[e >> 5], 1u << (e & 31));
    __syncwarp();
    for (int j = 0; j < p.k; ++j) {
      int id = warp_argmax(sel, E, tk, lane);
      if (lane == 0) {
        tk[id >> 5] |= 1u << (id & 31);
        out_ids[j] = (uint32_t)id;
      }
      __syncwarp();
    }
    if (lane == 0) {
      float z = 0.0f;
      for (int j = 0; j < p.k; ++j) z = __fadd_rn(z, s[out_ids[j]]);
      z = __fadd_rn(z, 1e-20f);
      for (int j = 0; j < p.k; ++j) out_w[j] = __fmul_rn(__fdiv_rn(s[out_ids[j]], z), p.routed_scale);
    }
  }
  __syncwarp();
}

// grid (ceil(T/TB), ceil(E/EB)); ws_logits [T, E] f32; the arrival counter of token block b is
// ws_count_end[-1 - b], the end of the workspace counting down: its address does not depend on T, so
// a workspace reused with another T keeps every counter at zero between calls (at the front, after
// the logits, a shorter call's counters would land on a longer call's logits)
// EW experts per warp (EB = 8 EW per CTA). EW = 1: tokens staged as bf16 and converted at each use
// (latency-bound small batches, most CTAs). EW = 2 (TB >= 4): the block's tokens staged once as f32
// in two float4 planes per token (xf[t][q][c] = elements 4q..4q+3 of chunk c, so a warp's loads are
// conflict-free) and each warp's two router rows applied to every staged token, which halves the
// conversions and shared-memory reads per multiply-add. Every logit sees the same operations in the
// same order either way.
template <int TB, int EW>
__global__ void __launch_bounds__(ROUTER_THREADS) route_kernel(RouteParams p, float* __restrict__ ws_logits,
                                                               unsigned* __restrict__ ws_count_end) {
  constexpr int EB = ROUTER_EB * EW;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_last;
  const int H = p.H, E = p.E;
  const int t0 = blockIdx.x * TB;
  const int nt = min(TB, p.T - t0);
  const int e0 = blockIdx.y * EB;
  const int chunks = H / 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint4* xs = reinterpret_cast<uint4*>(smem);  // EW = 1: [TB][H/8] bf16 chunks
  float4* xf = reinterpret_cast<float4*>(smem);  // EW = 2: [TB][2][H/8]
  pdl_wait();  // x may come from the kernel before
  pdl_trigger();

  for (int i = threadIdx.x; i < TB * chunks; i += ROUTER_THREADS) {
    const int t = i / chunks, c = i - t * chunks;
    const uint4 v = t < nt ? ldg_nc(p.x + (size_t)(t0 + t) * H + c * 8) : make_uint4(0, 0, 0, 0);
    if constexpr (EW == 1) {
      xs[i] = v;
    } else {
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
      const float2 a = __bfloat1622float2(h2[0]), b = __bfloat1622float2(h2[1]);
      const float2 cc = __bfloat1622float2(h2[2]), d = __bfloat1622float2(h2[3]);
      xf[(t * 2) * chunks + c] = make_float4(a.x, a.y, b.x, b.y);
      xf[(t * 2 + 1) * chunks + c] = make_float4(cc.x, cc.y, d.x, d.y);
    }
  }
  __syncthreads();

  if constexpr (EW == 2) {
    constexpr int LOADS = ROUTER_LOADS / 2;
    const int ea = e0 + 2 * warp, eb = ea + 1;
    if (ea < E) {
      const bool has_b = eb < E;
      const __nv_bfloat16* wa = p.w + (size_t)ea * H;
      const __nv_bfloat16* wb = p.w + (size_t)(has_b ? eb : ea) * H;
      float acc[2][TB];
#pragma unroll
      for (int t = 0; t < TB; ++t) acc[0][t] = acc[1][t] = 0.0f;
      for (int c0 = lane; c0 < chunks; c0 += LOADS * 32) {
        uint4 va[LOADS], vb[LOADS];
#pragma unroll
        for (int u = 0; u < LOADS; ++u)
          if (c0 + 32 * u < chunks) {
            va[u] = ldg_nc(wa + (c0 + 32 * u) * 8);
            vb[u] = ldg_nc(wb + (c0 + 32 * u) * 8);
          }
#pragma unroll
        for (int u = 0; u < LOADS; ++u) {
          const int c = c0 + 32 * u;
          if (c >= chunks) break;
          float fa[8], fb[8];
          const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&va[u]);
          const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&vb[u]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 x = __bfloat1622float2(a2[j]), y = __bfloat1622float2(b2[j]);
            fa[2 * j] = x.x;
            fa[2 * j + 1] = x.y;
            fb[2 * j] = y.x;
            fb[2 * j + 1] = y.y;
          }
#pragma unroll
          for (int t = 0; t < TB; ++t) {
            const float4 x0 = xf[(t * 2) * chunks + c], x1 = xf[(t * 2 + 1) * chunks + c];
            const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              acc[0][t] = __fmaf_rn(xv[j], fa[j], acc[0][t]);
              acc[1][t] = __fmaf_rn(xv[j], fb[j], acc[1][t]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
#pragma unroll
        for (int t = 0; t < TB; ++t) {
          float v = acc[r][t];
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(FULL, v, o));
          if (lane == 0 && t < nt && (r == 0 || has_b)) ws_logits[(size_t)(t0 + t) * E + (r ? eb : ea)] = v;
        }
      }
    }
  }

  // EW = 1: each warp owns expert e0 + warp; chunk loads are issued ROUTER_LOADS at a time
  for (int e = e0 + warp; EW == 1 && e < min(E, e0 + EB); e += ROUTER_WARPS) {
    float acc[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) acc[t] = 0.0f;
    const __nv_bfloat16* wr = p.w + (size_t)e * H;
    for (int c0 = lane; c0 < chunks; c0 += ROUTER_LOADS * 32) {
      uint4 wv[ROUTER_LOADS];
#pragma unroll
      for (int u = 0; u < ROUTER_LOADS; ++u)
        if (c0 + 32 * u < chunks) wv[u] = ldg_nc(wr + (c0 + 32 * u) * 8);
#pragma unroll
      for (int u = 0; u < ROUTER_LOADS; ++u) {
        const int c = c0 + 32 * u;
        if (c >= chunks) break;
        const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv[u]);
#pragma unroll
        for (int t = 0; t < TB; ++t) {
          uint4 xv = xs[t * chunks + c];
          const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 xf = __bfloat1622float2(x2[j]);
            const float2 wf = __bfloat1622float2(w2[j]);
            acc[t] = __fmaf_rn(xf.x, wf.x, acc[t]);
            acc[t] = __fmaf_rn(xf.y, wf.y, acc[t]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < TB; ++t) {
      float v = acc[t];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(FULL, v, o));
      if (lane == 0 && t < nt) ws_logits[(size_t)(t0 + t) * E + e] = v;
    }
  }

  // arrival: the last CTA of this token block selects
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&ws_count_end[-1 - (int)blockIdx.x], 1u);
    s_last = prev == gridDim.y - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* lg = reinterpret_cast<float*>(smem);  // reuse: [TB][E] logits
  float* aux = lg + (size_t)TB * E;            // [TB][max(E, 64)]
  const int auxw = E > 64 ? E : 64;
  uint32_t* taken = reinterpret_cast<uint32_t*>(aux + (size_t)TB * auxw);
  for (int i = threadIdx.x; i < nt * E; i += ROUTER_THREADS) lg[i] = __ldcg(ws_logits + (size_t)t0 * E + i);
  __syncthreads();
  for (int t = warp; t < nt; t += ROUTER_WARPS)
    select_token(p, lg + t * E, aux + t * auxw, taken + t * ((E + 31) / 32), t0 + t, lane);
  if (threadIdx.x == 0) ws_count_end[-1 - (int)blockIdx.x] = 0u;  // ready for the next call on this stream
}

static size_t route_smem(int TB, int EW, int H, int E) {
  const size_t stage = (size_t)TB * H * (EW == 2 ? 4 : 2);
  const size_t select = (size_t)TB * E * 4 + (size_t)TB * (E > 64 ? E : 64) * 4 + (size_t)TB * ((E + 31) / 32) * 4;
  return stage > select ? stage : select;
}

size_t route_workspace_bytes(int T, int E) {
  const size_t logits = ((size_t)T * E * 4 + 255) / 256 * 256;
  return logits + (size_t)(T > 0 ? T : 1) * 4;
}

template <int TB, int EW>
static moe_status launch_route(const RouteParams& p, float* logits, unsigned* counts, cudaStream_t st) {
  const size_t sm = route_smem(TB, EW, p.H, p.E);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(route_kernel<TB, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set[dev & 63] = true;
  }
  dim3 grid(ceil_div(p.T, TB), ceil_div(p.E, ROUTER_EB * EW));
  MOE_CUDA_TRY(launch_pdl(route_kernel<TB, EW>, grid, dim3(ROUTER_THREADS), sm, st, p, logits, counts));
  return MOE_OK;
}

// MOE_ROUTER_NARROW=1 keeps one expert per warp at every batch size (for comparison).
static bool route_narrow() {
  static const bool on = [] {
    const char* v = std::getenv("MOE_ROUTER_NARROW");
    return v && v[0] == '1';
  }();
  return on;
}

moe_status route_validate(const RouteParams& p) {
  if (p.T < 0 || p.H <= 0 || p.E <= 0 || p.k <= 0 || p.k > p.E || p.k > 32)
    return fail(MOE_ERR_INVALID, "moe_route: need T >= 0, 0 < k <= min(E, 32)");
  if (p.H % 8 != 0) return fail(MOE_ERR_INVALID, "moe_route: hidden must be a multiple of 8");
  if (p.E > ROUTER_MAX_E) return fail(MOE_ERR_INVALID, "moe_route: at most 1024 experts");
  if (p.mode < 0 || p.mode > 2) return fail(MOE_ERR_INVALID, "moe_route: unknown router mode");
  if (p.mode == MOE_ROUTER_SIGMOID_GROUP) {
    if (p.n_group <= 0 || p.n_group > 32 || p.E % p.n_group != 0 || p.topk_group <= 0 || p.topk_group > p.n_group)
      return fail(MOE_ERR_INVALID,
                  "moe_route: sigmoid-group routing needs 0 < topk_group <= n_group <= 32, E % n_group == 0");
    if (p.k > p.topk_group * (p.E / p.n_group))
      return fail(MOE_ERR_INVALID, "moe_route: k exceeds the experts of the kept groups");
  }
  if (!p.x || !p.w || !p.ids || !p.weights) return fail(MOE_ERR_INVALID, "moe_route: null pointer");
  if (((uintptr_t)p.x | (uintptr_t)p.w) & 15)
    return fail(MOE_ERR_INVALID, "moe_route: x and router weight must be 16-byte aligned");
  if (((uintptr_t)p.ids | (uintptr_t)p.weights | (uintptr_t)p.bias) & 3)
    return fail(MOE_ERR_INVALID, "moe_route: ids, weights and bias must be 4-byte aligned");
  return MOE_OK;
}

moe_status route_tokens(const RouteParams& p, void* ws, size_t ws_bytes, cudaStream_t st) {
  MOE_TRY(route_validate(p));
  if (p.T == 0) return MOE_OK;
  if (!ws || ws_bytes < route_workspace_bytes(p.T, p.E) || ((uintptr_t)ws & 15))
    return fail(MOE_ERR_INVALID,
                "moe_route: workspace missing, misaligned or smaller than moe_route_workspace_bytes");
  float* logits = static_cast<float*>(ws);
  // counters count down from the (4-byte aligned) end: T-independent addresses past every logit
  unsigned* counts = reinterpret_cast<unsigned*>(static_cast<char*>(ws) + (ws_bytes & ~(size_t)3));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // tokens per CTA: share each router-row load across tokens once the grid is wide enough
  const int eblocks = ceil_div(p.E, ROUTER_EB);
  int TB = 1;
  if ((int64_t)p.T * eblocks >= 16LL * sms) TB = 8;
  else if ((int64_t)p.T * eblocks >= 8LL * sms) TB = 4;
  else if ((int64_t)p.T * eblocks >= 4LL * sms) TB = 2;
  // large batches (4 or more tokens per CTA) take two experts per warp on f32-staged tokens
  const bool wide = TB >= 4 && route_smem(TB, 2, p.H, p.E) <= 200 * 1024 && !route_narrow();
  while (TB > 1 && route_smem(TB, 1, p.H, p.E) > 200 * 1024) TB >>= 1;
  if (route_smem(TB, 1, p.H, p.E) > 200 * 1024) return fail(MOE_ERR_INVALID, "moe_route: hidden too large");
  if (wide) return TB == 8 ? launch_route<8, 2>(p, logits, counts, st) : launch_route<4, 2>(p, logits, counts, st);
  switch (TB) {
    case 8: return launch_route<8, 1>(p, logits, counts, st);
    case 4: return launch_route<4, 1>(p, logits, counts, st);
    case 2: return launch_route<2, 1>(p, logits, counts, st);
    default: return launch_route<1, 1>(p, logits, counts, st);
  }
}

}  // namespace moe
