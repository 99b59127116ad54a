// expert_decode.cu — decode-size expert FFN: gate+up+SwiGLU, down + routing weight, combine.
//
// Reference: the fork kernel mistralrs_quant::indexed_moe_fused_decode called at
// src/moe/stages/gpu.rs:27-66 (quantize x, fused gate+up GEMV + act, down GEMV + weighted
// aggregate), its per-expert fallback run_expert (gpu.rs:162-167: silu(gate x) * (up x) -> down)
// and the cross-bank sum acc + y (gpu.rs:86-92, decode.rs:371-378).
//
// Work decomposition (B200): one CTA = 8 warps works on one (active expert, chunk of ROWT row
// tiles of 16 rows). KS = 8 / ROWT warps split the K dimension of each row tile and meet in
// shared memory. Each warp streams its weight fragments straight from HBM into registers with
// 16-byte non-allocating loads: the device weight layout is fragment-native, i.e. lane l's 16
// bytes of a (16-row tile, 32-column block) are exactly its A operand for two m16n8k16 tensor-core
// MMAs, so a warp reads 512 contiguous bytes per load instruction and never reshuffles. The
// expert's tokens (up to 32 per pass) sit in shared memory in B-fragment order and are reused by
// every row tile of the CTA. Q8_0 dequantises in registers to f16 (int8 -> f16 by the 0x6400
// exponent trick, minus the 1152 bias, times the block's f16 scale); activations are staged as f16
// with a per-token power-of-two scale, so nothing overflows f16 and the scale is undone exactly
// in the epilogue. BF16 weights feed bf16 MMAs directly.
#include "moe_internal.cuh"

namespace moe {

constexpr int EXP_THREADS = 256;
constexpr int EXP_WARPS = 8;
constexpr int MAX_TPP = 32;  // tokens per pass (4 n-tiles of 8)


// ---- weight fragment decoders -----------------------------------------------------------------

struct WQ8 {
  static constexpr bool kF16 = true;
  // 512 B per (tile, block); scales: per (tile, group of 4 blocks) 8 rows x 4 blocks x {s_g, s_g+8}
  __device__ static __forceinline__ const uint8_t* qptr(const ExpertParams& p, int e, int tile, int kb, int lane) {
    return p.wq + (int64_t)e * p.q_stride + ((int64_t)tile * p.kb_count + kb) * 512 + lane * 16;
  }
  __device__ static __forceinline__ const uint8_t* sptr(const ExpertParams& p, int e, int tile, int kbg, int lane) {
    const int kbg_count = (p.kb_count + 3) >> 2;
    return p.wsc + (int64_t)e * p.s_stride + ((int64_t)tile * kbg_count + kbg) * 128 + (lane >> 2) * 16;
  }
  // q: the lane's 16 quant bytes of one block; s2: {s_g, s_g+8} of that block (f16x2)
  __device__ static __forceinline__ void decode(uint4 q, uint32_t s2, uint32_t (&a0)[4], uint32_t (&a1)[4]) {
    const __half2 sg = __half2half2(__low2half(*reinterpret_cast<__half2*>(&s2)));
    const __half2 sh = __half2half2(__high2half(*reinterpret_cast<__half2*>(&s2)));
    const __half2 bias = __float2half2_rn(1152.0f);
    uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
    uint32_t* dst[2] = {a0, a1};
#pragma unroll
    for (int s = 0; s < 2; ++s) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t word = w[2 * s + h];
        uint32_t lo = __byte_perm(word, 0x64646464u, 0x4140);  // (row g)   1024 + u
        uint32_t hi = __byte_perm(word, 0x64646464u, 0x4342);  // (row g+8) 1024 + u
        __half2 vlo = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);
        __half2 vhi = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
        vlo = __hmul2(vlo, sg);
        vhi = __hmul2(vhi, sh);
        dst[s][2 * h + 0] = *reinterpret_cast<uint32_t*>(&vlo);
        dst[s][2 * h + 1] = *reinterpret_cast<uint32_t*>(&vhi);
      }
    }
  }
};

struct WBF16 {
  static constexpr bool kF16 = false;
  // 1 KB per (tile, block): two k16 steps of 512 B, lane's 16 B = its 8 A values.
  __device__ static __forceinline__ const uint8_t* qptr(const ExpertParams& p, int e, int tile, int kb, int lane) {
    return p.wq + (int64_t)e * p.q_stride + ((int64_t)tile * p.kb_count + kb) * 1024 + lane * 16;
  }
};

// ---- staging of the pass's activations into B-fragment order ------------------------------------
// xs word index of (token n, column pair kp): per (block, n-tile) 32 lanes x 4 words.
__device__ __forceinline__ int xs_word(int n, int k, int ntm) {
  const int kb = k >> 5, kk = k & 31, s = kk >> 4, k16 = kk & 15, h = k16 >> 3, c = (k16 & 7) >> 1;
  const int nt = n >> 3, g = n & 7;
  return ((kb * ntm + nt) * 32 + g * 4 + c) * 4 + s * 2 + h;
}

template <class WT, int ROWT>
__global__ void __launch_bounds__(EXP_THREADS, 2) expert_gemv_kernel(ExpertParams p) {
  constexpr int KS = EXP_WARPS / ROWT;
  extern __shared__ __align__(16) unsigned char smem[];
  const int a_idx = blockIdx.x / p.units_per_expert;
  const int chunk = blockIdx.x % p.units_per_expert;
  if (a_idx >= *p.n_active) return;
  const int e = p.active[a_idx];
  const int base = p.offsets[e];
  const int count = p.offsets[e + 1] - base;
  const int ntm = p.tpp >> 3;
  const int K = p.K;

  uint32_t* xs = reinterpret_cast<uint32_t*>(smem);                       // K * tpp halves
  float* red = reinterpret_cast<float*>(smem + (size_t)K * p.tpp * 2);    // [KS][ROWT*16][tpp]
  float* tscale = red + (size_t)KS * ROWT * 16 * p.tpp;                   // [tpp]
  int* srow = reinterpret_cast<int*>(tscale + MAX_TPP);                   // [tpp] source row
  int* spair = srow + MAX_TPP;                                            // [tpp] original pair

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rt_local = warp / KS, ks = warp % KS;
  const int tile = chunk * ROWT + rt_local;
  const bool tile_ok = tile < p.tiles;
  const int kb_per = (p.kb_count + KS - 1) / KS;
  const int kb_begin = min(ks * kb_per, p.kb_count), kb_end = min(kb_begin + kb_per, p.kb_count);

  for (int p0 = 0; p0 < count; p0 += p.tpp) {
    const int ntok = min(p.tpp, count - p0);
    const int nt_used = (ntok + 7) >> 3;
    // token bookkeeping
    if (threadIdx.x < p.tpp) {
      int n = threadIdx.x;
      if (n < ntok) {
        int pr = p.perm[base + p0 + n];
        spair[n] = pr;
        srow[n] = p.phase == 0 ? pr / p.width : base + p0 + n;
      } else {
        spair[n] = -1;
        srow[n] = -1;
      }
    }
    __syncthreads();
    // per-token scale: f16 staging normalises each row so its max magnitude is in [2^13, 2^14)
    for (int n = warp; n < p.tpp; n += EXP_WARPS) {
      float sc = 1.0f;
      if (WT::kF16 && n < ntok) {
        float m = 0.0f;
        if (p.phase == 0) {
          const __nv_bfloat162* row = reinterpret_cast<const __nv_bfloat162*>(p.x + (int64_t)srow[n] * K);
          for (int i = lane; i < K / 2; i += 32) {
            float2 v = __bfloat1622float2(row[i]);
            m = fmaxf(m, fmaxf(fabsf(v.x), fabsf(v.y)));
          }
        } else {
          const float2* row = reinterpret_cast<const float2*>(p.h_in + (int64_t)srow[n] * K);
          for (int i = lane; i < K / 2; i += 32) {
            float2 v = row[i];
            m = fmaxf(m, fmaxf(fabsf(v.x), fabsf(v.y)));
          }
        }
        m = warp_max(m);
        if (m > 0.0f && m < __int_as_float(0x7f800000)) {
          int ex;
          frexpf(m, &ex);  // m < 2^ex
          int sh = max(-100, min(100, ex - 14));
          sc = ldexpf(1.0f, sh);
        }
      }
      if (lane == 0) tscale[n] = sc;
    }
    __syncthreads();
    // convert + scatter into B-fragment order
    const int kpairs = K >> 1;
    for (int i = threadIdx.x; i < p.tpp * kpairs; i += EXP_THREADS) {
      const int n = i / kpairs, kp = i - n * kpairs, k = kp * 2;
      uint32_t word = 0u;
      if (n < ntok) {
        float2 v;
        if (p.phase == 0) v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(p.x + (int64_t)srow[n] * K)[kp]);
        else v = reinterpret_cast<const float2*>(p.h_in + (int64_t)srow[n] * K)[kp];
        if (WT::kF16) {
          const float inv = 1.0f / tscale[n];  // exact: power of two
          word = pack_f16x2(v.x * inv, v.y * inv);
        } else {
          word = pack_bf16x2(v.x, v.y);
        }
      }
      xs[xs_word(n, k, ntm)] = word;
    }
    __syncthreads();

    // ---- tensor-core main loop ----
    float acc[MAX_TPP / 8][4];
#pragma unroll
    for (int t = 0; t < MAX_TPP / 8; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;

    if (tile_ok) {
      constexpr int U = 4;
      if constexpr (WT::kF16) {
        for (int kb0 = kb_begin; kb0 < kb_end; kb0 += U) {
          uint4 q[U];
          uint32_t s2[U];
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (kb0 + u < kb_end) q[u] = ldg_stream(WT::qptr(p, e, tile, kb0 + u, lane));
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int kb = kb0 + u;
            if (kb < kb_end) {
              const uint32_t* sp = reinterpret_cast<const uint32_t*>(WT::sptr(p, e, tile, kb >> 2, lane));
              s2[u] = __ldg(sp + (kb & 3));
            }
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int kb = kb0 + u;
            if (kb < kb_end) {
              uint32_t a0[4], a1[4];
              WT::decode(q[u], s2[u], a0, a1);
#pragma unroll
              for (int t = 0; t < MAX_TPP / 8; ++t) {
                if (t < nt_used) {
                  uint4 b = lds128(xs + ((kb * ntm + t) * 32 + lane) * 4);
                  mma_f16(acc[t], a0, b.x, b.y);
                  mma_f16(acc[t], a1, b.z, b.w);
                }
              }
            }
          }
        }
      } else {
        for (int kb0 = kb_begin; kb0 < kb_end; kb0 += U) {
          uint4 q0[U], q1[U];
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (kb0 + u < kb_end) {
              const uint8_t* ptr = WT::qptr(p, e, tile, kb0 + u, lane);
              q0[u] = ldg_stream(ptr);
              q1[u] = ldg_stream(ptr + 512);
            }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int kb = kb0 + u;
            if (kb < kb_end) {
              uint32_t a0[4] = {q0[u].x, q0[u].y, q0[u].z, q0[u].w};
              uint32_t a1[4] = {q1[u].x, q1[u].y, q1[u].z, q1[u].w};
#pragma unroll
              for (int t = 0; t < MAX_TPP / 8; ++t) {
                if (t < nt_used) {
                  uint4 b = lds128(xs + ((kb * ntm + t) * 32 + lane) * 4);
                  mma_bf16(acc[t], a0, b.x, b.y);
                  mma_bf16(acc[t], a1, b.z, b.w);
                }
              }
            }
          }
        }
      }
    }

    // ---- K-split reduction through shared memory ----
    // C fragment: c0,c1 -> (row g, tokens 2c, 2c+1); c2,c3 -> (row g+8, same tokens)
    {
      const int g = lane >> 2, c = lane & 3;
      float* r = red + ((size_t)ks * ROWT * 16 + rt_local * 16) * p.tpp;
#pragma unroll
      for (int t = 0; t < MAX_TPP / 8; ++t) {
        if (t < ntm) {
          const int n0 = t * 8 + 2 * c;
          r[g * p.tpp + n0] = acc[t][0];
          r[g * p.tpp + n0 + 1] = acc[t][1];
          r[(g + 8) * p.tpp + n0] = acc[t][2];
          r[(g + 8) * p.tpp + n0 + 1] = acc[t][3];
        }
      }
    }
    __syncthreads();

    if (p.phase == 0) {
      // h[n][col] = silu(gate) * up, col = tile*8 + r; rows 0..7 of a tile are gate, 8..15 up
      const int cols = ROWT * 8;
      const int I = p.N >> 1;
      for (int i = threadIdx.x; i < ntok * cols; i += EXP_THREADS) {
        const int n = i / cols, cl = i - n * cols;
        const int rl = cl >> 3, r = cl & 7;
        const int tl = chunk * ROWT + rl;
        if (tl >= p.tiles) continue;
        float gsum = 0.0f, usum = 0.0f;
#pragma unroll
        for (int s = 0; s < KS; ++s) {
          gsum += red[((size_t)s * ROWT * 16 + rl * 16 + r) * p.tpp + n];
          usum += red[((size_t)s * ROWT * 16 + rl * 16 + 8 + r) * p.tpp + n];
        }
        const float sc = tscale[n];
        gsum *= sc;
        usum *= sc;
        const float hval = gsum / (1.0f + __expf(-gsum)) * usum;
        p.out[(int64_t)(base + p0 + n) * I + tl * 8 + r] = hval;
      }
    } else {
      const int rows = ROWT * 16;
      for (int i = threadIdx.x; i < ntok * rows; i += EXP_THREADS) {
        const int n = i / rows, rl = i - n * rows;
        const int row = chunk * ROWT * 16 + rl;
        if (row >= p.N) continue;
        float sum = 0.0f;
#pragma unroll
        for (int s = 0; s < KS; ++s) sum += red[((size_t)s * ROWT * 16 + rl) * p.tpp + n];
        const int pr = spair[n];
        p.out[(int64_t)pr * p.N + row] = sum * tscale[n] * p.route_w[pr];
      }
    }
    __syncthreads();
  }
}

// y[t][c] = sum_j ypair[t*width + j][c] (j in order) -> bf16; pairs with a bad id are skipped.
__global__ void combine_kernel(const float* __restrict__ ypair, const uint32_t* __restrict__ ids, int T, int width,
                               int H, int E, __nv_bfloat16* __restrict__ y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one float4 per thread
  const int64_t total = (int64_t)T * H / 4;
  if (i >= total) return;
  const int t = (int)(i / (H / 4));
  const int c4 = (int)(i - (int64_t)t * (H / 4));
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < width; ++j) {
    const int pr = t * width + j;
    if (ids[pr] >= (uint32_t)E) continue;
    float4 v = reinterpret_cast<const float4*>(ypair + (int64_t)pr * H)[c4];
    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
  }
  __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
  uint2 packed = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  reinterpret_cast<uint2*>(y + (int64_t)t * H)[c4] = packed;
}

// ---- host launchers -------------------------------------------------------------------------------

int choose_tpp(int K) {
  if ((size_t)K * 32 * 2 <= 72 * 1024) return 32;
  if ((size_t)K * 16 * 2 <= 96 * 1024) return 16;
  return 8;
}

size_t expert_smem_bytes(int K, int tpp) {
  return (size_t)K * tpp * 2 + (size_t)EXP_WARPS * 16 * tpp * 4 + MAX_TPP * 4 * 3 + 64;
}

template <class WT, int ROWT>
static moe_status launch_rowt(const ExpertParams& p, int grid, size_t smem, cudaStream_t st) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(expert_gemv_kernel<WT, ROWT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      200 * 1024));
    attr[dev & 63] = true;
  }
  expert_gemv_kernel<WT, ROWT><<<grid, EXP_THREADS, smem, st>>>(p);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

// rowt: row tiles per CTA (1, 2, 4 or 8); est_active: expected active experts (grid upper bound
// is min(E, n_pairs) experts, CTAs past the real count exit at once).
moe_status launch_expert_gemv(int wdtype, ExpertParams p, int max_active, int rowt, cudaStream_t st) {
  p.units_per_expert = ceil_div(p.tiles, rowt);
  const int grid = max_active * p.units_per_expert;
  if (grid <= 0) return MOE_OK;
  const size_t smem = expert_smem_bytes(p.K, p.tpp);
  if (wdtype == MOE_DTYPE_Q8_0) {
    switch (rowt) {
      case 1: return launch_rowt<WQ8, 1>(p, grid, smem, st);
      case 2: return launch_rowt<WQ8, 2>(p, grid, smem, st);
      case 4: return launch_rowt<WQ8, 4>(p, grid, smem, st);
      default: return launch_rowt<WQ8, 8>(p, grid, smem, st);
    }
  } else if (wdtype == MOE_DTYPE_BF16) {
    switch (rowt) {
      case 1: return launch_rowt<WBF16, 1>(p, grid, smem, st);
      case 2: return launch_rowt<WBF16, 2>(p, grid, smem, st);
      case 4: return launch_rowt<WBF16, 4>(p, grid, smem, st);
      default: return launch_rowt<WBF16, 8>(p, grid, smem, st);
    }
  }
  return fail(MOE_ERR_UNSUPPORTED, "decode expert kernel: weight format not built yet");
}

moe_status launch_combine(const float* ypair, const uint32_t* ids, int T, int width, int H, int E, void* y,
                          cudaStream_t st) {
  const int64_t total = (int64_t)T * H / 4;
  if (total == 0) return MOE_OK;
  const int threads = 256;
  combine_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(
      ypair, ids, T, width, H, E, static_cast<__nv_bfloat16*>(y));
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

}  // namespace moe
