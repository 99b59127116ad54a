// expert_decode.cu — decode-size expert FFN: gate+up+SwiGLU, down + routing weight, combine.
//
// Reference: the fork kernel mistralrs_quant::indexed_moe_fused_decode called at
// src/moe/stages/gpu.rs:27-66 (quantize x, fused gate+up GEMV + act, down GEMV + weighted
// aggregate), its per-expert fallback run_expert (gpu.rs:162-167: silu(gate x) * (up x) -> down)
// and the cross-bank sum acc + y (gpu.rs:86-92, decode.rs:371-378).
//
// Work decomposition (B200): one CTA = 8 warps works on one (active expert, chunk of ROWT row
// tiles of 16 rows). KS = 8 / ROWT warps split the K dimension of each row tile and meet in
// shared memory (KS = 1 keeps everything in registers). Each warp streams its weight fragments
// straight from HBM into registers with 16-byte non-allocating loads, three groups of four
// 32-column blocks in flight: the device weight layout is fragment-native, i.e. lane l's 16 bytes
// of a (16-row tile, 32-column block) are exactly its A operand for two m16n8k16 tensor-core MMAs,
// so a warp reads 512 contiguous bytes per load instruction and never reshuffles. The expert's
// tokens (up to 32 per pass) are staged once per CTA into shared memory in B-fragment order, one
// warp per token row with 16-byte loads, and reused by every row tile of the CTA.
//
// Precision: Q8_0 quants enter the MMA as exact f16 integers (int8 -> f16 through the 0x6400
// exponent trick minus the 1152 bias) and each block's f16 scale is applied in f32 to the MMA
// partial sum, so the weights are never rounded. Activations are staged as f16 with a per-token
// power-of-two scale (a bf16 value scaled into f16's range is exact); the scale is undone in the
// epilogue. BF16 weights feed bf16 MMAs with bf16 activations unchanged.
#include <type_traits>

#include "expert_frag.cuh"

namespace moe {

// PH: the pass (0 gate/up, 1 down) fixed at compile time, or -1 to read p.phase. Q8_0 units compile
// one kernel per pass, so each carries only its own token staging: gate/up copies rows converted
// by the plan launch (stage_prepped), down loads its f32 rows in one batch (stage_row_f32_batched).
template <class WT, int ROWT, int NTM, int WARPS, int PH>
__global__ void __launch_bounds__(WARPS * 32, 16 / WARPS) expert_gemv_kernel(ExpertParams p) {
  const int phase = PH >= 0 ? PH : p.phase;
  constexpr int KS = WARPS / ROWT;
  constexpr int THREADS = WARPS * 32;
  constexpr int STAGES = 3;
  constexpr int G = WT::GROUP;
  extern __shared__ __align__(16) unsigned char smem[];
  const int a_idx = blockIdx.x / p.units_per_expert;
  const int chunk = blockIdx.x % p.units_per_expert;
  // Gate/up follows the plan directly: wait for it. Down follows gate/up, so the plan (two kernels
  // back) has completed when it starts: it reads the plan's outputs through L2 and issues its first
  // weight loads before waiting for gate/up's h.
  if (phase == 0) {
    pdl_wait();
    pdl_trigger();
  }
  int e, es, base, count;  // es: the expert's weight slot
  if (p.act_rec) {  // one 16-byte load of the plan's record for this active index
    const int4 r = __ldcg(p.act_rec + a_idx);
    if (r.x < 0) return;
    e = r.x;
    es = r.y;
    base = r.z;
    count = r.w;
  } else {
    if (a_idx >= __ldcg(p.n_active)) return;
    e = __ldcg(p.active + a_idx);
    es = p.slot_of ? __ldcg(p.slot_of + e) : e;
    base = __ldcg(p.offsets + e);
    count = __ldcg(p.offsets + e + 1) - base;
  }
  (void)e;
  // a record that names a slot or a pair range outside the buffers latches an error and is skipped
  if (es < 0 || (p.n_wslots > 0 && es >= p.n_wslots) || base < 0 || count <= 0 || base + count > p.n_pairs) {
    if (threadIdx.x == 0 && p.err) atomicExch(p.err, (int)MOE_ERR_INVALID);
    return;
  }
  const int ntm = NTM;
  const int tpp = NTM * 8;
  const int K = p.K;

  uint32_t* xs = reinterpret_cast<uint32_t*>(smem);                      // K * tpp halves
  float* red = reinterpret_cast<float*>(smem + (size_t)K * tpp * 2);     // [KS][ROWT*16][tpp] (KS > 1)
  float* tscale = red + (KS > 1 ? (size_t)KS * ROWT * 16 * tpp : 0);     // [tpp]
  int* spair = reinterpret_cast<int*>(tscale + MAX_TPP);                 // [tpp] original pair

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rt_local = warp / KS, ks = warp % KS;
  const int tile = chunk * ROWT + rt_local;
  const bool tile_ok = tile < p.tiles;
  // K range of this warp: whole groups (a scale load always covers its group), balanced to within one
  const int groups = (p.kb_count + G - 1) / G;
  const int kb_begin = min(groups * ks / KS * G, p.kb_count);
  const int kb_end = min(groups * (ks + 1) / KS * G, p.kb_count);

  for (int p0 = 0; p0 < count; p0 += tpp) {
    const int ntok = min(tpp, count - p0);
    const int nt_used = (ntok + 7) >> 3;
    // first weight groups go out before the staging so HBM latency overlaps it
    typename WT::Stage st[STAGES];
    if (tile_ok) {
      WT::load(p, es, tile, kb_begin, kb_end, lane, st[0]);
      WT::load(p, es, tile, kb_begin + G, kb_end, lane, st[1]);
    }
    if (phase == 1 && p0 == 0) {  // h and the ypair rows belong to gate/up's grid until it completes
      pdl_wait();
      pdl_trigger();
    }
    if (threadIdx.x < tpp) {
      int pr = threadIdx.x < ntok ? p.perm[base + p0 + threadIdx.x] : -1;
      if (pr >= p.n_pairs || (threadIdx.x < ntok && pr < 0)) {  // outside the call's pairs: skipped, latched
        if (p.err) atomicExch(p.err, (int)MOE_ERR_INVALID);
        pr = -1;
      }
      spair[threadIdx.x] = pr;
    }
    __syncthreads();
    for (int n = warp; n < ntok; n += WARPS) {
      if (phase == 0 && spair[n] < 0) continue;
      const int src = phase == 0 ? spair[n] / p.width : base + p0 + n;
      if constexpr (PH == 0) {
        if (p.xq) stage_prepped(p, n, src, xs, ntm, tscale, lane);
        else stage_row<WT::kF16>(p, n, src, xs, ntm, tscale, lane);
      } else if constexpr (PH == 1) {
        if (p.K <= 1024) stage_row_f32_batched(p, n, src, xs, ntm, tscale, lane);
        else stage_row<WT::kF16>(p, n, src, xs, ntm, tscale, lane);
      } else {
        stage_row<WT::kF16>(p, n, src, xs, ntm, tscale, lane);
      }
    }
    if (PH == 0 && p.xq) cp_async_wait_all();
    __syncthreads();

    float acc[NTM][4];
#pragma unroll
    for (int t = 0; t < NTM; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
    if (tile_ok) {
      for (int kb0 = kb_begin; kb0 < kb_end; kb0 += STAGES * G) {
        WT::load(p, es, tile, kb0 + 2 * G, kb_end, lane, st[2]);
        WT::template compute<NTM>(st[0], kb0, kb_end, xs, ntm, nt_used, lane, acc);
        WT::load(p, es, tile, kb0 + 3 * G, kb_end, lane, st[0]);
        WT::template compute<NTM>(st[1], kb0 + G, kb_end, xs, ntm, nt_used, lane, acc);
        WT::load(p, es, tile, kb0 + 4 * G, kb_end, lane, st[1]);
        WT::template compute<NTM>(st[2], kb0 + 2 * G, kb_end, xs, ntm, nt_used, lane, acc);
      }
    }

    const int g = lane >> 2, c = lane & 3;
    if constexpr (KS == 1) {
      // complete sums in registers: c0,c1 -> (row g, tokens 2c, 2c+1); c2,c3 -> (row g+8, same)
      if (tile_ok) {
#pragma unroll
        for (int t = 0; t < NTM; ++t) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int n = t * 8 + 2 * c + j;
            if (t < nt_used && n < ntok) {
              const float sc = tscale[n];
              if (phase == 0) {
                const float gv = acc[t][j] * sc, uv = acc[t][2 + j] * sc;
                const int I = p.N >> 1;
                p.out[(int64_t)(base + p0 + n) * I + tile * 8 + g] = gv / (1.0f + __expf(-gv)) * uv;
              } else {
                const int pr = spair[n];
                if (pr < 0) continue;
                const float w = p.route_w[pr] * sc;
                float* o = p.out + (int64_t)pr * p.N + tile * 16;
                o[g] = acc[t][j] * w;
                o[g + 8] = acc[t][2 + j] * w;
              }
            }
          }
        }
      }
    } else {
      float* r = red + ((size_t)ks * ROWT * 16 + rt_local * 16) * tpp;
#pragma unroll
      for (int t = 0; t < NTM; ++t) {
        const int n0 = t * 8 + 2 * c;
        r[g * tpp + n0] = acc[t][0];
        r[g * tpp + n0 + 1] = acc[t][1];
        r[(g + 8) * tpp + n0] = acc[t][2];
        r[(g + 8) * tpp + n0 + 1] = acc[t][3];
      }
      __syncthreads();
      if (phase == 0) {
        const int cols = ROWT * 8;
        const int I = p.N >> 1;
        for (int i = threadIdx.x; i < ntok * cols; i += THREADS) {
          const int n = i / cols, cl = i - n * cols;
          const int rl = cl >> 3, rr = cl & 7;
          const int tl = chunk * ROWT + rl;
          if (tl >= p.tiles) continue;
          float gsum = 0.0f, usum = 0.0f;
#pragma unroll
          for (int s = 0; s < KS; ++s) {
            gsum += red[((size_t)s * ROWT * 16 + rl * 16 + rr) * tpp + n];
            usum += red[((size_t)s * ROWT * 16 + rl * 16 + 8 + rr) * tpp + n];
          }
          const float sc = tscale[n];
          gsum *= sc;
          usum *= sc;
          p.out[(int64_t)(base + p0 + n) * I + tl * 8 + rr] = gsum / (1.0f + __expf(-gsum)) * usum;
        }
      } else {
        const int rows = ROWT * 16;
        for (int i = threadIdx.x; i < ntok * rows; i += THREADS) {
          const int n = i / rows, rl = i - n * rows;
          const int row = chunk * ROWT * 16 + rl;
          if (row >= p.N) continue;
          float sum = 0.0f;
#pragma unroll
          for (int s = 0; s < KS; ++s) sum += red[((size_t)s * ROWT * 16 + rl) * tpp + n];
          const int pr = spair[n];
          if (pr < 0) continue;
          p.out[(int64_t)pr * p.N + row] = sum * tscale[n] * p.route_w[pr];
        }
      }
    }
    __syncthreads();
  }
}

// y[t][c] = sum_j ypair[t*width + j][c] (j in order) -> bf16; pairs with a bad id are skipped.
__global__ void combine_kernel(const float* __restrict__ ypair, const uint32_t* __restrict__ ids, int T, int width,
                               int H, int E, __nv_bfloat16* __restrict__ y, const int32_t* __restrict__ slot_of) {
  pdl_wait();  // ypair from the down projection
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one float4 per thread
  const int64_t total = (int64_t)T * H / 4;
  if (i >= total) return;
  const int t = (int)(i / (H / 4));
  const int c4 = (int)(i - (int64_t)t * (H / 4));
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < width; ++j) {
    const int pr = t * width + j;
    if (!pair_live(ids[pr], E, slot_of)) continue;
    float4 v = reinterpret_cast<const float4*>(ypair + (int64_t)pr * H)[c4];
    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
  }
  __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
  uint2 packed = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  reinterpret_cast<uint2*>(y + (int64_t)t * H)[c4] = packed;
}

// ---- host launchers -------------------------------------------------------------------------------

// Tokens per pass: enough n-tiles for the expected busiest expert (mean + 3 sd of a binomial
// count), within a shared-memory budget.
int choose_tpp(int K, double mean_tokens_per_expert) {
  const double m = mean_tokens_per_expert;
  const double want = m + 3.0 * sqrt(m > 0 ? m : 0) + 1.0;
  int tpp = want <= 8 ? 8 : want <= 16 ? 16 : want <= 24 ? 24 : 32;
  while (tpp > 8 && (size_t)K * tpp * 2 > 132 * 1024) tpp -= 8;
  return tpp;
}

size_t expert_smem_bytes(int K, int tpp, int rowt, int warps) {
  const int ks = warps / rowt;
  return (size_t)K * tpp * 2 + (ks > 1 ? (size_t)warps * 16 * tpp * 4 : 0) + MAX_TPP * 4 * 2 + 64;
}

template <class WT, int ROWT, int NTM, int WARPS, int PH>
static moe_status launch4(const ExpertParams& p, int grid, size_t smem, cudaStream_t st) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(expert_gemv_kernel<WT, ROWT, NTM, WARPS, PH>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr[dev & 63] = true;
  }
  MOE_CUDA_TRY(launch_pdl(expert_gemv_kernel<WT, ROWT, NTM, WARPS, PH>, dim3(grid), dim3(WARPS * 32), smem, st, p));
  return MOE_OK;
}

template <class WT, int ROWT, int NTM, int WARPS>
static moe_status launch3(const ExpertParams& p, int grid, size_t smem, cudaStream_t st) {
  if constexpr (std::is_same<WT, WQ8U>::value) {
    if (p.phase == 0) return launch4<WT, ROWT, NTM, WARPS, 0>(p, grid, smem, st);
    return launch4<WT, ROWT, NTM, WARPS, 1>(p, grid, smem, st);
  }
  return launch4<WT, ROWT, NTM, WARPS, -1>(p, grid, smem, st);
}

template <class WT, int ROWT, int WARPS>
static moe_status launch2(const ExpertParams& p, int grid, size_t smem, cudaStream_t st) {
  switch (p.tpp) {
    case 8: return launch3<WT, ROWT, 1, WARPS>(p, grid, smem, st);
    case 16: return launch3<WT, ROWT, 2, WARPS>(p, grid, smem, st);
    case 24: return launch3<WT, ROWT, 3, WARPS>(p, grid, smem, st);
    default: return launch3<WT, ROWT, 4, WARPS>(p, grid, smem, st);
  }
}

template <class WT>
static moe_status launch1(const ExpertParams& p, int grid, size_t smem, int rowt, cudaStream_t st) {
  switch (rowt) {
    case 1: return launch2<WT, 1, 8>(p, grid, smem, st);
    case 2: return launch2<WT, 2, 8>(p, grid, smem, st);
    case 4: return launch2<WT, 4, 8>(p, grid, smem, st);
    case 8: return launch2<WT, 8, 8>(p, grid, smem, st);
    default: return launch2<WT, 16, 16>(p, grid, smem, st);
  }
}

// rowt: row tiles per CTA (1, 2, 4 or 8 with 8 warps; 16 with 16 warps, one tile per warp). The
// grid covers min(E, n_pairs) experts; CTAs past the real count of active experts exit at once.
moe_status launch_expert_gemv(int wdtype, ExpertParams p, int max_active, int rowt, cudaStream_t st) {
  if (p.tpp % 8 || p.tpp < 8 || p.tpp > MAX_TPP) return fail(MOE_ERR_INVALID, "expert kernel: bad tokens per pass");
  if (p.K > 4096) return fail(MOE_ERR_UNSUPPORTED, "decode expert kernel: K > 4096");
  if (rowt != 1 && rowt != 2 && rowt != 4 && rowt != 8 && rowt != 16)
    return fail(MOE_ERR_INVALID, "expert kernel: bad row tiles per CTA");
  p.units_per_expert = ceil_div(p.tiles, rowt);
  const int grid = max_active * p.units_per_expert;
  if (grid <= 0) return MOE_OK;
  const size_t smem = expert_smem_bytes(p.K, p.tpp, rowt, rowt == 16 ? 16 : 8);
  if (wdtype == MOE_DTYPE_Q8_0 && p.tile_major) {
    if (p.K % 128 || p.N % 128) return fail(MOE_ERR_INVALID, "decode expert kernel: Q8_0 units need 128-multiples");
    return launch1<WQ8U>(p, grid, smem, rowt, st);
  }
  if (wdtype == MOE_DTYPE_Q8_0) return launch1<WQ8>(p, grid, smem, rowt, st);
  if (wdtype == MOE_DTYPE_BF16) return launch1<WBF16>(p, grid, smem, rowt, st);
  if (wdtype == MOE_DTYPE_Q2_0) {
    if (p.K % 128) return fail(MOE_ERR_INVALID, "decode expert kernel: Q2_0 needs K % 128 == 0");
    return launch1<WQ2>(p, grid, smem, rowt, st);
  }
  return fail(MOE_ERR_UNSUPPORTED, "decode expert kernel: weight format not built yet");
}

moe_status launch_combine(const float* ypair, const uint32_t* ids, int T, int width, int H, int E, void* y,
                          cudaStream_t st, const int32_t* slot_of) {
  const int64_t total = (int64_t)T * H / 4;
  if (total == 0) return MOE_OK;
  const int threads = 256;
  MOE_CUDA_TRY(launch_pdl(combine_kernel, dim3((unsigned)((total + threads - 1) / threads)), dim3(threads), 0, st,
                          ypair, ids, T, width, H, E, static_cast<__nv_bfloat16*>(y), slot_of));
  return MOE_OK;
}

}  // namespace moe
