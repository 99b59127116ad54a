// expert_stream.cu — decode expert FFN over Q8_0 units as a weight stream through shared memory.
//
// Same math as the decode GEMV of expert_decode.cu (reference: indexed_moe_fused_decode,
// src/moe/stages/gpu.rs:27-66, and run_expert, gpu.rs:162-167), same per-pair results bit for bit,
// different way of moving the weights. Decode is a weight stream: at T <= 256 tokens and k = 8 of
// 128 experts each weight byte meets at most ~16 tokens, so the kernel's rate is the HBM bytes it
// keeps in flight. The register-staged GEMV holds them in registers (three groups of 2.5 KB per
// warp), which caps the warps per SM; here they sit in a shared-memory ring filled by the copy
// engine:
//
//   * persistent CTAs, one per SM, walk the work items (active expert, 128-row unit row) in turn;
//   * one producer thread copies each item's 17 KB Q8_0 units (repack.cu: the 128 rows x 128
//     columns' fragments and scales, contiguous along K) with cp.async.bulk into a ring of up to
//     eight slots, each with a full / empty mbarrier pair; the copies run ahead across items, so an
//     item's first units are in flight while the previous item's epilogue runs;
//   * eight consumer warps stage the item's tokens once into B-fragment order (f16 with a per-token
//     power-of-two scale), then per unit each warp takes its 16-row tile's four blocks of fragments
//     and scales from the slot into registers, releases the slot, and runs the m16n8k16 MMAs with
//     the f32 post-scale exactly as the GEMV does (WQ8Stream<true>::compute, blocks in K order);
//   * the epilogue is the GEMV's: SwiGLU into h (gate/up) or times the routing weight into ypair.
// Every wait is bounded: a wait that runs out records MOE_ERR_TIMEOUT in the layer's error word and
// the CTA stops; the producer still waits (bounded) for its copies in flight before the CTA exits.
#include "expert_frag.cuh"

namespace moe {

constexpr int ST_CONSUMERS = 8;  // consumer warps: one 16-row tile of a 128-row unit each
constexpr int ST_THREADS = (ST_CONSUMERS + 1) * 32;
constexpr int ST_MAX_STAGES = 8;
constexpr int ST_HEADER = 256;   // barriers and the abort flag, ahead of the ring

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// One warp stages one token row, as stage_row<true> does (same scale, same f16 values, same layout),
// but with the lane's whole share of the row loaded at once: K <= 2048 bf16 (phase 0) or K <= 1024
// f32 (phase 1) is at most 8 chunks of 8 values per lane, so every load is in flight together
// instead of one L2 round trip per chunk, twice.
__device__ __forceinline__ void stage_row_batched(const ExpertParams& p, int n, int src_row, uint32_t* xs, int ntm,
                                                  float* tscale, int lane) {
  constexpr int MAXC = 8;
  const int chunks = p.K >> 3;
  float v[MAXC][8];
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = lane + 32 * i;
    if (c < chunks) load_chunk<true>(p, src_row, c, v[i]);
  }
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i)
    if (lane + 32 * i < chunks)
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[i][j]));
  m = warp_max(m);
  float inv = 1.0f, sc = 1.0f;
  if (m > 0.0f && m < __int_as_float(0x7f800000)) {
    int ex;
    frexpf(m, &ex);  // m < 2^ex
    const int sh = max(-100, min(100, ex - 14));
    sc = ldexpf(1.0f, sh);
    inv = ldexpf(1.0f, -sh);
  }
  if (lane == 0) tscale[n] = sc;
  const int nt = n >> 3, g = n & 7;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = lane + 32 * i;
    if (c >= chunks) continue;
    const int kb = c >> 2, s = (c >> 1) & 1, h = c & 1;
    uint32_t* dst = xs + ((kb * ntm + nt) * 32 + g * 4) * 4 + s * 2 + h;
#pragma unroll
    for (int q = 0; q < 4; ++q) dst[q * 4] = pack_f16x2(v[i][2 * q] * inv, v[i][2 * q + 1] * inv);
  }
}

template <int NTM>
__global__ void __launch_bounds__(ST_THREADS, 1) expert_stream_kernel(ExpertParams p, int stages) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + ST_MAX_STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + ST_MAX_STAGES);
  unsigned char* ring = smem + ST_HEADER;
  uint32_t* xs = reinterpret_cast<uint32_t*>(ring + (size_t)stages * Q8_UNIT_BYTES);
  constexpr int TPP = NTM * 8;
  float* tscale = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(xs) + (size_t)p.K * TPP * 2);
  int* spair = reinterpret_cast<int*>(tscale + MAX_TPP);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], ST_CONSUMERS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // Gate/up follows the plan directly; the down pass follows gate/up, so the plan (two kernels back)
  // has completed and its expert list can be read before the wait, which only h needs.
  if (p.phase == 0) {
    pdl_wait();
    pdl_trigger();
  }
  const int units_k = p.K / 128;  // units along K of one 128-row unit row
  const int chunks = p.N / 128;   // unit rows per expert
  const int n_items = __ldcg(p.n_active) * chunks;
  // a contiguous, expert-major range of items per CTA: consecutive items share their expert's tokens
  const int it_begin = (int)((int64_t)n_items * blockIdx.x / gridDim.x);
  const int it_end = (int)((int64_t)n_items * (blockIdx.x + 1) / gridDim.x);

  if (warp == ST_CONSUMERS) {  // ---- producer ----
    if (lane == 0) {
      uint32_t pos = 0;
      bool ok = true;
      for (int it = it_begin; it < it_end && ok; ++it) {
        const int a = it / chunks, c = it - a * chunks;
        const int e = __ldcg(p.active + a);
        const int es = p.slot_of ? __ldcg(p.slot_of + e) : e;
        const int count = __ldcg(p.offsets + e + 1) - __ldcg(p.offsets + e);
        const int passes = (count + TPP - 1) / TPP;
        const uint8_t* src = p.wq + (int64_t)es * p.q_stride + (int64_t)c * units_k * Q8_UNIT_BYTES;
        for (int ps = 0; ps < passes && ok; ++ps)
          for (int kc = 0; kc < units_k; ++kc, ++pos) {
            const int s = (int)(pos % (uint32_t)stages);
            if (pos >= (uint32_t)stages && !mbar_wait(&empty[s], ((pos / stages) - 1) & 1, abort_flag)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&full[s], Q8_UNIT_BYTES);
            bulk_load(ring + (size_t)s * Q8_UNIT_BYTES, src + (int64_t)kc * Q8_UNIT_BYTES, Q8_UNIT_BYTES, &full[s]);
          }
      }
      if (!ok) {
        *abort_flag = 1;
        if (p.err) atomicExch(p.err, (int32_t)MOE_ERR_TIMEOUT);
      }
      // no copy may still be writing into this CTA's shared memory when it exits
      const uint32_t first = pos > (uint32_t)stages ? pos - (uint32_t)stages : 0u;
      for (uint32_t q = first; q < pos; ++q) mbar_wait(&full[q % stages], (q / stages) & 1, nullptr);
    }
    return;
  }

  // ---- consumers ----
  bool waited = p.phase == 0;
  bool ok = true;
  uint32_t pos = 0;
  const int g = lane >> 2, cq = lane & 3;
  const int frag_off = warp * 4 * 512 + ((4 * g + (cq ^ ((g >> 1) & 3))) << 4);
  const int scale_off = 8 * 4 * 512 + warp * 128 + g * 16;
  int staged_e = -1, staged_p0 = -1;  // whose tokens xs holds
  for (int it = it_begin; it < it_end && ok; ++it) {
    const int a = it / chunks, c = it - a * chunks;
    const int e = __ldcg(p.active + a);
    const int base = __ldcg(p.offsets + e);
    const int count = __ldcg(p.offsets + e + 1) - base;
    const int tile = c * 8 + warp;
    for (int p0 = 0; p0 < count && ok; p0 += TPP) {
      const int ntok = min(TPP, count - p0);
      const int nt_used = (ntok + 7) >> 3;
      if (!waited) {  // h belongs to gate/up's grid until it completes
        pdl_wait();
        pdl_trigger();
        waited = true;
      }
      if (staged_e != e || staged_p0 != p0) {
        consumers_sync();  // the previous pass's reads of xs are done
        if (threadIdx.x < TPP) spair[threadIdx.x] = threadIdx.x < ntok ? p.perm[base + p0 + threadIdx.x] : -1;
        for (int n = warp; n < ntok; n += ST_CONSUMERS) {
          const int src = p.phase == 0 ? p.perm[base + p0 + n] / p.width : base + p0 + n;
          stage_row_batched(p, n, src, xs, NTM, tscale, lane);
        }
        consumers_sync();
        staged_e = e;
        staged_p0 = p0;
      }
      float acc[NTM][4];
#pragma unroll
      for (int t = 0; t < NTM; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
      for (int kc = 0; kc < units_k; ++kc, ++pos) {
        const int s = (int)(pos % (uint32_t)stages);
        if (!mbar_wait(&full[s], (pos / stages) & 1, abort_flag)) {
          ok = false;
          break;
        }
        const unsigned char* unit = ring + (size_t)s * Q8_UNIT_BYTES;
        WQ8U::Stage st;
#pragma unroll
        for (int u = 0; u < 4; ++u) st.q[u] = lds128(unit + frag_off + u * 512);
        st.s = lds128(unit + scale_off);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // in registers now: the slot may refill
        WQ8U::template compute<NTM>(st, kc * 4, p.kb_count, xs, NTM, nt_used, lane, acc);
      }
      if (!ok) break;
      // epilogue: complete sums in registers, c0,c1 -> (row g, tokens 2c, 2c+1); c2,c3 -> (row g+8)
#pragma unroll
      for (int t = 0; t < NTM; ++t) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int n = t * 8 + 2 * cq + j;
          if (t < nt_used && n < ntok) {
            const float sc = tscale[n];
            if (p.phase == 0) {
              const float gv = acc[t][j] * sc, uv = acc[t][2 + j] * sc;
              const int I = p.N >> 1;
              p.out[(int64_t)(base + p0 + n) * I + tile * 8 + g] = gv / (1.0f + __expf(-gv)) * uv;
            } else {
              const int pr = spair[n];
              const float w = p.route_w[pr] * sc;
              float* o = p.out + (int64_t)pr * p.N + tile * 16;
              o[g] = acc[t][j] * w;
              o[g + 8] = acc[t][2 + j] * w;
            }
          }
        }
      }
    }
  }
  if (!ok) {
    *abort_flag = 1;
    if (p.err && lane == 0) atomicExch(p.err, (int32_t)MOE_ERR_TIMEOUT);
  }
}

// Shared memory of one CTA: header, `stages` 17 KB slots, the staged tokens and their scales.
static size_t stream_smem(int K, int tpp, int stages) {
  return (size_t)ST_HEADER + (size_t)stages * Q8_UNIT_BYTES + (size_t)K * tpp * 2 + MAX_TPP * 4 * 2;
}

// Ring depth for a pass: as many slots (up to eight) as fit beside the tokens in 227 KB.
int stream_stages(int K, int tpp) {
  for (int s = ST_MAX_STAGES; s >= 3; --s)
    if (stream_smem(K, tpp, s) <= 227 * 1024) return s;
  return 0;
}

template <int NTM>
static moe_status launch_stream_t(const ExpertParams& p, int grid, int stages, cudaStream_t st) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(expert_stream_kernel<NTM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      227 * 1024));
    attr[dev & 63] = true;
  }
  MOE_CUDA_TRY(launch_pdl(expert_stream_kernel<NTM>, dim3(grid), dim3(ST_THREADS), stream_smem(p.K, NTM * 8, stages),
                          st, p, stages));
  return MOE_OK;
}

// The Q8_0 unit-layout expert pass through the shared-memory stream: grid = one CTA per SM (fewer
// when there are fewer items), items = max_active experts x N / 128 unit rows (CTAs whose items run
// past the real active count stop at once).
moe_status launch_expert_stream(ExpertParams p, int max_active, int sms, cudaStream_t st) {
  if (p.K % 128 || p.N % 128) return fail(MOE_ERR_INVALID, "expert stream: Q8_0 units need 128-multiples");
  if (p.K > (p.phase == 0 ? 2048 : 1024))
    return fail(MOE_ERR_UNSUPPORTED, "expert stream: rows wider than one batched staging load");
  if (p.tpp % 8 || p.tpp < 8 || p.tpp > MAX_TPP) return fail(MOE_ERR_INVALID, "expert stream: bad tokens per pass");
  const int stages = stream_stages(p.K, p.tpp);
  if (!stages) return fail(MOE_ERR_UNSUPPORTED, "expert stream: the tokens of one pass leave no room for the ring");
  const int items = max_active * (p.N / 128);
  const int grid = items < sms ? items : sms;
  if (grid <= 0) return MOE_OK;
  switch (p.tpp) {
    case 8: return launch_stream_t<1>(p, grid, stages, st);
    case 16: return launch_stream_t<2>(p, grid, stages, st);
    case 24: return launch_stream_t<3>(p, grid, stages, st);
    default: return launch_stream_t<4>(p, grid, stages, st);
  }
}

}  // namespace moe
