// expert_frag.cuh — the decode expert kernels' shared pieces: the Q8_0 / BF16 weight-fragment
// streams (device layout -> m16n8k16 A operands, exact int8 -> f16, per-block f32 scales) and the
// token staging into B-fragment order, used by expert_decode.cu (register-staged GEMV) and
// expert_stream.cu (shared-memory weight stream). Both compute a pair's sums in the same order, so
// they give the same bits.
#pragma once
#include "moe_internal.cuh"

namespace moe {

constexpr int MAX_TPP = 32;  // tokens per pass (4 n-tiles of 8)

// ---- weight fragment streams ---------------------------------------------------------------------

// Q8_0: per (tile, block) 512 B of quants; per (tile, group of 4 blocks) 128 B of scales holding
// {d(row g), d(row g+8)} for the 4 blocks at byte g*16. UNITS: the same fragments grouped in 17 KB
// units per (128-row tile, 128-column chunk), lane l's slot swizzled (repack.cu), scales inside the
// unit; a pipeline stage (4 blocks) is then one unit of the warp's 16-row tile.
template <bool UNITS>
struct WQ8Stream {
  static constexpr bool kF16 = true;
  static constexpr int GROUP = 4;  // blocks per pipeline stage
  struct Stage {
    uint4 q[GROUP];
    uint4 s;
  };
  __device__ static __forceinline__ void load(const ExpertParams& p, int e, int tile, int kb0, int kb_end, int lane,
                                              Stage& st) {
    const uint8_t* qb;
    const uint8_t* sb;
    if (UNITS) {  // kb0 % 4 == 0: blocks kb0 .. kb0 + 3 are the unit's four blocks
      const int g = lane >> 2, c = lane & 3;
      const uint8_t* unit =
          p.wq + (int64_t)e * p.q_stride + ((int64_t)(tile >> 3) * (p.kb_count >> 2) + (kb0 >> 2)) * Q8_UNIT_BYTES;
      qb = unit + (tile & 7) * 4 * 512 + ((4 * g + (c ^ ((g >> 1) & 3))) << 4);
      sb = unit + 8 * 4 * 512 + (tile & 7) * 128 + g * 16;
    } else {
      qb = p.wq + (int64_t)e * p.q_stride + ((int64_t)tile * p.kb_count + kb0) * 512 + lane * 16;
      const int kbg_count = (p.kb_count + 3) >> 2;
      sb = p.wsc + (int64_t)e * p.s_stride + ((int64_t)tile * kbg_count + (kb0 >> 2)) * 128 + (lane >> 2) * 16;
    }
#pragma unroll
    for (int u = 0; u < GROUP; ++u)
      if (kb0 + u < kb_end) st.q[u] = ldg_stream(qb + u * 512);
    if (kb0 < kb_end) st.s = ldg_stream(sb);
  }
  // exact int8 -> f16 of the lane's 16 quant bytes: a0 (k16 step 0), a1 (step 1). The device layout
  // stores u = q + 128 (the repack flips the sign bit), so 0x64 in the high byte makes 1024 + u.
  __device__ static __forceinline__ void quants(uint4 q, uint32_t (&a0)[4], uint32_t (&a1)[4]) {
    const __half2 bias = __float2half2_rn(1152.0f);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      uint32_t* dst = s ? a1 : a0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t lo = __byte_perm(w[2 * s + h], 0x64646464u, 0x4140);  // row g:   1024 + u
        uint32_t hi = __byte_perm(w[2 * s + h], 0x64646464u, 0x4342);  // row g+8: 1024 + u
        __half2 vlo = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);
        __half2 vhi = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
        dst[2 * h + 0] = *reinterpret_cast<uint32_t*>(&vlo);
        dst[2 * h + 1] = *reinterpret_cast<uint32_t*>(&vhi);
      }
    }
  }
  template <int NTM>
  __device__ static __forceinline__ void compute(const Stage& st, int kb0, int kb_end, const uint32_t* xs, int ntm,
                                                 int nt_used, int lane, float (&acc)[NTM][4]) {
    const uint32_t sw[4] = {st.s.x, st.s.y, st.s.z, st.s.w};
#pragma unroll
    for (int u = 0; u < GROUP; ++u) {
      const int kb = kb0 + u;
      if (kb >= kb_end) break;
      uint32_t a0[4], a1[4];
      quants(st.q[u], a0, a1);
      const __half2 s2 = *reinterpret_cast<const __half2*>(&sw[u]);
      const float slo = __low2float(s2), shi = __high2float(s2);
#pragma unroll
      for (int t = 0; t < NTM; ++t) {
        if (t < nt_used) {
          uint4 b = lds128(xs + ((kb * ntm + t) * 32 + lane) * 4);
          float tmp[4];
          mma_f16_zero(tmp, a0, b.x, b.y);
          mma_f16(tmp, a1, b.z, b.w);
          ffma2(acc[t][0], acc[t][1], slo, tmp[0], tmp[1]);
          ffma2(acc[t][2], acc[t][3], shi, tmp[2], tmp[3]);
        }
      }
    }
  }
};

// Q2_0 (repack.cu): per (tile, 128-column group) a lane's 16 B of codes (word w = the group's k16 steps
// 2w, 2w + 1) and 8 B of scales {d(g), d(g+8)} for the group's two 64-column blocks. A pair of codes
// becomes an exact f16x2 of (code - 1) by one shift, one mask-or (1024 + code) and one subtract of
// 1025; a block's four k16 MMAs chain in f32 and its scale is applied once in f32 afterwards.
struct WQ2 {
  static constexpr bool kF16 = true;
  static constexpr int GROUP = 4;  // 32-column blocks per stage: one 128-column group
  struct Stage {
    uint4 q;
    uint2 s;
  };
  __device__ static __forceinline__ void load(const ExpertParams& p, int e, int tile, int kb0, int kb_end, int lane,
                                              Stage& st) {
    if (kb0 >= kb_end) return;
    const int64_t grp = (int64_t)tile * (p.kb_count >> 2) + (kb0 >> 2);
    st.q = ldg_stream(p.wq + (int64_t)e * p.q_stride + grp * 512 + lane * 16);
    const uint2* sp = reinterpret_cast<const uint2*>(p.wsc + (int64_t)e * p.s_stride + grp * 64 + (lane >> 2) * 8);
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(st.s.x), "=r"(st.s.y) : "l"(sp));
  }
  template <int NTM>
  __device__ static __forceinline__ void compute(const Stage& st, int kb0, int kb_end, const uint32_t* xs, int ntm,
                                                 int nt_used, int lane, float (&acc)[NTM][4]) {
    const uint32_t w[4] = {st.q.x, st.q.y, st.q.z, st.q.w};
    const uint32_t sw[2] = {st.s.x, st.s.y};
    const __half2 bias = __float2half2_rn(1025.0f);
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      const int kb = kb0 + 2 * blk;  // the block's first 32-column block of the staged tokens
      if (kb >= kb_end) break;
      uint32_t a[4][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int sg = 4 * blk + s;  // k16 step within the group
        const uint32_t word = w[sg >> 1];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t v = ((word >> (2 * ((sg & 1) * 4 + q))) & 0x00030003u) | 0x64006400u;  // 1024 + code
          __half2 h = __hsub2(*reinterpret_cast<__half2*>(&v), bias);                     // code - 1
          a[s][q] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      const __half2 s2 = *reinterpret_cast<const __half2*>(&sw[blk]);
      const float slo = __low2float(s2), shi = __high2float(s2);
#pragma unroll
      for (int t = 0; t < NTM; ++t) {
        if (t < nt_used) {
          const uint4 b0 = lds128(xs + ((kb * ntm + t) * 32 + lane) * 4);
          const uint4 b1 = lds128(xs + (((kb + 1) * ntm + t) * 32 + lane) * 4);
          float tmp[4];
          mma_f16_zero(tmp, a[0], b0.x, b0.y);
          mma_f16(tmp, a[1], b0.z, b0.w);
          mma_f16(tmp, a[2], b1.x, b1.y);
          mma_f16(tmp, a[3], b1.z, b1.w);
          ffma2(acc[t][0], acc[t][1], slo, tmp[0], tmp[1]);
          ffma2(acc[t][2], acc[t][3], shi, tmp[2], tmp[3]);
        }
      }
    }
  }
};

// BF16: per (tile, block) 1 KB = two k16 steps of 512 B; lane's 16 B = its 8 A values.
using WQ8 = WQ8Stream<false>;
using WQ8U = WQ8Stream<true>;

struct WBF16 {
  static constexpr bool kF16 = false;
  static constexpr int GROUP = 2;
  struct Stage {
    uint4 q[GROUP][2];
  };
  __device__ static __forceinline__ void load(const ExpertParams& p, int e, int tile, int kb0, int kb_end, int lane,
                                              Stage& st) {
    const uint8_t* qb = p.wq + (int64_t)e * p.q_stride + ((int64_t)tile * p.kb_count + kb0) * 1024 + lane * 16;
#pragma unroll
    for (int u = 0; u < GROUP; ++u)
      if (kb0 + u < kb_end) {
        st.q[u][0] = ldg_stream(qb + u * 1024);
        st.q[u][1] = ldg_stream(qb + u * 1024 + 512);
      }
  }
  template <int NTM>
  __device__ static __forceinline__ void compute(const Stage& st, int kb0, int kb_end, const uint32_t* xs, int ntm,
                                                 int nt_used, int lane, float (&acc)[NTM][4]) {
#pragma unroll
    for (int u = 0; u < GROUP; ++u) {
      const int kb = kb0 + u;
      if (kb >= kb_end) break;
      const uint32_t a0[4] = {st.q[u][0].x, st.q[u][0].y, st.q[u][0].z, st.q[u][0].w};
      const uint32_t a1[4] = {st.q[u][1].x, st.q[u][1].y, st.q[u][1].z, st.q[u][1].w};
#pragma unroll
      for (int t = 0; t < NTM; ++t) {
        if (t < nt_used) {
          uint4 b = lds128(xs + ((kb * ntm + t) * 32 + lane) * 4);
          mma_bf16(acc[t], a0, b.x, b.y);
          mma_bf16(acc[t], a1, b.z, b.w);
        }
      }
    }
  }
};

// ---- staging ------------------------------------------------------------------------------------
// SMEM layout of the pass's activations: word ((kb * ntm + nt) * 32 + g * 4 + c) * 4 + s * 2 + h
// holds the (k, k+1) pair k = 32 kb + 16 s + 8 h + 2 c of token 8 nt + g: the B operand of
// m16n8k16 for lane 4g + c is then one 16-byte load {step0 b0b1, step0 b2b3, step1 b0b1, step1 b2b3}.
template <bool F16>
__device__ __forceinline__ void load_chunk(const ExpertParams& p, int src_row, int c, float (&v)[8]) {
  if (p.phase == 0) {
    uint4 raw = ldg_nc(p.x + (int64_t)src_row * p.K + c * 8);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(b2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float4* src = reinterpret_cast<const float4*>(p.h_in + (int64_t)src_row * p.K + c * 8);
    float4 f0 = src[0], f1 = src[1];
    v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
    v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
  }
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// One warp stages one token row converted beforehand (TokenPrep, plan.cu): the row's 16-byte pieces
// go straight to their B-fragment slots by asynchronous copies, all in flight together, and the
// row's scale is the one the conversion picked. The caller waits (cp_async_wait_all) and syncs.
__device__ __forceinline__ void stage_prepped(const ExpertParams& p, int n, int src_row, uint32_t* xs, int ntm,
                                              float* tscale, int lane) {
  const int pieces = p.K >> 3;  // per 32-column block four pieces of 16 bytes
  const uint4* srow = reinterpret_cast<const uint4*>(p.xq) + (size_t)src_row * pieces;
  const int nt = n >> 3, g = n & 7;
  for (int i = lane; i < pieces; i += 32) {
    const int kb = i >> 2, c = i & 3;
    cp_async16(xs + ((kb * ntm + nt) * 32 + g * 4 + c) * 4, srow + i);
  }
  if (lane == 0) tscale[n] = p.xq_scale[src_row];
}

// One warp stages one f32 row of at most 1024 values (the down pass's h) exactly as stage_row<true>
// does (same scale, same f16 values, same layout), with the lane's whole share loaded at once
// instead of one L2 round trip per chunk, twice.
__device__ __forceinline__ void stage_row_f32_batched(const ExpertParams& p, int n, int src_row, uint32_t* xs,
                                                      int ntm, float* tscale, int lane) {
  constexpr int MAXC = 4;
  const int chunks = p.K >> 3;
  float4 v[MAXC][2];
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = lane + 32 * i;
    if (c < chunks) {
      const float4* src = reinterpret_cast<const float4*>(p.h_in + (int64_t)src_row * p.K + c * 8);
      v[i][0] = src[0];
      v[i][1] = src[1];
    }
  }
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i)
    if (lane + 32 * i < chunks)
      m = fmaxf(fmaxf(fmaxf(m, fmaxf(fabsf(v[i][0].x), fabsf(v[i][0].y))), fmaxf(fabsf(v[i][0].z), fabsf(v[i][0].w))),
                fmaxf(fmaxf(fabsf(v[i][1].x), fabsf(v[i][1].y)), fmaxf(fabsf(v[i][1].z), fabsf(v[i][1].w))));
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
    dst[0] = pack_f16x2(v[i][0].x * inv, v[i][0].y * inv);
    dst[4] = pack_f16x2(v[i][0].z * inv, v[i][0].w * inv);
    dst[8] = pack_f16x2(v[i][1].x * inv, v[i][1].y * inv);
    dst[12] = pack_f16x2(v[i][1].z * inv, v[i][1].w * inv);
  }
}

// One warp stages one token row: (f16 path) the row's max magnitude gives a power-of-two scale
// that puts the row in [2^13, 2^14); the second sweep re-reads the row (L1/L2 hit), converts and
// scatters it into B-fragment order.
template <bool F16>
__device__ __forceinline__ void stage_row(const ExpertParams& p, int n, int src_row, uint32_t* xs, int ntm,
                                          float* tscale, int lane) {
  const int chunks = p.K >> 3;  // 8 elements per chunk
  float inv = 1.0f, sc = 1.0f;
  if (F16) {
    float m = 0.0f;
    for (int c = lane; c < chunks; c += 32) {
      float v[8];
      load_chunk<F16>(p, src_row, c, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
    }
    m = warp_max(m);
    if (m > 0.0f && m < __int_as_float(0x7f800000)) {
      int ex;
      frexpf(m, &ex);  // m < 2^ex
      const int sh = max(-100, min(100, ex - 14));
      sc = ldexpf(1.0f, sh);
      inv = ldexpf(1.0f, -sh);
    }
  }
  if (lane == 0) tscale[n] = sc;
  const int nt = n >> 3, g = n & 7;
  for (int c = lane; c < chunks; c += 32) {
    float v[8];
    load_chunk<F16>(p, src_row, c, v);
    const int kb = c >> 2, s = (c >> 1) & 1, h = c & 1;
    uint32_t* dst = xs + ((kb * ntm + nt) * 32 + g * 4) * 4 + s * 2 + h;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      dst[q * 4] = F16 ? pack_f16x2(v[2 * q] * inv, v[2 * q + 1] * inv) : pack_bf16x2(v[2 * q], v[2 * q + 1]);
  }
}

}  // namespace moe
