// expert_gemm_tc.cu — grouped expert GEMM on the 5th-generation tensor cores: prefill-size
// batches (Q4_K / FP8 / Q8_0) and decode batches of 4 or more tokens per expert (Q8_0).
//
// Reference: the fork's grouped MoE kernels behind MoEExperts::forward, driven by
// PrefillStream::dispatch (src/moe/prefill_stream.rs:1178-1216) and forward_batched (:2080-2102),
// with the expert math of run_expert (src/moe/stages/gpu.rs:162-167).
//
// A work item is one (expert, 128-row weight tile, <= BN-token tile) block of
//   gate/up:  H[tok, n] = SwiGLU over the tile's 64 gate and 64 up rows of X_e W^T
//   down:     Ypair[pair, n] = w_pair * (h_e W^T)[tok, n]
// computed as D[128 x N] (TMEM, f32) = A[128 x K] (weights, TMEM) * B[K x N] (tokens, shared memory)
// with tcgen05.mma kind::f16. The kernel is persistent (one or two CTAs per SM walking the items)
// and warp-specialised. Per 128-column K chunk:
//   * the token tile arrives by 2-D TMA loads (64 columns x 32 rows per box, SWIZZLE_128B) from the
//     gathered, f16-converted activations;
//   * the weight tile streams into a shared-memory ring by 1-D bulk copies; 8 or 16 warps dequantise
//     it (Q4_K: nibble -> f16 by the 0x6400 exponent trick, then d*sc*q - dmin*m in f16; FP8 e4m3:
//     cvt to f16 times the 128x128 block scale; Q8_0: byte -> f16 by the same trick, times the block
//     scale) and write the f16 operand straight into tensor memory with tcgen05.st, so the
//     dequantised weights never touch shared memory;
//   * one thread issues 8 MMAs (K = 16 each).
// With two accumulators the epilogue of one item overlaps the main loop of the next; with one, the
// CTA's other resident CTA covers it. Every wait is bounded: a wait that runs out sets
// MOE_ERR_TIMEOUT in the error word, the CTA stops issuing work, waits (bounded) for its own MMAs,
// frees its TMEM and returns.
//
// Weight layouts in HBM (tile-major, built by the repack kernels below):
//   FP8:  per (expert, 128-row tile, 128-column chunk) 16 KB of e4m3, rows of 128 B with 16-byte
//         chunk j of row r stored at j ^ (r % 8); the
//         128x128 block scale of that chunk in a separate f32 array.
//   Q4_K: per (expert, 128-row tile, 256-column super-block) the 128 rows' quant bytes (16 KB, same
//         chunk swizzle) and
//         their per-sub-block f16 pairs {d*sc, -dmin*m} (4 KB), precomputed at repack.
//   Q8_0: the decode GEMV's 17 KB units of m16n8k16 fragments (repack.cu); the dequant threads
//         gather their row's bytes from them.
// Gate/up tiles hold, per 16-row group, 8 gate rows then the 8 up rows of the same columns, so one
// warp holds a gate value and its up partner after tcgen05.ld (SwiGLU by one shuffle), and a 16-row
// MMA fragment of the decode GEMV holds 8 gate/up pairs.
#include <cuda.h>

#include <cstdlib>
#include <string>

#include "moe_internal.cuh"

namespace moe {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 128;
constexpr int A_COLS = BK / 2;        // tensor-memory columns of one dequantised weight stage
constexpr int EPI_WARPS = 4;

// Kernel shapes. Warps 0 .. DQW-1 dequantise, DQW issues MMAs, DQW+1 streams weight units, DQW+2
// streams token tiles, DQW+4 .. DQW+7 run the epilogue (tensor-memory lane quarter = warp % 4).
// Tensor memory: NACC f32 accumulators at columns [a BN, (a + 1) BN) (lane = weight row), used by
// successive work items in turn; stage s of the dequantised f16 weights at columns
// A_COL0 + 64 s .. +63 (lane = weight row, two K values per 32-bit column), the operand layout
// tcgen05.mma reads for A from tensor memory. One commit per chunk frees its weight stage and its
// token stage together, so both rings have STG stages.
//   Wide:  one CTA per SM, 16 dequant warps, 4 stages, 2 accumulators (epilogue of one item
//          overlaps the main loop of the next), 512 columns.
//   Pair:  two CTAs per SM, 8 dequant warps each, 2 stages, 1 accumulator, 256 columns: two MMA
//          issuers and two dequant pipelines per SM, each CTA's epilogue overlapping the other's
//          main loop.
//   Decode: see below.
// The dequant warps form DQG groups of DQW / DQG warps; group g takes the chunks q with
// q % DQG == g, each group covering all 128 rows (one warp per lane quarter) and the 4 column
// quarters of its chunks. One group per CTA works chunk by chunk in lockstep (the chunk's latency
// chain: ring read, convert, tcgen05.st, wait, hand-off); several groups keep as many chunks in
// flight.
template <int DQW_, int STG_, int NACC_, int RING_, int CTAS_, int BN_, int DQG_ = 1>
struct GemmShape {
  static constexpr int BN = BN_;                // tokens per work item (accumulator columns)
  static constexpr int B_BYTES = BN_ * BK * 2;  // one stage of f16 tokens
  static constexpr int DQW = DQW_;
  static constexpr int DQG = DQG_;
  static constexpr int WG = DQW_ / DQG_;   // warps per dequant group
  static constexpr int QPW = 16 / WG;      // 32-column quarters of a chunk each dequant thread covers
  static constexpr int STG = STG_;
  static constexpr int NACC = NACC_;
  static constexpr int RING = RING_;
  static constexpr int CTAS_PER_SM = CTAS_;
  static constexpr int MMA_WARP = DQW_;
  static constexpr int WLOAD_WARP = DQW_ + 1;
  static constexpr int TLOAD_WARP = DQW_ + 2;
  static constexpr int EPI_WARP0 = DQW_ + 4;
  static constexpr int THREADS = (DQW_ + 4 + EPI_WARPS) * 32;
  static constexpr int A_COL0 = NACC_ * BN_;
  static constexpr int TMEM_COLS = (A_COL0 + STG_ * A_COLS) <= 256 ? 256 : 512;
  static_assert(A_COL0 + STG_ * A_COLS <= TMEM_COLS, "tensor memory budget");
  static_assert(TMEM_COLS * CTAS_ <= 512, "co-resident CTAs must fit tensor memory together");
  static_assert(DQW_ % DQG_ == 0 && WG % 4 == 0 && 16 % WG == 0, "dequant groups cover whole lane quarters");
  // a group's chunks reuse its own stages and ring slots (both counts whole multiples of the groups),
  // so its parity waits never fall two phases behind: each stage and slot it waits on was last used
  // by the same group
  static_assert(STG_ % DQG_ == 0, "stages are whole multiples of the groups");
  static_assert(BN_ % 32 == 0 && BN_ <= 128, "token tiles are whole 32-row TMA boxes, N <= 128");
};
using WideShape = GemmShape<16, 4, 2, 4, 1, 128>;
using PairShape = GemmShape<8, 2, 1, 2, 2, 128>;
// Decode shapes: few tokens per expert, so the item count is set by the weight tiles and the kernel
// is a weight stream whose rate is the number of chunks in flight per SM. Two CTAs per SM (two
// MMA issuers and dequant pipelines) and small token tiles, which leave tensor memory for 3
// dequantised stages per CTA: 32-token items with 2 accumulators, or 64-token items with one.
using Decode32Shape = GemmShape<8, 3, 2, 6, 2, 32>;
using Decode64Shape = GemmShape<8, 3, 1, 4, 2, 64>;
constexpr int Q4K_UNIT = BM * 128 + BM * 32;
constexpr int TMA_ROWS = 32;  // token rows per TMA box  // Q4_K unit: quants + per-sub-block scale pairs
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, SWIZZLE_128B shared-memory matrix descriptor: rows of 128 bytes, 8-row groups 1024 bytes
// apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major), 16 B
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;             // version
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: f16 A and B, f32 accumulator, both K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// A from tensor memory (columns of 2 x f16 per lane), B from shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Four 32-bit columns per lane of this warp's 32-lane quarter.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint4& v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}


// ---- weight formats -----------------------------------------------------------------------------

struct GemmParams {
  const uint8_t* w;       // tile-major weights
  const float* wscale;    // FP8: [E][tiles][K/128][2] block scales (row halves of each 32-row group)
  int64_t w_stride;       // bytes per expert
  int tiles;              // 128-row tiles per expert
  int K;
  int N_rows;             // weight rows per expert (gate/up: 2I, down: H)
  int phase;              // 0: gate/up -> h (f32, sorted pairs); 1: down -> ypair
  const int32_t* tile_list;  // [n] (a_idx << 16) | ntile
  const int32_t* n_tiles;
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* perm;
  const float* tscale;    // per sorted row: power-of-two scale of the staged tokens
  const float* route_w;   // phase 1: routing weight per pair
  float* out;             // phase 0: h [pairs, N_rows/2]; phase 1: ypair [pairs, N_rows]
  int32_t* err;
  const int32_t* slot_of;  // [E] cache slot of each expert, or null: weights indexed by expert id
  int32_t* work;           // work-item counter of this launch (zero at launch)
};

// Weight formats. Weights stream through a shared-memory ring in "units" (one contiguous 1-D bulk
// copy each); each dequant thread then reads the 32 weights it owns of a 128-column chunk.
struct FP8W {
  static constexpr int UNIT_BYTES = BM * BK;  // one 128-column chunk of the tile: 16 KB
  static constexpr int CHUNKS_PER_UNIT = 1;
  struct Raw {
    uint4 q[2];
    float s;
  };
  __device__ static __forceinline__ const uint8_t* unit_src(const GemmParams& p, int e, int tile, int u) {
    return p.w + (int64_t)e * p.w_stride + ((int64_t)tile * (p.K / BK) + u) * UNIT_BYTES;
  }
  // thread (row r, quarter qq): 32 e4m3 bytes of chunk kc
  __device__ static __forceinline__ void read(const GemmParams& p, const unsigned char* unit, int e, int tile, int kc,
                                              int r, int qq, Raw& raw) {
    const unsigned char* row = unit + r * BK;
    raw.q[0] = *reinterpret_cast<const uint4*>(row + (((2 * qq) ^ (r & 7)) << 4));
    raw.q[1] = *reinterpret_cast<const uint4*>(row + (((2 * qq + 1) ^ (r & 7)) << 4));
    // merged gate/up tiles carry two scales per chunk: rows 8..15 of each 16-row group are up rows
    raw.s = __ldg(p.wscale + (((int64_t)e * p.tiles + tile) * (p.K / BK) + kc) * 2 + ((r >> 3) & 1));
  }
  __device__ static __forceinline__ void dequant(const Raw& raw, int, int, uint4 (&out)[4]) {
    const __half2 s2 = __float2half2_rn(raw.s);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t w[4] = {raw.q[i].x, raw.q[i].y, raw.q[i].z, raw.q[i].w};
      uint32_t h[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t lo, hi;
        const uint16_t wl = (uint16_t)(w[j] & 0xffff), wh = (uint16_t)(w[j] >> 16);
        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"(wl));
        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"(wh));
        __half2 a = __hmul2(*reinterpret_cast<__half2*>(&lo), s2);
        __half2 b = __hmul2(*reinterpret_cast<__half2*>(&hi), s2);
        h[2 * j] = *reinterpret_cast<uint32_t*>(&a);
        h[2 * j + 1] = *reinterpret_cast<uint32_t*>(&b);
      }
      out[2 * i] = make_uint4(h[0], h[1], h[2], h[3]);
      out[2 * i + 1] = make_uint4(h[4], h[5], h[6], h[7]);
    }
  }
  // 16-byte chunk index (within the 64-column atom row) of out[j]: 32 bytes -> chunks 4 (qq%2) + j
  __device__ static __forceinline__ int chunk_of(int qq, int j) { return (qq & 1) * 4 + j; }
};

struct Q4KW {
  static constexpr int UNIT_BYTES = Q4K_UNIT;  // one 256-column super-block of the tile: 20 KB
  static constexpr int CHUNKS_PER_UNIT = 2;
  struct Raw {
    uint4 q;     // 16 quant bytes: low nibbles of sub-block 2c, high nibbles of 2c + 1
    uint2 s;     // {d*sc, -dmin*m} f16 pairs of sub-blocks 2c and 2c + 1
  };
  __device__ static __forceinline__ const uint8_t* unit_src(const GemmParams& p, int e, int tile, int u) {
    return p.w + (int64_t)e * p.w_stride + ((int64_t)tile * (p.K / 256) + u) * UNIT_BYTES;
  }
  // thread (row r, quarter qq) of chunk kc: 64-column quarter c = 2 (kc % 2) + qq / 2 of the
  // super-block, quant bytes 32 c + 16 (qq % 2) .. +15
  __device__ static __forceinline__ void read(const GemmParams&, const unsigned char* unit, int, int, int kc, int r,
                                              int qq, Raw& raw) {
    const int c = ((kc & 1) << 1) | (qq >> 1);
    raw.q = *reinterpret_cast<const uint4*>(unit + r * 128 + (((2 * c + (qq & 1)) ^ (r & 7)) << 4));
    raw.s = *reinterpret_cast<const uint2*>(unit + BM * 128 + r * 32 + c * 8);
  }
  // out[0..1]: the 16 low-nibble weights (columns 16 (qq%2) .. +15 of the atom row),
  // out[2..3]: the 16 high-nibble weights (columns 32 + 16 (qq%2) .. +15)
  __device__ static __forceinline__ void dequant(const Raw& raw, int, int, uint4 (&out)[4]) {
    const __half2 bias = __float2half2_rn(1024.0f);
    const __half2 p0 = *reinterpret_cast<const __half2*>(&raw.s.x), p1 = *reinterpret_cast<const __half2*>(&raw.s.y);
    const __half2 d0 = __low2half2(p0), m0 = __high2half2(p0), d1 = __low2half2(p1), m1 = __high2half2(p1);
    const uint32_t w[4] = {raw.q.x, raw.q.y, raw.q.z, raw.q.w};
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t nl = w[t] & 0x0f0f0f0fu, nh = (w[t] >> 4) & 0x0f0f0f0fu;
      uint32_t a0 = __byte_perm(nl, 0x64646464u, 0x4140), a1 = __byte_perm(nl, 0x64646464u, 0x4342);
      uint32_t b0 = __byte_perm(nh, 0x64646464u, 0x4140), b1 = __byte_perm(nh, 0x64646464u, 0x4342);
      __half2 x0 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&a0), bias), d0, m0);
      __half2 x1 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&a1), bias), d0, m0);
      __half2 y0 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&b0), bias), d1, m1);
      __half2 y1 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&b1), bias), d1, m1);
      lo[2 * t] = *reinterpret_cast<uint32_t*>(&x0);
      lo[2 * t + 1] = *reinterpret_cast<uint32_t*>(&x1);
      hi[2 * t] = *reinterpret_cast<uint32_t*>(&y0);
      hi[2 * t + 1] = *reinterpret_cast<uint32_t*>(&y1);
    }
    out[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    out[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
    out[2] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    out[3] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
  }
  // 16-byte chunk index (within the 64-column atom row) of out[j]
  __device__ static __forceinline__ int chunk_of(int qq, int j) { return (j >> 1) * 4 + (qq & 1) * 2 + (j & 1); }
};

// Q8_0: the decode GEMV's units (repack.cu, repack_q8_units): per (expert, 128-row tile, 128-column
// chunk) 16 KB of m16n8k16 A fragments, [16-row tile s][block][slot 4g + (c ^ ((g >> 1) & 3))][16 B],
// lane (g, c)'s word j holding {row g, row g + 8} x columns 8j + 2c, +1 of the block (u = q + 128),
// then per s 128 B of {d(row g), d(row g + 8)} block-scale pairs at g * 16 + block * 4.
struct Q8W {
  static constexpr int UNIT_BYTES = Q8_UNIT_BYTES;  // 17 KB
  static constexpr int CHUNKS_PER_UNIT = 1;
  struct Raw {
    uint32_t p[8];  // word j's {column 8j + 2c, +1} bytes of this row for c = 2h, 2h + 1 at p[2j + h]
    uint32_t d;     // f16 block scale in the low half
  };
  __device__ static __forceinline__ const uint8_t* unit_src(const GemmParams& p, int e, int tile, int u) {
    return p.w + (int64_t)e * p.w_stride + ((int64_t)tile * (p.K / BK) + u) * UNIT_BYTES;
  }
  // thread (row r, quarter qq): row r's 32 quants of block qq, gathered from the four fragment slots
  // of its g (each holds rows g and g + 8), and its scale
  __device__ static __forceinline__ void read(const GemmParams&, const unsigned char* unit, int, int, int, int r,
                                              int qq, Raw& raw) {
    const int s16 = r >> 4, g = r & 7, up = (r >> 3) & 1;
    const unsigned char* blk = unit + (s16 * 4 + qq) * 512 + g * 64;
    const int f = (g >> 1) & 3;
    uint4 v[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] = *reinterpret_cast<const uint4*>(blk + ((c ^ f) << 4));
    const uint32_t sel = up ? 0x7632u : 0x5410u;  // bytes 2,3 (row g + 8) or 0,1 (row g) of two words
    const uint32_t w[4][4] = {{v[0].x, v[0].y, v[0].z, v[0].w},
                              {v[1].x, v[1].y, v[1].z, v[1].w},
                              {v[2].x, v[2].y, v[2].z, v[2].w},
                              {v[3].x, v[3].y, v[3].z, v[3].w}};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      raw.p[2 * j] = __byte_perm(w[0][j], w[1][j], sel);
      raw.p[2 * j + 1] = __byte_perm(w[2][j], w[3][j], sel);
    }
    raw.d = *reinterpret_cast<const uint16_t*>(unit + 8 * 4 * 512 + s16 * 128 + g * 16 + qq * 4 + up * 2);
  }
  // (1024 + u) by the 0x64 exponent byte, minus 1152 -> q exactly, times d: one f16 rounding;
  // out[j] = columns 8j .. 8j + 7 of the block in order
  __device__ static __forceinline__ void dequant(const Raw& raw, int, int, uint4 (&out)[4]) {
    const __half2 bias = __float2half2_rn(1152.0f);
    const uint32_t dd = raw.d | (raw.d << 16);
    const __half2 d2 = *reinterpret_cast<const __half2*>(&dd);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t h[4];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        uint32_t lo = __byte_perm(raw.p[2 * j + t], 0x64646464u, 0x4140);
        uint32_t hi = __byte_perm(raw.p[2 * j + t], 0x64646464u, 0x4342);
        __half2 a = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&lo), bias), d2);
        __half2 b = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&hi), bias), d2);
        h[2 * t] = *reinterpret_cast<uint32_t*>(&a);
        h[2 * t + 1] = *reinterpret_cast<uint32_t*>(&b);
      }
      out[j] = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
  __device__ static __forceinline__ int chunk_of(int qq, int j) { return (qq & 1) * 4 + j; }
};

// Weight-ring slots of a (format, shape): the shape's RING, or fewer when the format's units do not
// fit the shared memory left to each of the SM's CTAS_PER_SM CTAs (228 KB per SM, 1 KB reserved per
// CTA, a little static shared memory).
template <class W, class C>
__host__ __device__ constexpr int ring_slots() {
  constexpr int budget = 233472 / C::CTAS_PER_SM - 1024 - 64;
  constexpr int fit = (budget - C::STG * C::B_BYTES - 1024 - 512) / W::UNIT_BYTES;
  return fit < C::RING ? fit : C::RING;
}

template <class W, class C>
__host__ __device__ constexpr int gemm_smem_bytes() {
  return ring_slots<W, C>() * W::UNIT_BYTES + C::STG * C::B_BYTES + 1024 + 512;
}

// ---- the GEMM ------------------------------------------------------------------------------------
//
// Persistent: one or two CTAs per SM take the launch's work items from a global counter (one
// atomicAdd per item by the weight-streaming thread, which runs ahead of every other role and hands
// each index to them through a small shared-memory ring), item w = (token tile w / tiles, weight
// tile w % tiles), so CTAs running side by side share a token tile in L2 and stream different weight
// tiles. Taking items as they free up absorbs what a static split cannot: the SMs' different rates
// (measured: the CTAs of a static round-robin launch finished up to 15-25% apart) and items of
// different token counts. Warp roles, all hand-offs through mbarriers and all rings continuing
// across item boundaries:
//   * warps 0..15 dequantise chunk q (a global chunk counter) from the weight ring into tensor-memory
//     stage q % ASTAGES once the MMAs of chunk q - ASTAGES released it (stage_free), and arrive a_full;
//     after the last chunk of a weight unit they arrive raw_free for its ring slot;
//   * warp 16 (one lane) issues the 8 MMAs of each chunk into the item's accumulator (two
//     accumulators alternate between items), commits them to stage_free, and after the last
//     chunk commits acc_full; it waits acc_free before reusing an accumulator;
//   * warp 17 (one lane) streams weight units into the ring (1-D bulk copies, each after raw_free);
//   * warp 18 (one lane) streams token tiles into the B stages (2-D TMA, each after stage_free);
//   * warps 20..23 run the epilogue of item j while the next item computes: tensor-memory lane
//     quarter w % 4, per-column scales and destinations loaded before acc_full completes.
// A wait that runs past its limit (or sees another role give up) sets s_abort; every role stops at
// its next wait, the MMA warp drains its MMAs, the CTA waits (bounded) for the copies it issued,
// frees its tensor memory and returns.

struct Item {
  int e, es, base, n0, nval, nmma, tile;  // es: the expert's weight slot
};

// Work-item ring: the weight-streaming thread decodes the CTA's j-th item (its chain of dependent
// global loads: tile list -> active expert -> cache slot and offsets) and publishes it in slot
// j % ITEM_RING (e = -1 once the launch's counter has run past the last item), then arrives
// item_full; every consuming role (token loader, MMA issuer, each dequant and epilogue warp) copies
// it from shared memory and arrives item_free, after which the slot can take item j + ITEM_RING.
// The streaming thread runs ahead of the other roles, so none of them waits on those loads.
constexpr int ITEM_RING = 8;

template <class C>
__host__ __device__ constexpr int item_consumers() {
  return 2 + C::DQW + EPI_WARPS;
}

// The j-th item for a consuming role: 1 with *it filled, 0 when the launch has no more items, -1
// when the wait gave up (timeout or abort). Warp-collective when `warp_wide` (every lane gets the
// same result; lane 0 releases the slot), else called by one thread.
__device__ __forceinline__ int take_item(uint64_t* item_full, uint64_t* item_free, const Item* s_items, int j,
                                         volatile int* abort, bool warp_wide, Item* it) {
  const int slot = j % ITEM_RING;
  bool ok = mbar_wait(&item_full[slot], (j / ITEM_RING) & 1, abort);
  if (warp_wide) ok = __all_sync(FULL, ok);
  if (!ok) return -1;
  *it = s_items[slot];
  if (warp_wide) __syncwarp();
  if (!warp_wide || (threadIdx.x & 31) == 0) mbar_arrive(&item_free[slot]);
  return it->e >= 0 ? 1 : 0;
}

template <int BN>
__device__ __forceinline__ Item decode_item(const GemmParams& p, int w) {
  Item it;
  const int ti = w / p.tiles;
  it.tile = w % p.tiles;
  const int entry = __ldg(p.tile_list + ti);
  it.e = __ldg(p.active + (entry >> 16));
  it.es = p.slot_of ? __ldg(p.slot_of + it.e) : it.e;
  it.base = __ldg(p.offsets + it.e);
  const int count = __ldg(p.offsets + it.e + 1) - it.base;
  it.n0 = (entry & 0xffff) * BN;
  it.nval = min(BN, count - it.n0);
  it.nmma = (it.nval + 15) & ~15;  // M = 128 needs N % 16 == 0
  return it;
}

// Epilogue of one work item for the calling warp: tensor-memory lanes 32 quad .. +31 (weight rows)
// and the 16-column blocks cb0 <= cb < cb1 of accumulator columns (tokens). Gate/up: lanes 0..7 and
// 16..23 hold gate rows, the 8 lanes above each the matching up rows -> h = silu(g) * u. Down:
// ypair = w * (W h).
template <int BN>
__device__ __forceinline__ void epilogue_blocks(const GemmParams& p, const Item& it, uint32_t tbase, int quad, int lane,
                                                int cb0, int cb1) {
  // per-column scale (and, for the down projection, destination pair) of columns lane + 32 t
  float csc[BN / 32];
  int cpr[BN / 32];
#pragma unroll
  for (int t = 0; t < BN / 32; ++t) {
    const int n = lane + 32 * t;
    csc[t] = 0.0f;
    cpr[t] = 0;
    if (n < it.nval) {
      const int idx = it.base + it.n0 + n;
      csc[t] = __ldg(p.tscale + idx);
      if (p.phase == 1) {
        cpr[t] = __ldg(p.perm + idx);
        csc[t] *= __ldg(p.route_w + cpr[t]);
      }
    }
  }
#pragma unroll
  for (int cb = 0; cb < BN / 16; ++cb) {  // compile-time block index: csc / cpr stay in registers
    const int c0 = cb * 16;
    if (cb < cb0 || cb >= cb1 || c0 >= it.nmma) continue;
    float v[16];
    tmem_ld16(tbase + (uint32_t)c0, v);
    // All shuffles and arithmetic of the block first, with no branch between the 16 tokens, then the
    // predicated stores: a branch per token (the gate lanes' SiLU, or the valid-column test) makes
    // the scheduler run each token's shuffle -> exp -> reciprocal -> store chain to completion before
    // the next one starts (measured ~3,500 SM cycles per 16-token gate/up block, ~50 per down store).
    if (p.phase == 0) {
      const int col = it.tile * 64 + quad * 16 + (lane >> 4) * 8 + (lane & 7);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int n = c0 + i;
        const float sc = __shfl_sync(FULL, csc[n >> 5], n & 31);
        const float up = __shfl_down_sync(FULL, v[i], 8);
        const float g = v[i] * sc, uu = up * sc;  // meaningful on the gate lanes only
        v[i] = __fdividef(g, 1.0f + __expf(-g)) * uu;
      }
      float* dst = p.out + (int64_t)(it.base + it.n0 + c0) * (p.N_rows >> 1) + col;
      const bool gate_lane = !(lane & 8);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (gate_lane && c0 + i < it.nval) dst[(int64_t)i * (p.N_rows >> 1)] = v[i];
    } else {
      int pr[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int n = c0 + i;
        v[i] *= __shfl_sync(FULL, csc[n >> 5], n & 31);
        pr[i] = __shfl_sync(FULL, cpr[n >> 5], n & 31);
      }
      float* dst = p.out + it.tile * BM + quad * 32 + lane;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (c0 + i < it.nval) dst[(int64_t)pr[i] * p.N_rows] = v[i];
    }
  }
}

// With one accumulator (NACC == 1) the next item's MMAs wait for this item's epilogue. The gate/up
// epilogue (SiLU, 16-lane stores) is long enough that the dequant warps take part: warps sharing a
// lane quarter split the 8 column blocks (dequant warps w / 4 = 0, 1 take [0, 3) and [3, 6), the
// epilogue warp [6, 8)). The down epilogue is short; there the epilogue warps alone do it and the
// dequant warps run ahead into the next item.
template <class C>
__device__ __forceinline__ bool dequant_joins_epilogue(const GemmParams& p) {
  return C::NACC == 1 && C::DQG == 1 && C::BN == 128 && p.phase == 0;
}

template <class C>
__device__ __forceinline__ void epilogue_range(const GemmParams& p, int part, int* cb0, int* cb1) {
  if (!dequant_joins_epilogue<C>(p)) {
    *cb0 = 0;
    *cb1 = C::BN / 16;
  } else {
    *cb0 = part * 3;
    *cb1 = part == 2 ? C::BN / 16 : part * 3 + 3;
  }
}

template <class W, class C>
__global__ void __launch_bounds__(C::THREADS, C::CTAS_PER_SM)
    expert_gemm_kernel(GemmParams p, const __grid_constant__ CUtensorMap tmap) {
  constexpr int R = ring_slots<W, C>();
  static_assert(R >= 2 && R % C::DQG == 0, "weight ring: at least two slots, whole multiples of the groups");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned base, offset from the __shared__ array itself (not through an integer) so the
  // compiler keeps the shared address space and the ring reads stay shared-memory loads
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* sB = smem;                                // [C::STG][C::B_BYTES]
  unsigned char* sR = sB + C::STG * C::B_BYTES;           // [RING][UNIT_BYTES] raw weights
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(sR + R * W::UNIT_BYTES);
  uint64_t* raw_free = raw_full + R;
  uint64_t* b_full = raw_free + R;
  uint64_t* a_full = b_full + C::STG;
  uint64_t* stage_free = a_full + C::STG;  // MMAs of the stage's chunk done: weights and tokens reusable
  uint64_t* acc_full = stage_free + C::STG;
  uint64_t* acc_free = acc_full + C::NACC;
  uint64_t* mma_done = acc_free + C::NACC;
  uint64_t* item_full = mma_done + 1;
  uint64_t* item_free = item_full + ITEM_RING;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_free + ITEM_RING);
  __shared__ volatile int s_abort;
  __shared__ int s_units_issued, s_tiles_issued;
  __shared__ Item s_items[ITEM_RING];

  pdl_wait();  // the tile list, the gathered tokens and the error word come from earlier kernels
  pdl_trigger();
  // after any CTA gave up on a wait, the rest of the launch does no work
  if (p.err && *reinterpret_cast<volatile int32_t*>(p.err) == (int32_t)MOE_ERR_TIMEOUT) return;
  const int n_items = *p.n_tiles * p.tiles;
  if ((int)blockIdx.x >= n_items) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kchunks = p.K / BK;
  const int units = kchunks / W::CHUNKS_PER_UNIT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < R; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_free[s], W::CHUNKS_PER_UNIT * C::WG);  // each reading warp, once per chunk
    }
    for (int s = 0; s < C::STG; ++s) {
      mbar_init(&b_full[s], 1);
    }
    for (int s = 0; s < C::STG; ++s) {
      mbar_init(&a_full[s], C::WG);  // one arrival per warp of the chunk's dequant group
      mbar_init(&stage_free[s], 1);
    }
    for (int s = 0; s < C::NACC; ++s) {
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_free[s], EPI_WARPS + (dequant_joins_epilogue<C>(p) ? C::DQW : 0));
    }
    mbar_init(mma_done, 1);
    for (int s = 0; s < ITEM_RING; ++s) {
      mbar_init(&item_full[s], 1);
      mbar_init(&item_free[s], item_consumers<C>());
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
    s_units_issued = 0;
    s_tiles_issued = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  volatile int* abort = &s_abort;

  if (warp == C::WLOAD_WARP) {
    // ---------------- weight units -> ring ----------------
    if (lane == 0) {
      int g = 0;
      for (int j = 0; !*abort; ++j) {
        const int islot = j % ITEM_RING;
        if (j >= ITEM_RING && !mbar_wait(&item_free[islot], ((j / ITEM_RING) - 1) & 1, abort)) {
          s_abort = 1;
          break;
        }
        const int w = atomicAdd(p.work, 1);
        Item it;
        if (w < n_items) it = decode_item<C::BN>(p, w);
        else it.e = -1;
        s_items[islot] = it;
        mbar_arrive(&item_full[islot]);  // release: the item is visible to the roles that wait on it
        if (it.e < 0) break;
        for (int u = 0; u < units; ++u, ++g) {
          const int slot = g % R;
          if (g >= R && !mbar_wait(&raw_free[slot], ((g / R) - 1) & 1, abort)) {
            s_abort = 1;
            break;
          }
          mbar_expect_tx(&raw_full[slot], W::UNIT_BYTES);
          bulk_load(sR + slot * W::UNIT_BYTES, W::unit_src(p, it.es, it.tile, u), W::UNIT_BYTES, &raw_full[slot]);
          s_units_issued = g + 1;
        }
      }
    }
    __syncwarp();
  } else if (warp == C::TLOAD_WARP) {
    // ---------------- token tiles -> B stages ----------------
    if (lane == 0) {
      int q = 0;
      for (int j = 0; !*abort; ++j) {
        Item it;
        const int got = take_item(item_full, item_free, s_items, j, abort, false, &it);
        if (got <= 0) {
          if (got < 0) s_abort = 1;
          break;
        }
        const int boxes = (it.nmma + TMA_ROWS - 1) / TMA_ROWS;  // only the tile's own token rows
        for (int kc = 0; kc < kchunks; ++kc, ++q) {
          const int b = q % C::STG;
          if (q >= C::STG && !mbar_wait(&stage_free[b], ((q / C::STG) - 1) & 1, abort)) {
            s_abort = 1;
            break;
          }
          mbar_expect_tx(&b_full[b], 2 * boxes * TMA_ROWS * 128);
          for (int h = 0; h < 2; ++h)
            for (int j = 0; j < boxes; ++j)
              tma_load_2d(sB + b * C::B_BYTES + h * (C::BN * 128) + j * (TMA_ROWS * 128), &tmap, kc * BK + 64 * h,
                          it.base + it.n0 + j * TMA_ROWS, &b_full[b]);
          s_tiles_issued = q + 1;
        }
      }
    }
    __syncwarp();
  } else if (warp == C::MMA_WARP) {
    // ---------------- MMA issue ----------------
    if (lane == 0) {
      const uint64_t bdesc0 = smem_desc(smem_u32(sB));
      int q = 0;
      bool issued = false;  // a CTA may take no item at all when the others drain the counter first
      for (int j = 0; !*abort; ++j) {
        Item it;
        const int got = take_item(item_full, item_free, s_items, j, abort, false, &it);
        if (got <= 0) {
          if (got < 0) s_abort = 1;
          break;
        }
        const int acc = j % C::NACC;
        if (j >= C::NACC && !mbar_wait(&acc_free[acc], ((j / C::NACC) - 1) & 1, abort)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t idesc = idesc_f16(it.nmma);
        const uint32_t dcol = tmem + (uint32_t)(acc * C::BN);
        for (int kc = 0; kc < kchunks; ++kc, ++q) {
          const int sa = q % C::STG, b = q % C::STG;
          if (!mbar_wait(&a_full[sa], (q / C::STG) & 1, abort) || !mbar_wait(&b_full[b], (q / C::STG) & 1, abort)) {
            s_abort = 1;
            break;
          }
          tc_fence_after();
          const uint32_t acol = tmem + (uint32_t)(C::A_COL0 + sa * A_COLS);
          const uint64_t bd = bdesc0 + ((uint32_t)(b * C::B_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_ts(dcol, acol + (uint32_t)(k * 8), bd + (uint32_t)(((k >> 2) * (C::BN * 128) + (k & 3) * 32) >> 4),
                        idesc, (kc > 0 || k > 0) ? 1u : 0u);
          umma_commit(&stage_free[sa]);
          issued = true;
        }
        if (*abort) break;
        umma_commit(&acc_full[acc]);
      }
      // drain: every MMA this thread issued has completed once mma_done flips (no commit at all when
      // the CTA issued no MMA)
      if (issued) {
        umma_commit(mma_done);
        if (!mbar_wait(mma_done, 0, nullptr)) s_abort = 1;
      }
      // The commits of the last STG chunks arrive on stage_free barriers nobody else waits for any
      // more. Each arrive-on is a write to this CTA's shared memory: wait (bounded) until every one
      // has landed, so none can land after the CTA has exited, in the shared memory of whatever
      // CTA the SM runs next.
      for (int c = q > C::STG ? q - C::STG : 0; c < q; ++c)
        if (!mbar_wait(&stage_free[c % C::STG], (c / C::STG) & 1, nullptr)) s_abort = 1;
    }
    __syncwarp();
  } else if (warp >= C::EPI_WARP0) {
    // ---------------- epilogue ----------------
    const int quad = warp & 3;  // tensor-memory lanes 32 quad .. +31
    for (int j = 0;; ++j) {
      Item it;
      const int got = take_item(item_full, item_free, s_items, j, abort, true, &it);
      if (got <= 0) {
        if (got < 0 && lane == 0) s_abort = 1;
        break;
      }
      const int acc = j % C::NACC;
      const bool ok = __all_sync(FULL, mbar_wait(&acc_full[acc], (j / C::NACC) & 1, abort));
      if (!ok) {
        if (lane == 0) s_abort = 1;
        break;
      }
      tc_fence_after();
      int cb0, cb1;
      epilogue_range<C>(p, 2, &cb0, &cb1);
      epilogue_blocks<C::BN>(p, it, tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * C::BN), quad, lane, cb0, cb1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_free[acc]);
    }
  } else if (warp < C::DQW) {
    // ---------------- dequant ----------------
    // group grp = warp / WG takes the chunks q with q % DQG == grp; warp w owns tensor-memory lanes
    // 32 (w % 4) .. +31 (its weight rows, one per thread) and the QPW 32-column quarters
    // QPW ((w % WG) / 4) .. of each of its chunks
    const int grp = warp / C::WG;
    const int drow = threadIdx.x & (BM - 1), dq0 = ((warp % C::WG) >> 2) * C::QPW;
    const uint32_t lane_base = tmem + ((uint32_t)(drow & ~31) << 16) + (uint32_t)C::A_COL0;
    int q = 0, g = 0, j_item = 0;
    bool stop = false;
    while (!stop) {
      Item it;
      const int got = take_item(item_full, item_free, s_items, j_item, abort, true, &it);
      if (got <= 0) {
        stop = got < 0;
        break;
      }
      for (int kc = 0; kc < kchunks; ++kc, ++q) {
        if (C::DQG > 1 && q % C::DQG != grp) continue;
        const int gu = g + kc / W::CHUNKS_PER_UNIT, slot = gu % R;
        const bool ok_raw = mbar_wait(&raw_full[slot], (gu / R) & 1, abort);
        // the tcgen05 stores below are warp-collective: every lane takes the same branch
        stop = __any_sync(FULL, !ok_raw);
        if (stop) break;
        typename W::Raw raw[C::QPW];
#pragma unroll
        for (int d = 0; d < C::QPW; ++d) W::read(p, sR + slot * W::UNIT_BYTES, it.es, it.tile, kc, drow, dq0 + d, raw[d]);
        __syncwarp();  // this warp's reads of the unit are done (one arrival per warp and chunk)
        if (lane == 0) mbar_arrive(&raw_free[slot]);
        // prefill shapes (up to two quarters): convert before waiting for the stage, so the
        // conversion overlaps the MMAs still reading it; the decode shapes, whose MMAs rarely hold a
        // stage, convert one quarter at a time after the wait (fewer live registers)
        constexpr bool EARLY = C::QPW <= 2 && C::BN == 128;
        uint4 vals[EARLY ? C::QPW : 1][4];
        if (EARLY) {
#pragma unroll
          for (int d = 0; d < C::QPW; ++d) W::dequant(raw[d], kc, dq0 + d, vals[EARLY ? d : 0]);
        }
        const int sa = q % C::STG;
        const bool ok_a = q < C::STG || mbar_wait(&stage_free[sa], ((q / C::STG) - 1) & 1, abort);
        stop = __any_sync(FULL, !ok_a);
        if (stop) break;
        tc_fence_after();  // order the stores after the MMAs that read this stage
        const uint32_t stage = lane_base + (uint32_t)(sa * A_COLS);
#pragma unroll
        for (int d = 0; d < C::QPW; ++d) {
          const int dq = dq0 + d;
          const int vd = EARLY ? d : 0;
          if (!EARLY) W::dequant(raw[d], kc, dq, vals[0]);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj)
            tmem_st4(stage + (uint32_t)((dq >> 1) * 32 + W::chunk_of(dq, jj) * 4), vals[vd][jj]);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
      }
      g += units;
      if (dequant_joins_epilogue<C>(p) && !stop) {  // this item's share of the epilogue
        const bool ok_acc = mbar_wait(&acc_full[0], (j_item & 1), abort);
        stop = __any_sync(FULL, !ok_acc);
        if (stop) break;
        tc_fence_after();
        int cb0, cb1;
        epilogue_range<C>(p, warp >> 2, &cb0, &cb1);
        epilogue_blocks<C::BN>(p, it, tmem + ((uint32_t)(drow & ~31) << 16), warp & 3, lane, cb0, cb1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_free[0]);
      }
      ++j_item;
    }
    if (stop && lane == 0) s_abort = 1;
  }
  __syncthreads();

  // After an abort, wait (bounded) for the copies still in flight: the last RING weight units and the
  // last C::STG token tiles issued (earlier ones were consumed, so their phases completed).
  const bool failed = s_abort != 0;
  if (failed && threadIdx.x == 0) {
    for (int u = max(0, s_units_issued - R); u < s_units_issued; ++u)
      (void)mbar_wait(&raw_full[u % R], (u / R) & 1, nullptr);
    for (int c = max(0, s_tiles_issued - C::STG); c < s_tiles_issued; ++c)
      (void)mbar_wait(&b_full[c % C::STG], (c / C::STG) & 1, nullptr);
    if (p.err) atomicExch(p.err, (int)MOE_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
}

// ---- helpers around the GEMM ----------------------------------------------------------------------

// (a_idx, 128-token tile) entries of the active experts, in order; one CTA.
constexpr int TL_THREADS = 256;

// (a_idx << 16 | token tile) entries of the active experts, in active order. One CTA: each pass of
// TL_THREADS active experts computes its tile counts, scans them across the block and writes its
// entries; loads are independent per thread (a serial walk costs two dependent loads per expert).
__global__ void __launch_bounds__(TL_THREADS) tile_list_kernel(const int32_t* __restrict__ counts,
                                                               const int32_t* __restrict__ active,
                                                               const int32_t* __restrict__ n_active, int bn,
                                                               int32_t* __restrict__ list, int32_t* __restrict__ n_list) {
  __shared__ int s_warp[TL_THREADS / 32];
  __shared__ int s_base;
  pdl_wait();  // the plan's counts and active list
  pdl_trigger();
  const int na = *n_active;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  for (int a0 = 0; a0 < na; a0 += TL_THREADS) {
    const int a = a0 + threadIdx.x;
    const int nt = a < na ? (__ldg(counts + __ldg(active + a)) + bn - 1) / bn : 0;
    int incl = nt;  // inclusive scan within the warp, then across warps
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    int before = s_base;
    for (int w = 0; w < warp; ++w) before += s_warp[w];
    const int start = before + incl - nt;
    for (int j = 0; j < nt; ++j) list[start + j] = (a << 16) | j;
    __syncthreads();
    if (threadIdx.x == TL_THREADS - 1) s_base = start + nt;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    n_list[0] = s_base;
    n_list[1] = 0;  // work-item counters of the gate/up and down launches that follow
    n_list[2] = 0;
  }
}

// Sorted, f16 copy of the tokens (one warp per sorted pair): each row scaled by a power of two so
// its max magnitude lies in [2^13, 2^14) (exact for bf16 inputs), the scale kept per row. Only the
// first *n_valid sorted positions exist (the plan drops empty MOE_ID_NONE slots and bad ids), so
// warps past it return; a perm entry outside [0, n_pairs) is skipped as well.
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ xf, int K, int width,
                                   const int32_t* __restrict__ perm, int n_pairs, const int32_t* __restrict__ n_valid,
                                   __half* __restrict__ out, float* __restrict__ scale) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  pdl_wait();  // perm and the rows to gather come from earlier kernels
  pdl_trigger();
  if (warp >= n_pairs || warp >= *n_valid) return;
  const int pair = x ? perm[warp] : warp;
  if (pair < 0 || pair >= n_pairs) return;
  const int src = x ? pair / width : warp;
  float m = 0.0f;
  for (int c = lane; c < K / 8; c += 32) {
    if (x) {
      uint4 raw = ldg_nc(x + (int64_t)src * K + c * 8);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(b2[i]);
        m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    } else {
      const float4* r = reinterpret_cast<const float4*>(xf + (int64_t)src * K + c * 8);
      float4 a = r[0], b = r[1];
      m = fmaxf(m, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
      m = fmaxf(m, fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
    }
  }
  m = warp_max(m);
  float sc = 1.0f, inv = 1.0f;
  if (m > 0.0f && m < __int_as_float(0x7f800000)) {
    int ex;
    frexpf(m, &ex);
    const int sh = max(-100, min(100, ex - 14));
    sc = ldexpf(1.0f, sh);
    inv = ldexpf(1.0f, -sh);
  }
  if (lane == 0) scale[warp] = sc;
  for (int c = lane; c < K / 8; c += 32) {
    float v[8];
    if (x) {
      uint4 raw = ldg_nc(x + (int64_t)src * K + c * 8);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(b2[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else {
      const float4* r = reinterpret_cast<const float4*>(xf + (int64_t)src * K + c * 8);
      float4 a = r[0], b = r[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    uint4 o = make_uint4(pack_f16x2(v[0] * inv, v[1] * inv), pack_f16x2(v[2] * inv, v[3] * inv),
                         pack_f16x2(v[4] * inv, v[5] * inv), pack_f16x2(v[6] * inv, v[7] * inv));
    reinterpret_cast<uint4*>(out + (int64_t)warp * K)[c] = o;
  }
}

// ---- repack: GGML stacks -> tile-major layouts ------------------------------------------------------

// device row r of a merged gate/up tile t: group g = (r % 128) / 16, within-group i = r % 16;
// i < 8 -> gate row 64 t + 8 g + i, else up row 64 t + 8 g + (i - 8).
__device__ __forceinline__ void gu_src(int tile, int r, int* which, int* row) {
  const int g = r >> 4, i = r & 15;
  *which = i >= 8;
  *row = tile * 64 + g * 8 + (i & 7);
}

// FP8: one thread per (e, tile, kchunk, row): 128 bytes + the scale
__global__ void repack_fp8_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b,
                                  const float* __restrict__ sa, const float* __restrict__ sb, int E, int N_src, int K,
                                  uint8_t* __restrict__ dst, float* __restrict__ dscale) {
  const bool merged = b != nullptr;
  const int rows = merged ? 2 * N_src : N_src;
  const int tiles = rows / BM, kch = K / BK;
  const int64_t total = (int64_t)E * tiles * kch * BM;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int r = (int)(i % BM);
  int64_t rest = i / BM;
  const int kc = (int)(rest % kch);
  rest /= kch;
  const int tile = (int)(rest % tiles);
  const int e = (int)(rest / tiles);
  int which = 0, srow = tile * BM + r;
  if (merged) gu_src(tile, r, &which, &srow);
  const uint8_t* src = (which ? b : a) + ((int64_t)e * N_src + srow) * K + kc * BK;
  uint8_t* d = dst + (((int64_t)e * tiles + tile) * kch + kc) * (BM * BK) + r * BK;
  for (int j = 0; j < BK / 16; ++j)  // 16-byte chunk j of the row at j ^ (r % 8): conflict-free ring reads
    *reinterpret_cast<uint4*>(d + ((j ^ (r & 7)) << 4)) = *reinterpret_cast<const uint4*>(src + j * 16);
  // per (tile, chunk) two scales {rows of group half 0, rows of group half 1}: a merged tile holds gate
  // rows 64t..64t+63 and up rows 64t..64t+63, each inside one 128-row scale block of its projection;
  // an unmerged 128-row tile is one scale block, stored twice
  if (r == 0 || r == 8) {
    const float* ss = (which ? sb : sa);
    dscale[(((int64_t)e * tiles + tile) * kch + kc) * 2 + (r >> 3)] =
        ss[((int64_t)e * (N_src / 128) + srow / 128) * kch + kc];
  }
}

// Q4_K: one thread per (e, tile, super-block, row): 144 bytes (9 x 16)
// Q4_K: one thread per (e, tile, super-block, row). Unit layout per (e, tile, super-block):
// [128 rows][128 B] quants, then [128 rows][8 sub-blocks] f16 pairs {d*sc, -dmin*m} (the values the
// GGML formula multiplies and adds, rounded once to f16 exactly as the in-kernel dequant rounds them).
__global__ void repack_q4k_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b, int E, int N_src,
                                  int K, uint8_t* __restrict__ dst) {
  const bool merged = b != nullptr;
  const int rows = merged ? 2 * N_src : N_src;
  const int tiles = rows / BM, sbs = K / 256;
  const int64_t total = (int64_t)E * tiles * sbs * BM;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int r = (int)(i % BM);
  int64_t rest = i / BM;
  const int sb = (int)(rest % sbs);
  rest /= sbs;
  const int tile = (int)(rest % tiles);
  const int e = (int)(rest / tiles);
  int which = 0, srow = tile * BM + r;
  if (merged) gu_src(tile, r, &which, &srow);
  const uint8_t* src = (which ? b : a) + (((int64_t)e * N_src + srow) * sbs + sb) * 144;
  uint8_t* unit = dst + (((int64_t)e * tiles + tile) * sbs + sb) * Q4K_UNIT;
  for (int j = 0; j < 8; ++j)  // 16-byte chunk j of the row at j ^ (r % 8): conflict-free ring reads
    *reinterpret_cast<uint4*>(unit + r * 128 + ((j ^ (r & 7)) << 4)) = *reinterpret_cast<const uint4*>(src + 16 + j * 16);
  const float d = __half2float(*reinterpret_cast<const __half*>(src));
  const float dmin = __half2float(*reinterpret_cast<const __half*>(src + 2));
  const uint8_t* sc = src + 4;
  uint32_t pairs[8];
  for (int j = 0; j < 8; ++j) {
    int sv, mv;
    if (j < 4) {
      sv = sc[j] & 63;
      mv = sc[j + 4] & 63;
    } else {
      sv = (sc[j + 4] & 0xf) | ((sc[j - 4] >> 6) << 4);
      mv = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    __half2 h2 = __floats2half2_rn(d * (float)sv, -(dmin * (float)mv));
    pairs[j] = *reinterpret_cast<uint32_t*>(&h2);
  }
  uint4* sdst = reinterpret_cast<uint4*>(unit + BM * 128 + r * 32);
  sdst[0] = make_uint4(pairs[0], pairs[1], pairs[2], pairs[3]);
  sdst[1] = make_uint4(pairs[4], pairs[5], pairs[6], pairs[7]);
}

}  // namespace tc

// ---- host side --------------------------------------------------------------------------------------

using PFN_encodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode() {
  static PFN_encodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

// 2-D map over an f16 [rows, cols] row-major buffer, box 64 columns x 32 rows, SWIZZLE_128B.
moe_status make_row_tmap(void* map_out, const void* base, int64_t rows, int cols) {
  PFN_encodeTiled enc = get_encode();
  if (!enc) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (((uintptr_t)base & 15) || (cols * 2) % 16) return fail(MOE_ERR_INVALID, "tensor map: misaligned rows");
  CUtensorMap* m = static_cast<CUtensorMap*>(map_out);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)tc::TMA_ROWS};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return MOE_OK;
}

size_t tensor_map_bytes() { return sizeof(CUtensorMap); }

// Decode batches (a few tokens per expert: mean <= 16, or <= 24) take the 32- or 64-token decode
// shapes; prompts, whose busiest experts hold far more than the mean under skewed routing, the
// 128-token prefill shapes.
int tc_token_tile(int n_pairs, int E) {
  static const int forced = [] {  // MOE_TC_BN=32|64|128 pins the choice (tuning knob)
    const char* v = std::getenv("MOE_TC_BN");
    return v ? std::atoi(v) : 0;
  }();
  if (forced == 32 || forced == 64 || forced == 128) return forced;
  if ((int64_t)n_pairs <= 16ll * E) return 32;
  return (int64_t)n_pairs <= 24ll * E ? 64 : 128;
}

int64_t tc_weight_bytes(int wdtype, int N, int K) {
  if (wdtype == MOE_DTYPE_FP8_E4M3_B128) return (int64_t)N * K;
  if (wdtype == MOE_DTYPE_Q4_K) return (int64_t)(N / tc::BM) * (K / 256) * tc::Q4K_UNIT;
  if (wdtype == MOE_DTYPE_Q8_0) return (int64_t)(N / tc::BM) * (K / tc::BK) * Q8_UNIT_BYTES;
  return 0;
}
int64_t tc_scale_count(int wdtype, int N, int K) {
  return wdtype == MOE_DTYPE_FP8_E4M3_B128 ? (int64_t)(N / tc::BM) * (K / tc::BK) * 2 : 0;
}

moe_status tc_repack(int wdtype, const uint8_t* a, const uint8_t* b, const float* sa, const float* sb, int E, int N_src,
                     int K, uint8_t* dst, float* dscale, cudaStream_t st) {
  const int rows = b ? 2 * N_src : N_src;
  const int t = 256;
  if (wdtype == MOE_DTYPE_FP8_E4M3_B128) {
    const int64_t total = (int64_t)E * (rows / tc::BM) * (K / tc::BK) * tc::BM;
    tc::repack_fp8_kernel<<<(unsigned)((total + t - 1) / t), t, 0, st>>>(a, b, sa, sb, E, N_src, K, dst, dscale);
  } else if (wdtype == MOE_DTYPE_Q4_K) {
    const int64_t total = (int64_t)E * (rows / tc::BM) * (K / 256) * tc::BM;
    tc::repack_q4k_kernel<<<(unsigned)((total + t - 1) / t), t, 0, st>>>(a, b, E, N_src, K, dst);
  } else if (wdtype == MOE_DTYPE_Q8_0) {
    return repack_q8_units(a, b, E, N_src, K, dst, st);
  } else {
    return fail(MOE_ERR_UNSUPPORTED, "tensor-core path: weight format not built");
  }
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status tc_gather(const void* x_bf16, const float* x_f32, int K, int width, const int32_t* perm, int n_pairs,
                     const int32_t* n_valid, void* out_f16, float* scale, cudaStream_t st, bool pdl) {
  if (n_pairs <= 0) return MOE_OK;
  const int threads = 256;
  const int blocks = (int)(((int64_t)n_pairs * 32 + threads - 1) / threads);
  MOE_CUDA_TRY(launch_pdl_if(pdl, tc::gather_rows_kernel, dim3(blocks), dim3(threads), 0, st,
                          static_cast<const __nv_bfloat16*>(x_bf16), x_f32, K, width, perm, n_pairs, n_valid,
                          static_cast<__half*>(out_f16), scale));
  return MOE_OK;
}

moe_status tc_tile_list(const int32_t* counts, const int32_t* active, const int32_t* n_active, int bn, int32_t* list,
                        int32_t* n_list, cudaStream_t st) {
  if (bn != 32 && bn != 64 && bn != 128) return fail(MOE_ERR_INVALID, "tile list: bad token tile");
  MOE_CUDA_TRY(launch_pdl_if(bn < 128, tc::tile_list_kernel, dim3(1), dim3(tc::TL_THREADS), 0, st, counts, active,
                             n_active, bn, list, n_list));
  return MOE_OK;
}



template <class W, class C>
static moe_status launch_tc(const TcArgs& a, cudaStream_t st) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(tc::expert_gemm_kernel<W, C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      tc::gemm_smem_bytes<W, C>()));
    attr[dev & 63] = true;
  }
  tc::GemmParams p;
  p.w = a.w;
  p.wscale = a.wscale;
  p.w_stride = a.w_stride;
  p.tiles = a.N_rows / tc::BM;
  p.K = a.K;
  p.N_rows = a.N_rows;
  p.phase = a.phase;
  p.tile_list = a.tile_list;
  p.n_tiles = a.n_tiles;
  p.offsets = a.offsets;
  p.active = a.active;
  p.perm = a.perm;
  p.tscale = a.tscale;
  p.route_w = a.route_w;
  p.out = a.out;
  p.err = a.err;
  p.slot_of = a.slot_of;
  p.work = a.work;
  if (!p.work) return fail(MOE_ERR_INVALID, "tensor-core path: no work-item counter");
  static int sms[64] = {};
  if (!sms[dev & 63]) MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev));
  // persistent: CTAS_PER_SM CTAs per SM (or one per work item when there are fewer); the token
  // tiles of n_pairs sorted rows over at most max_active experts number at most n_pairs / BN + max_active
  const int64_t max_tiles = (int64_t)(a.n_pairs + C::BN - 1) / C::BN + a.max_active;
  const int grid = (int)std::min<int64_t>(max_tiles * p.tiles, (int64_t)sms[dev & 63] * C::CTAS_PER_SM);
  if (grid <= 0) return MOE_OK;
  // programmatic launch for the decode shapes only: measured, it slows the prefill pipeline
  MOE_CUDA_TRY(launch_pdl_if(C::BN < 128, tc::expert_gemm_kernel<W, C>, dim3(grid), dim3(C::THREADS),
                             tc::gemm_smem_bytes<W, C>(), st, p, *static_cast<const CUtensorMap*>(a.tmap)));
  return MOE_OK;
}

moe_status tc_gemm(int wdtype, const TcArgs& a, cudaStream_t st) {
  if (a.K % tc::BK || a.N_rows % tc::BM) return fail(MOE_ERR_INVALID, "tensor-core path: K % 128 or rows % 128");
  // MOE_TC_SHAPE=wide selects one 16-warp CTA per SM instead of two 8-warp CTAs (tuning knob)
  static const bool wide = [] {
    const char* v = std::getenv("MOE_TC_SHAPE");
    return v && std::string(v) == "wide";
  }();
  if (a.bn == tc::Decode32Shape::BN) {
    if (wdtype == MOE_DTYPE_FP8_E4M3_B128) return launch_tc<tc::FP8W, tc::Decode32Shape>(a, st);
    if (wdtype == MOE_DTYPE_Q4_K) return launch_tc<tc::Q4KW, tc::Decode32Shape>(a, st);
    if (wdtype == MOE_DTYPE_Q8_0) return launch_tc<tc::Q8W, tc::Decode32Shape>(a, st);
  } else if (a.bn == tc::Decode64Shape::BN) {
    if (wdtype == MOE_DTYPE_FP8_E4M3_B128) return launch_tc<tc::FP8W, tc::Decode64Shape>(a, st);
    if (wdtype == MOE_DTYPE_Q4_K) return launch_tc<tc::Q4KW, tc::Decode64Shape>(a, st);
    if (wdtype == MOE_DTYPE_Q8_0) return launch_tc<tc::Q8W, tc::Decode64Shape>(a, st);
  } else if (a.bn != tc::PairShape::BN) {
    return fail(MOE_ERR_INVALID, "tensor-core path: token tile must be 32, 64 or 128");
  }
  if (wdtype == MOE_DTYPE_FP8_E4M3_B128)
    return wide ? launch_tc<tc::FP8W, tc::WideShape>(a, st) : launch_tc<tc::FP8W, tc::PairShape>(a, st);
  if (wdtype == MOE_DTYPE_Q4_K)
    return wide ? launch_tc<tc::Q4KW, tc::WideShape>(a, st) : launch_tc<tc::Q4KW, tc::PairShape>(a, st);
  if (wdtype == MOE_DTYPE_Q8_0)
    return wide ? launch_tc<tc::Q8W, tc::WideShape>(a, st) : launch_tc<tc::Q8W, tc::PairShape>(a, st);
  return fail(MOE_ERR_UNSUPPORTED, "tensor-core path: weight format not built");
}

}  // namespace moe
