// expert_gemm_tc.cu — prefill-size grouped expert GEMM on the 5th-generation tensor cores.
//
// Reference: the fork's grouped MoE kernels behind MoEExperts::forward, driven by
// PrefillStream::dispatch (src/moe/prefill_stream.rs:1178-1216) and forward_batched (:2080-2102),
// with the expert math of run_expert (src/moe/stages/gpu.rs:162-167).
//
// One CTA computes one (expert, 128-row weight tile, <=128-token tile) block of
//   gate/up:  H[tok, n] = SwiGLU over the tile's 64 gate and 64 up rows of X_e W^T
//   down:     Ypair[pair, n] = w_pair * (h_e W^T)[tok, n]
// as D[128 x N] (TMEM, f32) = A[128 x K] (weights, shared memory) * B[K x N] (tokens, shared memory)
// with tcgen05.mma kind::f16 issued by one thread. Per 128-column K stage:
//   * the token tile arrives by two 2-D TMA loads (64 columns each, SWIZZLE_128B) from the
//     gathered, f16-converted activations, completing on an mbarrier;
//   * every thread dequantises 64 weights of one row (Q4_K: nibble -> f16 by the 0x6400 exponent
//     trick, then d*sc*q - dmin*m in f16; FP8 e4m3: cvt to f16 times the 128x128 block scale) and
//     writes them in the same SWIZZLE_128B K-major layout;
//   * one thread issues 8 MMAs (K = 16 each) and commits them to the stage's mbarrier, which gates
//     the reuse of that stage two steps later. Two stages keep dequant/TMA of stage k+1 under the
//     MMAs of stage k.
// Every wait is bounded: a wait that runs out sets MOE_ERR_TIMEOUT in the error word, the CTA
// stops issuing work, waits (bounded) for its own MMAs, frees its TMEM and returns.
//
// Weight layouts in HBM (tile-major, built by the repack kernels below):
//   FP8:  per (expert, 128-row tile, 128-column chunk) 16 KB of e4m3, row-major inside; the
//         128x128 block scale of that chunk in a separate f32 array.
//   Q4_K: per (expert, 128-row tile, 256-column super-block) the tile's 128 GGML blocks (144 B each).
// Gate/up tiles hold, per 32-row group, 16 gate rows then the 16 up rows of the same columns, so
// one warp holds a gate value and its up partner after tcgen05.ld (SwiGLU by one shuffle).
#include <cuda.h>

#include "moe_internal.cuh"

namespace moe {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 128;
constexpr int THREADS = 256;
constexpr int A_BYTES = BM * BK * 2;  // one stage of f16 weights
constexpr int B_BYTES = BN * BK * 2;  // one stage of f16 tokens
constexpr int STAGES = 2;
constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES) + 1024 /* alignment */ + 256 /* barriers */;
constexpr uint32_t WAIT_POLLS = 1u << 22;             // backstop on try_wait polls
constexpr uint64_t WAIT_NS = 200ull * 1000ull * 1000ull;  // a wait longer than 200 ms is declared stuck

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded parity wait: true when the phase completed, false after 200 ms (or WAIT_POLLS polls).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < WAIT_POLLS; ++i) {
    uint32_t done;
    asm volatile(
        "{.reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 63) == 63 && globaltimer_ns() - t0 > WAIT_NS) return false;
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
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

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
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

// Byte offset of the 16-byte chunk j (8 elements) of row r in a SWIZZLE_128B K-major atom.
__device__ __forceinline__ uint32_t sw128(int r, int j) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4)); }

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
};

struct FP8W {
  // thread (row r, half q) -> 64 weights of K-chunk kc: 4 x 16 B
  struct Raw {
    uint4 q[4];
    float s;
  };
  __device__ static __forceinline__ void load(const GemmParams& p, int e, int tile, int kc, int r, int q, Raw& raw) {
    const int kchunks = p.K / BK;
    const uint8_t* base = p.w + (int64_t)e * p.w_stride + ((int64_t)tile * kchunks + kc) * (BM * BK) + r * BK + q * 64;
#pragma unroll
    for (int i = 0; i < 4; ++i) raw.q[i] = ldg_stream(base + i * 16);
    // merged gate/up tiles carry two scales per chunk: rows 16..31 of each 32-row group are up rows
    raw.s = __ldg(p.wscale + (((int64_t)e * p.tiles + tile) * kchunks + kc) * 2 + ((r & 31) >> 4));
  }
  // 64 f16 values as 8 chunks of 16 bytes
  __device__ static __forceinline__ void dequant(const Raw& raw, uint4 (&out)[8]) {
    const __half2 s2 = __float2half2_rn(raw.s);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
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
};

struct Q4KW {
  struct Raw {
    uint4 hdr;   // d, dmin, scales[12]
    uint4 q[2];  // 32 bytes of nibbles
  };
  __device__ static __forceinline__ void load(const GemmParams& p, int e, int tile, int kc, int r, int q, Raw& raw) {
    const int sbs = p.K / 256;
    const int sb = kc >> 1;                    // super-block of this 128-column chunk
    const int c = ((kc & 1) << 1) | q;         // 64-column quarter of the super-block
    const uint8_t* blk = p.w + (int64_t)e * p.w_stride + ((int64_t)tile * sbs + sb) * (BM * 144) + r * 144;
    raw.hdr = ldg_nc(blk);
    raw.q[0] = ldg_stream(blk + 16 + c * 32);
    raw.q[1] = ldg_stream(blk + 16 + c * 32 + 16);
  }
  __device__ static __forceinline__ void dequant_c(const Raw& raw, int c, uint4 (&out)[8]) {
    const uint32_t hw[4] = {raw.hdr.x, raw.hdr.y, raw.hdr.z, raw.hdr.w};
    const __half2 dd = *reinterpret_cast<const __half2*>(&hw[0]);
    const float d = __low2float(dd), dmin = __high2float(dd);
    const uint8_t* sc = reinterpret_cast<const uint8_t*>(&hw[1]);
    float dl[2], ml[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = 2 * c + h;
      int s, m;
      if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
      } else {
        s = (sc[j + 4] & 0xf) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
      }
      dl[h] = d * (float)s;
      ml[h] = dmin * (float)m;
    }
    const __half2 bias = __float2half2_rn(1024.0f);
    const uint32_t w[8] = {raw.q[0].x, raw.q[0].y, raw.q[0].z, raw.q[0].w, raw.q[1].x, raw.q[1].y, raw.q[1].z, raw.q[1].w};
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // h = 0: low nibbles (sub-block 2c), 1: high nibbles (2c + 1)
      const __half2 d2 = __float2half2_rn(dl[h]);
      const __half2 m2 = __float2half2_rn(-ml[h]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {  // 8 bytes -> 8 weights per output chunk
        uint32_t o[4];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint32_t word = w[2 * i + t];
          const uint32_t nib = h ? (word >> 4) & 0x0f0f0f0fu : word & 0x0f0f0f0fu;
          uint32_t lo = __byte_perm(nib, 0x64646464u, 0x4140);  // 1024 + q
          uint32_t hi = __byte_perm(nib, 0x64646464u, 0x4342);
          __half2 a = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&lo), bias), d2, m2);
          __half2 b = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&hi), bias), d2, m2);
          o[2 * t] = *reinterpret_cast<uint32_t*>(&a);
          o[2 * t + 1] = *reinterpret_cast<uint32_t*>(&b);
        }
        out[4 * h + i] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
};

template <class W>
__device__ __forceinline__ void dequant_any(const typename W::Raw& raw, int c, uint4 (&out)[8]);
template <>
__device__ __forceinline__ void dequant_any<FP8W>(const FP8W::Raw& raw, int, uint4 (&out)[8]) {
  FP8W::dequant(raw, out);
}
template <>
__device__ __forceinline__ void dequant_any<Q4KW>(const Q4KW::Raw& raw, int c, uint4 (&out)[8]) {
  Q4KW::dequant_c(raw, c, out);
}

// ---- the GEMM ------------------------------------------------------------------------------------

template <class W>
__global__ void __launch_bounds__(THREADS, 1) expert_gemm_kernel(GemmParams p, const __grid_constant__ CUtensorMap tmap) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* sA = smem;                                // [STAGES][A_BYTES]
  unsigned char* sB = smem + STAGES * A_BYTES;             // [STAGES][B_BYTES]
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);  // TMA landed, per stage
  uint64_t* bar_mma = bar_full + STAGES;                   // MMAs of the stage done, per stage
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mma + STAGES);
  __shared__ int s_abort;
  __shared__ int s_last_tma, s_last_mma;  // last chunk whose TMA was issued / whose MMAs were committed

  const int tiles = p.tiles;
  const int ti = blockIdx.x / tiles;
  const int tile = blockIdx.x % tiles;
  if (ti >= *p.n_tiles) return;
  // after any CTA of this launch (or an earlier one) gave up on a wait, the rest do no work
  if (p.err && *reinterpret_cast<volatile int32_t*>(p.err) == (int32_t)MOE_ERR_TIMEOUT) return;
  const int entry = p.tile_list[ti];
  const int a_idx = entry >> 16, ntile = entry & 0xffff;
  const int e = p.active[a_idx];
  const int base = p.offsets[e];
  const int count = p.offsets[e + 1] - base;
  const int n0 = ntile * BN;
  const int nval = min(BN, count - n0);
  const int nmma = (nval + 15) & ~15;  // M = 128 needs N % 16 == 0
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kchunks = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_mma[s], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
    s_last_tma = -1;
    s_last_mma = -1;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // thread -> (row, 64-column half) of the weight tile for the dequant
  const int drow = threadIdx.x >> 1, dq = threadIdx.x & 1;
  typename W::Raw raw;
  W::load(p, e, tile, 0, drow, dq, raw);
  const uint32_t idesc = idesc_f16(nmma);
  bool ok = true;

  for (int kc = 0; kc < kchunks; ++kc) {
    const int s = kc & 1;
    if (kc >= STAGES) {  // the MMAs that read this stage two steps ago must be done
      if (!mbar_wait(&bar_mma[s], ((kc >> 1) - 1) & 1)) ok = false;
    }
    if (!ok) s_abort = 1;
    __syncthreads();
    if (s_abort) break;
    if (threadIdx.x == 0) {
      mbar_expect_tx(&bar_full[s], 2 * BN * 128);
      tma_load_2d(sB + s * B_BYTES, &tmap, kc * BK, base + n0, &bar_full[s]);
      tma_load_2d(sB + s * B_BYTES + BN * 128, &tmap, kc * BK + 64, base + n0, &bar_full[s]);
      s_last_tma = kc;
    }
    // dequantise this thread's 64 weights into the stage, prefetch the next chunk's bytes
    uint4 vals[8];
    dequant_any<W>(raw, ((kc & 1) << 1) | dq, vals);
    if (kc + 1 < kchunks) W::load(p, e, tile, kc + 1, drow, dq, raw);
    unsigned char* atom = sA + s * A_BYTES + dq * (BM * 128);
#pragma unroll
    for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(atom + sw128(drow, j)) = vals[j];
    fence_proxy_async();
    __syncthreads();
    if (threadIdx.x == 0) {
      if (!mbar_wait(&bar_full[s], (kc >> 1) & 1)) {
        s_abort = 1;
      } else {
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * A_BYTES), b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint32_t off = (k >> 2) * (BM * 128) + (k & 3) * 32;
          const uint32_t offb = (k >> 2) * (BN * 128) + (k & 3) * 32;
          umma_f16(tmem, smem_desc(a0 + off), smem_desc(b0 + offb), idesc, (kc > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&bar_mma[s]);
        s_last_mma = kc;
      }
    }
  }
  __syncthreads();
  // Wait (bounded) for this CTA's own work in flight: the last committed MMAs (which imply all
  // earlier ones) and, after an abort, the last issued TMA, before reading or freeing anything.
  bool have = !s_abort;
  if (s_last_mma >= 0 && !mbar_wait(&bar_mma[s_last_mma & 1], (s_last_mma >> 1) & 1)) have = false;
  if (s_abort && s_last_tma > s_last_mma) (void)mbar_wait(&bar_full[s_last_tma & 1], (s_last_tma >> 1) & 1);
  if (s_last_mma != kchunks - 1) have = false;
  if (!have && threadIdx.x == 0 && p.err) atomicExch(p.err, (int)MOE_ERR_TIMEOUT);
  tc_fence_after();

  if (have) {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (one weight row per thread) and the
    // token columns [64 (w / 4), +64) in steps of 16
    const int quad = warp & 3, chalf = warp >> 2;
    const int row = quad * 32 + lane;  // weight row within the tile
    for (int c0 = chalf * 64; c0 < chalf * 64 + 64; c0 += 16) {
      if (c0 >= nmma) break;
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0, v);
      if (p.phase == 0) {
        // lanes 0..15: gate rows, lanes 16..31: the matching up rows
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float up = __shfl_down_sync(FULL, v[i], 16);
          const int n = c0 + i;
          if (lane < 16 && n < nval) {
            const float sc = p.tscale[base + n0 + n];
            const float g = v[i] * sc, u = up * sc;
            const int col = tile * 64 + quad * 16 + lane;
            p.out[(int64_t)(base + n0 + n) * (p.N_rows >> 1) + col] = g / (1.0f + __expf(-g)) * u;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int n = c0 + i;
          if (n < nval) {
            const int pr = p.perm[base + n0 + n];
            p.out[(int64_t)pr * p.N_rows + tile * BM + row] = v[i] * p.tscale[base + n0 + n] * p.route_w[pr];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
}

// ---- helpers around the GEMM ----------------------------------------------------------------------

// (a_idx, 128-token tile) entries of the active experts, in order; one CTA.
__global__ void tile_list_kernel(const int32_t* __restrict__ counts, const int32_t* __restrict__ active,
                                 const int32_t* __restrict__ n_active, int32_t* __restrict__ list,
                                 int32_t* __restrict__ n_list) {
  if (threadIdx.x == 0) {
    int t = 0;
    const int na = *n_active;
    for (int a = 0; a < na; ++a) {
      const int nt = (counts[active[a]] + BN - 1) / BN;
      for (int j = 0; j < nt; ++j) list[t++] = (a << 16) | j;
    }
    *n_list = t;
  }
}

// Sorted, f16 copy of the tokens (one warp per sorted pair): each row scaled by a power of two so
// its max magnitude lies in [2^13, 2^14) (exact for bf16 inputs), the scale kept per row.
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ xf, int K, int width,
                                   const int32_t* __restrict__ perm, int n_pairs, __half* __restrict__ out,
                                   float* __restrict__ scale) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= n_pairs) return;
  const int src = x ? perm[warp] / width : warp;
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

// device row r of a merged gate/up tile t: group g = (r % 128) / 32, within-group i = r % 32;
// i < 16 -> gate row 64 t + 16 g + i, else up row 64 t + 16 g + (i - 16).
__device__ __forceinline__ void gu_src(int tile, int r, int* which, int* row) {
  const int g = r >> 5, i = r & 31;
  *which = i >= 16;
  *row = tile * 64 + g * 16 + (i & 15);
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
  for (int j = 0; j < BK; j += 16) *reinterpret_cast<uint4*>(d + j) = *reinterpret_cast<const uint4*>(src + j);
  // per (tile, chunk) two scales {rows of group half 0, rows of group half 1}: a merged tile holds gate
  // rows 64t..64t+63 and up rows 64t..64t+63, each inside one 128-row scale block of its projection;
  // an unmerged 128-row tile is one scale block, stored twice
  if (r == 0 || r == 16) {
    const float* ss = (which ? sb : sa);
    dscale[(((int64_t)e * tiles + tile) * kch + kc) * 2 + (r >> 4)] =
        ss[((int64_t)e * (N_src / 128) + srow / 128) * kch + kc];
  }
}

// Q4_K: one thread per (e, tile, super-block, row): 144 bytes (9 x 16)
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
  uint8_t* d = dst + (((int64_t)e * tiles + tile) * sbs + sb) * (BM * 144) + r * 144;
  for (int j = 0; j < 144; j += 16) *reinterpret_cast<uint4*>(d + j) = *reinterpret_cast<const uint4*>(src + j);
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

// 2-D map over an f16 [rows, cols] row-major buffer, box 64 columns x 128 rows, SWIZZLE_128B.
moe_status make_row_tmap(void* map_out, const void* base, int64_t rows, int cols) {
  PFN_encodeTiled enc = get_encode();
  if (!enc) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (((uintptr_t)base & 15) || (cols * 2) % 16) return fail(MOE_ERR_INVALID, "tensor map: misaligned rows");
  CUtensorMap* m = static_cast<CUtensorMap*>(map_out);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)tc::BN};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return MOE_OK;
}

size_t tensor_map_bytes() { return sizeof(CUtensorMap); }

int64_t tc_weight_bytes(int wdtype, int N, int K) {
  if (wdtype == MOE_DTYPE_FP8_E4M3_B128) return (int64_t)N * K;
  if (wdtype == MOE_DTYPE_Q4_K) return (int64_t)N * (K / 256) * 144;
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
  } else {
    return fail(MOE_ERR_UNSUPPORTED, "tensor-core path: weight format not built");
  }
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status tc_gather(const void* x_bf16, const float* x_f32, int K, int width, const int32_t* perm, int n_pairs,
                     void* out_f16, float* scale, cudaStream_t st) {
  if (n_pairs <= 0) return MOE_OK;
  const int threads = 256;
  const int blocks = (int)(((int64_t)n_pairs * 32 + threads - 1) / threads);
  tc::gather_rows_kernel<<<blocks, threads, 0, st>>>(static_cast<const __nv_bfloat16*>(x_bf16), x_f32, K, width, perm,
                                                     n_pairs, static_cast<__half*>(out_f16), scale);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status tc_tile_list(const int32_t* counts, const int32_t* active, const int32_t* n_active, int32_t* list,
                        int32_t* n_list, cudaStream_t st) {
  tc::tile_list_kernel<<<1, 32, 0, st>>>(counts, active, n_active, list, n_list);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}



template <class W>
static moe_status launch_tc(const TcArgs& a, cudaStream_t st) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(tc::expert_gemm_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      tc::SMEM_BYTES));
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
  const int grid = a.max_tiles * p.tiles;
  if (grid <= 0) return MOE_OK;
  tc::expert_gemm_kernel<W><<<grid, tc::THREADS, tc::SMEM_BYTES, st>>>(p, *static_cast<const CUtensorMap*>(a.tmap));
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status tc_gemm(int wdtype, const TcArgs& a, cudaStream_t st) {
  if (a.K % tc::BK || a.N_rows % tc::BM) return fail(MOE_ERR_INVALID, "tensor-core path: K % 128 or rows % 128");
  if (wdtype == MOE_DTYPE_FP8_E4M3_B128) return launch_tc<tc::FP8W>(a, st);
  if (wdtype == MOE_DTYPE_Q4_K) return launch_tc<tc::Q4KW>(a, st);
  return fail(MOE_ERR_UNSUPPORTED, "tensor-core path: weight format not built");
}

}  // namespace moe
