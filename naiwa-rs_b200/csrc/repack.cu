// repack.cu — GGML expert stacks -> the fragment-native device layout the decode kernels stream.
//
// Source: stacked [E, N, K] projections in GGML byte layout, the same bytes the reference slices per
// expert in expert_range (src/moe/expert.rs:123-145). Destination, per expert, per 16-row tile and
// 32-column block: 512 contiguous bytes (Q8_0 quants; 1 KB for BF16) in which lane l's 16 bytes
// are its m16n8k16 A-operand values for the block's two k16 steps:
//   byte/element j of a k16 step -> (row g + 8*((j>>1)&1), column (j>=4 ? 8 : 0) + 2c + (j&1)),
//   g = l/4, c = l%4.
// Q8_0 quants are stored biased (u = q + 128, the sign bit flipped) so the kernel's int8 -> f16
// conversion needs no XOR. Q8_0 scales go to a separate array: per tile and group of 4 blocks, 8 x 4 pairs {d(row g),
// d(row g+8)} (128 B), so one 16-byte load gives a lane its two rows' scales for 4 blocks.
// Gate and up are merged: tile t holds gate rows 8t..8t+7 then up rows 8t..8t+7, which puts a
// gate value and its up partner in the same thread after the MMA (SwiGLU in registers).
//
// Q8_0 units (hidden and inter multiples of 128): the same fragments and scales, grouped per
// (expert, 128-row tile, 128-column chunk) into one contiguous 17 KB unit that both the decode GEMV
// and the tcgen05 GEMM stream (the GEMM as one bulk copy):
//   [16-row tile s (8)][block (4)][fragment slot (32)][16 B]  then  [s (8)][128 B of scales],
// lane l = 4g + c's fragment stored in slot 4g + (c ^ ((g >> 1) & 3)) (the GEMM's dequant threads,
// one per weight row, read all four slots of their g; the swizzle spreads the eight g of a warp
// over all 32 banks).
//
// Q2_0 (the reference's resident-pool format: 64 weights per 18-byte block, f16 d, 2-bit codes,
// weight = (code - 1) d): per expert, per 16-row tile and 128-column group (two blocks), 512
// contiguous bytes of codes in which lane l = 4g + c's 16 bytes are four 32-bit words, word w
// holding the k16 steps 2w and 2w + 1 of the group: for step s and fragment pair q (0: row g, columns
// 2c..2c+1 of the step's first 8; 1: row g+8, same; 2: row g, columns 8+2c..; 3: row g+8, same), with
// p = (s & 1) * 4 + q, the pair's first code at bits 2p and its second at bits 16 + 2p, so one shift
// and one mask-or turn a pair into an f16x2 of 1024 + code. Scales apart: per tile and group, 8 x 8 B
// (lane g's {d(g), d(g+8)} of the group's two blocks).
#include "moe_internal.cuh"

namespace moe {

struct RepackSrc {
  const uint8_t* a;  // gate (merged) or the single projection
  const uint8_t* b;  // up (merged) or null
  int64_t expert_bytes;  // bytes of one expert in a source stack
  int N_src;             // rows per source projection
  int K;
};

__device__ __forceinline__ const uint8_t* src_row(const RepackSrc& s, int e, int tile, int r, int row_bytes) {
  if (s.b) {
    const uint8_t* base = r < 8 ? s.a : s.b;
    int row = tile * 8 + (r & 7);
    return base + (int64_t)e * s.expert_bytes + (int64_t)row * row_bytes;
  }
  return s.a + (int64_t)e * s.expert_bytes + (int64_t)(tile * 16 + r) * row_bytes;
}

__device__ __forceinline__ void frag_pos(int lane, int j, int* r, int* kk) {
  const int g = lane >> 2, c = lane & 3;
  *r = g + 8 * ((j >> 1) & 1);
  *kk = (j >= 4 ? 8 : 0) + 2 * c + (j & 1);
}

// one thread per (e, tile, kb, lane): 16 quant bytes
__global__ void repack_q8_kernel(RepackSrc s, int E, int tiles, uint8_t* __restrict__ dq) {
  const int KB = s.K / 32;
  const int64_t total = (int64_t)E * tiles * KB * 32;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int lane = (int)(i & 31);
  int64_t rest = i >> 5;
  const int kb = (int)(rest % KB); rest /= KB;
  const int tile = (int)(rest % tiles);
  const int e = (int)(rest / tiles);
  const int row_bytes = KB * 34;
  uint8_t out[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    int r, kk;
    frag_pos(lane, j & 7, &r, &kk);
    const int k = (j >> 3) * 16 + kk;
    out[j] = src_row(s, e, tile, r, row_bytes)[kb * 34 + 2 + k] ^ 0x80;  // stored as u = q + 128
  }
  uint4 v;
  memcpy(&v, out, 16);
  reinterpret_cast<uint4*>(dq)[i] = v;
}

// one thread per (e, tile, kbg, g): 16 bytes of scales
__global__ void repack_q8_scales_kernel(RepackSrc s, int E, int tiles, uint8_t* __restrict__ ds) {
  const int KB = s.K / 32, KBG = (KB + 3) / 4;
  const int64_t total = (int64_t)E * tiles * KBG * 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int g = (int)(i & 7);
  int64_t rest = i >> 3;
  const int kbg = (int)(rest % KBG); rest /= KBG;
  const int tile = (int)(rest % tiles);
  const int e = (int)(rest / tiles);
  const int row_bytes = KB * 34;
  uint16_t out[8];
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const int kb = kbg * 4 + b;
    uint16_t lo = 0, hi = 0;
    if (kb < KB) {
      const uint8_t* p0 = src_row(s, e, tile, g, row_bytes) + kb * 34;
      const uint8_t* p1 = src_row(s, e, tile, g + 8, row_bytes) + kb * 34;
      lo = (uint16_t)(p0[0] | (p0[1] << 8));
      hi = (uint16_t)(p1[0] | (p1[1] << 8));
    }
    out[2 * b] = lo;
    out[2 * b + 1] = hi;
  }
  uint4 v;
  memcpy(&v, out, 16);
  reinterpret_cast<uint4*>(ds)[i] = v;
}

// one thread per (e, tile, kb, k16 step, lane): 8 bf16 = 16 bytes
__global__ void repack_bf16_kernel(RepackSrc s, int E, int tiles, uint8_t* __restrict__ dq) {
  const int KB = s.K / 32;
  const int64_t total = (int64_t)E * tiles * KB * 64;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int lane = (int)(i & 31);
  const int step = (int)((i >> 5) & 1);
  int64_t rest = i >> 6;
  const int kb = (int)(rest % KB); rest /= KB;
  const int tile = (int)(rest % tiles);
  const int e = (int)(rest / tiles);
  const int row_bytes = s.K * 2;
  uint16_t out[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    int r, kk;
    frag_pos(lane, j, &r, &kk);
    const int k = kb * 32 + step * 16 + kk;
    const uint8_t* p = src_row(s, e, tile, r, row_bytes) + k * 2;
    out[j] = (uint16_t)(p[0] | (p[1] << 8));
  }
  uint4 v;
  memcpy(&v, out, 16);
  reinterpret_cast<uint4*>(dq)[i] = v;
}

// one thread per (e, 128-row tile, chunk, 16-row tile s, block, lane): 16 quant bytes, and for c == 0
// the {d(row g), d(row g + 8)} scale pair of the block
__global__ void repack_q8_units_kernel(RepackSrc s, int E, int tiles128, uint8_t* __restrict__ dst) {
  const int KB = s.K / 32, kch = s.K / 128;
  const int64_t total = (int64_t)E * tiles128 * kch * 8 * 4 * 32;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int lane = (int)(i & 31);
  const int blk = (int)((i >> 5) & 3);
  const int st16 = (int)((i >> 7) & 7);
  int64_t rest = i >> 10;
  const int kc = (int)(rest % kch); rest /= kch;
  const int t128 = (int)(rest % tiles128);
  const int e = (int)(rest / tiles128);
  const int tile = t128 * 8 + st16, kb = kc * 4 + blk;
  const int row_bytes = KB * 34;
  uint8_t out[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    int r, kk;
    frag_pos(lane, j & 7, &r, &kk);
    const int k = (j >> 3) * 16 + kk;
    out[j] = src_row(s, e, tile, r, row_bytes)[kb * 34 + 2 + k] ^ 0x80;  // stored as u = q + 128
  }
  uint4 v;
  memcpy(&v, out, 16);
  const int g = lane >> 2, c = lane & 3;
  uint8_t* unit = dst + (((int64_t)e * tiles128 + t128) * kch + kc) * Q8_UNIT_BYTES;
  reinterpret_cast<uint4*>(unit + (st16 * 4 + blk) * 512)[4 * g + (c ^ ((g >> 1) & 3))] = v;
  if (c == 0) {
    const uint8_t* p0 = src_row(s, e, tile, g, row_bytes) + kb * 34;
    const uint8_t* p1 = src_row(s, e, tile, g + 8, row_bytes) + kb * 34;
    const uint32_t pair = (uint32_t)(p0[0] | (p0[1] << 8)) | ((uint32_t)(p1[0] | (p1[1] << 8)) << 16);
    *reinterpret_cast<uint32_t*>(unit + 8 * 4 * 512 + st16 * 128 + g * 16 + blk * 4) = pair;
  }
}

static int blocks_for(int64_t n, int t) { return (int)((n + t - 1) / t); }

// merged: src a = gate [E, I, H], b = up [E, I, H] -> N = 2I device rows; else a = [E, N, K].
moe_status repack_q8_units(const uint8_t* a, const uint8_t* b, int E, int N_src, int K, uint8_t* dst,
                           cudaStream_t st) {
  const int rows = b ? 2 * N_src : N_src;
  if (rows % 128 || K % 128) return fail(MOE_ERR_INVALID, "Q8_0 units need 128-multiple rows and columns");
  RepackSrc s;
  s.a = a;
  s.b = b;
  s.N_src = N_src;
  s.K = K;
  s.expert_bytes = (int64_t)N_src * (K / 32) * 34;
  const int t = 256;
  repack_q8_units_kernel<<<blocks_for((int64_t)E * (rows / 128) * (K / 128) * 1024, t), t, 0, st>>>(s, E, rows / 128,
                                                                                                   dst);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

// one thread per (e, tile, 128-column group, lane): 16 bytes of codes
__global__ void repack_q2_kernel(RepackSrc s, int E, int tiles, uint8_t* __restrict__ dq) {
  const int GR = s.K / 128;
  const int64_t total = (int64_t)E * tiles * GR * 32;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int lane = (int)(i & 31);
  int64_t rest = i >> 5;
  const int gr = (int)(rest % GR); rest /= GR;
  const int tile = (int)(rest % tiles);
  const int e = (int)(rest / tiles);
  const int row_bytes = s.K / 64 * 18;
  const int g = lane >> 2, c = lane & 3;
  uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int step = 0; step < 8; ++step)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int r = g + 8 * (q & 1);
      const int col = gr * 128 + step * 16 + 8 * (q >> 1) + 2 * c;  // the pair's first column
      const uint8_t* row = src_row(s, e, tile, r, row_bytes);
      const uint8_t* blk = row + (col / 64) * 18;
      const int j0 = col % 64, j1 = j0 + 1;
      const uint32_t c0 = (blk[2 + j0 / 4] >> (2 * (j0 % 4))) & 3u;
      const uint32_t c1 = (blk[2 + j1 / 4] >> (2 * (j1 % 4))) & 3u;
      const int pq = (step & 1) * 4 + q;
      w[step >> 1] |= (c0 << (2 * pq)) | (c1 << (16 + 2 * pq));
    }
  reinterpret_cast<uint4*>(dq)[i] = make_uint4(w[0], w[1], w[2], w[3]);
}

// one thread per (e, tile, group, g): 8 bytes of scales {d(g), d(g+8)} of the group's two blocks
__global__ void repack_q2_scales_kernel(RepackSrc s, int E, int tiles, uint8_t* __restrict__ ds) {
  const int GR = s.K / 128;
  const int64_t total = (int64_t)E * tiles * GR * 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int g = (int)(i & 7);
  int64_t rest = i >> 3;
  const int gr = (int)(rest % GR); rest /= GR;
  const int tile = (int)(rest % tiles);
  const int e = (int)(rest / tiles);
  const int row_bytes = s.K / 64 * 18;
  uint16_t out[4];
#pragma unroll
  for (int b = 0; b < 2; ++b) {
    const uint8_t* p0 = src_row(s, e, tile, g, row_bytes) + (gr * 2 + b) * 18;
    const uint8_t* p1 = src_row(s, e, tile, g + 8, row_bytes) + (gr * 2 + b) * 18;
    out[2 * b] = (uint16_t)(p0[0] | (p0[1] << 8));
    out[2 * b + 1] = (uint16_t)(p1[0] | (p1[1] << 8));
  }
  uint2 v;
  memcpy(&v, out, 8);
  reinterpret_cast<uint2*>(ds)[i] = v;
}

// Device bytes of one expert's projection in the device layout.
int64_t device_q_bytes(int wdtype, int N, int K) {
  if (wdtype == MOE_DTYPE_Q8_0) return (int64_t)N * K;
  if (wdtype == MOE_DTYPE_BF16) return (int64_t)N * K * 2;
  if (wdtype == MOE_DTYPE_Q2_0) return (int64_t)N * K / 4;
  return 0;
}
int64_t device_s_bytes(int wdtype, int N, int K) {
  if (wdtype == MOE_DTYPE_Q8_0) return (int64_t)(N / 16) * ((K / 32 + 3) / 4) * 128;
  if (wdtype == MOE_DTYPE_Q2_0) return (int64_t)(N / 16) * (K / 128) * 64;
  return 0;
}

// merged: src a = gate [E, I, H], b = up [E, I, H] -> N = 2I device rows; else a = [E, N, K].
moe_status repack_projection(int wdtype, const uint8_t* a, const uint8_t* b, int E, int N_src, int K,
                             uint8_t* dq, uint8_t* ds, cudaStream_t st) {
  RepackSrc s;
  s.a = a;
  s.b = b;
  s.N_src = N_src;
  s.K = K;
  const int rows = b ? 2 * N_src : N_src;
  const int tiles = rows / 16;
  const int KB = K / 32;
  const int t = 256;
  if (wdtype == MOE_DTYPE_Q8_0) {
    s.expert_bytes = (int64_t)N_src * KB * 34;
    repack_q8_kernel<<<blocks_for((int64_t)E * tiles * KB * 32, t), t, 0, st>>>(s, E, tiles, dq);
    MOE_CUDA_TRY(cudaGetLastError());
    repack_q8_scales_kernel<<<blocks_for((int64_t)E * tiles * ((KB + 3) / 4) * 8, t), t, 0, st>>>(s, E, tiles, ds);
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
  }
  if (wdtype == MOE_DTYPE_Q2_0) {
    if (K % 128) return fail(MOE_ERR_INVALID, "repack: Q2_0 needs K % 128 == 0");
    s.expert_bytes = (int64_t)N_src * (K / 64) * 18;
    repack_q2_kernel<<<blocks_for((int64_t)E * tiles * (K / 128) * 32, t), t, 0, st>>>(s, E, tiles, dq);
    MOE_CUDA_TRY(cudaGetLastError());
    repack_q2_scales_kernel<<<blocks_for((int64_t)E * tiles * (K / 128) * 8, t), t, 0, st>>>(s, E, tiles, ds);
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
  }
  if (wdtype == MOE_DTYPE_BF16) {
    s.expert_bytes = (int64_t)N_src * K * 2;
    repack_bf16_kernel<<<blocks_for((int64_t)E * tiles * KB * 64, t), t, 0, st>>>(s, E, tiles, dq);
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
  }
  return fail(MOE_ERR_UNSUPPORTED, "repack: weight format not built yet");
}

}  // namespace moe
