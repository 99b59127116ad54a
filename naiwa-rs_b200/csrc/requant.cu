// requant.cu — expert stacks requantised to Q2_0 on the device (the reference's resident pool).
//
// The reference requantises the drafter's experts on the CPU through an f32 intermediate
// (resident.rs:120-182, quantize_q2_0 :46-88); here one thread per 64-weight block decodes the
// source block to f32 and runs the same scale-ladder search, every operation explicitly rounded so
// that the bytes match the CPU restatement exactly: the f16 scale candidates amax / {1, 1.25, 1.5,
// 1.75, 2}, codes clamp(round-half-away(x / d) + 1, 0, 3), the candidate with the least squared
// error (the first on ties), an all-zero block stored as d = 0 with every code 1.
#include "moe_internal.cuh"

namespace moe {

// source weight i (0..63) of the 64-weight block starting at column k0 of row `row`
__device__ __forceinline__ float src_weight(int dtype, const uint8_t* __restrict__ row, int k0, int i) {
  const int k = k0 + i;
  if (dtype == MOE_DTYPE_BF16) {
    const uint16_t b = (uint16_t)(row[2 * k] | (row[2 * k + 1] << 8));
    return __uint_as_float((uint32_t)b << 16);
  }
  if (dtype == MOE_DTYPE_Q8_0) {
    const uint8_t* blk = row + (k / 32) * 34;
    const float d = __half2float(__ushort_as_half((uint16_t)(blk[0] | (blk[1] << 8))));
    return __fmul_rn(d, (float)(int8_t)blk[2 + k % 32]);
  }
  // Q4_K: 8 sub-blocks of 32 per 256-weight super-block, w = (d sc) q - dmin m
  const uint8_t* blk = row + (k / 256) * 144;
  const float d = __half2float(__ushort_as_half((uint16_t)(blk[0] | (blk[1] << 8))));
  const float dmin = __half2float(__ushort_as_half((uint16_t)(blk[2] | (blk[3] << 8))));
  const uint8_t* sc6 = blk + 4;
  const int kk = k % 256, j = kk / 32;  // sub-block
  int sc, m;
  if (j < 4) {
    sc = sc6[j] & 63;
    m = sc6[j + 4] & 63;
  } else {
    sc = (sc6[j + 4] & 0xf) | ((sc6[j - 4] >> 6) << 4);
    m = (sc6[j + 4] >> 4) | ((sc6[j] >> 6) << 4);
  }
  const int c = kk / 64, h = (kk / 32) & 1, l = kk % 32;
  const uint8_t qb = blk[16 + 32 * c + l];
  const int q = h ? (qb >> 4) : (qb & 0xf);
  return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
}

__global__ void requant_q2_0_kernel(int dtype, const uint8_t* __restrict__ src, int64_t rows, int K, int64_t src_row_bytes,
                                    uint8_t* __restrict__ dst) {
  const int blocks_per_row = K / 64;
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= rows * blocks_per_row) return;
  const int64_t r = b / blocks_per_row;
  const int k0 = (int)(b % blocks_per_row) * 64;
  const uint8_t* row = src + r * src_row_bytes;
  float v[64];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    v[i] = src_weight(dtype, row, k0, i);
    amax = fmaxf(amax, fabsf(v[i]));
  }
  uint8_t* o = dst + b * 18;
  uint32_t packed[4] = {0u, 0u, 0u, 0u};
  uint16_t dbits = 0;
  if (amax == 0.0f) {
    packed[0] = packed[1] = packed[2] = packed[3] = 0x55555555u;  // every code 1: decodes to zero
  } else {
    const float ladder[5] = {1.0f, 1.25f, 1.5f, 1.75f, 2.0f};
    float best_err = __int_as_float(0x7f800000), best_scale = 0.0f;
    uint32_t best[4] = {0u, 0u, 0u, 0u};
#pragma unroll 1
    for (int f = 0; f < 5; ++f) {
      const float scale = __half2float(__float2half_rn(__fdiv_rn(amax, ladder[f])));
      if (scale == 0.0f) continue;
      const float inv = __fdiv_rn(1.0f, scale);
      float err = 0.0f;
      uint32_t codes[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        int cq = (int)roundf(__fmul_rn(v[j], inv)) + 1;
        cq = cq < 0 ? 0 : cq > 3 ? 3 : cq;
        codes[j / 16] |= (uint32_t)cq << (2 * (j % 16));
        const float res = __fsub_rn(v[j], __fmul_rn((float)cq - 1.0f, scale));
        err = __fadd_rn(err, __fmul_rn(res, res));
      }
      if (err < best_err) {
        best_err = err;
        best_scale = scale;
#pragma unroll
        for (int i = 0; i < 4; ++i) best[i] = codes[i];
      }
    }
    dbits = __half_as_ushort(__float2half_rn(best_scale));
#pragma unroll
    for (int i = 0; i < 4; ++i) packed[i] = best[i];
  }
  // byte layout: d (2 bytes) then 16 code bytes, weight j at bits 2*(j%4) of byte j/4 (little-endian
  // words of 16 codes each hold exactly those bytes)
  o[0] = (uint8_t)(dbits & 0xff);
  o[1] = (uint8_t)(dbits >> 8);
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int by = 0; by < 4; ++by) o[2 + 4 * i + by] = (uint8_t)(packed[i] >> (8 * by));
}

}  // namespace moe

using namespace moe;

extern "C" moe_status moe_requantize_q2_0(int src_dtype, const void* src, int E, int N, int K, void* dst,
                                          void* stream) {
  if (!src || !dst) return fail(MOE_ERR_INVALID, "moe_requantize_q2_0: null pointer");
  if (E <= 0 || N <= 0 || K <= 0 || K % 64)
    return fail(MOE_ERR_INVALID, "moe_requantize_q2_0: need E, N > 0 and K a multiple of 64");
  int64_t row_bytes;
  if (src_dtype == MOE_DTYPE_BF16) row_bytes = (int64_t)K * 2;
  else if (src_dtype == MOE_DTYPE_Q8_0) row_bytes = (int64_t)K / 32 * 34;
  else if (src_dtype == MOE_DTYPE_Q4_K) {
    if (K % 256) return fail(MOE_ERR_INVALID, "moe_requantize_q2_0: Q4_K rows need K % 256 == 0");
    row_bytes = (int64_t)K / 256 * 144;
  } else {
    return fail(MOE_ERR_UNSUPPORTED, "moe_requantize_q2_0: source must be BF16, Q8_0 or Q4_K");
  }
  const int64_t rows = (int64_t)E * N;
  const int64_t blocks = rows * (K / 64);
  const int t = 128;
  requant_q2_0_kernel<<<(unsigned)((blocks + t - 1) / t), t, 0, static_cast<cudaStream_t>(stream)>>>(
      src_dtype, static_cast<const uint8_t*>(src), rows, K, row_bytes, static_cast<uint8_t*>(dst));
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}
