// cpu_kernels.cpp — the CPU expert path's row dot products (cpu_kernels.h).
//
// Three builds of each dot, the widest the host reports taken at the first call: AVX-512 (F, BW, VL)
// + FMA + F16C, AVX2 + FMA + F16C, and portable scalar code, so the library loads on any x86-64 host.
// The vector builds widen each Q8_0 block's 32 int8 once (2 x 16 or 4 x 8 lanes) and multiply them
// into every activation vector of the call, then scale the block's partial sums by d in one FMA.
// On hosts other than x86-64 (an aarch64 Grace host, say) only the scalar build is compiled.
#include "cpu_kernels.h"

#if defined(__x86_64__)
#define MOE_CPU_X86 1
#include <immintrin.h>
#else
#define MOE_CPU_X86 0
#endif

#include <cstdlib>
#include <cstring>

namespace moe {
namespace {

inline float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ffu, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: renormalise
      exp = 127 - 15 + 1;
      while (!(man & 0x400u)) {
        man <<= 1;
        --exp;
      }
      bits = sign | (exp << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline float bf16_to_float(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

void dot_q8_0_scalar(const uint8_t* row, const float* const* xs, int nx, int K, float* out) {
  float acc[CPU_DOT_MAX_X] = {};
  for (int b = 0; b < K / 32; ++b) {
    const uint8_t* blk = row + b * 34;
    uint16_t dh;
    std::memcpy(&dh, blk, 2);
    const float d = half_to_float(dh);
    const int8_t* q = reinterpret_cast<const int8_t*>(blk + 2);
    for (int j = 0; j < nx; ++j) {
      const float* x = xs[j] + b * 32;
      float s = 0.0f;
      for (int i = 0; i < 32; ++i) s += (float)q[i] * x[i];
      acc[j] += d * s;
    }
  }
  for (int j = 0; j < nx; ++j) out[j] = acc[j];
}

void dot_bf16_scalar(const uint16_t* row, const float* const* xs, int nx, int K, float* out) {
  for (int j = 0; j < nx; ++j) {
    float s = 0.0f;
    for (int i = 0; i < K; ++i) s += bf16_to_float(row[i]) * xs[j][i];
    out[j] = s;
  }
}

#if MOE_CPU_X86
__attribute__((target("avx2,fma"))) inline float hsum(__m256 v) {
  __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_movehdup_ps(s));
  return _mm_cvtss_f32(s);
}

template <int NX>
__attribute__((target("avx2,fma,f16c"))) void dot_q8_0_avx2(const uint8_t* row, const float* const* xs, int K,
                                                             float* out) {
  __m256 acc[NX];
  for (int j = 0; j < NX; ++j) acc[j] = _mm256_setzero_ps();
  for (int b = 0; b < K / 32; ++b) {
    const uint8_t* blk = row + b * 34;
    uint16_t dh;
    std::memcpy(&dh, blk, 2);
    const __m256 d = _mm256_set1_ps(_cvtsh_ss(dh));
    __m256 w[4];
    for (int u = 0; u < 4; ++u)
      w[u] = _mm256_cvtepi32_ps(
          _mm256_cvtepi8_epi32(_mm_loadl_epi64(reinterpret_cast<const __m128i*>(blk + 2 + 8 * u))));
    for (int j = 0; j < NX; ++j) {
      const float* x = xs[j] + b * 32;
      __m256 s = _mm256_mul_ps(w[0], _mm256_loadu_ps(x));
      s = _mm256_fmadd_ps(w[1], _mm256_loadu_ps(x + 8), s);
      s = _mm256_fmadd_ps(w[2], _mm256_loadu_ps(x + 16), s);
      s = _mm256_fmadd_ps(w[3], _mm256_loadu_ps(x + 24), s);
      acc[j] = _mm256_fmadd_ps(d, s, acc[j]);
    }
  }
  for (int j = 0; j < NX; ++j) out[j] = hsum(acc[j]);
}

template <int NX>
__attribute__((target("avx2,fma"))) void dot_bf16_avx2(const uint16_t* row, const float* const* xs, int K,
                                                        float* out) {
  __m256 acc[NX];
  for (int j = 0; j < NX; ++j) acc[j] = _mm256_setzero_ps();
  int i = 0;
  for (; i + 8 <= K; i += 8) {
    const __m256 w = _mm256_castsi256_ps(_mm256_slli_epi32(
        _mm256_cvtepu16_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(row + i))), 16));
    for (int j = 0; j < NX; ++j) acc[j] = _mm256_fmadd_ps(w, _mm256_loadu_ps(xs[j] + i), acc[j]);
  }
  for (int j = 0; j < NX; ++j) {
    float s = hsum(acc[j]);
    for (int t = i; t < K; ++t) s += bf16_to_float(row[t]) * xs[j][t];
    out[j] = s;
  }
}

#define MOE_AVX512 __attribute__((target("avx512f,avx512bw,avx512vl,fma,f16c")))

template <int NX>
MOE_AVX512 void dot_q8_0_avx512(const uint8_t* row, const float* const* xs, int K, float* out) {
  __m512 acc[NX];
  for (int j = 0; j < NX; ++j) acc[j] = _mm512_setzero_ps();
  for (int b = 0; b < K / 32; ++b) {
    const uint8_t* blk = row + b * 34;
    uint16_t dh;
    std::memcpy(&dh, blk, 2);
    const __m512 d = _mm512_set1_ps(_cvtsh_ss(dh));
    const __m512 w0 = _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(blk + 2))));
    const __m512 w1 =
        _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(blk + 18))));
    for (int j = 0; j < NX; ++j) {
      const float* x = xs[j] + b * 32;
      const __m512 s = _mm512_fmadd_ps(w1, _mm512_loadu_ps(x + 16), _mm512_mul_ps(w0, _mm512_loadu_ps(x)));
      acc[j] = _mm512_fmadd_ps(d, s, acc[j]);
    }
  }
  for (int j = 0; j < NX; ++j) out[j] = _mm512_reduce_add_ps(acc[j]);
}

template <int NX>
MOE_AVX512 void dot_bf16_avx512(const uint16_t* row, const float* const* xs, int K, float* out) {
  __m512 acc[NX];
  for (int j = 0; j < NX; ++j) acc[j] = _mm512_setzero_ps();
  int i = 0;
  for (; i + 16 <= K; i += 16) {
    const __m512 w = _mm512_castsi512_ps(_mm512_slli_epi32(
        _mm512_cvtepu16_epi32(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(row + i))), 16));
    for (int j = 0; j < NX; ++j) acc[j] = _mm512_fmadd_ps(w, _mm512_loadu_ps(xs[j] + i), acc[j]);
  }
  for (int j = 0; j < NX; ++j) {
    float s = _mm512_reduce_add_ps(acc[j]);
    for (int t = i; t < K; ++t) s += bf16_to_float(row[t]) * xs[j][t];
    out[j] = s;
  }
}

MOE_AVX512 void dot_q8_0_avx512_any(const uint8_t* row, const float* const* xs, int nx, int K, float* out) {
  switch (nx) {
    case 1: return dot_q8_0_avx512<1>(row, xs, K, out);
    case 2: return dot_q8_0_avx512<2>(row, xs, K, out);
    case 3: return dot_q8_0_avx512<3>(row, xs, K, out);
    default: return dot_q8_0_avx512<4>(row, xs, K, out);
  }
}

MOE_AVX512 void dot_bf16_avx512_any(const uint16_t* row, const float* const* xs, int nx, int K, float* out) {
  switch (nx) {
    case 1: return dot_bf16_avx512<1>(row, xs, K, out);
    case 2: return dot_bf16_avx512<2>(row, xs, K, out);
    case 3: return dot_bf16_avx512<3>(row, xs, K, out);
    default: return dot_bf16_avx512<4>(row, xs, K, out);
  }
}

__attribute__((target("avx2,fma,f16c"))) void dot_q8_0_avx2_any(const uint8_t* row, const float* const* xs, int nx,
                                                                 int K, float* out) {
  switch (nx) {
    case 1: return dot_q8_0_avx2<1>(row, xs, K, out);
    case 2: return dot_q8_0_avx2<2>(row, xs, K, out);
    case 3: return dot_q8_0_avx2<3>(row, xs, K, out);
    default: return dot_q8_0_avx2<4>(row, xs, K, out);
  }
}

__attribute__((target("avx2,fma"))) void dot_bf16_avx2_any(const uint16_t* row, const float* const* xs, int nx, int K,
                                                            float* out) {
  switch (nx) {
    case 1: return dot_bf16_avx2<1>(row, xs, K, out);
    case 2: return dot_bf16_avx2<2>(row, xs, K, out);
    case 3: return dot_bf16_avx2<3>(row, xs, K, out);
    default: return dot_bf16_avx2<4>(row, xs, K, out);
  }
}

#endif  // MOE_CPU_X86

// 2: AVX-512 (F, BW, VL) + FMA + F16C; 1: AVX2 + FMA + F16C; 0: scalar
int host_isa() {
  static const int isa = [] {
#if MOE_CPU_X86
    __builtin_cpu_init();
    const bool avx2 =
        __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") && __builtin_cpu_supports("f16c");
    const bool avx512 = avx2 && __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
                        __builtin_cpu_supports("avx512vl");
    int isa = avx512 ? 2 : avx2 ? 1 : 0;
    if (const char* cap = std::getenv("MOE_CPU_ISA")) {  // lowers the choice, never raises it
      if (std::strcmp(cap, "scalar") == 0) isa = 0;
      else if (std::strcmp(cap, "avx2") == 0 && isa > 1) isa = 1;
    }
    return isa;
#else
    return 0;
#endif
  }();
  return isa;
}

}  // namespace

void cpu_dot_q8_0(const uint8_t* row, const float* const* xs, int nx, int K, float* out) {
  for (int j0 = 0; j0 < nx; j0 += CPU_DOT_MAX_X) {  // the row stays in cache across the chunks
    const int n = nx - j0 < CPU_DOT_MAX_X ? nx - j0 : CPU_DOT_MAX_X;
    const int isa = host_isa();
#if MOE_CPU_X86
    if (isa == 2) dot_q8_0_avx512_any(row, xs + j0, n, K, out + j0);
    else if (isa == 1) dot_q8_0_avx2_any(row, xs + j0, n, K, out + j0);
    else dot_q8_0_scalar(row, xs + j0, n, K, out + j0);
#else
    (void)isa;
    dot_q8_0_scalar(row, xs + j0, n, K, out + j0);
#endif
  }
}

void cpu_dot_bf16(const uint16_t* row, const float* const* xs, int nx, int K, float* out) {
  for (int j0 = 0; j0 < nx; j0 += CPU_DOT_MAX_X) {
    const int n = nx - j0 < CPU_DOT_MAX_X ? nx - j0 : CPU_DOT_MAX_X;
    const int isa = host_isa();
#if MOE_CPU_X86
    if (isa == 2) dot_bf16_avx512_any(row, xs + j0, n, K, out + j0);
    else if (isa == 1) dot_bf16_avx2_any(row, xs + j0, n, K, out + j0);
    else dot_bf16_scalar(row, xs + j0, n, K, out + j0);
#else
    (void)isa;
    dot_bf16_scalar(row, xs + j0, n, K, out + j0);
#endif
  }
}

const char* cpu_dot_isa() {
  const int isa = host_isa();
  return isa == 2 ? "avx512" : isa == 1 ? "avx2" : "scalar";
}

}  // namespace moe
