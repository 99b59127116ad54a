/*
 * moe_oracle.c — CPU restatement of the naiwa-rs MoE-layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library and the timed CPU baseline. It is
 * never linked into libmoe_b200.so. Built with -ffp-contract=off so every fused multiply-add is
 * the explicit fmaf written here (the device code uses __fmaf_rn at the same places), which is
 * what makes the router logits, the top-k ids and the permutation bit-exact comparable.
 *
 * Reference paths are inside flaneur2020/naiwa-rs. The arithmetic of the reference's MoE kernels
 * sits in its un-vendored fork (mistralrs-quant / mistralrs-core 0.9.4 at fork base bac32a67,
 * candle-core 0.11.0, Cargo.toml:10-20); where that is the case the function names the public
 * algorithm it restates instead.
 */
#include "moe_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------------ */
/* scalar formats                                                                              */
/* ------------------------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float orc_f16_to_f32(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

uint16_t orc_f32_to_f16(float f) {
  _Float16 v = (_Float16)f; /* IEEE round-to-nearest-even */
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

float orc_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

uint16_t orc_f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);                                          /* RNE */
  return (uint16_t)(u >> 16);
}

/* OCP FP8 E4M3 ("fn": no infinities, S.1111.111 is NaN, max 448). */
float orc_fp8e4m3_to_f32(uint8_t b) {
  int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
  float v;
  if (e == 15 && m == 7) return NAN;
  if (e == 0) v = ldexpf((float)m, -9);
  else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -v : v;
}

uint8_t orc_f32_to_fp8e4m3(float f) {
  uint8_t sign = (f2u(f) >> 31) ? 0x80 : 0;
  float a = fabsf(f);
  if (a != a) return sign | 0x7f;
  if (a >= 448.0f) return sign | 0x7e; /* saturate */
  if (a < 0.015625f) {                 /* subnormal: m * 2^-9, rounds up into 0x08 at m = 8 */
    float q = nearbyintf(a * 512.0f);
    return sign | (uint8_t)q;
  }
  int ex;
  (void)frexpf(a, &ex);
  int E = ex - 1;                              /* a in [2^E, 2^(E+1)) */
  float m = nearbyintf((ldexpf(a, -E) - 1.0f) * 8.0f);
  if (m >= 8.0f) { m = 0.0f; E += 1; }
  int code = ((E + 7) << 3) | (int)m;
  if (code > 0x7e) code = 0x7e;
  return sign | (uint8_t)code;
}

/* Deterministic exp shared bit-for-bit with the device (csrc/moe_math.cuh): Cody-Waite
 * reduction x = n*ln2 + r with a two-constant ln2 split, then the degree-7 Taylor polynomial of
 * e^r in Horner form with fused multiply-adds, then exact scaling by 2^n. Relative error is below
 * 2 ulp on the normal range; identical operations on both sides give identical bits. */
float orc_exp(float x) {
  if (x != x) return x;
  if (x > 0x1.62e430p+6f) return INFINITY;
  if (x < -104.0f) return 0.0f;
  float n = rintf(x * 0x1.715476p+0f);
  float r = fmaf(-n, 0x1.62e400p-1f, x);
  r = fmaf(-n, 0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;
  p = fmaf(p, r, 0x1.6c16c2p-10f);
  p = fmaf(p, r, 0x1.111112p-7f);
  p = fmaf(p, r, 0x1.555556p-5f);
  p = fmaf(p, r, 0x1.555556p-3f);
  p = fmaf(p, r, 0x1.000000p-1f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  if (ni > 127) { p = p * 0x1p127f; ni -= 127; }
  if (ni < -126) { p = p * 0x1p-64f; ni += 64; }
  return p * u2f((uint32_t)(ni + 127) << 23);
}

float orc_sigmoid(float x) { return 1.0f / (1.0f + orc_exp(-x)); }

float orc_silu(float x) { return x / (1.0f + orc_exp(-x)); }

/* ------------------------------------------------------------------------------------------ */
/* block formats                                                                               */
/* ------------------------------------------------------------------------------------------ */

/* GGML Q8_0 (public ggml quantize_row_q8_0 reference): d = amax/127 stored as f16,
 * q = round-half-away(x / d). Layout pinned by reference src/moe/tests.rs:101-102 (34 B / 32). */
void orc_q8_0_quantize(const float* x, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / 32; ++b) {
    const float* xb = x + b * 32;
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(xb[i]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint8_t* o = out + b * 34;
    uint16_t dh = orc_f32_to_f16(d);
    memcpy(o, &dh, 2);
    for (int i = 0; i < 32; ++i) o[2 + i] = (uint8_t)(int8_t)roundf(xb[i] * id);
  }
}

void orc_q8_0_dequantize(const uint8_t* blocks, int64_t n, float* out) {
  for (int64_t b = 0; b < n / 32; ++b) {
    const uint8_t* o = blocks + b * 34;
    uint16_t dh;
    memcpy(&dh, o, 2);
    float d = orc_f16_to_f32(dh);
    for (int i = 0; i < 32; ++i) out[b * 32 + i] = d * (float)(int8_t)o[2 + i];
  }
}

/* Q2_0, the reference's resident-pool format (src/moe/resident.rs:29-45): 64 weights per 18-byte
 * block, an f16 scale d then 16 bytes of 2-bit codes (weight j at bits 2*(j%4) of byte j/4), weight
 * value (code - 1) * d, so codes 0..3 stand for -1, 0, +1, +2. The quantiser restates
 * resident.rs:46-88: d is searched over amax / {1, 1.25, 1.5, 1.75, 2}, each rounded to f16; a
 * weight's code is clamp(round(x / d) + 1, 0, 3) with round-half-away; the candidate with the
 * smallest squared error is kept, the first on ties; an all-zero block is d = 0 with every code 1
 * (so it decodes to zeros), and a block whose candidates all round to d = 0 keeps codes 0 and d = 0. */
void orc_q2_0_quantize(const float* x, int64_t n, uint8_t* out) {
  static const float ladder[5] = {1.0f, 1.25f, 1.5f, 1.75f, 2.0f};
  for (int64_t b = 0; b < n / 64; ++b) {
    const float* xb = x + b * 64;
    uint8_t* o = out + b * 18;
    float amax = 0.0f;
    for (int i = 0; i < 64; ++i) amax = fmaxf(amax, fabsf(xb[i]));
    memset(o + 2, 0, 16);
    if (amax == 0.0f) {
      o[0] = o[1] = 0;
      memset(o + 2, 0x55, 16);
      continue;
    }
    float best_err = INFINITY, best_scale = 0.0f;
    uint8_t best[64], codes[64];
    memset(best, 0, sizeof(best));
    for (int f = 0; f < 5; ++f) {
      const float scale = orc_f16_to_f32(orc_f32_to_f16(amax / ladder[f]));
      if (scale == 0.0f) continue;
      const float inv = 1.0f / scale;
      float err = 0.0f;
      for (int j = 0; j < 64; ++j) {
        int c = (int)roundf(xb[j] * inv) + 1;
        c = c < 0 ? 0 : c > 3 ? 3 : c;
        codes[j] = (uint8_t)c;
        const float res = xb[j] - ((float)c - 1.0f) * scale;
        err += res * res;
      }
      if (err < best_err) {
        best_err = err;
        best_scale = scale;
        memcpy(best, codes, 64);
      }
    }
    const uint16_t dh = orc_f32_to_f16(best_scale);
    memcpy(o, &dh, 2);
    for (int j = 0; j < 64; ++j) o[2 + j / 4] |= (uint8_t)(best[j] << (2 * (j % 4)));
  }
}

void orc_q2_0_dequantize(const uint8_t* blocks, int64_t n, float* out) {
  for (int64_t b = 0; b < n / 64; ++b) {
    const uint8_t* o = blocks + b * 18;
    uint16_t dh;
    memcpy(&dh, o, 2);
    const float d = orc_f16_to_f32(dh);
    for (int j = 0; j < 64; ++j) out[b * 64 + j] = ((float)((o[2 + j / 4] >> (2 * (j % 4))) & 3) - 1.0f) * d;
  }
}

/* GGML Q4_K (public ggml block_q4_K): 8 sub-blocks of 32 with 6-bit scale/min pairs packed in
 * 12 bytes, w = d*sc*q - dmin*m. The packing and unpacking below are the published
 * get_scale_min_k4 rule; the quantizer is this oracle's own (a min/max fit per sub-block),
 * because any valid encoding serves as synthetic input. */
static void q4k_get_scale_min(int j, const uint8_t* s, int* sc, int* m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (s[j + 4] & 0xf) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

void orc_q4_k_quantize(const float* x, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / 256; ++b) {
    const float* xb = x + b * 256;
    uint8_t* o = out + b * 144;
    float scale[8], minv[8], max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
      float mn = xb[32 * j], mx = xb[32 * j];
      for (int i = 1; i < 32; ++i) { mn = fminf(mn, xb[32 * j + i]); mx = fmaxf(mx, xb[32 * j + i]); }
      if (mn > 0.0f) mn = 0.0f;
      scale[j] = (mx - mn) / 15.0f;
      minv[j] = -mn;
      max_scale = fmaxf(max_scale, scale[j]);
      max_min = fmaxf(max_min, minv[j]);
    }
    uint16_t dh = orc_f32_to_f16(max_scale / 63.0f), dmh = orc_f32_to_f16(max_min / 63.0f);
    float d = orc_f16_to_f32(dh), dmin = orc_f16_to_f32(dmh);
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
      sc[j] = d > 0.0f ? (int)fminf(63.0f, nearbyintf(scale[j] / d)) : 0;
      m[j] = dmin > 0.0f ? (int)fminf(63.0f, nearbyintf(minv[j] / dmin)) : 0;
    }
    memcpy(o, &dh, 2);
    memcpy(o + 2, &dmh, 2);
    uint8_t* s = o + 4;
    for (int j = 0; j < 4; ++j) {
      s[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
      s[j + 4] = (uint8_t)(m[j] | ((m[j + 4] >> 4) << 6));
      s[j + 8] = (uint8_t)((sc[j + 4] & 0xf) | ((m[j + 4] & 0xf) << 4));
    }
    uint8_t* qs = o + 16;
    for (int c = 0; c < 4; ++c) {
      for (int l = 0; l < 32; ++l) {
        int q2[2];
        for (int h = 0; h < 2; ++h) {
          int j = 2 * c + h;
          float dj = d * (float)sc[j], mj = dmin * (float)m[j];
          float q = dj > 0.0f ? nearbyintf((xb[32 * j + l] + mj) / dj) : 0.0f;
          q2[h] = q < 0.0f ? 0 : (q > 15.0f ? 15 : (int)q);
        }
        qs[32 * c + l] = (uint8_t)(q2[0] | (q2[1] << 4));
      }
    }
  }
}

void orc_q4_k_dequantize(const uint8_t* blocks, int64_t n, float* out) {
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* o = blocks + b * 144;
    uint16_t dh, dmh;
    memcpy(&dh, o, 2);
    memcpy(&dmh, o + 2, 2);
    float d = orc_f16_to_f32(dh), dmin = orc_f16_to_f32(dmh);
    const uint8_t* s = o + 4;
    const uint8_t* qs = o + 16;
    float* y = out + b * 256;
    for (int c = 0; c < 4; ++c) {
      for (int h = 0; h < 2; ++h) {
        int sc, m;
        q4k_get_scale_min(2 * c + h, s, &sc, &m);
        float dj = d * (float)sc, mj = dmin * (float)m;
        for (int l = 0; l < 32; ++l) {
          int q = h ? (qs[32 * c + l] >> 4) : (qs[32 * c + l] & 0xf);
          y[64 * c + 32 * h + l] = dj * (float)q - mj;
        }
      }
    }
  }
}

/* FP8 e4m3 with 128x128 f32 block scales, the public DeepSeek-V3 weight format:
 * scale = amax(block)/448, q = e4m3(w / scale), w' = f32(q) * scale. */
void orc_fp8_b128_quantize(const float* w, int n, int k, uint8_t* q, float* scales) {
  int nb = n / 128, kb = k / 128;
  for (int bi = 0; bi < nb; ++bi)
    for (int bj = 0; bj < kb; ++bj) {
      float amax = 0.0f;
      for (int r = 0; r < 128; ++r)
        for (int c = 0; c < 128; ++c) amax = fmaxf(amax, fabsf(w[(int64_t)(bi * 128 + r) * k + bj * 128 + c]));
      float s = amax > 0.0f ? amax / 448.0f : 1.0f;
      scales[bi * kb + bj] = s;
      for (int r = 0; r < 128; ++r)
        for (int c = 0; c < 128; ++c) {
          int64_t i = (int64_t)(bi * 128 + r) * k + bj * 128 + c;
          q[i] = orc_f32_to_fp8e4m3(w[i] / s);
        }
    }
}

void orc_fp8_b128_dequantize(const uint8_t* q, const float* scales, int n, int k, float* out) {
  int kb = k / 128;
  for (int r = 0; r < n; ++r)
    for (int c = 0; c < k; ++c) {
      int64_t i = (int64_t)r * k + c;
      out[i] = orc_fp8e4m3_to_f32(q[i]) * scales[(r / 128) * kb + c / 128];
    }
}

int64_t orc_block_bytes(int dtype, int64_t n_weights) {
  switch (dtype) {
    case 0: return n_weights * 2;
    case 1: return n_weights / 32 * 34;
    case 2: return n_weights / 256 * 144;
    case 3: return n_weights;
    case 4: return n_weights / 64 * 18;
    default: return -1;
  }
}

/* src/moe/expert.rs:123-145: row-block formats never cross an expert, so expert e of a stacked
 * [E, N, K] tensor is bytes [e*stride, (e+1)*stride) with stride = N * (K/block) * type_size. */
int orc_expert_range(int dtype, int E, int N, int K, int e, int64_t* begin, int64_t* end) {
  int block = dtype == 1 ? 32 : dtype == 2 ? 256 : dtype == 4 ? 64 : 1;
  if (K % block != 0 || e < 0 || e >= E) return -1;
  int64_t stride = orc_block_bytes(dtype, (int64_t)N * K);
  *begin = (int64_t)e * stride;
  *end = *begin + stride;
  return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* cache policy — src/moe/cached_layer.rs                                                      */
/* ------------------------------------------------------------------------------------------ */

/* Rust f32::total_cmp order as a signed integer key. */
static inline int32_t total_key(float f) {
  int32_t b = (int32_t)f2u(f);
  return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

/* cached_layer.rs:358-363: indices of the k largest logits, largest first, ties lowest index. */
int orc_top_k_ids(const float* logits, int n, int k, int* out) {
  int take = k < n ? k : n;
  char* used = calloc((size_t)n, 1);
  for (int j = 0; j < take; ++j) {
    int best = -1;
    for (int i = 0; i < n; ++i) {
      if (used[i]) continue;
      if (best < 0 || total_key(logits[i]) > total_key(logits[best])) best = i;
    }
    used[best] = 1;
    out[j] = best;
  }
  free(used);
  return take;
}

/* cached_layer.rs:367-379: every expert once, by votes (desc), then best rank, then id. */
int orc_union_by_votes(const int* const* rankings, const int* lens, int n_rankings, int* out) {
  int max_id = -1;
  for (int r = 0; r < n_rankings; ++r)
    for (int i = 0; i < lens[r]; ++i)
      if (rankings[r][i] > max_id) max_id = rankings[r][i];
  if (max_id < 0) return 0;
  int* votes = calloc((size_t)max_id + 1, sizeof(int));
  int* best = malloc(((size_t)max_id + 1) * sizeof(int));
  for (int e = 0; e <= max_id; ++e) best[e] = 1 << 30;
  for (int r = 0; r < n_rankings; ++r)
    for (int i = 0; i < lens[r]; ++i) {
      int e = rankings[r][i];
      votes[e] += 1;
      if (i < best[e]) best[e] = i;
    }
  int n = 0;
  for (int e = 0; e <= max_id; ++e)
    if (votes[e] > 0) out[n++] = e;
  /* insertion sort by (votes desc, best rank asc, id asc) */
  for (int i = 1; i < n; ++i) {
    int v = out[i], j = i - 1;
    while (j >= 0) {
      int u = out[j];
      int before = votes[v] > votes[u] || (votes[v] == votes[u] && (best[v] < best[u] || (best[v] == best[u] && v < u)));
      if (!before) break;
      out[j + 1] = u;
      --j;
    }
    out[j + 1] = v;
  }
  free(votes);
  free(best);
  return n;
}

/* cached_layer.rs:385-398: distinct missed experts ranked by summed router weight (total_cmp
 * desc, then id), truncated to min(ceil(frac * distinct), cap). Rows are concatenated in ids/ws
 * with row_lens giving each row's length. */
int orc_streamed_misses(const uint32_t* ids, const float* ws, const int* row_lens, int rows, float frac, int cap,
                        uint32_t* out) {
  if (frac <= 0.0f || cap == 0) return 0;
  int total = 0;
  for (int r = 0; r < rows; ++r) total += row_lens[r];
  uint32_t* uid = malloc(sizeof(uint32_t) * (size_t)(total + 1));
  float* wsum = malloc(sizeof(float) * (size_t)(total + 1));
  int nu = 0;
  for (int i = 0; i < total; ++i) {
    int f = -1;
    for (int j = 0; j < nu; ++j)
      if (uid[j] == ids[i]) { f = j; break; }
    if (f < 0) { uid[nu] = ids[i]; wsum[nu] = 0.0f; f = nu++; }
    wsum[f] += ws[i];
  }
  int take = (int)ceilf(frac * (float)nu);
  if (take > cap) take = cap;
  for (int i = 1; i < nu; ++i) {
    uint32_t a = uid[i];
    float wa = wsum[i];
    int j = i - 1;
    while (j >= 0 && (total_key(wa) > total_key(wsum[j]) || (total_key(wa) == total_key(wsum[j]) && a < uid[j]))) {
      uid[j + 1] = uid[j];
      wsum[j + 1] = wsum[j];
      --j;
    }
    uid[j + 1] = a;
    wsum[j + 1] = wa;
  }
  if (take > nu) take = nu;
  memcpy(out, uid, sizeof(uint32_t) * (size_t)take);
  free(uid);
  free(wsum);
  return take;
}

/* cached_layer.rs:401-410: the least recently used published resident outside `protect`,
 * ties to the lower expert id. */
int orc_lru_victim(const int* slot_expert, const int* slot_published, const uint64_t* last_use, int n_slots,
                   const int* protect, int n_protect, int* expert_out) {
  int best = -1;
  for (int s = 0; s < n_slots; ++s) {
    int e = slot_expert[s];
    if (e < 0 || !slot_published[s]) continue;
    int prot = 0;
    for (int p = 0; p < n_protect; ++p) prot |= protect[p] == e;
    if (prot) continue;
    if (best < 0 || last_use[s] < last_use[best] || (last_use[s] == last_use[best] && e < slot_expert[best])) best = s;
  }
  if (best >= 0 && expert_out) *expert_out = slot_expert[best];
  return best;
}

/* cached_layer.rs:344-355: the most routed expert not in a slot (ties lowest id); -1 when every
 * slot is taken or every expert is placed. */
int orc_fill_candidate(const int* slot_expert, int n_slots, const uint64_t* hit_counts, int n_experts) {
  int full = 1;
  for (int s = 0; s < n_slots; ++s) full &= slot_expert[s] >= 0;
  if (full) return -1;
  int best = -1;
  for (int e = 0; e < n_experts; ++e) {
    int taken = 0;
    for (int s = 0; s < n_slots; ++s) taken |= slot_expert[s] == e;
    if (taken) continue;
    if (best < 0 || hit_counts[e] > hit_counts[best]) best = e;
  }
  return best;
}

/* ------------------------------------------------------------------------------------------ */
/* router                                                                                      */
/* ------------------------------------------------------------------------------------------ */

/* logits[t, e] = x_t . w_e in f32 with a fixed reduction order that the device kernel follows
 * exactly: the row is cut into 8-element chunks, lane l of 32 owns chunks l, l+32, l+64, ... and
 * accumulates them in order with fused multiply-adds, then the 32 partial sums meet in a
 * butterfly (offsets 16, 8, 4, 2, 1; each step adds the partner's value to the own value).
 * Products of two bf16 are exact in f32. The router GEMV itself is in the reference's fork
 * (upstream of RoutedExperts::forward); its CPU copy for prediction is cached_layer.rs:1241-1242. */
void orc_router_logits(const uint16_t* x_bf16, const uint16_t* w_bf16, int T, int H, int E, float* logits) {
  int chunks = H / 8;
  for (int t = 0; t < T; ++t)
    for (int e = 0; e < E; ++e) {
      float acc[32], nxt[32];
      for (int l = 0; l < 32; ++l) {
        float a = 0.0f;
        for (int c = l; c < chunks; c += 32)
          for (int j = 0; j < 8; ++j) {
            int h = c * 8 + j;
            a = fmaf(orc_bf16_to_f32(x_bf16[(int64_t)t * H + h]), orc_bf16_to_f32(w_bf16[(int64_t)e * H + h]), a);
          }
        acc[l] = a;
      }
      for (int off = 16; off >= 1; off >>= 1) {
        for (int l = 0; l < 32; ++l) nxt[l] = acc[l] + acc[l ^ off];
        memcpy(acc, nxt, sizeof(acc));
      }
      logits[(int64_t)t * E + e] = acc[0];
    }
}

/* Sum of v[0..n) in the device's warp order: lane l adds v[l], v[l+32], ... then a butterfly. */
static float warp_order_sum(const float* v, int n) {
  float acc[32], nxt[32];
  for (int l = 0; l < 32; ++l) {
    float a = 0.0f;
    for (int i = l; i < n; i += 32) a = a + v[i];
    acc[l] = a;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    for (int l = 0; l < 32; ++l) nxt[l] = acc[l] + acc[l ^ off];
    memcpy(acc, nxt, sizeof(acc));
  }
  return acc[0];
}

/* Router modes (the fork's router is not in the reference tree; these restate the public model
 * descriptions the configs name):
 *  0 softmax over all E, top-k by logit, weight = p_j;
 *  1 top-k by logit, weight = e^(l_j - l_max) / sum_i<k e^(l_i - l_max)  (softmax renormalised
 *    over the k, Qwen3-MoE norm_topk_prob);
 *  2 DeepSeek-V3: s = sigmoid(l), selection score s + bias, group score = top-1 + top-2 of its
 *    group, keep topk_group groups, top-k inside them, weight = s_j / (sum_i s_i + 1e-20) * scale.
 * All rankings use the total order of cached_layer.rs:358-363 (ties to the lowest index). */
int orc_route(const float* logits, const float* bias, int T, int E, int k, int mode, int n_group, int topk_group,
              float routed_scale, uint32_t* ids, float* weights) {
  if (k > E || k <= 0) return -1;
  float* tmp = malloc(sizeof(float) * (size_t)E);
  float* sel = malloc(sizeof(float) * (size_t)E);
  int* order = malloc(sizeof(int) * (size_t)E);
  for (int t = 0; t < T; ++t) {
    const float* l = logits + (int64_t)t * E;
    uint32_t* id = ids + (int64_t)t * k;
    float* w = weights + (int64_t)t * k;
    if (mode == 0 || mode == 1) {
      orc_top_k_ids(l, E, k, order);
      float m = l[order[0]];
      if (mode == 0) {
        for (int e = 0; e < E; ++e) tmp[e] = orc_exp(l[e] - m);
        float z = warp_order_sum(tmp, E);
        for (int j = 0; j < k; ++j) { id[j] = (uint32_t)order[j]; w[j] = orc_exp(l[order[j]] - m) / z; }
      } else {
        float z = 0.0f;
        for (int j = 0; j < k; ++j) { tmp[j] = orc_exp(l[order[j]] - m); z = z + tmp[j]; }
        for (int j = 0; j < k; ++j) { id[j] = (uint32_t)order[j]; w[j] = tmp[j] / z; }
      }
    } else if (mode == 2) {
      if (n_group <= 0 || E % n_group != 0 || topk_group <= 0 || topk_group > n_group) { free(tmp); free(sel); free(order); return -1; }
      int gs = E / n_group;
      for (int e = 0; e < E; ++e) {
        tmp[e] = orc_sigmoid(l[e]);
        sel[e] = bias ? tmp[e] + bias[e] : tmp[e];
      }
      float gscore[256];
      int gtop[2];
      for (int g = 0; g < n_group; ++g) {
        int nt = orc_top_k_ids(sel + g * gs, gs, 2, gtop);
        gscore[g] = nt == 2 ? sel[g * gs + gtop[0]] + sel[g * gs + gtop[1]] : sel[g * gs + gtop[0]];
      }
      int gsel[256];
      orc_top_k_ids(gscore, n_group, topk_group, gsel);
      float* masked = malloc(sizeof(float) * (size_t)E);
      for (int e = 0; e < E; ++e) masked[e] = -INFINITY;
      for (int i = 0; i < topk_group; ++i)
        for (int j = 0; j < gs; ++j) masked[gsel[i] * gs + j] = sel[gsel[i] * gs + j];
      orc_top_k_ids(masked, E, k, order);
      free(masked);
      float z = 0.0f;
      for (int j = 0; j < k; ++j) z = z + tmp[order[j]];
      z = z + 1e-20f;
      for (int j = 0; j < k; ++j) { id[j] = (uint32_t)order[j]; w[j] = tmp[order[j]] / z * routed_scale; }
    } else {
      free(tmp); free(sel); free(order);
      return -1;
    }
  }
  free(tmp);
  free(sel);
  free(order);
  return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* permute                                                                                     */
/* ------------------------------------------------------------------------------------------ */

/* Stable counting sort of the routed pairs by expert. The reference groups pairs per bank in
 * pair order (gpu.rs:103-132) and per row in input order (rings.rs:146-156); a stable sort keeps
 * exactly that order inside each expert. Ids equal to 0xFFFFFFFF (the library's MOE_ID_NONE, an
 * empty slot) are skipped; returns -1 on any other id >= E (route.rs:52-68). */
int orc_permute(const uint32_t* ids, int n_pairs, int E, int32_t* counts, int32_t* offsets, int32_t* perm,
                int32_t* active, int32_t* n_active) {
  if (E <= 0 || n_pairs < 0) return -1;
  for (int e = 0; e < E; ++e) counts[e] = 0;
  for (int p = 0; p < n_pairs; ++p) {
    if (ids[p] == 0xFFFFFFFFu) continue;
    if (ids[p] >= (uint32_t)E) return -1;
    counts[ids[p]]++;
  }
  offsets[0] = 0;
  for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
  int32_t* fill = calloc((size_t)E, sizeof(int32_t));
  for (int p = 0; p < n_pairs; ++p) {
    uint32_t e = ids[p];
    if (e == 0xFFFFFFFFu) continue;
    perm[offsets[e] + fill[e]++] = p;
  }
  free(fill);
  int na = 0;
  for (int e = 0; e < E; ++e)
    if (counts[e] > 0) active[na++] = e;
  *n_active = na;
  return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* expert FFN + combine                                                                        */
/* ------------------------------------------------------------------------------------------ */

/* The dequantised reference the reference's own tests compare against
 * (prefill_stream.rs:1936-1950 and the fallback run_expert, gpu.rs:162-167):
 * y_t = sum_j w_tj * down_e(silu(gate_e x_t) * up_e x_t), accumulated in double. */
void orc_moe_forward_f32(const float* x, const uint32_t* ids, const float* w, int T, int k, int E, int H, int I,
                         const float* gate, const float* up, const float* down, float* y) {
  double* h = malloc(sizeof(double) * (size_t)I);
  double* acc = malloc(sizeof(double) * (size_t)H);
  for (int t = 0; t < T; ++t) {
    const float* xt = x + (int64_t)t * H;
    for (int n = 0; n < H; ++n) acc[n] = 0.0;
    for (int j = 0; j < k; ++j) {
      uint32_t e = ids[(int64_t)t * k + j];
      double wt = w[(int64_t)t * k + j];
      if (e >= (uint32_t)E) continue;
      const float* g = gate + (int64_t)e * I * H;
      const float* u = up + (int64_t)e * I * H;
      const float* d = down + (int64_t)e * H * I;
      for (int n = 0; n < I; ++n) {
        double sg = 0.0, su = 0.0;
        for (int c = 0; c < H; ++c) {
          sg += (double)g[(int64_t)n * H + c] * xt[c];
          su += (double)u[(int64_t)n * H + c] * xt[c];
        }
        h[n] = sg / (1.0 + exp(-sg)) * su;
      }
      for (int n = 0; n < H; ++n) {
        double s = 0.0;
        for (int c = 0; c < I; ++c) s += (double)d[(int64_t)n * I + c] * h[c];
        acc[n] += wt * s;
      }
    }
    for (int n = 0; n < H; ++n) y[(int64_t)t * H + n] = (float)acc[n];
  }
  free(h);
  free(acc);
}

/* The same dequantised reference over quantised stacks, computed expert by expert on n_threads so
 * that full-size layers (config 3's 512-token chunks, config 5's 7168 x 2048 FP8 experts) can be
 * checked on every token: only one expert's f32 weights exist at a time, and the token sums run in
 * double. Per token the experts are added in expert order instead of slot order, which moves the
 * double sum by far less than one f32 ulp of the result. Returns -1 on bad arguments. */
typedef struct {
  int dtype, E, H, I, T, k;
  const uint8_t *gate, *up, *down;
  const float *gs, *us, *ds;
  const float* x;
  const float* w;
  int e;                 /* current expert */
  const int* pairs;      /* its pairs (t * k + j), in pair order */
  int np;
  float *fg, *fu, *fd;   /* its dequantised [I, H], [I, H], [H, I] */
  double* h;             /* [np, I] */
  double* yp;            /* [np, H] */
  double* acc;           /* [T, H] */
  atomic_int next;
  int phase;
} ref_job;

static void dequant_rows(int dtype, const uint8_t* q, const float* scales, int N, int K, int r0, int r1, float* out) {
  const int64_t row_bytes = orc_block_bytes(dtype, K);
  if (dtype == 3) { /* FP8: the block scale of (row, column) */
    const int kb = K / 128;
    for (int r = r0; r < r1; ++r)
      for (int c = 0; c < K; ++c)
        out[(int64_t)r * K + c] = orc_fp8e4m3_to_f32(q[(int64_t)r * K + c]) * scales[(r / 128) * kb + c / 128];
    return;
  }
  for (int r = r0; r < r1; ++r) {
    const uint8_t* src = q + (int64_t)r * row_bytes;
    float* dst = out + (int64_t)r * K;
    if (dtype == 0) {
      for (int c = 0; c < K; ++c) {
        uint16_t b;
        memcpy(&b, src + 2 * c, 2);
        dst[c] = orc_bf16_to_f32(b);
      }
    } else if (dtype == 1) {
      orc_q8_0_dequantize(src, K, dst);
    } else if (dtype == 4) {
      orc_q2_0_dequantize(src, K, dst);
    } else {
      orc_q4_k_dequantize(src, K, dst);
    }
  }
}

static double dot_f64(const float* a, const double* b, int n) {
  double s[4] = {0, 0, 0, 0};
  int i = 0;
  for (; i + 4 <= n; i += 4)
    for (int l = 0; l < 4; ++l) s[l] += (double)a[i + l] * b[i + l];
  for (; i < n; ++i) s[0] += (double)a[i] * b[i];
  return (s[0] + s[1]) + (s[2] + s[3]);
}

static double dot_f32x(const float* a, const float* b, int n) {
  double s[4] = {0, 0, 0, 0};
  int i = 0;
  for (; i + 4 <= n; i += 4)
    for (int l = 0; l < 4; ++l) s[l] += (double)a[i + l] * b[i + l];
  for (; i < n; ++i) s[0] += (double)a[i] * b[i];
  return (s[0] + s[1]) + (s[2] + s[3]);
}

static void* ref_worker(void* arg) {
  ref_job* J = (ref_job*)arg;
  const int CH = 32;
  const int e = J->e, H = J->H, I = J->I;
  if (J->phase == 0) { /* dequantise the expert: items are 32-row chunks of the three matrices */
    const int gi = (I + CH - 1) / CH, di = (H + CH - 1) / CH;
    for (;;) {
      int it = atomic_fetch_add(&J->next, 1);
      if (it >= 2 * gi + di) break;
      const int64_t gub = orc_block_bytes(J->dtype, (int64_t)I * H);
      const int scn = J->dtype == 3 ? (I / 128) * (H / 128) : 0;
      if (it < 2 * gi) {
        const int which = it / gi, r0 = (it % gi) * CH, r1 = r0 + CH < I ? r0 + CH : I;
        const uint8_t* src = (which ? J->up : J->gate) + (int64_t)e * gub;
        const float* sc = J->dtype == 3 ? (which ? J->us : J->gs) + (int64_t)e * scn : NULL;
        dequant_rows(J->dtype, src, sc, I, H, r0, r1, which ? J->fu : J->fg);
      } else {
        const int r0 = (it - 2 * gi) * CH, r1 = r0 + CH < H ? r0 + CH : H;
        const float* sc = J->dtype == 3 ? J->ds + (int64_t)e * scn : NULL;
        dequant_rows(J->dtype, J->down + (int64_t)e * gub, sc, H, I, r0, r1, J->fd);
      }
    }
  } else if (J->phase == 1) { /* h = silu(gate x) * (up x) per pair, in double */
    const int per = (I + CH - 1) / CH;
    for (;;) {
      int it = atomic_fetch_add(&J->next, 1);
      if (it >= J->np * per) break;
      const int q = it / per, n0 = (it % per) * CH, n1 = n0 + CH < I ? n0 + CH : I;
      const float* xt = J->x + (int64_t)(J->pairs[q] / J->k) * H;
      for (int n = n0; n < n1; ++n) {
        const double sg = dot_f32x(J->fg + (int64_t)n * H, xt, H);
        const double su = dot_f32x(J->fu + (int64_t)n * H, xt, H);
        J->h[(int64_t)q * I + n] = sg / (1.0 + exp(-sg)) * su;
      }
    }
  } else if (J->phase == 2) { /* down per pair */
    const int per = (H + CH - 1) / CH;
    for (;;) {
      int it = atomic_fetch_add(&J->next, 1);
      if (it >= J->np * per) break;
      const int q = it / per, n0 = (it % per) * CH, n1 = n0 + CH < H ? n0 + CH : H;
      for (int n = n0; n < n1; ++n) J->yp[(int64_t)q * H + n] = dot_f64(J->fd + (int64_t)n * I, J->h + (int64_t)q * I, I);
    }
  } else { /* weighted sum into the tokens, pairs in order, by column chunk */
    const int per = (H + CH - 1) / CH;
    for (;;) {
      int it = atomic_fetch_add(&J->next, 1);
      if (it >= per) break;
      const int n0 = it * CH, n1 = n0 + CH < H ? n0 + CH : H;
      for (int q = 0; q < J->np; ++q) {
        const int p = J->pairs[q];
        const double wt = J->w[p];
        double* at = J->acc + (int64_t)(p / J->k) * H;
        for (int n = n0; n < n1; ++n) at[n] += wt * J->yp[(int64_t)q * H + n];
      }
    }
  }
  return NULL;
}

int orc_moe_forward_ref(int dtype, const uint8_t* gate, const uint8_t* up, const uint8_t* down, const float* gs,
                        const float* us, const float* ds, const float* x, const uint32_t* ids, const float* w, int T,
                        int k, int E, int H, int I, int n_threads, float* y) {
  if (dtype < 0 || dtype > 4 || T < 0 || k <= 0 || E <= 0 || H <= 0 || I <= 0) return -1;
  if ((dtype == 3 && (H % 128 || I % 128 || !gs || !us || !ds)) || (dtype == 1 && (H % 32 || I % 32)) ||
      (dtype == 2 && (H % 256 || I % 256)) || (dtype == 4 && (H % 64 || I % 64)))
    return -1;
  if (n_threads < 1) n_threads = 1;
  const int n = T * k;
  int* count = calloc((size_t)E, sizeof(int));
  for (int p = 0; p < n; ++p)
    if (ids[p] < (uint32_t)E) count[ids[p]]++;
  int maxc = 0;
  for (int e = 0; e < E; ++e) maxc = count[e] > maxc ? count[e] : maxc;
  ref_job J;
  memset(&J, 0, sizeof(J));
  J.dtype = dtype; J.E = E; J.H = H; J.I = I; J.T = T; J.k = k;
  J.gate = gate; J.up = up; J.down = down; J.gs = gs; J.us = us; J.ds = ds; J.x = x; J.w = w;
  int* pairs = malloc(sizeof(int) * (size_t)(maxc > 0 ? maxc : 1));
  J.pairs = pairs;
  J.fg = malloc(sizeof(float) * (size_t)I * H);
  J.fu = malloc(sizeof(float) * (size_t)I * H);
  J.fd = malloc(sizeof(float) * (size_t)H * I);
  J.h = malloc(sizeof(double) * (size_t)(maxc > 0 ? maxc : 1) * I);
  J.yp = malloc(sizeof(double) * (size_t)(maxc > 0 ? maxc : 1) * H);
  J.acc = calloc((size_t)T * H + 1, sizeof(double));
  pthread_t* th = malloc(sizeof(pthread_t) * (size_t)n_threads);
  for (int e = 0; e < E; ++e) {
    if (!count[e]) continue;
    int np = 0;
    for (int p = 0; p < n; ++p)
      if (ids[p] == (uint32_t)e) pairs[np++] = p;
    J.e = e;
    J.np = np;
    for (int phase = 0; phase < 4; ++phase) {
      J.phase = phase;
      atomic_store(&J.next, 0);
      for (int i = 1; i < n_threads; ++i) pthread_create(&th[i], NULL, ref_worker, &J);
      ref_worker(&J);
      for (int i = 1; i < n_threads; ++i) pthread_join(th[i], NULL);
    }
  }
  for (int64_t i = 0; i < (int64_t)T * H; ++i) y[i] = (float)J.acc[i];
  free(th);
  free(pairs);
  free(J.fg);
  free(J.fu);
  free(J.fd);
  free(J.h);
  free(J.yp);
  free(J.acc);
  free(count);
  return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* timed CPU baseline                                                                          */
/* ------------------------------------------------------------------------------------------ */

/* Restates the reference's CPU expert path, mistralrs_quant::fused_moe_decode as described at
 * src/moe/stages/cpu_miss.rs:13-54: pass 1 runs gate+up+SiLU once per distinct (expert, row)
 * pair with a non-zero weight (weight-0 padding is skipped, cpu_miss.rs:90-100); pass 2 runs down
 * and the router-weighted sum per row. Activations stay f32 (the x86 fused kernel keeps them f32,
 * prefill_stream.rs:1960-1963); weights are read as Q8_0 blocks and dequantised on the fly.
 * Work items are spread over n_threads with a shared atomic counter. */
static inline float q8_dot(const uint8_t* row_blocks, const float* x, int K) {
  float sum = 0.0f;
  for (int b = 0; b < K / 32; ++b) {
    const uint8_t* o = row_blocks + (int64_t)b * 34;
    uint16_t dh;
    memcpy(&dh, o, 2);
    const int8_t* q = (const int8_t*)(o + 2);
    const float* xb = x + b * 32;
    float s[8] = {0};
    for (int i = 0; i < 32; ++i) s[i & 7] += (float)q[i] * xb[i]; /* 8 lanes: vectorises */
    sum += orc_f16_to_f32(dh) * (((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7])));
  }
  return sum;
}

typedef struct {
  const uint8_t *gate, *up, *down;
  const float* x;
  const uint32_t* ids;
  const float* w;
  int T, k, E, H, I;
  int n_pairs;
  const int* pair_e;
  const int* pair_t;
  int* slot_of; /* [T*k] -> pair index or -1 */
  float* h;     /* [n_pairs, I] */
  float* y;
  atomic_int next;
  int phase;
  int chunk;
} fused_job;

static void* fused_worker(void* arg) {
  fused_job* J = (fused_job*)arg;
  const int64_t grow = (int64_t)J->H / 32 * 34; /* bytes of one gate/up row */
  const int64_t drow = (int64_t)J->I / 32 * 34; /* bytes of one down row */
  if (J->phase == 1) {
    int per = (J->I + J->chunk - 1) / J->chunk;
    int items = J->n_pairs * per;
    for (;;) {
      int it = atomic_fetch_add(&J->next, 1);
      if (it >= items) break;
      int p = it / per, c0 = (it % per) * J->chunk, c1 = c0 + J->chunk < J->I ? c0 + J->chunk : J->I;
      int e = J->pair_e[p];
      const float* xt = J->x + (int64_t)J->pair_t[p] * J->H;
      const uint8_t* g = J->gate + (int64_t)e * J->I * grow;
      const uint8_t* u = J->up + (int64_t)e * J->I * grow;
      for (int n = c0; n < c1; ++n) {
        float gv = q8_dot(g + n * grow, xt, J->H), uv = q8_dot(u + n * grow, xt, J->H);
        J->h[(int64_t)p * J->I + n] = gv / (1.0f + expf(-gv)) * uv;
      }
    }
  } else {
    int per = (J->H + J->chunk - 1) / J->chunk;
    int items = J->T * per;
    for (;;) {
      int it = atomic_fetch_add(&J->next, 1);
      if (it >= items) break;
      int t = it / per, c0 = (it % per) * J->chunk, c1 = c0 + J->chunk < J->H ? c0 + J->chunk : J->H;
      float* yt = J->y + (int64_t)t * J->H;
      for (int n = c0; n < c1; ++n) yt[n] = 0.0f;
      for (int j = 0; j < J->k; ++j) {
        int p = J->slot_of[t * J->k + j];
        if (p < 0) continue;
        float wt = J->w[t * J->k + j];
        int e = J->pair_e[p];
        const uint8_t* d = J->down + (int64_t)e * J->H * drow;
        const float* hp = J->h + (int64_t)p * J->I;
        for (int n = c0; n < c1; ++n) yt[n] += wt * q8_dot(d + n * drow, hp, J->I);
      }
    }
  }
  return NULL;
}

int orc_fused_moe_decode_q8_0(const uint8_t* gate, const uint8_t* up, const uint8_t* down, const float* x,
                              const uint32_t* ids, const float* w, int T, int k, int E, int H, int I, int n_threads,
                              float* y) {
  if (H % 32 || I % 32) return -1;
  int n = T * k;
  int* pair_e = malloc(sizeof(int) * (size_t)n);
  int* pair_t = malloc(sizeof(int) * (size_t)n);
  int* slot_of = malloc(sizeof(int) * (size_t)n);
  int np = 0;
  for (int i = 0; i < n; ++i) {
    slot_of[i] = -1;
    if (ids[i] >= (uint32_t)E) { free(pair_e); free(pair_t); free(slot_of); return -1; }
    if (w[i] == 0.0f) continue;
    int t = i / k, found = -1;
    for (int q = 0; q < np; ++q)
      if (pair_t[q] == t && pair_e[q] == (int)ids[i]) { found = q; break; }
    if (found < 0) { pair_e[np] = (int)ids[i]; pair_t[np] = t; found = np++; }
    slot_of[i] = found;
  }
  float* h = malloc(sizeof(float) * (size_t)(np > 0 ? np : 1) * I);
  fused_job J;
  memset(&J, 0, sizeof(J));
  J.gate = gate; J.up = up; J.down = down; J.x = x; J.ids = ids; J.w = w;
  J.T = T; J.k = k; J.E = E; J.H = H; J.I = I; J.n_pairs = np;
  J.pair_e = pair_e; J.pair_t = pair_t; J.slot_of = slot_of; J.h = h; J.y = y;
  if (n_threads < 1) n_threads = 1;
  pthread_t* th = malloc(sizeof(pthread_t) * (size_t)n_threads);
  for (int phase = 1; phase <= 2; ++phase) {
    J.phase = phase;
    J.chunk = 64;
    atomic_store(&J.next, 0);
    for (int i = 1; i < n_threads; ++i) pthread_create(&th[i], NULL, fused_worker, &J);
    fused_worker(&J);
    for (int i = 1; i < n_threads; ++i) pthread_join(th[i], NULL);
  }
  free(th);
  free(h);
  free(pair_e);
  free(pair_t);
  free(slot_of);
  return 0;
}
