/*
 * cpu_baseline.c — the reference's CPU expert path restated for speed, for timing only.
 *
 * TEST INFRASTRUCTURE ONLY: bench.py times it as the reference arm (--impl reference) and as the
 * cpu_baseline leg; nothing in libmoe_b200.so links or calls it, and the parity tests keep using the
 * strict-order oracle in moe_oracle.c as the checker (tests/test_oracle.py pins this file to it).
 *
 * What it restates: the miss stage's CPU decode, mistralrs_quant::fused_moe_decode as the reference
 * calls it (src/moe/stages/cpu_miss.rs:21-54, CpuExperts::forward src/moe/expert.rs:59-117). The
 * fused kernel itself lives in the reference's un-vendored fork; its structure as the reference
 * describes it is two passes over Q8_0 weights with f32 activations (prefill_stream.rs:1960-1963):
 *   pass 1: gate+up+SiLU once per distinct (expert, row) pair with a non-zero routing weight
 *           (weight-0 padding is skipped, cpu_miss.rs:90-100);
 *   pass 2: down, then the router-weighted sum per row.
 * It runs on a thread pool (the reference uses rayon). This restatement is written to be fast, not
 * to follow a fixed summation order: AVX2 + FMA + F16C, and each expert's weight rows are read once
 * per call and multiplied into every token routed to that expert (up to four tokens per register
 * block), so a call streams each active expert's 5,013,504 Q8_0 bytes once, the DRAM-bound cost
 * the reference measures (design.md:248-249).
 *
 * Threads: a persistent pool created by the first call with a given thread count (the calling
 * thread takes part); work items are handed out by an atomic counter.
 */
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define BL_MAX_THREADS 256
#define BL_ROWS 16  /* weight rows per work item */
#define BL_NX 4     /* tokens per register block */

/* ---- thread pool ---------------------------------------------------------------------------- */

typedef void (*bl_fn)(void* ctx, int item);

typedef struct {
  pthread_mutex_t mu;
  pthread_cond_t go, done;
  int n_threads;    /* including the caller */
  uint64_t gen;     /* bumped per parallel_for */
  int running;      /* workers still inside the current job */
  bl_fn fn;
  void* ctx;
  int items;
  atomic_int next;
  pthread_t th[BL_MAX_THREADS];
} bl_pool;

static bl_pool* g_pool = NULL;
static pthread_mutex_t g_pool_mu = PTHREAD_MUTEX_INITIALIZER;

static void bl_drain(bl_pool* p) {
  for (;;) {
    int it = atomic_fetch_add(&p->next, 1);
    if (it >= p->items) break;
    p->fn(p->ctx, it);
  }
}

static void* bl_worker(void* arg) {
  bl_pool* p = (bl_pool*)arg;
  uint64_t seen = 0;
  for (;;) {
    pthread_mutex_lock(&p->mu);
    while (p->gen == seen) pthread_cond_wait(&p->go, &p->mu);
    seen = p->gen;
    pthread_mutex_unlock(&p->mu);
    bl_drain(p);
    pthread_mutex_lock(&p->mu);
    if (--p->running == 0) pthread_cond_signal(&p->done);
    pthread_mutex_unlock(&p->mu);
  }
  return NULL;
}

static bl_pool* bl_get_pool(int n_threads) {
  pthread_mutex_lock(&g_pool_mu);
  if (!g_pool || g_pool->n_threads != n_threads) {
    /* a pool with another size is left running idle: the baseline uses one size per process */
    bl_pool* p = calloc(1, sizeof(bl_pool));
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->go, NULL);
    pthread_cond_init(&p->done, NULL);
    p->n_threads = n_threads;
    for (int i = 1; i < n_threads; ++i) pthread_create(&p->th[i], NULL, bl_worker, p);
    g_pool = p;
  }
  bl_pool* p = g_pool;
  pthread_mutex_unlock(&g_pool_mu);
  return p;
}

static void bl_parallel_for(bl_pool* p, int items, bl_fn fn, void* ctx) {
  if (items <= 0) return;
  pthread_mutex_lock(&p->mu);
  p->fn = fn;
  p->ctx = ctx;
  p->items = items;
  atomic_store(&p->next, 0);
  p->running = p->n_threads - 1;
  p->gen++;
  pthread_cond_broadcast(&p->go);
  pthread_mutex_unlock(&p->mu);
  bl_drain(p);
  pthread_mutex_lock(&p->mu);
  while (p->running > 0) pthread_cond_wait(&p->done, &p->mu);
  pthread_mutex_unlock(&p->mu);
}

/* ---- Q8_0 row x tokens ------------------------------------------------------------------------ */

static inline float bl_hsum(__m256 v) {
  __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_movehdup_ps(s));
  return _mm_cvtss_f32(s);
}

/* out[j] = row . xs[j] for j < nx (nx <= BL_NX): a Q8_0 row of K/32 blocks (f16 d, 32 int8). */
static void bl_q8_dots(const uint8_t* row, const float* const* xs, int nx, int K, float* out) {
  __m256 acc[BL_NX];
  for (int j = 0; j < BL_NX; ++j) acc[j] = _mm256_setzero_ps();
  for (int b = 0; b < K / 32; ++b) {
    const uint8_t* blk = row + (size_t)b * 34;
    uint16_t dh;
    memcpy(&dh, blk, 2);
    const __m256 d = _mm256_set1_ps(_cvtsh_ss(dh));
    const __m128i q16a = _mm_loadu_si128((const __m128i*)(blk + 2));
    const __m128i q16b = _mm_loadu_si128((const __m128i*)(blk + 18));
    const __m256 w0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(q16a));
    const __m256 w1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(q16a, 8)));
    const __m256 w2 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(q16b));
    const __m256 w3 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(q16b, 8)));
    for (int j = 0; j < nx; ++j) {
      const float* x = xs[j] + b * 32;
      __m256 s = _mm256_mul_ps(w0, _mm256_loadu_ps(x));
      s = _mm256_fmadd_ps(w1, _mm256_loadu_ps(x + 8), s);
      s = _mm256_fmadd_ps(w2, _mm256_loadu_ps(x + 16), s);
      s = _mm256_fmadd_ps(w3, _mm256_loadu_ps(x + 24), s);
      acc[j] = _mm256_fmadd_ps(d, s, acc[j]);
    }
  }
  for (int j = 0; j < nx; ++j) out[j] = bl_hsum(acc[j]);
}

/* ---- the two passes --------------------------------------------------------------------------- */

typedef struct {
  const uint8_t *gate, *up, *down;
  const float* x;
  int H, I, E;
  int n_active;
  const int* active;     /* [n_active] experts with pairs */
  const int* off;        /* [E + 1] pair offsets by expert */
  const int* pair_tok;   /* [P] token of each pair, expert-major */
  const float* pair_w;   /* [P] summed routing weight of each pair */
  const int* tok_off;    /* [T + 1] the pairs of each token (indices into tok_pairs) */
  const int* tok_pairs;  /* pairs per token, in first-slot order */
  float* h;              /* [P, I] */
  float* yp;             /* [P, H] */
  float* y;              /* [T, H] */
  int gu_chunks, dn_chunks, y_chunks;
} bl_job;

static void bl_pass1(void* ctx, int item) { /* (active expert, 16 gate/up rows) */
  bl_job* J = (bl_job*)ctx;
  const int e = J->active[item / J->gu_chunks], n0 = (item % J->gu_chunks) * BL_ROWS;
  const int n1 = n0 + BL_ROWS < J->I ? n0 + BL_ROWS : J->I;
  const size_t rb = (size_t)J->H / 32 * 34;
  const uint8_t* g = J->gate + (size_t)e * J->I * rb;
  const uint8_t* u = J->up + (size_t)e * J->I * rb;
  for (int p0 = J->off[e]; p0 < J->off[e + 1]; p0 += BL_NX) {
    const int nx = J->off[e + 1] - p0 < BL_NX ? J->off[e + 1] - p0 : BL_NX;
    const float* xs[BL_NX];
    for (int j = 0; j < nx; ++j) xs[j] = J->x + (size_t)J->pair_tok[p0 + j] * J->H;
    for (int n = n0; n < n1; ++n) {
      float gv[BL_NX], uv[BL_NX];
      bl_q8_dots(g + (size_t)n * rb, xs, nx, J->H, gv);
      bl_q8_dots(u + (size_t)n * rb, xs, nx, J->H, uv);
      for (int j = 0; j < nx; ++j) J->h[(size_t)(p0 + j) * J->I + n] = gv[j] / (1.0f + expf(-gv[j])) * uv[j];
    }
  }
}

static void bl_pass2(void* ctx, int item) { /* (active expert, 16 down rows) */
  bl_job* J = (bl_job*)ctx;
  const int e = J->active[item / J->dn_chunks], n0 = (item % J->dn_chunks) * BL_ROWS;
  const int n1 = n0 + BL_ROWS < J->H ? n0 + BL_ROWS : J->H;
  const size_t rb = (size_t)J->I / 32 * 34;
  const uint8_t* d = J->down + (size_t)e * J->H * rb;
  for (int p0 = J->off[e]; p0 < J->off[e + 1]; p0 += BL_NX) {
    const int nx = J->off[e + 1] - p0 < BL_NX ? J->off[e + 1] - p0 : BL_NX;
    const float* hs[BL_NX];
    for (int j = 0; j < nx; ++j) hs[j] = J->h + (size_t)(p0 + j) * J->I;
    for (int n = n0; n < n1; ++n) {
      float v[BL_NX];
      bl_q8_dots(d + (size_t)n * rb, hs, nx, J->I, v);
      for (int j = 0; j < nx; ++j) J->yp[(size_t)(p0 + j) * J->H + n] = v[j];
    }
  }
}

static void bl_pass3(void* ctx, int item) { /* (token, 256 columns): the weighted sum */
  bl_job* J = (bl_job*)ctx;
  const int t = item / J->y_chunks, c0 = (item % J->y_chunks) * 256;
  const int c1 = c0 + 256 < J->H ? c0 + 256 : J->H;
  float* yt = J->y + (size_t)t * J->H;
  for (int c = c0; c < c1; ++c) yt[c] = 0.0f;
  for (int q = J->tok_off[t]; q < J->tok_off[t + 1]; ++q) {
    const int p = J->tok_pairs[q];
    const float w = J->pair_w[p];
    const float* src = J->yp + (size_t)p * J->H;
    for (int c = c0; c < c1; ++c) yt[c] += w * src[c];
  }
}

/* y [T, H] f32 = sum over each token's routed (expert, weight) slots of weight * down(silu(gate x) *
 * (up x)) on Q8_0 stacks [E, I, H/32*34] / [E, H, I/32*34]; slots with weight 0 or id >= E are
 * skipped, a token's repeated expert runs once with the weights summed. Returns -1 on bad shapes. */
int orc_baseline_decode_q8_0(const uint8_t* gate, const uint8_t* up, const uint8_t* down, const float* x,
                             const uint32_t* ids, const float* w, int T, int k, int E, int H, int I, int n_threads,
                             float* y) {
  if (H % 32 || I % 32 || T < 0 || k <= 0 || E <= 0) return -1;
  if (n_threads < 1) n_threads = 1;
  if (n_threads > BL_MAX_THREADS) n_threads = BL_MAX_THREADS;
  const int n = T * k;
  int* pe = malloc(sizeof(int) * (size_t)(n + 1));  /* distinct (token, expert) pairs in slot order */
  int* pt = malloc(sizeof(int) * (size_t)(n + 1));
  float* pw = malloc(sizeof(float) * (size_t)(n + 1));
  int* tok_off = malloc(sizeof(int) * (size_t)(T + 1));
  int P = 0;
  for (int t = 0; t < T; ++t) {
    tok_off[t] = P;
    for (int j = 0; j < k; ++j) {
      const uint32_t e = ids[(size_t)t * k + j];
      const float wt = w[(size_t)t * k + j];
      if (e >= (uint32_t)E || wt == 0.0f) continue;
      int q = tok_off[t];
      while (q < P && pe[q] != (int)e) ++q;
      if (q < P) {
        pw[q] += wt;
      } else {
        pe[P] = (int)e;
        pt[P] = t;
        pw[P] = wt;
        ++P;
      }
    }
  }
  tok_off[T] = P;
  /* expert-major order of the pairs (stable) */
  int* off = calloc((size_t)E + 1, sizeof(int));
  for (int p = 0; p < P; ++p) off[pe[p] + 1]++;
  for (int e = 0; e < E; ++e) off[e + 1] += off[e];
  int* fill = malloc(sizeof(int) * (size_t)E);
  memcpy(fill, off, sizeof(int) * (size_t)E);
  int* pair_tok = malloc(sizeof(int) * (size_t)(P + 1));
  float* pair_w = malloc(sizeof(float) * (size_t)(P + 1));
  int* tok_pairs = malloc(sizeof(int) * (size_t)(P + 1));
  for (int p = 0; p < P; ++p) {
    const int s = fill[pe[p]]++;
    pair_tok[s] = pt[p];
    pair_w[s] = pw[p];
    tok_pairs[p] = s; /* token-major slot order -> expert-major pair index */
  }
  int* active = malloc(sizeof(int) * (size_t)E);
  int na = 0;
  for (int e = 0; e < E; ++e)
    if (off[e + 1] > off[e]) active[na++] = e;
  bl_job J;
  memset(&J, 0, sizeof(J));
  J.gate = gate; J.up = up; J.down = down; J.x = x;
  J.H = H; J.I = I; J.E = E;
  J.n_active = na; J.active = active; J.off = off;
  J.pair_tok = pair_tok; J.pair_w = pair_w; J.tok_off = tok_off; J.tok_pairs = tok_pairs;
  J.h = malloc(sizeof(float) * (size_t)(P + 1) * I);
  J.yp = malloc(sizeof(float) * (size_t)(P + 1) * H);
  J.y = y;
  J.gu_chunks = (I + BL_ROWS - 1) / BL_ROWS;
  J.dn_chunks = (H + BL_ROWS - 1) / BL_ROWS;
  J.y_chunks = (H + 255) / 256;
  bl_pool* pool = bl_get_pool(n_threads);
  bl_parallel_for(pool, na * J.gu_chunks, bl_pass1, &J);
  bl_parallel_for(pool, na * J.dn_chunks, bl_pass2, &J);
  bl_parallel_for(pool, T * J.y_chunks, bl_pass3, &J);
  free(J.h);
  free(J.yp);
  free(active);
  free(tok_pairs);
  free(pair_w);
  free(pair_tok);
  free(fill);
  free(off);
  free(tok_off);
  free(pw);
  free(pt);
  free(pe);
  return 0;
}
