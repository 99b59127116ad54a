/*
 * moe_oracle.h — CPU restatement of the naiwa-rs MoE-layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links, loads or calls this code.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it, as the checker
 * and as the timed CPU baseline.
 *
 * Every function cites the reference file:line it restates (paths inside flaneur2020/naiwa-rs).
 * Where the reference's arithmetic lives in its un-vendored mistral.rs / candle fork
 * (mistralrs-quant 0.9.4, candle-core 0.11.0; Cargo.toml:10-20), the function restates the
 * published algorithm and names it.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar formats ---------------------------------------------------------------------- */
float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);
float orc_bf16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16(float f);
float orc_fp8e4m3_to_f32(uint8_t b);
uint8_t orc_f32_to_fp8e4m3(float f);

/* deterministic exp / sigmoid / silu shared bit-for-bit with the device code */
float orc_exp(float x);
float orc_sigmoid(float x);
float orc_silu(float x);

/* ---- block formats (GGML layouts) -------------------------------------------------------- */
/* Q8_0: 34-byte blocks {f16 d; int8 qs[32]} (reference src/moe/tests.rs:101-102). */
void orc_q8_0_quantize(const float* x, int64_t n, uint8_t* out);
void orc_q8_0_dequantize(const uint8_t* blocks, int64_t n, float* out);
/* Q4_K: 144-byte super-blocks of 256 {f16 d; f16 dmin; u8 scales[12]; u8 qs[128]}. */
void orc_q2_0_quantize(const float* x, int64_t n, uint8_t* out);
void orc_q2_0_dequantize(const uint8_t* blocks, int64_t n, float* out);
void orc_q4_k_quantize(const float* x, int64_t n, uint8_t* out);
void orc_q4_k_dequantize(const uint8_t* blocks, int64_t n, float* out);
/* FP8 e4m3 with one f32 scale per 128x128 block of an [N, K] matrix (N, K multiples of 128). */
void orc_fp8_b128_quantize(const float* w, int n, int k, uint8_t* q, float* scales);
void orc_fp8_b128_dequantize(const uint8_t* q, const float* scales, int n, int k, float* out);

int64_t orc_block_bytes(int dtype, int64_t n_weights); /* dtype codes follow include/moe_b200.h */
/* Byte range [begin, end) of expert e inside a stacked [E, N, K] tensor (src/moe/expert.rs:123-145).
 * Returns 0 on success, -1 when K is not a multiple of the block size or e >= E. */
int orc_expert_range(int dtype, int E, int N, int K, int e, int64_t* begin, int64_t* end);

/* ---- cache policy (src/moe/cached_layer.rs) --------------------------------------------- */
int orc_top_k_ids(const float* logits, int n, int k, int* out);
int orc_union_by_votes(const int* const* rankings, const int* lens, int n_rankings, int* out);
int orc_streamed_misses(const uint32_t* ids, const float* ws, const int* row_lens, int rows,
                        float frac, int cap, uint32_t* out);
/* slots: expert (-1 empty), published flag, last_use. Returns slot index or -1; *expert_out. */
int orc_lru_victim(const int* slot_expert, const int* slot_published, const uint64_t* last_use,
                   int n_slots, const int* protect, int n_protect, int* expert_out);
int orc_fill_candidate(const int* slot_expert, int n_slots, const uint64_t* hit_counts, int n_experts);

/* ---- router -------------------------------------------------------------------------------- */
void orc_router_logits(const uint16_t* x_bf16, const uint16_t* w_bf16, int T, int H, int E, float* logits);
/* mode: 0 softmax, 1 softmax + renormalise over the top-k, 2 sigmoid + group-limited top-k */
int orc_route(const float* logits, const float* bias, int T, int E, int k, int mode, int n_group,
              int topk_group, float routed_scale, uint32_t* ids, float* weights);

/* ---- permute ------------------------------------------------------------------------------- */
int orc_permute(const uint32_t* ids, int n_pairs, int E, int32_t* counts, int32_t* offsets,
                int32_t* perm, int32_t* active, int32_t* n_active);

/* ---- expert FFN + combine (dequantised f32 reference) ------------------------------------ */
/* gate, up: [E, I, H] f32; down: [E, H, I] f32; x: [T, H] f32; ids/w: [T, k]; y: [T, H] f32. */
void orc_moe_forward_f32(const float* x, const uint32_t* ids, const float* w, int T, int k, int E, int H,
                         int I, const float* gate, const float* up, const float* down, float* y);
/* orc_moe_forward_f32 over quantised stacks (dtype codes of include/moe_b200.h; FP8 block scales in
 * gs/us/ds), expert by expert on n_threads; ids >= E are skipped. */
int orc_moe_forward_ref(int dtype, const uint8_t* gate, const uint8_t* up, const uint8_t* down, const float* gs,
                        const float* us, const float* ds, const float* x, const uint32_t* ids, const float* w, int T,
                        int k, int E, int H, int I, int n_threads, float* y);

/* ---- timed CPU baseline: two-pass fused decode over Q8_0 stacks -------------------------- */
/* gate/up/down are GGML Q8_0 stacks [E, I, H], [E, I, H], [E, H, I]. x f32 [T, H]. */
int orc_fused_moe_decode_q8_0(const uint8_t* gate, const uint8_t* up, const uint8_t* down, const float* x,
                              const uint32_t* ids, const float* w, int T, int k, int E, int H, int I,
                              int n_threads, float* y);

/* ---- timed CPU baseline, fast restatement (cpu_baseline.c): same result as
 * orc_fused_moe_decode_q8_0 up to summation order; AVX2, persistent thread pool ------------------ */
int orc_baseline_decode_q8_0(const uint8_t* gate, const uint8_t* up, const uint8_t* down, const float* x,
                             const uint32_t* ids, const float* w, int T, int k, int E, int H, int I, int n_threads,
                             float* y);

#ifdef __cplusplus
}
#endif
#endif
