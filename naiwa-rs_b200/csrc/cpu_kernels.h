// cpu_kernels.h — host-side dot products of the CPU expert path (cpu_executor.cu), in plain C++.
//
// A weight row (GGML bytes: Q8_0 blocks of {f16 d, 32 int8}, or bf16 values) times up to
// CPU_DOT_MAX_X f32 activation vectors in one pass over the row, so each block is read and widened
// once per call however many of the expert's tokens use it. Q8_0 dots are sum over blocks of
// d * (sum of q * x); the f32 accumulation order is fixed per build of the function, not per call.
#pragma once
#include <cstdint>

namespace moe {

constexpr int CPU_DOT_MAX_X = 4;

// out[j] = row . xs[j] for j < nx, K a multiple of 32 for Q8_0 (vectors taken CPU_DOT_MAX_X at a
// time, each chunk one pass over the row).
void cpu_dot_q8_0(const uint8_t* row, const float* const* xs, int nx, int K, float* out);
void cpu_dot_bf16(const uint16_t* row, const float* const* xs, int nx, int K, float* out);

// The instruction set the dots were dispatched to on this host: "avx512", "avx2" or "scalar".
const char* cpu_dot_isa();

}  // namespace moe
