// moe_common.cuh — shared device helpers of libmoe_b200.so (sm_100a only).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "moe_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libmoe_b200 is built for sm_100a only"
#endif

namespace moe {

// ---- host-side error plumbing --------------------------------------------------------------

void set_error(const std::string& msg);
moe_status fail(moe_status st, const std::string& msg);
moe_status cuda_fail(cudaError_t e, const char* what);
const std::string& last_error_message();  // this thread's last failure message

#define MOE_CUDA_TRY(expr)                                   \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return ::moe::cuda_fail(_e, #expr); \
  } while (0)

#define MOE_TRY(expr)                      \
  do {                                     \
    moe_status _s = (expr);                \
    if (_s != MOE_OK) return _s;           \
  } while (0)

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// ---- mbarriers and bulk copies (shared memory) -------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

constexpr uint32_t WAIT_POLLS = 1u << 22;               // backstop on try_wait polls
constexpr long long WAIT_CYCLES = 400ll * 1000ll * 1000ll;  // ~200 ms of SM clock: a longer wait is declared stuck

// Bounded parity wait: true when the phase completed; false after WAIT_CYCLES SM clocks (or
// WAIT_POLLS polls), or as soon as another role of the CTA gave up (*abort set; nullptr: no such
// check). The clock is read only once the first poll failed: the common, already-completed case
// costs one try_wait.
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;}"
      : "=r"(done)
      : "r"(a), "r"(parity)
      : "memory");
  return done != 0;
}

// The same test with a suspend-time hint: a thread whose phase is not complete sleeps until it
// completes (or about SUSPEND_NS pass) instead of spinning, so waiting roles leave the issue slots
// to the dequantising warps.
constexpr uint32_t SUSPEND_NS = 1u << 20;
__device__ __forceinline__ bool mbar_try_sleep(uint32_t a, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      "selp.u32 %0, 1, 0, p;}"
      : "=r"(done)
      : "r"(a), "r"(parity), "r"(SUSPEND_NS)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try(a, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 0; i < WAIT_POLLS; ++i) {
    if (mbar_try_sleep(a, parity)) return true;
    if ((abort && *abort) || clock64() - t0 > WAIT_CYCLES) return false;
  }
  return false;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---- programmatic dependent launch ---------------------------------------------------------
// The forward's kernels are launched with launch_pdl: each may start while the kernel before it in
// the stream is still running, so its CTAs become resident and do their set-up (barriers, tensor
// memory, for the down GEMV the first weight loads) during the other's tail. The contract every
// such kernel keeps: pdl_wait() (which returns once the preceding kernel has completed and its
// writes are visible; at once when there is no programmatic dependency) comes before any access to
// data an earlier kernel wrote or reads, and pdl_trigger() (which lets the next kernel launch)
// only after pdl_wait(). A kernel that starts therefore knows that every kernel two or more
// places before it has completed. MOE_PDL=0 launches everything plainly.

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();

// allow = false launches plainly (the kernel's pdl_wait / pdl_trigger are then no-ops).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_if(bool allow, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = allow && pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  return launch_pdl_if(true, kernel, grid, block, smem, st, std::forward<Args>(args)...);
}

// ---- device helpers -------------------------------------------------------------------------

constexpr unsigned FULL = 0xffffffffu;

// Deterministic exp, bit-identical to the CPU oracle's orc_exp: Cody-Waite reduction with a
// two-constant ln2 split, the degree-7 Taylor polynomial of e^r in Horner form with fused
// multiply-adds, then exact scaling by 2^n. Every operation is an explicitly rounded intrinsic so
// the compiler cannot contract or reorder it.
__device__ __forceinline__ float det_exp(float x) {
  if (x != x) return x;
  if (x > 0x1.62e430p+6f) return __int_as_float(0x7f800000);
  if (x < -104.0f) return 0.0f;
  float n = rintf(__fmul_rn(x, 0x1.715476p+0f));
  float r = __fmaf_rn(-n, 0x1.62e400p-1f, x);
  r = __fmaf_rn(-n, 0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
  p = __fmaf_rn(p, r, 0x1.111112p-7f);
  p = __fmaf_rn(p, r, 0x1.555556p-5f);
  p = __fmaf_rn(p, r, 0x1.555556p-3f);
  p = __fmaf_rn(p, r, 0x1.000000p-1f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ni = (int)n;
  if (ni > 127) { p = __fmul_rn(p, 0x1p127f); ni -= 127; }
  if (ni < -126) { p = __fmul_rn(p, 0x1p-64f); ni += 64; }
  return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

__device__ __forceinline__ float det_sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, det_exp(-x))); }

// Rust f32::total_cmp order as an unsigned key (larger key = later in the order).
__device__ __forceinline__ uint32_t total_key_u(float f) {
  int32_t b = __float_as_int(f);
  b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
  return (uint32_t)b ^ 0x80000000u;
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once per launch). The
// data is read-only for the kernel's lifetime, so the asm is not volatile and may be scheduled freely.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ldg_nc(const void* p) {
  uint4 v;
  asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16-byte shared load as a plain C++ access, so the compiler keeps it ordered against barriers.
__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// D = A(16x16, row) * B(16x8, col) + C, f32 accumulate (warp-level tensor-core MMA).
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D = A * B (no accumulator input): the first MMA of a block-scaled partial sum.
__device__ __forceinline__ void mma_f16_zero(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "{.reg .f32 z; mov.f32 z, 0f00000000;\n"
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {z,z,z,z};}"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (d0, d1) += s * (t0, t1) as one packed f32x2 fused multiply-add (sm_100).
__device__ __forceinline__ void ffma2(float& d0, float& d1, float s, float t0, float t1) {
  asm(
      "{.reg .b64 t, c, s2;\n"
      "mov.b64 t, {%2, %3};\n"
      "mov.b64 c, {%0, %1};\n"
      "mov.b64 s2, {%4, %4};\n"
      "fma.rn.f32x2 c, s2, t, c;\n"
      "mov.b64 {%0, %1}, c;}"
      : "+f"(d0), "+f"(d1)
      : "f"(t0), "f"(t1), "f"(s));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
  return v;
}

// Exclusive scan of v over the block (blockDim.x == 1024), returns the prefix, *total the sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = warp_sums[lane];
    int z = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(FULL, z, o);
      if (lane >= o) z += y;
    }
    warp_sums[lane] = z - s;  // exclusive warp base
    if (lane == 31) warp_sums[32] = z;
  }
  __syncthreads();
  int r = x - v + warp_sums[warp];
  *total = warp_sums[32];
  __syncthreads();
  return r;
}

// Expert parallelism: bit r set when token t has a slot whose id falls in rank r's experts
// [r * epr, (r + 1) * epr); *bad = 1 for an id past world * epr (skipped). world <= 64.
__device__ __forceinline__ uint64_t token_rank_mask(const uint32_t* __restrict__ ids, int t, int k, int epr, int world,
                                                    int* bad) {
  uint64_t m = 0;
  const uint32_t limit = (uint32_t)epr * (uint32_t)world;
  for (int j = 0; j < k; ++j) {
    const uint32_t id = ids[(int64_t)t * k + j];
    if (id == MOE_ID_NONE) continue;
    if (id >= limit) {
      *bad = 1;
      continue;
    }
    m |= 1ull << (id / (uint32_t)epr);
  }
  return m;
}

// A routed pair runs when its id names an expert (< E) that is resident: with an expert cache,
// slot_of[id] >= 0; without one (slot_of null) every expert is. MOE_ID_NONE and non-resident
// experts are skipped; ids >= E other than MOE_ID_NONE are the caller's error.
__device__ __forceinline__ bool pair_live(uint32_t id, int E, const int32_t* slot_of) {
  return id < (uint32_t)E && (!slot_of || slot_of[id] >= 0);
}

}  // namespace moe
