// route_noalloc.cu — the router entry point for callers that cannot allocate device memory.
//
// moe_route_tokens needs a workspace (router logits plus per-token-block arrival counters) that
// the caller allocates. Some callers have no way to do that: a host binding that owns no CUDA
// allocator (a thin FFI crate that only forwards pointers it was given), code that runs while a
// stream capture is active (cudaMalloc is not a stream operation and breaks the capture), or an
// application that hands the library a fixed device-memory budget up front. This variant runs the
// same router kernel with its workspace in a file-scope device array instead.
//
// The array is static: every GPU that loads the library holds its MOE_ROUTE_NOALLOC_MAX_BYTES
// until the process exits, and every call on a device shares it. A call leaves the logits of its
// tokens in the array; the arrival counters are cleared on the caller's stream at the start of
// each call, so a call never depends on what an earlier one left. Two calls whose kernels overlap
// on the GPU (different streams, no ordering between them) race on the array and produce garbage.
#include <mutex>

#include "moe_internal.cuh"

namespace moe {

static __device__ __align__(256) unsigned char g_route_noalloc_scratch[MOE_ROUTE_NOALLOC_MAX_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the static array on the current device. Host code must not pass the symbol
// itself to a kernel: on the host it names a stand-in object, not device memory.
moe_status scratch_address(void** out) {
  int dev = 0;
  MOE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(MOE_ERR_INVALID, "moe_route_tokens_noalloc: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_route_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_route_noalloc_scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MOE_OK;
}
}  // namespace

}  // namespace moe

using namespace moe;

extern "C" moe_status moe_route_tokens_noalloc(const void* x, const void* w_router, const float* bias, int T, int H,
                                               int E, int k, int mode, int n_group, int topk_group,
                                               float routed_scale, uint32_t* ids, float* weights, void* stream) {
  if (T < 0 || E <= 0) return fail(MOE_ERR_INVALID, "moe_route_tokens_noalloc: need T >= 0 and E > 0");
  const size_t need = route_workspace_bytes(T, E);
  if (need > (size_t)MOE_ROUTE_NOALLOC_MAX_BYTES)
    return fail(MOE_ERR_INVALID, "moe_route_tokens_noalloc: T * E too large for the static scratch (needs " +
                                     std::to_string(need) + " bytes, the array holds " +
                                     std::to_string((size_t)MOE_ROUTE_NOALLOC_MAX_BYTES) + ")");
  RouteParams p{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w_router), bias, ids,
                weights, T, H, E, k, mode, n_group, topk_group, routed_scale};
  // every argument is checked before anything is enqueued, so a rejected call leaves the stream
  // (and a capture in progress on it) untouched
  MOE_TRY(route_validate(p));
  if (T == 0) return MOE_OK;
  void* scratch = nullptr;
  MOE_TRY(scratch_address(&scratch));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the arrival counters sit after the 256-byte-aligned logits and must start at zero
  const size_t logits = ((size_t)T * E * 4 + 255) / 256 * 256;
  MOE_CUDA_TRY(cudaMemsetAsync(static_cast<char*>(scratch) + logits, 0, need - logits, st));
  return route_tokens(p, scratch, need, st);
}
