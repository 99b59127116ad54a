// doorbell.cu — host <-> device hand-off rings over mapped pinned memory.
//
// Reference: src/doorbell/doorbell.cu:15-149 (the ring kernels), mapped.rs:18-141 (the mapped
// allocation, volatile loads, release stores, bounded host waits), payload_ring.rs:14-81 (seq +
// consumed header, a ring of slots), d2h/topk.rs:20-125 (top-k ids to the host),
// h2d/result.rs:27-123 (CPU results back to the device).
//
// One moe_ring is a cudaHostAllocMapped allocation: a 64-byte header {seq, consumed, status} and
// `depth` slots. The producer writes a slot's payload, makes it visible (device:
// __threadfence_system; host: a release fence) and then publishes with a release store of
// seq + 1; the consumer waits for seq >= target with acquire loads, reads the slot and publishes
// consumed = target, which is what lets the producer reuse the slot (seq - consumed < depth).
//   * device -> host (moe_ring_publish_from_device / moe_ring_host_take): a one-block kernel copies
//     up to two device segments into the slot, the host thread waits without a stream sync;
//   * host -> device (moe_ring_host_publish / moe_ring_device_take): the host writes the slot, a
//     one-block kernel waits for it and copies it into device memory.
// Unlike the reference's device spin, every device wait here is bounded (about one second of
// %globaltimer): a wait that runs out records MOE_ERR_TIMEOUT in the header's status word and the
// kernel returns without touching its destination, so the context stays usable and the next
// moe_ring_check reports it. Host waits take a timeout in microseconds.
#include <algorithm>
#include <chrono>
#include <cstring>
#include <thread>

#include "moe_internal.cuh"

namespace moe {

constexpr int RING_THREADS = 256;
constexpr size_t RING_HEADER = 64;
constexpr uint64_t RING_DEVICE_WAIT_NS = 1000ull * 1000ull * 1000ull;  // 1 s

struct RingHeader {
  uint32_t seq;       // producer: number of slots published
  uint32_t consumed;  // consumer: number of slots read out
  int32_t status;     // device waits that ran out record MOE_ERR_TIMEOUT here
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t ring_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Block-wide copy of n bytes; 16-byte steps when both ends and n allow it.
__device__ __forceinline__ void block_copy(unsigned char* dst, const unsigned char* src, size_t n) {
  if ((((uintptr_t)dst | (uintptr_t)src | n) & 15) == 0) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    const uint4* s = reinterpret_cast<const uint4*>(src);
    for (size_t i = threadIdx.x; i < n / 16; i += blockDim.x) d[i] = s[i];
  } else {
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
}

// Waits (thread 0, bounded) until the condition on the mapped header holds; the verdict is shared
// with the block. want_seq: wait for seq >= target; else wait for seq - consumed < depth.
__device__ bool ring_wait(RingHeader* h, bool want_seq, uint32_t target, uint32_t depth) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const uint64_t t0 = ring_now_ns();
    int ok = 0;
    for (;;) {
      if (want_seq) {
        if ((int32_t)(ld_acquire_sys(&h->seq) - target) >= 0) ok = 1;
      } else {
        if (target - ld_acquire_sys(&h->consumed) < depth) ok = 1;  // target = the seq being written
      }
      if (ok || ring_now_ns() - t0 > RING_DEVICE_WAIT_NS) break;
      __nanosleep(256);
    }
    if (!ok) atomicExch(&h->status, (int32_t)MOE_ERR_TIMEOUT);
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Device -> host: slot (seq_index % depth) <- src0[0:n0] ++ src1[0:n1], then seq = seq_index + 1.
__global__ void __launch_bounds__(RING_THREADS) ring_publish_kernel(RingHeader* h, unsigned char* slots,
                                                                    size_t slot_bytes, uint32_t depth,
                                                                    uint32_t seq_index, const unsigned char* src0,
                                                                    size_t n0, const unsigned char* src1, size_t n1) {
  if (!ring_wait(h, false, seq_index, depth)) return;
  unsigned char* slot = slots + (size_t)(seq_index % depth) * slot_bytes;
  block_copy(slot, src0, n0);
  if (src1) block_copy(slot + n0, src1, n1);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // the payload is visible to the host before the counter moves
    st_release_sys(&h->seq, seq_index + 1);
  }
}

// Host -> device: wait for seq >= target, dst <- slot ((target - 1) % depth), then consumed = target.
__global__ void __launch_bounds__(RING_THREADS) ring_take_kernel(RingHeader* h, const unsigned char* slots,
                                                                 size_t slot_bytes, uint32_t depth, uint32_t target,
                                                                 unsigned char* dst, size_t n) {
  if (!ring_wait(h, true, target, depth)) return;
  const unsigned char* slot = slots + (size_t)((target - 1) % depth) * slot_bytes;
  block_copy(dst, slot, n);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // every read of the slot retired before the host may overwrite it
    st_release_sys(&h->consumed, target);
  }
}

}  // namespace moe

using namespace moe;

struct moe_ring {
  int dev = 0;
  uint32_t depth = 0;
  size_t slot_bytes = 0;
  unsigned char* host = nullptr;  // mapped allocation, host view
  unsigned char* devp = nullptr;  // same bytes, device view
  uint32_t next_publish = 0;      // producer side: seq value of the next publish
};

static RingHeader* host_header(moe_ring* r) { return reinterpret_cast<RingHeader*>(r->host); }

static uint32_t host_load_acquire(const uint32_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
static void host_store_release(uint32_t* p, uint32_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }

// Spin briefly, then yield-poll until pred() or the timeout (microseconds, < 0: no limit).
template <class Pred>
static bool host_wait(Pred pred, int64_t timeout_us) {
  const auto t0 = std::chrono::steady_clock::now();
  for (int i = 0;; ++i) {
    if (pred()) return true;
    if (timeout_us >= 0 &&
        std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count() >
            timeout_us)
      return false;
    if (i > 2048) std::this_thread::yield();
  }
}

extern "C" {

moe_status moe_ring_create(int device, int depth, size_t slot_bytes, moe_ring** out) {
  if (!out) return fail(MOE_ERR_INVALID, "moe_ring_create: null out");
  *out = nullptr;
  if (depth < 1 || depth > 1024 || slot_bytes == 0)
    return fail(MOE_ERR_INVALID, "moe_ring_create: need 1 <= depth <= 1024 and slot_bytes > 0");
  DeviceGuard guard(device);
  if (!guard.ok) return fail(MOE_ERR_CUDA, "moe_ring_create: cannot select device");
  moe_ring* r = new moe_ring();
  r->dev = device;
  r->depth = (uint32_t)depth;
  r->slot_bytes = (slot_bytes + 15) & ~(size_t)15;
  const size_t bytes = RING_HEADER + r->slot_bytes * (size_t)depth;
  void* h = nullptr;
  cudaError_t e = cudaHostAlloc(&h, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) {
    delete r;
    return cuda_fail(e, "cudaHostAlloc(mapped ring)");
  }
  std::memset(h, 0, bytes);  // a consumer that runs first sees zeros, never stale bytes
  void* d = nullptr;
  e = cudaHostGetDevicePointer(&d, h, 0);
  if (e != cudaSuccess) {
    cudaFreeHost(h);
    delete r;
    return cuda_fail(e, "cudaHostGetDevicePointer(ring)");
  }
  r->host = static_cast<unsigned char*>(h);
  r->devp = static_cast<unsigned char*>(d);
  *out = r;
  return MOE_OK;
}

void moe_ring_destroy(moe_ring* r) {
  if (!r) return;
  if (r->host) cudaFreeHost(r->host);
  delete r;
}

size_t moe_ring_slot_bytes(const moe_ring* r) { return r ? r->slot_bytes : 0; }

moe_status moe_ring_publish_from_device(moe_ring* r, const void* src0, size_t n0, const void* src1, size_t n1,
                                        void* stream, uint32_t* seq_out) {
  if (!r) return fail(MOE_ERR_INVALID, "moe_ring_publish_from_device: null ring");
  if (!src0 || (n1 && !src1)) return fail(MOE_ERR_INVALID, "moe_ring_publish_from_device: null source");
  if (n0 + n1 > r->slot_bytes) return fail(MOE_ERR_INVALID, "moe_ring_publish_from_device: payload exceeds the slot");
  DeviceGuard guard(r->dev);
  const uint32_t s = r->next_publish;
  ring_publish_kernel<<<1, RING_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<RingHeader*>(r->devp), r->devp + RING_HEADER, r->slot_bytes, r->depth, s,
      static_cast<const unsigned char*>(src0), n0, static_cast<const unsigned char*>(src1), n1);
  MOE_CUDA_TRY(cudaGetLastError());
  r->next_publish = s + 1;
  if (seq_out) *seq_out = s + 1;
  return MOE_OK;
}

moe_status moe_ring_host_take(moe_ring* r, uint32_t target, void* dst, size_t n, int64_t timeout_us) {
  if (!r) return fail(MOE_ERR_INVALID, "moe_ring_host_take: null ring");
  if (n > r->slot_bytes || (n && !dst)) return fail(MOE_ERR_INVALID, "moe_ring_host_take: bad destination");
  RingHeader* h = host_header(r);
  if (!host_wait([&] { return (int32_t)(host_load_acquire(&h->seq) - target) >= 0 || host_load_acquire(
                                  reinterpret_cast<uint32_t*>(&h->status)) != 0; },
                 timeout_us))
    return fail(MOE_ERR_TIMEOUT, "moe_ring_host_take: the device did not publish in time");
  if ((int32_t)(host_load_acquire(&h->seq) - target) < 0)
    return fail(MOE_ERR_TIMEOUT, "moe_ring_host_take: a device-side ring wait ran out");
  std::memcpy(dst, r->host + RING_HEADER + (size_t)((target - 1) % r->depth) * r->slot_bytes, n);
  host_store_release(&h->consumed, target);
  return MOE_OK;
}

moe_status moe_ring_host_publish(moe_ring* r, const void* src, size_t n, int64_t timeout_us, uint32_t* seq_out) {
  if (!r) return fail(MOE_ERR_INVALID, "moe_ring_host_publish: null ring");
  if (n > r->slot_bytes || (n && !src)) return fail(MOE_ERR_INVALID, "moe_ring_host_publish: bad payload");
  RingHeader* h = host_header(r);
  const uint32_t s = r->next_publish;
  if (!host_wait([&] { return s - host_load_acquire(&h->consumed) < r->depth; }, timeout_us))
    return fail(MOE_ERR_TIMEOUT, "moe_ring_host_publish: the ring stayed full (the device did not consume)");
  std::memcpy(r->host + RING_HEADER + (size_t)(s % r->depth) * r->slot_bytes, src, n);
  host_store_release(&h->seq, s + 1);  // release: the payload is visible before the counter
  r->next_publish = s + 1;
  if (seq_out) *seq_out = s + 1;
  return MOE_OK;
}

moe_status moe_ring_device_take(moe_ring* r, uint32_t target, void* dst, size_t n, void* stream) {
  if (!r) return fail(MOE_ERR_INVALID, "moe_ring_device_take: null ring");
  if (n > r->slot_bytes || (n && !dst)) return fail(MOE_ERR_INVALID, "moe_ring_device_take: bad destination");
  if (target == 0) return fail(MOE_ERR_INVALID, "moe_ring_device_take: targets start at 1");
  DeviceGuard guard(r->dev);
  ring_take_kernel<<<1, RING_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<RingHeader*>(r->devp), r->devp + RING_HEADER, r->slot_bytes, r->depth, target,
      static_cast<unsigned char*>(dst), n);
  MOE_CUDA_TRY(cudaGetLastError());
  return MOE_OK;
}

moe_status moe_ring_check(moe_ring* r, void* stream) {
  if (!r) return fail(MOE_ERR_INVALID, "moe_ring_check: null ring");
  DeviceGuard guard(r->dev);
  MOE_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  RingHeader* h = host_header(r);
  const int32_t st = __atomic_exchange_n(&h->status, 0, __ATOMIC_ACQ_REL);
  if (st != 0) return fail((moe_status)st, "moe_ring: a device-side wait ran out (its producer never published)");
  return MOE_OK;
}

void moe_ring_counters(const moe_ring* r, uint32_t* seq, uint32_t* consumed) {
  if (!r) return;
  const RingHeader* h = reinterpret_cast<const RingHeader*>(r->host);
  if (seq) *seq = __atomic_load_n(&h->seq, __ATOMIC_ACQUIRE);
  if (consumed) *consumed = __atomic_load_n(&h->consumed, __ATOMIC_ACQUIRE);
}

}  // extern "C"
