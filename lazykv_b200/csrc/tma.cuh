// TMA bulk copies and bounded mbarrier waits (sm_90+ PTX, used on sm_100a by attention.cu).
#pragma once

#include "common.cuh"

namespace lkv {

// Status word of the kernels with bounded waits: 0, or the first LKV_DEV_* code a kernel recorded.
// Internal linkage (the library is built without relocatable device code): each translation unit
// that includes this header has its own and reads it with tu_device_status; lkv_device_status
// combines those of attention.cu and select.cu.
static __device__ int g_device_status = 0;
// Optional mirror of the status word in pinned, mapped host memory (set by lkv_status_attach): a
// kernel that records a status also sets it with a system-scope atomic, so the host can poll it
// between steps without synchronising with the device.
static __device__ int* g_status_host = nullptr;
constexpr int LKV_DEV_WAIT_TIMEOUT = 1;       // an mbarrier wait ran out of iterations
constexpr int LKV_DEV_LIST_OVERFLOW = 2;      // a CTA's item list would not fit its shared memory (host sizing error)
constexpr uint32_t kMaxWaitIters = 1u << 21;  // tries; each may suspend up to kWaitHintNs
constexpr uint32_t kWaitHintNs = 1000;        // suspend-time hint of one try (the wait ends sooner when the phase completes)

// This translation unit's status word into *status (cleared after the read when `clear`).
static inline cudaError_t tu_device_status(int* status, int clear) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_device_status, sizeof(int));
  if (e == cudaSuccess && clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
  }
  return e;
}

// Points this translation unit's kernels on the current device at the host mirror (device address
// of a mapped host int, or null to detach).
static inline cudaError_t tu_status_attach(int* mirror) { return cudaMemcpyToSymbol(g_status_host, &mirror, sizeof(mirror)); }

// Records `code` in the status word (the first code wins) and in its host mirror, if attached.
__device__ __forceinline__ void record_status(int code) {
  atomicCAS(&g_device_status, 0, code);
  int* h = g_status_host;
  if (h != nullptr) atomicCAS_system(h, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes initialised mbarriers visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// A plain arrival (no transaction bytes): completes the phase of a count-1 barrier by itself.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One bulk copy global -> this CTA's shared memory (16-byte aligned addresses, size a multiple of
// 16), completing `bytes` of transaction count on `bar`. No multicast.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// An L2 policy under which the lines a load brings in are the first to be evicted. The streamed
// blocks, records and block bounds are read once per call; under this policy they do not push the
// reused lines out of L2 (lists, bitmaps, partials, counters and the kernels' own instructions).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// tma_load_1d under an L2 cache policy.
__device__ __forceinline__ void tma_load_1d_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
               : "memory");
}

// Waits for the phase of `bar` with the given parity. Each try may suspend the thread (up to the
// hint) until the phase completes, so a waiting warp does not spin on issue slots. Gives up after
// `iters` tries (kMaxWaitIters: about two seconds at most), records LKV_DEV_WAIT_TIMEOUT and
// returns false.
__device__ __forceinline__ bool mbar_wait_n(uint64_t* bar, uint32_t parity, uint32_t iters) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < iters; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity), "r"(kWaitHintNs)
        : "memory");
    if (done) return true;
  }
  record_status(LKV_DEV_WAIT_TIMEOUT);
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) { return mbar_wait_n(bar, parity, kMaxWaitIters); }

}  // namespace lkv
