// The cross-GPU exchange of a context-sharded layer's partials over NVLink, with plain peer stores
// instead of a collective: every rank writes its (out, lse) rows straight into each peer's inbox,
// raises a per-group arrival counter there, waits (bounded) until every rank's rows of the group
// are in its own inbox, and merges them by log-sum-exp (lazykv/exact.py:69-85, the n-way form of
// merge_lse). One launch per layer replaces an all-gather and a merge launch. The reference runs on
// one GPU and has no counterpart.
//
// Memory. Each rank allocates one region with cudaMalloc (so that its base is an IPC-exportable
// allocation) and exports it with cudaIpcGetMemHandle; every rank opens its peers' regions with
// cudaIpcOpenMemHandle (peer access enabled lazily). Region layout, for R rows of D channels:
//   counters [kXgGroupsMax] uint32 at 0        arrivals per row group, written by every rank
//   epochs   [kXgGroupsMax] uint32 at 4 KiB    this rank's completed exchanges per group (local)
//   inbox    [2][world][R][D + 4] float32 at 8 KiB: rank r's rows of an exchange with epoch e sit
//            in half e & 1 (o [D], then lse, then padding), so a rank that runs one exchange ahead
//            never overwrites rows a slower peer may still read.
// Counters only grow: after e exchanges every rank has added e to each group's counter of every
// rank, so "every rank's rows of exchange e are here" is counter >= e * world, whatever a faster
// rank already added for e + 1. A rank starts exchange e + 2 only after its exchange e + 1 saw every
// peer's rows of e + 1, which each peer wrote after it finished reading exchange e; so half e & 1 is
// free again when it is rewritten.
//
// Ordering: the CTA stores its rows to the peers (generic stores over NVLink) and synchronises,
// then one thread issues a system-scope fence and a relaxed system-scope add on each peer's counter
// (release pattern); the reader's thread 0 polls its own counter with system-scope acquire loads,
// the CTA synchronises, and every thread reads the rows through L2 (.cg).
//
// The wait is bounded: after kXgWaitIters polls (each with a suspend hint) the CTA records
// LKV_DEV_WAIT_TIMEOUT in the status word (lkv_device_status, lkv_status_poll), writes its rows
// from its own partial alone, and still counts the exchange as done, so the next call neither
// hangs nor reads stale halves of a live peer.
#include "tma.cuh"

namespace lkv {
namespace {

constexpr int kXgMaxWorld = 64;
constexpr int kXgGroupsMax = 1024;
constexpr size_t kXgCountersOff = 0, kXgEpochsOff = 4096, kXgInboxOff = 8192;
constexpr int kXgRowsPerGroup = 4;
constexpr int kXgThreads = 128;
constexpr uint32_t kXgWaitIters = 1u << 22;  // polls; each may suspend up to kXgSleepNs
constexpr uint32_t kXgSleepNs = 200;

inline int xg_groups(int rows) { return (rows + kXgRowsPerGroup - 1) / kXgRowsPerGroup; }
__host__ __device__ inline size_t xg_row_floats(int d) { return (size_t)d + 4; }
inline size_t xg_region_bytes(int rows, int d, int world) {
  return kXgInboxOff + 2 * (size_t)world * rows * xg_row_floats(d) * sizeof(float);
}

struct XgParams {
  const float* out;     // [rows, d] this rank's partial output (float32)
  const float* lse;     // [rows]    its log-sum-exp (natural log)
  unsigned char* base[kXgMaxWorld];  // every rank's region (this rank's own at [rank])
  int world, rank, rows, d;
  void* merged;         // [rows, d] in out_dtype
  int out_bf16;
  float* merged_lse;    // [rows] (optional)
  uint32_t wait_iters;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_add_sys(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One CTA per group of kXgRowsPerGroup rows: push this rank's rows of the group to every rank, add
// one to the group's counter there, wait for every rank's rows of this exchange, merge them.
__global__ void __launch_bounds__(kXgThreads) exchange_merge_kernel(const __grid_constant__ XgParams p) {
  __shared__ uint32_t sh_e;
  __shared__ int sh_ok;
  const int c = blockIdx.x;
  const int r0 = c * kXgRowsPerGroup, r1 = min(p.rows, r0 + kXgRowsPerGroup);
  const int nr = r1 - r0;
  const int D = p.d, D4 = p.d / 4;
  const size_t rf = xg_row_floats(D);
  pdl_wait();  // the attention's partial
  pdl_release();
  uint32_t* epochs = reinterpret_cast<uint32_t*>(p.base[p.rank] + kXgEpochsOff);
  if (threadIdx.x == 0) sh_e = epochs[c] + 1u;
  __syncthreads();
  const uint32_t e = sh_e;
  const size_t half = e & 1u;
  // Push: this rank's rows r0..r1 into slot `rank` of half e & 1 of every rank's inbox.
  for (int r = 0; r < p.world; ++r) {
    float* dst = reinterpret_cast<float*>(p.base[r] + kXgInboxOff) + ((half * p.world + p.rank) * p.rows + r0) * rf;
    for (int i = threadIdx.x; i < nr * D4; i += blockDim.x) {
      const int row = i / D4, q = i - row * D4;
      *reinterpret_cast<float4*>(dst + row * rf + 4 * q) = *reinterpret_cast<const float4*>(p.out + (size_t)(r0 + row) * D + 4 * q);
    }
    for (int row = threadIdx.x; row < nr; row += blockDim.x) dst[row * rf + D] = p.lse[r0 + row];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // the rows before the arrivals
    for (int r = 0; r < p.world; ++r) red_add_sys(reinterpret_cast<uint32_t*>(p.base[r] + kXgCountersOff) + c, 1u);
    // Every rank's rows of exchange e are here once the counter reaches e * world.
    const uint32_t* cnt = reinterpret_cast<const uint32_t*>(p.base[p.rank] + kXgCountersOff) + c;
    const uint32_t target = e * (uint32_t)p.world;
    uint32_t it = 0;
    bool ok = (int32_t)(ld_acquire_sys(cnt) - target) >= 0;
    while (!ok && it < p.wait_iters) {
      __nanosleep(kXgSleepNs);
      ++it;
      ok = (int32_t)(ld_acquire_sys(cnt) - target) >= 0;
    }
    if (!ok) record_status(LKV_DEV_WAIT_TIMEOUT);
    sh_ok = ok ? 1 : 0;
    epochs[c] = e;
  }
  __syncthreads();
  __threadfence();  // thread 0's acquire, then the barrier: the rows it saw arrive are read after this
  const bool ok = sh_ok != 0;
  const float* inbox = reinterpret_cast<const float*>(p.base[p.rank] + kXgInboxOff) + half * p.world * p.rows * rf;
  for (int i = threadIdx.x; i < nr * D; i += blockDim.x) {
    const int row = r0 + i / D, ch = i % D;
    float o, l;
    if (ok) {
      float M = -INFINITY;
      for (int r = 0; r < p.world; ++r) M = fmaxf(M, __ldcg(inbox + ((size_t)r * p.rows + row) * rf + D));
      float num = 0.0f, den = 0.0f;
      if (M != -INFINITY) {
        for (int r = 0; r < p.world; ++r) {
          const float* src = inbox + ((size_t)r * p.rows + row) * rf;
          const float lr = __ldcg(src + D);
          if (lr == -INFINITY) continue;
          const float w = expf(lr - M);
          num = fmaf(w, __ldcg(src + ch), num);
          den += w;
        }
      }
      const bool empty = !(den > 0.0f);
      o = empty ? 0.0f : num / den;
      l = empty ? -INFINITY : M + logf(den);
    } else {  // a peer did not arrive in time: this rank's own partial (the status word says so)
      o = p.out[(size_t)row * D + ch];
      l = p.lse[row];
    }
    if (p.out_bf16)
      static_cast<__nv_bfloat16*>(p.merged)[(size_t)row * D + ch] = __float2bfloat16_rn(o);
    else
      static_cast<float*>(p.merged)[(size_t)row * D + ch] = o;
    if (ch == 0 && p.merged_lse != nullptr) p.merged_lse[row] = l;
  }
}

uint32_t g_xg_wait_iters = kXgWaitIters;

}  // namespace

cudaError_t exchange_device_status(int* status, int clear) { return tu_device_status(status, clear); }
cudaError_t exchange_status_attach(int* mirror) { return tu_status_attach(mirror); }
int exchange_set_wait_iters(int64_t v) {
  if (v < 1 || v > (int64_t)kXgWaitIters) return fail(LKV_ERR_ARG, "lkv_debug_set: exchange wait bound %lld outside [1, %u]", (long long)v, kXgWaitIters);
  g_xg_wait_iters = (uint32_t)v;
  return LKV_OK;
}

}  // namespace lkv

using namespace lkv;

extern "C" {

size_t lkv_exchange_region_bytes(int rows, int d, int world) {
  if (rows <= 0 || d <= 0 || world <= 0) return 0;
  return xg_region_bytes(rows, d, world);
}

int lkv_exchange_alloc(int rows, int d, int world, void** base, void* ipc_handle) {
  if (base == nullptr || ipc_handle == nullptr) return fail(LKV_ERR_PTR, "lkv_exchange_alloc: null pointer");
  if (rows <= 0 || d <= 0 || d % 4 != 0 || world <= 0 || world > kXgMaxWorld || xg_groups(rows) > kXgGroupsMax)
    return fail(LKV_ERR_ARG, "lkv_exchange_alloc: rows %d, d %d (a multiple of 4), world %d (at most %d)", rows, d, world, kXgMaxWorld);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, xg_region_bytes(rows, d, world));
  if (e == cudaSuccess) e = cudaMemset(p, 0, xg_region_bytes(rows, d, world));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_exchange_alloc: %s", cudaGetErrorString(e));
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *base = p;
  return LKV_OK;
}

int lkv_exchange_open(const void* ipc_handle, void** peer_base) {
  if (ipc_handle == nullptr || peer_base == nullptr) return fail(LKV_ERR_PTR, "lkv_exchange_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_exchange_open: %s", cudaGetErrorString(e));
  }
  *peer_base = p;
  return LKV_OK;
}

int lkv_exchange_close(void* peer_base) {
  if (peer_base == nullptr) return fail(LKV_ERR_PTR, "lkv_exchange_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(peer_base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_exchange_close: %s", cudaGetErrorString(e));
  }
  return LKV_OK;
}

int lkv_exchange_free(void* base) {
  if (base == nullptr) return fail(LKV_ERR_PTR, "lkv_exchange_free: null pointer");
  cudaError_t e = cudaFree(base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_exchange_free: %s", cudaGetErrorString(e));
  }
  return LKV_OK;
}

int lkv_exchange_merge(const float* out, const float* lse, int rows, int d, int world, int rank, void* const* bases, void* merged, int out_dtype,
                       float* merged_lse, void* stream) {
  if (out == nullptr || lse == nullptr || bases == nullptr || merged == nullptr) return fail(LKV_ERR_PTR, "lkv_exchange_merge: null pointer");
  if (!dtype_ok(out_dtype)) return fail(LKV_ERR_ARG, "lkv_exchange_merge: bad output dtype %d", out_dtype);
  if (rows <= 0 || d <= 0 || d % 4 != 0 || world <= 0 || world > kXgMaxWorld || rank < 0 || rank >= world || xg_groups(rows) > kXgGroupsMax)
    return fail(LKV_ERR_ARG, "lkv_exchange_merge: rows %d, d %d, rank %d of %d", rows, d, rank, world);
  if (!aligned(out, 16)) return fail(LKV_ERR_PTR, "lkv_exchange_merge: the partial output must be 16-byte aligned");
  XgParams p{};
  for (int r = 0; r < world; ++r) {
    if (bases[r] == nullptr || !aligned(bases[r], 256)) return fail(LKV_ERR_PTR, "lkv_exchange_merge: region of rank %d missing or misaligned", r);
    p.base[r] = static_cast<unsigned char*>(bases[r]);
  }
  p.out = out;
  p.lse = lse;
  p.world = world;
  p.rank = rank;
  p.rows = rows;
  p.d = d;
  p.merged = merged;
  p.out_bf16 = out_dtype == LKV_BF16;
  p.merged_lse = merged_lse;
  p.wait_iters = g_xg_wait_iters;
  cudaError_t e = launch_pdl(exchange_merge_kernel, dim3(xg_groups(rows)), dim3(kXgThreads), 0, as_stream(stream), 0, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_exchange_merge: %s", cudaGetErrorString(e));
  }
  return LKV_OK;
}

}  // extern "C"
