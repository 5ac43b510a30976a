// Device-side residency of the tier: admit (lazykv/tiered.py:389-487) and the fetch of the misses.
//
// The reference keeps its residency tables in numpy and brings the selection to the host to update
// them; here they live on the device and the update is one kernel per decode step and layer (one
// CTA per KV head), with the reference's rule unchanged:
//  * a chosen block whose block_slot is -1 misses;
//  * victims are the slots not holding a chosen block, least recently used first, ties by slot
//    index (np.argsort(last_used[free], kind="stable")), assigned to the misses in chosen order;
//  * an evicted block gets block_slot = -1 and evicted_at = step; a filled slot gets its block and
//    last_used = step; every chosen slot gets last_used = step (the gather's put_along_axis).
// Table conventions are the reference's: slot_block [h, n_slots] (block or -1), block_slot
// [h, cap] (pool index 1..n_slots or -1), last_used [h, n_slots] and evicted_at [h, cap] int64.
// The fetch kernel then copies each miss from the host store (pairs in the model dtype, or int8
// records dequantised exactly as lazykv/quant.py:unpack) into its slot of the pool
// [n_slots + 2, h, 2, bs, d].
#include <atomic>
#include <new>
#include "admit.cuh"
#include "common.cuh"

namespace lkv {
namespace {

constexpr int kAdmitThreads = 1024;

__device__ uint32_t admit_scan(uint32_t v, uint32_t* warp_sums) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = warp_sums[lane];
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += x;
    }
    warp_sums[lane] = wi - w;
  }
  __syncthreads();
  const uint32_t r = warp_sums[warp] + incl - v;
  __syncthreads();
  return r;
}

// The m smallest of n distinct 64-bit keys in keys[0, n) (shared memory) move to keys[0, m), in no
// particular order: a radix select of the m-th smallest over the bits in which the keys differ (8
// per pass, from the top), then a stable compaction of the keys at or below it. Each thread holds
// its contiguous share of at most kAdmitSelPer keys in registers across the compaction.
constexpr int kAdmitSelPer = 16;
constexpr int kAdmitSelMax = kAdmitSelPer * kAdmitThreads;

__device__ void select_smallest(uint64_t* keys, int n, int m, uint32_t* warp_sums) {
  __shared__ unsigned long long sh_min, sh_max;
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sh_rem;
  __shared__ uint64_t sh_prefix;
  if (threadIdx.x == 0) {
    sh_min = ~0ull;
    sh_max = 0ull;
    sh_rem = (uint32_t)m;
  }
  __syncthreads();
  unsigned long long lmin = ~0ull, lmax = 0ull;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    lmin = min(lmin, (unsigned long long)keys[i]);
    lmax = max(lmax, (unsigned long long)keys[i]);
  }
  atomicMin(&sh_min, lmin);
  atomicMax(&sh_max, lmax);
  __syncthreads();
  const int hb = 63 - __clzll((long long)(sh_min ^ sh_max));  // the top bit in which keys differ (n >= 2 distinct keys)
  uint64_t mask = hb >= 63 ? 0ull : ~((2ull << hb) - 1ull);    // the bits above it, equal in every key
  uint64_t prefix = (uint64_t)sh_min & mask;
  for (int shift = (hb / 8) * 8; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint64_t x = keys[i];
      if ((x & mask) == prefix) atomicAdd(&hist[(x >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // the digit holding the rem-th smallest of the keys under the prefix
      uint32_t rem = sh_rem, acc = 0u;
      int dg = 255;
      for (int b = 0; b < 256; ++b) {
        if (acc + hist[b] >= rem) {
          dg = b;
          break;
        }
        acc += hist[b];
      }
      sh_rem = rem - acc;
      sh_prefix = prefix | ((uint64_t)dg << shift);
    }
    __syncthreads();
    prefix = sh_prefix;
    mask |= 255ull << shift;
  }
  const uint64_t t = prefix;  // the m-th smallest key
  // Stable compaction of the keys <= t (exactly m: the keys are distinct).
  const int seg = (n + blockDim.x - 1) / blockDim.x;
  const int lo = min(n, (int)threadIdx.x * seg), hi = min(n, lo + seg);
  uint64_t mine[kAdmitSelPer];
  uint32_t cnt = 0;
#pragma unroll
  for (int e = 0; e < kAdmitSelPer; ++e) {
    mine[e] = lo + e < hi ? keys[lo + e] : ~0ull;
    cnt += (lo + e < hi && mine[e] <= t) ? 1u : 0u;
  }
  uint32_t pos = admit_scan(cnt, warp_sums);  // barriers: every read above precedes every write below
#pragma unroll
  for (int e = 0; e < kAdmitSelPer; ++e)
    if (lo + e < hi && mine[e] <= t) keys[pos++] = mine[e];
  __syncthreads();
}

// One CTA per KV head. Shared memory: per slot a 64-bit LRU key (last_used + 4 << 24 | slot), and a
// kept flag; the free slots are bitonic-sorted by key.
__global__ void __launch_bounds__(kAdmitThreads) admit_kernel(const int32_t* __restrict__ chosen, int k, int64_t chosen_ld,
                                                               int32_t* __restrict__ block_slot, int cap, int32_t* __restrict__ slot_block,
                                                               int64_t* __restrict__ last_used, int n_slots, int64_t* __restrict__ evicted_at,
                                                               int64_t step, int32_t* __restrict__ miss_blk, int32_t* __restrict__ miss_slot,
                                                               int32_t* __restrict__ n_miss, int32_t* __restrict__ slots_out, int64_t slots_ld,
                                                               int64_t* __restrict__ miss_total) {
  extern __shared__ uint64_t keys[];  // [P]
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t sh_nfree, sh_nmiss;
  unsigned char* kept = reinterpret_cast<unsigned char*>(keys + 0);  // reused below, see layout
  const int j = blockIdx.x;
  int P = 1;
  while (P < n_slots) P <<= 1;
  kept = reinterpret_cast<unsigned char*>(keys + P);
  const int32_t* ch = chosen + (int64_t)j * chosen_ld;
  int32_t* bslot = block_slot + (int64_t)j * cap;
  int32_t* sblock = slot_block + (int64_t)j * n_slots;
  int64_t* lu = last_used + (int64_t)j * n_slots;

  for (int s = threadIdx.x; s < n_slots; s += blockDim.x) kept[s] = 0;
  __syncthreads();
  // Hits mark their slot kept.
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const int b = ch[i];
    const int s = (b >= 0 && b < cap) ? bslot[b] : -1;
    if (s >= 1 && s <= n_slots) kept[s - 1] = 1;
  }
  __syncthreads();
  // Free slots, compacted in slot order, then sorted by (last_used, slot).
  const int seg = (n_slots + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * seg, hi = min(n_slots, lo + seg);
  uint32_t nf = 0;
  for (int s = lo; s < hi; ++s) nf += !kept[s];
  uint32_t pos = admit_scan(nf, warp_sums);
  for (int s = lo; s < hi; ++s)
    if (!kept[s]) keys[pos++] = ((uint64_t)(lu[s] + 4) << 24) | (uint64_t)s;
  if (threadIdx.x == blockDim.x - 1) sh_nfree = pos;
  // The misses' count first: only that many victims are needed, the smallest keys in order.
  {
    const int segm = (k + blockDim.x - 1) / blockDim.x;
    const int mlo = threadIdx.x * segm, mhi = min(k, mlo + segm);
    uint32_t nm0 = 0;
    for (int i = mlo; i < mhi; ++i) {
      const int b = ch[i];
      nm0 += (b >= 0 && b < cap && bslot[b] < 1);
    }
    const uint32_t before = admit_scan(nm0, warp_sums);
    if (threadIdx.x == blockDim.x - 1) sh_nmiss = before + nm0;
  }
  __syncthreads();
  int n_free = (int)sh_nfree;
  const int m = (int)min(sh_nmiss, (uint32_t)n_free);
  if (m == 0) {
    n_free = 0;  // all hits: no victim needed, nothing to sort
  } else if (m < n_free && n_free > 2048 && n_free <= kAdmitSelMax) {
    select_smallest(keys, n_free, m, warp_sums);  // keys[0, m) = the m smallest, unsorted
    n_free = m;
  }
  int PF = 1;  // the keys left are sorted: the next power of two above their count
  while (PF < n_free) PF <<= 1;
  for (int i = n_free + threadIdx.x; i < PF; i += blockDim.x) keys[i] = ~0ull;
  __syncthreads();
  for (int size = 2; size <= PF; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < PF / 2; i += blockDim.x) {
        const int a = 2 * i - (i & (stride - 1)), b = a + stride;
        const bool asc = (a & size) == 0;
        const uint64_t x = keys[a], y = keys[b];
        if ((x > y) == asc) {
          keys[a] = y;
          keys[b] = x;
        }
      }
      __syncthreads();
    }
  }
  // Misses, ranked in chosen order.
  const int segk = (k + blockDim.x - 1) / blockDim.x;
  const int klo = threadIdx.x * segk, khi = min(k, klo + segk);
  uint32_t nm = 0;
  for (int i = klo; i < khi; ++i) {
    const int b = ch[i];
    nm += (b >= 0 && b < cap && bslot[b] < 1);
  }
  uint32_t rank = admit_scan(nm, warp_sums);
  if (threadIdx.x == blockDim.x - 1) sh_nmiss = rank + nm;
  // Evict every victim's old block first (old blocks are never chosen), then assign.
  for (int i = klo; i < khi; ++i) {
    const int b = ch[i];
    if (!(b >= 0 && b < cap && bslot[b] < 1)) continue;
    const int v = rank < (uint32_t)n_free ? (int)(keys[rank] & 0xffffffull) : -1;
    if (v >= 0) {
      const int old = sblock[v];
      if (old >= 0) {
        bslot[old] = -1;
        if (evicted_at != nullptr) evicted_at[(int64_t)j * cap + old] = step;
      }
    }
    ++rank;
  }
  __syncthreads();
  rank -= nm;
  for (int i = klo; i < khi; ++i) {
    const int b = ch[i];
    if (!(b >= 0 && b < cap && bslot[b] < 1)) continue;
    const int v = rank < (uint32_t)n_free ? (int)(keys[rank] & 0xffffffull) : -1;
    if (v >= 0) {
      sblock[v] = b;
      bslot[b] = v + 1;
      lu[v] = step;
      miss_blk[(int64_t)j * k + rank] = b;
      miss_slot[(int64_t)j * k + rank] = v + 1;
    }
    ++rank;
  }
  __syncthreads();
  // Every chosen slot was used at this step.
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const int b = ch[i];
    const int s = (b >= 0 && b < cap) ? bslot[b] : -1;
    if (s >= 1 && s <= n_slots) lu[s - 1] = step;
    if (slots_out != nullptr) slots_out[(int64_t)j * slots_ld + i] = s;
  }
  if (threadIdx.x == 0) {
    const int nm_j = (int)min(sh_nmiss, (uint32_t)n_free);
    n_miss[j] = nm_j;
    if (miss_total != nullptr && nm_j > 0) atomicAdd(reinterpret_cast<unsigned long long*>(miss_total), (unsigned long long)nm_j);
  }
}

// The admit with the head's tables staged in shared memory (admit.cuh: admit_head), one CTA per
// KV head, used when the staged tables fit in shared memory.
__global__ void __launch_bounds__(kAdmitCtaThreads) admit_staged_kernel(const int32_t* __restrict__ chosen, int k, int64_t chosen_ld,
                                                                         const __grid_constant__ AdmitArgs a) {
  extern __shared__ __align__(16) unsigned char admit_smem[];
  const int j = blockIdx.x;
  admit_stage_lu(a, j, admit_smem);  // last_used is the predecessor's to leave alone: only the chosen ids are its
  pdl_wait();                        // the selection's chosen ids
  pdl_release();                     // the fetch may be placed (it waits for this grid's completion)
  admit_head(a, j, chosen + (int64_t)j * chosen_ld, k, admit_smem, true);
}

// Copy (or dequantise) the misses of every head into their slots; warps stride over the misses.
// An int8 record is first staged whole in the warp's shared memory (16-byte loads, once over the
// link when the store is host memory), then dequantised from there.
constexpr int kFetchWarps = 8;

template <typename T>
__global__ void __launch_bounds__(32 * kFetchWarps) fetch_misses_kernel(const void* __restrict__ store, int store_kind, int64_t width,
                                                                        T* __restrict__ pool, int h, int bs, int d, int k,
                                                                        const int32_t* __restrict__ miss_blk,
                                                                        const int32_t* __restrict__ miss_slot,
                                                                        const int32_t* __restrict__ n_miss) {
  extern __shared__ __align__(16) unsigned char stage_all[];
  const int j = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned char* stage = stage_all + (size_t)warp * ((width + 15) / 16 * 16);
  pdl_wait();  // the admit's miss lists
  pdl_release();  // the attention's CTAs may be placed (they wait for this grid's completion)
  const int n = n_miss[j];
  const int n1 = bs * d, n2 = 2 * n1;
  for (int m = blockIdx.x * kFetchWarps + warp; m < n; m += gridDim.x * kFetchWarps) {
    const int b = miss_blk[(int64_t)j * k + m], slot = miss_slot[(int64_t)j * k + m];
    T* dst = pool + ((int64_t)slot * h + j) * n2;
    if (store_kind == LKV_COLD_INT8) {
      const uint4* rec = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(store) + ((int64_t)b * h + j) * width);
      for (int e = lane; e < (int)(width / 16); e += 32) reinterpret_cast<uint4*>(stage)[e] = rec[e];
      __syncwarp();
      const __half* ks = reinterpret_cast<const __half*>(stage + 2 * n1);
      const __half* kz = ks + d;
      const __half* vs = ks + 2 * d;
      const __half* vz = vs + bs;
      if constexpr (sizeof(T) == 2) {
        // bf16 slots (d a multiple of 8): lane e takes 8 consecutive values of one token, so one
        // 8-byte code load, the scales as 16-byte loads (keys: per channel) or one value (values:
        // per token), and one 16-byte store. Same arithmetic as below: (q + 128) * scale (exact),
        // then + zero (one rounding), then rounded to bf16.
        for (int e8 = lane; e8 < n2 / 8; e8 += 32) {
          const int e = 8 * e8;
          const int kv = e / n1, rem = e - kv * n1, t = rem / d, c = rem - t * d;
          const uint2 cw = *reinterpret_cast<const uint2*>(stage + e);
          const uint32_t w[2] = {cw.x ^ 0x80808080u, cw.y ^ 0x80808080u};  // (q + 128) as unsigned bytes
          float sc[8], z[8];
          if (kv == 0) {
            const uint4 sv = *reinterpret_cast<const uint4*>(ks + c), zv = *reinterpret_cast<const uint4*>(kz + c);
            const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w}, zw[4] = {zv.x, zv.y, zv.z, zv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&sw[i]));
              const float2 bz = __half22float2(*reinterpret_cast<const __half2*>(&zw[i]));
              sc[2 * i] = a.x, sc[2 * i + 1] = a.y, z[2 * i] = bz.x, z[2 * i + 1] = bz.y;
            }
          } else {
            const float s1 = __half2float(vs[t]), z1 = __half2float(vz[t]);
#pragma unroll
            for (int i = 0; i < 8; ++i) sc[i] = s1, z[i] = z1;
          }
          uint32_t out[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float q0 = (float)((w[i / 2] >> (16 * (i & 1))) & 0xffu), q1 = (float)((w[i / 2] >> (16 * (i & 1) + 8)) & 0xffu);
            const float v0 = __fadd_rn(__fmul_rn(q0, sc[2 * i]), z[2 * i]), v1 = __fadd_rn(__fmul_rn(q1, sc[2 * i + 1]), z[2 * i + 1]);
            const __nv_bfloat162 pr = __floats2bfloat162_rn(v0, v1);
            out[i] = *reinterpret_cast<const uint32_t*>(&pr);
          }
          *reinterpret_cast<uint4*>(dst + e) = make_uint4(out[0], out[1], out[2], out[3]);
        }
        __syncwarp();
        continue;
      }
      for (int e = lane; e < n2; e += 32) {
        const int kv = e / n1, rem = e % n1, t = rem / d, c = rem % d;
        const float q = (float)reinterpret_cast<const int8_t*>(stage)[e];
        const float sc = __half2float(kv ? vs[t] : ks[c]), z = __half2float(kv ? vz[t] : kz[c]);
        dst[e] = from_f32<T>(__fadd_rn(__fmul_rn(__fadd_rn(q, 128.0f), sc), z));  // quant.py:103-104
      }
      __syncwarp();
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(store) + ((int64_t)b * h + j) * n2);
      uint4* o = reinterpret_cast<uint4*>(dst);
      for (int e = lane; e < n2 * (int)sizeof(T) / 16; e += 32) o[e] = src[e];
    }
  }
}

// fetch_misses_kernel for int8 records into bf16 slots at bs 16, d 64: a warp takes one miss at a
// time (admit.cuh: fetch_record_i8_bf16).
__global__ void __launch_bounds__(32 * kFetchWarps) fetch_misses_i8_bf16_kernel(const uint8_t* __restrict__ store, __nv_bfloat16* __restrict__ pool,
                                                                               int h, int k, const int32_t* __restrict__ miss_blk,
                                                                               const int32_t* __restrict__ miss_slot,
                                                                               const int32_t* __restrict__ n_miss) {
  __shared__ __align__(16) unsigned char stage_all[kFetchWarps * kFetchStageBytes];
  const int j = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  unsigned char* stage = stage_all + warp * kFetchStageBytes;
  pdl_wait();     // the admit's miss lists
  pdl_release();  // the attention's CTAs may be placed (they wait for this grid's completion)
  const int n = n_miss[j];
  for (int m = blockIdx.x * kFetchWarps + warp; m < n; m += gridDim.x * kFetchWarps) {
    const int b = miss_blk[(int64_t)j * k + m], slot = miss_slot[(int64_t)j * k + m];
    fetch_record_i8_bf16(store + ((int64_t)b * h + j) * kRecBytes16x64, pool + ((int64_t)slot * h + j) * 2048, stage);
  }
}

}  // namespace
}  // namespace lkv

using namespace lkv;

extern "C" int lkv_tier_admit(const int32_t* chosen, int h, int k, int64_t chosen_ld, int32_t* block_slot, int cap, int32_t* slot_block,
                              int64_t* last_used, int n_slots, int64_t* evicted_at, int64_t step, const void* store, int store_kind,
                              void* pool, int bs, int d, int dtype, int32_t* miss_blk, int32_t* miss_slot, int32_t* n_miss,
                              int32_t* slots_out, int64_t slots_ld, int64_t* miss_total, void* stream) {
  if (!dtype_ok(dtype)) return fail(LKV_ERR_ARG, "lkv_tier_admit: bad dtype %d", dtype);
  if (store_kind != LKV_COLD_INT8 && store_kind != LKV_COLD_PAIRS) return fail(LKV_ERR_ARG, "lkv_tier_admit: bad store kind %d", store_kind);
  if (h <= 0 || k <= 0 || cap <= 0 || n_slots < k) return fail(LKV_ERR_ARG, "lkv_tier_admit: need h, k, cap > 0 and n_slots >= k (%d < %d)", n_slots, k);
  if (n_slots > (1 << 16)) return fail(LKV_ERR_ARG, "lkv_tier_admit: %d slots above 65536", n_slots);
  if (chosen == nullptr || block_slot == nullptr || slot_block == nullptr || last_used == nullptr || store == nullptr || pool == nullptr ||
      miss_blk == nullptr || miss_slot == nullptr || n_miss == nullptr)
    return fail(LKV_ERR_PTR, "lkv_tier_admit: null pointer");
  if (!aligned(store, 16) || !aligned(pool, 16)) return fail(LKV_ERR_PTR, "lkv_tier_admit: store and pool must be 16-byte aligned");
  if (bs % 8 || d % 8 || bs > 128 || d > 256) return fail(LKV_ERR_ARG, "lkv_tier_admit: bs and d must be multiples of 8 (bs <= 128, d <= 256)");
  int P = 1;
  while (P < n_slots) P <<= 1;
  cudaStream_t st = as_stream(stream);
  // The staged admit when its tables fit in shared memory (keys, last_used, chosen, their slots,
  // slot_block, the kept flags); else the one that works on the tables in global memory.
  const size_t staged = admit_smem_bytes(n_slots, k);
  if (staged <= 200 * 1024) {
    AdmitArgs aa{};
    aa.block_slot = block_slot;
    aa.cap = cap;
    aa.slot_block = slot_block;
    aa.last_used = last_used;
    aa.n_slots = n_slots;
    aa.evicted_at = evicted_at;
    aa.step = step;
    aa.miss_blk = miss_blk;
    aa.miss_slot = miss_slot;
    aa.n_miss = n_miss;
    aa.slots_out = slots_out;
    aa.slots_ld = slots_ld;
    aa.miss_total = miss_total;
    cudaError_t e = cudaSuccess;
    if (staged > 48 * 1024) {
      // The attribute is raised once per device to the largest size a call has needed.
      static std::atomic<int> set_bytes[64];
      int dev = 0;
      e = cudaGetDevice(&dev);
      std::atomic<int>& cur = set_bytes[dev & 63];
      if (e == cudaSuccess && cur.load() < (int)staged) {
        e = cudaFuncSetAttribute(admit_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)staged);
        if (e == cudaSuccess) cur.store((int)staged);
      }
    }
    if (e == cudaSuccess) e = launch_pdl(admit_staged_kernel, dim3(h), dim3(kAdmitCtaThreads), staged, st, 0, chosen, k, chosen_ld, aa);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(LKV_ERR_CUDA, "lkv_tier_admit(admit): %s", cudaGetErrorString(e));
    }
  } else {
    const size_t smem = (size_t)P * 8 + (size_t)((n_slots + 15) / 16 * 16);
    if (smem > 200 * 1024) return fail(LKV_ERR_ARG, "lkv_tier_admit: %d slots need %zu bytes of shared memory", n_slots, smem);
    if (smem > 48 * 1024) cudaFuncSetAttribute(admit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    admit_kernel<<<h, kAdmitThreads, smem, st>>>(chosen, k, chosen_ld, block_slot, cap, slot_block, last_used, n_slots, evicted_at, step,
                                                  miss_blk, miss_slot, n_miss, slots_out, slots_ld, miss_total);
    if (int rc = launched("lkv_tier_admit(admit)")) return rc;
  }
  const int64_t width = lkv_packed_pair_bytes(bs, d);
  if (store_kind == LKV_COLD_INT8 && dtype == LKV_BF16 && bs == 16 && d == 64) {
    // Up to four CTAs per SM over the heads, enough for every selected block to miss.
    int per_head = (k + kFetchWarps - 1) / kFetchWarps;
    const int cap_ctas = (4 * kNumSMs + h - 1) / h;
    if (per_head > cap_ctas) per_head = cap_ctas;
    cudaError_t e = launch_pdl(fetch_misses_i8_bf16_kernel, dim3(per_head, h), dim3(32 * kFetchWarps), 0, st, 0, static_cast<const uint8_t*>(store),
                               static_cast<__nv_bfloat16*>(pool), h, k, (const int32_t*)miss_blk, (const int32_t*)miss_slot, (const int32_t*)n_miss);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(LKV_ERR_CUDA, "lkv_tier_admit(fetch): %s", cudaGetErrorString(e));
    }
    return launched("lkv_tier_admit(fetch)");
  }
  const int fetch_ctas = (k + kFetchWarps - 1) / kFetchWarps < 32 ? (k + kFetchWarps - 1) / kFetchWarps : 32;
  dim3 grid(fetch_ctas, h);
  const size_t fsmem = store_kind == LKV_COLD_INT8 ? (size_t)kFetchWarps * ((width + 15) / 16 * 16) : 0;
  if (fsmem > 200 * 1024) return fail(LKV_ERR_ARG, "lkv_tier_admit: records of %lld bytes are too wide to stage", (long long)width);
  cudaError_t e = cudaSuccess;
  if (dtype == LKV_BF16) {
    auto kern = fetch_misses_kernel<__nv_bfloat16>;
    if (fsmem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsmem);
    e = launch_pdl(kern, grid, dim3(32 * kFetchWarps), fsmem, st, 0, store, store_kind, width, static_cast<__nv_bfloat16*>(pool), h, bs, d, k,
                   (const int32_t*)miss_blk, (const int32_t*)miss_slot, (const int32_t*)n_miss);
  } else {
    auto kern = fetch_misses_kernel<float>;
    if (fsmem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsmem);
    e = launch_pdl(kern, grid, dim3(32 * kFetchWarps), fsmem, st, 0, store, store_kind, width, static_cast<float*>(pool), h, bs, d, k,
                   (const int32_t*)miss_blk, (const int32_t*)miss_slot, (const int32_t*)n_miss);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_tier_admit(fetch): %s", cudaGetErrorString(e));
  }
  return launched("lkv_tier_admit(fetch)");
}

// The bitmap of a given selection: one CTA per head clears the head's words, then sets the bit of
// every listed id in [0, 32 * words); -1 entries (padding) and ids past the bitmap are skipped.
__global__ void __launch_bounds__(256) mark_blocks_kernel(const int32_t* __restrict__ ids, int k, int64_t ld, uint32_t* __restrict__ bitmap,
                                                          int words) {
  const int j = blockIdx.x;
  uint32_t* row = bitmap + (int64_t)j * words;
  for (int w = threadIdx.x; w < words; w += blockDim.x) row[w] = 0u;
  __syncthreads();
  const int32_t* r = ids + (int64_t)j * ld;
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const int b = r[i];
    if (b >= 0 && b < words * 32) atomicOr(row + (b >> 5), 1u << (b & 31));
  }
}

extern "C" int lkv_mark_blocks(const int32_t* ids, int h, int k, int64_t ids_ld, uint32_t* bitmap, int bitmap_words, void* stream) {
  if (h <= 0 || k < 0 || bitmap_words <= 0 || ids_ld < k) return fail(LKV_ERR_ARG, "lkv_mark_blocks: need h, bitmap_words > 0, k >= 0, ids_ld >= k");
  if (bitmap == nullptr || (k > 0 && ids == nullptr)) return fail(LKV_ERR_PTR, "lkv_mark_blocks: null pointer");
  mark_blocks_kernel<<<h, 256, 0, as_stream(stream)>>>(ids, k, ids_ld, bitmap, bitmap_words);
  return launched("lkv_mark_blocks");
}

// ---- Ragged rows, cold tier in pinned host memory: the records a step attends, staged ----
//
// One CTA per 256-candidate chunk of a (sequence, KV head) row (the score kernel's work list); a
// warp per candidate block not in the row's excluded bitmap reads its record over the link with
// 16-byte loads (five in flight per lane) and stores it at the block's staged row, so that the
// attention that follows reads it from HBM. The rows of head 0 also write the staged table entry of
// each candidate (its staged row, or -1 where the block table names no store row).
constexpr int kStageWarps = 8;
constexpr int kStageChunk = 256;
constexpr int kStageInflight = 5;

__global__ void __launch_bounds__(32 * kStageWarps) ragged_stage_kernel(const uint4* __restrict__ records, int64_t n_records, int heads, int width16,
                                                                        const int32_t* __restrict__ table, int64_t table_stride,
                                                                        const int2* __restrict__ work, const int4* __restrict__ row_info,
                                                                        const uint32_t* __restrict__ excluded, int bitmap_words, uint4* __restrict__ stage,
                                                                        int64_t stage_rows, const int32_t* __restrict__ stage_first,
                                                                        int32_t* __restrict__ stage_table, int64_t stage_stride) {
  const int2 wk = work[blockIdx.x];
  const int row = wk.x, first = wk.y;
  const int seq = row / heads, head = row - seq * heads;
  const int end = min(first + kStageChunk, row_info[row].z);
  const int64_t sf = stage_first[seq];
  const int32_t* tab = table + (int64_t)seq * table_stride;
  if (head == 0) {
    for (int c = first + (int)threadIdx.x; c < end; c += blockDim.x) {
      const int src = tab[1 + c];
      stage_table[(int64_t)seq * stage_stride + 1 + c] = (src >= 0 && src < n_records && sf + c < stage_rows) ? (int32_t)(sf + c) : -1;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t* ex = excluded != nullptr ? excluded + (int64_t)row * bitmap_words : nullptr;
  for (int c = first + warp; c < end; c += kStageWarps) {
    const int b = 1 + c;
    if (ex != nullptr && ((ex[b >> 5] >> (b & 31)) & 1u)) continue;
    const int src = tab[b];
    if (src < 0 || src >= n_records || sf + c >= stage_rows) continue;
    const uint4* s = records + ((int64_t)src * heads + head) * width16;
    uint4* d = stage + ((sf + c) * heads + head) * width16;
    for (int base = 0; base < width16; base += 32 * kStageInflight) {
      uint4 v[kStageInflight];
#pragma unroll
      for (int u = 0; u < kStageInflight; ++u) {
        const int i = base + 32 * u + lane;
        if (i < width16) v[u] = __ldcs(s + i);
      }
#pragma unroll
      for (int u = 0; u < kStageInflight; ++u) {
        const int i = base + 32 * u + lane;
        if (i < width16) d[i] = v[u];
      }
    }
  }
}

extern "C" int lkv_ragged_stage_records(const uint8_t* records, int64_t n_records, int heads, int width, const int32_t* table, int64_t table_stride,
                                        const int32_t* work, int n_work, const int32_t* row_info, const uint32_t* excluded, int bitmap_words,
                                        uint8_t* stage, int64_t stage_rows, const int32_t* stage_first, int32_t* stage_table, int64_t stage_stride,
                                        void* stream) {
  const char* who = "lkv_ragged_stage_records";
  if (records == nullptr || table == nullptr || work == nullptr || row_info == nullptr || stage == nullptr || stage_first == nullptr ||
      stage_table == nullptr)
    return fail(LKV_ERR_PTR, "%s: null pointer", who);
  if (heads <= 0 || width <= 0 || width % 16 || n_work < 0 || n_records <= 0 || stage_rows <= 0 || (excluded != nullptr && bitmap_words <= 0))
    return fail(LKV_ERR_ARG, "%s: bad shape (heads %d, width %d, work %d)", who, heads, width, n_work);
  if (!aligned(records, 16) || !aligned(stage, 16) || !aligned(work, 8) || !aligned(row_info, 16))
    return fail(LKV_ERR_PTR, "%s: records and stage must be 16-byte aligned (work 8, row info 16)", who);
  if (n_work == 0) return LKV_OK;
  ragged_stage_kernel<<<n_work, 32 * kStageWarps, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint4*>(records), n_records, heads, width / 16, table, table_stride, reinterpret_cast<const int2*>(work),
      reinterpret_cast<const int4*>(row_info), excluded, bitmap_words, reinterpret_cast<uint4*>(stage), stage_rows, stage_first, stage_table,
      stage_stride);
  return launched(who);
}

// ---- Decode-time KV append into the pool's current block ----
//
// T tokens of keys and values (element (head, token, channel) at head * s_head + token * s_tok +
// channel, in elements) into a pool slot [h, 2, bs, d] at token positions fill .. fill + T - 1: one
// launch in place of a copy per half. Elements move as raw 2- or 4-byte words.
template <typename W>
__global__ void __launch_bounds__(256) append_tokens_kernel(const W* __restrict__ k, int64_t ksh, int64_t kst, const W* __restrict__ v, int64_t vsh,
                                                            int64_t vst, W* __restrict__ slot, int h, int t, int d, int bs, int fill) {
  const int64_t n = (int64_t)h * t * d;  // elements per half
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < 2 * n; i += (int64_t)gridDim.x * blockDim.x) {
    const int half = i >= n ? 1 : 0;
    const int64_t r = i - half * n;
    const int c = (int)(r % d);
    const int64_t ht = r / d;
    const int tok = (int)(ht % t), head = (int)(ht / t);
    const W* src = half ? v + head * vsh + tok * vst : k + head * ksh + tok * kst;
    slot[((int64_t)head * 2 + half) * bs * d + (int64_t)(fill + tok) * d + c] = src[c];
  }
}

extern "C" int lkv_append_tokens(const void* k, int64_t k_s_head, int64_t k_s_tok, const void* v, int64_t v_s_head, int64_t v_s_tok, int h, int t,
                                 int d, int dtype, void* slot, int bs, int fill, void* stream) {
  if (!dtype_ok(dtype)) return fail(LKV_ERR_ARG, "lkv_append_tokens: bad dtype %d", dtype);
  if (k == nullptr || v == nullptr || slot == nullptr) return fail(LKV_ERR_PTR, "lkv_append_tokens: null pointer");
  if (h <= 0 || t <= 0 || d <= 0 || bs <= 0 || fill < 0 || fill + t > bs)
    return fail(LKV_ERR_ARG, "lkv_append_tokens: %d tokens at fill %d do not fit a block of %d", t, fill, bs);
  const int64_t total = 2ll * h * t * d;
  const int blocks = (int)((total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024);
  cudaStream_t st = as_stream(stream);
  if (dtype == LKV_BF16)
    append_tokens_kernel<uint16_t><<<blocks, 256, 0, st>>>(static_cast<const uint16_t*>(k), k_s_head, k_s_tok, static_cast<const uint16_t*>(v),
                                                            v_s_head, v_s_tok, static_cast<uint16_t*>(slot), h, t, d, bs, fill);
  else
    append_tokens_kernel<uint32_t><<<blocks, 256, 0, st>>>(static_cast<const uint32_t*>(k), k_s_head, k_s_tok, static_cast<const uint32_t*>(v),
                                                            v_s_head, v_s_tok, static_cast<uint32_t*>(slot), h, t, d, bs, fill);
  return launched("lkv_append_tokens");
}

// ---- One resident-split decode step in one call (lkv_split_step) ----

struct lkv_split_events {
  cudaEvent_t fork;     // the selection is done: the admit may start
  cudaEvent_t done;     // the admit is done
  bool pending;         // done has been recorded at least once
};

extern "C" int lkv_split_events_create(lkv_split_events** out) {
  if (out == nullptr) return fail(LKV_ERR_PTR, "lkv_split_events_create: null pointer");
  auto* ev = new (std::nothrow) lkv_split_events{};
  if (ev == nullptr) return fail(LKV_ERR_ARG, "lkv_split_events_create: out of host memory");
  cudaError_t e = cudaEventCreateWithFlags(&ev->fork, cudaEventDisableTiming);
  if (e == cudaSuccess) {
    e = cudaEventCreateWithFlags(&ev->done, cudaEventDisableTiming);
    if (e != cudaSuccess) cudaEventDestroy(ev->fork);
  }
  if (e != cudaSuccess) {
    delete ev;
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_split_events_create: %s", cudaGetErrorString(e));
  }
  *out = ev;
  return LKV_OK;
}

extern "C" int lkv_split_events_destroy(lkv_split_events* ev) {
  if (ev == nullptr) return LKV_OK;
  cudaEventDestroy(ev->fork);
  cudaEventDestroy(ev->done);
  cudaGetLastError();  // a context torn down at exit: nothing left to release
  delete ev;
  return LKV_OK;
}

extern "C" int lkv_split_join(lkv_split_events* ev, void* stream) {
  if (ev == nullptr) return fail(LKV_ERR_PTR, "lkv_split_join: null events");
  if (!ev->pending) return LKV_OK;
  const cudaError_t e = cudaStreamWaitEvent(as_stream(stream), ev->done, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_split_join: %s", cudaGetErrorString(e));
  }
  return LKV_OK;
}

extern "C" int lkv_split_wait(lkv_split_events* ev) {
  if (ev == nullptr) return fail(LKV_ERR_PTR, "lkv_split_wait: null events");
  if (!ev->pending) return LKV_OK;
  const cudaError_t e = cudaEventSynchronize(ev->done);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_split_wait: %s", cudaGetErrorString(e));
  }
  return LKV_OK;
}

extern "C" int lkv_split_step(const lkv_split_step_args* a, lkv_split_events* ev, void* stream, void* admit_stream) {
  if (a == nullptr || ev == nullptr) return fail(LKV_ERR_PTR, "lkv_split_step: null arguments or events");
  cudaStream_t st = as_stream(stream), side = as_stream(admit_stream);
  if (st == side) return fail(LKV_ERR_ARG, "lkv_split_step: the admit needs a stream of its own");
  if (int rc = lkv_split_join(ev, stream)) return rc;
  if (!a->selected) {
    if (int rc = lkv_quest_topk_resident(a->q, a->q_dtype, a->hq, a->h, a->d, a->kmin, a->kmax, a->meta_dtype, a->m_head, a->first_block, a->n_cand,
                                         a->k, a->bound_mode, a->chosen, a->chosen_ld, a->block_slot, a->cap, a->hot, a->hot_ld, a->bitmap,
                                         a->bitmap_words, a->sel_workspace, a->sel_workspace_bytes, stream))
      return rc;
  }
  cudaError_t e = cudaEventRecord(ev->fork, st);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_split_step(fork): %s", cudaGetErrorString(e));
  }
  if (int rc = lkv_exact_attention(a->q, a->hq, a->h, a->d, a->bs, a->hot_set, a->cold_set, a->scale, a->out, a->out_dtype, a->lse, nullptr, nullptr,
                                   a->att_workspace, a->att_workspace_bytes, stream))
    return rc;
  // Launched after the attention, so that the attention's CTAs are placed first.
  e = cudaStreamWaitEvent(side, ev->fork, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_split_step(wait): %s", cudaGetErrorString(e));
  }
  if (int rc = lkv_tier_admit(a->chosen, a->h, a->k, a->chosen_ld, a->block_slot, a->cap, a->slot_block, a->last_used, a->n_slots, a->evicted_at,
                              a->step, a->store, a->store_kind, a->pool, a->bs, a->d, a->pool_dtype, a->miss_blk, a->miss_slot, a->n_miss, nullptr, 0,
                              a->miss_total, admit_stream))
    return rc;
  e = cudaEventRecord(ev->done, side);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_split_step(done): %s", cudaGetErrorString(e));
  }
  ev->pending = true;
  return LKV_OK;
}
