// The device admit of one KV head and the fetch of one missed block: the device functions of the
// staged admit kernel and the vectorised fetch kernel (tier.cu).
//
// Admit (lazykv/tiered.py:389-463), for one head, by one CTA of kAdmitCtaThreads threads:
//  * a chosen block whose block_slot is -1 misses;
//  * victims are the slots not holding a chosen block, least recently used first, ties by slot
//    index (np.argsort(last_used[free], kind="stable")), assigned to the misses in chosen order;
//  * an evicted block gets block_slot = -1 and evicted_at = step; a filled slot gets its block and
//    last_used = step; every chosen slot gets last_used = step (the gather's put_along_axis).
// Tables: slot_block [h, n_slots] (block or -1), block_slot [h, cap] (pool index 1..n_slots or -1),
// last_used [h, n_slots] and evicted_at [h, cap] int64. The head's chosen ids, each chosen block's
// current slot (one gather of block_slot), slot_block and last_used are staged in shared memory;
// every phase works on the staged copies and the changes go back at the end.
#pragma once

#include "common.cuh"

namespace lkv {

constexpr int kAdmitCtaThreads = 1024;

struct AdmitArgs {
  int32_t* block_slot;
  int cap;
  int32_t* slot_block;
  int64_t* last_used;
  int n_slots;
  int64_t* evicted_at;
  int64_t step;
  int32_t* miss_blk;   // [h, k]
  int32_t* miss_slot;  // [h, k]
  int32_t* n_miss;     // [h]
  int32_t* slots_out;  // [h, slots_ld] (optional)
  int64_t slots_ld;
  int64_t* miss_total;  // optional: every head's misses added to it (a running count)
};

// Shared-memory bytes of admit_head for n_slots slots and k chosen blocks.
__host__ __device__ inline size_t admit_smem_bytes(int n_slots, int k) {
  int P = 1;
  while (P < n_slots) P <<= 1;
  return (size_t)P * 8 + (size_t)n_slots * 8 + (size_t)k * 8 + (size_t)n_slots * 4 + (size_t)((n_slots + 15) / 16 * 16);
}

// Exclusive block-wide scan (every thread of the CTA calls it; up to 32 warps).
__device__ __forceinline__ uint32_t admit_block_scan(uint32_t v, uint32_t* warp_sums) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = lane < nw ? warp_sums[lane] : 0u;
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

// Stages head j's last_used where admit_head reads it (all threads of the CTA; no barrier at the
// end): a kernel can do this before it waits for the chosen ids.
__device__ __forceinline__ void admit_stage_lu(const AdmitArgs& a, int j, unsigned char* smem) {
  int P = 1;
  while (P < a.n_slots) P <<= 1;
  int64_t* lu_s = reinterpret_cast<int64_t*>(smem + (size_t)P * 8);
  const int64_t* lu = a.last_used + (int64_t)j * a.n_slots;
  for (int s = threadIdx.x; s < a.n_slots; s += blockDim.x) lu_s[s] = lu[s];
}

// The admit of head j with the chosen ids ch [k] (global memory), by the whole CTA. smem holds
// admit_smem_bytes(n_slots, k) bytes; when `lu_staged` the head's last_used is already in place
// (admit_stage_lu). Writes the tables back, the miss lists, n_miss[j] and slots_out[j].
static __device__ void admit_head(const AdmitArgs& a, int j, const int32_t* ch, int k, unsigned char* smem, bool lu_staged) {
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t sh_nfree, sh_nmiss;
  const int n_slots = a.n_slots, cap = a.cap;
  int P = 1;
  while (P < n_slots) P <<= 1;
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem);
  int64_t* lu_s = reinterpret_cast<int64_t*>(keys + P);
  int32_t* ch_s = reinterpret_cast<int32_t*>(lu_s + n_slots);
  int32_t* cs_s = ch_s + k;
  int32_t* sb_s = cs_s + k;
  unsigned char* kept = reinterpret_cast<unsigned char*>(sb_s + n_slots);
  int32_t* bslot = a.block_slot + (int64_t)j * cap;
  int32_t* sblock = a.slot_block + (int64_t)j * n_slots;
  int64_t* lu = a.last_used + (int64_t)j * n_slots;
  for (int s = threadIdx.x; s < n_slots; s += blockDim.x) {
    sb_s[s] = sblock[s];
    if (!lu_staged) lu_s[s] = lu[s];
    kept[s] = 0;
  }
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const int b = __ldcg(ch + i);
    ch_s[i] = b;
    cs_s[i] = (b >= 0 && b < cap) ? bslot[b] : -1;
  }
  __syncthreads();
  // Hits mark their slot kept.
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const int sl = cs_s[i];
    if (sl >= 1 && sl <= n_slots) kept[sl - 1] = 1;
  }
  __syncthreads();
  // Free slots, compacted in slot order, then sorted by (last_used, slot). Only the free slots are
  // sorted (with as many slots as the selection keeps, they are exactly the victims): a bitonic
  // sort over the next power of two above their count.
  const int seg = (n_slots + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * seg, hi = min(n_slots, lo + seg);
  uint32_t nf = 0;
  for (int s = lo; s < hi; ++s) nf += !kept[s];
  uint32_t pos = admit_block_scan(nf, warp_sums);
  for (int s = lo; s < hi; ++s)
    if (!kept[s]) keys[pos++] = ((uint64_t)(lu_s[s] + 4) << 24) | (uint64_t)s;
  if (threadIdx.x == blockDim.x - 1) sh_nfree = pos;
  __syncthreads();
  const int n_free = (int)sh_nfree;
  int PF = 1;
  while (PF < n_free) PF <<= 1;
  for (int i = n_free + threadIdx.x; i < PF; i += blockDim.x) keys[i] = ~0ull;
  __syncthreads();
  for (int size = 2; size <= PF; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < PF / 2; i += blockDim.x) {
        const int x0 = 2 * i - (i & (stride - 1)), x1 = x0 + stride;
        const bool asc = (x0 & size) == 0;
        const uint64_t x = keys[x0], y = keys[x1];
        if ((x > y) == asc) {
          keys[x0] = y;
          keys[x1] = x;
        }
      }
      __syncthreads();
    }
  }
  // Misses, ranked in chosen order; each takes the next victim: the victim's old block is evicted,
  // the slot gets the missed block (old blocks are never chosen, so no entry is written twice).
  const int segk = (k + blockDim.x - 1) / blockDim.x;
  const int klo = threadIdx.x * segk, khi = min(k, klo + segk);
  uint32_t nm = 0;
  for (int i = klo; i < khi; ++i) {
    const int b = ch_s[i];
    nm += (b >= 0 && b < cap && cs_s[i] < 1);
  }
  uint32_t rank = admit_block_scan(nm, warp_sums);
  if (threadIdx.x == blockDim.x - 1) sh_nmiss = rank + nm;
  for (int i = klo; i < khi; ++i) {
    const int b = ch_s[i];
    if (!(b >= 0 && b < cap && cs_s[i] < 1)) continue;
    const int v = rank < (uint32_t)n_free ? (int)(keys[rank] & 0xffffffull) : -1;
    if (v >= 0) {
      const int old = sb_s[v];
      if (old >= 0) {
        bslot[old] = -1;
        if (a.evicted_at != nullptr) a.evicted_at[(int64_t)j * cap + old] = a.step;
      }
      sb_s[v] = b;
      lu_s[v] = a.step;
      cs_s[i] = v + 1;
      bslot[b] = v + 1;
      a.miss_blk[(int64_t)j * k + rank] = b;
      a.miss_slot[(int64_t)j * k + rank] = v + 1;
    }
    ++rank;
  }
  __syncthreads();
  // Every chosen slot was used at this step.
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const int sl = cs_s[i];
    if (sl >= 1 && sl <= n_slots) lu_s[sl - 1] = a.step;
    if (a.slots_out != nullptr) a.slots_out[(int64_t)j * a.slots_ld + i] = sl;
  }
  __syncthreads();
  for (int s = threadIdx.x; s < n_slots; s += blockDim.x) {
    sblock[s] = sb_s[s];
    lu[s] = lu_s[s];
  }
  if (threadIdx.x == 0) {
    const int nm_j = (int)min(sh_nmiss, (uint32_t)n_free);
    a.n_miss[j] = nm_j;
    if (a.miss_total != nullptr && nm_j > 0) atomicAdd(reinterpret_cast<unsigned long long*>(a.miss_total), (unsigned long long)nm_j);
  }
}

// One warp dequantises the int8 record at `rec` (global, 2,368 bytes: bs 16, d 64) into the bf16
// slot row `dst` (2,048 values: keys then values, token-major). `stage` is this warp's 2,944 bytes of
// shared memory (16-byte aligned): the record, then its 64 key scales and 64 zeros as float32. A code
// becomes (q + 128) as a float exactly by a byte permute into 2^23 + (q + 128) and one subtraction
// (two values at a time); then (q + 128) * scale + zero (the product is exact, so the fused form
// rounds once, as the product and sum do) and the bf16 rounding: unpack's values bit for bit.
constexpr int kRecBytes16x64 = 2368;
constexpr int kFetchStageBytes = 2944;

__device__ __forceinline__ void fetch_record_i8_bf16(const uint8_t* rec_g, __nv_bfloat16* dst_g, unsigned char* stage) {
  const int lane = threadIdx.x & 31;
  float* kf = reinterpret_cast<float*>(stage + kRecBytes16x64 + 64);  // 2,432: 16-byte aligned
  const uint4* rec = reinterpret_cast<const uint4*>(rec_g);
#pragma unroll
  for (int e = lane; e < kRecBytes16x64 / 16; e += 32) reinterpret_cast<uint4*>(stage)[e] = rec[e];
  __syncwarp();
  {  // key scales and zeros (float16 at 2,048 and 2,176) as float32: lane l converts channels 2l, 2l + 1
    const __half2 sc2 = reinterpret_cast<const __half2*>(stage + 2048)[lane];
    const __half2 zr2 = reinterpret_cast<const __half2*>(stage + 2176)[lane];
    reinterpret_cast<float2*>(kf)[lane] = __half22float2(sc2);
    reinterpret_cast<float2*>(kf + 64)[lane] = __half22float2(zr2);
  }
  __syncwarp();
  uint4* dst = reinterpret_cast<uint4*>(dst_g);
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int e8 = lane + 32 * it;  // chunk of 8 values: chunks 0..127 keys, 128..255 values
    const int kv = e8 >> 7, t = (e8 >> 3) & 15, c = (e8 & 7) * 8;
    const uint2 cw = *reinterpret_cast<const uint2*>(stage + 8 * e8);
    const uint32_t a0 = cw.x ^ 0x80808080u, a1 = cw.y ^ 0x80808080u;
    const float2 m23 = make_float2(-8388608.0f, -8388608.0f);
    float2 q[4];
    q[0] = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(a0, 0x4b000000u, 0x7650)), __uint_as_float(__byte_perm(a0, 0x4b000000u, 0x7651))), m23);
    q[1] = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(a0, 0x4b000000u, 0x7652)), __uint_as_float(__byte_perm(a0, 0x4b000000u, 0x7653))), m23);
    q[2] = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(a1, 0x4b000000u, 0x7650)), __uint_as_float(__byte_perm(a1, 0x4b000000u, 0x7651))), m23);
    q[3] = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(a1, 0x4b000000u, 0x7652)), __uint_as_float(__byte_perm(a1, 0x4b000000u, 0x7653))), m23);
    float2 sc[4], zr[4];
    if (kv == 0) {  // keys: per channel
      const float4 s0 = *reinterpret_cast<const float4*>(kf + c), s1 = *reinterpret_cast<const float4*>(kf + c + 4);
      const float4 z0 = *reinterpret_cast<const float4*>(kf + 64 + c), z1 = *reinterpret_cast<const float4*>(kf + 64 + c + 4);
      sc[0] = make_float2(s0.x, s0.y), sc[1] = make_float2(s0.z, s0.w), sc[2] = make_float2(s1.x, s1.y), sc[3] = make_float2(s1.z, s1.w);
      zr[0] = make_float2(z0.x, z0.y), zr[1] = make_float2(z0.z, z0.w), zr[2] = make_float2(z1.x, z1.y), zr[3] = make_float2(z1.z, z1.w);
    } else {  // values: per token (float16 at 2,304 and 2,336)
      const float s1 = __half2float(reinterpret_cast<const __half*>(stage + 2304)[t]);
      const float z1 = __half2float(reinterpret_cast<const __half*>(stage + 2336)[t]);
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[i] = make_float2(s1, s1), zr[i] = make_float2(z1, z1);
    }
    uint32_t out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 v = __ffma2_rn(q[i], sc[i], zr[i]);
      const __nv_bfloat162 pr = __floats2bfloat162_rn(v.x, v.y);
      out[i] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    dst[e8] = make_uint4(out[0], out[1], out[2], out[3]);
  }
  __syncwarp();  // the stage is read before the next record lands in it
}

}  // namespace lkv
