// K3: Quest bound scoring and device-side top-k (lazykv/selection.py:38-62, lazykv/tiered.py:383-387).
//
// Scoring: one thread per (KV head, candidate block). The bound is max over the head's query group
// of q+ . kmax + q- . kmin (selection.py:49-53), no 1/sqrt(d). Each dot product is accumulated left
// to right over the channels with one rounded float32 product and one rounded float32 add per
// channel (no fused multiply-add); in bf16 mode each dot product is rounded to bf16 and their sum
// rounded to bf16 again, as the reference's two bf16 matmuls and bf16 add are. The result is a
// 64-bit key (orderable bound << 32 | ~candidate) so that descending key order is descending bound
// with ties broken by ascending block id, the canonical order the tests hold the kernel to.
//
// Selection: one CTA per KV head. An 8-pass MSB-first radix select over the keys (in the
// workspace, L2-resident) finds the k-th largest key exactly (keys are unique); the keys at or
// above it are compacted into shared memory, bitonic-sorted descending and written out as block
// ids. The optional bitmap marks the selected block ids for the exact pass's complement.
#include <cooperative_groups.h>

#include <mutex>

#include "common.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace lkv {
namespace {

constexpr int kSelectThreads = 1024;
constexpr int kMaxK = 16384;             // shared-memory sort capacity (128 KiB of keys)
constexpr int kScoreTileBytes = 16384;   // one metadata array's tile per CTA

// Rows (candidates) per scoring CTA: a 16 KiB tile of each of kmin and kmax, at most 256 rows.
inline int score_rows(int d, size_t es) {
  const int r = kScoreTileBytes / (int)(d * es);
  return r < 256 ? r : 256;
}

// One thread per candidate row of a tile. The CTA first copies the tile's kmin and kmax rows
// (contiguous in memory) into shared memory with coalesced 16-byte loads, storing 16-byte chunk c
// of row t at chunk position (c + t % 8) mod chunks (a rotation within the row, so rows of fewer
// than 8 chunks stay in place): a quarter-warp reading chunk c of 8 consecutive rows then
// touches 8 distinct bank groups, while each thread still walks its row's channels in order.
// Position of 16-byte chunk c of tile row t (row_bytes = chunks * 16): a rotation by t when the
// chunk count is a power of two (shift and mask), else by t % 8.
__device__ __forceinline__ int tile_pos(int t, int c, int chunks, int row_bytes) {
  if ((chunks & (chunks - 1)) == 0) return t * row_bytes + (((c + t) & (chunks - 1)) << 4);
  int cc = c + (t & 7) % chunks;
  if (cc >= chunks) cc -= chunks;
  return t * row_bytes + cc * 16;
}

// Row and chunk of the u-th 16-byte chunk of a tile.
__device__ __forceinline__ void tile_rc(int u, int chunks, int& t, int& c) {
  if ((chunks & (chunks - 1)) == 0) {
    const int sh = __ffs(chunks) - 1;
    t = u >> sh;
    c = u & (chunks - 1);
  } else {
    t = u / chunks;
    c = u % chunks;
  }
}

// Query staging for the scoring kernels: q+ and q- transposed to [channel][row] with the rows
// padded to an even count GP, so one channel's rows are adjacent and pair up in float32x2 ops.
template <int G>
constexpr int qpad() { return G < 2 ? 2 : G; }

template <typename TQ, int G>
__device__ __forceinline__ void stage_query(const TQ* q, int j, int d, float* qs) {
  constexpr int GP = qpad<G>();
  for (int e = threadIdx.x; e < GP * d; e += blockDim.x) {
    const int c = e / GP, r = e % GP;
    const float v = r < G ? to_f32<TQ>(q[(int64_t)j * G * d + (int64_t)r * d + c]) : 0.0f;
    const float vp = fmaxf(v, 0.0f);   // q.clamp_min(0)
    qs[e] = vp;
    qs[GP * d + e] = __fsub_rn(v, vp);  // q - qp
  }
}

// The bound of tile row t, in the channel order and with the roundings of the header comment.
// When the query and the metadata are both bf16 every product is exact in float32 (8 x 8 significant
// bits), so a fused multiply-add rounds exactly as the separate product and add do, and the rows
// pair up in float32x2 FMAs. Otherwise products round, and separate scalar multiplies and adds are
// used (a float32x2 multiply followed by a float32x2 add was measured to give fused results on this
// toolchain, which that order rules out).
template <typename TQ, typename TM, int G>
__device__ __forceinline__ float row_bound(const unsigned char* tile_max, const unsigned char* tile_min, int t, int d, const float* qs,
                                           int bound_mode) {
  constexpr int GP = qpad<G>();
  if constexpr (sizeof(TQ) == 2 && sizeof(TM) == 2) {
    constexpr int NP = GP / 2;
    const int chunks = d / 8;
    float2 a[NP], b[NP];
#pragma unroll
    for (int r = 0; r < NP; ++r) a[r] = b[r] = make_float2(0.0f, 0.0f);
    const float2* qp = reinterpret_cast<const float2*>(qs);
    const float2* qn = reinterpret_cast<const float2*>(qs + GP * d);
    for (int c = 0; c < chunks; ++c) {
      const int pos = tile_pos(t, c, chunks, d * 2);
      const uint4 x = *reinterpret_cast<const uint4*>(tile_max + pos), y = *reinterpret_cast<const uint4*>(tile_min + pos);
      const uint32_t wx[4] = {x.x, x.y, x.z, x.w}, wy[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float mx = __uint_as_float((i & 1) ? (wx[i / 2] & 0xffff0000u) : (wx[i / 2] << 16));
        const float mn = __uint_as_float((i & 1) ? (wy[i / 2] & 0xffff0000u) : (wy[i / 2] << 16));
        const float2 x2 = make_float2(mx, mx), n2 = make_float2(mn, mn);
#pragma unroll
        for (int r = 0; r < NP; ++r) {
          a[r] = __ffma2_rn(qp[(c * 8 + i) * NP + r], x2, a[r]);
          b[r] = __ffma2_rn(qn[(c * 8 + i) * NP + r], n2, b[r]);
        }
      }
    }
    float best = -INFINITY;
#pragma unroll
    for (int r = 0; r < G; ++r) {
      const float ar = (r & 1) ? a[r / 2].y : a[r / 2].x, br = (r & 1) ? b[r / 2].y : b[r / 2].x;
      const float sc = bound_mode == LKV_BF16 ? bf16_round(__fadd_rn(bf16_round(ar), bf16_round(br))) : __fadd_rn(ar, br);
      best = fmaxf(best, sc);
    }
    return best;
  }
  const int row_bytes = d * (int)sizeof(TM);
  const int chunks = row_bytes / 16;
  float a[G], b[G];
#pragma unroll
  for (int r = 0; r < G; ++r) a[r] = b[r] = 0.0f;
  constexpr int PER = 16 / (int)sizeof(TM);
  const float* qp = qs;
  const float* qn = qs + GP * d;
  for (int c = 0; c < chunks; ++c) {
    const int pos = tile_pos(t, c, chunks, row_bytes);
    float mx[8], mn[8];
    if constexpr (PER == 8) {
      const uint4 x = *reinterpret_cast<const uint4*>(tile_max + pos), y = *reinterpret_cast<const uint4*>(tile_min + pos);
      const uint32_t wx[4] = {x.x, x.y, x.z, x.w}, wy[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        mx[2 * i] = __uint_as_float(wx[i] << 16);
        mx[2 * i + 1] = __uint_as_float(wx[i] & 0xffff0000u);
        mn[2 * i] = __uint_as_float(wy[i] << 16);
        mn[2 * i + 1] = __uint_as_float(wy[i] & 0xffff0000u);
      }
    } else {
      const float4 x = *reinterpret_cast<const float4*>(tile_max + pos), y = *reinterpret_cast<const float4*>(tile_min + pos);
      mx[0] = x.x; mx[1] = x.y; mx[2] = x.z; mx[3] = x.w;
      mn[0] = y.x; mn[1] = y.y; mn[2] = y.z; mn[3] = y.w;
    }
    const int c0 = c * PER;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
#pragma unroll
      for (int r = 0; r < G; ++r) {
        a[r] = __fadd_rn(a[r], __fmul_rn(qp[(c0 + i) * GP + r], mx[i]));
        b[r] = __fadd_rn(b[r], __fmul_rn(qn[(c0 + i) * GP + r], mn[i]));
      }
    }
  }
  float best = -INFINITY;
#pragma unroll
  for (int r = 0; r < G; ++r) {
    const float sc = bound_mode == LKV_BF16 ? bf16_round(__fadd_rn(bf16_round(a[r]), bf16_round(b[r]))) : __fadd_rn(a[r], b[r]);
    best = fmaxf(best, sc);
  }
  return best;
}

// hist0 (optional, [h][256], zero on entry): per KV head, the count of keys by the top 8 bits of the
// orderable bound, i.e. the first radix pass of the select, accumulated with one global atomic per
// non-empty bin and CTA. keys (optional) [h][n_cand]; the bounds (optional) go to out_bound (float32)
// or out_bound16 (bf16, bf16 bound mode only) with row stride bound_ld.
template <typename TQ, typename TM, int G>
__global__ void quest_score_kernel(const TQ* __restrict__ q, int d, const TM* __restrict__ kmin, const TM* __restrict__ kmax,
                                   int64_t m_head, int first_block, int n_cand, int bound_mode, uint64_t* __restrict__ keys,
                                   float* __restrict__ out_bound, uint32_t* __restrict__ hist0, __nv_bfloat16* __restrict__ out_bound16,
                                   int64_t bound_ld) {
  __shared__ uint32_t sh_hist[256];
  extern __shared__ __align__(16) float qs[];  // q+ [d][GP], q- [d][GP], then the two tiles
  const int rows = blockDim.x;
  const int row_bytes = d * (int)sizeof(TM);
  const int chunks = row_bytes / 16;
  unsigned char* tile_max = reinterpret_cast<unsigned char*>(qs + 2 * qpad<G>() * d);
  unsigned char* tile_min = tile_max + (size_t)rows * row_bytes;
  const int j = blockIdx.y;
  const int c_first = blockIdx.x * rows;
  const int n_rows = min(rows, n_cand - c_first);
  pdl_wait();  // the query, the metadata and the workspace are the predecessor's to finish with
  pdl_release();
  stage_query<TQ, G>(q, j, d, qs);
  const unsigned char* gmax = reinterpret_cast<const unsigned char*>(kmax + (int64_t)j * m_head + (int64_t)(first_block + c_first) * d);
  const unsigned char* gmin = reinterpret_cast<const unsigned char*>(kmin + (int64_t)j * m_head + (int64_t)(first_block + c_first) * d);
  for (int u = threadIdx.x; u < n_rows * chunks; u += blockDim.x) {
    int t, c;
    tile_rc(u, chunks, t, c);
    const int pos = tile_pos(t, c, chunks, row_bytes);
    cp_async16(tile_max + pos, reinterpret_cast<const uint4*>(gmax) + u);
    cp_async16(tile_min + pos, reinterpret_cast<const uint4*>(gmin) + u);
  }
  for (int b = threadIdx.x; b < 256; b += blockDim.x) sh_hist[b] = 0;
  cp_async_wait_all();
  __syncthreads();
  const int t = threadIdx.x;
  uint32_t digit = 256u;
  if (t < n_rows) {
    const float best = row_bound<TQ, TM, G>(tile_max, tile_min, t, d, qs, bound_mode);
    const int ci = c_first + t;
    const uint32_t ob = orderable(best);
    if (keys != nullptr) keys[(int64_t)j * n_cand + ci] = ((uint64_t)ob << 32) | (uint64_t)(0xffffffffu - (uint32_t)ci);
    const float nb = best == 0.0f ? 0.0f : best;
    if (out_bound != nullptr) out_bound[(int64_t)j * bound_ld + ci] = nb;
    if (out_bound16 != nullptr) out_bound16[(int64_t)j * bound_ld + ci] = __float2bfloat16_rn(nb);  // exact: a bf16-rounded bound
    digit = ob >> 24;
  }
  if (hist0 == nullptr) return;
  const uint32_t peers = __match_any_sync(0xffffffffu, digit);
  if (digit < 256u && (t & 31) == __ffs(peers) - 1) atomicAdd(&sh_hist[digit], __popc(peers));
  __syncthreads();
  for (int b = threadIdx.x; b < 256; b += blockDim.x)
    if (sh_hist[b]) atomicAdd(&hist0[(int64_t)j * 256 + b], sh_hist[b]);
}

// Finds the digit (8 bits at `shift` of the 32-bit bound) holding the `remaining`-th largest among
// the keys counted in `hist`; warp 0 scans the 256 bins from the top.
__device__ void pick_digit(const uint32_t* hist, uint32_t* sh_digit, uint32_t* sh_remaining, uint32_t* sh_bincount) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    uint32_t cnt[8];
    uint32_t sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      cnt[i] = hist[255 - 8 * lane - i];
      sum += cnt[i];
    }
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const uint32_t excl = incl - sum;
    const uint32_t rem = *sh_remaining;
    if (excl < rem && incl >= rem) {
      uint32_t acc = excl;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (acc + cnt[i] >= rem) {
          *sh_digit = 255 - 8 * lane - i;
          *sh_bincount = cnt[i];
          *sh_remaining = rem - acc;
          break;
        }
        acc += cnt[i];
      }
    }
  }
}

// Exclusive block-wide scan of one value per thread (1024 threads); returns the prefix and writes
// the total to *total.
__device__ uint32_t block_scan(uint32_t v, uint32_t* warp_sums, uint32_t* total) {
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
    const uint32_t w = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0u;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += x;
    }
    warp_sums[lane] = wi - w;
    if (lane == 31) *total = wi;
  }
  __syncthreads();
  const uint32_t r = warp_sums[warp] + incl - v;
  __syncthreads();
  return r;
}

// One CTA per KV head. Keys (orderable bound << 32 | ~candidate) are staged in shared memory when
// they fit. An MSB-first radix select over the 32-bit bound (4 passes; 2 for bf16 bounds, whose low
// 16 bits carry no order) finds the k-th largest bound T and
// how many keys at T are needed; those are the lowest candidate ids at T (the tie rule), picked by a
// block-wide scan in candidate order. The k selected keys, in ascending candidate order after the
// scan, are written out as block ids either in that order (by_block) or bitonic-sorted descending
// (descending bound, ascending id: the order of top_blocks); the bitmap marks them.
__global__ void __launch_bounds__(kSelectThreads) topk_kernel(const uint64_t* __restrict__ keys_all, int n_cand, int k, int first_block,
                                                             int32_t* __restrict__ out_blocks, int out_ld, uint32_t* __restrict__ bitmap,
                                                             int bitmap_words, int stage_keys, int by_block, int n_passes) {
  extern __shared__ uint64_t smem64[];  // sel [P], then (when staged) keys [n_cand]
  __shared__ uint32_t hist[256];
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t sh_digit, sh_remaining, sh_bincount, sh_total;
  const int j = blockIdx.x;
  int P = 1;
  const int kk = k < n_cand ? k : n_cand;
  while (P < kk) P <<= 1;
  uint64_t* sel = smem64;
  const uint64_t* keys = keys_all + (int64_t)j * n_cand;
  if (stage_keys) {
    uint64_t* ks = smem64 + (P < 2 ? 2 : P);  // 16-byte aligned
    if ((reinterpret_cast<uintptr_t>(keys) & 15) == 0) {
      // 16-byte async copies for the even-sized body, a plain load for an odd last key.
      const int pairs = n_cand / 2;
      for (int i = threadIdx.x; i < pairs; i += blockDim.x) cp_async16(ks + 2 * i, keys + 2 * i);
      if ((n_cand & 1) && threadIdx.x == 0) ks[n_cand - 1] = keys[n_cand - 1];
      cp_async_wait_all();
    } else {
      for (int i = threadIdx.x; i < n_cand; i += blockDim.x) ks[i] = keys[i];
    }
    keys = ks;
  }
  if (bitmap != nullptr)
    for (int w = threadIdx.x; w < bitmap_words; w += blockDim.x) bitmap[(int64_t)j * bitmap_words + w] = 0u;
  if (threadIdx.x == 0) {
    sh_remaining = (uint32_t)kk;
    sh_bincount = 0;
  }
  __syncthreads();

  uint32_t prefix = 0, mask = 0;
  bool take_all_equal = (kk >= n_cand);
  for (int pass = 0; pass < n_passes && !take_all_equal; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    // Keys share their top bits (sign and exponent) heavily, so lanes holding the same digit add
    // their count once per warp instead of contending on one shared-memory word.
    for (int i0 = 0; i0 < n_cand; i0 += blockDim.x) {
      const int i = i0 + threadIdx.x;
      const uint32_t hi = i < n_cand ? (uint32_t)(keys[i] >> 32) : 0u;
      const bool counted = i < n_cand && (hi & mask) == prefix;
      const uint32_t digit = counted ? ((hi >> shift) & 255u) : 256u;
      const uint32_t peers = __match_any_sync(0xffffffffu, digit);
      if (counted && (threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
    }
    __syncthreads();
    pick_digit(hist, &sh_digit, &sh_remaining, &sh_bincount);
    __syncthreads();
    prefix |= sh_digit << shift;
    mask |= 255u << shift;
    take_all_equal = (sh_bincount == sh_remaining);
    __syncthreads();
  }
  const uint32_t need_equal = take_all_equal ? 0xffffffffu : sh_remaining;

  // Compaction in candidate order: thread t owns the contiguous range [t*seg, (t+1)*seg).
  const int seg = (n_cand + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * seg, hi_end = min(n_cand, lo + seg);
  uint32_t n_gt = 0, n_eq = 0;
  for (int i = lo; i < hi_end; ++i) {
    const uint32_t h = (uint32_t)(keys[i] >> 32) & mask;
    n_gt += (kk >= n_cand) || h > prefix;
    n_eq += (kk < n_cand) && h == prefix;
  }
  const uint32_t eq_before = block_scan(n_eq, warp_sums, &sh_total);
  // Equal keys taken by this thread: those whose rank among equals is below need_equal.
  uint32_t take_eq = 0;
  if (eq_before < need_equal) take_eq = min(n_eq, need_equal - eq_before);
  const uint32_t pos0 = block_scan(n_gt + take_eq, warp_sums, &sh_total);
  uint32_t pos = pos0, eq_seen = 0;
  for (int i = lo; i < hi_end; ++i) {
    const uint64_t key = keys[i];
    const uint32_t h = (uint32_t)(key >> 32) & mask;
    bool take = (kk >= n_cand) || h > prefix;
    if (!take && h == prefix) take = eq_seen++ < take_eq;
    if (take && pos < (uint32_t)P) sel[pos++] = key;
  }
  __syncthreads();
  for (int i = kk + threadIdx.x; i < P; i += blockDim.x) sel[i] = 0ull;
  __syncthreads();
  // Bitonic sort, descending (skipped for ascending block-id order: the scan wrote that order).
  for (int size = 2; size <= (by_block ? 1 : P); size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < P / 2; i += blockDim.x) {
        const int lo2 = 2 * i - (i & (stride - 1));
        const int hi2 = lo2 + stride;
        const bool desc = (lo2 & size) == 0;
        const uint64_t a = sel[lo2], b = sel[hi2];
        if ((a < b) == desc) {
          sel[lo2] = b;
          sel[hi2] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < kk; i += blockDim.x) {
    const uint32_t ci = 0xffffffffu - (uint32_t)(sel[i] & 0xffffffffull);
    const int blk = first_block + (int)ci;
    out_blocks[(int64_t)j * out_ld + i] = blk;
    if (bitmap != nullptr && blk / 32 < bitmap_words) atomicOr(&bitmap[(int64_t)j * bitmap_words + blk / 32], 1u << (blk % 32));
  }
}

// ---- the cluster-wide select of the k smallest... largest keys, ascending block-id output ----------
//
// After the score kernel (keys in the workspace, L2-resident, and the first radix pass's histogram
// per head), one thread-block cluster of C CTAs per KV head finishes the selection: CTA c stages a
// contiguous slice of the keys in shared memory; every CTA reads the first pass's totals and picks
// the same digit; each further pass counts its slice, a cluster barrier, and every CTA sums the C
// histograms through distributed shared memory and picks the same digit. Compaction: one
// block-wide scan of packed (above, equal) counts per CTA, the CTAs' totals exchanged the same way;
// the exclusive sums over lower ranks give each CTA its output offset and its share of the tied keys
// (lowest ids first), so the selected ids come out in ascending block-id order with no sort. Every
// CTA reaches every cluster barrier (no early exit).

// The resident split (lkv_quest_topk_resident): for each chosen block, its slot before this step's
// admit (block_slot [h, bs_ld], 1.. or -1) goes to hot [h, hot_ld] at the block's position, -1 for a
// block not resident, and the bitmap marks only the resident ones, so that an exact pass over the
// bitmap's complement covers the misses and the admit can run after, or beside, the attention.
struct ResidentOut {
  const int32_t* block_slot;  // null: the plain selection
  int64_t bs_ld;
  int32_t* hot;
  int64_t hot_ld;
};

constexpr int kClusterThreads = 256;
constexpr int kClusterMax = 16;
constexpr int kClusterMaxPer = 4096;   // keys per CTA (in shared memory)
constexpr int kHistHeads = 64;         // heads the first-pass histograms are kept for
constexpr size_t kHistBytes = (size_t)kHistHeads * 256 * sizeof(uint32_t);  // at the workspace's start
constexpr size_t kFailOffset = kHistBytes;       // per-head failure words of the TMA-scored selection
constexpr size_t kKeysOffset = kHistBytes + 256;  // then the keys (64-bit, or 32-bit in the TMA-scored selection)

__global__ void __launch_bounds__(kClusterThreads) topk_cluster_kernel(const uint64_t* __restrict__ keys_all, uint32_t* __restrict__ hist0,
                                                                     int n_cand, int k, int first_block, int n_passes, int per,
                                                                     int32_t* __restrict__ out_blocks, int out_ld, uint32_t* __restrict__ bitmap,
                                                                     int bitmap_words, const ResidentOut res) {
  cg::cluster_group cluster = cg::this_cluster();
  const int c = (int)cluster.block_rank();
  const int C = (int)cluster.num_blocks();
  const int j = blockIdx.y;
  const int tid = threadIdx.x;
  extern __shared__ __align__(16) uint64_t keys[];  // [per]
  __shared__ uint32_t hist[3][256];   // this rank's counts of passes 1..3
  __shared__ uint32_t ghist[256];     // totals of the current pass
  __shared__ uint32_t counts[2];      // this rank's (above, equal) totals
  __shared__ uint32_t lower[kClusterMax][2];
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t sh_digit, sh_remaining, sh_bincount, sh_total, sh_pos0, sh_eq0;

  const int lo = min(n_cand, c * per);
  const int hi = min(n_cand, lo + per);
  const int cnt = hi - lo;
  const uint64_t* src = keys_all + (int64_t)j * n_cand + lo;
  pdl_wait();  // the keys and first-pass counts of the score kernel
  pdl_release();
  for (int i = tid; i < cnt; i += blockDim.x) keys[i] = src[i];
  if (c == 0 && bitmap != nullptr)
    for (int w = tid; w < bitmap_words; w += blockDim.x) bitmap[(int64_t)j * bitmap_words + w] = 0u;
  for (int b = tid; b < 256; b += blockDim.x) ghist[b] = hist0[(int64_t)j * 256 + b];
  const int kk = k < n_cand ? k : n_cand;
  if (tid == 0) {
    sh_remaining = (uint32_t)kk;
    sh_bincount = 0;
  }
  __syncthreads();
  uint32_t prefix = 0, mask = 0;
  bool take_all = kk >= n_cand;
  for (int pass = 0; pass < n_passes && !take_all; ++pass) {
    const int shift = 24 - 8 * pass;
    if (pass > 0) {
      uint32_t* hp = hist[pass - 1];
      for (int b = tid; b < 256; b += blockDim.x) hp[b] = 0;
      __syncthreads();
      for (int i0 = 0; i0 < cnt; i0 += blockDim.x) {
        const int i = i0 + tid;
        const uint32_t h32 = i < cnt ? (uint32_t)(keys[i] >> 32) : 0u;
        const bool counted = i < cnt && (h32 & mask) == prefix;
        const uint32_t digit = counted ? ((h32 >> shift) & 255u) : 256u;
        const uint32_t peers = __match_any_sync(0xffffffffu, digit);
        if (counted && (tid & 31) == __ffs(peers) - 1) atomicAdd(&hp[digit], __popc(peers));
      }
      cluster.sync();  // every rank's counts of this pass are final
      for (int b = tid; b < 256; b += blockDim.x) {
        uint32_t v[kClusterMax];
#pragma unroll
        for (int r = 0; r < kClusterMax; ++r) v[r] = r < C ? *cluster.map_shared_rank(&hp[b], r) : 0u;  // all in flight at once
        uint32_t sum = 0;
#pragma unroll
        for (int r = 0; r < kClusterMax; ++r) sum += v[r];
        ghist[b] = sum;
      }
      __syncthreads();
    }
    pick_digit(ghist, &sh_digit, &sh_remaining, &sh_bincount);
    __syncthreads();
    prefix |= sh_digit << shift;
    mask |= 255u << shift;
    take_all = (sh_bincount == sh_remaining);
    __syncthreads();
  }
  const uint32_t need = take_all ? 0xffffffffu : sh_remaining;
  const bool all = kk >= n_cand;

  // ---- compaction in candidate order across the cluster ----
  const int seg = (cnt + blockDim.x - 1) / blockDim.x;
  const int tlo = min(cnt, tid * seg), thi = min(cnt, tlo + seg);
  uint32_t n_gt = 0, n_eq = 0;
  for (int i = tlo; i < thi; ++i) {
    const uint32_t h32 = (uint32_t)(keys[i] >> 32) & mask;
    n_gt += all || h32 > prefix;
    n_eq += !all && h32 == prefix;
  }
  const uint32_t pre = block_scan(n_gt | (n_eq << 16), warp_sums, &sh_total);  // per <= 4096: both fit 16 bits
  if (tid == 0) {
    counts[0] = sh_total & 0xffffu;
    counts[1] = sh_total >> 16;
  }
  cluster.sync();  // every rank's totals are published; every rank has read the first-pass histogram
  if (c == 0)
    for (int b = tid; b < 256; b += blockDim.x) hist0[(int64_t)j * 256 + b] = 0u;  // zero for the next call
  if (tid < c) {
    lower[tid][0] = *cluster.map_shared_rank(&counts[0], tid);
    lower[tid][1] = *cluster.map_shared_rank(&counts[1], tid);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t eqb = 0, posb = 0;
    for (int r = 0; r < c; ++r) {
      const uint32_t take = eqb < need ? min(lower[r][1], need - eqb) : 0u;
      posb += lower[r][0] + take;
      eqb += lower[r][1];
    }
    sh_pos0 = posb;
    sh_eq0 = eqb;
  }
  __syncthreads();
  const uint32_t gt_before = pre & 0xffffu, eq_before_t = pre >> 16;
  const uint32_t e0 = sh_eq0;
  const uint32_t room = e0 < need ? need - e0 : 0u;  // tied keys this rank may still take
  uint32_t pos = sh_pos0 + gt_before + min(eq_before_t, room);
  const uint32_t take_eq = eq_before_t < room ? min(n_eq, room - eq_before_t) : 0u;
  uint32_t eq_seen = 0;
  for (int i = tlo; i < thi; ++i) {
    const uint32_t h32 = (uint32_t)(keys[i] >> 32) & mask;
    bool take = all || h32 > prefix;
    if (!take && h32 == prefix) take = eq_seen++ < take_eq;
    if (take && pos < (uint32_t)kk) {
      const int blk = first_block + lo + i;
      out_blocks[(int64_t)j * out_ld + pos] = blk;
      int32_t slot = 1;
      if (res.block_slot != nullptr) {
        slot = __ldcg(res.block_slot + (int64_t)j * res.bs_ld + blk);
        res.hot[(int64_t)j * res.hot_ld + pos] = slot >= 1 ? slot : -1;
      }
      if (bitmap != nullptr && slot >= 1 && blk / 32 < bitmap_words) atomicOr(&bitmap[(int64_t)j * bitmap_words + blk / 32], 1u << (blk % 32));
      ++pos;
    }
  }
  cluster.sync();  // each rank's shared memory stays alive until every rank has read it
}

// Cluster size for n candidates: a power of two giving ~512 keys per CTA, at most 16; 0 when a
// CTA would need more than kClusterMaxPer keys.
inline int cluster_size_for(int n_cand) {
  int c = 1;
  while (c < kClusterMax && (n_cand + c - 1) / c > 512) c <<= 1;
  if ((n_cand + c - 1) / c > kClusterMaxPer) return 0;
  return c;
}

int launch_topk_cluster(int h, cudaStream_t st, const uint64_t* keys, uint32_t* hist0, int n_cand, int k, int first_block, int n_passes,
                        int32_t* out_blocks, int out_ld, uint32_t* bitmap, int bitmap_words, const ResidentOut& res) {
  static bool attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(topk_cluster_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(topk_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kClusterMaxPer * sizeof(uint64_t)));
    if (e != cudaSuccess) return fail(LKV_ERR_CUDA, "lkv_quest_topk(cluster select) attributes: %s", cudaGetErrorString(e));
    attr_set[dev & 63] = true;
  }
  const int C = cluster_size_for(n_cand);
  const int per = (n_cand + C - 1) / C;
  cudaError_t e = launch_pdl(topk_cluster_kernel, dim3(C, h), dim3(kClusterThreads), (size_t)per * sizeof(uint64_t), st, C, keys, hist0, n_cand,
                             k, first_block, n_passes, per, out_blocks, out_ld, bitmap, bitmap_words, res);
  if (e != cudaSuccess) return fail(LKV_ERR_CUDA, "lkv_quest_topk(cluster select, %d CTAs x %d heads): %s", C, h, cudaGetErrorString(e));
  return LKV_OK;
}

// ---- selection in two launches: TMA scoring, then a cluster select per head ------------------------
//
// For a bf16 query and bf16 metadata at head_dim 64, block-id order, at most 16,384 candidates per
// head and 64 heads.
//
// quest_score_tma_kernel: P x h CTAs (P = ceil(n_cand / 256)); CTA c of head j scores its 256
// candidates. Their kmax and kmin rows arrive by tensor-map TMA (boxes of 128 rows, 128-byte
// swizzle: chunk x of row r at chunk x ^ (r & 7)), and thread t scores row t as quest_score_kernel
// does (same channel order and roundings). The orderable 32-bit bound goes to the head's keys in the
// workspace and its top 8 bits to the head's first-pass histogram (one global atomic per non-empty
// bin and CTA).
//
// quest_pick_kernel, launched right behind it (programmatic dependent launch: its CTAs are placed
// while the scoring runs and wait for its completion): a cluster of 8 CTAs x 1024 threads per head,
// one key per thread (two above 8,192 candidates). Every CTA picks the first digit from the
// histogram; each further radix pass counts the CTA's keys in shared memory, a cluster barrier
// completes the pass and every CTA sums the cluster's histograms through distributed shared memory.
// The compaction exchanges each CTA's (above, tied) totals the same way: a CTA's output offset and
// its share of the tied keys (lowest ids first) come from the totals of the CTAs before it, so the
// ids come out in ascending block-id order; each warp ORs its 32 candidates' bits into the bitmap.
// Rank 0 returns the histogram and the head's failure word to zero for the next call.
//
// No CTA waits for a CTA outside its cluster, and a cluster's CTAs are scheduled together. The
// scoring's TMA waits are bounded: a wait that runs out records LKV_DEV_WAIT_TIMEOUT (status word
// and host mirror) and sets the head's failure word, and the select then writes the failure's
// poison for the head (every listed id -1 and an empty bitmap, so that an exact pass over the
// complement still covers every candidate). A CTA whose wait ran out waits (bounded) for its copy
// before it exits, so no bulk copy lands in the shared memory of a finished CTA.

constexpr int kScThreads = 128;                        // candidates per CTA (one thread each)
constexpr int kScBoxRows = 128;
constexpr int kScBoxes = kScThreads / kScBoxRows;       // boxes per metadata array
constexpr int kScBox = kScBoxRows * 128;               // bytes of one box: 128 rows of 64 bf16
constexpr size_t kScSmem = 1024 + 2 * kScBoxes * (size_t)kScBox;  // the kmax boxes, then the kmin boxes
constexpr int kPkThreads = 1024;
constexpr int kPkCluster = 8;
constexpr int kPkMaxKpt = 2;
constexpr int kPkMaxCand = kPkCluster * kPkThreads * kPkMaxKpt;  // 16,384
constexpr uint32_t kScExitWaitIters = 1u << 22;      // bound of the wait for a copy still in flight at exit

struct SelParams {
  CUtensorMap tmax, tmin;  // [h][rows][64] bf16, box {64, 128, 1}, 128-byte swizzle
  const __nv_bfloat16* q;
  int n_cand, k, first_block, n_passes, bound_mode;
  int32_t* out_blocks;
  int out_ld;
  uint32_t* bitmap;
  int bitmap_words;
  float* out_bound;
  uint32_t* hist0;  // [h][256] first-pass counts: zero on entry, left zero
  uint32_t* fail;   // [h] set when a scoring wait ran out: zero on entry, left zero
  uint32_t* keys;   // [h][n_cand] orderable bounds
  uint32_t wait_iters;  // bound of each TMA wait (tries)
  int stall;            // test hook: 1 = wait on a barrier that nothing completes before scoring
  ResidentOut res;      // the resident split (null block_slot: off)
};

// One 3-D tile load global -> this CTA's shared memory under an L2 cache policy. No multicast.
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar, uint64_t pol) {
  asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(pol)
               : "memory");
}

// row_bound's bf16 x bf16 arithmetic on a swizzled box row (d = 64: 8 chunks of 16 bytes).
template <int G>
__device__ __forceinline__ float row_bound_swz(const unsigned char* bmax, const unsigned char* bmin, int r, const float* qs, int bound_mode) {
  constexpr int GP = qpad<G>();
  constexpr int NP = GP / 2;
  float2 a[NP], b[NP];
#pragma unroll
  for (int x = 0; x < NP; ++x) a[x] = b[x] = make_float2(0.0f, 0.0f);
  const float2* qp = reinterpret_cast<const float2*>(qs);
  const float2* qn = reinterpret_cast<const float2*>(qs + GP * 64);
#pragma unroll 2
  for (int c = 0; c < 8; ++c) {
    const int pos = r * 128 + ((c ^ (r & 7)) << 4);
    const uint4 x = *reinterpret_cast<const uint4*>(bmax + pos), y = *reinterpret_cast<const uint4*>(bmin + pos);
    const uint32_t wx[4] = {x.x, x.y, x.z, x.w}, wy[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float mx = __uint_as_float((i & 1) ? (wx[i / 2] & 0xffff0000u) : (wx[i / 2] << 16));
      const float mn = __uint_as_float((i & 1) ? (wy[i / 2] & 0xffff0000u) : (wy[i / 2] << 16));
      const float2 x2 = make_float2(mx, mx), n2 = make_float2(mn, mn);
      if constexpr (NP % 2 == 0) {  // the rows' q+ and q- of one channel in 16-byte loads
#pragma unroll
        for (int w = 0; w < NP; w += 2) {
          const float4 p4 = reinterpret_cast<const float4*>(qp)[((c * 8 + i) * NP + w) / 2];
          const float4 n4 = reinterpret_cast<const float4*>(qn)[((c * 8 + i) * NP + w) / 2];
          a[w] = __ffma2_rn(make_float2(p4.x, p4.y), x2, a[w]);
          a[w + 1] = __ffma2_rn(make_float2(p4.z, p4.w), x2, a[w + 1]);
          b[w] = __ffma2_rn(make_float2(n4.x, n4.y), n2, b[w]);
          b[w + 1] = __ffma2_rn(make_float2(n4.z, n4.w), n2, b[w + 1]);
        }
      } else {
#pragma unroll
        for (int w = 0; w < NP; ++w) {
          a[w] = __ffma2_rn(qp[(c * 8 + i) * NP + w], x2, a[w]);
          b[w] = __ffma2_rn(qn[(c * 8 + i) * NP + w], n2, b[w]);
        }
      }
    }
  }
  float best = -INFINITY;
#pragma unroll
  for (int w = 0; w < G; ++w) {
    const float ar = (w & 1) ? a[w / 2].y : a[w / 2].x, br = (w & 1) ? b[w / 2].y : b[w / 2].x;
    const float sc = bound_mode == LKV_BF16 ? bf16_round(__fadd_rn(bf16_round(ar), bf16_round(br))) : __fadd_rn(ar, br);
    best = fmaxf(best, sc);
  }
  return best;
}

template <int G>
__global__ void __launch_bounds__(kScThreads) quest_score_tma_kernel(const __grid_constant__ SelParams sp) {
  const int j = blockIdx.y, c = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  extern __shared__ unsigned char sc_raw[];
  unsigned char* tiles = sc_raw + ((1024 - (smem_u32(sc_raw) & 1023)) & 1023);
  __shared__ __align__(16) float qs[2 * qpad<G>() * 64];
  __shared__ __align__(8) uint64_t bar[2];  // [0] the tiles; [1] the test hook's (never completed)
  __shared__ uint32_t hist[256];

  const int n_cand = sp.n_cand;
  const int lo = c * kScThreads;
  const int cnt = min(kScThreads, n_cand - lo);
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // the query, the metadata and the workspace are the predecessor's to finish with
  pdl_release();  // the select's CTAs may be placed now (they wait for this grid's completion)
  if (tid == 0) {  // the bounds first: the query is staged while they are in flight
    const int r0 = sp.first_block + lo;
    const uint64_t pol = l2_evict_first_policy();  // the bounds are read once per call
    mbar_arrive_expect_tx(&bar[0], (uint32_t)(2 * kScBoxes * kScBox));
#pragma unroll
    for (int bx = 0; bx < kScBoxes; ++bx) {
      tma_load_3d_hint(tiles + bx * kScBox, &sp.tmax, 0, r0 + bx * kScBoxRows, j, &bar[0], pol);
      tma_load_3d_hint(tiles + (kScBoxes + bx) * kScBox, &sp.tmin, 0, r0 + bx * kScBoxRows, j, &bar[0], pol);
    }
  }
  stage_query<__nv_bfloat16, G>(sp.q, j, 64, qs);
  for (int b = tid; b < 256; b += kScThreads) hist[b] = 0u;
  uint32_t got = 1u;
  if (sp.stall && tid == 0) got = mbar_wait_n(&bar[1], 0, sp.wait_iters) ? 1u : 0u;  // test hook: runs out
  if (got) got = mbar_wait_n(&bar[0], 0, sp.wait_iters) ? 1u : 0u;
  const bool ok = __syncthreads_and((int)got) != 0;  // also the barrier of the staged query and the histogram

  uint32_t key = 0u;
  if (tid < cnt) {
    if (ok) {
      const int bx = tid / kScBoxRows, r = tid % kScBoxRows;
      const float best = row_bound_swz<G>(tiles + bx * kScBox, tiles + (kScBoxes + bx) * kScBox, r, qs, sp.bound_mode);
      key = orderable(best);
      if (sp.out_bound != nullptr) sp.out_bound[(int64_t)j * n_cand + lo + tid] = best == 0.0f ? 0.0f : best;
    }
    sp.keys[(int64_t)j * n_cand + lo + tid] = key;
  }
  const uint32_t digit = tid < cnt ? key >> 24 : 256u;
  const uint32_t peers = __match_any_sync(0xffffffffu, digit);
  if (digit < 256u && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
  __syncthreads();
  for (int b = tid; b < 256; b += kScThreads)
    if (hist[b] != 0u) atomicAdd(&sp.hist0[(int64_t)j * 256 + b], hist[b]);
  if (tid == 0 && !ok) {
    atomicOr(&sp.fail[j], 1u);
    mbar_wait_n(&bar[0], 0, kScExitWaitIters);  // the copy may still be landing: no exit before it does
  }
}

// The cluster barrier that only keeps shared memory alive: arrive without release semantics (no
// data is published by it), so it does not wait for this CTA's global stores to complete.
__device__ __forceinline__ void cluster_sync_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\nbarrier.cluster.wait.aligned;" ::: "memory");
}

// CTA c of the head's cluster owns whole bitmap words: words [w_c, w_{c+1}) of the words the
// candidates span, 32 x KPT per CTA at most. Thread t holds block 32 * w_c + t (+ 1024 per further
// key), a candidate when it lies in [first_block, first_block + n_cand); so a warp's 32 blocks are
// exactly one bitmap word, which its lane 0 stores whole (no zeroing pass, no atomics), and the
// CTAs' candidates follow one another in block order.
template <int KPT>
__global__ void __launch_bounds__(kPkThreads) quest_pick_kernel(const __grid_constant__ SelParams sp) {
  cg::cluster_group cluster = cg::this_cluster();
  const int c = (int)cluster.block_rank(), C = (int)cluster.num_blocks();
  const int j = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
  __shared__ uint32_t hist[2][256];  // this CTA's counts of the current pass (alternating buffers)
  __shared__ uint32_t ghist[256];    // the cluster's totals (the first pass: the scoring's histogram)
  __shared__ uint32_t counts[2];     // this CTA's (above, tied) totals
  __shared__ uint32_t lower[kPkCluster][2];
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t sh_digit, sh_remaining, sh_bincount, sh_total, sh_pos0, sh_eq0;

  const int n_cand = sp.n_cand, first = sp.first_block;
  const int wf = first / 32, wl = (first + n_cand - 1) / 32;  // the words the candidates span
  const int nw = wl - wf + 1;
  const int w_lo = wf + (int)((int64_t)nw * c / C), w_hi = wf + (int)((int64_t)nw * (c + 1) / C);
  const int W = sp.bitmap_words;
  pdl_wait();  // the keys, the histogram and the failure word of the scoring
  pdl_release();  // the next kernel's CTAs may be placed now (they wait for this grid's completion)
  const bool failed = __ldcg(&sp.fail[j]) != 0u;
  uint32_t keys[KPT];
  bool have[KPT];
#pragma unroll
  for (int kp = 0; kp < KPT; ++kp) {
    const int b = 32 * w_lo + kp * kPkThreads + tid;  // block id
    have[kp] = b < 32 * w_hi && b >= first && b < first + n_cand;
    keys[kp] = have[kp] ? __ldcg(sp.keys + (int64_t)j * n_cand + (b - first)) : 0u;
  }
  if (tid < 256) ghist[tid] = __ldcg(&sp.hist0[(int64_t)j * 256 + tid]);
  const int kk = sp.k < n_cand ? sp.k : n_cand;
  if (tid == 0) {
    sh_remaining = (uint32_t)kk;
    sh_bincount = 0u;
  }
  __syncthreads();
  uint32_t prefix = 0u, mask = 0u;
  const bool all = kk >= n_cand;
  bool take_all = all;
  for (int pass = 0; pass < sp.n_passes && !take_all; ++pass) {  // the same digits in every CTA of the cluster
    const int shift = 24 - 8 * pass;
    if (pass > 0) {
      uint32_t* hp = hist[pass & 1];
      if (tid < 256) hp[tid] = 0u;
      __syncthreads();
#pragma unroll
      for (int kp = 0; kp < KPT; ++kp) {
        const bool counted = have[kp] && (keys[kp] & mask) == prefix;
        const uint32_t digit = counted ? ((keys[kp] >> shift) & 255u) : 256u;
        const uint32_t peers = __match_any_sync(0xffffffffu, digit);
        if (counted && lane == __ffs(peers) - 1) atomicAdd(&hp[digit], __popc(peers));
      }
      cluster.sync();  // every CTA's counts of this pass are final
      if (tid < 256) {
        uint32_t v[kPkCluster];
#pragma unroll
        for (int r = 0; r < kPkCluster; ++r) v[r] = r < C ? *cluster.map_shared_rank(&hp[tid], r) : 0u;  // all in flight at once
        uint32_t sum = 0;
#pragma unroll
        for (int r = 0; r < kPkCluster; ++r) sum += v[r];
        ghist[tid] = sum;
      }
      __syncthreads();
    }
    pick_digit(ghist, &sh_digit, &sh_remaining, &sh_bincount);
    __syncthreads();
    prefix |= sh_digit << shift;
    mask |= 255u << shift;
    take_all = (sh_bincount == sh_remaining);  // uniform: every CTA summed the same counts
    __syncthreads();
  }
  const uint32_t need = take_all ? 0xffffffffu : sh_remaining;

  // ---- compaction in candidate order across the cluster ----
  uint32_t pre[KPT], run = 0u;
  bool gt[KPT], eq[KPT];
#pragma unroll
  for (int kp = 0; kp < KPT; ++kp) {
    const uint32_t km = keys[kp] & mask;
    gt[kp] = have[kp] && (all || km > prefix || (take_all && km == prefix));
    eq[kp] = have[kp] && !all && !take_all && km == prefix;
    pre[kp] = run + block_scan((gt[kp] ? 1u : 0u) | ((eq[kp] ? 1u : 0u) << 16), warp_sums, &sh_total);  // <= 2,048 each: 16 bits
    run += sh_total;
  }
  if (tid == 0) {
    counts[0] = run & 0xffffu;
    counts[1] = run >> 16;
  }
  cluster.sync();  // every CTA's totals are published; every CTA has read the histogram
  if (tid < C) {
    lower[tid][0] = *cluster.map_shared_rank(&counts[0], tid);
    lower[tid][1] = *cluster.map_shared_rank(&counts[1], tid);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t eqb = 0, posb = 0;
    for (int r = 0; r < c; ++r) {
      const uint32_t take = eqb < need ? min(lower[r][1], need - eqb) : 0u;
      posb += lower[r][0] + take;
      eqb += lower[r][1];
    }
    sh_pos0 = posb;
    sh_eq0 = eqb;
  }
  __syncthreads();
  // Every exchange is done: from here on only global stores, then a barrier that keeps the shared
  // memory alive for the other CTAs' reads above.
  const uint32_t room = sh_eq0 < need ? need - sh_eq0 : 0u;  // tied keys this CTA may still take
#pragma unroll
  for (int kp = 0; kp < KPT; ++kp) {
    const int b = 32 * w_lo + kp * kPkThreads + tid;
    const uint32_t gt_before = pre[kp] & 0xffffu, eq_before = pre[kp] >> 16;
    const uint32_t pos = sh_pos0 + gt_before + min(eq_before, room);
    const bool take = !failed && (gt[kp] || (eq[kp] && eq_before < room)) && pos < (uint32_t)kk;
    if (take) sp.out_blocks[(int64_t)j * sp.out_ld + pos] = b;
    bool mark = take;
    if (take && sp.res.block_slot != nullptr) {  // the resident split: the slot before this step's admit
      const int32_t slot = __ldcg(sp.res.block_slot + (int64_t)j * sp.res.bs_ld + b);
      sp.res.hot[(int64_t)j * sp.res.hot_ld + pos] = slot >= 1 ? slot : -1;
      mark = slot >= 1;
    }
    const uint32_t word = __ballot_sync(0xffffffffu, mark);  // bit l: block 32 * (b / 32) + l
    if (sp.bitmap != nullptr && lane == 0 && b < 32 * w_hi && b / 32 < W) sp.bitmap[(int64_t)j * W + b / 32] = word;
  }
  if (sp.bitmap != nullptr) {  // the words outside the candidates' span: zero (first and last CTA)
    if (c == 0)
      for (int w = tid; w < min(wf, W); w += blockDim.x) sp.bitmap[(int64_t)j * W + w] = 0u;
    if (c == C - 1)
      for (int w = wl + 1 + tid; w < W; w += blockDim.x) sp.bitmap[(int64_t)j * W + w] = 0u;
  }
  if (failed) {  // a scoring wait ran out: every listed id -1 (the bitmap words above are empty)
    const int p0 = (int)((int64_t)sp.k * c / C), p1 = (int)((int64_t)sp.k * (c + 1) / C);
    for (int p = p0 + tid; p < p1; p += blockDim.x) {
      sp.out_blocks[(int64_t)j * sp.out_ld + p] = -1;
      if (sp.res.block_slot != nullptr) sp.res.hot[(int64_t)j * sp.res.hot_ld + p] = -1;
    }
  }
  if (c == 0 && tid < 256) sp.hist0[(int64_t)j * 256 + tid] = 0u;  // zero for the next call (every CTA read it before the barrier above)
  cluster_sync_relaxed();  // no CTA leaves while another may still read its shared memory; every CTA read the failure word
  if (c == 0 && tid == 0) sp.fail[j] = 0u;
}

// Whether the TMA-scored select takes this call (bf16 query and metadata, head_dim 64, block-id
// order, G in {1, 2, 4, 8}, at most kPkMaxCand candidates and kHistHeads heads); fills its maps.
bool select_plan(int g, int q_dtype, int meta_dtype, int h, int d, const void* kmin, const void* kmax, int64_t m_head, int first_block,
                 int n_cand, int order, SelParams& sp) {
  if (q_dtype != LKV_BF16 || meta_dtype != LKV_BF16 || d != 64 || order != LKV_ORDER_BLOCK) return false;
  if (g != 1 && g != 2 && g != 4 && g != 8) return false;
  if (n_cand > kPkMaxCand || h > kHistHeads) return false;
  const int nw = (first_block + n_cand - 1) / 32 - first_block / 32 + 1;  // bitmap words the candidates span
  if ((nw + kPkCluster - 1) / kPkCluster > kPkMaxKpt * kPkThreads / 32) return false;
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[3] = {64, (cuuint64_t)first_block + (cuuint64_t)n_cand, (cuuint64_t)h};
  const cuuint64_t strides[2] = {128, (cuuint64_t)m_head * 2};
  const cuuint32_t box[3] = {64, kScBoxRows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  for (int i = 0; i < 2; ++i) {
    CUresult r = encode_tiled(i == 0 ? &sp.tmax : &sp.tmin, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(i == 0 ? kmax : kmin), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
  }
  return true;
}

// Test hooks (lkv_debug_set): the bound of the selection's TMA waits, and a one-shot stall.
uint32_t g_sel_wait_iters = kMaxWaitIters;
int g_sel_stall_next = 0;

template <int G>
cudaError_t launch_score_tma_g(const SelParams& sp, int h, cudaStream_t st) {
  static bool attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(quest_score_tma_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kScSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev & 63] = true;
  }
  const int P = (sp.n_cand + kScThreads - 1) / kScThreads;
  return launch_pdl(quest_score_tma_kernel<G>, dim3(P, h), dim3(kScThreads), kScSmem, st, 0, sp);
}

int launch_select(int g, const SelParams& sp, int h, cudaStream_t st) {
  cudaError_t e = cudaErrorInvalidValue;
  switch (g) {
    case 1: e = launch_score_tma_g<1>(sp, h, st); break;
    case 2: e = launch_score_tma_g<2>(sp, h, st); break;
    case 4: e = launch_score_tma_g<4>(sp, h, st); break;
    case 8: e = launch_score_tma_g<8>(sp, h, st); break;
    default: return fail(LKV_ERR_ARG, "lkv_quest_topk: query group %d not in {1,2,4,8}", g);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_quest_topk(score, %d heads): %s", h, cudaGetErrorString(e));
  }
  // The select: 8-CTA clusters, one per head (a portable cluster size: always schedulable); each
  // CTA takes ceil(words / 8) bitmap words, 32 blocks a word, 1,024 blocks a key per thread.
  const int nw = (sp.first_block + sp.n_cand - 1) / 32 - sp.first_block / 32 + 1;
  const int kpt = (nw + kPkCluster - 1) / kPkCluster > kPkThreads / 32 ? 2 : 1;
  e = kpt == 1 ? launch_pdl(quest_pick_kernel<1>, dim3(kPkCluster, h), dim3(kPkThreads), 0, st, kPkCluster, sp)
               : launch_pdl(quest_pick_kernel<2>, dim3(kPkCluster, h), dim3(kPkThreads), 0, st, kPkCluster, sp);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_quest_topk(select, %d heads): %s", h, cudaGetErrorString(e));
  }
  return LKV_OK;
}

// Keys of gathered candidates: (orderable bound << 32) | ~id, so the select decodes the id itself.
__global__ void merge_keys_kernel(const float* __restrict__ bounds, const int32_t* __restrict__ ids, int n, int64_t ld,
                                  uint64_t* __restrict__ keys) {
  const int j = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float b = bounds[(int64_t)j * ld + i];
    const uint32_t id = (uint32_t)ids[(int64_t)j * ld + i];
    keys[(int64_t)j * n + i] = ((uint64_t)orderable(b) << 32) | (uint64_t)(0xffffffffu - id);
  }
}

template <typename TQ, typename TM>
int launch_score(int g, int h, int d, cudaStream_t st, const void* q, const void* kmin, const void* kmax, int64_t m_head, int first_block,
                 int n_cand, int bound_mode, uint64_t* keys, float* out_bound, uint32_t* hist0, __nv_bfloat16* out_bound16 = nullptr,
                 int64_t bound_ld = -1) {
  if (bound_ld < 0) bound_ld = n_cand;
  const int rows = score_rows(d, sizeof(TM));
  dim3 grid((n_cand + rows - 1) / rows, h);
  const size_t smem = 2 * (size_t)(g < 2 ? 2 : g) * d * sizeof(float) + 2 * (size_t)rows * d * sizeof(TM);
#define LKV_SCORE(G)                                                                                                   \
  case G: {                                                                                                            \
    auto kern = quest_score_kernel<TQ, TM, G>;                                                                         \
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);          \
    cudaError_t le = launch_pdl(kern, grid, dim3(rows), smem, st, 0, static_cast<const TQ*>(q), d, static_cast<const TM*>(kmin),      \
                                static_cast<const TM*>(kmax), m_head, first_block, n_cand, bound_mode, keys, out_bound, hist0, out_bound16, bound_ld); \
    if (le != cudaSuccess) return fail(LKV_ERR_CUDA, "lkv_quest_topk(score): %s", cudaGetErrorString(le));             \
    break;                                                                                                             \
  }
  switch (g) {
    LKV_SCORE(1)
    LKV_SCORE(2)
    LKV_SCORE(4)
    LKV_SCORE(8)
    default:
      return fail(LKV_ERR_ARG, "lkv_quest_topk: query group %d not in {1,2,4,8}", g);
  }
#undef LKV_SCORE
  return LKV_OK;
}


// ---- global top-k over every shard's gathered bounds --------------------------------------------
//
// The shards of a context-sharded layer hold contiguous, ascending candidate ranges, rank after
// rank. Each rank scores its own candidates (lkv_quest_bounds) and the bounds of all ranks are
// all-gathered into [world][h][ld]; every rank then runs this kernel on the same gathered bounds, so
// all of them agree on one selection: the k highest bounds of the whole context, ties at the k-th
// bound to the lower block ids, i.e. the set lkv_quest_topk picks over the unsharded candidates.
// Each rank writes only its own part: the chosen candidates inside its range, as local ids in
// ascending order, padded with -1, and its own bitmap.
//
// One CTA of kSelectThreads threads per KV head, no shared key copy: MSB-first radix passes over the
// orderable 32-bit form of the bound (2 for bf16 bounds, 4 for float32), each a histogram of the
// keys that match the digits found so far; then the number of keys at the threshold in lower ranks
// (the ties they take first) and a block-wide scan over this rank's range in candidate order.
constexpr int kMaxWorld = 64;

struct GatherSel {
  const void* bounds;   // [world][h][ld], bf16 or float32
  int bf16;             // bounds are bf16
  int world, h;
  int64_t ld;           // row stride (elements)
  int seg_start[kMaxWorld + 1];  // prefix sums of the ranks' candidate counts
  int k, n_passes, rank;
  int out_base;         // local id of the rank's first candidate
  int32_t* out;         // [h][out_ld]
  int out_ld, out_cols; // columns written (chosen ids, then -1)
  uint32_t* bitmap;     // [h][bitmap_words] or null
  int bitmap_words;
  ResidentOut res;      // the resident split (null block_slot: off), on local ids
};

__device__ __forceinline__ uint32_t gathered_key(const GatherSel& p, int r, int j, int i) {
  const int64_t at = ((int64_t)r * p.h + j) * p.ld + i;
  if (p.bf16) {
    const uint16_t u = static_cast<const uint16_t*>(p.bounds)[at];
    return orderable(__uint_as_float((uint32_t)u << 16));
  }
  return orderable(static_cast<const float*>(p.bounds)[at]);
}

__global__ void __launch_bounds__(kSelectThreads) topk_gathered_kernel(const __grid_constant__ GatherSel p) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t sh_digit, sh_remaining, sh_bincount, sh_total, sh_eq_before;
  const int j = blockIdx.x;
  const int tid = threadIdx.x;
  const int n_total = p.seg_start[p.world];
  const int kk = p.k < n_total ? p.k : n_total;
  pdl_wait();  // the gathered bounds are the collective's to finish writing
  pdl_release();
  if (tid == 0) {
    sh_remaining = (uint32_t)kk;
    sh_bincount = 0;
    sh_eq_before = 0;
  }
  uint32_t prefix = 0, mask = 0;
  bool take_all = kk >= n_total;
  for (int pass = 0; pass < p.n_passes && !take_all; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = tid; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    for (int r = 0; r < p.world; ++r) {
      const int n_r = p.seg_start[r + 1] - p.seg_start[r];
      for (int i0 = 0; i0 < n_r; i0 += blockDim.x) {
        const int i = i0 + tid;
        const uint32_t key = i < n_r ? gathered_key(p, r, j, i) : 0u;
        const bool counted = i < n_r && (key & mask) == prefix;
        const uint32_t digit = counted ? ((key >> shift) & 255u) : 256u;
        const uint32_t peers = __match_any_sync(0xffffffffu, digit);
        if (counted && (tid & 31) == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
      }
    }
    __syncthreads();
    pick_digit(hist, &sh_digit, &sh_remaining, &sh_bincount);
    __syncthreads();
    prefix |= sh_digit << shift;
    mask |= 255u << shift;
    take_all = (sh_bincount == sh_remaining);
    __syncthreads();
  }
  const bool all = kk >= n_total;
  const uint32_t need = take_all ? 0xffffffffu : sh_remaining;  // keys at the threshold to take, lowest ids first
  // Keys at the threshold in the lower ranks: they come first.
  if (!all && !take_all) {
    uint32_t eq = 0;
    for (int r = 0; r < p.rank; ++r) {
      const int n_r = p.seg_start[r + 1] - p.seg_start[r];
      for (int i = tid; i < n_r; i += blockDim.x) eq += (gathered_key(p, r, j, i) & mask) == prefix;
    }
    eq = __reduce_add_sync(0xffffffffu, eq);
    if ((tid & 31) == 0 && eq) atomicAdd(&sh_eq_before, eq);
  }
  if (p.bitmap != nullptr)
    for (int w = tid; w < p.bitmap_words; w += blockDim.x) p.bitmap[(int64_t)j * p.bitmap_words + w] = 0u;
  __syncthreads();
  // This rank's range, in candidate order: thread t owns a contiguous piece.
  const int n_my = p.seg_start[p.rank + 1] - p.seg_start[p.rank];
  const int seg = (n_my + blockDim.x - 1) / blockDim.x;
  const int tlo = min(n_my, tid * seg), thi = min(n_my, tlo + seg);
  uint32_t n_gt = 0, n_eq = 0;
  for (int i = tlo; i < thi; ++i) {
    const uint32_t key = gathered_key(p, p.rank, j, i) & mask;
    n_gt += all || key > prefix;
    n_eq += !all && key == prefix;
  }
  const uint32_t gt_before = block_scan(n_gt, warp_sums, &sh_total);
  const uint32_t n_gt_all = sh_total;
  const uint32_t eq_before_t = block_scan(n_eq, warp_sums, &sh_total);
  const uint32_t e0 = sh_eq_before;
  const uint32_t room = need == 0xffffffffu ? 0xffffffffu : (e0 < need ? need - e0 : 0u);  // ties this rank may take
  const uint32_t n_sel = n_gt_all + min(sh_total, room);
  uint32_t pos = gt_before + min(eq_before_t, room);
  const uint32_t take_eq = eq_before_t < room ? min(n_eq, room - eq_before_t) : 0u;
  uint32_t eq_seen = 0;
  int32_t* out = p.out + (int64_t)j * p.out_ld;
  for (int i = tlo; i < thi; ++i) {
    const uint32_t key = gathered_key(p, p.rank, j, i) & mask;
    bool take = all || key > prefix;
    if (!take && key == prefix) take = eq_seen++ < take_eq;
    if (take && pos < (uint32_t)p.out_cols) {
      const int blk = p.out_base + i;
      out[pos] = blk;
      int32_t slot = 1;
      if (p.res.block_slot != nullptr) {
        slot = __ldcg(p.res.block_slot + (int64_t)j * p.res.bs_ld + blk);
        p.res.hot[(int64_t)j * p.res.hot_ld + pos] = slot >= 1 ? slot : -1;
      }
      if (p.bitmap != nullptr && slot >= 1 && blk / 32 < p.bitmap_words) atomicOr(&p.bitmap[(int64_t)j * p.bitmap_words + blk / 32], 1u << (blk % 32));
      ++pos;
    }
  }
  for (int c = (int)n_sel + tid; c < p.out_cols; c += blockDim.x) {
    out[c] = -1;
    if (p.res.block_slot != nullptr) p.res.hot[(int64_t)j * p.res.hot_ld + c] = -1;
  }
}

}  // namespace
}  // namespace lkv

namespace lkv {
cudaError_t select_device_status(int* status, int clear) { return tu_device_status(status, clear); }
cudaError_t select_status_attach(int* mirror) { return tu_status_attach(mirror); }
}  // namespace lkv

using namespace lkv;

extern "C" {

int lkv_debug_set(int key, int64_t value) {
  switch (key) {
    case LKV_DEBUG_SELECT_WAIT_ITERS:
      if (value < 1 || value > (int64_t)kMaxWaitIters) return fail(LKV_ERR_ARG, "lkv_debug_set: wait bound %lld outside [1, %u]", (long long)value, kMaxWaitIters);
      g_sel_wait_iters = (uint32_t)value;
      return LKV_OK;
    case LKV_DEBUG_SELECT_STALL_NEXT:
      g_sel_stall_next = value != 0;
      return LKV_OK;
    case LKV_DEBUG_EXCHANGE_WAIT_ITERS:
      return exchange_set_wait_iters(value);
    default:
      return fail(LKV_ERR_ARG, "lkv_debug_set: unknown key %d", key);
  }
}

size_t lkv_quest_topk_workspace(int h, int n_cand) {
  return kKeysOffset + (size_t)(h > 0 ? h : 0) * (size_t)(n_cand > 0 ? n_cand : 0) * sizeof(uint64_t);
}

}  // extern "C"

namespace lkv {
namespace {

int quest_topk_impl(const void* q, int q_dtype, int hq, int h, int d, const void* kmin, const void* kmax, int meta_dtype, int64_t m_head,
                    int first_block, int n_cand, int k, int bound_mode, int order, int32_t* out_blocks, int out_ld, float* out_bound,
                    uint32_t* bitmap, int bitmap_words, void* workspace, size_t workspace_bytes, void* stream,
                    const ResidentOut& res = ResidentOut{nullptr, 0, nullptr, 0}) {
  if (!dtype_ok(q_dtype) || !dtype_ok(meta_dtype) || !dtype_ok(bound_mode))
    return fail(LKV_ERR_ARG, "lkv_quest_topk: bad dtype (q %d, meta %d, bound %d)", q_dtype, meta_dtype, bound_mode);
  if (h <= 0 || hq <= 0 || hq % h != 0) return fail(LKV_ERR_ARG, "lkv_quest_topk: %d query heads do not group over %d KV heads", hq, h);
  if (d <= 0 || d % 8 != 0 || d > 256) return fail(LKV_ERR_ARG, "lkv_quest_topk: head_dim %d unsupported", d);
  if (n_cand <= 0 || k <= 0 || k > n_cand) return fail(LKV_ERR_ARG, "lkv_quest_topk: need 0 < k <= n_cand (k=%d, n_cand=%d)", k, n_cand);
  if (k > kMaxK && order != LKV_ORDER_BLOCK) return fail(LKV_ERR_ARG, "lkv_quest_topk: k=%d exceeds %d", k, kMaxK);
  if (first_block < 0) return fail(LKV_ERR_ARG, "lkv_quest_topk: negative first block");
  if (out_ld < k) return fail(LKV_ERR_ARG, "lkv_quest_topk: output row stride %d < k=%d", out_ld, k);
  if (order != LKV_ORDER_BOUND && order != LKV_ORDER_BLOCK) return fail(LKV_ERR_ARG, "lkv_quest_topk: bad order %d", order);
  if (q == nullptr || kmin == nullptr || kmax == nullptr || out_blocks == nullptr || workspace == nullptr)
    return fail(LKV_ERR_PTR, "lkv_quest_topk: null pointer");
  if (!aligned(kmin, 16) || !aligned(kmax, 16) || (m_head * (int64_t)dtype_size(meta_dtype)) % 16 != 0)
    return fail(LKV_ERR_PTR, "lkv_quest_topk: metadata rows must be 16-byte aligned");
  if (workspace_bytes < lkv_quest_topk_workspace(h, n_cand))
    return fail(LKV_ERR_WORKSPACE, "lkv_quest_topk: workspace %zu < %zu bytes", workspace_bytes, lkv_quest_topk_workspace(h, n_cand));
  if (bitmap != nullptr && bitmap_words * 32ll < (int64_t)first_block + n_cand)
    return fail(LKV_ERR_ARG, "lkv_quest_topk: bitmap of %d words cannot hold block %d", bitmap_words, first_block + n_cand - 1);
  const int g = hq / h;
  cudaStream_t st = as_stream(stream);
  // A bf16 bound's orderable 32-bit form has constant low 16 bits for a given sign, so its top 16
  // bits order the keys: two 8-bit passes reach the k-th bound; ties go to the scan.
  const int n_passes = bound_mode == LKV_BF16 ? 2 : 4;
  uint32_t* hist0 = static_cast<uint32_t*>(workspace);  // first-pass histograms, zero between calls
  uint64_t* keys = reinterpret_cast<uint64_t*>(static_cast<unsigned char*>(workspace) + kKeysOffset);
  // bf16 query and metadata at head_dim 64, block-id order: TMA scoring, then a cluster per head
  // selects (its launch placed while the scoring runs).
  {
    SelParams sp{};
    if (select_plan(g, q_dtype, meta_dtype, h, d, kmin, kmax, m_head, first_block, n_cand, order, sp)) {
      sp.q = static_cast<const __nv_bfloat16*>(q);
      sp.n_cand = n_cand;
      sp.k = k;
      sp.first_block = first_block;
      sp.n_passes = n_passes;
      sp.bound_mode = bound_mode;
      sp.out_blocks = out_blocks;
      sp.out_ld = out_ld;
      sp.bitmap = bitmap;
      sp.bitmap_words = bitmap_words;
      sp.out_bound = out_bound;
      sp.hist0 = hist0;
      sp.fail = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(workspace) + kFailOffset);
      sp.keys = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(workspace) + kKeysOffset);
      sp.wait_iters = g_sel_wait_iters;
      sp.stall = g_sel_stall_next;
      sp.res = res;
      g_sel_stall_next = 0;
      return launch_select(g, sp, h, st);
    }
  }
  // Ascending block-id order with at most kHistHeads heads: the score kernel also counts the first
  // radix pass, and a cluster per head finishes the select from the keys.
  const bool cluster = order == LKV_ORDER_BLOCK && h <= kHistHeads && cluster_size_for(n_cand) > 0;
  if (!cluster && k > kMaxK) return fail(LKV_ERR_ARG, "lkv_quest_topk: k=%d exceeds %d", k, kMaxK);
  if (!cluster && res.block_slot != nullptr)
    return fail(LKV_ERR_ARG, "lkv_quest_topk_resident: needs block order, at most %d heads and %d candidates", kHistHeads, kClusterMax * kClusterMaxPer);
  uint32_t* h0 = cluster ? hist0 : nullptr;
  int rc;
  if (q_dtype == LKV_BF16 && meta_dtype == LKV_BF16)
    rc = launch_score<__nv_bfloat16, __nv_bfloat16>(g, h, d, st, q, kmin, kmax, m_head, first_block, n_cand, bound_mode, keys, out_bound, h0);
  else if (q_dtype == LKV_F32 && meta_dtype == LKV_F32)
    rc = launch_score<float, float>(g, h, d, st, q, kmin, kmax, m_head, first_block, n_cand, bound_mode, keys, out_bound, h0);
  else if (q_dtype == LKV_BF16 && meta_dtype == LKV_F32)
    rc = launch_score<__nv_bfloat16, float>(g, h, d, st, q, kmin, kmax, m_head, first_block, n_cand, bound_mode, keys, out_bound, h0);
  else
    rc = launch_score<float, __nv_bfloat16>(g, h, d, st, q, kmin, kmax, m_head, first_block, n_cand, bound_mode, keys, out_bound, h0);
  if (rc) return rc;
  if ((rc = launched("lkv_quest_topk(score)"))) return rc;
  if (cluster) {
    if ((rc = launch_topk_cluster(h, st, keys, hist0, n_cand, k, first_block, n_passes, out_blocks, out_ld, bitmap, bitmap_words, res))) return rc;
    return launched("lkv_quest_topk(cluster select)");
  }
  int P = 1;
  while (P < k) P <<= 1;
  const size_t sel_smem = (size_t)(P < 2 ? 2 : P) * sizeof(uint64_t);
  const int stage_keys = sel_smem + (size_t)n_cand * sizeof(uint64_t) <= 200 * 1024;
  const size_t smem = sel_smem + (stage_keys ? (size_t)n_cand * sizeof(uint64_t) : 0);
  if (smem > 48 * 1024) cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  topk_kernel<<<h, kSelectThreads, smem, st>>>(keys, n_cand, k, first_block, out_blocks, out_ld, bitmap, bitmap_words, stage_keys,
                                                order == LKV_ORDER_BLOCK, n_passes);
  return launched("lkv_quest_topk(select)");
}

}  // namespace
}  // namespace lkv

extern "C" {

int lkv_quest_topk(const void* q, int q_dtype, int hq, int h, int d, const void* kmin, const void* kmax,
                   int meta_dtype, int64_t m_head, int first_block, int n_cand, int k, int bound_mode, int order,
                   int32_t* out_blocks, int out_ld, float* out_bound, uint32_t* bitmap, int bitmap_words,
                   void* workspace, size_t workspace_bytes, void* stream) {
  return quest_topk_impl(q, q_dtype, hq, h, d, kmin, kmax, meta_dtype, m_head, first_block, n_cand, k, bound_mode, order, out_blocks, out_ld,
                         out_bound, bitmap, bitmap_words, workspace, workspace_bytes, stream);
}

int lkv_quest_topk_resident(const void* q, int q_dtype, int hq, int h, int d, const void* kmin, const void* kmax, int meta_dtype, int64_t m_head,
                            int first_block, int n_cand, int k, int bound_mode, int32_t* out_blocks, int out_ld, const int32_t* block_slot,
                            int cap, int32_t* hot, int64_t hot_ld, uint32_t* bitmap, int bitmap_words, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (block_slot == nullptr || hot == nullptr) return fail(LKV_ERR_PTR, "lkv_quest_topk_resident: null pointer");
  if (cap < first_block + n_cand || hot_ld < k) return fail(LKV_ERR_ARG, "lkv_quest_topk_resident: block_slot of %d blocks or hot row of %lld < k", cap,
                                                           (long long)hot_ld);
  const ResidentOut res{block_slot, (int64_t)cap, hot, hot_ld};
  return quest_topk_impl(q, q_dtype, hq, h, d, kmin, kmax, meta_dtype, m_head, first_block, n_cand, k, bound_mode, LKV_ORDER_BLOCK, out_blocks,
                         out_ld, nullptr, bitmap, bitmap_words, workspace, workspace_bytes, stream, res);
}

int lkv_quest_topk_admit(const void* q, int q_dtype, int hq, int h, int d, const void* kmin, const void* kmax, int meta_dtype, int64_t m_head,
                         int first_block, int n_cand, int k, int bound_mode, int32_t* out_blocks, int out_ld, float* out_bound,
                         uint32_t* bitmap, int bitmap_words, void* workspace, size_t workspace_bytes, int32_t* block_slot, int cap,
                         int32_t* slot_block, int64_t* last_used, int n_slots, int64_t* evicted_at, int64_t step, const void* store,
                         int store_kind, void* pool, int bs, int dtype, int32_t* miss_blk, int32_t* miss_slot, int32_t* n_miss,
                         int32_t* slots_out, int64_t slots_ld, int64_t* miss_total, void* stream) {
  // The admit's arguments are checked before anything is launched, as lkv_tier_admit checks them.
  if (!dtype_ok(dtype)) return fail(LKV_ERR_ARG, "lkv_quest_topk_admit: bad dtype %d", dtype);
  if (store_kind != LKV_COLD_INT8 && store_kind != LKV_COLD_PAIRS) return fail(LKV_ERR_ARG, "lkv_quest_topk_admit: bad store kind %d", store_kind);
  if (h <= 0 || k <= 0 || cap <= 0 || n_slots < k) return fail(LKV_ERR_ARG, "lkv_quest_topk_admit: need h, k, cap > 0 and n_slots >= k (%d < %d)", n_slots, k);
  if (n_slots > (1 << 16)) return fail(LKV_ERR_ARG, "lkv_quest_topk_admit: %d slots above 65536", n_slots);
  if (block_slot == nullptr || slot_block == nullptr || last_used == nullptr || store == nullptr || pool == nullptr || miss_blk == nullptr ||
      miss_slot == nullptr || n_miss == nullptr)
    return fail(LKV_ERR_PTR, "lkv_quest_topk_admit: null pointer");
  if (!aligned(store, 16) || !aligned(pool, 16)) return fail(LKV_ERR_PTR, "lkv_quest_topk_admit: store and pool must be 16-byte aligned");
  if (bs % 8 || d % 8 || bs > 128 || d > 256) return fail(LKV_ERR_ARG, "lkv_quest_topk_admit: bs and d must be multiples of 8 (bs <= 128, d <= 256)");
  if ((int64_t)first_block + n_cand > cap) return fail(LKV_ERR_ARG, "lkv_quest_topk_admit: candidates end past the %d blocks of block_slot", cap);
  const int rc = quest_topk_impl(q, q_dtype, hq, h, d, kmin, kmax, meta_dtype, m_head, first_block, n_cand, k, bound_mode, LKV_ORDER_BLOCK,
                                 out_blocks, out_ld, out_bound, bitmap, bitmap_words, workspace, workspace_bytes, stream);
  if (rc != LKV_OK) return rc;
  return lkv_tier_admit(out_blocks, h, k, out_ld, block_slot, cap, slot_block, last_used, n_slots, evicted_at, step, store, store_kind, pool, bs, d,
                        dtype, miss_blk, miss_slot, n_miss, slots_out, slots_ld, miss_total, stream);
}

size_t lkv_topk_merge_workspace(int h, int n) { return lkv_quest_topk_workspace(h, n); }

int lkv_topk_merge(const float* bounds, const int32_t* ids, int h, int n, int64_t ld, int k, int bound_mode, int order, int32_t* out_blocks,
                   int out_ld, uint32_t* bitmap, int bitmap_words, void* workspace, size_t workspace_bytes, void* stream) {
  if (!dtype_ok(bound_mode)) return fail(LKV_ERR_ARG, "lkv_topk_merge: bad bound mode %d", bound_mode);
  if (h <= 0 || n <= 0 || k <= 0 || k > n || ld < n) return fail(LKV_ERR_ARG, "lkv_topk_merge: need 0 < k <= n <= ld (h=%d, n=%d, k=%d)", h, n, k);
  if (k > kMaxK) return fail(LKV_ERR_ARG, "lkv_topk_merge: k=%d exceeds %d", k, kMaxK);
  if (out_ld < k) return fail(LKV_ERR_ARG, "lkv_topk_merge: output row stride %d < k=%d", out_ld, k);
  if (order != LKV_ORDER_BOUND && order != LKV_ORDER_BLOCK) return fail(LKV_ERR_ARG, "lkv_topk_merge: bad order %d", order);
  if (bounds == nullptr || ids == nullptr || out_blocks == nullptr || workspace == nullptr) return fail(LKV_ERR_PTR, "lkv_topk_merge: null pointer");
  if (workspace_bytes < lkv_topk_merge_workspace(h, n))
    return fail(LKV_ERR_WORKSPACE, "lkv_topk_merge: workspace %zu < %zu bytes", workspace_bytes, lkv_topk_merge_workspace(h, n));
  cudaStream_t st = as_stream(stream);
  uint64_t* keys = reinterpret_cast<uint64_t*>(static_cast<unsigned char*>(workspace) + kKeysOffset);
  merge_keys_kernel<<<dim3((n + 255) / 256, h), 256, 0, st>>>(bounds, ids, n, ld, keys);
  if (int rc = launched("lkv_topk_merge(keys)")) return rc;
  int P = 1;
  while (P < k) P <<= 1;
  const size_t sel_smem = (size_t)(P < 2 ? 2 : P) * sizeof(uint64_t);
  const int stage_keys = sel_smem + (size_t)n * sizeof(uint64_t) <= 200 * 1024;
  const size_t smem = sel_smem + (stage_keys ? (size_t)n * sizeof(uint64_t) : 0);
  if (smem > 48 * 1024) cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  topk_kernel<<<h, kSelectThreads, smem, st>>>(keys, n, k, 0, out_blocks, out_ld, bitmap, bitmap_words, stage_keys, order == LKV_ORDER_BLOCK,
                                                bound_mode == LKV_BF16 ? 2 : 4);
  return launched("lkv_topk_merge(select)");
}

int lkv_quest_bounds(const void* q, int q_dtype, int hq, int h, int d, const void* kmin, const void* kmax, int meta_dtype, int64_t m_head,
                     int first_block, int n_cand, int bound_mode, void* bounds, int bounds_dtype, int64_t bounds_ld, void* stream) {
  if (!dtype_ok(q_dtype) || !dtype_ok(meta_dtype) || !dtype_ok(bound_mode) || !dtype_ok(bounds_dtype))
    return fail(LKV_ERR_ARG, "lkv_quest_bounds: bad dtype (q %d, meta %d, bound %d, out %d)", q_dtype, meta_dtype, bound_mode, bounds_dtype);
  if (bounds_dtype == LKV_BF16 && bound_mode != LKV_BF16) return fail(LKV_ERR_ARG, "lkv_quest_bounds: float32 bounds do not fit bf16 output");
  if (h <= 0 || hq <= 0 || hq % h != 0) return fail(LKV_ERR_ARG, "lkv_quest_bounds: %d query heads do not group over %d KV heads", hq, h);
  if (d <= 0 || d % 8 != 0 || d > 256) return fail(LKV_ERR_ARG, "lkv_quest_bounds: head_dim %d unsupported", d);
  if (n_cand <= 0 || first_block < 0 || bounds_ld < n_cand)
    return fail(LKV_ERR_ARG, "lkv_quest_bounds: need n_cand > 0, first_block >= 0, bounds_ld >= n_cand (%d, %d, %lld)", n_cand, first_block,
                (long long)bounds_ld);
  if (q == nullptr || kmin == nullptr || kmax == nullptr || bounds == nullptr) return fail(LKV_ERR_PTR, "lkv_quest_bounds: null pointer");
  if (!aligned(kmin, 16) || !aligned(kmax, 16) || (m_head * (int64_t)dtype_size(meta_dtype)) % 16 != 0)
    return fail(LKV_ERR_PTR, "lkv_quest_bounds: metadata rows must be 16-byte aligned");
  const int g = hq / h;
  cudaStream_t st = as_stream(stream);
  float* b32 = bounds_dtype == LKV_F32 ? static_cast<float*>(bounds) : nullptr;
  __nv_bfloat16* b16 = bounds_dtype == LKV_BF16 ? static_cast<__nv_bfloat16*>(bounds) : nullptr;
  int rc;
  if (q_dtype == LKV_BF16 && meta_dtype == LKV_BF16)
    rc = launch_score<__nv_bfloat16, __nv_bfloat16>(g, h, d, st, q, kmin, kmax, m_head, first_block, n_cand, bound_mode, nullptr, b32, nullptr, b16, bounds_ld);
  else if (q_dtype == LKV_F32 && meta_dtype == LKV_F32)
    rc = launch_score<float, float>(g, h, d, st, q, kmin, kmax, m_head, first_block, n_cand, bound_mode, nullptr, b32, nullptr, b16, bounds_ld);
  else if (q_dtype == LKV_BF16 && meta_dtype == LKV_F32)
    rc = launch_score<__nv_bfloat16, float>(g, h, d, st, q, kmin, kmax, m_head, first_block, n_cand, bound_mode, nullptr, b32, nullptr, b16, bounds_ld);
  else
    rc = launch_score<float, __nv_bfloat16>(g, h, d, st, q, kmin, kmax, m_head, first_block, n_cand, bound_mode, nullptr, b32, nullptr, b16, bounds_ld);
  if (rc) return rc;
  return launched("lkv_quest_bounds");
}

int lkv_topk_gathered(const void* bounds, int bounds_dtype, int world, int h, int64_t ld, const int32_t* seg_n, int k, int rank, int out_base,
                      int32_t* out_local, int out_ld, int out_cols, uint32_t* bitmap, int bitmap_words, void* stream) {
  return lkv_topk_gathered_resident(bounds, bounds_dtype, world, h, ld, seg_n, k, rank, out_base, out_local, out_ld, out_cols, bitmap, bitmap_words,
                                    nullptr, 0, nullptr, 0, stream);
}

int lkv_topk_gathered_resident(const void* bounds, int bounds_dtype, int world, int h, int64_t ld, const int32_t* seg_n, int k, int rank,
                               int out_base, int32_t* out_local, int out_ld, int out_cols, uint32_t* bitmap, int bitmap_words,
                               const int32_t* block_slot, int cap, int32_t* hot, int64_t hot_ld, void* stream) {
  if (bounds_dtype != LKV_BF16 && bounds_dtype != LKV_F32) return fail(LKV_ERR_ARG, "lkv_topk_gathered: bounds must be bf16 or float32");
  if (world <= 0 || world > kMaxWorld || rank < 0 || rank >= world) return fail(LKV_ERR_ARG, "lkv_topk_gathered: rank %d of %d (at most %d)", rank, world, kMaxWorld);
  if (h <= 0 || k <= 0 || out_base < 0 || seg_n == nullptr) return fail(LKV_ERR_ARG, "lkv_topk_gathered: need h, k > 0, out_base >= 0, counts");
  if (bounds == nullptr || out_local == nullptr) return fail(LKV_ERR_PTR, "lkv_topk_gathered: null pointer");
  GatherSel p{};
  p.seg_start[0] = 0;
  for (int r = 0; r < world; ++r) {
    if (seg_n[r] < 0 || seg_n[r] > ld) return fail(LKV_ERR_ARG, "lkv_topk_gathered: rank %d has %d candidates (row stride %lld)", r, seg_n[r], (long long)ld);
    if ((int64_t)p.seg_start[r] + seg_n[r] > INT32_MAX) return fail(LKV_ERR_ARG, "lkv_topk_gathered: too many candidates");
    p.seg_start[r + 1] = p.seg_start[r] + seg_n[r];
  }
  if (p.seg_start[world] <= 0) return fail(LKV_ERR_ARG, "lkv_topk_gathered: no candidates");
  const int n_my = seg_n[rank];
  const int most = k < n_my ? k : n_my;  // at most this many of the chosen fall in this rank's range
  if (out_cols < most || out_ld < out_cols)
    return fail(LKV_ERR_ARG, "lkv_topk_gathered: %d output columns (row stride %d) cannot hold up to %d chosen ids", out_cols, out_ld, most);
  if (bitmap != nullptr && bitmap_words * 32ll < (int64_t)out_base + n_my)
    return fail(LKV_ERR_ARG, "lkv_topk_gathered: bitmap of %d words cannot hold local block %d", bitmap_words, out_base + n_my - 1);
  p.bounds = bounds;
  p.bf16 = bounds_dtype == LKV_BF16;
  p.world = world;
  p.h = h;
  p.ld = ld;
  p.k = k;
  p.n_passes = bounds_dtype == LKV_BF16 ? 2 : 4;
  p.rank = rank;
  p.out_base = out_base;
  p.out = out_local;
  p.out_ld = out_ld;
  p.out_cols = out_cols;
  p.bitmap = bitmap;
  p.bitmap_words = bitmap_words;
  if (block_slot != nullptr) {
    if (hot == nullptr || hot_ld < out_cols || cap < out_base + n_my)
      return fail(LKV_ERR_ARG, "lkv_topk_gathered_resident: hot rows of %lld < %d columns, or block_slot of %d blocks", (long long)hot_ld, out_cols, cap);
    p.res = ResidentOut{block_slot, (int64_t)cap, hot, hot_ld};
  }
  cudaError_t e = launch_pdl(topk_gathered_kernel, dim3(h), dim3(kSelectThreads), 0, as_stream(stream), 0, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv_topk_gathered: %s", cudaGetErrorString(e));
  }
  return LKV_OK;
}

}  // extern "C"

// ---- allocation-free top-k -------------------------------------------------------------------
//
// Some callers cannot allocate device memory at the point where they select blocks: an
// allocator-free serving runtime, code running inside an allocator callback or under a
// framework's memory guard, or a host that has reserved all device memory up front. For them,
// lkv_quest_topk_noalloc keeps its scratch (the 64-bit (bound, block) keys the score kernel writes
// and the select kernel reads) in the fixed array below instead of a caller workspace.

namespace lkv {
namespace {

// 4 MiB of keys: h * n_cand <= 524,288 (e.g. 8 KV heads x 65,536 candidate blocks, a 1M-token
// context in 16-token blocks). Every device that loads the library holds it until exit.
constexpr size_t kNoAllocScratchBytes = kKeysOffset + (4u << 20);
static __device__ __align__(256) uint64_t g_topk_scratch[kNoAllocScratchBytes / sizeof(uint64_t)];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_topk_scratch on the current device, looked up once per device. In host
// code the array's name is only a stand-in for the symbol, never an address to pass to a kernel.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(LKV_ERR_CUDA, "lkv_quest_topk_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(LKV_ERR_ARG, "lkv_quest_topk_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_topk_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(LKV_ERR_CUDA, "lkv_quest_topk_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return LKV_OK;
}

}  // namespace
}  // namespace lkv

extern "C" int lkv_quest_topk_noalloc(const void* q, int q_dtype, int hq, int h, int d, const void* kmin,
                                      const void* kmax, int meta_dtype, int64_t m_head, int first_block, int n_cand,
                                      int k, int bound_mode, int order, int32_t* out_blocks, int out_ld, float* out_bound,
                                      uint32_t* bitmap, int bitmap_words, void* stream) {
  const size_t need = lkv_quest_topk_workspace(h, n_cand);
  if (need > kNoAllocScratchBytes)
    return fail(LKV_ERR_ARG, "lkv_quest_topk_noalloc: %d heads x %d candidates need %zu bytes of scratch, above its fixed %zu (h * n_cand <= %zu)",
                h, n_cand, need, kNoAllocScratchBytes, (kNoAllocScratchBytes - kKeysOffset) / sizeof(uint64_t));
  void* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  // The array's first kKeysOffset bytes are the block-order paths' counters (the first-pass
  // histograms and the TMA-scored selection's failure words), which must read zero on entry:
  // __device__ storage starts zeroed and every complete call leaves them zero (a call whose bounded
  // wait ran out too: its select resets them). A call that returns an error may have launched a
  // kernel that counts without the one that zeroes, so they are cleared then (an asynchronous memset
  // on the stream, which allocates nothing). The keys after the counters need no clearing: every key
  // a select reads was written by the same call. Calls whose kernels overlap on the GPU share the
  // array and race.
  const int rc = lkv_quest_topk(q, q_dtype, hq, h, d, kmin, kmax, meta_dtype, m_head, first_block, n_cand, k, bound_mode, order,
                                out_blocks, out_ld, out_bound, bitmap, bitmap_words, scratch, kNoAllocScratchBytes, stream);
  if (rc != LKV_OK) cudaMemsetAsync(scratch, 0, kKeysOffset, as_stream(stream));
  return rc;
}

// ---- ragged rows: many sequences' selections in two launches -------------------------------
//
// Continuous batching puts sequences of different lengths in one decode step. Row r = seq * heads
// + head has n_cand(r) candidate blocks (logical blocks 1 .. n_cand) and keeps k(r) of them; its
// blocks live anywhere in a paged store, found through the sequence's block table (logical block ->
// store row), and the metadata kmin / kmax are [heads][store rows][d]. The score kernel takes a
// flattened list of (row, first candidate) chunks of up to 256 candidates, so long and short rows
// cost in proportion to their candidates; it computes each candidate's bound exactly as
// quest_score_kernel does (same channel order and roundings) and stores its orderable form. The
// select kernel is one CTA per row: a radix select over its keys in shared memory, then the kept
// blocks in ascending id order (ties to the lowest ids, as the single-sequence select), and the
// row's bitmap.

namespace lkv {
namespace {

constexpr int kRaggedMaxCand = 16384;  // candidates of a row: the select keeps its keys in shared memory

template <typename TQ, typename TM, int G>
__global__ void ragged_score_kernel(const TQ* __restrict__ q, int d, const TM* __restrict__ kmin, const TM* __restrict__ kmax, int64_t m_head,
                                    int64_t n_store, int heads, const int32_t* __restrict__ table, int64_t table_stride,
                                    const int2* __restrict__ work, const int2* __restrict__ row_sel, int bound_mode, uint32_t* __restrict__ keys,
                                    int64_t key_stride) {
  extern __shared__ __align__(16) float qs[];  // q+ [d][GP], q- [d][GP], then the two tiles
  __shared__ int sh_store[256];
  const int rows = blockDim.x;
  const int row_bytes = d * (int)sizeof(TM);
  const int chunks = row_bytes / 16;
  unsigned char* tile_max = reinterpret_cast<unsigned char*>(qs + 2 * qpad<G>() * d);
  unsigned char* tile_min = tile_max + (size_t)rows * row_bytes;
  const int2 w = work[blockIdx.x];
  const int r = w.x, c_first = w.y;
  const int n_cand = row_sel[r].x;
  const int n_rows = min(rows, n_cand - c_first);
  if (n_rows <= 0) return;
  const int head = r % heads;
  const int32_t* tab = table + (int64_t)(r / heads) * table_stride;
  stage_query<TQ, G>(q, r, d, qs);
  for (int t = threadIdx.x; t < n_rows; t += blockDim.x) {
    const int srow = __ldg(tab + 1 + c_first + t);
    sh_store[t] = (srow >= 0 && srow < n_store) ? srow : -1;  // outside the store: no load, lowest key
  }
  __syncthreads();
  for (int u = threadIdx.x; u < n_rows * chunks; u += blockDim.x) {
    int t, c;
    tile_rc(u, chunks, t, c);
    const int srow = sh_store[t];
    if (srow < 0) continue;
    const int pos = tile_pos(t, c, chunks, row_bytes);
    const int64_t off = (int64_t)head * m_head + (int64_t)srow * d;
    cp_async16(tile_max + pos, reinterpret_cast<const uint4*>(kmax + off) + c);
    cp_async16(tile_min + pos, reinterpret_cast<const uint4*>(kmin + off) + c);
  }
  cp_async_wait_all();
  __syncthreads();
  const int t = threadIdx.x;
  if (t < n_rows) {
    uint32_t key = 0u;
    if (sh_store[t] >= 0) key = orderable(row_bound<TQ, TM, G>(tile_max, tile_min, t, d, qs, bound_mode));
    keys[(int64_t)r * key_stride + c_first + t] = key;
  }
}

// One CTA (kSelectThreads) per row: out[r][0 .. k) the kept logical blocks ascending, bitmap row r.
__global__ void __launch_bounds__(kSelectThreads) ragged_topk_kernel(const uint32_t* __restrict__ keys, int64_t key_stride,
                                                                      const int2* __restrict__ row_sel, int n_passes, int32_t* __restrict__ out,
                                                                      int64_t out_stride, uint32_t* __restrict__ bitmap, int bitmap_words) {
  extern __shared__ uint32_t ks[];
  __shared__ uint32_t hist[256], warp_sums[32];
  __shared__ uint32_t sh_digit, sh_remaining, sh_bincount, sh_total;
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const int n = min(row_sel[r].x, kRaggedMaxCand);
  const int k = min(row_sel[r].y, n);
  const uint32_t* src = keys + (int64_t)r * key_stride;
  for (int i = tid; i < n; i += blockDim.x) ks[i] = src[i];
  if (bitmap != nullptr)
    for (int wd = tid; wd < bitmap_words; wd += blockDim.x) bitmap[(int64_t)r * bitmap_words + wd] = 0u;
  if (tid == 0) {
    sh_remaining = (uint32_t)k;
    sh_bincount = 0u;
  }
  __syncthreads();
  uint32_t prefix = 0u, mask = 0u;
  bool take_all = k >= n;
  for (int pass = 0; pass < n_passes && !take_all && k > 0; ++pass) {
    const int shift = 24 - 8 * pass;
    if (tid < 256) hist[tid] = 0u;
    __syncthreads();
    for (int base = 0; base < n; base += blockDim.x) {
      const int i = base + tid;
      const uint32_t key = i < n ? ks[i] : 0u;
      const bool counted = i < n && (key & mask) == prefix;
      const uint32_t digit = counted ? ((key >> shift) & 255u) : 256u;
      const uint32_t peers = __match_any_sync(0xffffffffu, digit);
      if (counted && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
    }
    __syncthreads();
    pick_digit(hist, &sh_digit, &sh_remaining, &sh_bincount);
    __syncthreads();
    prefix |= sh_digit << shift;
    mask |= 255u << shift;
    take_all = sh_bincount == sh_remaining;  // uniform: every thread read the same shared values
    __syncthreads();
  }
  // Taken: keys above the prefix, then the first `need` keys at it in id order (all when take_all).
  const uint32_t need = take_all ? 0xffffffffu : sh_remaining;
  const bool all = k >= n;
  const int per = (n + (int)blockDim.x - 1) / (int)blockDim.x;
  const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
  uint32_t gt = 0, eq = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t m = ks[i] & mask;
    if (all || m > prefix || (take_all && m == prefix)) ++gt;
    else if (m == prefix) ++eq;
  }
  const uint32_t pre = block_scan(gt | (eq << 16), warp_sums, &sh_total);
  uint32_t pos_gt = pre & 0xffffu, pos_eq = pre >> 16;  // taken-above and tied keys before this thread's ids
  if (k > 0)
    for (int i = i0; i < i1; ++i) {
      const uint32_t m = ks[i] & mask;
      const bool above = all || m > prefix || (take_all && m == prefix);
      uint32_t pos = 0xffffffffu;
      if (above) {
        pos = pos_gt + min(pos_eq, need);
        ++pos_gt;
      } else if (m == prefix) {
        if (pos_eq < need) pos = pos_gt + pos_eq;
        ++pos_eq;
      }
      if (pos < (uint32_t)k) {
        const int blk = 1 + i;
        out[(int64_t)r * out_stride + pos] = blk;
        if (bitmap != nullptr && blk / 32 < bitmap_words) atomicOr(&bitmap[(int64_t)r * bitmap_words + blk / 32], 1u << (blk % 32));
      }
    }
}

template <typename TQ, typename TM>
int launch_ragged_score(int g, int d, int heads, cudaStream_t st, const void* q, const void* kmin, const void* kmax, int64_t m_head,
                        int64_t n_store, const int32_t* table, int64_t table_stride, const int2* work, int n_work, const int2* row_sel,
                        int bound_mode, uint32_t* keys, int64_t key_stride) {
  const int rows = 256;
  auto smem_for = [&](int gp) { return (size_t)2 * gp * d * sizeof(float) + 2 * (size_t)rows * d * sizeof(TM); };
  const TQ* qq = static_cast<const TQ*>(q);
  const TM* mn = static_cast<const TM*>(kmin);
  const TM* mx = static_cast<const TM*>(kmax);
#define LKV_RAGGED_SCORE(GG)                                                                                                       \
  {                                                                                                                                \
    auto kern = ragged_score_kernel<TQ, TM, GG>;                                                                                   \
    const size_t smem = smem_for(qpad<GG>());                                                                                      \
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                    \
    kern<<<n_work, rows, smem, st>>>(qq, d, mn, mx, m_head, n_store, heads, table, table_stride, work, row_sel, bound_mode, keys, \
                                     key_stride);                                                                                  \
    return launched("lkv_ragged_quest_topk(score)");                                                                              \
  }
  switch (g) {
    case 1: LKV_RAGGED_SCORE(1)
    case 2: LKV_RAGGED_SCORE(2)
    case 4: LKV_RAGGED_SCORE(4)
    case 8: LKV_RAGGED_SCORE(8)
    default: return fail(LKV_ERR_ARG, "lkv_ragged_quest_topk: query group %d not in {1,2,4,8}", g);
  }
#undef LKV_RAGGED_SCORE
}

}  // namespace
}  // namespace lkv

extern "C" {

size_t lkv_ragged_topk_workspace(int rows, int max_cand) {
  if (rows <= 0 || max_cand <= 0) return 0;
  return (size_t)rows * (size_t)max_cand * sizeof(uint32_t);
}

int lkv_ragged_quest_topk(const void* q, int q_dtype, int rows, int g, int d, int heads, const void* kmin, const void* kmax, int meta_dtype,
                          int64_t m_head, int64_t n_store, const int32_t* table, int64_t table_stride, const int32_t* row_sel, int max_cand,
                          const int32_t* work, int n_work, int bound_mode, int32_t* out_blocks, int64_t out_stride, uint32_t* bitmap,
                          int bitmap_words, void* workspace, size_t workspace_bytes, void* stream) {
  const char* who = "lkv_ragged_quest_topk";
  if (!dtype_ok(q_dtype) || !dtype_ok(meta_dtype) || !dtype_ok(bound_mode) || q_dtype != meta_dtype)
    return fail(LKV_ERR_ARG, "%s: query and metadata must share a dtype (q %d, meta %d, bound %d)", who, q_dtype, meta_dtype, bound_mode);
  if (rows <= 0 || heads <= 0 || rows % heads != 0) return fail(LKV_ERR_ARG, "%s: %d rows do not group over %d KV heads", who, rows, heads);
  if (d <= 0 || d % 8 != 0 || d > 256) return fail(LKV_ERR_ARG, "%s: head_dim %d unsupported", who, d);
  if (max_cand <= 0 || max_cand > kRaggedMaxCand) return fail(LKV_ERR_ARG, "%s: max_cand %d outside [1, %d]", who, max_cand, kRaggedMaxCand);
  if (n_work <= 0 || n_store <= 0 || table_stride <= max_cand || out_stride <= 0)
    return fail(LKV_ERR_ARG, "%s: bad sizes (work %d, store %lld, table stride %lld)", who, n_work, (long long)n_store, (long long)table_stride);
  if (q == nullptr || kmin == nullptr || kmax == nullptr || table == nullptr || row_sel == nullptr || work == nullptr || out_blocks == nullptr ||
      workspace == nullptr)
    return fail(LKV_ERR_PTR, "%s: null pointer", who);
  if (!aligned(kmin, 16) || !aligned(kmax, 16) || (m_head * (int64_t)dtype_size(meta_dtype)) % 16 != 0)
    return fail(LKV_ERR_PTR, "%s: metadata rows must be 16-byte aligned", who);
  if (!aligned(work, 8) || !aligned(row_sel, 8)) return fail(LKV_ERR_PTR, "%s: work and row_sel must be 8-byte aligned", who);
  if (workspace_bytes < lkv_ragged_topk_workspace(rows, max_cand))
    return fail(LKV_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", who, workspace_bytes, lkv_ragged_topk_workspace(rows, max_cand));
  if (bitmap != nullptr && bitmap_words * 32ll < (int64_t)max_cand + 1)
    return fail(LKV_ERR_ARG, "%s: bitmap of %d words cannot hold block %d", who, bitmap_words, max_cand);
  cudaStream_t st = as_stream(stream);
  uint32_t* keys = static_cast<uint32_t*>(workspace);
  const int2* wk = reinterpret_cast<const int2*>(work);
  const int2* rs = reinterpret_cast<const int2*>(row_sel);
  int rc = q_dtype == LKV_BF16 ? launch_ragged_score<__nv_bfloat16, __nv_bfloat16>(g, d, heads, st, q, kmin, kmax, m_head, n_store, table, table_stride,
                                                                                  wk, n_work, rs, bound_mode, keys, max_cand)
                               : launch_ragged_score<float, float>(g, d, heads, st, q, kmin, kmax, m_head, n_store, table, table_stride, wk, n_work,
                                                                  rs, bound_mode, keys, max_cand);
  if (rc) return rc;
  const size_t smem = (size_t)max_cand * sizeof(uint32_t);
  if (smem > 48 * 1024) cudaFuncSetAttribute(ragged_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  ragged_topk_kernel<<<rows, kSelectThreads, smem, st>>>(keys, max_cand, rs, bound_mode == LKV_BF16 ? 2 : 4, out_blocks, out_stride, bitmap,
                                                         bitmap_words);
  return launched("lkv_ragged_quest_topk(select)");
}

}  // extern "C"
