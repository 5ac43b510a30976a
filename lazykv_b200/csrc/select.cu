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
#include <mutex>

#include "common.cuh"

namespace lkv {
namespace {

constexpr int kScoreThreads = 128;
constexpr int kSelectThreads = 1024;
constexpr int kMaxK = 16384;  // shared-memory sort capacity (128 KiB of keys)

template <typename TQ, typename TM, int G>
__global__ void __launch_bounds__(kScoreThreads) quest_score_kernel(
    const TQ* __restrict__ q, int d, const TM* __restrict__ kmin, const TM* __restrict__ kmax,
    int64_t m_head, int first_block, int n_cand, int bound_mode, uint64_t* __restrict__ keys,
    float* __restrict__ out_bound) {
  extern __shared__ float qs[];  // qp [G][d] then qn [G][d]
  const int j = blockIdx.y;
  for (int e = threadIdx.x; e < G * d; e += blockDim.x) {
    const float v = to_f32<TQ>(q[(int64_t)j * G * d + e]);
    const float vp = fmaxf(v, 0.0f);      // q.clamp_min(0)
    qs[e] = vp;
    qs[G * d + e] = __fsub_rn(v, vp);     // q - qp
  }
  __syncthreads();
  const int ci = blockIdx.x * blockDim.x + threadIdx.x;
  if (ci >= n_cand) return;
  const int64_t row = (int64_t)j * m_head + (int64_t)(first_block + ci) * d;
  const TM* pmax = kmax + row;
  const TM* pmin = kmin + row;
  float a[G], b[G];
#pragma unroll
  for (int r = 0; r < G; ++r) a[r] = b[r] = 0.0f;
  for (int c0 = 0; c0 < d; c0 += 8) {
    float mx[8], mn[8];
    Vec8<TM>::load(pmax + c0, mx);
    Vec8<TM>::load(pmin + c0, mn);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int r = 0; r < G; ++r) {
        a[r] = __fadd_rn(a[r], __fmul_rn(qs[r * d + c0 + i], mx[i]));
        b[r] = __fadd_rn(b[r], __fmul_rn(qs[G * d + r * d + c0 + i], mn[i]));
      }
    }
  }
  float best = -INFINITY;
#pragma unroll
  for (int r = 0; r < G; ++r) {
    float s = bound_mode == LKV_BF16 ? bf16_round(__fadd_rn(bf16_round(a[r]), bf16_round(b[r]))) : __fadd_rn(a[r], b[r]);
    best = fmaxf(best, s);
  }
  const uint64_t key = ((uint64_t)orderable(best) << 32) | (uint64_t)(0xffffffffu - (uint32_t)ci);
  keys[(int64_t)j * n_cand + ci] = key;
  if (out_bound != nullptr) out_bound[(int64_t)j * n_cand + ci] = best == 0.0f ? 0.0f : best;
}

// Finds, among keys matching `prefix` under `mask`, the digit at `shift` holding the `remaining`-th
// largest; called by all threads after `hist` is complete. Warp 0 scans the 256 bins from the top.
__device__ void pick_digit(const uint32_t* hist, uint32_t* sh_digit, uint32_t* sh_remaining,
                           uint32_t* sh_bincount) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    // Lane l owns bins 255-8l .. 248-8l (highest first).
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

__global__ void __launch_bounds__(kSelectThreads) topk_kernel(
    const uint64_t* __restrict__ keys_all, int n_cand, int k, int first_block,
    int32_t* __restrict__ out_blocks, int out_ld, uint32_t* __restrict__ bitmap, int bitmap_words) {
  extern __shared__ uint64_t sel[];  // [P]
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sh_digit, sh_remaining, sh_bincount, sh_count;
  __shared__ uint64_t sh_thr;
  const int j = blockIdx.x;
  const uint64_t* keys = keys_all + (int64_t)j * n_cand;
  if (bitmap != nullptr)
    for (int w = threadIdx.x; w < bitmap_words; w += blockDim.x) bitmap[(int64_t)j * bitmap_words + w] = 0u;

  uint64_t prefix = 0, mask = 0;
  if (threadIdx.x == 0) {
    sh_remaining = (uint32_t)k;
    sh_count = 0;
  }
  bool done = (k >= n_cand);
  for (int pass = 0; pass < 8 && !done; ++pass) {
    const int shift = 56 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n_cand; i += blockDim.x) {
      const uint64_t key = keys[i];
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    pick_digit(hist, &sh_digit, &sh_remaining, &sh_bincount);
    __syncthreads();
    prefix |= (uint64_t)sh_digit << shift;
    mask |= (uint64_t)255u << shift;
    // Every key matching the prefix is taken: the threshold is the prefix itself.
    done = (sh_bincount == sh_remaining);
    __syncthreads();
  }
  if (threadIdx.x == 0) sh_thr = (k >= n_cand) ? 0ull : prefix;
  __syncthreads();
  const uint64_t thr = sh_thr;
  int P = 1;
  const int kk = k < n_cand ? k : n_cand;
  while (P < kk) P <<= 1;
  for (int i = threadIdx.x; i < n_cand; i += blockDim.x) {
    const uint64_t key = keys[i];
    if (key >= thr) {
      const uint32_t pos = atomicAdd(&sh_count, 1u);
      if (pos < (uint32_t)P) sel[pos] = key;
    }
  }
  __syncthreads();
  for (int i = kk + threadIdx.x; i < P; i += blockDim.x) sel[i] = 0ull;
  __syncthreads();
  // Bitonic sort, descending.
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < P / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t a = sel[lo], b = sel[hi];
        if ((a < b) == desc) {
          sel[lo] = b;
          sel[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < kk; i += blockDim.x) {
    const uint32_t ci = 0xffffffffu - (uint32_t)(sel[i] & 0xffffffffull);
    const int blk = first_block + (int)ci;
    out_blocks[(int64_t)j * out_ld + i] = blk;
    if (bitmap != nullptr && blk / 32 < bitmap_words)
      atomicOr(&bitmap[(int64_t)j * bitmap_words + blk / 32], 1u << (blk % 32));
  }
}

template <typename TQ, typename TM>
int launch_score(int g, dim3 grid, size_t smem, cudaStream_t st, const void* q, int d, const void* kmin,
                 const void* kmax, int64_t m_head, int first_block, int n_cand, int bound_mode,
                 uint64_t* keys, float* out_bound) {
#define LKV_SCORE(G)                                                                            \
  case G:                                                                                       \
    quest_score_kernel<TQ, TM, G><<<grid, kScoreThreads, smem, st>>>(                           \
        static_cast<const TQ*>(q), d, static_cast<const TM*>(kmin), static_cast<const TM*>(kmax), \
        m_head, first_block, n_cand, bound_mode, keys, out_bound);                              \
    break;
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

}  // namespace
}  // namespace lkv

using namespace lkv;

extern "C" {

size_t lkv_quest_topk_workspace(int h, int n_cand) {
  return (size_t)(h > 0 ? h : 0) * (size_t)(n_cand > 0 ? n_cand : 0) * sizeof(uint64_t);
}

int lkv_quest_topk(const void* q, int q_dtype, int hq, int h, int d, const void* kmin, const void* kmax,
                   int meta_dtype, int64_t m_head, int first_block, int n_cand, int k, int bound_mode,
                   int32_t* out_blocks, int out_ld, float* out_bound, uint32_t* bitmap, int bitmap_words,
                   void* workspace, size_t workspace_bytes, void* stream) {
  if (!dtype_ok(q_dtype) || !dtype_ok(meta_dtype) || !dtype_ok(bound_mode))
    return fail(LKV_ERR_ARG, "lkv_quest_topk: bad dtype (q %d, meta %d, bound %d)", q_dtype, meta_dtype, bound_mode);
  if (h <= 0 || hq <= 0 || hq % h != 0) return fail(LKV_ERR_ARG, "lkv_quest_topk: %d query heads do not group over %d KV heads", hq, h);
  if (d <= 0 || d % 8 != 0 || d > 256) return fail(LKV_ERR_ARG, "lkv_quest_topk: head_dim %d unsupported", d);
  if (n_cand <= 0 || k <= 0 || k > n_cand) return fail(LKV_ERR_ARG, "lkv_quest_topk: need 0 < k <= n_cand (k=%d, n_cand=%d)", k, n_cand);
  if (k > kMaxK) return fail(LKV_ERR_ARG, "lkv_quest_topk: k=%d exceeds %d", k, kMaxK);
  if (first_block < 0) return fail(LKV_ERR_ARG, "lkv_quest_topk: negative first block");
  if (out_ld < k) return fail(LKV_ERR_ARG, "lkv_quest_topk: output row stride %d < k=%d", out_ld, k);
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
  uint64_t* keys = static_cast<uint64_t*>(workspace);
  dim3 grid((n_cand + kScoreThreads - 1) / kScoreThreads, h);
  const size_t smem = 2 * (size_t)g * d * sizeof(float);
  int rc;
  if (q_dtype == LKV_BF16 && meta_dtype == LKV_BF16)
    rc = launch_score<__nv_bfloat16, __nv_bfloat16>(g, grid, smem, st, q, d, kmin, kmax, m_head, first_block, n_cand, bound_mode, keys, out_bound);
  else if (q_dtype == LKV_F32 && meta_dtype == LKV_F32)
    rc = launch_score<float, float>(g, grid, smem, st, q, d, kmin, kmax, m_head, first_block, n_cand, bound_mode, keys, out_bound);
  else if (q_dtype == LKV_BF16 && meta_dtype == LKV_F32)
    rc = launch_score<__nv_bfloat16, float>(g, grid, smem, st, q, d, kmin, kmax, m_head, first_block, n_cand, bound_mode, keys, out_bound);
  else
    rc = launch_score<float, __nv_bfloat16>(g, grid, smem, st, q, d, kmin, kmax, m_head, first_block, n_cand, bound_mode, keys, out_bound);
  if (rc) return rc;
  if ((rc = launched("lkv_quest_topk(score)"))) return rc;
  int P = 1;
  while (P < k) P <<= 1;
  const size_t sel_smem = (size_t)P * sizeof(uint64_t);
  if (sel_smem > 48 * 1024) cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sel_smem);
  topk_kernel<<<h, kSelectThreads, sel_smem, st>>>(keys, n_cand, k, first_block, out_blocks, out_ld, bitmap, bitmap_words);
  return launched("lkv_quest_topk(select)");
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
constexpr size_t kNoAllocScratchBytes = 4u << 20;
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
                                      int k, int bound_mode, int32_t* out_blocks, int out_ld, float* out_bound,
                                      uint32_t* bitmap, int bitmap_words, void* stream) {
  const size_t need = lkv_quest_topk_workspace(h, n_cand);
  if (need > kNoAllocScratchBytes)
    return fail(LKV_ERR_ARG, "lkv_quest_topk_noalloc: %d heads x %d candidates need %zu bytes of scratch, above its fixed %zu (h * n_cand <= %zu)",
                h, n_cand, need, kNoAllocScratchBytes, kNoAllocScratchBytes / sizeof(uint64_t));
  void* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  // Nothing in the scratch has to start at zero: the score kernel writes every key the select
  // kernel reads. Calls whose kernels overlap on the GPU share the array and race.
  return lkv_quest_topk(q, q_dtype, hq, h, d, kmin, kmax, meta_dtype, m_head, first_block, n_cand, k, bound_mode,
                        out_blocks, out_ld, out_bound, bitmap, bitmap_words, scratch, kNoAllocScratchBytes, stream);
}
