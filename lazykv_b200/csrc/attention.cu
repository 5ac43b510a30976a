// K4/K5/K6: split decode attention over listed or remaining blocks, and the log-sum-exp merge.
//
// One launch serves either pass of lazykv/exact.py's set split, or both at once:
//  * hot segment (lazykv/tiered.py:465-487 + lazykv/attention.py:125-136): the key sequence of KV
//    head j is the n_list listed blocks, read in place through an optional block->slot map (no
//    gather copy); the last listed block is the current block with `last_fill` live tokens
//    (selection.py:65-69); a listed id of -1 is padding (no load, no keys), which lets heads list
//    different numbers of blocks (a shard's part of a global selection);
//  * cold segment (lazykv/exact.py:88-127): blocks [first, first + n) minus a per-head exclusion
//    bitmap, read from int8 records with the dequantisation fused (quant.py:103-104: float32
//    affine, then rounded to the model dtype, i.e. what a fetch puts in a slot), or from pairs in
//    the model dtype.
// Each CTA takes a share of the items of one KV head and emits online-softmax partials (running
// max m in the log2 domain, sum l, unnormalised o) for the head's G query rows, per segment; the
// partials are folded into per-segment (out = o / l, lse) and into their merge. A partial over no
// key is (m = -inf, l = 0), which the fold turns into lse = -inf and out = 0, as
// cpu_partial_attention does (exact.py:108-110).
//
// Three kernels do the partial work:
//  * attn_stream_kernel (bf16, d 64 or 128, bs 16, G <= 8, stores in device memory: the metric's
//    and the long-context geometry): tensor-core contractions, int8 records dequantised straight
//    into mma fragments, a balanced split of every segment over one CTA per SM, and the fold done by the head's last CTA
//    (no second launch); described at the kernel;
//  * attn_tma_kernel (stores in device memory, G = 4, bs = 16, d in {64, 128}): each warp streams
//    its items through a private ring of shared-memory stages filled by TMA bulk copies
//    (cp.async.bulk, one mbarrier per stage, bounded waits); the block ids, slot rows and exclusion
//    bits of the warp's items are prefetched into registers so issuing never waits on a dependent
//    global load; dot products and accumulations use packed float32x2 FMAs;
//  * attn_ldg_kernel (any other geometry, and stores in mapped host memory read over the link):
//    the same arithmetic with vectorised loads straight from global memory.
// The last two emit one partial per CTA and a combine kernel folds them.
// Lane layout (CUDA-core kernels) in a warp: CG = d/16 channel groups x TL = 32/CG token lanes; a lane holds 16
// channels of the G query rows and of its accumulators and takes tokens tl, tl + TL, ... of a block.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <type_traits>
#include <mutex>

#include "tma.cuh"

namespace lkv {
namespace {

int* g_status_word = nullptr;  // the host mirror of the status word (lkv_status_attach)

constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kMinChunk = 16;             // blocks per CTA at least (4 per warp)
constexpr int kTargetCtas = 2 * kNumSMs;  // two resident CTAs per SM
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLazy = 8.0f;  // log2-domain headroom of the lazy rescaling (weights <= 256)

enum SegKind { SEG_LIST = 0, SEG_RANGE_REC = 1, SEG_RANGE_PAIRS = 2 };

struct Seg {
  int kind;
  // strided pairs in the model dtype: hot pool, full cache, or a pairs cold store (element strides)
  const void* k_base;
  const void* v_base;
  int64_t s_row, s_head, s_tok;
  // int8 records [blocks, h, width]
  const uint8_t* records;
  int64_t width;
  // listed items
  const int32_t* blocks;
  int n_list, last_fill;
  const int32_t* slot_of;
  int64_t slot_stride;
  int64_t n_rows;  // storage rows addressable from k_base / v_base (0 = unknown)
  // range items
  int first_block;
  const uint32_t* excluded;
  int bitmap_words;
  // split of the items over CTAs
  int n_items, chunk, n_splits;
};

struct AttnParams {
  const void* q;
  int hq, h, bs;
  float scale_log2;
  Seg seg[2];
  int n_segs, n_splits_total;
  float* part;  // [h][n_splits_total][G][D + 2]
};

int splits_for(int n_items, int target) {
  if (n_items <= 0) return 0;
  int s = (n_items + kMinChunk - 1) / kMinChunk;
  if (s > target) s = target;
  if (s < 1) s = 1;
  const int chunk = (n_items + s - 1) / s;
  return (n_items + chunk - 1) / chunk;
}

void set_split(Seg& S, int target) {
  S.n_splits = splits_for(S.n_items, target);
  S.chunk = S.n_splits > 0 ? (S.n_items + S.n_splits - 1) / S.n_splits : 0;
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// A dequantised cold value as the model dtype holds it: the exact pass attends to what a fetch
// would put in a slot (unpack in the model dtype), so under bf16 each value is rounded once more.
template <typename T>
__device__ __forceinline__ float as_model(float x) {
  if constexpr (sizeof(T) == 2) return __bfloat162float(__float2bfloat16_rn(x));
  return x;
}
template <typename T>
__device__ __forceinline__ float2 as_model2(float2 x) {
  if constexpr (sizeof(T) == 2) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(x.x, x.y);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(&b);
    return f2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  return x;
}

__device__ __forceinline__ bool range_excluded(const Seg& S, int j, int blk) {
  return S.excluded != nullptr && blk / 32 < S.bitmap_words &&
         ((__ldg(S.excluded + (int64_t)j * S.bitmap_words + blk / 32) >> (blk % 32)) & 1u);
}

// ============================================================================================
// attn_ldg_kernel: plain loads, any supported geometry, any memory (device or mapped host)
// ============================================================================================

template <typename T, int N>
__device__ __forceinline__ void load_chunk(const T* p, float* out) {
  if constexpr (N % 8 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 8) Vec8<T>::load(p + i, out + i);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f32<T>(p[i]);
  }
}

// N int8 codes -> (code + 128) as float.
template <int N>
__device__ __forceinline__ void load_codes(const uint8_t* p, float* out) {
  if constexpr (N == 16) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int b = 0; b < 4; ++b) out[4 * i + b] = (float)(int8_t)((w[i] >> (8 * b)) & 0xffu) + 128.0f;
  } else if constexpr (N == 4) {
    uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(p));
#pragma unroll
    for (int b = 0; b < 4; ++b) out[b] = (float)(int8_t)((w >> (8 * b)) & 0xffu) + 128.0f;
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = (float)(int8_t)p[i] + 128.0f;
  }
}

__device__ __forceinline__ float ldh(const uint8_t* p) { return __half2float(__ldg(reinterpret_cast<const __half*>(p))); }

template <int G, int D>
__device__ void write_cta_partial(const float (&sh_m)[kWarps][G], const float (&sh_l)[kWarps][G], const float (&sh_o)[kWarps][G][D],
                                  float* out) {
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int r = e / D, c = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sh_m[w][r]);
    float O = 0.0f, Lr = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float f = sh_m[w][r] == -INFINITY ? 0.0f : exp2f(sh_m[w][r] - M);
        O = fmaf(sh_o[w][r][c], f, O);
        Lr = fmaf(sh_l[w][r], f, Lr);
      }
    }
    out[2 * G + r * D + c] = O;
    if (c == 0) {
      out[r] = M;
      out[G + r] = Lr;
    }
  }
}

template <typename T, int G, int D>
__global__ void __launch_bounds__(kThreads) attn_ldg_kernel(const AttnParams p) {
  constexpr int CG = D >= 128 ? 8 : 4;
  constexpr int CPL = D / CG;
  constexpr int TL = 32 / CG;
  __shared__ float sh_m[kWarps][G], sh_l[kWarps][G];
  __shared__ float sh_o[kWarps][G][D];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cg = lane % CG, tl = lane / CG;
  const int j = blockIdx.y;
  int split = blockIdx.x, si = 0;
  if (p.n_segs > 1 && split >= p.seg[0].n_splits) {
    si = 1;
    split -= p.seg[0].n_splits;
  }
  const Seg& S = p.seg[si];
  const bool int8 = S.kind == SEG_RANGE_REC;
  const int c0 = cg * CPL;

  float qr[G][CPL];
  {
    const T* q = static_cast<const T*>(p.q) + (int64_t)j * G * D;
#pragma unroll
    for (int r = 0; r < G; ++r) {
      load_chunk<T, CPL>(q + r * D + c0, qr[r]);
#pragma unroll
      for (int c = 0; c < CPL; ++c) qr[r][c] *= p.scale_log2;
    }
  }
  float m[G], l[G], o[G][CPL];
#pragma unroll
  for (int r = 0; r < G; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) o[r][c] = 0.0f;
  }

  const int begin = split * S.chunk;
  const int end = min(S.n_items, begin + S.chunk);
  for (int it = begin + warp; it < end; it += kWarps) {
    int blk, live = p.bs;
    if (S.kind == SEG_LIST) {
      blk = __ldg(S.blocks + (int64_t)j * S.n_list + it);
      if (blk < 0) continue;  // padding
      if (it == S.n_list - 1) live = S.last_fill;
    } else {
      blk = S.first_block + it;
      if (range_excluded(S, j, blk)) continue;
    }
    const T* kp = nullptr;
    const T* vp = nullptr;
    const uint8_t* rec = nullptr;
    float ks[CPL], kz[CPL];
    if (int8) {
      rec = S.records + ((int64_t)blk * p.h + j) * S.width;
      const uint8_t* sc = rec + 2ll * p.bs * D;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        ks[c] = ldh(sc + 2 * (c0 + c));
        kz[c] = ldh(sc + 2 * D + 2 * (c0 + c));
      }
    } else {
      const int64_t row = (S.kind == SEG_LIST && S.slot_of != nullptr) ? (int64_t)__ldg(S.slot_of + (int64_t)j * S.slot_stride + blk) : (int64_t)blk;
      kp = static_cast<const T*>(S.k_base) + row * S.s_row + (int64_t)j * S.s_head;
      vp = static_cast<const T*>(S.v_base) + row * S.s_row + (int64_t)j * S.s_head;
    }
    for (int t0 = 0; t0 < p.bs; t0 += TL) {
      const int t = t0 + tl;
      float kv[CPL];
      if (int8) {
        load_codes<CPL>(rec + (int64_t)t * D + c0, kv);
#pragma unroll
        for (int c = 0; c < CPL; ++c) kv[c] = as_model<T>(fmaf(kv[c], ks[c], kz[c]));
      } else {
        load_chunk<T, CPL>(kp + t * S.s_tok + c0, kv);
      }
      float s[G];
#pragma unroll
      for (int r = 0; r < G; ++r) {
        float acc = 0.0f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) acc = fmaf(qr[r][c], kv[c], acc);
        s[r] = acc;
      }
#pragma unroll
      for (int r = 0; r < G; ++r) {
#pragma unroll
        for (int off = 1; off < CG; off <<= 1) s[r] += __shfl_xor_sync(0xffffffffu, s[r], off);
        if (t >= live) s[r] = -INFINITY;
      }
      float pr[G];
#pragma unroll
      for (int r = 0; r < G; ++r) {
        float mb = s[r];
#pragma unroll
        for (int off = CG; off < 32; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
        if (mb > m[r]) {
          const float alpha = exp2f(m[r] - mb);  // 0 when m was -inf
          l[r] *= alpha;
#pragma unroll
          for (int c = 0; c < CPL; ++c) o[r][c] *= alpha;
          m[r] = mb;
        }
        pr[r] = m[r] == -INFINITY ? 0.0f : exp2f(s[r] - m[r]);
        l[r] += pr[r];
      }
      if (int8) {
        const uint8_t* sc = rec + 2ll * p.bs * D + 4 * D;
        const float vs = ldh(sc + 2 * t), vz = ldh(sc + 2 * p.bs + 2 * t);
        load_codes<CPL>(rec + (int64_t)p.bs * D + (int64_t)t * D + c0, kv);
#pragma unroll
        for (int c = 0; c < CPL; ++c) kv[c] = as_model<T>(fmaf(kv[c], vs, vz));
      } else {
        load_chunk<T, CPL>(vp + t * S.s_tok + c0, kv);
      }
#pragma unroll
      for (int r = 0; r < G; ++r)
#pragma unroll
        for (int c = 0; c < CPL; ++c) o[r][c] = fmaf(pr[r], kv[c], o[r][c]);
    }
  }

  // Reduce over the token lanes (m is uniform within the warp; the CG lanes of a token hold the
  // same l, so the sum over token lanes is the block sum).
#pragma unroll
  for (int r = 0; r < G; ++r) {
#pragma unroll
    for (int off = CG; off < 32; off <<= 1) {
      l[r] += __shfl_xor_sync(0xffffffffu, l[r], off);
#pragma unroll
      for (int c = 0; c < CPL; ++c) o[r][c] += __shfl_xor_sync(0xffffffffu, o[r][c], off);
    }
  }
  if (tl == 0) {
#pragma unroll
    for (int r = 0; r < G; ++r) {
#pragma unroll
      for (int c = 0; c < CPL; ++c) sh_o[warp][r][c0 + c] = o[r][c];
      if (cg == 0) {
        sh_m[warp][r] = m[r];
        sh_l[warp][r] = l[r];
      }
    }
  }
  __syncthreads();
  write_cta_partial<G, D>(sh_m, sh_l, sh_o, p.part + ((int64_t)j * p.n_splits_total + blockIdx.x) * G * (D + 2));
}

// ============================================================================================
// attn_tma_kernel: per-warp TMA rings, G = 4, bs = 16, d in {64, 128}, stores in device memory
// ============================================================================================

template <typename T, int D>
struct TmaCfg {
  static constexpr int G = 4, BS = 16;
  static constexpr int CG = D / 16, CPL = 16, TL = 32 / CG, TPL = BS / TL;
  static constexpr int PAIR = 2 * BS * D * (int)sizeof(T);
  static constexpr int REC = 2 * BS * D + 4 * D + 4 * BS;
  static constexpr int RAW = PAIR > REC ? PAIR : REC;
  static constexpr int STAGE = (RAW + 127) / 128 * 128;
  static constexpr int STAGES = STAGE <= 4096 ? 4 : 3;
  static constexpr int SCL_K = CG * (CPL + 4);             // padded per channel group
  static constexpr int SCL = 2 * SCL_K + 2 * BS;           // ks, kz, (vs, vz) per token
  static constexpr size_t SMEM = (size_t)kWarps * STAGES * STAGE + (size_t)kWarps * STAGES * 8 + (size_t)kWarps * SCL * 4 +
                                 (size_t)kWarps * G * D * 4 + (size_t)kWarps * 2 * G * 4;
};

// Lane channel order: for bf16 the two 16-byte halves of a lane's 32 bytes are read in swapped
// order on every other quarter-warp, so the 8 lanes of an LDS.128 phase hit 8 distinct bank groups.
template <typename T>
__device__ __forceinline__ int half_swap(int lane) {
  return sizeof(T) == 2 ? ((lane >> 2) & 1) : 0;
}

// 16 consecutive channels of a row (lane order) as 8 float2.
template <typename T>
__device__ __forceinline__ void lds_row16(const T* row, int swap, float2 (&x)[8]);

template <>
__device__ __forceinline__ void lds_row16<__nv_bfloat16>(const __nv_bfloat16* row, int swap, float2 (&x)[8]) {
  const uint4* p = reinterpret_cast<const uint4*>(row);
  const uint4 a = p[swap], b = p[1 - swap];
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = f2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
}

template <>
__device__ __forceinline__ void lds_row16<float>(const float* row, int, float2 (&x)[8]) {
  const float4* p = reinterpret_cast<const float4*>(row);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = p[i];
    x[2 * i] = f2(v.x, v.y);
    x[2 * i + 1] = f2(v.z, v.w);
  }
}

// 16 int8 codes (lane order) -> 8 float2 of (code + 128), exactly: the byte is placed in the low
// mantissa bits of 2^23 and 2^23 is subtracted.
__device__ __forceinline__ void codes16(const uint8_t* p, float2 (&u)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
  const float2 minus_magic = f2(-8388608.0f, -8388608.0f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // __byte_perm selector 0x765b: byte b of the code word, then bytes 1-3 of 0x4b000000.
    const float2 lo = f2(__uint_as_float(__byte_perm(w[i], 0x4b000000u, 0x7650)), __uint_as_float(__byte_perm(w[i], 0x4b000000u, 0x7651)));
    const float2 hi = f2(__uint_as_float(__byte_perm(w[i], 0x4b000000u, 0x7652)), __uint_as_float(__byte_perm(w[i], 0x4b000000u, 0x7653)));
    u[2 * i] = __fadd2_rn(lo, minus_magic);
    u[2 * i + 1] = __fadd2_rn(hi, minus_magic);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) attn_tma_kernel(const AttnParams p) {
  using C = TmaCfg<T, D>;
  constexpr int G = C::G, BS = C::BS, CG = C::CG, CPL = C::CPL, TL = C::TL, TPL = C::TPL, STAGES = C::STAGES;
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cg = lane % CG, tl = lane / CG;
  const int j = blockIdx.y;
  int split = blockIdx.x, si = 0;
  if (p.n_segs > 1 && split >= p.seg[0].n_splits) {
    si = 1;
    split -= p.seg[0].n_splits;
  }
  const Seg& S = p.seg[si];
  const bool list = S.kind == SEG_LIST;
  const bool rec = S.kind == SEG_RANGE_REC;

  unsigned char* stages = smem + (size_t)warp * STAGES * C::STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)kWarps * STAGES * C::STAGE) + warp * STAGES;
  float* scl = reinterpret_cast<float*>(smem + (size_t)kWarps * STAGES * C::STAGE + (size_t)kWarps * STAGES * 8) + warp * C::SCL;
  float* sh_o = reinterpret_cast<float*>(smem + (size_t)kWarps * STAGES * C::STAGE + (size_t)kWarps * STAGES * 8 + (size_t)kWarps * C::SCL * 4);
  float* sh_ml = sh_o + kWarps * G * D;  // [warp][m(G) | l(G)]

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // The lane's channels: physical = c0 + 8 * ((ci >> 3) ^ swap) + (ci & 7), ci = 0..15; records use
  // the natural order (16 codes are one 16-byte read).
  const int c0 = cg * CPL;
  const int swap = rec ? 0 : half_swap<T>(lane);
  float2 q2[G][8];
  {
    const T* q = static_cast<const T*>(p.q) + (int64_t)j * G * D;
#pragma unroll
    for (int r = 0; r < G; ++r) {
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const int c = c0 + 8 * ((w >> 2) ^ swap) + 2 * (w & 3);
        q2[r][w] = f2(to_f32<T>(q[r * D + c]) * p.scale_log2, to_f32<T>(q[r * D + c + 1]) * p.scale_log2);
      }
    }
  }
  float m[G], l[G];
  float2 o2[G][8];
#pragma unroll
  for (int r = 0; r < G; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) o2[r][w] = f2(0.0f, 0.0f);
  }

  const int begin = split * S.chunk;
  const int end = min(S.n_items, begin + S.chunk);

  // Per-warp item cache: for list segments, lane i holds the storage row of the warp's item
  // (batch * 32 + i); for range segments, lane i holds exclusion word (w0 + i) of the chunk.
  int row_cache = 0, cache_batch = -1;
  uint32_t excl_word = 0;
  const int w0 = (S.first_block + begin) / 32;
  if (!list) {
    const int w = w0 + lane;
    excl_word = (S.excluded != nullptr && w < S.bitmap_words && w * 32 < S.first_block + end)
                    ? __ldg(S.excluded + (int64_t)j * S.bitmap_words + w) : 0u;
  }
  // Next item at or after `it` (stepping by kWarps) that is not excluded, or `end`.
  auto next_item = [&](int it) -> int {
    if (list) return it < end ? it : end;
    while (it < end) {
      const int blk = S.first_block + it;
      const int wi = blk / 32 - w0;
      uint32_t word;
      if (wi < 32) {
        word = __shfl_sync(0xffffffffu, excl_word, wi);
      } else {
        word = (S.excluded != nullptr && blk / 32 < S.bitmap_words) ? __ldg(S.excluded + (int64_t)j * S.bitmap_words + blk / 32) : 0u;
      }
      if (!((word >> (blk % 32)) & 1u)) return it;
      it += kWarps;
    }
    return end;
  };
  // Storage row of the listed item `it`, the n-th of this warp (all lanes call it together).
  auto list_row = [&](int it, int n) -> int64_t {
    const int batch = n >> 5;
    if (batch != cache_batch) {
      const int my_it = begin + warp + (batch * 32 + lane) * kWarps;
      int r = 0;
      if (my_it < end) {
        const int blk = __ldg(S.blocks + (int64_t)j * S.n_list + my_it);
        r = blk < 0 ? -1 : (S.slot_of != nullptr ? __ldg(S.slot_of + (int64_t)j * S.slot_stride + blk) : blk);
      }
      row_cache = r;
      cache_batch = batch;
    }
    return (int64_t)__shfl_sync(0xffffffffu, row_cache, n & 31);
  };
  uint32_t pad_bits = 0;  // stages holding a padding item (no copy, nothing to attend)
  // Issue the copies of item `it` (the n-th of this warp) into stage `s`; lane 0 issues.
  auto issue = [&](int it, int n, int s) {
    unsigned char* dst = stages + (size_t)s * C::STAGE;
    if (list) {
      const int64_t row = list_row(it, n);
      pad_bits = (pad_bits & ~(1u << s)) | ((row < 0 ? 1u : 0u) << s);
      if (row < 0) {
        if (lane == 0) mbar_arrive(&bars[s]);
      } else if (lane == 0) {
        const T* kp = static_cast<const T*>(S.k_base) + row * S.s_row + (int64_t)j * S.s_head;
        const T* vp = static_cast<const T*>(S.v_base) + row * S.s_row + (int64_t)j * S.s_head;
        constexpr uint32_t half = BS * D * sizeof(T);
        mbar_arrive_expect_tx(&bars[s], 2 * half);
        tma_load_1d(dst, kp, half, &bars[s]);
        tma_load_1d(dst + half, vp, half, &bars[s]);
      }
    } else if (lane == 0) {
      const int blk = S.first_block + it;
      if (rec) {
        mbar_arrive_expect_tx(&bars[s], (uint32_t)S.width);
        tma_load_1d(dst, S.records + ((int64_t)blk * p.h + j) * S.width, (uint32_t)S.width, &bars[s]);
      } else {
        const T* kp = static_cast<const T*>(S.k_base) + (int64_t)blk * S.s_row + (int64_t)j * S.s_head;
        mbar_arrive_expect_tx(&bars[s], C::PAIR);
        tma_load_1d(dst, kp, C::PAIR, &bars[s]);
      }
    }
  };

  int issue_it = next_item(begin + warp), n_issued = 0;
#pragma unroll 1
  for (int s = 0; s < STAGES; ++s) {
    if (issue_it < end) {
      issue(issue_it, n_issued, s);
      ++n_issued;
      issue_it = next_item(issue_it + kWarps);
    }
  }

  uint32_t phase = 0;
  int s = 0, n_done = 0;
  bool ok = true;
#pragma unroll 1
  for (int it = next_item(begin + warp); it < end; it = next_item(it + kWarps)) {
    ok = __all_sync(0xffffffffu, mbar_wait(&bars[s], (phase >> s) & 1u));
    if (!ok) break;
    phase ^= 1u << s;
    ++n_done;
    if ((pad_bits >> s) & 1u) {  // padding: nothing to attend; the stage is free
      if (issue_it < end) {
        issue(issue_it, n_issued, s);
        ++n_issued;
        issue_it = next_item(issue_it + kWarps);
      }
      s = (s + 1 == STAGES) ? 0 : s + 1;
      continue;
    }
    const unsigned char* st = stages + (size_t)s * C::STAGE;
    const int live = (list && it == S.n_list - 1) ? S.last_fill : BS;

    // ---- scores of the lane's TPL tokens ----
    float sc[G][TPL];
    float2 ks2[8], kz2[8];
    if (rec) {
      // Scales of this record as float: K per channel (padded per channel group), V per token.
      const __half* hs = reinterpret_cast<const __half*>(st + 2 * BS * D);
      for (int c = lane; c < D; c += 32) {
        const int g = c / CPL, ci = c % CPL;
        scl[g * (CPL + 4) + ci] = __half2float(hs[c]);
        scl[C::SCL_K + g * (CPL + 4) + ci] = __half2float(hs[D + c]);
      }
      if (lane < BS) {
        scl[2 * C::SCL_K + 2 * lane] = __half2float(hs[2 * D + lane]);
        scl[2 * C::SCL_K + 2 * lane + 1] = __half2float(hs[2 * D + BS + lane]);
      }
      __syncwarp();
      const float4* a = reinterpret_cast<const float4*>(scl + cg * (CPL + 4));
      const float4* b = reinterpret_cast<const float4*>(scl + C::SCL_K + cg * (CPL + 4));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 x = a[i], y = b[i];
        ks2[2 * i] = f2(x.x, x.y);
        ks2[2 * i + 1] = f2(x.z, x.w);
        kz2[2 * i] = f2(y.x, y.y);
        kz2[2 * i + 1] = f2(y.z, y.w);
      }
    }
#pragma unroll
    for (int i = 0; i < TPL; ++i) {
      const int t = tl + TL * i;
      float2 k2[8];
      if (rec) {
        float2 u[8];
        codes16(st + t * D + c0, u);
#pragma unroll
        for (int w = 0; w < 8; ++w) k2[w] = as_model2<T>(__ffma2_rn(u[w], ks2[w], kz2[w]));
      } else {
        lds_row16<T>(reinterpret_cast<const T*>(st) + t * D + c0, swap, k2);
      }
#pragma unroll
      for (int r = 0; r < G; ++r) {
        float2 acc = __fmul2_rn(q2[r][0], k2[0]);
#pragma unroll
        for (int w = 1; w < 8; ++w) acc = __ffma2_rn(q2[r][w], k2[w], acc);
        sc[r][i] = acc.x + acc.y;
      }
    }
    // ---- softmax update (lazy rescaling) ----
    // m is a reference maximum, not the running one: weights exp2(s - m) may reach 2^kLazy before
    // the accumulators are rescaled, so a block needs the warp-wide maximum only when one of its
    // scores passes m + kLazy (one vote instead of a max reduction per row and block).
    bool need = false;
#pragma unroll
    for (int r = 0; r < G; ++r) {
#pragma unroll
      for (int i = 0; i < TPL; ++i) {
#pragma unroll
        for (int off = 1; off < CG; off <<= 1) sc[r][i] += __shfl_xor_sync(0xffffffffu, sc[r][i], off);
        if (tl + TL * i >= live) sc[r][i] = -INFINITY;
        need |= sc[r][i] > m[r] + kLazy;
      }
    }
    if (__any_sync(0xffffffffu, need)) {
#pragma unroll
      for (int r = 0; r < G; ++r) {
        float mb = -INFINITY;
#pragma unroll
        for (int i = 0; i < TPL; ++i) mb = fmaxf(mb, sc[r][i]);
#pragma unroll
        for (int off = CG; off < 32; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
        if (mb > m[r] + kLazy) {
          const float alpha = exp2f(m[r] - mb);  // 0 when m was -inf
          l[r] *= alpha;
          const float2 a2 = f2(alpha, alpha);
#pragma unroll
          for (int w = 0; w < 8; ++w) o2[r][w] = __fmul2_rn(o2[r][w], a2);
          m[r] = mb;
        }
      }
    }
    float pr[G][TPL];
#pragma unroll
    for (int r = 0; r < G; ++r) {
#pragma unroll
      for (int i = 0; i < TPL; ++i) {
        pr[r][i] = m[r] == -INFINITY ? 0.0f : exp2f(sc[r][i] - m[r]);
        l[r] += pr[r][i];
      }
    }
    // ---- values ----
#pragma unroll
    for (int i = 0; i < TPL; ++i) {
      const int t = tl + TL * i;
      float2 v2[8];
      if (rec) {
        codes16(st + BS * D + t * D + c0, v2);
        const float vs = scl[2 * C::SCL_K + 2 * t], vz = scl[2 * C::SCL_K + 2 * t + 1];
        const float2 vs2 = f2(vs, vs), vz2 = f2(vz, vz);
#pragma unroll
        for (int x = 0; x < 8; ++x) v2[x] = as_model2<T>(__ffma2_rn(v2[x], vs2, vz2));
      } else {
        lds_row16<T>(reinterpret_cast<const T*>(st) + BS * D + t * D + c0, swap, v2);
      }
#pragma unroll
      for (int r = 0; r < G; ++r) {
        const float2 pp = f2(pr[r][i], pr[r][i]);
#pragma unroll
        for (int x = 0; x < 8; ++x) o2[r][x] = __ffma2_rn(pp, v2[x], o2[r][x]);
      }
    }
    __syncwarp();  // every lane is done with stage s (and the scale scratch) before it is refilled
    if (issue_it < end) {
      issue(issue_it, n_issued, s);
      ++n_issued;
      issue_it = next_item(issue_it + kWarps);
    }
    s = (s + 1 == STAGES) ? 0 : s + 1;
  }
  // After a timed-out wait, wait (bounded) for the copies still in flight before the CTA's shared
  // memory can be reused.
  for (int k = n_done; !ok && k < n_issued; ++k) {
    if (!__all_sync(0xffffffffu, mbar_wait(&bars[s], (phase >> s) & 1u))) break;
    phase ^= 1u << s;
    s = (s + 1 == STAGES) ? 0 : s + 1;
  }

  // ---- warp reduction over the token lanes, then across warps ----
  // Lanes that read their two 16-byte halves swapped hold the accumulators of channels c0+8.. first;
  // put them back in channel order before lanes of different parity are summed.
  if (swap) {
#pragma unroll
    for (int r = 0; r < G; ++r)
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float2 t = o2[r][w];
        o2[r][w] = o2[r][w + 4];
        o2[r][w + 4] = t;
      }
  }
#pragma unroll
  for (int r = 0; r < G; ++r) {
#pragma unroll
    for (int off = CG; off < 32; off <<= 1) {
      l[r] += __shfl_xor_sync(0xffffffffu, l[r], off);
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        o2[r][w].x += __shfl_xor_sync(0xffffffffu, o2[r][w].x, off);
        o2[r][w].y += __shfl_xor_sync(0xffffffffu, o2[r][w].y, off);
      }
    }
  }
  if (tl == 0) {
#pragma unroll
    for (int r = 0; r < G; ++r) {
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const int c = c0 + 2 * w;
        sh_o[(warp * G + r) * D + c] = o2[r][w].x;
        sh_o[(warp * G + r) * D + c + 1] = o2[r][w].y;
      }
      if (cg == 0) {
        sh_ml[warp * 2 * G + r] = m[r];
        sh_ml[warp * 2 * G + G + r] = l[r];
      }
    }
  }
  __syncthreads();
  float* out = p.part + ((int64_t)j * p.n_splits_total + blockIdx.x) * G * (D + 2);
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int r = e / D, c = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sh_ml[w * 2 * G + r]);
    float O = 0.0f, Lr = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mw = sh_ml[w * 2 * G + r];
        const float f = mw == -INFINITY ? 0.0f : exp2f(mw - M);
        O = fmaf(sh_o[(w * G + r) * D + c], f, O);
        Lr = fmaf(sh_ml[w * 2 * G + G + r], f, Lr);
      }
    }
    out[2 * G + r * D + c] = O;
    if (c == 0) {
      out[r] = M;
      out[G + r] = Lr;
    }
  }
}

// ============================================================================================
// tensor-core helpers (bf16, d = 64, bs = 16)
// ============================================================================================
//
// Per item (one block of one KV head) a warp runs two small contractions on the tensor cores with
// mma.sync.m16n8k16 (bf16 operands, float32 accumulators):
//   S^T [16 tokens x 8 rows]   = K [16 x 64] . Q^T [64 x 8]      (4 k-steps; rows >= G are zero)
//   O^T [64 channels x 8 rows] += V^T [64 x 16] . P^T [16 x 8]   (4 m-tiles)
// bf16 K and V tiles reach shared memory as 16 rows x 128 bytes in the 128-byte swizzle (16-byte
// chunk c of row r stored at chunk c ^ (r & 7)) by tensor-map TMA loads, so ldmatrix reads them
// without bank conflicts. The products of bf16 operands are exact in float32; P (float32) enters
// the second contraction as the sum of three bf16 terms (hi + mid + lo, 24 significant bits), each
// a separate MMA, so the result keeps float32 accuracy. The score fragment becomes the P^T operand
// with movmatrix (an 8x8 transpose in registers).

// The stream kernel's geometry per head_dim (bs 16). A bf16 K or V tile is 16 tokens x D channels
// in 128-byte swizzled rows of 64 channels: one 2 KiB sub-tile per 64 channels, each its own tile
// load. An int8 record is K codes [16][D], V codes [16][D], then the K scales and zeros (fp16 [D]
// each) and the V scales and zeros (fp16 [16] each) (lazykv/quant.py:90-105).
template <int D>
struct MmaGeom {
  static_assert(D == 64 || D == 128, "head_dim");
  static constexpr int HALVES = D / 64;                 // 64-channel sub-tiles per tile
  static constexpr int TILE = 16 * D * 2;               // one K or V tile (bytes)
  static constexpr int HOT = 2 * TILE;                  // K tile + V tile
  static constexpr int REC = 32 * D + 4 * D + 64;       // int8 record: 2,368 bytes at D 64, 4,672 at D 128
  static constexpr int OFF_KS = 32 * D, OFF_VS = 36 * D, OFF_VZ = 36 * D + 32;
  static constexpr int KF = (REC + 127) / 128 * 128;    // the record's K scales, zeros as float32 [D] each
  static constexpr int STAGE = HOT;                     // a stage holds a tile pair or a record
  static constexpr int WARPS = D == 64 ? 16 : 8;        // WARPS x 2 stages of ring in shared memory
  static_assert(KF + 8 * D <= STAGE, "the record and its float32 scales inside one stage");
};
constexpr int kMmaRec = MmaGeom<64>::REC;  // int8 record at bs 16, d 64

struct MmaParams {
  AttnParams p;
  CUtensorMap tk[2], tv[2];  // per segment: K and V maps of a list or pairs segment
  int head_major[2];         // map coordinate order: (0, 0, head, row) instead of (0, 0, row, head)
};

// One 4-D tile load global -> this CTA's shared memory under an L2 cache policy. No multicast.
__device__ __forceinline__ void tma_load_4d_hint(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint64_t* bar,
                                                 uint64_t pol) {
  asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(
                   dst),
               "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(pol)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x by the hardware approximation (PTX ex2.approx.ftz.f32: relative error about 2^-22, subnormal
// results flushed to zero; 2^-inf = 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t movtrans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// (lo, hi) -> bf16x2 with lo in the low half; and back to float2 (exact).
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&b);
}
__device__ __forceinline__ float2 unpack_bf2(uint32_t w) { return f2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u)); }

// Splits (a, b) into three bf16x2 terms whose sum is (a, b) to 24 significant bits: each term is the
// bf16 rounding of what the previous ones left, and each residual (x - term) is exact in float32.
__device__ __forceinline__ void split3(float a, float b, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
  const float2 neg1 = f2(-1.0f, -1.0f);
  hi = pack_bf2(a, b);
  const float2 r = __ffma2_rn(unpack_bf2(hi), neg1, f2(a, b));
  mid = pack_bf2(r.x, r.y);
  const float2 r2 = __ffma2_rn(unpack_bf2(mid), neg1, r);
  lo = pack_bf2(r2.x, r2.y);
}

__device__ __forceinline__ uint32_t swz(int row, int chunk) { return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4)); }

// ============================================================================================
// attn_stream_kernel: balanced, warp-streaming tensor-core split decode
// (bf16, d = 64 or 128, bs = 16, G <= 8, stores in device memory)
// ============================================================================================
//
// Grid: P CTAs per KV head (P = kStreamCtasPerSm x SMs / h, raised when a CTA's items would not
// fit its list), MmaGeom<D>::WARPS warps per CTA (16 at d 64, 8 at d 128, so that two stages per
// warp fit in shared memory).
//
// Work split. A head's items are, per segment, the listed blocks (padding counted, then skipped)
// or the blocks of the range that the exclusion bitmap leaves. CTA i of P takes the i-th P-th of
// every segment's items: every CTA gets the same mix of bf16 tile pairs and int8 records whatever
// the selection left in the range. One CTA per SM, so no CTA waits on another for issue slots.
//
// Set-up (whole CTA): the range's items are counted by a popcount over the bitmap; the CTA's items
// are written to a shared-memory list as storage rows (list ids through the slot map; range blocks
// as the complement of the bitmap, placed by a block-wide scan of per-word counts).
// Streaming (each warp): warp w takes the w-th share of the CTA's items of each segment (segment 0's
// first); its items pass through its private ring of StreamCfg::STAGES stages (4 KiB at d 64, 8 KiB
// at d 128) that lane 0 fills by TMA (tile-mode loads of the K and V tiles in the 128-byte swizzle,
// one per 64 channels, or one bulk copy of the record) and refills as soon as the item in a stage
// has been used.
//
// Int8 records go from shared memory straight into mma fragments, with a fixed permutation of the
// channels (the contraction does not depend on the order): for S^T = K . Q^T lane (g, t) holds the
// D/4 channels (D/4)t .. (D/4)t + D/4 - 1 of tokens g and g + 8 (16-byte code loads, the K scales of
// those channels); for O^T += V^T . P^T lane g holds channels (D/8)g .. (D/8)g + D/8 - 1 of tokens 2t, 2t+1, 2t+8, 2t+9
// (four 8-byte loads). The query fragments follow the same permutation and the output channels are
// put back in order when the state is parked. Each value is (code + 128) * scale + zero in float32
// (one rounding) and then rounded to bf16: what a fetch would put in a slot (quant.py:103-104).
//
// Each warp keeps one online-softmax state (log2 domain, lazy rescaling) and parks it in shared
// memory when its items move to the next segment and at the end (then in the idle ring); the CTA
// folds its warps' parked
// states into one partial per segment in the workspace; the last CTA of the head (a per-head counter
// in the workspace, zero before and after the call) folds the head's partials into the outputs.

constexpr int kStreamCtasPerSm = 1;
constexpr int kStreamListCap = 3072;       // items per CTA
constexpr int kStreamCounterBytes = 4096;  // per-head CTA counters at the workspace start (h <= 1024)

template <int G, int D>
struct StreamCfg {
  static constexpr int NW = MmaGeom<D>::WARPS;
  static constexpr int THREADS = 32 * NW;
  static constexpr int STAGES = 2;  // per warp (the loop is unrolled over them)
  static constexpr int STAGE = MmaGeom<D>::STAGE;
  static constexpr int SLOT = G * D + 2 * G;    // floats of a parked state: o [G][D], m [G], l [G]
  static constexpr int RING = NW * STAGES * STAGE;
  static constexpr int PARK = NW * 2 * SLOT * 4;  // each warp's state per segment
  static constexpr int LIST = kStreamListCap * 4;
  static constexpr int BARS = NW * STAGES * 8;
  static constexpr size_t SMEM = 1024 + (size_t)RING + PARK + LIST + BARS;
  // Floats of one (CTA, set) partial in the workspace: o [G][D], m [G], l [G], padded to 16 bytes so
  // the rows of o are float4-aligned for every G.
  static constexpr int PART = (G * D + 2 * G + 3) / 4 * 4;
  static_assert(SMEM <= 227 * 1024, "shared memory of one CTA");
};

struct StreamParams {
  AttnParams p;              // segments in item order; segment s's partials are set s
  CUtensorMap tk[2], tv[2];  // K / V maps of tile segments
  int head_major[2];
  int per_head;              // P
  unsigned int* counters;    // [h]: zero on entry, left zero
  float* part;               // [h][P][2][PART]: o [G][D], m [G], l [G] per (CTA, set)
  void* out;                 // [hq, D] in TO (optional)
  float* lse;                // [hq] (optional)
  float* seg_out;            // [2, hq, D] (optional)
  float* seg_lse;            // [2, hq] (optional)
  // Ragged rows (batched sequences, one row per (sequence, KV head) = seq * heads + head); all null
  // for a single sequence, where row = KV head = blockIdx.y, CTA = blockIdx.x and P = per_head.
  const int4* sched;         // per CTA: (row, index in the row, the row's CTAs, the row's first partial)
  const int4* row_info;      // per row: (items of the list segment, last_fill, blocks of the range, 0)
  const int32_t* table;      // range blocks through block tables: record row = table[seq * table_stride + block]
  int64_t table_stride;
  int heads;                 // KV heads of a sequence (the pool's and the records' head index is row % heads)
};

// In-range blocks of bitmap word w that the exclusion bitmap of row j leaves (n_items: the row's blocks).
__device__ __forceinline__ uint32_t range_word_bits(const Seg& S, int n_items, int j, int w) {
  const int f = S.first_block, e = S.first_block + n_items;  // blocks [f, e)
  const int lo = max(f, 32 * w) - 32 * w, hi = min(e, 32 * w + 32) - 32 * w;
  if (hi <= lo) return 0u;
  const uint32_t in = (hi - lo == 32 ? 0xffffffffu : ((1u << (hi - lo)) - 1u)) << lo;
  const uint32_t ex = (S.excluded != nullptr && w < S.bitmap_words) ? __ldg(S.excluded + (int64_t)j * S.bitmap_words + w) : 0u;
  return in & ~ex;
}

// Block-wide exclusive prefix sum of v (every thread of the CTA calls it); *total gets the sum.
__device__ __forceinline__ int block_excl_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += u;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int s = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= off) s += u;
    }
    if (lane < nw) warp_sums[lane] = s;  // inclusive
    if (lane == nw - 1) *total = s;
  }
  __syncthreads();
  const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + incl - v;
  __syncthreads();  // warp_sums may be reused right after
  return before;
}

// 4 int8 codes (one word) -> (code + 128) as 4 floats (exact: 2^23 magic).
__device__ __forceinline__ void codes4(uint32_t w, float2& lo, float2& hi) {
  const uint32_t a = w ^ 0x80808080u;
  const float2 mm = f2(-8388608.0f, -8388608.0f);
  lo = __fadd2_rn(f2(__uint_as_float(__byte_perm(a, 0x4b000000u, 0x7650)), __uint_as_float(__byte_perm(a, 0x4b000000u, 0x7651))), mm);
  hi = __fadd2_rn(f2(__uint_as_float(__byte_perm(a, 0x4b000000u, 0x7652)), __uint_as_float(__byte_perm(a, 0x4b000000u, 0x7653))), mm);
}

// (code + 128) of byte `sel` of words a and c (already xor-ed with 0x80808080), as a float pair.
__device__ __forceinline__ float2 code_pair(uint32_t a, uint32_t c, uint32_t sel) {
  return __fadd2_rn(f2(__uint_as_float(__byte_perm(a, 0x4b000000u, sel)), __uint_as_float(__byte_perm(c, 0x4b000000u, sel))),
                    f2(-8388608.0f, -8388608.0f));
}

__device__ __forceinline__ float2 h2f2(uint32_t w) { return __half22float2(*reinterpret_cast<const __half2*>(&w)); }

template <int G, int D, typename TO, bool RAGGED>
__global__ void __launch_bounds__(MmaGeom<D>::WARPS * 32, kStreamCtasPerSm) attn_stream_kernel(const __grid_constant__ StreamParams sp) {
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "query group");
  using C = StreamCfg<G, D>;
  using GM = MmaGeom<D>;
  constexpr int NW = C::NW;
  constexpr int KS = D / 16;  // k-steps of S^T = K . Q^T, and m-tiles of O^T
  constexpr int CH = D / 4;   // channels of a record's K row that lane (g, t) holds
  constexpr int NS = C::STAGES;
  const AttnParams& p = sp.p;
  extern __shared__ unsigned char smem_raw[];
  __shared__ int sh_bad, sh_last, sh_total, sh_lo[2];
  __shared__ int warp_sums[32];
  __shared__ uint64_t fold_bar;  // the last CTA's bulk copy of the head's partials
  unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  unsigned char* ring = smem;
  float* park = reinterpret_cast<float*>(smem + C::RING);
  int* list = reinterpret_cast<int*>(smem + C::RING + C::PARK);
  uint64_t* bars_all = reinterpret_cast<uint64_t*>(smem + C::RING + C::PARK + C::LIST);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // The CTA's row: j (query group, lists, bitmap, outputs, counter), its KV head hj in the pool and
  // the records, the CTA's index ci among the row's P, the row's first partial pbase, the fill of its
  // current block. A single sequence (RAGGED false) has them from the grid and the parameters; ragged
  // rows from the schedule, kept in shared memory and read where used, so that none stays in a
  // register across the streaming loop.
  __shared__ int sh_rp[6];  // j, ci, P, pbase, hj, last_fill
  auto rp = [&](int i) -> int {
    if constexpr (RAGGED) return *reinterpret_cast<volatile int*>(&sh_rp[i]);
    switch (i) {
      case 0: case 4: return (int)blockIdx.y;
      case 1: return (int)blockIdx.x;
      case 2: return sp.per_head;
      case 3: return (int)blockIdx.y * sp.per_head;
      default: return p.seg[0].last_fill;
    }
  };
  uint64_t* bars = bars_all + warp * NS;
  if (threadIdx.x == 0) {
    sh_bad = 0;
    mbar_init(&fold_bar, 1);
    if constexpr (RAGGED) {
      const int4 e = sp.sched[blockIdx.x];
      sh_rp[0] = e.x, sh_rp[1] = e.y, sh_rp[2] = e.z, sh_rp[3] = e.w, sh_rp[4] = e.x % sp.heads;
      sh_rp[5] = sp.row_info[e.x].y;
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }

  pdl_wait();  // the lists, the bitmap and the workspace are the predecessor's to finish with
  pdl_release();
  if constexpr (RAGGED) __syncthreads();  // sh_rp
  const int j = rp(0);
  // ---- set-up: counts, this CTA's item range, its list of storage rows ----
  // A list segment's count is its length; a range's is a popcount over the bitmap. In the common
  // case (segment 0 a list, segment 1 a range of at most kSetupWords words per thread) the list's
  // loads are issued first and the range is listed in one pass over the bitmap while they fly.
  constexpr int kSetupWords = 1;
  const Seg& S0 = p.seg[0];
  const Seg& S1 = p.seg[1];
  // The row's item counts (list length, range blocks) and the fill of its current block.
  int n_seg0 = S0.n_items, n_seg1 = p.n_segs > 1 ? S1.n_items : 0;  // the row's list items and range blocks
  // A range block's record row: the block itself, or its entry in the sequence's block table.
  const int32_t* table = nullptr;
  if constexpr (RAGGED) {
    const int4 ri = sp.row_info[j];
    n_seg0 = ri.x, n_seg1 = ri.z;
    table = sp.table + (int64_t)(j / sp.heads) * sp.table_stride;
  }
  const bool fast = p.n_segs == 2 && S0.kind == SEG_LIST && S1.kind != SEG_LIST &&
                    (n_seg1 <= 0 || (S1.first_block + n_seg1 - 1) / 32 - S1.first_block / 32 < kSetupWords * C::THREADS);
  int64_t cnt0 = 0, cnt1 = 0, la0 = 0, lb0 = 0, la1 = 0, lb1 = 0;
  int n_a = 0, n_b = 0;
  if (fast) {
    cnt0 = n_seg0;
    la0 = cnt0 * rp(1) / rp(2);
    lb0 = cnt0 * (rp(1) + 1) / rp(2);
    n_a = (int)(lb0 - la0);
    // The list's first C::THREADS items: id, then slot row (dependent loads, in flight during the scan).
    int hot_row = -1;
    const int64_t hit = la0 + threadIdx.x;
    if (hit < lb0) {
      const int blk = __ldg(S0.blocks + (int64_t)j * S0.n_list + hit);
      int64_t row = blk < 0 ? -1 : (S0.slot_of != nullptr ? __ldg(S0.slot_of + (int64_t)j * S0.slot_stride + blk) : blk);
      hot_row = row >= S0.n_rows ? -1 : (int)row;
    }
    // The range: this thread's kSetupWords consecutive words, their counts, a block-wide scan.
    uint32_t bits[kSetupWords];
    int mine = 0;
    const int w0 = S1.first_block / 32 + threadIdx.x * kSetupWords;
#pragma unroll
    for (int k = 0; k < kSetupWords; ++k) {
      bits[k] = n_seg1 > 0 ? range_word_bits(S1, n_seg1, j, w0 + k) : 0u;
      mine += __popc(bits[k]);
    }
    const int before = block_excl_scan(mine, warp_sums, &sh_total);
    cnt1 = sh_total;
    la1 = cnt1 * rp(1) / rp(2);
    lb1 = cnt1 * (rp(1) + 1) / rp(2);
    n_b = (int)(lb1 - la1);
    if (n_a + n_b <= kStreamListCap) {
      // The range's items in [la1, lb1) lie in a contiguous run of words. Each word's bits and first
      // ordinal go to shared memory (the ring, idle until streaming starts); then warp w lists the
      // run's words w, w + NW, ..., one lane per bit (its ordinal: the word's plus the set bits below it).
      static_assert(kSetupWords == 1, "one word per thread in the warp-cooperative listing");
      uint32_t* wbits = reinterpret_cast<uint32_t*>(ring);
      int* word_ord = reinterpret_cast<int*>(ring) + C::THREADS;
      __shared__ int sh_wrun[2];
      if (threadIdx.x == 0) {
        sh_wrun[0] = C::THREADS;
        sh_wrun[1] = -1;
      }
      wbits[threadIdx.x] = bits[0];
      word_ord[threadIdx.x] = before;
      __syncthreads();
      if (before < lb1 && before + __popc(bits[0]) > la1) {  // this word holds items of the slice
        atomicMin(&sh_wrun[0], (int)threadIdx.x);
        atomicMax(&sh_wrun[1], (int)threadIdx.x);
      }
      __syncthreads();
      const uint32_t below = (1u << lane) - 1u;
      for (int t = sh_wrun[0] + warp; t <= sh_wrun[1]; t += NW) {
        const uint32_t b = wbits[t];
        if (!((b >> lane) & 1u)) continue;
        const int64_t ord = word_ord[t] + __popc(b & below);
        if (ord < la1 || ord >= lb1) continue;
        const int blk = 32 * (S1.first_block / 32 + t) + lane;
        int rrow = blk;
        if (table != nullptr) {  // a table entry outside the store lists nothing
          rrow = __ldg(table + blk);
          if (rrow < 0 || rrow >= S1.n_rows) rrow = -1;
        }
        list[n_a + (ord - la1)] = S1.kind == SEG_RANGE_REC ? rrow : (rrow < S1.n_rows ? rrow : -1);
      }
      // The ring's words were written through the generic proxy; the tile copies that refill it go
      // through the async proxy after the barrier that ends the set-up.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      if (hit < lb0) list[threadIdx.x] = hot_row;
      for (int64_t it = lb0 > la0 + C::THREADS ? la0 + C::THREADS + threadIdx.x : lb0; it < lb0; it += blockDim.x) {
        const int blk = __ldg(S0.blocks + (int64_t)j * S0.n_list + it);
        int64_t row = blk < 0 ? -1 : (S0.slot_of != nullptr ? __ldg(S0.slot_of + (int64_t)j * S0.slot_stride + blk) : blk);
        list[it - la0] = row >= S0.n_rows ? -1 : (int)row;
      }
    }
  } else {
    for (int s = 0; s < p.n_segs; ++s) {
      const Seg& S = p.seg[s];
      int64_t c = (s == 0 ? n_seg0 : n_seg1);
      if (S.kind != SEG_LIST && (s == 0 ? n_seg0 : n_seg1) > 0) {
        const int w0 = S.first_block / 32, w1 = (S.first_block + (s == 0 ? n_seg0 : n_seg1) - 1) / 32;
        int mine = 0;
        for (int w = w0 + threadIdx.x; w <= w1; w += blockDim.x) mine += __popc(range_word_bits(S, (s == 0 ? n_seg0 : n_seg1), j, w));
        block_excl_scan(mine, warp_sums, &sh_total);
        c = sh_total;
      }
      if (s == 0) cnt0 = c; else cnt1 = c;
    }
    // This CTA's share of each segment (ordinals [la, lb)); the list holds segment 0's items first.
    la0 = cnt0 * rp(1) / rp(2);
    lb0 = cnt0 * (rp(1) + 1) / rp(2);
    la1 = cnt1 * rp(1) / rp(2);
    lb1 = cnt1 * (rp(1) + 1) / rp(2);
    n_a = (int)(lb0 - la0);
    n_b = (int)(lb1 - la1);
    if (n_a + n_b <= kStreamListCap) {
      for (int s = 0; s < p.n_segs; ++s) {
        const Seg& S = p.seg[s];
        const int64_t la = s == 0 ? la0 : la1, lb = s == 0 ? lb0 : lb1;
        int* dst = list + (s == 0 ? 0 : n_a);
        if (la >= lb) continue;
        if (S.kind == SEG_LIST) {
          for (int64_t it = la + threadIdx.x; it < lb; it += blockDim.x) {
            const int blk = __ldg(S.blocks + (int64_t)j * S.n_list + it);
            int64_t row = blk < 0 ? -1 : (S.slot_of != nullptr ? __ldg(S.slot_of + (int64_t)j * S.slot_stride + blk) : blk);
            if (row >= S.n_rows) row = -1;  // outside the tensor maps: nothing to load
            dst[it - la] = (int)row;
          }
        } else {
          // Ordinal of each word's first kept block by a block-wide scan, chunk by chunk.
          const int w0 = S.first_block / 32, w1 = (S.first_block + (s == 0 ? n_seg0 : n_seg1) - 1) / 32;
          int64_t run = 0;
          for (int c0 = w0; c0 <= w1 && run < lb; c0 += blockDim.x) {
            const int w = c0 + threadIdx.x;
            uint32_t bits = w <= w1 ? range_word_bits(S, (s == 0 ? n_seg0 : n_seg1), j, w) : 0u;
            const int before = block_excl_scan(__popc(bits), warp_sums, &sh_total);
            int64_t ord = run + before;
            while (bits != 0u && ord < lb) {
              const int b = __ffs(bits) - 1;
              bits &= bits - 1u;
              if (ord >= la) {
                int rrow = 32 * w + b;
                if (table != nullptr) {
                  rrow = __ldg(table + rrow);
                  if (rrow < 0 || rrow >= S.n_rows) rrow = -1;
                }
                dst[ord - la] = S.kind == SEG_RANGE_REC ? rrow : (rrow < S.n_rows ? rrow : -1);
              }
              ++ord;
            }
            run += sh_total;
          }
        }
      }
    }
  }
  if (threadIdx.x == 0) {
    sh_lo[0] = (int)la0;
    sh_lo[1] = (int)la1;
    if (n_a + n_b > kStreamListCap) {  // the host sizes P so that this cannot happen
      sh_bad = 2;
      record_status(LKV_DEV_LIST_OVERFLOW);
    }
  }
  __syncthreads();

  // ---- streaming: this warp's share of the list ----
  // Its items: list[ha, ha + hn) of segment 0, then list[n_a + ca, n_a + ca + cn) of segment 1. The
  // split is fixed, so a call's result does not depend on timing.
  const int ha = n_a * warp / NW, hn = sh_bad ? 0 : n_a * (warp + 1) / NW - ha;
  const int ca = n_b * warp / NW, cn = sh_bad ? 0 : n_b * (warp + 1) / NW - ca;
  const int n_mine = hn + cn;
  auto list_index = [&](int k) { return k < hn ? ha + k : n_a + ca + (k - hn); };

  const int g = lane >> 2, t = lane & 3;
  uint32_t bq[KS][2], bqp[KS][2];
  {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(static_cast<const __nv_bfloat16*>(p.q) + ((int64_t)j * G + (g < G ? g : 0)) * D);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      bq[ks][0] = g < G ? q[(16 * ks + 2 * t) / 2] : 0u;
      bq[ks][1] = g < G ? q[(16 * ks + 2 * t + 8) / 2] : 0u;
      bqp[ks][0] = g < G ? q[(CH * t + 4 * ks) / 2] : 0u;
      bqp[ks][1] = g < G ? q[(CH * t + 4 * ks + 2) / 2] : 0u;
    }
  }
  uint32_t koff[4], voff[4];
  {
    const int i = lane >> 3, r7 = lane & 7;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      koff[x] = swz(r7 + 8 * (i & 1), 2 * x + (i >> 1));
      voff[x] = swz(r7 + 8 * (i >> 1), 2 * x + (i & 1));
    }
  }
  unsigned char* stage0 = ring + warp * NS * C::STAGE;
  // Per set: whether its items are int8 records (else bf16 tile pairs through the tensor maps).
  const bool rec0 = p.seg[0].kind == SEG_RANGE_REC, rec1 = p.n_segs > 1 && p.seg[1].kind == SEG_RANGE_REC;
  // The warp's item holding the current block (the last listed block, `last_fill` live tokens), if any.
  const int fill_k = (p.seg[0].kind == SEG_LIST && lb0 == n_seg0 && hn > 0 && ha + hn == n_a) ? hn - 1 : -1;
  const uint64_t stream_pol = l2_evict_first_policy();  // every item is read once
  // Lane 0 fills stage s with the warp's k-th item (or arrives for a padding item).
  auto issue = [&](int k, int s) {
    if (lane != 0) return;
    const int set = k < hn ? 0 : 1;
    const int row = list[list_index(k)];
    if (row < 0) {
      mbar_arrive(&bars[s]);
      return;
    }
    unsigned char* dst = stage0 + s * C::STAGE;
    if (set ? rec1 : rec0) {
      const Seg& S = p.seg[set];
      mbar_arrive_expect_tx(&bars[s], (uint32_t)GM::REC);
      tma_load_1d_hint(dst, S.records + ((int64_t)row * p.h + rp(4)) * S.width, (uint32_t)GM::REC, &bars[s], stream_pol);
    } else {
      mbar_arrive_expect_tx(&bars[s], (uint32_t)GM::HOT);
      const int hm = sp.head_major[set];
      const int hj = rp(4);
      const int c2 = hm ? hj : row, c3 = hm ? row : hj;
#pragma unroll
      for (int hf = 0; hf < GM::HALVES; ++hf) {  // channels 64 hf .. 64 hf + 63 of the K and V tiles
        tma_load_4d_hint(smem_u32(dst + 2048 * hf), &sp.tk[set], 64 * hf, 0, c2, c3, &bars[s], stream_pol);
        tma_load_4d_hint(smem_u32(dst + GM::TILE + 2048 * hf), &sp.tv[set], 64 * hf, 0, c2, c3, &bars[s], stream_pol);
      }
    }
  };
  int n_issued = 0;
#pragma unroll
  for (int s = 0; s < NS; ++s)
    if (s < n_mine) {
      issue(s, s);
      ++n_issued;
    }

  // Online-softmax state. The running maxima m (log2 domain) start at a finite -1e30 so that no
  // score needs a test for an empty state: the first finite score always rescales (by 2^-huge = 0),
  // and a masked score (-inf) gives 2^-inf = 0. thr = (m + kLazy) / scale_log2 is the raw-score
  // threshold of the lazy rescaling (scale_log2 > 0), nm = -m.
  constexpr float kNoMax = -1e30f;
  const float sl2 = p.scale_log2, inv_sl2 = 1.0f / p.scale_log2;
  float o[KS][4];
  float m0, m1, nm0, nm1, thr0, thr1, l0, l1;
  auto reset_state = [&]() {
    m0 = m1 = kNoMax;
    nm0 = nm1 = -kNoMax;
    thr0 = thr1 = (kNoMax + kLazy) * inv_sl2;
    l0 = l1 = 0.0f;
#pragma unroll
    for (int a = 0; a < KS; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) o[a][b] = 0.0f;
  };
  reset_state();
  const int r0 = 2 * t, r1 = 2 * t + 1;
  // Parks the state of `set` in this warp's slot for it (channels back in natural order). A row that
  // saw no key is parked as (m = -inf, l = 0).
  auto park_state = [&](int set) {
    float la = l0, lb = l1;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      la += __shfl_xor_sync(0xffffffffu, la, off);
      lb += __shfl_xor_sync(0xffffffffu, lb, off);
    }
    float* slot = park + (warp * 2 + set) * C::SLOT;
    const bool perm = set ? rec1 : rec0;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      const int c0 = perm ? (D / 8) * g + 2 * mt : 16 * mt + g;
      const int c1 = perm ? (D / 8) * g + 2 * mt + 1 : 16 * mt + g + 8;
      if (r0 < G) {
        slot[r0 * D + c0] = o[mt][0];
        slot[r0 * D + c1] = o[mt][2];
      }
      if (r1 < G) {
        slot[r1 * D + c0] = o[mt][1];
        slot[r1 * D + c1] = o[mt][3];
      }
    }
    if (g == 0) {
      if (r0 < G) {
        slot[G * D + r0] = la > 0.0f ? m0 : -INFINITY;
        slot[G * D + G + r0] = la;
      }
      if (r1 < G) {
        slot[G * D + r1] = lb > 0.0f ? m1 : -INFINITY;
        slot[G * D + G + r1] = lb;
      }
    }
  };

  // Lane offsets inside a stage (bytes): record K codes of tokens g and g + 8 at channels CH t..,
  // V codes of tokens 2t, 2t+1, 2t+8, 2t+9 at channels (D/8)g.., V scales / zeros of those tokens,
  // and the float32 K scales / zeros of channels CH t.. in the stage's tail.
  const int ok0 = g * D + CH * t, ok8 = (g + 8) * D + CH * t;
  const int ov0 = 16 * D + (2 * t) * D + (D / 8) * g, ov1 = ov0 + D, ov8 = ov0 + 8 * D, ov9 = ov0 + 9 * D;
  const int ovs = GM::OFF_VS + 4 * t, ovz = GM::OFF_VZ + 4 * t;

  // One item in the stage at `st`: scores, softmax update and the O contraction. REC: an int8
  // record dequantised in registers (permuted channels); else a bf16 tile pair read by ldmatrix.
  auto item = [&](auto rec_tag, unsigned char* st, bool masked) {
    constexpr bool REC = decltype(rec_tag)::value;
    const uint32_t st32 = smem_u32(st);
    float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if constexpr (REC) {
      // The record's 64 K scales and 64 K zeros (float16) become float32 once per warp, in the
      // stage's unused tail; lane (g, t) then reads those of its channels CH t .. CH t + CH - 1.
      float* kf = reinterpret_cast<float*>(st + GM::KF);
      if constexpr (D == 64) {
        const uint2 hw = *reinterpret_cast<const uint2*>(st + GM::OFF_KS + 8 * lane);
        const float2 f01 = h2f2(hw.x), f23 = h2f2(hw.y);
        *reinterpret_cast<float4*>(kf + 4 * lane) = make_float4(f01.x, f01.y, f23.x, f23.y);
      } else {
        const uint4 hw = *reinterpret_cast<const uint4*>(st + GM::OFF_KS + 16 * lane);
        const float2 f01 = h2f2(hw.x), f23 = h2f2(hw.y), f45 = h2f2(hw.z), f67 = h2f2(hw.w);
        *reinterpret_cast<float4*>(kf + 8 * lane) = make_float4(f01.x, f01.y, f23.x, f23.y);
        *reinterpret_cast<float4*>(kf + 8 * lane + 4) = make_float4(f45.x, f45.y, f67.x, f67.y);
      }
      uint32_t wg0[KS], wg8[KS];
#pragma unroll
      for (int v = 0; v < KS / 4; ++v) {
        const uint4 cg0 = *reinterpret_cast<const uint4*>(st + ok0 + 16 * v);
        const uint4 cg8 = *reinterpret_cast<const uint4*>(st + ok8 + 16 * v);
        wg0[4 * v] = cg0.x, wg0[4 * v + 1] = cg0.y, wg0[4 * v + 2] = cg0.z, wg0[4 * v + 3] = cg0.w;
        wg8[4 * v] = cg8.x, wg8[4 * v + 1] = cg8.y, wg8[4 * v + 2] = cg8.z, wg8[4 * v + 3] = cg8.w;
      }
      __syncwarp();
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const float4 sc = *reinterpret_cast<const float4*>(kf + CH * t + 4 * ks);
        const float4 zc = *reinterpret_cast<const float4*>(kf + D + CH * t + 4 * ks);
        const float2 s01 = f2(sc.x, sc.y), s23 = f2(sc.z, sc.w), z01 = f2(zc.x, zc.y), z23 = f2(zc.z, zc.w);
        float2 ua, ub, va, vb;
        codes4(wg0[ks], ua, ub);
        codes4(wg8[ks], va, vb);
        const float2 k0 = __ffma2_rn(ua, s01, z01), k1 = __ffma2_rn(va, s01, z01);
        const float2 k2 = __ffma2_rn(ub, s23, z23), k3 = __ffma2_rn(vb, s23, z23);
        const uint32_t a[4] = {pack_bf2(k0.x, k0.y), pack_bf2(k1.x, k1.y), pack_bf2(k2.x, k2.y), pack_bf2(k3.x, k3.y)};
        if (ks & 1)
          mma_bf16(sb, a, bqp[ks][0], bqp[ks][1]);
        else
          mma_bf16(sa, a, bqp[ks][0], bqp[ks][1]);
      }
    } else {
#pragma unroll
      for (int ks = 0; ks < KS; ks += 2) {
        uint32_t a[4], b[4];
        ldsm_x4(st32 + 2048 * (ks >> 2) + koff[ks & 3], a);
        ldsm_x4(st32 + 2048 * ((ks + 1) >> 2) + koff[(ks + 1) & 3], b);
        mma_bf16(sa, a, bq[ks][0], bq[ks][1]);
        mma_bf16(sb, b, bq[ks + 1][0], bq[ks + 1][1]);
      }
    }
    // Raw scores: a0, a1 (token g, rows 2t, 2t+1), a2, a3 (token g + 8).
    float a0 = sa[0] + sb[0], a1 = sa[1] + sb[1], a2 = sa[2] + sb[2], a3 = sa[3] + sb[3];
    if (!REC && masked) {
      const int last_fill = rp(5);
      if (g >= last_fill) a0 = a1 = -INFINITY;
      if (g + 8 >= last_fill) a2 = a3 = -INFINITY;
    }
    // ---- softmax update (log2 domain, lazy rescaling) ----
    if (__any_sync(0xffffffffu, a0 > thr0 || a2 > thr0 || a1 > thr1 || a3 > thr1)) {
      float mb0 = fmaxf(a0, a2) * sl2, mb1 = fmaxf(a1, a3) * sl2;
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mb0 = fmaxf(mb0, __shfl_xor_sync(0xffffffffu, mb0, off));
        mb1 = fmaxf(mb1, __shfl_xor_sync(0xffffffffu, mb1, off));
      }
      if (mb0 > m0 + kLazy) {
        const float alpha = exp2f(m0 - mb0);
        l0 *= alpha;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          o[mt][0] *= alpha;
          o[mt][2] *= alpha;
        }
        m0 = mb0;
        nm0 = -mb0;
        thr0 = (mb0 + kLazy) * inv_sl2;
      }
      if (mb1 > m1 + kLazy) {
        const float alpha = exp2f(m1 - mb1);
        l1 *= alpha;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          o[mt][1] *= alpha;
          o[mt][3] *= alpha;
        }
        m1 = mb1;
        nm1 = -mb1;
        thr1 = (mb1 + kLazy) * inv_sl2;
      }
    }
    const float p0 = ex2(fmaf(a0, sl2, nm0)), p2 = ex2(fmaf(a2, sl2, nm0));
    const float p1 = ex2(fmaf(a1, sl2, nm1)), p3 = ex2(fmaf(a3, sl2, nm1));
    l0 += p0 + p2;
    l1 += p1 + p3;
    uint32_t h01, md01, s01, h23, md23, s23;
    split3(p0, p1, h01, md01, s01);
    split3(p2, p3, h23, md23, s23);
    const uint32_t bh0 = movtrans(h01), bh1 = movtrans(h23);
    const uint32_t bm0 = movtrans(md01), bm1 = movtrans(md23);
    const uint32_t bl0 = movtrans(s01), bl1 = movtrans(s23);

    // ---- O^T += V^T . P^T ----
    if constexpr (REC) {
      // Lane g's D / 8 channels of tokens 2t, 2t+1, 2t+8, 2t+9, as D / 32 words each.
      uint32_t e0[D / 32], e1[D / 32], e2[D / 32], e3[D / 32];
      if constexpr (D == 64) {
        const uint2 c0 = *reinterpret_cast<const uint2*>(st + ov0);
        const uint2 c1 = *reinterpret_cast<const uint2*>(st + ov1);
        const uint2 c2 = *reinterpret_cast<const uint2*>(st + ov8);
        const uint2 c3 = *reinterpret_cast<const uint2*>(st + ov9);
        e0[0] = c0.x ^ 0x80808080u, e0[1] = c0.y ^ 0x80808080u, e1[0] = c1.x ^ 0x80808080u, e1[1] = c1.y ^ 0x80808080u;
        e2[0] = c2.x ^ 0x80808080u, e2[1] = c2.y ^ 0x80808080u, e3[0] = c3.x ^ 0x80808080u, e3[1] = c3.y ^ 0x80808080u;
      } else {
        const uint4 c0 = *reinterpret_cast<const uint4*>(st + ov0);
        const uint4 c1 = *reinterpret_cast<const uint4*>(st + ov1);
        const uint4 c2 = *reinterpret_cast<const uint4*>(st + ov8);
        const uint4 c3 = *reinterpret_cast<const uint4*>(st + ov9);
        e0[0] = c0.x ^ 0x80808080u, e0[1] = c0.y ^ 0x80808080u, e0[2] = c0.z ^ 0x80808080u, e0[3] = c0.w ^ 0x80808080u;
        e1[0] = c1.x ^ 0x80808080u, e1[1] = c1.y ^ 0x80808080u, e1[2] = c1.z ^ 0x80808080u, e1[3] = c1.w ^ 0x80808080u;
        e2[0] = c2.x ^ 0x80808080u, e2[1] = c2.y ^ 0x80808080u, e2[2] = c2.z ^ 0x80808080u, e2[3] = c2.w ^ 0x80808080u;
        e3[0] = c3.x ^ 0x80808080u, e3[1] = c3.y ^ 0x80808080u, e3[2] = c3.z ^ 0x80808080u, e3[3] = c3.w ^ 0x80808080u;
      }
      const float2 vs01 = h2f2(*reinterpret_cast<const uint32_t*>(st + ovs));
      const float2 vs89 = h2f2(*reinterpret_cast<const uint32_t*>(st + ovs + 16));
      const float2 vz01 = h2f2(*reinterpret_cast<const uint32_t*>(st + ovz));
      const float2 vz89 = h2f2(*reinterpret_cast<const uint32_t*>(st + ovz + 16));
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
        const int wi = mt >> 1;
        const uint32_t sel0 = 0x7650u + 2 * (mt & 1), sel1 = sel0 + 1;
        const float2 v00 = __ffma2_rn(code_pair(e0[wi], e1[wi], sel0), vs01, vz01);  // channel (D/8)g+2mt, tokens 2t, 2t+1
        const float2 v01 = __ffma2_rn(code_pair(e0[wi], e1[wi], sel1), vs01, vz01);  // channel (D/8)g+2mt+1
        const float2 v80 = __ffma2_rn(code_pair(e2[wi], e3[wi], sel0), vs89, vz89);  // tokens 2t+8, 2t+9
        const float2 v81 = __ffma2_rn(code_pair(e2[wi], e3[wi], sel1), vs89, vz89);
        const uint32_t a[4] = {pack_bf2(v00.x, v00.y), pack_bf2(v01.x, v01.y), pack_bf2(v80.x, v80.y), pack_bf2(v81.x, v81.y)};
        mma_bf16(o[mt], a, bl0, bl1);
        mma_bf16(o[mt], a, bm0, bm1);
        mma_bf16(o[mt], a, bh0, bh1);
      }
    } else {
      const uint32_t vt = st32 + GM::TILE;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
        uint32_t a[4];
        ldsm_x4_t(vt + 2048 * (mt >> 2) + voff[mt & 3], a);
        mma_bf16(o[mt], a, bl0, bl1);
        mma_bf16(o[mt], a, bm0, bm1);
        mma_bf16(o[mt], a, bh0, bh1);
      }
    }
  };

  // The ring: item k sits in stage k % NS; the loop is unrolled over the stages so that every
  // stage address and barrier is a constant, and the n-th use of a stage waits on parity n & 1.
  int n_done = 0;
  bool ok = true;
  const bool parked_mid = hn > 0 && n_mine > hn;
#pragma unroll 1
  for (int base = 0; base < n_mine && ok; base += NS) {
    const uint32_t par = (uint32_t)(base / NS) & 1u;
#pragma unroll
    for (int u = 0; u < NS; ++u) {
      const int k = base + u;
      if (k >= n_mine) break;
      if (!__all_sync(0xffffffffu, mbar_wait(&bars[u], par))) {
        ok = false;
        break;
      }
      ++n_done;
      if (k == hn && hn > 0) {  // segment 0 done: park its state, start segment 1's
        park_state(0);
        reset_state();
      }
      if (list[list_index(k)] >= 0) {
        unsigned char* st = stage0 + u * C::STAGE;
        if (k < hn ? rec0 : rec1)
          item(std::true_type{}, st, false);
        else
          item(std::false_type{}, st, k == fill_k);
      }
      __syncwarp();  // every lane is done with the stage before it is refilled
      if (k + NS < n_mine) {
        issue(k + NS, u);
        ++n_issued;
      }
    }
  }
  const int cur_set = n_mine == 0 ? -1 : (n_mine > hn ? 1 : 0);
  // After a timed-out wait, wait (bounded) for the copies still in flight: items n_done .. n_issued-1.
  if (!ok) {
    for (int k = n_done; k < n_issued; ++k) {
      const int u = k % NS;
      if (!__all_sync(0xffffffffu, mbar_wait(&bars[u], (uint32_t)(k / NS) & 1u))) break;
    }
    if (lane == 0) atomicExch(&sh_bad, 1);
  }
  if (cur_set >= 0) park_state(cur_set);
  // A set this warp holds no state of: empty (m = -inf).
  if (lane < G) {
    if (cur_set != 0 && !parked_mid) park[(warp * 2 + 0) * C::SLOT + G * D + lane] = -INFINITY;
    if (cur_set != 1) park[(warp * 2 + 1) * C::SLOT + G * D + lane] = -INFINITY;
  }
  __syncthreads();

  // ---- fold the warps' parked states into this CTA's partials ----
  // Partials live set-major per row: set s of CTA ci at part[(2 * pbase + s * P + ci) * PART], so a
  // head's set-0 partials are contiguous. When only the merged output is wanted (no per-set
  // outputs), the CTA folds both sets into ONE partial (set 0): per row, lane l of one warp holds
  // the maximum of warp (l % NW)'s state of set (l / NW); the lanes agree on the maximum M and the
  // sum L by shuffles, the weights 2^(m - M) go to shared memory, and every thread folds output
  // elements with them. Otherwise each set is folded on its own, one partial per set.
  const int64_t part_stride = C::PART;
  const int ci = rp(1), P = rp(2), pbase = rp(3);
  const bool merge_sets = sp.seg_out == nullptr;
  const int n_folds = merge_sets ? 1 : 2;  // partials this CTA writes
  const int per_fold = merge_sets ? 2 * NW : NW;  // parked states per partial
  auto mine = [&](int set) { return sp.part + ((int64_t)2 * pbase + (int64_t)set * P + ci) * part_stride; };
  __shared__ float fold_w[2 * 8][2 * NW > 32 ? 2 * NW : 32];  // [(partial, row)][state] weights
  static_assert(2 * NW <= 32, "one lane per parked state");
  for (int pr = warp; pr < n_folds * G; pr += NW) {
    const int f_set = pr / G, r = pr % G;
    // lane -> (warp, set) of the parked state it weighs
    const int sw = merge_sets ? lane % NW : lane, sset = merge_sets ? lane / NW : f_set;
    const bool live = lane < per_fold && !sh_bad;
    const float* sl = park + (sw * 2 + sset) * C::SLOT;
    const float mw = live ? sl[G * D + r] : -INFINITY;
    float M = mw;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    const float f = (M == -INFINITY || mw == -INFINITY) ? 0.0f : exp2f(mw - M);
    float L = f != 0.0f ? f * sl[G * D + G + r] : 0.0f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    if (lane < per_fold) fold_w[pr][lane] = f;
    if (lane == 0) {
      mine(f_set)[G * D + r] = M;
      mine(f_set)[G * D + G + r] = L;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n_folds * G * D; e += blockDim.x) {
    const int f_set = e / (G * D), r = (e / D) % G, c = e % D;
    const float* wr = fold_w[f_set * G + r];
    float O = 0.0f;
#pragma unroll
    for (int w = 0; w < per_fold; ++w) {
      const int sw = merge_sets ? w % NW : w, sset = merge_sets ? w / NW : f_set;
      if (wr[w] != 0.0f) O = fmaf(park[(sw * 2 + sset) * C::SLOT + r * D + c], wr[w], O);  // a zero weight: the slot may be unset
    }
    mine(f_set)[r * D + c] = O;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) sh_last = atomicAdd(&sp.counters[j], 1u) == (unsigned)(P - 1);
  __syncthreads();
  if (!sh_last) return;
  __threadfence();

  // ---- the head's last CTA: fold its P partials per set into the outputs ----
  // The head's partials of each folded set are contiguous in the workspace: one bulk copy brings
  // them into the idle ring (when they fit); per (set, row) a warp finds the maximum, the weights
  // and the sum by shuffles (lanes over the partials); then every thread folds one output element.
  const float* hp = sp.part + (int64_t)2 * pbase * part_stride;  // set s, partial k at hp + (s * P + k) * PART
  const int nset = merge_sets ? 1 : p.n_segs;
  const size_t head_bytes = (size_t)nset * P * C::PART * sizeof(float);
  const bool bulk = head_bytes <= (size_t)C::RING;
  bool got = true;
  if (bulk && threadIdx.x == 0) {
    asm volatile("fence.proxy.async;" ::: "memory");  // the partials (generic stores of other CTAs) before the bulk reads
    mbar_arrive_expect_tx(&fold_bar, (uint32_t)head_bytes);
    for (size_t off = 0; off < head_bytes; off += 32768) {
      const uint32_t n = (uint32_t)(head_bytes - off < 32768 ? head_bytes - off : 32768);
      tma_load_1d(ring + off, reinterpret_cast<const unsigned char*>(hp) + off, n, &fold_bar);
    }
  }
  if (bulk) got = __syncthreads_and(mbar_wait(&fold_bar, 0));
  const float* parts = bulk ? reinterpret_cast<const float*>(ring) : hp;
  auto part_at = [&](int set, int k) { return parts + ((int64_t)set * P + k) * part_stride; };
  // The weights of up to 32 partials per (set, row) live in fold_w; more partials go through the
  // workspace one pass per row (P <= 32 covers kStreamCtasPerSm x SMs / h for h >= 5 on B200).
  __shared__ float setM[2 * 8], setL[2 * 8];
  if (P <= 32 && got) {
    for (int pr = warp; pr < nset * G; pr += NW) {
      const int set = pr / G, r = pr % G;
      const float mk = lane < P ? (bulk ? part_at(set, lane)[G * D + r] : __ldcg(part_at(set, lane) + G * D + r)) : -INFINITY;
      float M = mk;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      const float f = (M == -INFINITY || mk == -INFINITY) ? 0.0f : exp2f(mk - M);
      float L = 0.0f;
      if (f != 0.0f) L = f * (bulk ? part_at(set, lane)[G * D + G + r] : __ldcg(part_at(set, lane) + G * D + G + r));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      if (lane < P) fold_w[pr][lane] = f;
      if (lane == 0) {
        setM[pr] = M;
        setL[pr] = L;
      }
    }
    __syncthreads();
  }
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int r = e / D, c = e % D;
    float O0 = 0.0f, O1 = 0.0f, M0 = -INFINITY, M1 = -INFINITY, L0 = 0.0f, L1 = 0.0f;
#pragma unroll
    for (int set = 0; set < 2; ++set) {
      if (set >= nset || !got) break;
      float O = 0.0f, M = -INFINITY, L = 0.0f;
      if (P <= 32) {
        const float* wr = fold_w[set * G + r];
#pragma unroll 4
        for (int k = 0; k < P; ++k) {
          const float* pk = part_at(set, k) + r * D + c;
          O = fmaf(bulk ? *pk : __ldcg(pk), wr[k], O);
        }
        M = setM[set * G + r];
        L = setL[set * G + r];
      } else {  // more partials than a warp's lanes: straight from the workspace
        for (int k = 0; k < P; ++k) M = fmaxf(M, __ldcg(hp + ((int64_t)set * P + k) * part_stride + G * D + r));
        if (M != -INFINITY)
          for (int k = 0; k < P; ++k) {
            const float* pk = hp + ((int64_t)set * P + k) * part_stride;
            const float mk = __ldcg(pk + G * D + r);
            if (mk == -INFINITY) continue;
            const float f = exp2f(mk - M);
            O = fmaf(__ldcg(pk + r * D + c), f, O);
            L = fmaf(__ldcg(pk + G * D + G + r), f, L);
          }
      }
      if (set == 0) {
        O0 = O; M0 = M; L0 = L;
      } else {
        O1 = O; M1 = M; L1 = L;
      }
    }
    const int64_t row = (int64_t)j * G + r;
    if (sp.seg_out != nullptr) {
#pragma unroll
      for (int set = 0; set < 2; ++set) {
        if (set >= nset) break;
        const float Os = set == 0 ? O0 : O1, Ms = set == 0 ? M0 : M1, Ls = set == 0 ? L0 : L1;
        const bool empty = !(Ls > 0.0f);
        sp.seg_out[(int64_t)set * p.hq * D + row * D + c] = empty ? 0.0f : Os / Ls;
        if (c == 0 && sp.seg_lse != nullptr) sp.seg_lse[(int64_t)set * p.hq + row] = empty ? -INFINITY : (Ms + log2f(Ls)) * kLn2;
      }
    }
    if (sp.out != nullptr || sp.lse != nullptr) {
      const float M = fmaxf(M0, M1);
      float O = 0.0f, L = 0.0f;
      if (M != -INFINITY) {
        if (M0 != -INFINITY) {
          const float f = exp2f(M0 - M);
          O = fmaf(O0, f, O);
          L = fmaf(L0, f, L);
        }
        if (M1 != -INFINITY) {
          const float f = exp2f(M1 - M);
          O = fmaf(O1, f, O);
          L = fmaf(L1, f, L);
        }
      }
      const bool empty = !(L > 0.0f);
      if (sp.out != nullptr) static_cast<TO*>(sp.out)[row * D + c] = from_f32<TO>(empty ? 0.0f : O / L);
      if (c == 0 && sp.lse != nullptr) sp.lse[row] = empty ? -INFINITY : (M + log2f(L)) * kLn2;
    }
  }
  if (threadIdx.x == 0) sp.counters[j] = 0u;  // ready for the next call
}

// ============================================================================================
// combine and merge
// ============================================================================================

// Fold the splits of each segment (segment 0: [0, n0), segment 1: [n0, n0 + n1)) of each (head,
// query row) into per-segment (out, lse) and their merge. One CTA per (head, row): the threads split
// the channels x the splits so the partials are read with independent loads. Outputs may be null.
constexpr int kCombineThreads = 1024;
constexpr int kCombineMaxSplits = 1024;  // (m, l) of up to this many splits are staged in shared memory

// One CTA per (KV head, query row): the splits' (m, l) are staged in shared memory, then
// kCombineThreads / D split lanes per channel accumulate the rescaled partial outputs, so every
// thread has only a few independent global loads in flight.
template <typename TO, int G, int D>
__global__ void __launch_bounds__(kCombineThreads) attn_combine_kernel(const float* __restrict__ part, int n0, int n1, TO* __restrict__ out,
                                                                       float* __restrict__ lse, float* __restrict__ seg_out,
                                                                       float* __restrict__ seg_lse, int hq) {
  constexpr int KS = kCombineThreads / D;  // split lanes per channel
  __shared__ float sm_m[kCombineMaxSplits], sm_l[kCombineMaxSplits];
  __shared__ float red_m[kCombineThreads / 32];
  __shared__ float acc_o[KS][D];
  __shared__ float acc_l[KS];
  __shared__ float seg_M[2], seg_L[2];
  __shared__ float seg_O[2][D];
  const int j = blockIdx.x, r = blockIdx.y;
  const int nt = n0 + n1;
  const int c = threadIdx.x % D, k = threadIdx.x / D;
  const int64_t stride = G * (D + 2);
  const float* base = part + (int64_t)j * nt * stride;
  const bool staged = nt <= kCombineMaxSplits;
  if (staged)
    for (int sp = threadIdx.x; sp < nt; sp += kCombineThreads) {
      sm_m[sp] = base[sp * stride + r];
      sm_l[sp] = base[sp * stride + G + r];
    }
  __syncthreads();
#pragma unroll
  for (int sgi = 0; sgi < 2; ++sgi) {
    const int a = sgi == 0 ? 0 : n0, b = sgi == 0 ? n0 : nt;
    float mloc = -INFINITY;
    for (int sp = a + threadIdx.x; sp < b; sp += kCombineThreads) mloc = fmaxf(mloc, staged ? sm_m[sp] : base[sp * stride + r]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, off));
    if ((threadIdx.x & 31) == 0) red_m[threadIdx.x >> 5] = mloc;
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCombineThreads / 32; ++w) M = fmaxf(M, red_m[w]);
    float O = 0.0f, L = 0.0f;
    if (M != -INFINITY) {
#pragma unroll 4
      for (int sp = a + k; sp < b; sp += KS) {
        const float* ps = base + sp * stride;
        const float ms = staged ? sm_m[sp] : ps[r];
        const float f = ms == -INFINITY ? 0.0f : exp2f(ms - M);
        O = fmaf(ps[2 * G + r * D + c], f, O);
        L = fmaf(staged ? sm_l[sp] : ps[G + r], f, L);
      }
    }
    acc_o[k][c] = O;
    if (c == 0) acc_l[k] = L;
    __syncthreads();
    if (k == 0) {
      float Os = 0.0f, Ls = 0.0f;
#pragma unroll
      for (int q = 0; q < KS; ++q) {
        Os += acc_o[q][c];
        Ls += acc_l[q];
      }
      seg_O[sgi][c] = Os;
      if (c == 0) {
        seg_M[sgi] = M;
        seg_L[sgi] = Ls;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x >= D) return;
  const int64_t row = (int64_t)j * G + r;
  if (seg_out != nullptr) {
#pragma unroll
    for (int sgi = 0; sgi < 2; ++sgi) {
      const bool empty = !(seg_L[sgi] > 0.0f);
      seg_out[(int64_t)sgi * hq * D + row * D + c] = empty ? 0.0f : seg_O[sgi][c] / seg_L[sgi];
      if (c == 0 && seg_lse != nullptr) seg_lse[(int64_t)sgi * hq + row] = empty ? -INFINITY : (seg_M[sgi] + log2f(seg_L[sgi])) * kLn2;
    }
  }
  if (out != nullptr) {
    const float M = fmaxf(seg_M[0], seg_M[1]);
    float O = 0.0f, L = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int sgi = 0; sgi < 2; ++sgi) {
        if (seg_M[sgi] == -INFINITY) continue;
        const float f = exp2f(seg_M[sgi] - M);
        O = fmaf(seg_O[sgi][c], f, O);
        L = fmaf(seg_L[sgi], f, L);
      }
    }
    const bool empty = !(L > 0.0f);
    out[row * D + c] = from_f32<TO>(empty ? 0.0f : O / L);
    if (c == 0 && lse != nullptr) lse[row] = empty ? -INFINITY : (M + log2f(L)) * kLn2;
  }
}

template <typename T>
__global__ void lse_merge_kernel(const float* __restrict__ outs, int64_t out_stride, const float* __restrict__ lses, int64_t lse_stride, int n_parts,
                                 int64_t rows, int d, T* __restrict__ out, float* __restrict__ lse_out) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= rows * d) return;
  const int64_t r = e / d;
  float M = -INFINITY;
  for (int k = 0; k < n_parts; ++k) M = fmaxf(M, lses[k * lse_stride + r]);
  float acc = 0.0f, lse = -INFINITY;
  if (M != -INFINITY) {
    float sum = 0.0f;
    for (int k = 0; k < n_parts; ++k) sum += expf(lses[k * lse_stride + r] - M);
    lse = M + logf(sum);
    for (int k = 0; k < n_parts; ++k) {
      const float w = expf(lses[k * lse_stride + r] - lse);
      acc = fmaf(w, outs[(int64_t)k * out_stride + e], acc);
    }
  }
  out[e] = from_f32<T>(acc);
  if (lse_out != nullptr && e % d == 0) lse_out[r] = lse;
}

size_t partial_bytes(int h, int g, int d, int n_splits) { return (size_t)h * n_splits * g * (d + 2) * sizeof(float); }

// ---- dispatch ---------------------------------------------------------------------------------

bool is_host_mapped(const void* ptr) {
  if (ptr == nullptr) return false;
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
    cudaGetLastError();
    return true;  // unknown to CUDA: do not hand it to TMA
  }
  return a.type == cudaMemoryTypeHost || a.type == cudaMemoryTypeUnregistered;
}

// Whether the TMA kernel handles this launch: G = 4, bs = 16, d in {64, 128}, contiguous 16-channel
// token rows, every store in device memory.
bool tma_ok(const AttnParams& p, int g, int d) {
  if (g != 4 || p.bs != 16 || (d != 64 && d != 128)) return false;
  for (int i = 0; i < p.n_segs; ++i) {
    const Seg& S = p.seg[i];
    if (S.n_items == 0) continue;
    if (S.kind == SEG_RANGE_REC) {
      if (is_host_mapped(S.records)) return false;
    } else {
      if (S.s_tok != d || is_host_mapped(S.k_base) || is_host_mapped(S.v_base)) return false;
    }
  }
  return true;
}

template <typename T, int D>
int launch_tma(const AttnParams& p, cudaStream_t st) {
  using C = TmaCfg<T, D>;
  static uint64_t attr_set = 0;  // one bit per device
  auto k = attn_tma_kernel<T, D>;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set & bit)) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
    if (e != cudaSuccess) {
      cudaGetLastError();  // not left behind for a later launch check
      return fail(LKV_ERR_CUDA, "attention: shared memory attribute: %s", cudaGetErrorString(e));
    }
    attr_set |= bit;
  }
  k<<<dim3(p.n_splits_total, p.h), kThreads, C::SMEM, st>>>(p);
  return LKV_OK;
}

template <typename T, typename TO, int G, int D>
int launch_all(AttnParams& p, bool use_tma, TO* out, float* lse, float* seg_out, float* seg_lse, cudaStream_t st) {
  if (p.n_splits_total > 0) {
    dim3 grid(p.n_splits_total, p.h);
    if (use_tma) {
      if constexpr (G == 4 && (D == 64 || D == 128)) {
        if (int rc = launch_tma<T, D>(p, st)) return rc;
      }
    } else {
      attn_ldg_kernel<T, G, D><<<grid, kThreads, 0, st>>>(p);
    }
  }
  const int n0 = p.seg[0].n_splits, n1 = p.n_segs > 1 ? p.seg[1].n_splits : 0;
  attn_combine_kernel<TO, G, D><<<dim3(p.h, G), kCombineThreads, 0, st>>>(p.part, n0, n1, out, lse, seg_out, seg_lse, p.hq);
  return launched("lkv attention");
}

template <typename T, typename TO>
int dispatch(int g, int d, AttnParams& p, TO* out, float* lse, float* seg_out, float* seg_lse, cudaStream_t st) {
  const bool use_tma = tma_ok(p, g, d);
#define LKV_D(G, D) \
  if (d == D) return launch_all<T, TO, G, D>(p, use_tma, out, lse, seg_out, seg_lse, st);
#define LKV_G(G)   \
  if (g == G) {    \
    LKV_D(G, 16)   \
    LKV_D(G, 64)   \
    LKV_D(G, 128)  \
  }
  LKV_G(1)
  LKV_G(2)
  LKV_G(4)
  LKV_G(8)
#undef LKV_G
#undef LKV_D
  return fail(LKV_ERR_ARG, "attention: query group %d / head_dim %d not built (groups 1,2,4,8; head_dim 16,64,128)", g, d);
}

int common_checks(const char* who, const void* q, int hq, int h, int d, int bs, int dtype, const void* ws) {
  if (!dtype_ok(dtype)) return fail(LKV_ERR_ARG, "%s: bad dtype %d", who, dtype);
  if (h <= 0 || hq <= 0 || hq % h != 0) return fail(LKV_ERR_ARG, "%s: %d query heads do not group over %d KV heads", who, hq, h);
  const int tl = 32 / (d >= 128 ? 8 : 4);
  if (bs <= 0 || bs % tl != 0) return fail(LKV_ERR_ARG, "%s: block size %d must be a multiple of %d", who, bs, tl);
  if (q == nullptr || ws == nullptr) return fail(LKV_ERR_PTR, "%s: null pointer", who);
  return LKV_OK;
}

int fill_hot(const char* who, Seg& S, int h, int d, int bs, const lkv_hot_set* hs) {
  if (hs->k_base == nullptr || hs->v_base == nullptr || hs->blocks == nullptr) return fail(LKV_ERR_PTR, "%s: null hot-set pointer", who);
  if (hs->n_list <= 0) return fail(LKV_ERR_ARG, "%s: empty block list", who);
  if (hs->last_fill < 0 || hs->last_fill > bs) return fail(LKV_ERR_ARG, "%s: last_fill %d outside [0, %d]", who, hs->last_fill, bs);
  const size_t es = dtype_size(hs->dtype);
  if (!aligned(hs->k_base, 16) || !aligned(hs->v_base, 16) || (hs->s_row * es) % 16 || (hs->s_head * es) % 16 || (hs->s_tok * es) % 16)
    return fail(LKV_ERR_PTR, "%s: KV rows must be 16-byte aligned", who);
  S = Seg{};
  S.kind = SEG_LIST;
  S.k_base = hs->k_base; S.v_base = hs->v_base; S.s_row = hs->s_row; S.s_head = hs->s_head; S.s_tok = hs->s_tok;
  S.blocks = hs->blocks; S.n_list = hs->n_list; S.last_fill = hs->last_fill; S.slot_of = hs->slot_of; S.slot_stride = hs->slot_stride;
  S.n_rows = hs->n_rows > 0 ? hs->n_rows : 0;
  S.n_items = hs->n_list;
  (void)h; (void)d;
  return LKV_OK;
}

int fill_cold(const char* who, Seg& S, int h, int d, int bs, int dtype, const lkv_cold_set* cs) {
  if (cs->kind != LKV_COLD_INT8 && cs->kind != LKV_COLD_PAIRS) return fail(LKV_ERR_ARG, "%s: bad cold kind %d", who, cs->kind);
  if (cs->n_blocks < 0 || cs->first_block < 0) return fail(LKV_ERR_ARG, "%s: bad block range", who);
  if (cs->n_blocks > 0 && cs->store == nullptr) return fail(LKV_ERR_PTR, "%s: null cold store", who);
  if (cs->store != nullptr && !aligned(cs->store, 16)) return fail(LKV_ERR_PTR, "%s: cold store must be 16-byte aligned", who);
  S = Seg{};
  if (cs->kind == LKV_COLD_INT8) {
    S.kind = SEG_RANGE_REC;
    S.records = static_cast<const uint8_t*>(cs->store);
    S.width = lkv_packed_pair_bytes(bs, d);
  } else {
    // pairs [blocks, h, 2, bs, d]: a "row" is a block
    S.kind = SEG_RANGE_PAIRS;
    S.k_base = cs->store;
    S.v_base = static_cast<const char*>(cs->store) + (size_t)bs * d * dtype_size(dtype);
    S.s_row = (int64_t)h * 2 * bs * d; S.s_head = 2ll * bs * d; S.s_tok = d;
    S.n_rows = (int64_t)cs->first_block + cs->n_blocks;
  }
  S.first_block = cs->first_block; S.excluded = cs->excluded; S.bitmap_words = cs->bitmap_words;
  S.n_items = cs->n_blocks;
  return LKV_OK;
}

// Split the target CTA count between two segments in proportion to their bytes.
// hot_item / cold_item: the cost of one item of each segment (bytes for the CUDA-core kernels, time
// for the tensor-core one). Each segment gets at least one CTA; the total stays within total_ctas + 1.
void split_two(Seg& hot, Seg& cold, int h, double hot_item, double cold_item, int total_ctas) {
  const int target = (total_ctas + h - 1) / h;
  const double wh = (double)hot.n_items * hot_item, wc = (double)cold.n_items * cold_item;
  int th = wh + wc > 0 ? (int)(target * wh / (wh + wc) + 0.5) : 0;
  if (hot.n_items > 0 && th < 1) th = 1;
  int tc = target - th;
  if (cold.n_items > 0 && tc < 1) tc = 1;
  set_split(hot, th);
  set_split(cold, tc);
}

// ---- the tensor-core path -----------------------------------------------------------------

// K and V maps of a list or pairs segment: 4-D bf16 tensors (channel, token, row, head) with a box of
// one 16 x 64 block, 128-byte swizzle. The row and head dimensions are ordered by stride.
bool make_kv_maps(const Seg& S, int h, int d, CUtensorMap* tk, CUtensorMap* tv, int* head_major) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr || S.n_rows <= 0) return false;
  const int64_t es = 2;
  const int64_t st = S.s_tok * es, sr = S.s_row * es, sh = S.s_head * es;
  const bool hm = sh < sr;
  // Boxes of 64 channels x 16 tokens (128-byte swizzled rows); a 128-channel tile is two boxes.
  const cuuint64_t dims[4] = {(cuuint64_t)d, 16, (cuuint64_t)(hm ? h : S.n_rows), (cuuint64_t)(hm ? S.n_rows : h)};
  const cuuint64_t strides[3] = {(cuuint64_t)st, (cuuint64_t)(hm ? sh : sr), (cuuint64_t)(hm ? sr : sh)};
  const cuuint32_t box[4] = {64, 16, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  for (int i = 0; i < 2; ++i) {
    CUresult r = encode_tiled(i == 0 ? tk : tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(i == 0 ? S.k_base : S.v_base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
  }
  *head_major = hm ? 1 : 0;
  return true;
}

// Whether the stream kernel takes this launch (bf16, d 64 or 128, bs 16, G <= 8, stores in device
// memory, d-channel token rows); fills the tensor maps of its list / pairs segments.
bool mma_plan(const AttnParams& p, int g, int d, bool bf16, MmaParams& mp) {
  if (!bf16 || (d != 64 && d != 128) || p.bs != 16 || (g != 1 && g != 2 && g != 4 && g != 8)) return false;
  if (!(p.scale_log2 > 0.0f)) return false;  // its lazy rescaling compares raw scores against (m + 8) / scale
  for (int i = 0; i < p.n_segs; ++i) {
    const Seg& S = p.seg[i];
    if (S.n_items == 0) continue;
    if (S.kind == SEG_RANGE_REC) {
      if (S.width != (d == 64 ? MmaGeom<64>::REC : MmaGeom<128>::REC) || is_host_mapped(S.records)) return false;
    } else {
      if (S.s_tok != d || is_host_mapped(S.k_base) || is_host_mapped(S.v_base)) return false;
      if (!make_kv_maps(S, p.h, d, &mp.tk[i], &mp.tv[i], &mp.head_major[i])) return false;
    }
  }
  return true;
}

// SMs of the current device (cached per device; the B200 count when no device answers).
int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return kNumSMs;
  }
  int& c = cached[dev & 63];
  if (c == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
      cudaGetLastError();
      v = kNumSMs;
    }
    c = v;
  }
  return c;
}

// CTAs per KV head of the stream kernel: kStreamCtasPerSm per SM over the heads, or more when a
// CTA's items could exceed its list (n_ub: an upper bound of a head's items; a CTA holds at most
// ceil(n / P) items of each of the two segments, so ceil(n_ub / P) + 2 in all). When the list
// forces more than one wave of CTAs, P is chosen among [need, 3 need] (at most 32, the fold's fast
// path, unless need is more) to minimise the waves times
// a CTA's share (items plus a fixed cost of kStreamCtaCost items for its set-up and fold), so that
// the last wave is not left mostly empty (64 heads x 4 CTAs on 148 SMs would be 1.73 waves).
constexpr int64_t kStreamCtaCost = 64;
int stream_per_head(int h, int64_t n_ub) {
  const int sms = kStreamCtasPerSm * sm_count();
  const int hh = h > 0 ? h : 1;
  int per = sms / hh;
  const int64_t need = (n_ub + kStreamListCap - 3) / (kStreamListCap - 2);
  if (need <= per) return per < 1 ? 1 : per;
  int64_t best_p = need, best_cost = -1;
  const int64_t top = 3 * need < 32 ? 3 * need : (need > 32 ? need : 32);
  for (int64_t P = need; P <= top; ++P) {
    const int64_t waves = (hh * P + sms - 1) / sms;
    const int64_t cost = waves * (kStreamCtaCost + (n_ub + P - 1) / P);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_p = P;
    }
  }
  return (int)best_p;
}
size_t stream_partial_bytes(int h, int g, int d, int64_t n_ub) {
  const int part = (g * d + 2 * g + 3) / 4 * 4;
  return (size_t)h * stream_per_head(h, n_ub) * 2 * part * sizeof(float);
}
int64_t stream_item_bound(const AttnParams& p) {
  int64_t n = 0;
  for (int s = 0; s < p.n_segs; ++s) n += p.seg[s].n_items;
  return n;
}

template <int G, int D, typename TO>
int launch_stream(const StreamParams& sp, cudaStream_t st) {
  using C = StreamCfg<G, D>;
  static uint64_t attr_set = 0;  // one bit per device
  // Ragged rows run at head_dim 64 only (run_attention_ragged checks it).
  auto k = attn_stream_kernel<G, D, TO, false>;
  if constexpr (D == 64)
    if (sp.sched != nullptr) k = attn_stream_kernel<G, D, TO, true>;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set & bit)) {  // every instance: a single sequence's and (head_dim 64) ragged rows'
    cudaError_t e = cudaFuncSetAttribute(attn_stream_kernel<G, D, TO, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
    if constexpr (D == 64)
      if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_stream_kernel<G, D, TO, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
    if (e != cudaSuccess) {
      cudaGetLastError();  // not left behind for a later launch check
      return fail(LKV_ERR_CUDA, "attention: shared memory attribute: %s", cudaGetErrorString(e));
    }
    attr_set |= bit;
  }
  const dim3 grid = sp.sched != nullptr ? dim3(sp.per_head) : dim3(sp.per_head, sp.p.h);  // ragged: per_head holds the CTAs
  cudaError_t e = launch_pdl(k, grid, dim3(C::THREADS), C::SMEM, st, 0, sp);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LKV_ERR_CUDA, "lkv attention: %s", cudaGetErrorString(e));
  }
  return launched("lkv attention");
}

// Splits, workspace check and launch of one attention call. The workspace starts with
// kStreamCounterBytes of per-head counters (zero before and after every call), then the partials.
template <typename T, typename TO>
int run_attention(const char* who, AttnParams& p, int g, int d, TO* out, float* lse, float* seg_out, float* seg_lse, void* workspace,
                  size_t workspace_bytes, cudaStream_t st) {
  if (workspace_bytes < (size_t)kStreamCounterBytes)
    return fail(LKV_ERR_WORKSPACE, "%s: workspace %zu < %d bytes", who, workspace_bytes, kStreamCounterBytes);
  if (!aligned(workspace, 16)) return fail(LKV_ERR_PTR, "%s: workspace must be 16-byte aligned", who);
  p.part = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kStreamCounterBytes);
  const size_t avail = workspace_bytes - kStreamCounterBytes;
  MmaParams mp{};
  const bool mma = p.h <= kStreamCounterBytes / 4 && mma_plan(p, g, d, sizeof(T) == 2, mp);
  if (mma) {
    if constexpr (sizeof(T) == 2) {
      StreamParams sp{};
      sp.p = p;
      for (int i = 0; i < 2; ++i) {
        sp.tk[i] = mp.tk[i];
        sp.tv[i] = mp.tv[i];
        sp.head_major[i] = mp.head_major[i];
      }
      const int64_t n_ub = stream_item_bound(p);
      sp.per_head = stream_per_head(p.h, n_ub);
      sp.counters = static_cast<unsigned int*>(workspace);
      sp.part = p.part;
      sp.out = out;
      sp.lse = lse;
      sp.seg_out = seg_out;
      sp.seg_lse = seg_lse;
      const size_t need = stream_partial_bytes(p.h, g, d, n_ub);
      if (avail < need) return fail(LKV_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", who, workspace_bytes, need + kStreamCounterBytes);
      if (d == 128) {
        switch (g) {
          case 1: return launch_stream<1, 128, TO>(sp, st);
          case 2: return launch_stream<2, 128, TO>(sp, st);
          case 4: return launch_stream<4, 128, TO>(sp, st);
          default: return launch_stream<8, 128, TO>(sp, st);
        }
      }
      switch (g) {
        case 1: return launch_stream<1, 64, TO>(sp, st);
        case 2: return launch_stream<2, 64, TO>(sp, st);
        case 4: return launch_stream<4, 64, TO>(sp, st);
        default: return launch_stream<8, 64, TO>(sp, st);
      }
    }
  }
  if (p.n_segs == 1) {
    set_split(p.seg[0], (kTargetCtas + p.h - 1) / p.h);
    p.n_splits_total = p.seg[0].n_splits;
  } else {
    split_two(p.seg[0], p.seg[1], p.h, 4096, 2368, kTargetCtas);
    p.n_splits_total = p.seg[0].n_splits + p.seg[1].n_splits;
  }
  const size_t need = partial_bytes(p.h, g, d, p.n_splits_total);
  if (avail < need) return fail(LKV_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", who, workspace_bytes, need + kStreamCounterBytes);
  return dispatch<T, TO>(g, d, p, out, lse, seg_out, seg_lse, st);
}

// Ragged rows: one launch of the stream kernel over a host-built schedule (see lkv_ragged_schedule).
template <typename TO>
int run_attention_ragged(const char* who, AttnParams& p, int g, int d, const int4* sched, int n_ctas, int n_parts, const int4* row_info,
                         const int32_t* table, int64_t table_stride, int heads, TO* out, float* lse, void* workspace, size_t workspace_bytes,
                         cudaStream_t st) {
  const int rows = p.hq / g;
  if (rows > kStreamCounterBytes / 4) return fail(LKV_ERR_ARG, "%s: %d rows > %d", who, rows, kStreamCounterBytes / 4);
  const size_t need = (size_t)kStreamCounterBytes + (size_t)n_parts * 2 * ((g * 64 + 2 * g + 3) / 4 * 4) * sizeof(float);
  if (workspace_bytes < need) return fail(LKV_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", who, workspace_bytes, need);
  if (!aligned(workspace, 16)) return fail(LKV_ERR_PTR, "%s: workspace must be 16-byte aligned", who);
  p.part = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kStreamCounterBytes);
  MmaParams mp{};
  if (d != 64 || !mma_plan(p, g, d, true, mp))
    return fail(LKV_ERR_ARG, "%s: ragged rows need bf16, head_dim 64, block size 16, a group of 1, 2, 4 or 8, a positive scale and device-resident stores", who);
  StreamParams sp{};
  sp.p = p;
  for (int i = 0; i < 2; ++i) {
    sp.tk[i] = mp.tk[i];
    sp.tv[i] = mp.tv[i];
    sp.head_major[i] = mp.head_major[i];
  }
  sp.per_head = n_ctas;
  sp.counters = static_cast<unsigned int*>(workspace);
  sp.part = p.part;
  sp.out = out;
  sp.lse = lse;
  sp.sched = sched;
  sp.row_info = row_info;
  sp.table = table;
  sp.table_stride = table_stride;
  sp.heads = heads;
  switch (g) {
    case 1: return launch_stream<1, 64, TO>(sp, st);
    case 2: return launch_stream<2, 64, TO>(sp, st);
    case 4: return launch_stream<4, 64, TO>(sp, st);
    default: return launch_stream<8, 64, TO>(sp, st);
  }
}

}  // namespace
}  // namespace lkv

using namespace lkv;

extern "C" {

int lkv_ragged_schedule(const int32_t* row_items, int rows, int n_sms, int32_t* sched, int max_ctas, int* n_parts) {
  if (row_items == nullptr || sched == nullptr || n_parts == nullptr || rows <= 0 || n_sms <= 0)
    return -fail(LKV_ERR_ARG, "lkv_ragged_schedule: bad arguments");
  int64_t total = 0;
  for (int r = 0; r < rows; ++r) {
    if (row_items[r] < 0) return -fail(LKV_ERR_ARG, "lkv_ragged_schedule: row %d has %d items", r, row_items[r]);
    total += row_items[r];
  }
  // Items per CTA: about four waves of one CTA per SM, at least 64 items and at most what a CTA's
  // list holds (two segments, each rounded up).
  int64_t chunk = (total + 4LL * n_sms - 1) / (4LL * n_sms);
  if (chunk < 64) chunk = 64;
  if (chunk > kStreamListCap - 2) chunk = kStreamListCap - 2;
  int n = 0, parts = 0;
  for (int r = 0; r < rows; ++r) {
    const int P = (int)((row_items[r] + chunk - 1) / chunk) > 0 ? (int)((row_items[r] + chunk - 1) / chunk) : 1;
    if (n + P > max_ctas) return -fail(LKV_ERR_WORKSPACE, "lkv_ragged_schedule: more than %d CTAs", max_ctas);
    for (int c = 0; c < P; ++c, ++n) {
      sched[4 * n + 0] = r;
      sched[4 * n + 1] = c;
      sched[4 * n + 2] = P;
      sched[4 * n + 3] = parts;
    }
    parts += P;
  }
  *n_parts = parts;
  return n;
}

size_t lkv_ragged_attention_workspace(int g, int n_parts) {
  if (g <= 0 || n_parts < 0) return 0;
  return (size_t)kStreamCounterBytes + (size_t)n_parts * 2 * ((g * 64 + 2 * g + 3) / 4 * 4) * sizeof(float);
}

int lkv_ragged_exact_attention(const void* q, int rows, int g, int d, int bs, int heads, const lkv_hot_set* hot, const uint8_t* records,
                               int64_t n_records, const int32_t* table, int64_t table_stride, const uint32_t* excluded, int bitmap_words,
                               const int32_t* row_info, const int32_t* sched, int n_ctas, int n_parts, float scale, void* out, int out_dtype,
                               float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  const char* who = "lkv_ragged_exact_attention";
  if (hot == nullptr || records == nullptr || table == nullptr || row_info == nullptr || sched == nullptr || q == nullptr)
    return fail(LKV_ERR_PTR, "%s: null pointer", who);
  if (rows <= 0 || heads <= 0 || rows % heads != 0 || n_ctas <= 0 || n_parts < n_ctas || n_records <= 0)
    return fail(LKV_ERR_ARG, "%s: bad shape (rows %d, heads %d, CTAs %d, partials %d)", who, rows, heads, n_ctas, n_parts);
  if (int rc = common_checks(who, q, rows * g, heads, d, bs, hot->dtype, workspace)) return rc;
  if (hot->dtype != LKV_BF16 || !dtype_ok(out_dtype)) return fail(LKV_ERR_ARG, "%s: ragged rows are bf16", who);
  if (out == nullptr && lse == nullptr) return fail(LKV_ERR_PTR, "%s: no output", who);
  AttnParams p{};
  p.q = q; p.hq = rows * g; p.h = heads; p.bs = bs; p.scale_log2 = scale * kLog2e;
  if (int rc = fill_hot(who, p.seg[0], heads, d, bs, hot)) return rc;
  // The range: candidate blocks from 1, as many as the longest row; each row's own count is in row_info.
  lkv_cold_set cs{records, LKV_COLD_INT8, 1, (int)(n_records > INT32_MAX ? INT32_MAX : n_records), excluded, bitmap_words};
  if (int rc = fill_cold(who, p.seg[1], heads, d, bs, LKV_BF16, &cs)) return rc;
  p.seg[1].n_rows = n_records;  // bounds the table's entries
  p.n_segs = 2;
  cudaStream_t st = as_stream(stream);
  const int4* sc = reinterpret_cast<const int4*>(sched);
  const int4* ri = reinterpret_cast<const int4*>(row_info);
  if (!aligned(sched, 16) || !aligned(row_info, 16)) return fail(LKV_ERR_PTR, "%s: schedule and row info must be 16-byte aligned", who);
  if (out_dtype == LKV_BF16)
    return run_attention_ragged<__nv_bfloat16>(who, p, g, d, sc, n_ctas, n_parts, ri, table, table_stride, heads, static_cast<__nv_bfloat16*>(out), lse,
                                               workspace, workspace_bytes, st);
  return run_attention_ragged<float>(who, p, g, d, sc, n_ctas, n_parts, ri, table, table_stride, heads, static_cast<float*>(out), lse, workspace,
                                     workspace_bytes, st);
}

int lkv_device_status(int* status, int clear) {
  if (status == nullptr) return fail(LKV_ERR_PTR, "lkv_device_status: null pointer");
  int a = 0, b = 0, c = 0;
  cudaError_t e = tu_device_status(&a, clear);
  if (e == cudaSuccess) e = select_device_status(&b, clear);
  if (e == cudaSuccess) e = exchange_device_status(&c, clear);
  if (e != cudaSuccess) return fail(LKV_ERR_CUDA, "lkv_device_status: %s", cudaGetErrorString(e));
  *status = a != 0 ? a : (b != 0 ? b : c);
  return LKV_OK;
}

int lkv_status_attach(void) {
  static std::mutex mu;
  static int* host_word = nullptr;  // pinned, mapped, portable: one word for every device
  std::lock_guard<std::mutex> lock(mu);
  cudaError_t e = cudaSuccess;
  if (host_word == nullptr) {
    void* p = nullptr;
    e = cudaHostAlloc(&p, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable);
    if (e != cudaSuccess) return fail(LKV_ERR_CUDA, "lkv_status_attach: cudaHostAlloc: %s", cudaGetErrorString(e));
    host_word = static_cast<int*>(p);
    __atomic_store_n(host_word, 0, __ATOMIC_SEQ_CST);
    g_status_word = host_word;
  }
  int* dev_word = nullptr;
  e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&dev_word), host_word, 0);
  if (e == cudaSuccess) e = tu_status_attach(dev_word);
  if (e == cudaSuccess) e = select_status_attach(dev_word);
  if (e == cudaSuccess) e = exchange_status_attach(dev_word);
  if (e != cudaSuccess) return fail(LKV_ERR_CUDA, "lkv_status_attach: %s", cudaGetErrorString(e));
  return LKV_OK;
}

int lkv_status_poll(int* status, int clear) {
  if (status == nullptr) return fail(LKV_ERR_PTR, "lkv_status_poll: null pointer");
  int* w = g_status_word;
  if (w == nullptr) return fail(LKV_ERR_ARG, "lkv_status_poll: lkv_status_attach has not been called");
  *status = clear ? __atomic_exchange_n(w, 0, __ATOMIC_SEQ_CST) : __atomic_load_n(w, __ATOMIC_SEQ_CST);
  return LKV_OK;
}

size_t lkv_attention_workspace(int h, int hq, int d, int n_items) {
  if (h <= 0 || hq <= 0) return 0;
  const int s = splits_for(n_items, (kTargetCtas + h - 1) / h);
  const size_t a = partial_bytes(h, hq / h, d, s), b = stream_partial_bytes(h, hq / h, d, n_items > 0 ? n_items : 0);
  return kStreamCounterBytes + (a > b ? a : b);
}

size_t lkv_exact_attention_workspace(int h, int hq, int d, int n_list, int n_blocks) {
  if (h <= 0 || hq <= 0) return 0;
  const int per_head = (kTargetCtas + h - 1) / h + 1;  // any split of the target between the segments
  const int64_t n_ub = (int64_t)(n_list > 0 ? n_list : 0) + (n_blocks > 0 ? n_blocks : 0);
  const size_t a = partial_bytes(h, hq / h, d, per_head), b = stream_partial_bytes(h, hq / h, d, n_ub);
  return kStreamCounterBytes + (a > b ? a : b);
}

int lkv_hot_attention(const void* q, int hq, int h, int d, int bs, const void* k_base, const void* v_base, int dtype, int64_t s_row,
                      int64_t s_head, int64_t s_tok, int64_t n_rows, const int32_t* blocks, int n_list, const int32_t* slot_of,
                      int64_t slot_stride, int last_fill, float scale, float* out, float* lse, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (int rc = common_checks("lkv_hot_attention", q, hq, h, d, bs, dtype, workspace)) return rc;
  if (out == nullptr || lse == nullptr) return fail(LKV_ERR_PTR, "lkv_hot_attention: null pointer");
  lkv_hot_set hs{k_base, v_base, dtype, s_row, s_head, s_tok, blocks, n_list, slot_of, slot_stride, last_fill, n_rows};
  AttnParams p{};
  p.q = q; p.hq = hq; p.h = h; p.bs = bs; p.scale_log2 = scale * kLog2e;
  if (int rc = fill_hot("lkv_hot_attention", p.seg[0], h, d, bs, &hs)) return rc;
  p.n_segs = 1;
  cudaStream_t st = as_stream(stream);
  return dtype == LKV_BF16 ? run_attention<__nv_bfloat16, float>("lkv_hot_attention", p, hq / h, d, out, lse, nullptr, nullptr, workspace, workspace_bytes, st)
                           : run_attention<float, float>("lkv_hot_attention", p, hq / h, d, out, lse, nullptr, nullptr, workspace, workspace_bytes, st);
}

int lkv_cold_attention(const void* q, int hq, int h, int d, int bs, const void* cold, int cold_kind, int dtype, int first_block,
                       int n_blocks, const uint32_t* excluded, int bitmap_words, float scale, float* out, float* lse, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (int rc = common_checks("lkv_cold_attention", q, hq, h, d, bs, dtype, workspace)) return rc;
  if (out == nullptr || lse == nullptr) return fail(LKV_ERR_PTR, "lkv_cold_attention: null pointer");
  lkv_cold_set cs{cold, cold_kind, first_block, n_blocks, excluded, bitmap_words};
  AttnParams p{};
  p.q = q; p.hq = hq; p.h = h; p.bs = bs; p.scale_log2 = scale * kLog2e;
  if (int rc = fill_cold("lkv_cold_attention", p.seg[0], h, d, bs, dtype, &cs)) return rc;
  p.n_segs = 1;
  cudaStream_t st = as_stream(stream);
  return dtype == LKV_BF16 ? run_attention<__nv_bfloat16, float>("lkv_cold_attention", p, hq / h, d, out, lse, nullptr, nullptr, workspace, workspace_bytes, st)
                           : run_attention<float, float>("lkv_cold_attention", p, hq / h, d, out, lse, nullptr, nullptr, workspace, workspace_bytes, st);
}

int lkv_exact_attention(const void* q, int hq, int h, int d, int bs, const lkv_hot_set* hot, const lkv_cold_set* cold, float scale,
                        void* out, int out_dtype, float* lse, float* part_out, float* part_lse, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (hot == nullptr || cold == nullptr) return fail(LKV_ERR_PTR, "lkv_exact_attention: null set");
  if (int rc = common_checks("lkv_exact_attention", q, hq, h, d, bs, hot->dtype, workspace)) return rc;
  if (!dtype_ok(out_dtype)) return fail(LKV_ERR_ARG, "lkv_exact_attention: bad output dtype %d", out_dtype);
  if (out == nullptr && part_out == nullptr) return fail(LKV_ERR_PTR, "lkv_exact_attention: no output");
  AttnParams p{};
  p.q = q; p.hq = hq; p.h = h; p.bs = bs; p.scale_log2 = scale * kLog2e;
  if (int rc = fill_hot("lkv_exact_attention", p.seg[0], h, d, bs, hot)) return rc;
  if (int rc = fill_cold("lkv_exact_attention", p.seg[1], h, d, bs, hot->dtype, cold)) return rc;
  p.n_segs = 2;
  cudaStream_t st = as_stream(stream);
  const int g = hq / h;
  const bool bf = hot->dtype == LKV_BF16;
  const char* who = "lkv_exact_attention";
  if (out_dtype == LKV_BF16)
    return bf ? run_attention<__nv_bfloat16, __nv_bfloat16>(who, p, g, d, static_cast<__nv_bfloat16*>(out), lse, part_out, part_lse, workspace, workspace_bytes, st)
              : run_attention<float, __nv_bfloat16>(who, p, g, d, static_cast<__nv_bfloat16*>(out), lse, part_out, part_lse, workspace, workspace_bytes, st);
  return bf ? run_attention<__nv_bfloat16, float>(who, p, g, d, static_cast<float*>(out), lse, part_out, part_lse, workspace, workspace_bytes, st)
            : run_attention<float, float>(who, p, g, d, static_cast<float*>(out), lse, part_out, part_lse, workspace, workspace_bytes, st);
}

int lkv_lse_merge(const float* outs, const float* lses, int n_parts, int64_t rows, int d, void* out, int out_dtype, float* lse_out,
                  void* stream) {
  if (!dtype_ok(out_dtype)) return fail(LKV_ERR_ARG, "lkv_lse_merge: bad dtype %d", out_dtype);
  if (n_parts <= 0 || rows < 0 || d <= 0) return fail(LKV_ERR_ARG, "lkv_lse_merge: bad shape");
  if (outs == nullptr || lses == nullptr || out == nullptr) return fail(LKV_ERR_PTR, "lkv_lse_merge: null pointer");
  if (rows == 0) return LKV_OK;
  const int64_t n = rows * d;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (out_dtype == LKV_BF16)
    lse_merge_kernel<__nv_bfloat16><<<blocks, 256, 0, as_stream(stream)>>>(outs, rows * d, lses, rows, n_parts, rows, d,
                                                                          static_cast<__nv_bfloat16*>(out), lse_out);
  else
    lse_merge_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(outs, rows * d, lses, rows, n_parts, rows, d, static_cast<float*>(out), lse_out);
  return launched("lkv_lse_merge");
}

int lkv_lse_merge_packed(const float* parts, int n_parts, int64_t rows, int d, void* out, int out_dtype, float* lse_out, void* stream) {
  if (!dtype_ok(out_dtype)) return fail(LKV_ERR_ARG, "lkv_lse_merge_packed: bad dtype %d", out_dtype);
  if (n_parts <= 0 || rows < 0 || d <= 0) return fail(LKV_ERR_ARG, "lkv_lse_merge_packed: bad shape");
  if (parts == nullptr || out == nullptr) return fail(LKV_ERR_PTR, "lkv_lse_merge_packed: null pointer");
  if (rows == 0) return LKV_OK;
  const int64_t n = rows * d, stride = rows * (d + 1);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (out_dtype == LKV_BF16)
    lse_merge_kernel<__nv_bfloat16><<<blocks, 256, 0, as_stream(stream)>>>(parts, stride, parts + n, stride, n_parts, rows, d,
                                                                          static_cast<__nv_bfloat16*>(out), lse_out);
  else
    lse_merge_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(parts, stride, parts + n, stride, n_parts, rows, d, static_cast<float*>(out), lse_out);
  return launched("lkv_lse_merge_packed");
}

}  // extern "C"
