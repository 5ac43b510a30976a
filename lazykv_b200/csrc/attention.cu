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
// Each CTA takes a chunk of one segment's items for one KV head and emits an online-softmax partial
// (running max m in the log2 domain, sum l, unnormalised o) for the head's G query rows. A combine
// kernel folds the chunks into per-segment (out = o / l, lse) and into their merge. A partial over
// no key is (m = -inf, l = 0), which the combine turns into lse = -inf and out = 0, as
// cpu_partial_attention does (exact.py:108-110).
//
// Two kernels do the partial work:
//  * attn_tma_kernel (stores in device memory, G = 4, bs = 16, d in {64, 128}): each warp streams
//    its items through a private ring of shared-memory stages filled by TMA bulk copies
//    (cp.async.bulk, one mbarrier per stage, bounded waits); the block ids, slot rows and exclusion
//    bits of the warp's items are prefetched into registers so issuing never waits on a dependent
//    global load; dot products and accumulations use packed float32x2 FMAs;
//  * attn_ldg_kernel (any other geometry, and stores in mapped host memory read over the link):
//    the same arithmetic with vectorised loads straight from global memory.
// Lane layout in a warp: CG = d/16 channel groups x TL = 32/CG token lanes; a lane holds 16
// channels of the G query rows and of its accumulators and takes tokens tl, tl + TL, ... of a block.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "tma.cuh"

namespace lkv {
namespace {

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
// attn_mma_kernel: tensor-core split decode (bf16, d = 64, bs = 16, G <= 8), stores in device memory
// ============================================================================================
//
// Per item (one block of one KV head) a warp runs two small contractions on the tensor cores with
// mma.sync.m16n8k16 (bf16 operands, float32 accumulators):
//   S^T [16 tokens x 8 rows]   = K [16 x 64] . Q^T [64 x 8]      (4 k-steps; rows >= G are zero)
//   O^T [64 channels x 8 rows] += V^T [64 x 16] . P^T [16 x 8]   (4 m-tiles)
// K and V reach shared memory as bf16 tiles of 16 rows x 128 bytes in the 128-byte swizzle
// (16-byte chunk c of row r stored at chunk c ^ (r & 7)), so ldmatrix reads them without bank
// conflicts: hot blocks and cold pairs by tensor-map TMA loads (cp.async.bulk.tensor, SWIZZLE_128B),
// int8 cold records by a bulk copy of the raw record that the warp dequantises into its own tile
// (float32 affine of quant.py:103-104, rounded to bf16: what a fetch puts in a slot). The products
// of bf16 operands are exact in float32; P (float32) enters the second contraction as the sum of
// three bf16 terms (hi + mid + lo, 24 significant bits), each a separate MMA, so the result keeps
// float32 accuracy. The score fragment becomes the P^T operand with movmatrix (an 8x8 transpose in
// registers). Softmax bookkeeping follows the CUDA-core kernels: log2 domain, lazy rescaling.

constexpr int kMmaWarps = 4;
constexpr int kMmaThreads = 32 * kMmaWarps;
constexpr int kMmaStages = 2;
constexpr int kMmaTile = 2048;                  // 16 x 64 bf16, swizzled
constexpr int kMmaHotStage = 2 * kMmaTile;      // K tile + V tile
constexpr int kMmaRec = 2368;                   // int8 record at bs 16, d 64
constexpr int kMmaRecStage = 2432;              // record stage stride (a multiple of 128 bytes)
constexpr int kMmaCtasPerSm = 6;
constexpr int kMmaTargetCtas = kMmaCtasPerSm * kNumSMs;
constexpr int kMmaHotBody = kMmaWarps * kMmaStages * kMmaHotStage;                            // hot / pairs stages
constexpr int kMmaColdBody = kMmaWarps * 2 * kMmaTile + kMmaWarps * kMmaStages * kMmaRecStage;  // tiles + record stages
constexpr int kMmaBody = kMmaHotBody > kMmaColdBody ? kMmaHotBody : kMmaColdBody;
static_assert(kMmaBody >= kMmaWarps * 8 * 64 * 4 + kMmaWarps * 2 * 8 * 4, "epilogue scratch exceeds the body");
constexpr size_t kMmaSmem = 1024 + kMmaBody + kMmaWarps * kMmaStages * 8;

struct MmaParams {
  AttnParams p;
  CUtensorMap tk[2], tv[2];  // per segment: K and V maps of a list or pairs segment
  int head_major[2];         // map coordinate order: (0, 0, head, row) instead of (0, 0, row, head)
};

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint64_t* bar) {
  asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
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

// Splits (a, b) into three bf16x2 terms whose sum is (a, b) to 24 significant bits.
__device__ __forceinline__ void split3(float a, float b, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
  hi = pack_bf2(a, b);
  const float2 r = __fadd2_rn(f2(a, b), f2(-unpack_bf2(hi).x, -unpack_bf2(hi).y));
  mid = pack_bf2(r.x, r.y);
  const float2 r2 = __fadd2_rn(r, f2(-unpack_bf2(mid).x, -unpack_bf2(mid).y));
  lo = pack_bf2(r2.x, r2.y);
}

// 8 int8 codes -> 4 float2 of (code + 128), exactly (2^23 magic, as codes16).
__device__ __forceinline__ void codes8(uint2 w, float2 (&u)[4]) {
  const uint32_t a = w.x ^ 0x80808080u, b = w.y ^ 0x80808080u;
  const float2 mm = f2(-8388608.0f, -8388608.0f);
  u[0] = __fadd2_rn(f2(__uint_as_float(__byte_perm(a, 0x4b000000u, 0x7650)), __uint_as_float(__byte_perm(a, 0x4b000000u, 0x7651))), mm);
  u[1] = __fadd2_rn(f2(__uint_as_float(__byte_perm(a, 0x4b000000u, 0x7652)), __uint_as_float(__byte_perm(a, 0x4b000000u, 0x7653))), mm);
  u[2] = __fadd2_rn(f2(__uint_as_float(__byte_perm(b, 0x4b000000u, 0x7650)), __uint_as_float(__byte_perm(b, 0x4b000000u, 0x7651))), mm);
  u[3] = __fadd2_rn(f2(__uint_as_float(__byte_perm(b, 0x4b000000u, 0x7652)), __uint_as_float(__byte_perm(b, 0x4b000000u, 0x7653))), mm);
}

__device__ __forceinline__ uint32_t swz(int row, int chunk) { return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4)); }

// Dequantises the int8 record at `raw` (kq | vq | k_scale | k_zero | v_scale | v_zero, bs 16, d 64)
// into bf16 K and V tiles in the swizzled layout. Lane: channel group gq = lane & 7 (8 channels),
// tokens 4 * (lane >> 3) + i, i = 0..3. Each value is (code + 128) * scale + zero in float32 (one
// rounding, as quant.py's unpack), then rounded to bf16.
__device__ __forceinline__ void dequant_record(const unsigned char* raw, unsigned char* kt, unsigned char* vt, int lane) {
  const int gq = lane & 7, t0 = 4 * (lane >> 3);
  // Swizzled chunk offsets of tokens t0 + i: t0 & 7 is 0 or 4, so (t & 7) = (t0 & 7) + i.
  uint32_t dst[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = (uint32_t)((t0 + i) * 128 + ((gq ^ ((t0 & 7) + i)) << 4));
  float2 ks2[4], kz2[4];
  {
    const uint4 a = *reinterpret_cast<const uint4*>(raw + 2048 + 16 * gq);
    const uint4 b = *reinterpret_cast<const uint4*>(raw + 2048 + 128 + 16 * gq);
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      ks2[x] = __half22float2(*reinterpret_cast<const __half2*>(&wa[x]));
      kz2[x] = __half22float2(*reinterpret_cast<const __half2*>(&wb[x]));
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 u[4];
    codes8(*reinterpret_cast<const uint2*>(raw + (t0 + i) * 64 + 8 * gq), u);
    float2 k[4];
#pragma unroll
    for (int x = 0; x < 4; ++x) k[x] = __ffma2_rn(u[x], ks2[x], kz2[x]);
    uint4 o;
    o.x = pack_bf2(k[0].x, k[0].y);
    o.y = pack_bf2(k[1].x, k[1].y);
    o.z = pack_bf2(k[2].x, k[2].y);
    o.w = pack_bf2(k[3].x, k[3].y);
    *reinterpret_cast<uint4*>(kt + dst[i]) = o;
  }
  // Per-token V scales of tokens t0..t0+3: four f16 each, one 8-byte load.
  const uint2 vsw = *reinterpret_cast<const uint2*>(raw + 2304 + 2 * t0);
  const uint2 vzw = *reinterpret_cast<const uint2*>(raw + 2336 + 2 * t0);
  const float2 vs01 = __half22float2(*reinterpret_cast<const __half2*>(&vsw.x)), vs23 = __half22float2(*reinterpret_cast<const __half2*>(&vsw.y));
  const float2 vz01 = __half22float2(*reinterpret_cast<const __half2*>(&vzw.x)), vz23 = __half22float2(*reinterpret_cast<const __half2*>(&vzw.y));
  const float vs[4] = {vs01.x, vs01.y, vs23.x, vs23.y}, vz[4] = {vz01.x, vz01.y, vz23.x, vz23.y};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 vs2 = f2(vs[i], vs[i]), vz2 = f2(vz[i], vz[i]);
    float2 u[4];
    codes8(*reinterpret_cast<const uint2*>(raw + 1024 + (t0 + i) * 64 + 8 * gq), u);
    float2 v[4];
#pragma unroll
    for (int x = 0; x < 4; ++x) v[x] = __ffma2_rn(u[x], vs2, vz2);
    uint4 o;
    o.x = pack_bf2(v[0].x, v[0].y);
    o.y = pack_bf2(v[1].x, v[1].y);
    o.z = pack_bf2(v[2].x, v[2].y);
    o.w = pack_bf2(v[3].x, v[3].y);
    *reinterpret_cast<uint4*>(vt + dst[i]) = o;
  }
}

template <int G>
__global__ void __launch_bounds__(kMmaThreads, kMmaCtasPerSm) attn_mma_kernel(const __grid_constant__ MmaParams mp) {
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "query group");
  constexpr int D = 64, BS = 16;
  const AttnParams& p = mp.p;
  extern __shared__ unsigned char smem_raw[];
  __shared__ int sh_bad;
  unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int j = blockIdx.y;
  int split = blockIdx.x, si = 0;
  if (p.n_segs > 1 && split >= p.seg[0].n_splits) {
    si = 1;
    split -= p.seg[0].n_splits;
  }
  const Seg& S = p.seg[si];
  const bool list = S.kind == SEG_LIST;
  const bool rec = S.kind == SEG_RANGE_REC;
  const CUtensorMap* tk = &mp.tk[si];
  const CUtensorMap* tv = &mp.tv[si];
  const bool head_major = mp.head_major[si] != 0;

  // Shared memory: hot/pairs segments use kMmaStages stages of (K tile, V tile) per warp; record
  // segments a (K tile, V tile) pair per warp followed by kMmaStages raw record stages per warp.
  unsigned char* tiles = smem + warp * 2 * kMmaTile;  // record segments only
  unsigned char* stage0 = rec ? smem + kMmaWarps * 2 * kMmaTile + warp * kMmaStages * kMmaRecStage : smem + warp * kMmaStages * kMmaHotStage;
  const int stage_stride = rec ? kMmaRecStage : kMmaHotStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kMmaBody) + warp * kMmaStages;
  if (threadIdx.x == 0) sh_bad = 0;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kMmaStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // Q^T fragments (bf16, exact): b0 = q[g][16ks + 2t .. +1], b1 = q[g][16ks + 2t + 8 .. +9].
  uint32_t bq[4][2];
  {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(static_cast<const __nv_bfloat16*>(p.q) + ((int64_t)j * G + (g < G ? g : 0)) * D);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      bq[ks][0] = g < G ? q[(16 * ks + 2 * t) / 2] : 0u;
      bq[ks][1] = g < G ? q[(16 * ks + 2 * t + 8) / 2] : 0u;
    }
  }
  // ldmatrix lane offsets within a tile: K (non-transposed, k-step ks) and V (transposed, m-tile mt).
  uint32_t koff[4], voff[4];
  {
    const int i = lane >> 3, r7 = lane & 7;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      koff[x] = swz(r7 + 8 * (i & 1), 2 * x + (i >> 1));
      voff[x] = swz(r7 + 8 * (i >> 1), 2 * x + (i & 1));
    }
  }

  float o[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) o[a][b] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

  const int begin = split * S.chunk;
  const int end = min(S.n_items, begin + S.chunk);
  uint32_t excl_word = 0;
  const int w0 = (S.first_block + begin) / 32;
  if (!list) {
    const int w = w0 + lane;
    excl_word = (S.excluded != nullptr && w < S.bitmap_words && w * 32 < S.first_block + end)
                    ? __ldg(S.excluded + (int64_t)j * S.bitmap_words + w) : 0u;
  }
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
      it += kMmaWarps;
    }
    return end;
  };
  int row_cache = 0, cache_batch = -1;
  auto list_row = [&](int n) -> int {
    const int batch = n >> 5;
    if (batch != cache_batch) {
      const int my_it = begin + warp + (batch * 32 + lane) * kMmaWarps;
      int r = 0;
      if (my_it < end) {
        const int blk = __ldg(S.blocks + (int64_t)j * S.n_list + my_it);
        r = blk < 0 ? -1 : (S.slot_of != nullptr ? __ldg(S.slot_of + (int64_t)j * S.slot_stride + blk) : blk);
      }
      row_cache = r;
      cache_batch = batch;
    }
    return __shfl_sync(0xffffffffu, row_cache, n & 31);
  };
  uint32_t pad_bits = 0;  // stages holding a padding item (no copy, nothing to attend)
  auto issue = [&](int it, int n, int s) {
    unsigned char* dst = stage0 + s * stage_stride;
    const int row = list ? list_row(n) : S.first_block + it;
    pad_bits = (pad_bits & ~(1u << s)) | ((row < 0 ? 1u : 0u) << s);
    if (row < 0) {
      if (lane == 0) mbar_arrive(&bars[s]);
    } else if (lane == 0) {
      if (rec) {
        mbar_arrive_expect_tx(&bars[s], (uint32_t)kMmaRec);
        tma_load_1d(dst, S.records + ((int64_t)row * p.h + j) * S.width, (uint32_t)kMmaRec, &bars[s]);
      } else {
        mbar_arrive_expect_tx(&bars[s], (uint32_t)kMmaHotStage);
        const int c2 = head_major ? j : row, c3 = head_major ? row : j;
        tma_load_4d(smem_u32(dst), tk, 0, 0, c2, c3, &bars[s]);
        tma_load_4d(smem_u32(dst + kMmaTile), tv, 0, 0, c2, c3, &bars[s]);
      }
    }
  };

  int issue_it = next_item(begin + warp), n_issued = 0;
#pragma unroll 1
  for (int s = 0; s < kMmaStages; ++s) {
    if (issue_it < end) {
      issue(issue_it, n_issued, s);
      ++n_issued;
      issue_it = next_item(issue_it + kMmaWarps);
    }
  }

  uint32_t phase = 0;
  int s = 0, n_done = 0;
  bool ok = true;
#pragma unroll 1
  for (int it = next_item(begin + warp); it < end; it = next_item(it + kMmaWarps)) {
    ok = __all_sync(0xffffffffu, mbar_wait(&bars[s], (phase >> s) & 1u));
    if (!ok) break;
    phase ^= 1u << s;
    ++n_done;
    unsigned char* st = stage0 + s * stage_stride;
    if ((pad_bits >> s) & 1u) {  // padding: nothing to attend; the stage is free
      if (issue_it < end) {
        issue(issue_it, n_issued, s);
        ++n_issued;
        issue_it = next_item(issue_it + kMmaWarps);
      }
      s = (s + 1 == kMmaStages) ? 0 : s + 1;
      continue;
    }
    uint32_t kt, vt;
    if (rec) {
      dequant_record(st, tiles, tiles + kMmaTile, lane);
      __syncwarp();
      // The raw stage is free again: refill it before the contractions.
      if (issue_it < end) {
        issue(issue_it, n_issued, s);
        ++n_issued;
        issue_it = next_item(issue_it + kMmaWarps);
      }
      kt = smem_u32(tiles);
      vt = kt + kMmaTile;
    } else {
      kt = smem_u32(st);
      vt = kt + kMmaTile;
    }

    // ---- S^T = K . Q^T ----
    float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ks = 0; ks < 4; ks += 2) {
      uint32_t a[4], b[4];
      ldsm_x4(kt + koff[ks], a);
      ldsm_x4(kt + koff[ks + 1], b);
      mma_bf16(sa, a, bq[ks][0], bq[ks][1]);
      mma_bf16(sb, b, bq[ks + 1][0], bq[ks + 1][1]);
    }
    // Lane scores: x0 (token g, row 2t), x1 (token g, row 2t+1), x2 / x3 (token g + 8).
    float x0 = (sa[0] + sb[0]) * p.scale_log2, x1 = (sa[1] + sb[1]) * p.scale_log2;
    float x2 = (sa[2] + sb[2]) * p.scale_log2, x3 = (sa[3] + sb[3]) * p.scale_log2;
    if (list && it == S.n_list - 1) {
      if (g >= S.last_fill) x0 = x1 = -INFINITY;
      if (g + 8 >= S.last_fill) x2 = x3 = -INFINITY;
    }
    // ---- softmax update (lazy rescaling, as the CUDA-core kernels) ----
    const bool need = x0 > m0 + kLazy || x2 > m0 + kLazy || x1 > m1 + kLazy || x3 > m1 + kLazy;
    if (__any_sync(0xffffffffu, need)) {
      float mb0 = fmaxf(x0, x2), mb1 = fmaxf(x1, x3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mb0 = fmaxf(mb0, __shfl_xor_sync(0xffffffffu, mb0, off));
        mb1 = fmaxf(mb1, __shfl_xor_sync(0xffffffffu, mb1, off));
      }
      if (mb0 > m0 + kLazy) {
        const float alpha = exp2f(m0 - mb0);  // 0 when m0 was -inf
        l0 *= alpha;
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          o[mt][0] *= alpha;
          o[mt][2] *= alpha;
        }
        m0 = mb0;
      }
      if (mb1 > m1 + kLazy) {
        const float alpha = exp2f(m1 - mb1);
        l1 *= alpha;
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          o[mt][1] *= alpha;
          o[mt][3] *= alpha;
        }
        m1 = mb1;
      }
    }
    const float p0 = m0 == -INFINITY ? 0.0f : ex2(x0 - m0);
    const float p2 = m0 == -INFINITY ? 0.0f : ex2(x2 - m0);
    const float p1 = m1 == -INFINITY ? 0.0f : ex2(x1 - m1);
    const float p3 = m1 == -INFINITY ? 0.0f : ex2(x3 - m1);
    l0 += p0 + p2;
    l1 += p1 + p3;
    // ---- P^T operand: three bf16 terms, transposed into the B layout ----
    uint32_t h01, m01, s01, h23, m23, s23;
    split3(p0, p1, h01, m01, s01);
    split3(p2, p3, h23, m23, s23);
    const uint32_t bh0 = movtrans(h01), bh1 = movtrans(h23);
    const uint32_t bm0 = movtrans(m01), bm1 = movtrans(m23);
    const uint32_t bl0 = movtrans(s01), bl1 = movtrans(s23);
    // ---- O^T += V^T . P^T ----
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      uint32_t a[4];
      ldsm_x4_t(vt + voff[mt], a);
      mma_bf16(o[mt], a, bl0, bl1);
      mma_bf16(o[mt], a, bm0, bm1);
      mma_bf16(o[mt], a, bh0, bh1);
    }
    __syncwarp();  // every lane is done with the stage (and the tiles) before they are refilled
    if (!rec && issue_it < end) {
      issue(issue_it, n_issued, s);
      ++n_issued;
      issue_it = next_item(issue_it + kMmaWarps);
    }
    s = (s + 1 == kMmaStages) ? 0 : s + 1;
  }
  // After a timed-out wait, wait (bounded) for the copies still in flight.
  for (int k = n_done; !ok && k < n_issued; ++k) {
    if (!__all_sync(0xffffffffu, mbar_wait(&bars[s], (phase >> s) & 1u))) break;
    phase ^= 1u << s;
    s = (s + 1 == kMmaStages) ? 0 : s + 1;
  }
  if (!ok && lane == 0) atomicExch(&sh_bad, 1);

  // ---- epilogue: per-warp partials through shared memory (the stages are idle now) ----
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  __syncthreads();
  float* out = p.part + ((int64_t)j * p.n_splits_total + blockIdx.x) * G * (D + 2);
  if (sh_bad) {
    for (int e = threadIdx.x; e < G * (D + 2); e += blockDim.x) out[e] = e < G ? -INFINITY : 0.0f;
    return;
  }
  float* sh_o = reinterpret_cast<float*>(smem);           // [warp][G][D]
  float* sh_ml = sh_o + kMmaWarps * G * D;                // [warp][m(G) | l(G)]
  const int r0 = 2 * t, r1 = 2 * t + 1;
#pragma unroll
  for (int mt = 0; mt < 4; ++mt) {
    if (r0 < G) {
      sh_o[(warp * G + r0) * D + 16 * mt + g] = o[mt][0];
      sh_o[(warp * G + r0) * D + 16 * mt + g + 8] = o[mt][2];
    }
    if (r1 < G) {
      sh_o[(warp * G + r1) * D + 16 * mt + g] = o[mt][1];
      sh_o[(warp * G + r1) * D + 16 * mt + g + 8] = o[mt][3];
    }
  }
  if (g == 0) {
    if (r0 < G) {
      sh_ml[warp * 2 * G + r0] = m0;
      sh_ml[warp * 2 * G + G + r0] = l0;
    }
    if (r1 < G) {
      sh_ml[warp * 2 * G + r1] = m1;
      sh_ml[warp * 2 * G + G + r1] = l1;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int r = e / D, c = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kMmaWarps; ++w) M = fmaxf(M, sh_ml[w * 2 * G + r]);
    float O = 0.0f, Lr = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kMmaWarps; ++w) {
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
    if (e != cudaSuccess) return fail(LKV_ERR_CUDA, "attention: shared memory attribute: %s", cudaGetErrorString(e));
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

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    else
      cudaGetLastError();
  }
  return fn;
}

// K and V maps of a list or pairs segment: 4-D bf16 tensors (channel, token, row, head) with a box of
// one 16 x 64 block, 128-byte swizzle. The row and head dimensions are ordered by stride.
bool make_kv_maps(const Seg& S, int h, CUtensorMap* tk, CUtensorMap* tv, int* head_major) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr || S.n_rows <= 0) return false;
  const int64_t es = 2;
  const int64_t st = S.s_tok * es, sr = S.s_row * es, sh = S.s_head * es;
  const bool hm = sh < sr;
  const cuuint64_t dims[4] = {64, 16, (cuuint64_t)(hm ? h : S.n_rows), (cuuint64_t)(hm ? S.n_rows : h)};
  const cuuint64_t strides[3] = {(cuuint64_t)st, (cuuint64_t)(hm ? sh : sr), (cuuint64_t)(hm ? sr : sh)};
  const cuuint32_t box[4] = {64, 16, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  for (int i = 0; i < 2; ++i) {
    CUresult r = enc(i == 0 ? tk : tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(i == 0 ? S.k_base : S.v_base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
  }
  *head_major = hm ? 1 : 0;
  return true;
}

// Whether the tensor-core kernel takes this launch (bf16, d 64, bs 16, G <= 8, stores in device
// memory, 64-channel token rows); fills the tensor maps of its list / pairs segments.
bool mma_plan(const AttnParams& p, int g, int d, bool bf16, MmaParams& mp) {
  if (!bf16 || d != 64 || p.bs != 16 || (g != 1 && g != 2 && g != 4 && g != 8)) return false;
  for (int i = 0; i < p.n_segs; ++i) {
    const Seg& S = p.seg[i];
    if (S.n_items == 0) continue;
    if (S.kind == SEG_RANGE_REC) {
      if (S.width != kMmaRec || is_host_mapped(S.records)) return false;
    } else {
      if (S.s_tok != d || is_host_mapped(S.k_base) || is_host_mapped(S.v_base)) return false;
      if (!make_kv_maps(S, p.h, &mp.tk[i], &mp.tv[i], &mp.head_major[i])) return false;
    }
  }
  return true;
}

template <int G>
int launch_mma(const MmaParams& mp, cudaStream_t st) {
  static uint64_t attr_set = 0;  // one bit per device
  auto k = attn_mma_kernel<G>;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set & bit)) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMmaSmem);
    if (e != cudaSuccess) return fail(LKV_ERR_CUDA, "attention: shared memory attribute: %s", cudaGetErrorString(e));
    attr_set |= bit;
  }
  k<<<dim3(mp.p.n_splits_total, mp.p.h), kMmaThreads, kMmaSmem, st>>>(mp);
  return LKV_OK;
}

// Splits, workspace check and launch of one attention call (partials + combine).
template <typename T, typename TO>
int run_attention(const char* who, AttnParams& p, int g, int d, TO* out, float* lse, float* seg_out, float* seg_lse, size_t workspace_bytes,
                  cudaStream_t st) {
  MmaParams mp{};
  const bool mma = mma_plan(p, g, d, sizeof(T) == 2, mp);
  const int total = mma ? kMmaTargetCtas : kTargetCtas;
  if (p.n_segs == 1) {
    set_split(p.seg[0], (total + p.h - 1) / p.h);
    p.n_splits_total = p.seg[0].n_splits;
  } else {
    if (mma) {
      // Tensor-core costs per item, relative: a listed block 1; a cold record about 2.5 (the fused
      // dequantisation), of which the range's excluded blocks (about the listed ones) cost little.
      const double n_cold = p.seg[1].n_items > 0 ? p.seg[1].n_items : 1;
      const double live = fmax(0.0, n_cold - fmax(0.0, p.seg[0].n_items - 2.0)) / n_cold;
      const double cold_cost = p.seg[1].kind == SEG_RANGE_REC ? 2.5 : 1.0;
      split_two(p.seg[0], p.seg[1], p.h, 1.0, cold_cost * live + 0.05, total);
    } else {
      split_two(p.seg[0], p.seg[1], p.h, 4096, 2368, total);
    }
    p.n_splits_total = p.seg[0].n_splits + p.seg[1].n_splits;
  }
  const size_t need = partial_bytes(p.h, g, d, p.n_splits_total);
  if (workspace_bytes < need) return fail(LKV_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", who, workspace_bytes, need);
  if (!mma) return dispatch<T, TO>(g, d, p, out, lse, seg_out, seg_lse, st);
  if constexpr (sizeof(T) == 2) {
    mp.p = p;
    int rc = LKV_OK;
    if (p.n_splits_total > 0) {
      switch (g) {
        case 1: rc = launch_mma<1>(mp, st); break;
        case 2: rc = launch_mma<2>(mp, st); break;
        case 4: rc = launch_mma<4>(mp, st); break;
        default: rc = launch_mma<8>(mp, st); break;
      }
    }
    if (rc) return rc;
    const int n0 = p.seg[0].n_splits, n1 = p.n_segs > 1 ? p.seg[1].n_splits : 0;
    switch (g) {
      case 1: attn_combine_kernel<TO, 1, 64><<<dim3(p.h, 1), kCombineThreads, 0, st>>>(p.part, n0, n1, out, lse, seg_out, seg_lse, p.hq); break;
      case 2: attn_combine_kernel<TO, 2, 64><<<dim3(p.h, 2), kCombineThreads, 0, st>>>(p.part, n0, n1, out, lse, seg_out, seg_lse, p.hq); break;
      case 4: attn_combine_kernel<TO, 4, 64><<<dim3(p.h, 4), kCombineThreads, 0, st>>>(p.part, n0, n1, out, lse, seg_out, seg_lse, p.hq); break;
      default: attn_combine_kernel<TO, 8, 64><<<dim3(p.h, 8), kCombineThreads, 0, st>>>(p.part, n0, n1, out, lse, seg_out, seg_lse, p.hq); break;
    }
    return launched("lkv attention");
  }
  return fail(LKV_ERR_ARG, "%s: unreachable", who);
}

}  // namespace
}  // namespace lkv

using namespace lkv;

extern "C" {

int lkv_device_status(int* status, int clear) {
  if (status == nullptr) return fail(LKV_ERR_PTR, "lkv_device_status: null pointer");
  cudaError_t e = cudaMemcpyFromSymbol(status, g_device_status, sizeof(int));
  if (e == cudaSuccess && clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
  }
  if (e != cudaSuccess) return fail(LKV_ERR_CUDA, "lkv_device_status: %s", cudaGetErrorString(e));
  return LKV_OK;
}

size_t lkv_attention_workspace(int h, int hq, int d, int n_items) {
  if (h <= 0 || hq <= 0) return 0;
  const int s = splits_for(n_items, (kMmaTargetCtas + h - 1) / h);
  const size_t b = partial_bytes(h, hq / h, d, s);
  return b > 0 ? b : 16;
}

size_t lkv_exact_attention_workspace(int h, int hq, int d, int n_list, int n_blocks) {
  if (h <= 0 || hq <= 0) return 0;
  Seg a{}, b{};
  a.n_items = n_list;
  b.n_items = n_blocks;
  split_two(a, b, h, 4096, 2368, kMmaTargetCtas);
  const int per_head = (kMmaTargetCtas + h - 1) / h + 1;  // any split of the target between the segments
  const size_t s = partial_bytes(h, hq / h, d, per_head > a.n_splits + b.n_splits ? per_head : a.n_splits + b.n_splits);
  return s > 0 ? s : 16;
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
  p.part = static_cast<float*>(workspace);
  cudaStream_t st = as_stream(stream);
  return dtype == LKV_BF16 ? run_attention<__nv_bfloat16, float>("lkv_hot_attention", p, hq / h, d, out, lse, nullptr, nullptr, workspace_bytes, st)
                           : run_attention<float, float>("lkv_hot_attention", p, hq / h, d, out, lse, nullptr, nullptr, workspace_bytes, st);
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
  p.part = static_cast<float*>(workspace);
  cudaStream_t st = as_stream(stream);
  return dtype == LKV_BF16 ? run_attention<__nv_bfloat16, float>("lkv_cold_attention", p, hq / h, d, out, lse, nullptr, nullptr, workspace_bytes, st)
                           : run_attention<float, float>("lkv_cold_attention", p, hq / h, d, out, lse, nullptr, nullptr, workspace_bytes, st);
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
  p.part = static_cast<float*>(workspace);
  cudaStream_t st = as_stream(stream);
  const int g = hq / h;
  const bool bf = hot->dtype == LKV_BF16;
  const char* who = "lkv_exact_attention";
  if (out_dtype == LKV_BF16)
    return bf ? run_attention<__nv_bfloat16, __nv_bfloat16>(who, p, g, d, static_cast<__nv_bfloat16*>(out), lse, part_out, part_lse, workspace_bytes, st)
              : run_attention<float, __nv_bfloat16>(who, p, g, d, static_cast<__nv_bfloat16*>(out), lse, part_out, part_lse, workspace_bytes, st);
  return bf ? run_attention<__nv_bfloat16, float>(who, p, g, d, static_cast<float*>(out), lse, part_out, part_lse, workspace_bytes, st)
            : run_attention<float, float>(who, p, g, d, static_cast<float*>(out), lse, part_out, part_lse, workspace_bytes, st);
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
