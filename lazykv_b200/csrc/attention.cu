// K4/K5/K6: split decode attention over listed or remaining blocks, and the log-sum-exp merge.
//
// One launch serves either pass of lazykv/exact.py's set split, or both at once:
//  * hot segment (lazykv/tiered.py:465-487 + lazykv/attention.py:125-136): the key sequence of KV
//    head j is the n_list listed blocks, read in place through an optional block->slot map (no
//    gather copy); the last listed block is the current block with `last_fill` live tokens
//    (selection.py:65-69);
//  * cold segment (lazykv/exact.py:88-127): blocks [first, first + n) minus a per-head exclusion
//    bitmap, read from int8 records with the dequantisation fused (quant.py:103-104, float32
//    affine), or from pairs in the model dtype.
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
        for (int c = 0; c < CPL; ++c) kv[c] = fmaf(kv[c], ks[c], kz[c]);
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
        for (int c = 0; c < CPL; ++c) kv[c] = fmaf(kv[c], vs, vz);
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
  float m[G], l[G], zs[G];
  float2 o2[G][8];
#pragma unroll
  for (int r = 0; r < G; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
    zs[r] = 0.0f;
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
        r = S.slot_of != nullptr ? __ldg(S.slot_of + (int64_t)j * S.slot_stride + blk) : blk;
      }
      row_cache = r;
      cache_batch = batch;
    }
    return (int64_t)__shfl_sync(0xffffffffu, row_cache, n & 31);
  };
  // Issue the copies of item `it` (the n-th of this warp) into stage `s`; lane 0 issues.
  auto issue = [&](int it, int n, int s) {
    unsigned char* dst = stages + (size_t)s * C::STAGE;
    if (list) {
      const int64_t row = list_row(it, n);
      if (lane == 0) {
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
        for (int w = 0; w < 8; ++w) k2[w] = __ffma2_rn(u[w], ks2[w], kz2[w]);
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
          zs[r] *= alpha;
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
        // o += p * (u * vs + vz) = (p * vs) * u + p * vz; the second term is channel-independent.
        codes16(st + BS * D + t * D + c0, v2);
        const float vs = scl[2 * C::SCL_K + 2 * t], vz = scl[2 * C::SCL_K + 2 * t + 1];
#pragma unroll
        for (int r = 0; r < G; ++r) {
          const float w = pr[r][i] * vs;
          zs[r] = fmaf(pr[r][i], vz, zs[r]);
          const float2 ww = f2(w, w);
#pragma unroll
          for (int x = 0; x < 8; ++x) o2[r][x] = __ffma2_rn(ww, v2[x], o2[r][x]);
        }
      } else {
        lds_row16<T>(reinterpret_cast<const T*>(st) + BS * D + t * D + c0, swap, v2);
#pragma unroll
        for (int r = 0; r < G; ++r) {
          const float2 pp = f2(pr[r][i], pr[r][i]);
#pragma unroll
          for (int x = 0; x < 8; ++x) o2[r][x] = __ffma2_rn(pp, v2[x], o2[r][x]);
        }
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
    const float2 z2 = f2(zs[r], zs[r]);
#pragma unroll
    for (int w = 0; w < 8; ++w) o2[r][w] = __fadd2_rn(o2[r][w], z2);
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
// combine and merge
// ============================================================================================

// Fold the splits of each segment (segment 0: [0, n0), segment 1: [n0, n0 + n1)) of each (head,
// query row) into per-segment (out, lse) and their merge. One CTA per (head, row): the threads split
// the channels x the splits so the partials are read with independent loads. Outputs may be null.
constexpr int kCombineThreads = 256;

template <typename TO, int G, int D>
__global__ void __launch_bounds__(kCombineThreads) attn_combine_kernel(const float* __restrict__ part, int n0, int n1, TO* __restrict__ out,
                                                                       float* __restrict__ lse, float* __restrict__ seg_out,
                                                                       float* __restrict__ seg_lse, int hq) {
  constexpr int KS = kCombineThreads / D;  // split lanes per channel
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
#pragma unroll
  for (int sgi = 0; sgi < 2; ++sgi) {
    const int a = sgi == 0 ? 0 : n0, b = sgi == 0 ? n0 : nt;
    float mloc = -INFINITY;
    for (int sp = a + threadIdx.x; sp < b; sp += kCombineThreads) mloc = fmaxf(mloc, base[sp * stride + r]);
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
        const float ms = ps[r];
        const float f = ms == -INFINITY ? 0.0f : exp2f(ms - M);
        O = fmaf(ps[2 * G + r * D + c], f, O);
        L = fmaf(ps[G + r], f, L);
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
__global__ void lse_merge_kernel(const float* __restrict__ outs, const float* __restrict__ lses, int n_parts, int64_t rows, int d,
                                 T* __restrict__ out, float* __restrict__ lse_out) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= rows * d) return;
  const int64_t r = e / d;
  float M = -INFINITY;
  for (int k = 0; k < n_parts; ++k) M = fmaxf(M, lses[k * rows + r]);
  float acc = 0.0f, lse = -INFINITY;
  if (M != -INFINITY) {
    float sum = 0.0f;
    for (int k = 0; k < n_parts; ++k) sum += expf(lses[k * rows + r] - M);
    lse = M + logf(sum);
    for (int k = 0; k < n_parts; ++k) {
      const float w = expf(lses[k * rows + r] - lse);
      acc = fmaf(w, outs[(int64_t)k * rows * d + e], acc);
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
  }
  S.first_block = cs->first_block; S.excluded = cs->excluded; S.bitmap_words = cs->bitmap_words;
  S.n_items = cs->n_blocks;
  return LKV_OK;
}

// Split the target CTA count between two segments in proportion to their bytes.
void split_two(Seg& hot, Seg& cold, int h, int hot_item_bytes, int cold_item_bytes) {
  const int target = (kTargetCtas + h - 1) / h;
  const double wh = (double)hot.n_items * hot_item_bytes, wc = (double)cold.n_items * cold_item_bytes;
  int th = wh + wc > 0 ? (int)(target * wh / (wh + wc) + 0.5) : 0;
  if (hot.n_items > 0 && th < 1) th = 1;
  int tc = target - th;
  if (cold.n_items > 0 && tc < 1) tc = 1;
  set_split(hot, th);
  set_split(cold, tc);
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
  const int s = splits_for(n_items, (kTargetCtas + h - 1) / h);
  const size_t b = partial_bytes(h, hq / h, d, s);
  return b > 0 ? b : 16;
}

size_t lkv_exact_attention_workspace(int h, int hq, int d, int n_list, int n_blocks) {
  if (h <= 0 || hq <= 0) return 0;
  Seg a{}, b{};
  a.n_items = n_list;
  b.n_items = n_blocks;
  split_two(a, b, h, 4096, 2368);
  const size_t s = partial_bytes(h, hq / h, d, a.n_splits + b.n_splits);
  return s > 0 ? s : 16;
}

int lkv_hot_attention(const void* q, int hq, int h, int d, int bs, const void* k_base, const void* v_base, int dtype, int64_t s_row,
                      int64_t s_head, int64_t s_tok, const int32_t* blocks, int n_list, const int32_t* slot_of, int64_t slot_stride,
                      int last_fill, float scale, float* out, float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = common_checks("lkv_hot_attention", q, hq, h, d, bs, dtype, workspace)) return rc;
  if (out == nullptr || lse == nullptr) return fail(LKV_ERR_PTR, "lkv_hot_attention: null pointer");
  lkv_hot_set hs{k_base, v_base, dtype, s_row, s_head, s_tok, blocks, n_list, slot_of, slot_stride, last_fill};
  AttnParams p{};
  p.q = q; p.hq = hq; p.h = h; p.bs = bs; p.scale_log2 = scale * kLog2e;
  if (int rc = fill_hot("lkv_hot_attention", p.seg[0], h, d, bs, &hs)) return rc;
  p.n_segs = 1;
  set_split(p.seg[0], (kTargetCtas + h - 1) / h);
  p.n_splits_total = p.seg[0].n_splits;
  p.part = static_cast<float*>(workspace);
  if (workspace_bytes < partial_bytes(h, hq / h, d, p.n_splits_total))
    return fail(LKV_ERR_WORKSPACE, "lkv_hot_attention: workspace %zu < %zu bytes", workspace_bytes, partial_bytes(h, hq / h, d, p.n_splits_total));
  cudaStream_t st = as_stream(stream);
  return dtype == LKV_BF16 ? dispatch<__nv_bfloat16, float>(hq / h, d, p, out, lse, nullptr, nullptr, st)
                           : dispatch<float, float>(hq / h, d, p, out, lse, nullptr, nullptr, st);
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
  set_split(p.seg[0], (kTargetCtas + h - 1) / h);
  p.n_splits_total = p.seg[0].n_splits;
  p.part = static_cast<float*>(workspace);
  if (workspace_bytes < partial_bytes(h, hq / h, d, p.n_splits_total))
    return fail(LKV_ERR_WORKSPACE, "lkv_cold_attention: workspace %zu < %zu bytes", workspace_bytes, partial_bytes(h, hq / h, d, p.n_splits_total));
  cudaStream_t st = as_stream(stream);
  return dtype == LKV_BF16 ? dispatch<__nv_bfloat16, float>(hq / h, d, p, out, lse, nullptr, nullptr, st)
                           : dispatch<float, float>(hq / h, d, p, out, lse, nullptr, nullptr, st);
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
  split_two(p.seg[0], p.seg[1], h, 4096, 2368);
  p.n_splits_total = p.seg[0].n_splits + p.seg[1].n_splits;
  p.part = static_cast<float*>(workspace);
  if (workspace_bytes < partial_bytes(h, hq / h, d, p.n_splits_total))
    return fail(LKV_ERR_WORKSPACE, "lkv_exact_attention: workspace %zu < %zu bytes", workspace_bytes, partial_bytes(h, hq / h, d, p.n_splits_total));
  cudaStream_t st = as_stream(stream);
  const int g = hq / h;
  const bool bf = hot->dtype == LKV_BF16;
  if (out_dtype == LKV_BF16)
    return bf ? dispatch<__nv_bfloat16, __nv_bfloat16>(g, d, p, static_cast<__nv_bfloat16*>(out), lse, part_out, part_lse, st)
              : dispatch<float, __nv_bfloat16>(g, d, p, static_cast<__nv_bfloat16*>(out), lse, part_out, part_lse, st);
  return bf ? dispatch<__nv_bfloat16, float>(g, d, p, static_cast<float*>(out), lse, part_out, part_lse, st)
            : dispatch<float, float>(g, d, p, static_cast<float*>(out), lse, part_out, part_lse, st);
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
    lse_merge_kernel<__nv_bfloat16><<<blocks, 256, 0, as_stream(stream)>>>(outs, lses, n_parts, rows, d, static_cast<__nv_bfloat16*>(out), lse_out);
  else
    lse_merge_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(outs, lses, n_parts, rows, d, static_cast<float*>(out), lse_out);
  return launched("lkv_lse_merge");
}

}  // extern "C"
