// K4/K5/K6: split decode attention over listed or remaining blocks, and the log-sum-exp merge.
//
// One kernel serves both passes of lazykv/exact.py's set split:
//  * hot (lazykv/tiered.py:465-487 + lazykv/attention.py:125-136): the key sequence of KV head j is
//    the n_list listed blocks, read in place through an optional block->slot map (no gather copy);
//    the last listed block is the current block with `last_fill` live tokens (selection.py:65-69);
//  * cold (lazykv/exact.py:88-127): blocks [first, first + n) minus a per-head exclusion bitmap,
//    read from int8 records with the dequantisation fused (quant.py:103-104), or from pairs.
// Each CTA takes a chunk of blocks of one KV head and emits an online-softmax partial (running max m
// in the log2 domain, sum l, unnormalised o) for the head's G query rows; a second kernel combines
// the chunks into (out = o / l, lse) per query row. A partial over no key is (m = -inf, l = 0),
// which the combine turns into lse = -inf and out = 0, as cpu_partial_attention does (exact.py:108-110).
//
// Lane layout in a warp: CG channel groups x TL token lanes (CG = 4 for d <= 64, 8 for d = 128); a
// lane holds CPL = d / CG channels of the G query rows and of its output accumulators, and takes
// tokens tl, tl + TL, ... of each block. Scores are reduced over the CG lanes of a token, block
// maxima over the TL token lanes. Blocks of a chunk are dealt round-robin to the CTA's 4 warps.
#include "common.cuh"

namespace lkv {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kMinChunk = 16;               // blocks per CTA at least (4 per warp)
constexpr int kTargetCtas = 3 * kNumSMs;    // about three resident CTAs per SM
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnParams {
  const void* q;
  int hq, h, bs;
  float scale_log2;
  // strided pairs in the model dtype (hot pool, full cache, or a bf16/f32 cold store)
  const void* k_base;
  const void* v_base;
  int64_t s_row, s_head, s_tok;
  // int8 records [blocks, h, width]
  const uint8_t* records;
  int64_t width;
  // item -> block: listed (blocks != null) or a range with an exclusion bitmap
  const int32_t* blocks;
  int n_list, last_fill;
  const int32_t* slot_of;
  int64_t slot_stride;
  int first_block;
  const uint32_t* excluded;
  int bitmap_words;
  int n_items, chunk, n_splits;
  float* part;  // [h][n_splits][G][D + 2]
};

int choose_splits(int n_items, int h) {
  if (n_items <= 0) return 0;
  int by_size = (n_items + kMinChunk - 1) / kMinChunk;
  int by_grid = (kTargetCtas + h - 1) / h;
  int s = by_size < by_grid ? by_size : by_grid;
  if (s < 1) s = 1;
  const int chunk = (n_items + s - 1) / s;
  return (n_items + chunk - 1) / chunk;
}

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

template <typename T, int G, int D, bool INT8>
__global__ void __launch_bounds__(kThreads) attn_partial_kernel(const AttnParams p) {
  constexpr int CG = D >= 128 ? 8 : 4;
  constexpr int CPL = D / CG;
  constexpr int TL = 32 / CG;
  __shared__ float sh_m[kWarps][G], sh_l[kWarps][G];
  __shared__ float sh_o[kWarps][G][D];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cg = lane % CG, tl = lane / CG;
  const int j = blockIdx.y, split = blockIdx.x;
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

  const int begin = split * p.chunk;
  const int end = min(p.n_items, begin + p.chunk);
  for (int it = begin + warp; it < end; it += kWarps) {
    int blk, live = p.bs;
    if (p.blocks != nullptr) {
      blk = __ldg(p.blocks + (int64_t)j * p.n_list + it);
      if (it == p.n_list - 1) live = p.last_fill;
    } else {
      blk = p.first_block + it;
      if (p.excluded != nullptr && blk / 32 < p.bitmap_words &&
          ((__ldg(p.excluded + (int64_t)j * p.bitmap_words + blk / 32) >> (blk % 32)) & 1u))
        continue;
    }
    const T* kp = nullptr;
    const T* vp = nullptr;
    const uint8_t* rec = nullptr;
    float ks[CPL], kz[CPL];
    if constexpr (INT8) {
      rec = p.records + ((int64_t)blk * p.h + j) * p.width;
      const uint8_t* sc = rec + 2ll * p.bs * D;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        ks[c] = ldh(sc + 2 * (c0 + c));
        kz[c] = ldh(sc + 2 * D + 2 * (c0 + c));
      }
    } else {
      const int64_t row = p.slot_of != nullptr ? (int64_t)__ldg(p.slot_of + (int64_t)j * p.slot_stride + blk) : (int64_t)blk;
      kp = static_cast<const T*>(p.k_base) + row * p.s_row + (int64_t)j * p.s_head;
      vp = static_cast<const T*>(p.v_base) + row * p.s_row + (int64_t)j * p.s_head;
    }
    for (int t0 = 0; t0 < p.bs; t0 += TL) {
      const int t = t0 + tl;
      float kv[CPL];
      if constexpr (INT8) {
        load_codes<CPL>(rec + (int64_t)t * D + c0, kv);
#pragma unroll
        for (int c = 0; c < CPL; ++c) kv[c] = fmaf(kv[c], ks[c], kz[c]);
      } else {
        load_chunk<T, CPL>(kp + t * p.s_tok + c0, kv);
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
      if constexpr (INT8) {
        const uint8_t* sc = rec + 2ll * p.bs * D + 4 * D;
        const float vs = ldh(sc + 2 * t), vz = ldh(sc + 2 * p.bs + 2 * t);
        load_codes<CPL>(rec + (int64_t)p.bs * D + (int64_t)t * D + c0, kv);
#pragma unroll
        for (int c = 0; c < CPL; ++c) kv[c] = fmaf(kv[c], vs, vz);
      } else {
        load_chunk<T, CPL>(vp + t * p.s_tok + c0, kv);
      }
#pragma unroll
      for (int r = 0; r < G; ++r)
#pragma unroll
        for (int c = 0; c < CPL; ++c) o[r][c] = fmaf(pr[r], kv[c], o[r][c]);
    }
  }

  // Reduce over the token lanes (m is uniform within the warp).
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
        // l was accumulated once per token lane and once per channel group: the CG lanes of a
        // token hold the same value, so the sum over token lanes is the block sum.
        sh_l[warp][r] = l[r];
      }
    }
  }
  __syncthreads();
  float* out = p.part + ((int64_t)j * p.n_splits + split) * G * (D + 2);
  for (int e = threadIdx.x; e < G * D; e += kThreads) {
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

// Combine the n_splits partials of each (head, query row) into (out = o / l, lse).
template <int G, int D>
__global__ void attn_combine_kernel(const float* __restrict__ part, int n_splits, float* __restrict__ out,
                                    float* __restrict__ lse) {
  const int j = blockIdx.x;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int r = e / D, c = e % D;
    float M = -INFINITY;
    for (int s = 0; s < n_splits; ++s) M = fmaxf(M, part[((int64_t)j * n_splits + s) * G * (D + 2) + r]);
    float O = 0.0f, L = 0.0f;
    if (M != -INFINITY) {
      for (int s = 0; s < n_splits; ++s) {
        const float* ps = part + ((int64_t)j * n_splits + s) * G * (D + 2);
        const float ms = ps[r];
        if (ms == -INFINITY) continue;
        const float f = exp2f(ms - M);
        L = fmaf(ps[G + r], f, L);
        O = fmaf(ps[2 * G + r * D + c], f, O);
      }
    }
    const int64_t row = (int64_t)j * G + r;
    const bool empty = !(L > 0.0f);
    out[row * D + c] = empty ? 0.0f : O / L;
    if (c == 0) lse[row] = empty ? -INFINITY : (M + log2f(L)) * kLn2;
  }
}

template <typename T>
__global__ void lse_merge_kernel(const float* __restrict__ outs, const float* __restrict__ lses, int n_parts,
                                 int64_t rows, int d, T* __restrict__ out, float* __restrict__ lse_out) {
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

template <typename T, int G, int D>
int launch_attn(AttnParams& p, bool int8, float* out, float* lse, cudaStream_t st) {
  if (p.n_splits > 0) {
    dim3 grid(p.n_splits, p.h);
    if (int8)
      attn_partial_kernel<T, G, D, true><<<grid, kThreads, 0, st>>>(p);
    else
      attn_partial_kernel<T, G, D, false><<<grid, kThreads, 0, st>>>(p);
  }
  const int threads = G * D < 1024 ? G * D : 1024;
  attn_combine_kernel<G, D><<<p.h, threads, 0, st>>>(p.part, p.n_splits, out, lse);
  return launched("lkv attention");
}

template <typename T>
int dispatch_attn(int g, int d, AttnParams& p, bool int8, float* out, float* lse, cudaStream_t st) {
#define LKV_D(G, D) \
  if (d == D) return launch_attn<T, G, D>(p, int8, out, lse, st);
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

int common_checks(const char* who, const void* q, int hq, int h, int d, int bs, int dtype, float* out, float* lse, void* ws) {
  if (!dtype_ok(dtype)) return fail(LKV_ERR_ARG, "%s: bad dtype %d", who, dtype);
  if (h <= 0 || hq <= 0 || hq % h != 0) return fail(LKV_ERR_ARG, "%s: %d query heads do not group over %d KV heads", who, hq, h);
  const int tl = 32 / (d >= 128 ? 8 : 4);
  if (bs <= 0 || bs % tl != 0) return fail(LKV_ERR_ARG, "%s: block size %d must be a multiple of %d", who, bs, tl);
  if (q == nullptr || out == nullptr || lse == nullptr || ws == nullptr) return fail(LKV_ERR_PTR, "%s: null pointer", who);
  return LKV_OK;
}

}  // namespace
}  // namespace lkv

using namespace lkv;

extern "C" {

size_t lkv_attention_workspace(int h, int hq, int d, int n_items) {
  if (h <= 0 || hq <= 0) return 0;
  const int s = choose_splits(n_items, h);
  const size_t b = partial_bytes(h, hq / h, d, s);
  return b > 0 ? b : 16;
}

int lkv_hot_attention(const void* q, int hq, int h, int d, int bs, const void* k_base, const void* v_base,
                      int dtype, int64_t s_row, int64_t s_head, int64_t s_tok, const int32_t* blocks,
                      int n_list, const int32_t* slot_of, int64_t slot_stride, int last_fill, float scale,
                      float* out, float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = common_checks("lkv_hot_attention", q, hq, h, d, bs, dtype, out, lse, workspace)) return rc;
  if (k_base == nullptr || v_base == nullptr || blocks == nullptr) return fail(LKV_ERR_PTR, "lkv_hot_attention: null pointer");
  if (n_list <= 0) return fail(LKV_ERR_ARG, "lkv_hot_attention: empty block list");
  if (last_fill < 0 || last_fill > bs) return fail(LKV_ERR_ARG, "lkv_hot_attention: last_fill %d outside [0, %d]", last_fill, bs);
  const size_t es = dtype_size(dtype);
  if (!aligned(k_base, 16) || !aligned(v_base, 16) || (s_row * es) % 16 || (s_head * es) % 16 || (s_tok * es) % 16)
    return fail(LKV_ERR_PTR, "lkv_hot_attention: KV rows must be 16-byte aligned");
  AttnParams p{};
  p.q = q; p.hq = hq; p.h = h; p.bs = bs; p.scale_log2 = scale * kLog2e;
  p.k_base = k_base; p.v_base = v_base; p.s_row = s_row; p.s_head = s_head; p.s_tok = s_tok;
  p.blocks = blocks; p.n_list = n_list; p.last_fill = last_fill; p.slot_of = slot_of; p.slot_stride = slot_stride;
  p.n_items = n_list;
  p.n_splits = choose_splits(n_list, h);
  p.chunk = (n_list + p.n_splits - 1) / p.n_splits;
  p.part = static_cast<float*>(workspace);
  if (workspace_bytes < partial_bytes(h, hq / h, d, p.n_splits))
    return fail(LKV_ERR_WORKSPACE, "lkv_hot_attention: workspace %zu < %zu bytes", workspace_bytes, partial_bytes(h, hq / h, d, p.n_splits));
  cudaStream_t st = as_stream(stream);
  return dtype == LKV_BF16 ? dispatch_attn<__nv_bfloat16>(hq / h, d, p, false, out, lse, st)
                           : dispatch_attn<float>(hq / h, d, p, false, out, lse, st);
}

int lkv_cold_attention(const void* q, int hq, int h, int d, int bs, const void* cold, int cold_kind, int dtype,
                       int first_block, int n_blocks, const uint32_t* excluded, int bitmap_words, float scale,
                       float* out, float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = common_checks("lkv_cold_attention", q, hq, h, d, bs, dtype, out, lse, workspace)) return rc;
  if (cold_kind != LKV_COLD_INT8 && cold_kind != LKV_COLD_PAIRS) return fail(LKV_ERR_ARG, "lkv_cold_attention: bad cold kind %d", cold_kind);
  if (n_blocks < 0 || first_block < 0) return fail(LKV_ERR_ARG, "lkv_cold_attention: bad block range");
  if (n_blocks > 0 && cold == nullptr) return fail(LKV_ERR_PTR, "lkv_cold_attention: null cold store");
  if (cold != nullptr && !aligned(cold, 16)) return fail(LKV_ERR_PTR, "lkv_cold_attention: cold store must be 16-byte aligned");
  AttnParams p{};
  p.q = q; p.hq = hq; p.h = h; p.bs = bs; p.scale_log2 = scale * kLog2e;
  if (cold_kind == LKV_COLD_INT8) {
    p.records = static_cast<const uint8_t*>(cold);
    p.width = lkv_packed_pair_bytes(bs, d);
  } else {
    // pairs [blocks, h, 2, bs, d]: a "row" is a block
    p.k_base = cold;
    p.v_base = static_cast<const char*>(cold) + (size_t)bs * d * dtype_size(dtype);
    p.s_row = (int64_t)h * 2 * bs * d; p.s_head = 2ll * bs * d; p.s_tok = d;
  }
  p.first_block = first_block; p.excluded = excluded; p.bitmap_words = bitmap_words;
  p.n_items = n_blocks;
  p.n_splits = choose_splits(n_blocks, h);
  p.chunk = p.n_splits > 0 ? (n_blocks + p.n_splits - 1) / p.n_splits : 0;
  p.part = static_cast<float*>(workspace);
  if (workspace_bytes < partial_bytes(h, hq / h, d, p.n_splits))
    return fail(LKV_ERR_WORKSPACE, "lkv_cold_attention: workspace %zu < %zu bytes", workspace_bytes, partial_bytes(h, hq / h, d, p.n_splits));
  cudaStream_t st = as_stream(stream);
  const bool int8 = cold_kind == LKV_COLD_INT8;
  return dtype == LKV_BF16 ? dispatch_attn<__nv_bfloat16>(hq / h, d, p, int8, out, lse, st)
                           : dispatch_attn<float>(hq / h, d, p, int8, out, lse, st);
}

int lkv_lse_merge(const float* outs, const float* lses, int n_parts, int64_t rows, int d, void* out, int out_dtype,
                  float* lse_out, void* stream) {
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
