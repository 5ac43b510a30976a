// int8 record codec and block metadata (K2 quantise-on-write, K7 dequantise-on-read, a4 min/max).
//
// Record layout, lazykv/quant.py:52-56 and :85-86, for one (block, head) pair:
//   kq int8 [bs][d] | vq int8 [bs][d] | k_scale f16 [d] | k_zero f16 [d] | v_scale f16 [bs] | v_zero f16 [bs]
// Keys are quantised per channel (range over the block's tokens), values per token (range over
// head_dim), lazykv/quant.py:83-84. Arithmetic follows lazykv/quant.py:59-70 and :103-104 operation
// by operation in float32 with explicit round-to-nearest intrinsics, so that no multiply-add is
// contracted and the bytes match the reference's CPU pack bit for bit.
#include <float.h>

#include "common.cuh"

namespace lkv {
namespace {

constexpr float kLevels = 255.0f;  // lazykv/quant.py:43

struct RecordLayout {
  int bs, d;
  int64_t width;
  __host__ __device__ int64_t kq() const { return 0; }
  __host__ __device__ int64_t vq() const { return (int64_t)bs * d; }
  __host__ __device__ int64_t ks() const { return 2ll * bs * d; }
  __host__ __device__ int64_t kz() const { return 2ll * bs * d + 2ll * d; }
  __host__ __device__ int64_t vs() const { return 2ll * bs * d + 4ll * d; }
  __host__ __device__ int64_t vz() const { return 2ll * bs * d + 4ll * d + 2ll * bs; }
};

__device__ __forceinline__ float half_at(const uint8_t* p) { return __half2float(*reinterpret_cast<const __half*>(p)); }

// One float32 dequantised value: (q + 128) * scale + zero, each operation rounded (quant.py:103-104).
__device__ __forceinline__ float dequant(int8_t q, float scale, float zero) {
  return __fadd_rn(__fmul_rn(__fadd_rn((float)q, 128.0f), scale), zero);
}

// One code: rint((x - mn) / scale) clamped to [0, 255], minus 128 (quant.py:69).
__device__ __forceinline__ int8_t quantise(float x, float mn, float scale) {
  float q = rintf(__fdiv_rn(__fsub_rn(x, mn), scale));
  q = fminf(fmaxf(q, 0.0f), kLevels);
  return (int8_t)((int)q - 128);
}

// ---- block min/max --------------------------------------------------------------------------

template <typename T>
__global__ void block_minmax_kernel(const T* __restrict__ keys, int n_blocks, int bs, int d,
                                    int64_t s_head, int64_t s_block, int64_t s_tok, T* kmin,
                                    T* kmax, int64_t m_head, int first_block) {
  const int j = blockIdx.y;
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (int64_t)n_blocks * d) return;
  const int b = (int)(e / d), c = (int)(e % d);
  const T* p = keys + j * s_head + b * s_block + c;
  float mn = to_f32<T>(p[0]), mx = mn;
  for (int t = 1; t < bs; ++t) {
    float x = to_f32<T>(p[t * s_tok]);
    mn = fminf(mn, x);
    mx = fmaxf(mx, x);
  }
  const int64_t o = j * m_head + (int64_t)(first_block + b) * d + c;
  kmin[o] = from_f32<T>(mn);
  kmax[o] = from_f32<T>(mx);
}

// ---- pack -------------------------------------------------------------------------------------

// One CTA per (block, head) pair; the pair is staged in shared memory as float.
template <typename T>
__global__ void pack_kernel(const T* __restrict__ pairs, int h, int bs, int d, uint8_t* records,
                            int64_t width, T* kmin, T* kmax, int64_t m_head, int first_block,
                            T* deq) {
  extern __shared__ float smem[];
  const int n = bs * d;
  float* x = smem;                 // [2][bs][d]
  float* kmn = x + 2 * n;          // [d]
  float* ksc = kmn + d;            // [d]
  float* vmn = ksc + d;            // [bs]
  float* vsc = vmn + bs;           // [bs]
  const int64_t p = blockIdx.x;    // pair index = block * h + head
  const int j = (int)(p % h), b = (int)(p / h);
  const T* src = pairs + p * 2 * n;
  for (int e = threadIdx.x; e < 2 * n; e += blockDim.x) x[e] = to_f32<T>(src[e]);
  __syncthreads();

  const RecordLayout L{bs, d, width};
  uint8_t* rec = records + p * width;
  // Keys: range over tokens, one (scale, zero) per channel.
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float mn = x[c], mx = mn;
    for (int t = 1; t < bs; ++t) {
      mn = fminf(mn, x[t * d + c]);
      mx = fmaxf(mx, x[t * d + c]);
    }
    float sc = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), kLevels), FLT_MIN);
    kmn[c] = mn;
    ksc[c] = sc;
    reinterpret_cast<__half*>(rec + L.ks())[c] = __float2half_rn(sc);
    reinterpret_cast<__half*>(rec + L.kz())[c] = __float2half_rn(mn);
  }
  // Values: range over channels, one (scale, zero) per token; one warp per token.
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, n_warps = blockDim.x / 32;
  for (int t = warp; t < bs; t += n_warps) {
    float mn = INFINITY, mx = -INFINITY;
    for (int c = lane; c < d; c += 32) {
      mn = fminf(mn, x[n + t * d + c]);
      mx = fmaxf(mx, x[n + t * d + c]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) {
      float sc = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), kLevels), FLT_MIN);
      vmn[t] = mn;
      vsc[t] = sc;
      reinterpret_cast<__half*>(rec + L.vs())[t] = __float2half_rn(sc);
      reinterpret_cast<__half*>(rec + L.vz())[t] = __float2half_rn(mn);
    }
  }
  __syncthreads();
  int8_t* kq = reinterpret_cast<int8_t*>(rec + L.kq());
  int8_t* vq = reinterpret_cast<int8_t*>(rec + L.vq());
  for (int e = threadIdx.x; e < n; e += blockDim.x) {
    const int t = e / d, c = e % d;
    const int8_t a = quantise(x[e], kmn[c], ksc[c]);
    const int8_t v = quantise(x[n + e], vmn[t], vsc[t]);
    kq[e] = a;
    vq[e] = v;
    if (deq != nullptr || kmin != nullptr) {
      // What unpack would return in the model dtype: from the stored float16 scale and zero.
      x[e] = to_f32<T>(from_f32<T>(dequant(a, __half2float(__float2half_rn(ksc[c])), __half2float(__float2half_rn(kmn[c])))));
      x[n + e] = to_f32<T>(from_f32<T>(dequant(v, __half2float(__float2half_rn(vsc[t])), __half2float(__float2half_rn(vmn[t])))));
    }
  }
  if (deq == nullptr && kmin == nullptr) return;
  __syncthreads();
  if (deq != nullptr) {
    T* dst = deq + p * 2 * n;
    for (int e = threadIdx.x; e < 2 * n; e += blockDim.x) dst[e] = from_f32<T>(x[e]);
  }
  if (kmin != nullptr) {
    // Metadata over the dequantised keys, lazykv/tiered.py:191-194.
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
      float mn = x[c], mx = mn;
      for (int t = 1; t < bs; ++t) {
        mn = fminf(mn, x[t * d + c]);
        mx = fmaxf(mx, x[t * d + c]);
      }
      const int64_t o = j * m_head + (int64_t)(first_block + b) * d + c;
      kmin[o] = from_f32<T>(mn);
      kmax[o] = from_f32<T>(mx);
    }
  }
}

// ---- unpack / fetch ------------------------------------------------------------------------

// Dequantise record `src` into pair `dst` [2][bs][d]; 8 elements per thread iteration.
template <typename T>
__device__ __forceinline__ void unpack_one(const uint8_t* __restrict__ src, T* __restrict__ dst,
                                           const RecordLayout& L, int tid, int nthreads) {
  const int n = L.bs * L.d;
  for (int e8 = tid; e8 < (2 * n) / 8; e8 += nthreads) {
    const int e = e8 * 8;
    const int kv = e / n, rem = e % n, t = rem / L.d, c0 = rem % L.d;
    const uint2 raw = *reinterpret_cast<const uint2*>(src + (kv ? L.vq() : L.kq()) + rem);
    const int8_t* q = reinterpret_cast<const int8_t*>(&raw);
    float out[8];
    if (kv == 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) out[i] = dequant(q[i], half_at(src + L.ks() + 2 * (c0 + i)), half_at(src + L.kz() + 2 * (c0 + i)));
    } else {
      const float s = half_at(src + L.vs() + 2 * t), z = half_at(src + L.vz() + 2 * t);
#pragma unroll
      for (int i = 0; i < 8; ++i) out[i] = dequant(q[i], s, z);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[e + i] = from_f32<T>(out[i]);
  }
}

template <typename T>
__global__ void unpack_kernel(const uint8_t* __restrict__ records, int64_t n, RecordLayout L, T* out) {
  const int64_t r = blockIdx.x;
  unpack_one<T>(records + r * L.width, out + r * 2 * L.bs * L.d, L, threadIdx.x, blockDim.x);
}

template <typename T>
__global__ void fetch_kernel(const void* __restrict__ src, int src_kind, const int64_t* __restrict__ src_rows,
                             T* dst, const int64_t* __restrict__ dst_rows, RecordLayout L) {
  const int64_t i = blockIdx.x;
  const int64_t s = src_rows[i], o = dst_rows[i];
  const int n2 = 2 * L.bs * L.d;
  T* d = dst + o * n2;
  if (src_kind == LKV_COLD_INT8) {
    unpack_one<T>(static_cast<const uint8_t*>(src) + s * L.width, d, L, threadIdx.x, blockDim.x);
  } else {
    const uint4* a = reinterpret_cast<const uint4*>(static_cast<const T*>(src) + s * n2);
    uint4* b = reinterpret_cast<uint4*>(d);
    const int n16 = n2 * (int)sizeof(T) / 16;
    for (int e = threadIdx.x; e < n16; e += blockDim.x) b[e] = a[e];
  }
}

int check_geometry(int bs, int d) {
  if (bs <= 0 || d <= 0 || bs % 8 != 0 || d % 8 != 0 || bs > 128 || d > 256)
    return fail(LKV_ERR_ARG, "unsupported block geometry bs=%d d=%d (multiples of 8, bs<=128, d<=256)", bs, d);
  return LKV_OK;
}

}  // namespace
}  // namespace lkv

using namespace lkv;

extern "C" {

int lkv_block_minmax(const void* keys, int dtype, int h, int n_blocks, int bs, int d, int64_t s_head,
                     int64_t s_block, int64_t s_tok, void* kmin, void* kmax, int64_t m_head,
                     int first_block, void* stream) {
  if (!dtype_ok(dtype)) return fail(LKV_ERR_ARG, "lkv_block_minmax: bad dtype %d", dtype);
  if (keys == nullptr || kmin == nullptr || kmax == nullptr) return fail(LKV_ERR_PTR, "lkv_block_minmax: null pointer");
  if (h <= 0 || n_blocks < 0 || bs <= 0 || d <= 0) return fail(LKV_ERR_ARG, "lkv_block_minmax: bad shape");
  if (n_blocks == 0) return LKV_OK;
  dim3 grid((unsigned)((int64_t(n_blocks) * d + 255) / 256), h);
  if (dtype == LKV_BF16)
    block_minmax_kernel<__nv_bfloat16><<<grid, 256, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(keys), n_blocks, bs, d, s_head, s_block, s_tok,
        static_cast<__nv_bfloat16*>(kmin), static_cast<__nv_bfloat16*>(kmax), m_head, first_block);
  else
    block_minmax_kernel<float><<<grid, 256, 0, as_stream(stream)>>>(
        static_cast<const float*>(keys), n_blocks, bs, d, s_head, s_block, s_tok,
        static_cast<float*>(kmin), static_cast<float*>(kmax), m_head, first_block);
  return launched("lkv_block_minmax");
}

int lkv_pack_int8(const void* pairs, int dtype, int n_blocks, int h, int bs, int d, uint8_t* records,
                  void* kmin, void* kmax, int64_t m_head, int first_block, void* deq, void* stream) {
  if (!dtype_ok(dtype)) return fail(LKV_ERR_ARG, "lkv_pack_int8: bad dtype %d", dtype);
  if (int rc = check_geometry(bs, d)) return rc;
  if (pairs == nullptr || records == nullptr) return fail(LKV_ERR_PTR, "lkv_pack_int8: null pointer");
  if ((kmin == nullptr) != (kmax == nullptr)) return fail(LKV_ERR_PTR, "lkv_pack_int8: kmin and kmax go together");
  if (!aligned(records, 16)) return fail(LKV_ERR_PTR, "lkv_pack_int8: records must be 16-byte aligned");
  if (n_blocks < 0 || h <= 0) return fail(LKV_ERR_ARG, "lkv_pack_int8: bad shape");
  const int64_t n_pairs = (int64_t)n_blocks * h;
  if (n_pairs == 0) return LKV_OK;
  const size_t smem = (2 * bs * d + 2 * d + 2 * bs) * sizeof(float);
  const int64_t width = lkv_packed_pair_bytes(bs, d);
  if (dtype == LKV_BF16) {
    auto k = pack_kernel<__nv_bfloat16>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<(unsigned)n_pairs, 256, smem, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(pairs), h, bs, d, records, width,
        static_cast<__nv_bfloat16*>(kmin), static_cast<__nv_bfloat16*>(kmax), m_head, first_block,
        static_cast<__nv_bfloat16*>(deq));
  } else {
    auto k = pack_kernel<float>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<(unsigned)n_pairs, 256, smem, as_stream(stream)>>>(
        static_cast<const float*>(pairs), h, bs, d, records, width, static_cast<float*>(kmin),
        static_cast<float*>(kmax), m_head, first_block, static_cast<float*>(deq));
  }
  return launched("lkv_pack_int8");
}

int lkv_unpack_int8(const uint8_t* records, int64_t n, int bs, int d, void* out, int out_dtype, void* stream) {
  if (!dtype_ok(out_dtype)) return fail(LKV_ERR_ARG, "lkv_unpack_int8: bad dtype %d", out_dtype);
  if (int rc = check_geometry(bs, d)) return rc;
  if (records == nullptr || out == nullptr) return fail(LKV_ERR_PTR, "lkv_unpack_int8: null pointer");
  if (!aligned(records, 16)) return fail(LKV_ERR_PTR, "lkv_unpack_int8: records must be 16-byte aligned");
  if (n <= 0) return n == 0 ? LKV_OK : fail(LKV_ERR_ARG, "lkv_unpack_int8: negative count");
  RecordLayout L{bs, d, lkv_packed_pair_bytes(bs, d)};
  if (out_dtype == LKV_BF16)
    unpack_kernel<__nv_bfloat16><<<(unsigned)n, 128, 0, as_stream(stream)>>>(records, n, L, static_cast<__nv_bfloat16*>(out));
  else
    unpack_kernel<float><<<(unsigned)n, 128, 0, as_stream(stream)>>>(records, n, L, static_cast<float*>(out));
  return launched("lkv_unpack_int8");
}

int lkv_fetch_pairs(const void* src, int src_kind, const int64_t* src_rows, void* dst,
                    const int64_t* dst_rows, int64_t n, int bs, int d, int dtype, void* stream) {
  if (!dtype_ok(dtype)) return fail(LKV_ERR_ARG, "lkv_fetch_pairs: bad dtype %d", dtype);
  if (src_kind != LKV_COLD_INT8 && src_kind != LKV_COLD_PAIRS) return fail(LKV_ERR_ARG, "lkv_fetch_pairs: bad source kind %d", src_kind);
  if (int rc = check_geometry(bs, d)) return rc;
  if (n == 0) return LKV_OK;
  if (src == nullptr || dst == nullptr || src_rows == nullptr || dst_rows == nullptr) return fail(LKV_ERR_PTR, "lkv_fetch_pairs: null pointer");
  if (!aligned(src, 16) || !aligned(dst, 16)) return fail(LKV_ERR_PTR, "lkv_fetch_pairs: pools must be 16-byte aligned");
  RecordLayout L{bs, d, lkv_packed_pair_bytes(bs, d)};
  if (dtype == LKV_BF16)
    fetch_kernel<__nv_bfloat16><<<(unsigned)n, 128, 0, as_stream(stream)>>>(src, src_kind, src_rows, static_cast<__nv_bfloat16*>(dst), dst_rows, L);
  else
    fetch_kernel<float><<<(unsigned)n, 128, 0, as_stream(stream)>>>(src, src_kind, src_rows, static_cast<float*>(dst), dst_rows, L);
  return launched("lkv_fetch_pairs");
}

}  // extern "C"
