// Error state and small queries of the C ABI (include/lkv.h).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "common.cuh"

namespace lkv {

static thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

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

// ---- tensor maps, encoded once per distinct set of arguments ------------------------------------
//
// cuTensorMapEncodeTiled is a pure function of its arguments (the address, sizes, strides, box and
// modes), so a map encoded once can be reused by every later launch over the same buffer: an eager
// decode loop that calls the kernels with the same stores every step then pays the encoding once.
// A fixed table of distinct argument sets, looked up by a hash of the arguments (a short linear
// probe from the hashed slot; a miss with every probed slot taken replaces the first of them),
// under a mutex.

namespace {

struct MapKey {
  CUtensorMapDataType dt;
  cuuint32_t rank;
  void* base;
  cuuint64_t dims[5];
  cuuint64_t strides[4];
  cuuint32_t box[5];
  cuuint32_t estr[5];
  CUtensorMapInterleave il;
  CUtensorMapSwizzle sw;
  CUtensorMapL2promotion l2;
  CUtensorMapFloatOOBfill oob;
};

constexpr int kMapCacheSize = 512;  // a power of two
constexpr int kMapProbe = 8;
struct MapEntry {
  bool used;
  MapKey key;
  CUtensorMap map;
};
MapEntry g_maps[kMapCacheSize];
std::mutex g_map_mu;

// FNV-1a over the key's bytes (padding zeroed by the caller).
uint64_t map_hash(const MapKey& k) {
  const unsigned char* p = reinterpret_cast<const unsigned char*>(&k);
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < sizeof(MapKey); ++i) h = (h ^ p[i]) * 1099511628211ull;
  return h;
}

}  // namespace

CUresult encode_tiled(CUtensorMap* out, CUtensorMapDataType dt, cuuint32_t rank, void* base, const cuuint64_t* dims, const cuuint64_t* strides,
                      const cuuint32_t* box, const cuuint32_t* estr, CUtensorMapInterleave il, CUtensorMapSwizzle sw, CUtensorMapL2promotion l2,
                      CUtensorMapFloatOOBfill oob) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr || rank < 1 || rank > 5) return CUDA_ERROR_NOT_SUPPORTED;
  MapKey key;
  memset(&key, 0, sizeof(key));  // padding and unused dimensions compare equal
  key.dt = dt;
  key.rank = rank;
  key.base = base;
  for (cuuint32_t i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
    key.estr[i] = estr[i];
    if (i + 1 < rank) key.strides[i] = strides[i];
  }
  key.il = il;
  key.sw = sw;
  key.l2 = l2;
  key.oob = oob;
  const int home = (int)(map_hash(key) & (kMapCacheSize - 1));
  std::lock_guard<std::mutex> lock(g_map_mu);
  int free_slot = -1;
  for (int p = 0; p < kMapProbe; ++p) {
    MapEntry& e = g_maps[(home + p) & (kMapCacheSize - 1)];
    if (!e.used) {
      if (free_slot < 0) free_slot = (home + p) & (kMapCacheSize - 1);
      continue;
    }
    if (memcmp(&e.key, &key, sizeof(key)) == 0) {
      *out = e.map;
      return CUDA_SUCCESS;
    }
  }
  const CUresult r = enc(out, dt, rank, base, dims, strides, box, estr, il, sw, l2, oob);
  if (r == CUDA_SUCCESS) {
    MapEntry& e = g_maps[free_slot >= 0 ? free_slot : home];
    e.used = true;
    e.key = key;
    e.map = *out;
  }
  return r;
}

int launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(LKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return LKV_OK;
}

}  // namespace lkv

extern "C" {

const char* lkv_version(void) { return "lkv_sm100 0.1"; }

size_t lkv_last_error(char* buf, size_t len) {
  size_t n = strlen(lkv::g_last_error);
  if (buf != nullptr && len > 0) {
    size_t m = n < len - 1 ? n : len - 1;
    memcpy(buf, lkv::g_last_error, m);
    buf[m] = '\0';
  }
  return n;
}

int lkv_shard_plan(int n_sealed, int k_total, int world, int rank, int32_t* out) {
  if (out == nullptr) return lkv::fail(LKV_ERR_PTR, "lkv_shard_plan: null output");
  if (n_sealed < 2 || world < 1 || rank < 0 || rank >= world || k_total < 1)
    return lkv::fail(LKV_ERR_ARG, "lkv_shard_plan: bad plan (n_sealed %d, k %d, world %d, rank %d)", n_sealed, k_total, world, rank);
  // Contiguous ranges of ceil(n_sealed / world) sealed blocks; block 0 (the sink) is not a
  // candidate. The budget is shared in proportion to the candidates, the remainder one block each
  // to the lowest ranks that have room.
  const int per = (n_sealed + world - 1) / world;
  int cand[1024];
  if (world > 1024) return lkv::fail(LKV_ERR_ARG, "lkv_shard_plan: world %d above 1024", world);
  int total = 0;
  for (int r = 0; r < world; ++r) {
    const int lo = r * per < n_sealed ? r * per : n_sealed, hi = (r + 1) * per < n_sealed ? (r + 1) * per : n_sealed;
    const int first = lo > 1 ? lo : 1;
    cand[r] = hi > first ? hi - first : 0;
    total += cand[r];
  }
  if (k_total > total) return lkv::fail(LKV_ERR_ARG, "lkv_shard_plan: budget %d above the %d candidates", k_total, total);
  int given = 0, mine = 0;
  for (int r = 0; r < world; ++r) {
    const int kr = (int)((int64_t)k_total * cand[r] / total);
    given += kr;
    if (r == rank) mine = kr;
  }
  for (int r = 0; r < world && given < k_total; ++r) {
    const int kr = (int)((int64_t)k_total * cand[r] / total);
    if (kr < cand[r]) {
      ++given;
      if (r == rank) ++mine;
    }
  }
  const int lo = rank * per < n_sealed ? rank * per : n_sealed, hi = (rank + 1) * per < n_sealed ? (rank + 1) * per : n_sealed;
  out[0] = lo;
  out[1] = hi;
  out[2] = lo > 1 ? lo : 1;
  out[3] = cand[rank];
  out[4] = mine;
  return LKV_OK;
}

int64_t lkv_packed_pair_bytes(int bs, int d) {
  // lazykv/quant.py:46-49: two int8 payloads, float16 scale+zero per channel (keys) and per token (values).
  return 2ll * bs * d + 2ll * 2 * d + 2ll * 2 * bs;
}

}  // extern "C"
