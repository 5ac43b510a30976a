// Error state and small queries of the C ABI (include/lkv.h).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

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
