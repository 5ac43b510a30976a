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

int64_t lkv_packed_pair_bytes(int bs, int d) {
  // lazykv/quant.py:46-49: two int8 payloads, float16 scale+zero per channel (keys) and per token (values).
  return 2ll * bs * d + 2ll * 2 * d + 2ll * 2 * bs;
}

}  // extern "C"
