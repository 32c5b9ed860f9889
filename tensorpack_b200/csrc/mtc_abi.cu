// C-ABI housekeeping: version, per-thread error text, device queries.
#include <string>

#include "mtc_internal.h"

namespace mtc {
namespace {
thread_local std::string g_last_error;
}

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

}  // namespace mtc

extern "C" int mtc_abi_version(void) { return MTC_ABI_VERSION; }

extern "C" const char* mtc_last_error(void) { return mtc::g_last_error.c_str(); }

extern "C" int mtc_device_sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
    mtc::set_error("mtc_device_sm_count: no CUDA device %d", device);
    return MTC_ERR_CUDA;
  }
  return n;
}

extern "C" int mtc_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  mtc::clear_error();
  MTC_REQUIRE(dst && src, "mtc_copy_async: null pointer");
  MTC_REQUIRE(((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0,
              "mtc_copy_async: pointers not 16-byte aligned");
  if (bytes == 0) return MTC_OK;
  MTC_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, mtc::as_stream(stream)),
                 "mtc_copy_async");
  return MTC_OK;
}
