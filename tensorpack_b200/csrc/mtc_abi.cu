// C-ABI housekeeping: version, per-thread error text, device queries, the
// wait limit of the kernels' bounded pipeline waits.
#include <atomic>
#include <string>

#include "mtc_internal.h"

namespace mtc {
namespace {
thread_local std::string g_last_error;

#ifndef MTC_SOURCE_HASH
#define MTC_SOURCE_HASH "unknown"
#endif
// Read from the file by the build script (tensorpack_b200/build.py) to tell
// whether this library was built from the sources next to it.
__attribute__((used)) const char kSourceHash[] = "MTC_SOURCE_HASH=" MTC_SOURCE_HASH;
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

namespace {
constexpr unsigned long long kDefaultWaitNs = 2000000000ull;
std::atomic<unsigned long long> g_wait_ns{kDefaultWaitNs};
std::atomic<uint32_t> g_withheld{0};
}  // namespace

unsigned long long wait_limit_ns() { return g_wait_ns.load(std::memory_order_relaxed); }
uint32_t take_withheld_bytes() { return g_withheld.exchange(0u); }

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

extern "C" int mtc_set_wait_limit_ns(uint64_t ns) {
  mtc::clear_error();
  mtc::g_wait_ns.store(ns ? ns : mtc::kDefaultWaitNs);
  return MTC_OK;
}

extern "C" int mtc_debug_withhold_bytes(uint32_t bytes) {
  mtc::clear_error();
  MTC_REQUIRE((bytes & 15u) == 0 && bytes <= 4096u, "mtc_debug_withhold_bytes: %u is not a multiple of 16 in 0..4096",
              bytes);
  mtc::g_withheld.store(bytes);
  return MTC_OK;
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
