// Host-side helpers shared by the C-ABI entry points: per-thread error text
// and CUDA status checks.  Never exits or aborts: every failure becomes a
// negative return code plus a message for mtc_last_error().
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/mtc_b200.h"

namespace mtc {

void set_error(const char* fmt, ...);
void clear_error();

inline int cuda_fail(cudaError_t e, const char* what) {
  set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return MTC_ERR_CUDA;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Launch-error check after a <<<>>> launch.
#define MTC_CHECK_LAUNCH(what)                                      \
  do {                                                              \
    cudaError_t e_ = cudaGetLastError();                            \
    if (e_ != cudaSuccess) return ::mtc::cuda_fail(e_, what);       \
  } while (0)

#define MTC_CHECK_CUDA(call, what)                                  \
  do {                                                              \
    cudaError_t e_ = (call);                                        \
    if (e_ != cudaSuccess) return ::mtc::cuda_fail(e_, what);       \
  } while (0)

#define MTC_REQUIRE(cond, ...)                                      \
  do {                                                              \
    if (!(cond)) {                                                  \
      ::mtc::set_error(__VA_ARGS__);                                \
      return MTC_ERR_INVALID;                                       \
    }                                                               \
  } while (0)

// The epilogue argument of the C ABI, checked (act in range) and flattened
// for kernel parameters; NULL means none.
struct EpiArg {
  const float* bias = nullptr;
  int act = MTC_ACT_NONE;
};
inline int read_epilogue(const mtc_epilogue* ep, EpiArg* out, const char* who) {
  *out = EpiArg();
  if (!ep) return MTC_OK;
  if (ep->act < MTC_ACT_NONE || ep->act > MTC_ACT_GELU_TANH) {
    set_error("%s: unknown activation %d", who, ep->act);
    return MTC_ERR_INVALID;
  }
  if (ep->bias && (reinterpret_cast<uintptr_t>(ep->bias) & 3)) {
    set_error("%s: bias not 4-byte aligned", who);
    return MTC_ERR_INVALID;
  }
  out->bias = ep->bias;
  out->act = ep->act;
  return MTC_OK;
}

// Limit of every bounded pipeline wait of the next launches, in ns (2 s
// unless mtc_set_wait_limit_ns changed it), and the diagnostic hold of
// mtc_debug_withhold_bytes, taken (and cleared) by the next strip launch.
unsigned long long wait_limit_ns();
uint32_t take_withheld_bytes();

// Shared launch helpers (mtc_prefill.cu): the X row gather into fp16 Xp and
// the TMA descriptor of Xp used by the prefill and decode kernels.
int launch_gather_x(const float* X, long long ldx, int K, int Kp, const int32_t* row_perm, int M, __half* Xp,
                    uint32_t* status, cudaStream_t st);
int encode_xp_map(CUtensorMap* map, const __half* Xp, int Kp, int M, int box_rows, const char* who);
int encode_xp_blocks_map(CUtensorMap* map, const __half* Xp, int Kp, int rows, int nblk, const char* who);

}  // namespace mtc
