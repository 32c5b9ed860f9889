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

// Shared launch helpers (mtc_prefill.cu): the X row gather into fp16 Xp and
// the TMA descriptor of Xp used by the prefill and decode kernels.
int launch_gather_x(const float* X, long long ldx, int K, int Kp, const int32_t* row_perm, int M, __half* Xp,
                    uint32_t* status, cudaStream_t st);
int encode_xp_map(CUtensorMap* map, const __half* Xp, int Kp, int M, int box_rows, const char* who);

}  // namespace mtc
