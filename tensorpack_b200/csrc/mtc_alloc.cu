// GPU candidate search of the MTC rate-distortion allocators.
//
// Restates the per-block scale search of mtc/core/allocation.py:106-160
// (called by rd_candidates, allocation.py:200-235, for every level of
// QuadtreeRD, mtc/core/quadtree.py:93-95): for every s x s block and one
// precision mode, try every clipping ratio alpha of the mode's grid and both
// scale signs, keep the scale with the smallest importance-weighted squared
// error.  One thread per block walks the candidates in the reference's order
// with the reference's arithmetic (fp32 codes and errors, fp64 row
// weighting, no fused multiply-add), so distortions and scales match the
// reference bit for bit.
#include <math.h>

#include "mtc_internal.h"

namespace mtc {
namespace {

__device__ __forceinline__ double round_bf16_value(double x) {
  // nearest bf16 value: 8 significant bits, fp32 exponent range (allocation.py:97-103)
  if (x == 0.0) return x;
  int e;
  const double m = frexp(x, &e);
  return ldexp(rint(m * 256.0) / 256.0, e);
}

__global__ void rd_search_kernel(const float* __restrict__ W, int K, int N, int s, const double* __restrict__ h,
                                 float lo, float hi, double qmag, const float* __restrict__ alphas, int n_alpha,
                                 int n_sign, int bf16, double* __restrict__ out_d, float* __restrict__ out_s) {
  const int nbn = N / s;
  const long long nb = (long long)(K / s) * nbn;
  const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nb) return;
  const int bi = (int)(b / nbn), bj = (int)(b % nbn);
  const float* blk = W + (long long)bi * s * N + (long long)bj * s;
  float amax = 0.0f;
  for (int r = 0; r < s; ++r)
    for (int c = 0; c < s; ++c) amax = fmaxf(amax, fabsf(blk[(long long)r * N + c]));
  if (amax < 1e-30f) amax = 1.0f;
  double best_d = INFINITY;
  float best_s = 0.0f;
  for (int ia = 0; ia < n_alpha; ++ia) {
    for (int isg = 0; isg < n_sign; ++isg) {
      const float sgn = isg == 0 ? 1.0f : -1.0f;
      float sc = (float)((double)__fmul_rn(__fmul_rn(sgn, alphas[ia]), amax) / qmag);
      if (bf16) sc = (float)round_bf16_value((double)sc);
      const float inv = __fdiv_rn(1.0f, sc);
      double dist = 0.0;
      for (int r = 0; r < s; ++r) {
        float acc = 0.0f;
        const float* row = blk + (long long)r * N;
        for (int c = 0; c < s; ++c) {
          const float x = row[c];
          float q = rintf(__fmul_rn(x, inv));
          if (q < lo) q = lo;
          else if (q > hi) q = hi;
          const float e = __fsub_rn(x, __fmul_rn(q, sc));
          acc = __fadd_rn(acc, __fmul_rn(e, e));
        }
        dist = __dadd_rn(dist, __dmul_rn(h[bi * s + r], (double)acc));
      }
      if (dist < best_d) {
        best_d = dist;
        best_s = sc;
      }
    }
  }
  out_d[b] = best_d;
  out_s[b] = best_s;
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" int mtc_rd_search(const float* W, int32_t K, int32_t N, int32_t block_size, const double* h_norm,
                             int32_t mode, const float* alphas, int32_t n_alpha, int32_t bf16_scales,
                             double* out_dist, float* out_scale, void* stream) {
  clear_error();
  MTC_REQUIRE(W && h_norm && alphas && out_dist && out_scale, "mtc_rd_search: null pointer argument");
  MTC_REQUIRE(block_size > 0 && K % block_size == 0 && N % block_size == 0,
              "mtc_rd_search: shape (%d, %d) not divisible by block size %d", K, N, block_size);
  int lo, hi;
  switch (mode) {
    case 2: lo = -2; hi = 1; break;
    case 3: lo = -4; hi = 3; break;
    case 4: lo = -8; hi = 7; break;
    case 5: lo = -16; hi = 15; break;
    case 6: lo = -32; hi = 31; break;
    case 8: lo = -128; hi = 127; break;
    case 16: lo = -32768; hi = 32767; break;
    default: set_error("mtc_rd_search: mode %d has no scale", mode); return MTC_ERR_INVALID;
  }
  MTC_REQUIRE(n_alpha > 0, "mtc_rd_search: empty alpha grid");
  const double qmag = (double)(-lo > hi ? -lo : hi);
  const long long nb = (long long)(K / block_size) * (N / block_size);
  const int threads = 128;
  const long long blocks = (nb + threads - 1) / threads;
  MTC_REQUIRE(blocks < (1ll << 31), "mtc_rd_search: too many blocks");
  rd_search_kernel<<<(unsigned)blocks, threads, 0, as_stream(stream)>>>(
      W, K, N, block_size, h_norm, (float)lo, (float)hi, qmag, alphas, n_alpha, mode == 16 ? 1 : 2, bf16_scales,
      out_dist, out_scale);
  MTC_CHECK_LAUNCH("mtc_rd_search");
  return MTC_OK;
}
