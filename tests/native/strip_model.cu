// CPU model of the strip-stream decode kernel, for the format tests only.
//
// It walks the batch records exactly as strip_kernel does and runs the same
// per-lane code (lane_fast / lane_generic from mtc_strip.cuh) for all 32
// lanes of every step.  The two mma.sync.m16n8k16 of a step are evaluated
// from the lanes' registers with the PTX fragment layout of that shape
// (A: a0 = (row g, k 2t..2t+1), a1 = (row g+8, k 2t..2t+1), a2 = (row g,
// k 2t+8..2t+9), a3 = (row g+8, k 2t+8..2t+9); B: b0 = (k 2t..2t+1, col g),
// b1 = (k 2t+8..2t+9, col g); D: c0..c3 = (g, 2t), (g, 2t+1), (g+8, 2t),
// (g+8, 2t+1)), and the results are read back with the kernel's selection
// (lane 4g + g/2, elements g & 1 and 2 + (g & 1)).  Accumulation is in fp64
// here, so results differ from the GPU's fp32 sums by rounding only.
//
// Wide streams (MTC_STRIP_WIDE) are followed the same way: a wide group
// step's four MMAs are evaluated from the lanes' two A-fragment sets.
//
// Never part of the GEMM path: the library in tensorpack_b200/ has no CPU
// product; this file is built into tests/native/libstrip_model.so.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <vector>

#include "../../tensorpack_b200/csrc/mtc_strip.cuh"

using namespace mtc::strip;

namespace {

constexpr int MT = kMaxM;

template <int C, bool G>
void fast_lanes(const uint8_t* st, int n0, int n1, bool full, const uint16_t* x16, int kpad, uint32_t a[32][8],
                uint32_t b[32][MT][2]) {
  for (int L = 0; L < 32; ++L) {
    if (full)
      lane_fast<C, G, true, MT>(st, n0, n1, L, x16, kpad, a[L], b[L]);
    else
      lane_fast<C, G, false, MT>(st, n0, n1, L, x16, kpad, a[L], b[L]);
  }
}

// D = A (16x16) x B (16x8) of one mma from the lanes' fragments.
void mma_model(const uint32_t a[32][8], int half, const uint32_t b[32][MT][2], int m, double D[16][8]) {
  double A[16][16], B[16][8];
  for (int L = 0; L < 32; ++L) {
    const int g = L >> 2, t = L & 3;
    const uint32_t* r = a[L] + 4 * half;
    auto lo = [](uint32_t v) { return (double)h2f((uint16_t)(v & 0xFFFFu)); };
    auto hi = [](uint32_t v) { return (double)h2f((uint16_t)(v >> 16)); };
    A[g][2 * t] = lo(r[0]), A[g][2 * t + 1] = hi(r[0]);
    A[g + 8][2 * t] = lo(r[1]), A[g + 8][2 * t + 1] = hi(r[1]);
    A[g][2 * t + 8] = lo(r[2]), A[g][2 * t + 9] = hi(r[2]);
    A[g + 8][2 * t + 8] = lo(r[3]), A[g + 8][2 * t + 9] = hi(r[3]);
    B[2 * t][g] = lo(b[L][m][0]), B[2 * t + 1][g] = hi(b[L][m][0]);
    B[2 * t + 8][g] = lo(b[L][m][1]), B[2 * t + 9][g] = hi(b[L][m][1]);
  }
  for (int i = 0; i < 16; ++i)
    for (int j = 0; j < 8; ++j) {
      double s = 0.0;
      for (int k = 0; k < 16; ++k) s += A[i][k] * B[k][j];
      D[i][j] = s;
    }
}

}  // namespace

template <int C>
void wide_lanes(const uint8_t* st, int n, bool full, const uint16_t* x16, int kpad, uint32_t a[32][8],
                uint32_t a2[32][8], uint32_t b[32][MT][2]) {
  for (int L = 0; L < 32; ++L) {
    if (full)
      lane_wide<C, true, MT>(st, n, L, x16, kpad, a[L], a2[L], b[L]);
    else
      lane_wide<C, false, MT>(st, n, L, x16, kpad, a[L], a2[L], b[L]);
  }
}

extern "C" int strip_model_gemm(const uint8_t* stream, const uint32_t* batch_off, const uint32_t* strip_batch,
                                int n_strips, int tk, int K, int N, int exp2, const float* X, int M,
                                const int32_t* pr, const int32_t* pc, float* Y, uint32_t flags) {
  const bool wide = (flags & kWide) != 0;
  if (M < 1 || M > MT) return -1;
  const int kpad = tk * 32;
  std::vector<uint16_t> x16((size_t)MT * kpad, 0);
  for (int m = 0; m < M; ++m)
    for (int k = 0; k < K; ++k) x16[(size_t)m * kpad + k] = f2h(X[(size_t)m * K + (pr ? pr[k] : k)]);
  const int n_batches = (int)strip_batch[n_strips];
  std::vector<double> part((size_t)n_batches * MT * 8, 0.0);
  static uint32_t a[32][8], a2[32][8], b[32][MT][2];
  for (int bi = 0; bi < n_batches; ++bi) {
    const uint8_t* base = stream + batch_off[bi];
    const uint32_t nst = ldu32(base + 4);
    const uint8_t* st = base + pad16(8 + 4 * (int)nst);
    double* out = part.data() + (size_t)bi * MT * 8;
    uint32_t run_d = 0;
    int run_left = 0;
    for (uint32_t s = 0; s < nst; ++s) {
      // inside a run the kernel reuses the run's first descriptor
      uint32_t d = ldu32(base + 8 + 4 * s);
      if (run_left > 0) {
        d = run_d;
        --run_left;
      } else if (desc_run(d) > 1) {
        run_d = d;
        run_left = desc_run(d) - 1;
      }
      const int kind = desc_kind(d), n0 = desc_n0(d), n1 = desc_n1(d);
      const bool full = desc_full(d);
      if (full != full_counts(kind, n0, n1, wide)) return -3;
      if (wide && kind < kU2) {
        // four MMAs (columns 0-1, 2-3 of quartet 0 from a, 4-5, 6-7 of quartet 1
        // from a2) sharing one B fragment; every quad's diagonal covers all 8 columns
        switch (kind) {
          case kG2: wide_lanes<0>(st, n0, full, x16.data(), kpad, a, a2, b); break;
          case kG3: wide_lanes<1>(st, n0, full, x16.data(), kpad, a, a2, b); break;
          case kG4: wide_lanes<2>(st, n0, full, x16.data(), kpad, a, a2, b); break;
          case kG5: wide_lanes<3>(st, n0, full, x16.data(), kpad, a, a2, b); break;
          case kG6: wide_lanes<4>(st, n0, full, x16.data(), kpad, a, a2, b); break;
          default: wide_lanes<5>(st, n0, full, x16.data(), kpad, a, a2, b); break;
        }
        for (int m = 0; m < MT; ++m)
          for (int j = 0; j < 4; ++j) {
            double D[16][8];
            mma_model(j < 2 ? a : a2, j & 1, b, m, D);
            for (int g = 0; g < 8; ++g) {
              const int t = g >> 1, sel = g & 1;
              const double c[4] = {D[g][2 * t], D[g][2 * t + 1], D[g + 8][2 * t], D[g + 8][2 * t + 1]};
              out[m * 8 + 2 * j] += c[sel];
              out[m * 8 + 2 * j + 1] += c[2 + sel];
            }
          }
      } else if (kind == kGeneric) {
        for (int L = 0; L < 32; ++L) {
          float g[MT][4] = {};
          lane_generic<MT>(st, n0, n1, L, x16.data(), kpad, g);
          for (int m = 0; m < MT; ++m)
            for (int c = 0; c < 4; ++c) out[m * 8 + 4 * (L >> 4) + c] += g[m][c];
        }
      } else {
        switch (kind) {
          case kG2: fast_lanes<0, true>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kG3: fast_lanes<1, true>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kG4: fast_lanes<2, true>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kG5: fast_lanes<3, true>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kG6: fast_lanes<4, true>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kG8: fast_lanes<5, true>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kU2: fast_lanes<0, false>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kU3: fast_lanes<1, false>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kU4: fast_lanes<2, false>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kU5: fast_lanes<3, false>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kU6: fast_lanes<4, false>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          case kU8: fast_lanes<5, false>(st, n0, n1, full, x16.data(), kpad, a, b); break;
          default: return -2;
        }
        for (int m = 0; m < MT; ++m)
          for (int half = 0; half < 2; ++half) {
            double D[16][8];
            mma_model(a, half, b, m, D);
            for (int g = 0; g < 8; ++g) {  // the kernel's read-back: lane 4g + g/2
              const int t = g >> 1, sel = g & 1, h = g >> 2;
              const double c[4] = {D[g][2 * t], D[g][2 * t + 1], D[g + 8][2 * t], D[g + 8][2 * t + 1]};
              out[m * 8 + 4 * h + 2 * half] += c[sel];
              out[m * 8 + 4 * h + 2 * half + 1] += c[2 + sel];
            }
          }
      }
      st += desc_bytes(d);
    }
  }
  const double inv = ldexp(1.0, -exp2);
  for (int s = 0; s < n_strips; ++s)
    for (int f = 0; f < 8; ++f) {
      const int n = 8 * s + f;
      if (n >= N) continue;
      for (int m = 0; m < M; ++m) {
        double sum = 0.0;
        for (uint32_t bi = strip_batch[s]; bi < strip_batch[s + 1]; ++bi) sum += part[((size_t)bi * MT + m) * 8 + f];
        Y[(size_t)m * N + (pc ? pc[n] : n)] = (float)(sum * inv);
      }
    }
  return 0;
}

// Pack one lane's 16 codes with the class recipes and decode them again
// (format self-test).  Returns 0 on success, 1 on a placement collision.


extern "C" int strip_model_lane_roundtrip(int cls, const int32_t* q16, int32_t* out16, uint32_t* words) {
  int q[4][4];
  for (int i = 0; i < 16; ++i) q[i / 4][i % 4] = q16[i];
  uint32_t A[4], B;
  if (!mtc::strip::pack_lane(cls, q, A, &B)) return 1;
  // the 16-bit secondary planes travel as 16 bits and are spread again by the decoder
  uint32_t Bw = B;
  if (sec_bytes(cls) == 2) Bw = spread16((B & 0xFFu) | ((B >> 8) & 0xFF00u));
  uint32_t a[8];
  switch (cls) {
    case 0: decode_lane<0>(A, Bw, a); break;
    case 1: decode_lane<1>(A, Bw, a); break;
    case 2: decode_lane<2>(A, Bw, a); break;
    case 3: decode_lane<3>(A, Bw, a); break;
    case 4: decode_lane<4>(A, Bw, a); break;
    default: decode_lane<5>(A, Bw, a); break;
  }
  for (int k = 0; k < 8; ++k)
    for (int hh = 0; hh < 2; ++hh) {
      const float v = h2f((uint16_t)(a[k] >> (16 * hh)));
      out16[(pair_row(k) + hh) * 4 + pair_col(k)] = (int32_t)v;
    }
  for (int i = 0; i < 4; ++i) words[i] = A[i];
  words[4] = B;
  return 0;
}
