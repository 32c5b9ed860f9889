// Strip stream: the decode-sized (M <= 4) layout of a packed MTC matrix and
// the per-lane arithmetic that consumes it.  Shared by the host builder
// (mtc_strip_build.cu), the GPU kernel (mtc_strip.cu) and the CPU model of
// the kernel's lanes used by the format tests; every function here is
// __host__ __device__ so that all three run the same decode.
//
// Replaces, for decode-sized M, the reference's packed GEMM
// (mtc/kernels/gemm.py:124-210, 541-574) over MTC-QT / MTC-QT-P leaves
// (mtc/core/quadtree.py:40-171, mtc/core/permutation.py:15-21).
//
// Layout.  A strip is 8 output features (stored column order) over all of K.
// It is cut into 8x8 groups (8 k-rows x 8 features).  A group covered by one
// leaf is a "group" item; a group split into four 4x4 leaves contributes its
// micro-blocks (4 k x 4 features) as "micro" items.  P0 items carry nothing
// and are dropped.  Items of P16 or with a scale that is not exact in fp16
// are "generic" micro items (fp32 path).  Items are sorted by kind (group
// classes P2..P8, micro classes P2..P8, generic) and packed into steps:
//
//   group step: up to 8 groups of one class (512 weights);
//   micro / generic step: up to 16 micro-blocks of each column half (quartet)
//   of the strip.
//
// One warp consumes one step with two mma.sync.m16n8k16 per lane.  Lane L
// (quad g = L >> 2, t = L & 3) owns one 4x4 micro-block of quartet h = L >> 4:
// its 16 codes become the two A fragments (rows g / g+8 = two feature
// columns, k slots 2t, 2t+1, 2t+8, 2t+9 = the micro-block's four k rows) and
// its B fragment is x * scale at those four k rows, placed in B column g.
// Only the diagonal D[g][g], D[g+8][g] of each product is used: every quad
// sums its own four micro-blocks, so the lanes of a warp need not share k
// rows, and sorting by class makes every step branch-free.
//
// Step record (16-byte aligned):
//   group:   [n u32 entries: fp16(scale * 2^exp2) | group row (8 k) << 16, pad16]
//            [plane A: 4n lanes x prim_bytes][plane B: 4n lanes x sec_bytes][pad16]
//   micro:   [n0 + n1 u32 entries: fp16 scale | micro row (4 k) << 16, pad16]
//            [plane A][plane B][pad16]      (lanes of quartet 0, then quartet 1)
//   generic: [n0 + n1 x (fp32 scale * 2^exp2, micro row | mode << 16), pad16]
//            [n0 + n1 x 32 B: the 16 codes as LSB-first m-bit two's complement]
//   group in a wide stream (MTC_STRIP_WIDE): up to 16 groups; lane L takes
//            group L >> 1, k half L & 1 and both quartets, whose two
//            micro-blocks sit side by side in each plane (2n lanes).
// Batch record (one bulk copy, never crossing a strip):
//   [u32 strip][u32 n_steps][n_steps u32 step descriptors][pad16][steps]
// Step descriptor: bits 0-3 kind, 4 full step, 5-9 n0 (groups for a group
// step), 10-14 n1, 15-21 step bytes / 16, 22-31 length of the run of
// identical full steps that starts here (1 for other steps).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>

namespace mtc {
namespace strip {

enum Kind : int {
  kG2 = 0, kG3, kG4, kG5, kG6, kG8,   // group steps by mode
  kU2, kU3, kU4, kU5, kU6, kU8,       // micro steps by mode
  kGeneric,                           // fp32 path (P16, inexact scales)
  kKinds
};

constexpr int kGenericSlot = 32;      // bytes of codes per generic micro-block (P16: 16 x 16 bit)
constexpr int kMaxM = 4;              // tokens per call

__host__ __device__ constexpr int pad16(int x) { return (x + 15) & ~15; }

// class index 0..5 <-> mode P2, P3, P4, P5, P6, P8
__host__ __device__ constexpr int mode_of_class(int c) {
  return c == 0 ? 2 : c == 1 ? 3 : c == 2 ? 4 : c == 3 ? 5 : c == 4 ? 6 : 8;
}
__host__ __device__ constexpr int class_of_mode(int m) {
  return m == 2 ? 0 : m == 3 ? 1 : m == 4 ? 2 : m == 5 ? 3 : m == 6 ? 4 : m == 8 ? 5 : -1;
}
// Per-lane bytes (16 codes) of the primary and secondary planes.
__host__ __device__ constexpr int prim_bytes(int c) {
  return c <= 1 ? 4 : c <= 4 ? 8 : 16;
}
__host__ __device__ constexpr int sec_bytes(int c) { return c == 1 || c == 3 ? 2 : c == 4 ? 4 : 0; }
__host__ __device__ constexpr int bias_of_class(int c) { return 1 << (mode_of_class(c) - 1); }

// Step descriptor fields.  A step is "full" when every lane has an item
// (8 groups, or 16 micro-blocks of each quartet); its lane offsets are then
// compile-time constants.  The first step of a run of identical full steps
// (same kind) carries the run's length, so the kernel loops over the run
// without reading the following descriptors.
//
// Wide streams (flag kWide): a group step holds up to 16 groups and lane L
// takes both column quartets of group L >> 1, k half L & 1 (32 weights, four
// MMAs sharing one B fragment).  Micro and generic steps are the same in both
// forms.
constexpr uint32_t kWide = 1u;        // stream flag (MTC_STRIP_WIDE)
constexpr uint32_t kMergeModes = 2u;  // build flag (MTC_STRIP_MERGE_MODES): P2 packed as P3, P6 as P8
__host__ __device__ constexpr int group_step_max(bool wide) { return wide ? 16 : 8; }
__host__ __device__ constexpr bool full_counts(int kind, int n0, int n1, bool wide = false) {
  return kind < kU2 ? n0 == group_step_max(wide) : (n0 == 16 && n1 == 16);
}
constexpr int kMaxRun = 1023;  // 10-bit run length
__host__ __device__ constexpr uint32_t make_desc(int kind, int n0, int n1, int bytes, int run = 1,
                                                 bool wide = false) {
  return (uint32_t)kind | ((uint32_t)(full_counts(kind, n0, n1, wide) ? 1 : 0) << 4) | ((uint32_t)n0 << 5) |
         ((uint32_t)n1 << 10) | ((uint32_t)(bytes >> 4) << 15) | ((uint32_t)run << 22);
}
__host__ __device__ inline int desc_kind(uint32_t d) { return (int)(d & 15u); }
__host__ __device__ inline bool desc_full(uint32_t d) { return (d >> 4) & 1u; }
__host__ __device__ inline int desc_n0(uint32_t d) { return (int)((d >> 5) & 31u); }
__host__ __device__ inline int desc_n1(uint32_t d) { return (int)((d >> 10) & 31u); }
__host__ __device__ inline int desc_bytes(uint32_t d) { return (int)(((d >> 15) & 127u) << 4); }
__host__ __device__ inline int desc_run(uint32_t d) { return (int)(d >> 22); }

// Bytes of a step record (the same in wide streams: a wide group step of n
// groups has 2 n lanes of two micro-blocks each).
__host__ __device__ inline int step_bytes(int kind, int n0, int n1) {
  if (kind < kU2) {
    const int c = kind, lanes = 4 * n0;
    return pad16(pad16(4 * n0) + lanes * (prim_bytes(c) + sec_bytes(c)));
  }
  const int nl = n0 + n1;
  if (kind == kGeneric) return pad16(8 * nl) + kGenericSlot * nl;
  const int c = kind - kU2;
  return pad16(pad16(4 * nl) + nl * (prim_bytes(c) + sec_bytes(c)));
}

// ---------------------------------------------------------------------------
// Code placement ("recipes").  A lane's 16 codes form 8 fp16 pairs, one per
// A-fragment register: pair k holds column c = (k & 1) + 2 (k >> 2) of the
// micro-block at k rows r0 = 2 ((k >> 1) & 1) (low half) and r0 + 1 (high
// half).  Pair k is built as
//     v = ((A[pw] >> prs) & (field(pbits) << p)) | 0x6400_6400
//       | (shift(B, ss) & (field(sbits) << (p + pbits)))
// which is the fp16 pair 1024 + 2^p u (u = q + 2^(m-1), the biased code),
// and q = v * 2^-p - (1024 * 2^-p + 2^(m-1)) follows from one exact HFMA2.
// B is the secondary plane word (16-bit planes spread to bytes 0 and 2);
// shift(B, s) = s >= 0 ? B >> s : B << -s.  The packer derives every bit's
// position from the same recipe, so the two cannot disagree.
// ---------------------------------------------------------------------------
struct Recipe {
  int pw, prs, p, pbits, ss, sbits;
};

__host__ __device__ constexpr Recipe recipe(int c, int k) {
  // P2: five pairs at p = 0, 2, .., 8 of word 0, three more from word 0 >> 10
  // P3: as P2's first four (p = 0..6) from A and A >> 8, high bit from B << 2 / B << 1
  // P4: nibble pairs at p = 0, 4 of A[w] and A[w] >> 8
  // P5: P4 layout, high bit from B << (4 - k/2)
  // P6: P4 layout, high 2-bit field from B shifted by -4, -2, 4, 6
  // P8: byte pairs (bytes j, j + 2) of A[k / 2]
  return c == 0 ? (k < 5 ? Recipe{0, 0, 2 * k, 2, 0, 0} : Recipe{0, 10, 2 * (k - 5), 2, 0, 0})
       : c == 1 ? (k < 4 ? Recipe{0, 0, 2 * k, 2, -2, 1} : Recipe{0, 8, 2 * (k - 4), 2, -1, 1})
       : c == 2 ? Recipe{k >> 2, 8 * ((k & 3) >> 1), 4 * (k & 1), 4, 0, 0}
       : c == 3 ? Recipe{k >> 2, 8 * ((k & 3) >> 1), 4 * (k & 1), 4, -(4 - (k >> 1)), 1}
       : c == 4 ? Recipe{k >> 2, 8 * ((k & 3) >> 1), 4 * (k & 1), 4,
                         (k >> 1) == 0 ? -4 : (k >> 1) == 1 ? -2 : (k >> 1) == 2 ? 4 : 6, 2}
                : Recipe{k >> 1, 8 * (k & 1), 0, 8, 0, 0};
}
__host__ __device__ constexpr int pair_col(int k) { return (k & 1) + 2 * (k >> 2); }
__host__ __device__ constexpr int pair_row(int k) { return 2 * ((k >> 1) & 1); }
__host__ __device__ constexpr uint32_t field2(int bits) { return ((1u << bits) - 1u) * 0x00010001u; }

// fp16 bits of an exactly representable normal value (compile-time constants).
__host__ __device__ constexpr uint16_t f16c(double v) {
  uint16_t sign = v < 0 ? 0x8000u : 0u;
  double a = v < 0 ? -v : v;
  if (a == 0.0) return sign;
  int e = 0;
  while (a >= 2.0) { a /= 2.0; ++e; }
  while (a < 1.0) { a *= 2.0; --e; }
  return (uint16_t)(sign | (uint16_t)((e + 15) << 10) | (uint16_t)((a - 1.0) * 1024.0));
}
__host__ __device__ constexpr uint32_t f16x2c(double v) { return (uint32_t)f16c(v) * 0x00010001u; }

// ---------------------------------------------------------------------------
// Scalar helpers with identical host and device results.
// ---------------------------------------------------------------------------
__host__ __device__ inline float h2f(uint16_t b) {
  __half_raw r;
  r.x = b;
  return __half2float(__half(r));
}
__host__ __device__ inline uint16_t f2h(float f) {
  __half_raw r = __half_raw(__float2half_rn(f));
  return r.x;
}

__host__ __device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
#ifdef __CUDA_ARCH__
  return __byte_perm(a, b, s);
#else
  const uint64_t x = ((uint64_t)b << 32) | a;
  uint32_t r = 0;
  for (int i = 0; i < 4; ++i) r |= (uint32_t)((x >> (8 * ((s >> (4 * i)) & 7u))) & 0xFFu) << (8 * i);
  return r;
#endif
}
// Two fp16 lanes: round(a * b + c) and round(a * b).
__host__ __device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
#ifdef __CUDA_ARCH__
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
#else
  // Every use in the decoder is exact (small integers), so fp32 evaluation
  // followed by one rounding gives the device result.
  uint32_t r = 0;
  for (int i = 0; i < 2; ++i) {
    const float v = h2f((uint16_t)(a >> 16 * i)) * h2f((uint16_t)(b >> 16 * i)) + h2f((uint16_t)(c >> 16 * i));
    r |= (uint32_t)f2h(v) << 16 * i;
  }
  return r;
#endif
}
__host__ __device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
#ifdef __CUDA_ARCH__
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
#else
  // The fp32 product of two fp16 values is exact; one rounding to fp16
  // matches mul.rn.f16x2 (subnormal results included).
  uint32_t r = 0;
  for (int i = 0; i < 2; ++i)
    r |= (uint32_t)f2h(h2f((uint16_t)(a >> 16 * i)) * h2f((uint16_t)(b >> 16 * i))) << 16 * i;
  return r;
#endif
}

// (a & b) | c and a | (b & c) as single LOP3s; c / the mask come in
// registers so both constants of a pair are available to one instruction.
template <uint32_t B>
__host__ __device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t c) {
#ifdef __CUDA_ARCH__
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "n"(B), "r"(c));
  return r;
#else
  return (a & B) | c;
#endif
}
template <uint32_t C>
__host__ __device__ __forceinline__ uint32_t lop3_or_and(uint32_t a, uint32_t b) {
#ifdef __CUDA_ARCH__
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xF8;" : "=r"(r) : "r"(a), "r"(b), "n"(C));
  return r;
#else
  return a | (b & C);
#endif
}

__host__ __device__ __forceinline__ uint32_t ldu32(const uint8_t* p) {
#ifdef __CUDA_ARCH__
  return *reinterpret_cast<const uint32_t*>(p);
#else
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
#endif
}
__host__ __device__ __forceinline__ uint32_t ldu16(const uint8_t* p) {
#ifdef __CUDA_ARCH__
  return *reinterpret_cast<const uint16_t*>(p);
#else
  uint16_t v;
  memcpy(&v, p, 2);
  return v;
#endif
}
__host__ __device__ __forceinline__ void ldwords(const uint8_t* p, uint32_t* w, int n) {
#ifdef __CUDA_ARCH__
  if (n == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
  } else if (n == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x, w[1] = v.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
#else
  memcpy(w, p, 4 * n);
#endif
}

// ---------------------------------------------------------------------------
// Lane decode: 16 codes -> 8 fp16 pairs of exact signed codes q.
// ---------------------------------------------------------------------------
template <int C, int K>
__host__ __device__ __forceinline__ uint32_t decode_pair(const uint32_t* A, uint32_t B) {
  constexpr Recipe r = recipe(C, K);
  constexpr uint32_t kMagic = 0x64006400u;
  uint32_t v;
  if constexpr (r.pbits == 8) {
    v = prmt(A[r.pw], 0x64646464u, (K & 1) ? 0x4341u : 0x4240u);  // bytes j and j + 2 over 0x64
  } else {
    v = lop3_and_or<(field2(r.pbits) << r.p)>(A[r.pw] >> r.prs, kMagic);
    if constexpr (r.sbits > 0) {
      const uint32_t s = r.ss >= 0 ? (B >> (r.ss >= 0 ? r.ss : 0)) : (B << (r.ss < 0 ? -r.ss : 0));
      v = lop3_or_and<(field2(r.sbits) << (r.p + r.pbits))>(v, s);
    }
  }
  constexpr double scale = 1.0 / (double)(1 << r.p);
  constexpr double offset = -(1024.0 * scale + (double)(1 << (mode_of_class(C) - 1)));
  return hfma2(v, f16x2c(scale), f16x2c(offset));
}

template <int C>
__host__ __device__ __forceinline__ void decode_lane(const uint32_t* A, uint32_t B, uint32_t a[8]) {
  a[0] = decode_pair<C, 0>(A, B);
  a[1] = decode_pair<C, 1>(A, B);
  a[2] = decode_pair<C, 2>(A, B);
  a[3] = decode_pair<C, 3>(A, B);
  a[4] = decode_pair<C, 4>(A, B);
  a[5] = decode_pair<C, 5>(A, B);
  a[6] = decode_pair<C, 6>(A, B);
  a[7] = decode_pair<C, 7>(A, B);
}

// Place the 16 codes of one lane per the class's recipes: A = primary plane
// words, B = secondary word in spread form (16-bit planes in bytes 0 and 2).
// Returns false if a recipe would place two bits on one position.
__host__ inline bool pack_lane(int cls, const int q[4][4], uint32_t A[4], uint32_t* B) {
  A[0] = A[1] = A[2] = A[3] = 0;
  *B = 0;
  uint32_t usedA[4] = {0, 0, 0, 0}, usedB = 0;
  const int m = mode_of_class(cls), bias = 1 << (m - 1);
  for (int k = 0; k < 8; ++k) {
    const Recipe rc = recipe(cls, k);
    for (int hh = 0; hh < 2; ++hh) {
      const uint32_t u = (uint32_t)(q[pair_row(k) + hh][pair_col(k)] + bias);
      for (int i = 0; i < rc.pbits; ++i) {
        const int pos = rc.p + i + 16 * hh + rc.prs;
        if (pos < 0 || pos > 31 || (usedA[rc.pw] >> pos & 1u)) return false;
        usedA[rc.pw] |= 1u << pos;
        A[rc.pw] |= ((u >> i) & 1u) << pos;
      }
      for (int i = 0; i < rc.sbits; ++i) {
        const int pos = rc.p + rc.pbits + i + 16 * hh + rc.ss;
        if (pos < 0 || pos > 31 || (usedB >> pos & 1u)) return false;
        usedB |= 1u << pos;
        *B |= ((u >> (rc.pbits + i)) & 1u) << pos;
      }
    }
  }
  return true;
}

// Spread a 16-bit secondary plane word to bytes 0 and 2.
__host__ __device__ __forceinline__ uint32_t spread16(uint32_t b16) { return prmt(b16, 0u, 0x4140u); }

// ---------------------------------------------------------------------------
// Lane operands of one step.
// ---------------------------------------------------------------------------
// Lane -> item mapping.  Group step with n groups: lane L takes group
// (L & 15) >> 1, k half L & 1 (rows 0-3 or 4-7), quartet L >> 4; valid when
// (L & 15) < 2 n; plane index (L & 15) + (L >> 4) 2 n.  Micro / generic step:
// lane L takes entry L (quartet 0, L < n0) or n0 + L - 16 (quartet 1,
// L - 16 < n1).
struct LaneSlot {
  bool valid;
  int idx;    // plane / entry index of the lane
  int eidx;   // entry index (group steps: the group)
  int lanes;  // plane entries in the step
  int nent;   // entries in the step
};

__host__ __device__ __forceinline__ LaneSlot lane_slot(bool group, int n0, int n1, int lane) {
  LaneSlot s;
  const int i = lane & 15, h = lane >> 4;
  if (group) {
    s.valid = i < 2 * n0;
    s.idx = s.valid ? i + h * 2 * n0 : 0;
    s.eidx = s.valid ? (i >> 1) : 0;
    s.lanes = 4 * n0;
    s.nent = n0;
  } else {
    s.valid = h ? (i < n1) : (i < n0);
    s.idx = s.valid ? (h ? n0 + i : i) : 0;
    s.eidx = s.idx;
    s.lanes = n0 + n1;
    s.nent = n0 + n1;
  }
  return s;
}

// A fragments (a[0..3]: columns 0, 1; a[4..7]: columns 2, 3) and B fragments
// (x * scale at the lane's k rows, per token) of a fast-class lane.  Invalid
// lanes decode whatever sits at plane index 0 and get a zero scale, so their
// products are zero.  FULL steps take every lane, so all offsets are
// constants.
template <int C, bool GROUP, bool FULL, int MT>
__host__ __device__ __forceinline__ void lane_fast(const uint8_t* step, int n0, int n1, int lane,
                                                   const uint16_t* x16, int kpad, uint32_t a[8],
                                                   uint32_t b[MT][2]) {
  constexpr int PB = prim_bytes(C), SB = sec_bytes(C);
  uint32_t e;
  const uint8_t *pa, *pb;
  if constexpr (FULL) {
    constexpr int NENT = GROUP ? 8 : 32, E = pad16(4 * NENT);
    e = ldu32(step + 4 * (GROUP ? ((lane & 15) >> 1) : lane));
    pa = step + E + lane * PB;
    pb = step + E + 32 * PB + lane * SB;
  } else {
    const LaneSlot s = lane_slot(GROUP, n0, n1, lane);
    e = s.valid ? ldu32(step + 4 * s.eidx) : 0u;
    const uint8_t* planes = step + pad16(4 * s.nent);
    pa = planes + s.idx * PB;
    pb = planes + s.lanes * PB + s.idx * SB;
  }
  uint32_t A[PB / 4];
  ldwords(pa, A, PB / 4);
  uint32_t B = 0;
  if constexpr (SB == 2) B = spread16(ldu16(pb));
  if constexpr (SB == 4) B = ldu32(pb);
  decode_lane<C>(A, B, a);
  const int xo = GROUP ? (int)(e >> 16) * 8 + (lane & 1) * 4 : (int)(e >> 16) * 4;
  const uint32_t s2 = prmt(e, e, 0x1010u);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const uint8_t* xp = reinterpret_cast<const uint8_t*>(x16 + (size_t)m * kpad + xo);
    uint32_t xw[2];
    ldwords(xp, xw, 2);
    b[m][0] = hmul2(xw[0], s2);
    b[m][1] = hmul2(xw[1], s2);
  }
}

// Wide group step lane: group L >> 1, k half L & 1, both quartets.  a0 / a1
// are the A fragments of quartet 0 / 1 (columns 0-3 / 4-7 of the strip); b is
// shared by the four MMAs.  Plane A holds the lane's two micro-blocks side by
// side (2 prim_bytes), plane B likewise (2 sec_bytes).
template <int C, bool FULL, int MT>
__host__ __device__ __forceinline__ void lane_wide(const uint8_t* step, int n, int lane, const uint16_t* x16,
                                                   int kpad, uint32_t a0[8], uint32_t a1[8], uint32_t b[MT][2]) {
  constexpr int PB = prim_bytes(C), SB = sec_bytes(C);
  const bool valid = FULL || lane < 2 * n;
  const int idx = valid ? lane : 0;
  const int lanes = FULL ? 32 : 2 * n;
  const int E = FULL ? 64 : pad16(4 * n);
  const uint32_t e = valid ? ldu32(step + 4 * (lane >> 1)) : 0u;
  const uint8_t* pa = step + E + idx * 2 * PB;
  const uint8_t* pb = step + E + lanes * 2 * PB + idx * 2 * SB;
  uint32_t A[2 * PB / 4];
  if constexpr (PB == 16) {
    ldwords(pa, A, 4);
    ldwords(pa + 16, A + 4, 4);
  } else {
    ldwords(pa, A, 2 * PB / 4);
  }
  uint32_t B0 = 0, B1 = 0;
  if constexpr (SB == 2) {
    const uint32_t w = ldu32(pb);
    B0 = spread16(w & 0xFFFFu);
    B1 = spread16(w >> 16);
  }
  if constexpr (SB == 4) {
    uint32_t w[2];
    ldwords(pb, w, 2);
    B0 = w[0];
    B1 = w[1];
  }
  decode_lane<C>(A, B0, a0);
  decode_lane<C>(A + PB / 4, B1, a1);
  const int xo = (int)(e >> 16) * 8 + (lane & 1) * 4;
  const uint32_t s2 = prmt(e, e, 0x1010u);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const uint8_t* xp = reinterpret_cast<const uint8_t*>(x16 + (size_t)m * kpad + xo);
    uint32_t xw[2];
    ldwords(xp, xw, 2);
    b[m][0] = hmul2(xw[0], s2);
    b[m][1] = hmul2(xw[1], s2);
  }
}

// Generic lane: fp32 products into g[m][c] (c = column of the lane's quartet).
// Code i of the micro-block (row-major) is the m-bit field at bit i m of the
// lane's 32-byte slot, read through a two-byte window.
template <int MT>
__host__ __device__ __forceinline__ void lane_generic(const uint8_t* step, int n0, int n1, int lane,
                                                      const uint16_t* x16, int kpad, float g[MT][4]) {
  const LaneSlot s = lane_slot(false, n0, n1, lane);
  if (!s.valid) return;
  const uint32_t e0 = ldu32(step + 8 * s.idx), e1 = ldu32(step + 8 * s.idx + 4);
  float sc;
  memcpy(&sc, &e0, 4);
  const int row4 = (int)(e1 & 0xFFFFu), mode = (int)((e1 >> 16) & 31u);
  const uint8_t* codes = step + pad16(8 * s.nent) + kGenericSlot * s.idx;
  float xr[MT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int r = 0; r < 4; ++r) xr[m][r] = h2f(x16[(size_t)m * kpad + row4 * 4 + r]) * sc;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int bit = i * mode;
    const uint32_t win = (uint32_t)codes[bit >> 3] | ((uint32_t)codes[(bit >> 3) + 1] << 8) |
                         ((uint32_t)codes[(bit >> 3) + 2 < kGenericSlot ? (bit >> 3) + 2 : kGenericSlot - 1] << 16);
    const uint32_t u = (win >> (bit & 7)) & ((1u << mode) - 1u);
    const float q = (float)((int)(u << (32 - mode)) >> (32 - mode));
    const int r = i >> 2, c = i & 3;
#pragma unroll
    for (int m = 0; m < MT; ++m) g[m][c] += q * xr[m][r];
  }
}

}  // namespace strip
}  // namespace mtc
