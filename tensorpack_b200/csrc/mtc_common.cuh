// Device-side helpers shared by the MTC kernels: the tile-stream format,
// micro-block decoders, and thin PTX wrappers (mbarrier, bulk copies, mma).
//
// Tile stream format (all kernels agree on it; the repack writes it):
//   * W (stored permuted, K x N) is cut into 32x32 tiles, each tile into an
//     8x8 grid of 4x4 micro-blocks (mb).  Micro-blocks are numbered in Z
//     order: z = i2 j2 i1 j1 i0 j0 (i = mb row, j = mb column, bit 2 first),
//     so every quadtree leaf (edge 4..32, aligned) is a contiguous z range.
//   * Codes are stored biased, u = q + 2^(m-1), split into a primary plane of
//     width wp and a secondary plane of width ws:  P2 (2,0) P3 (2,1)
//     P4 (4,0) P5 (4,1) P6 (4,2) P8 (8,0); P16 keeps signed int16 codes.
//   * An mb is read as two halves h = 0, 1 (mb columns 2h and 2h+1); a half
//     holds four code pairs j = 0..3: pair j = (column 2h + (j>>1),
//     rows 2(j&1) and 2(j&1)+1) as (lo, hi).  Plane layouts per mb:
//       width 1 (2 B):  code (h, j, lo/hi) at bit 4h + j + 8*hi
//       width 2 (4 B):  code (h, j, lo/hi) at bit 8h + 2j + 16*hi
//       width 4 (8 B):  word h, code (j, lo/hi) at bit 4(j&1) + 8(j>>1) + 16*hi
//       width 8 (16 B): half h = 2 words, word j>>1, byte (j&1) + 2*hi
//       P16   (32 B):   half h = 4 words, word j = lo16 | hi16 << 16 (signed)
//     These positions let one LOP3 against 0x6400 (fp16 1024.0) produce two
//     fp16 values (1024 + 2^p u) that one HFMA2 turns into exact codes.
//   * Primary planes of the tile's mbs are concatenated in z order, then the
//     secondary planes; offsets are prefix sums over z (computed in-kernel).
//     Primary offsets are multiples of 4 bytes, secondary offsets multiples
//     of 2, so secondary planes are read in 16-bit units.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mtc_b200.h"


namespace mtc {

constexpr int kTile = 32;
constexpr int kMbPerTile = 64;
constexpr uint32_t kMagic = 0x64006400u;  // two fp16 1024.0

__host__ __device__ constexpr int pad16(int x) { return (x + 15) & ~15; }

// Primary / secondary plane bytes per micro-block for each mode.
__host__ __device__ inline int mb_prim_bytes(int m) {
  switch (m) {
    case 2: case 3: return 4;
    case 4: case 5: case 6: return 8;
    case 8: return 16;
    case 16: return 32;
    default: return 0;
  }
}
__host__ __device__ inline int mb_sec_bytes(int m) {
  switch (m) {
    case 3: case 5: return 2;
    case 6: return 4;
    default: return 0;
  }
}
__host__ __device__ inline int prim_width(int m) {
  switch (m) {
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 8: return 8;
    case 16: return 16;
    default: return 0;
  }
}

// Leaf-table entry fields.
__device__ __forceinline__ int lt_mode(uint32_t e) { return e & 31u; }
__device__ __forceinline__ int lt_prim(uint32_t e) { return ((e >> 8) & 15u) * 4; }
__device__ __forceinline__ int lt_sec(uint32_t e) { return ((e >> 12) & 3u) * 2; }
__device__ __forceinline__ bool lt_slow(uint32_t e) { return (e >> 14) & 1u; }
__device__ __forceinline__ float lt_scale(uint32_t e) { return __uint_as_float(e & 0xffff0000u); }
// Leaf-table entry and scale of leaf L (sw = scale words per leaf, 1 or 2).
__device__ __forceinline__ uint32_t lt_entry(const uint32_t* ltab, int L, int sw) { return ltab[L * sw]; }
__device__ __forceinline__ float lt_scale_of(const uint32_t* ltab, int L, int sw) {
  return sw == 2 ? __uint_as_float(ltab[2 * L + 1]) : lt_scale(ltab[L]);
}

// Z order <-> (mb row, mb column) inside a tile.
__host__ __device__ inline int z_of(int i, int j) {
  return ((i >> 2) & 1) << 5 | ((j >> 2) & 1) << 4 | ((i >> 1) & 1) << 3 | ((j >> 1) & 1) << 2 |
         (i & 1) << 1 | (j & 1);
}
__host__ __device__ inline int z_row(int z) {
  return ((z >> 5) & 1) << 2 | ((z >> 3) & 1) << 1 | ((z >> 1) & 1);
}
__host__ __device__ inline int z_col(int z) {
  return ((z >> 4) & 1) << 2 | ((z >> 2) & 1) << 1 | (z & 1);
}

// Leaf index of micro-block z given the tile's leaf-start mask.
__device__ __forceinline__ int leaf_of(uint64_t start, int z) {
  uint64_t m = (z >= 63) ? ~0ull : ((2ull << z) - 1ull);
  return __popcll(start & m) - 1;
}

// ---------------------------------------------------------------------------
// Code extraction helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t lop_or(uint32_t x, uint32_t mask) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(x), "r"(mask), "r"(kMagic));
  return r;
}
__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__host__ __device__ constexpr uint32_t h2const(uint16_t bits) {
  return (uint32_t)bits | ((uint32_t)bits << 16);
}

// fp16 bit pattern of an exactly representable normal (or zero) value,
// evaluated at compile time for the decoder constants.
__host__ __device__ constexpr uint16_t f16_bits(double v) {
  uint16_t sign = v < 0 ? 0x8000u : 0u;
  double a = v < 0 ? -v : v;
  if (a == 0.0) return sign;
  int e = 0;
  while (a >= 2.0) { a /= 2.0; ++e; }
  while (a < 1.0) { a *= 2.0; --e; }
  return (uint16_t)(sign | (uint16_t)((e + 15) << 10) | (uint16_t)((a - 1.0) * 1024.0));
}
__host__ __device__ constexpr uint32_t k2(double v) { return h2const(f16_bits(v)); }

// Load helpers (generic pointers into shared or global memory).
__device__ __forceinline__ uint32_t ld32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t ld16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// Pair decoders: each returns two exact fp16 codes (lo row, hi row).
// A field of a p-bit position inside each 16-bit half, OR-ed into 1024.0,
// reads 1024 + 2^p u; scaling by 2^-p and subtracting 1024 2^-p + bias is
// exact because every intermediate is a small integer.
template <int J>
__device__ __forceinline__ uint32_t pair_p2(uint32_t v) {  // v = plane word >> 8h
  constexpr double c = 1.0 / double(1 << (2 * J));
  return hfma2u(lop_or(v, 0x00030003u << (2 * J)), k2(c), k2(-1024.0 * c - 2.0));
}
template <int J>
__device__ __forceinline__ uint32_t nib_field(uint32_t w) {  // P4-style nibble plane word
  return lop_or((J >> 1) ? (w >> 8) : w, (J & 1) ? 0x00F000F0u : 0x000F000Fu);
}
template <int J>
__device__ __forceinline__ uint32_t pair_p4(uint32_t w) {
  constexpr double c = (J & 1) ? 1.0 / 16.0 : 1.0;
  return hfma2u(nib_field<J>(w), k2(c), k2(-1024.0 * c - 8.0));
}
template <int J>
__device__ __forceinline__ uint32_t pair_p8(uint32_t w0, uint32_t w1) {
  uint32_t w = (J >> 1) ? w1 : w0;
  return hfma2u(lop_or((J & 1) ? (w >> 8) : w, 0x00FF00FFu), k2(1.0), k2(-1152.0));
}
// P3: primary crumb plane (u & 3) + bit plane (u >> 2); v1 = bit plane >> 4h.
template <int J>
__device__ __forceinline__ uint32_t pair_p3(uint32_t v, uint32_t v1) {
  constexpr double c2 = 1.0 / double(1 << (2 * J));
  constexpr double c1 = 4.0 / double(1 << J);
  uint32_t inner = hfma2u(lop_or(v1, 0x00010001u << J), k2(c1), k2(-1024.0 * c1 - 4.0 - 1024.0 * c2));
  return hfma2u(lop_or(v, 0x00030003u << (2 * J)), k2(c2), inner);
}
// P5: nibble plane + bit plane (u >> 4); P6: nibble plane + crumb plane (u >> 4).
template <int MODE, int J>
__device__ __forceinline__ uint32_t pair_p56(uint32_t w, uint32_t vs) {
  constexpr double c4 = (J & 1) ? 1.0 / 16.0 : 1.0;
  constexpr double bias = (MODE == 5) ? 16.0 : 32.0;
  constexpr double cs = (MODE == 5) ? 16.0 / double(1 << J) : 16.0 / double(1 << (2 * J));
  constexpr uint32_t mask = (MODE == 5) ? (0x00010001u << J) : (0x00030003u << (2 * J));
  uint32_t inner = hfma2u(lop_or(vs, mask), k2(cs), k2(-1024.0 * cs - bias - 1024.0 * c4));
  return hfma2u(nib_field<J>(w), k2(c4), inner);
}

// Decode one half micro-block into four fp16x2 registers holding the exact
// codes q (pairs j = 0..3), for every mode except P16 and P0.
// prim/sec point at this mb's primary / secondary plane bytes.
__device__ __forceinline__ void decode_half_codes(int mode, const uint8_t* prim, const uint8_t* sec,
                                                  int h, uint32_t q[4]) {
  switch (mode) {
    case 2: {
      uint32_t v = ld32(prim) >> (8 * h);
      q[0] = pair_p2<0>(v); q[1] = pair_p2<1>(v); q[2] = pair_p2<2>(v); q[3] = pair_p2<3>(v);
      break;
    }
    case 4: {
      uint32_t w = ld32(prim + 4 * h);
      q[0] = pair_p4<0>(w); q[1] = pair_p4<1>(w); q[2] = pair_p4<2>(w); q[3] = pair_p4<3>(w);
      break;
    }
    case 8: {
      uint32_t w0 = ld32(prim + 8 * h), w1 = ld32(prim + 8 * h + 4);
      q[0] = pair_p8<0>(w0, w1); q[1] = pair_p8<1>(w0, w1);
      q[2] = pair_p8<2>(w0, w1); q[3] = pair_p8<3>(w0, w1);
      break;
    }
    case 3: {
      uint32_t v = ld32(prim) >> (8 * h);
      uint32_t v1 = __byte_perm(ld16(sec), 0u, 0x4140) >> (4 * h);
      q[0] = pair_p3<0>(v, v1); q[1] = pair_p3<1>(v, v1);
      q[2] = pair_p3<2>(v, v1); q[3] = pair_p3<3>(v, v1);
      break;
    }
    case 5: {
      uint32_t w = ld32(prim + 4 * h);
      uint32_t vs = __byte_perm(ld16(sec), 0u, 0x4140) >> (4 * h);
      q[0] = pair_p56<5, 0>(w, vs); q[1] = pair_p56<5, 1>(w, vs);
      q[2] = pair_p56<5, 2>(w, vs); q[3] = pair_p56<5, 3>(w, vs);
      break;
    }
    case 6: {
      uint32_t w = ld32(prim + 4 * h);
      uint32_t vs = (ld16(sec) | (ld16(sec + 2) << 16)) >> (8 * h);
      q[0] = pair_p56<6, 0>(w, vs); q[1] = pair_p56<6, 1>(w, vs);
      q[2] = pair_p56<6, 2>(w, vs); q[3] = pair_p56<6, 3>(w, vs);
      break;
    }
    default:
      q[0] = q[1] = q[2] = q[3] = 0u;
  }
}

// Integer codes of one half micro-block (exact path used by the dequant
// kernel and the repack self-check): code[2j + hi].
__device__ __forceinline__ void decode_half_int(int mode, const uint8_t* prim, const uint8_t* sec,
                                                int h, int code[8]) {
  if (mode == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) code[i] = 0;
    return;
  }
  if (mode == 16) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w = ld32(prim + 16 * h + 4 * j);
      code[2 * j] = (int)(int16_t)(w & 0xffffu);
      code[2 * j + 1] = (int)(int16_t)(w >> 16);
    }
    return;
  }
  const int wp = prim_width(mode);
  const int bias = 1 << (mode - 1);
  uint32_t pw0 = 0, pw1 = 0, sv = 0;
  if (wp == 2) pw0 = ld32(prim);
  if (wp == 4) pw0 = ld32(prim + 4 * h);
  if (wp == 8) { pw0 = ld32(prim + 8 * h); pw1 = ld32(prim + 8 * h + 4); }
  if (mode == 3 || mode == 5) sv = ld16(sec);
  if (mode == 6) sv = ld16(sec) | (ld16(sec + 2) << 16);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int hi = 0; hi < 2; ++hi) {
      uint32_t u = 0;
      if (wp == 2) u = (pw0 >> (8 * h + 2 * j + 16 * hi)) & 3u;
      if (wp == 4) u = (pw0 >> (4 * (j & 1) + 8 * (j >> 1) + 16 * hi)) & 15u;
      if (wp == 8) u = (((j >> 1) ? pw1 : pw0) >> (8 * ((j & 1) + 2 * hi))) & 255u;
      if (mode == 3) u |= ((sv >> (4 * h + j + 8 * hi)) & 1u) << 2;
      if (mode == 5) u |= ((sv >> (4 * h + j + 8 * hi)) & 1u) << 4;
      if (mode == 6) u |= ((sv >> (8 * h + 2 * j + 16 * hi)) & 3u) << 4;
      code[2 * j + hi] = (int)u - bias;
    }
  }
}

// fp16 weights W*2^e of one half micro-block as four f16x2 registers:
// pair j = (row lo, row hi) of column 2h + (j>>1).
__device__ __forceinline__ void decode_half_w16(uint32_t entry, float scale, const uint8_t* prim,
                                                const uint8_t* sec, int h, float pow2e, uint32_t r[4]) {
  const int mode = lt_mode(entry);
  if (mode == 0) {
    r[0] = r[1] = r[2] = r[3] = 0u;
    return;
  }
  if (mode == 16 || lt_slow(entry)) {
    int code[8];
    decode_half_int(mode, prim, sec, h, code);
    const float s = scale * pow2e;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __half2 v = __floats2half2_rn(__fmul_rn((float)code[2 * j], s), __fmul_rn((float)code[2 * j + 1], s));
      r[j] = *reinterpret_cast<uint32_t*>(&v);
    }
    return;
  }
  uint32_t q[4];
  decode_half_codes(mode, prim, sec, h, q);
  __half s16 = __float2half_rn(scale * pow2e);
  const uint32_t s2 = h2const(*reinterpret_cast<uint16_t*>(&s16));
#pragma unroll
  for (int j = 0; j < 4; ++j) r[j] = hmul2u(q[j], s2);
}

// Decode, for one tile record, the aligned 2x2 micro-block group owned by
// this lane into fp16 (W * 2^e) pairs.  All 32 lanes of the warp must call
// it together (it scans group sizes with shuffles).  Lane (g, t) =
// (lane >> 2, lane & 3) owns group (t, jj = g >> 1) and column half h = g & 1;
// R[k] (k = 2 di + dj) is micro-block (2t + di, 2jj + dj), pairs j = 0..3 as
// in decode_half_w16.
__device__ __forceinline__ int group_of_lane(int lane) {
  const int t = lane & 3, jj = lane >> 3;
  return ((t >> 1) << 3) | ((jj >> 1) << 2) | ((t & 1) << 1) | (jj & 1);
}

// Per-lane constants of the group decode, computed once per kernel.
struct GroupLane {
  int z0;       // first micro-block (Z order) of this lane's group
  int h;        // column half
  int src[4];   // scan partner lane for distance 1, 2, 4, 8 (own lane if none)
  uint32_t live;  // bit i set when the partner for distance 2^i exists
};

__device__ __forceinline__ GroupLane make_group_lane(int lane) {
  GroupLane c;
  const int G = group_of_lane(lane);
  c.z0 = 4 * G;
  c.h = (lane >> 2) & 1;
  c.live = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int Gs = G - (1 << i);
    const int ts = ((Gs >> 3) & 1) << 1 | ((Gs >> 1) & 1);
    const int js = ((Gs >> 2) & 1) << 1 | (Gs & 1);
    c.src[i] = (Gs >= 0) ? (8 * js + ts) : lane;
    if (Gs >= 0) c.live |= 1u << i;
  }
  return c;
}

// Four micro-blocks of one mode, consecutive in the plane regions: the
// group of a leaf of edge >= 8.  pb / sb = plane bytes per micro-block.
template <int MODE>
__device__ __forceinline__ void decode_run4(const uint8_t* prim, const uint8_t* sec, int h, uint32_t s2,
                                            uint32_t R[4][4]) {
  constexpr int pb = (MODE == 2 || MODE == 3) ? 4 : (MODE == 8 ? 16 : 8);
  constexpr int sb = (MODE == 3 || MODE == 5) ? 2 : (MODE == 6 ? 4 : 0);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t q[4];
    decode_half_codes(MODE, prim + k * pb, sec + k * sb, h, q);
#pragma unroll
    for (int j = 0; j < 4; ++j) R[k][j] = hmul2u(q[j], s2);
  }
}

// ---------------------------------------------------------------------------
// Mode-uniform ("two-plane") decoder used when the lanes of a warp hold
// groups of different modes: one instruction sequence for P2..P8 driven by a
// per-mode parameter table, so no lane waits on another lane's branch.
//   q = fma(prim_field, c, fma(sec_field, cs, K))
// prim_field = (x_j & pmask_j) | 1024.0, sec_field likewise with smask_j
// (zero mask for single-plane modes: the field then reads 1024 exactly and K
// cancels it).  All intermediate values are small integers, so exact.
// ---------------------------------------------------------------------------
struct DecRow {  // 20 words per mode: pmask[4] smask[4] c[4] cs[4] K[4]
  uint32_t w[20];
};

__host__ __device__ constexpr DecRow make_dec_row(int mode) {
  DecRow r{};
  const int wp = (mode == 2 || mode == 3) ? 2 : (mode == 8 ? 8 : 4);
  const int ws = (mode == 3 || mode == 5) ? 1 : (mode == 6 ? 2 : 0);
  const double bias = double(1 << (mode - 1));
  for (int j = 0; j < 4; ++j) {
    uint32_t pm = 0;
    int pos = 0;
    if (wp == 2) { pm = 0x00030003u << (2 * j); pos = 2 * j; }
    if (wp == 4) { pm = (j & 1) ? 0x00F000F0u : 0x000F000Fu; pos = (j & 1) ? 4 : 0; }
    if (wp == 8) { pm = 0x00FF00FFu; pos = 0; }
    uint32_t sm = 0;
    double cs = 0.0;
    if (ws == 1) { sm = 0x00010001u << j; cs = double(1 << wp) / double(1 << j); }
    if (ws == 2) { sm = 0x00030003u << (2 * j); cs = double(1 << wp) / double(1 << (2 * j)); }
    const double c = 1.0 / double(1 << pos);
    r.w[j] = pm;
    r.w[4 + j] = sm;
    r.w[8 + j] = k2(c);
    r.w[12 + j] = k2(cs);
    r.w[16 + j] = k2(-1024.0 * cs - bias - 1024.0 * c);
  }
  return r;
}

// decode class of a mode: 0 = P0, 1..6 = P2, P3, P4, P5, P6, P8, 7 = P16
__device__ __forceinline__ int dec_class_of(int m) {
  return m > 8 ? 7 : (int)((0x675432170ull >> (4 * m)) & 15ull);
}

// mode -> row of the parameter table (2,3,4,5,6,8 -> 0..5)
__device__ __forceinline__ int dec_row_index(int mode) { return (0x5F43210u >> (4 * (mode - 2))) & 15u; }

// The table, built at compile time (rows for modes 2, 3, 4, 5, 6, 8).
static __constant__ DecRow kDecTable[6] = {make_dec_row(2), make_dec_row(3), make_dec_row(4),
                                           make_dec_row(5), make_dec_row(6), make_dec_row(8)};

// Copy the table (6 rows x 20 words) into shared memory; call by one warp.
__device__ __forceinline__ void load_dec_table(uint32_t* dst, int lane) {
  const uint32_t* src = reinterpret_cast<const uint32_t*>(kDecTable);
  for (int i = lane; i < 120; i += 32) dst[i] = src[i];
}

// One micro-block half with the table row `tab` (P2..P8).
__device__ __forceinline__ void decode_half_uniform(const uint32_t* tab, int mode, const uint8_t* prim,
                                                    const uint8_t* sec, int h, uint32_t s2, uint32_t r[4]) {
  const int wp = (mode == 2 || mode == 3) ? 2 : (mode == 8 ? 8 : 4);
  const int ws = (mode == 3 || mode == 5) ? 1 : (mode == 6 ? 2 : 0);
  const int offA = (wp == 2) ? 0 : (wp == 4 ? 4 * h : 8 * h);
  const int offB = (wp == 8) ? 8 * h + 4 : offA;
  const uint32_t A = ld32(prim + offA) >> ((wp == 2) ? 8 * h : 0);
  const uint32_t B = ld32(prim + offB) >> ((wp == 2) ? 8 * h : 0);
  const uint32_t x[4] = {A, A >> (wp == 8 ? 8 : 0), B >> (wp == 4 ? 8 : 0), B >> (wp == 2 ? 0 : 8)};
  uint32_t S = 0;
  if (ws == 1) S = __byte_perm(ld16(sec), 0u, 0x4140) >> (4 * h);
  if (ws == 2) S = (ld16(sec) | (ld16(sec + 2) << 16)) >> (8 * h);
  const uint4 pm = *reinterpret_cast<const uint4*>(tab);
  const uint4 sm = *reinterpret_cast<const uint4*>(tab + 4);
  const uint4 c = *reinterpret_cast<const uint4*>(tab + 8);
  const uint4 cs = *reinterpret_cast<const uint4*>(tab + 12);
  const uint4 K = *reinterpret_cast<const uint4*>(tab + 16);
  r[0] = hmul2u(hfma2u(lop_or(x[0], pm.x), c.x, hfma2u(lop_or(S, sm.x), cs.x, K.x)), s2);
  r[1] = hmul2u(hfma2u(lop_or(x[1], pm.y), c.y, hfma2u(lop_or(S, sm.y), cs.y, K.y)), s2);
  r[2] = hmul2u(hfma2u(lop_or(x[2], pm.z), c.z, hfma2u(lop_or(S, sm.z), cs.z, K.z)), s2);
  r[3] = hmul2u(hfma2u(lop_or(x[3], pm.w), c.w, hfma2u(lop_or(S, sm.w), cs.w, K.w)), s2);
}

// One micro-block half of decode class c (0 = P0 zeros; 1..6 = P2, P3, P4,
// P5, P6, P8) through the table decoder, without branches: lanes of
// different classes run the same instructions, and several calls can be
// interleaved by the compiler.  Both 16-bit secondary words are always read
// (they lie inside the staged records, or just past them in shared memory).
// tab = the decoder table in shared memory.
__device__ __forceinline__ void decode_half_class(const uint32_t* tab, int c, const uint8_t* prim,
                                                  const uint8_t* sec, int h, uint32_t s2, uint32_t r[4]) {
  const int cc = c > 0 ? c : 1;
  const bool w2 = cc <= 2, w8 = cc == 6, w4 = !w2 && !w8;       // primary plane width 2 / 4 / 8
  const bool s1 = cc == 2 || cc == 4, s2w = cc == 5;             // secondary plane width 1 / 2
  const int offA = w2 ? 0 : (w4 ? 4 * h : 8 * h);
  const int offB = w8 ? 8 * h + 4 : offA;
  const uint32_t A = ld32(prim + offA) >> (w2 ? 8 * h : 0);
  const uint32_t B = ld32(prim + offB) >> (w2 ? 8 * h : 0);
  const uint32_t x0 = A, x1 = A >> (w8 ? 8 : 0), x2 = B >> (w4 ? 8 : 0), x3 = B >> (w2 ? 0 : 8);
  const uint32_t lo = ld16(sec), hi = ld16(sec + 2);
  const uint32_t S = s1 ? (__byte_perm(lo, 0u, 0x4140) >> (4 * h)) : (s2w ? ((lo | (hi << 16)) >> (8 * h)) : 0u);
  const uint32_t* row = tab + 20 * (cc - 1);
  const uint4 pm = *reinterpret_cast<const uint4*>(row);
  const uint4 sm = *reinterpret_cast<const uint4*>(row + 4);
  const uint4 cf = *reinterpret_cast<const uint4*>(row + 8);
  const uint4 cs = *reinterpret_cast<const uint4*>(row + 12);
  const uint4 K = *reinterpret_cast<const uint4*>(row + 16);
  const uint32_t sc = c > 0 ? s2 : 0u;
  r[0] = hmul2u(hfma2u(lop_or(x0, pm.x), cf.x, hfma2u(lop_or(S, sm.x), cs.x, K.x)), sc);
  r[1] = hmul2u(hfma2u(lop_or(x1, pm.y), cf.y, hfma2u(lop_or(S, sm.y), cs.y, K.y)), sc);
  r[2] = hmul2u(hfma2u(lop_or(x2, pm.z), cf.z, hfma2u(lop_or(S, sm.z), cs.z, K.z)), sc);
  r[3] = hmul2u(hfma2u(lop_or(x3, pm.w), cf.w, hfma2u(lop_or(S, sm.w), cs.w, K.w)), sc);
}

// Four micro-blocks of one leaf (a group), decode class c, through the table
// decoder (lanes of different classes run the same instructions).
__device__ __forceinline__ void decode_run4_class(const uint32_t* tab, int c, const uint8_t* prim,
                                                  const uint8_t* sec, int h, uint32_t s2, uint32_t R[4][4]) {
  const int pb = c == 6 ? 16 : (c <= 2 ? 4 : 8);
  const int sb = (c == 2 || c == 4) ? 2 : (c == 5 ? 4 : 0);
#pragma unroll
  for (int k = 0; k < 4; ++k) decode_half_class(tab, c, prim + k * pb, sec + k * sb, h, s2, R[k]);
}

// Any group through the per-micro-block path (four 4x4 leaves of possibly
// different modes, P16, inexact fp16 scales).  prim / sec = group base.
__device__ __forceinline__ void decode_group_generic(const uint32_t* ltab, uint64_t leaf_start, int G,
                                                     const uint8_t* prim, const uint8_t* sec, int sw, int h,
                                                     float pow2e, uint32_t R[4][4]) {
  const int z0 = 4 * G;
  const int l0 = leaf_of(leaf_start, z0);
  const bool single = ((leaf_start >> (z0 + 1)) & 7ull) == 0ull;
  uint32_t po = 0, so = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int L = single ? l0 : l0 + k;
    const uint32_t e = lt_entry(ltab, L, sw);
    decode_half_w16(e, lt_scale_of(ltab, L, sw), prim + po, sec + so, h, pow2e, R[k]);
    po += lt_prim(e);
    so += lt_sec(e);
  }
}

// One micro-block half of a known mode, scaled: four fp16x2 weight pairs.
template <int MODE>
__device__ __forceinline__ void decode_mb_half(const uint8_t* prim, const uint8_t* sec, int h, uint32_t s2,
                                               uint32_t r[4]) {
  uint32_t q[4];
  decode_half_codes(MODE, prim, sec, h, q);
#pragma unroll
  for (int j = 0; j < 4; ++j) r[j] = hmul2u(q[j], s2);
}

__device__ __forceinline__ uint32_t half2_bits(float v) {
  __half x = __float2half_rn(v);
  return h2const(*reinterpret_cast<uint16_t*>(&x));
}

__device__ __forceinline__ void decode_group_w16(const uint8_t* rec, uint16_t n_leaves, uint16_t prim_bytes,
                                                 uint64_t leaf_start, int sw, const GroupLane& c, float pow2e,
                                                 const uint32_t* dtab, uint32_t R[4][4]) {
  const uint32_t* ltab = reinterpret_cast<const uint32_t*>(rec);
  const uint8_t* prim_base = rec + pad16(4 * sw * n_leaves);
  const uint8_t* sec_base = prim_base + pad16(prim_bytes);
  const int l0 = leaf_of(leaf_start, c.z0);
  const bool single = ((leaf_start >> (c.z0 + 1)) & 7ull) == 0ull;
  const uint32_t e0 = lt_entry(ltab, l0, sw);
  uint32_t v;
  if (single) {
    v = 4u * ((uint32_t)lt_prim(e0) | ((uint32_t)lt_sec(e0) << 16));
  } else {
    v = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t e = lt_entry(ltab, l0 + k, sw);
      v += (uint32_t)lt_prim(e) | ((uint32_t)lt_sec(e) << 16);
    }
  }
  // exclusive scan of group sizes over the 16 groups in Z order
  uint32_t incl = v;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t u = __shfl_sync(0xffffffffu, incl, c.src[i]);
    if (c.live & (1u << i)) incl += u;
  }
  const uint32_t ex = incl - v;
  const uint8_t* prim = prim_base + (ex & 0xffffu);
  const uint8_t* sec = sec_base + (ex >> 16);
  const int mode0 = lt_mode(e0);
  const bool fast = single && mode0 != 16 && !lt_slow(e0);
  const int mode_l0 = __shfl_sync(0xffffffffu, mode0, 0);
  if (__all_sync(0xffffffffu, fast && mode0 == mode_l0)) {
    // every lane holds a single-leaf group of the same mode: specialised path
    const uint32_t s2 = half2_bits(lt_scale_of(ltab, l0, sw) * pow2e);
    switch (mode_l0) {
      case 2: decode_run4<2>(prim, sec, c.h, s2, R); return;
      case 3: decode_run4<3>(prim, sec, c.h, s2, R); return;
      case 4: decode_run4<4>(prim, sec, c.h, s2, R); return;
      case 5: decode_run4<5>(prim, sec, c.h, s2, R); return;
      case 6: decode_run4<6>(prim, sec, c.h, s2, R); return;
      case 8: decode_run4<8>(prim, sec, c.h, s2, R); return;
      default:
#pragma unroll
        for (int k = 0; k < 4; ++k) R[k][0] = R[k][1] = R[k][2] = R[k][3] = 0u;
        return;
    }
  }
  // Modes differ across the warp: every micro-block of P0..P8 with an fp16-exact
  // scale goes through the branch-free table decoder (all lanes run the same
  // instructions, and the four decodes interleave); the rest (P16, flagged
  // slow, inexact scale) decode as zeros there and are redone per lane below.
  uint32_t po = 0, so = 0;
  bool generic = false;
  uint32_t ent[4];
  float scl[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int L = single ? l0 : l0 + k;
    ent[k] = lt_entry(ltab, L, sw);
    scl[k] = lt_scale_of(ltab, L, sw);
    const int m = lt_mode(ent[k]);
    const float sv = scl[k] * pow2e;
    const __half hs = __float2half_rn(sv);
    const bool exact = __half2float(hs) == sv;
    int cls = dec_class_of(m);
    if (m != 0 && (lt_slow(ent[k]) || !exact)) cls = 7;
    if (cls == 7) generic = true;
    decode_half_class(dtab, cls == 7 ? 0 : cls, prim + po, sec + so, c.h,
                      h2const(*reinterpret_cast<const uint16_t*>(&hs)), R[k]);
    po += lt_prim(ent[k]);
    so += lt_sec(ent[k]);
  }
  if (__any_sync(0xffffffffu, generic)) {
    po = 0;
    so = 0;
#pragma unroll 1
    for (int k = 0; k < 4; ++k) {
      const uint32_t e = k == 0 ? ent[0] : k == 1 ? ent[1] : k == 2 ? ent[2] : ent[3];
      const float sk = k == 0 ? scl[0] : k == 1 ? scl[1] : k == 2 ? scl[2] : scl[3];
      const int m = lt_mode(e);
      const float sv = sk * pow2e;
      const bool exact = __half2float(__float2half_rn(sv)) == sv;
      if (m == 16 || (m != 0 && (lt_slow(e) || !exact))) {
        uint32_t r[4];
        decode_half_w16(e, sk, prim + po, sec + so, c.h, pow2e, r);
        if (k == 0) { R[0][0] = r[0]; R[0][1] = r[1]; R[0][2] = r[2]; R[0][3] = r[3]; }
        if (k == 1) { R[1][0] = r[0]; R[1][1] = r[1]; R[1][2] = r[2]; R[1][3] = r[3]; }
        if (k == 2) { R[2][0] = r[0]; R[2][1] = r[1]; R[2][2] = r[2]; R[2][3] = r[3]; }
        if (k == 3) { R[3][0] = r[0]; R[3][1] = r[1]; R[3][2] = r[2]; R[3][3] = r[3]; }
      }
      po += lt_prim(e);
      so += lt_sec(e);
    }
  }
}

// ---------------------------------------------------------------------------
// mbarrier / bulk-copy / mma wrappers
// ---------------------------------------------------------------------------

// ---------------------------------------------------------------------------
// Output epilogue (mtc_epilogue of the C ABI): y = act(x + bias[j]).
// ---------------------------------------------------------------------------
struct Epi {
  const float* bias;  // nullable
  int act;            // MTC_ACT_*
};

__device__ __forceinline__ float epi_act(float x, int act) {
  switch (act) {
    case MTC_ACT_RELU:
      return x < 0.0f ? 0.0f : x;  // NaN passes through, as in torch.relu
    case MTC_ACT_SILU:
      return x / (1.0f + expf(-x));
    case MTC_ACT_GELU_TANH: {
      // GELU, tanh form (Hendrycks & Gimpel): sqrt(2/pi) and 0.044715
      const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
      return 0.5f * x * (1.0f + tanhf(u));
    }
    default:
      return x;
  }
}

__device__ __forceinline__ float epi_apply(const Epi& e, float x, long long j) {
  if (e.bias) x += __ldg(e.bias + j);
  return e.act ? epi_act(x, e.act) : x;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Programmatic dependent launch (kernels launched with
// cudaLaunchAttributeProgrammaticStreamSerialization): the next kernel in the
// stream may start once every CTA of this one has called launch_dependents;
// griddep_wait blocks until the previous kernel has completed and its memory
// is visible.  Both are no-ops for kernels launched without the attribute.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// try_wait with a suspend-time hint: a waiting thread sleeps until the phase
// completes (or ~20 us pass) instead of re-issuing the test, so idle roles do
// not take issue slots from the working warps.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: returns false (and the caller aborts) after `limit_ns`.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}
// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace mtc
