// Dequantisation of one staged sub-stage into a tensor-core operand tile,
// shared by the prefill (tcgen05, CTA pairs) and decode (tcgen05, swap-AB)
// kernels.  The format of the staged data is the one mtc_repack_stage_plan /
// mtc_repack_stage_fill build (include/mtc_b200.h).
#pragma once

#include "mtc_common.cuh"

namespace mtc {

// Shared by the prefill and decode kernels: the dequantisation of one staged
// sub-stage (four tiles of a column band in two k-tile rows) into the W tile
// the tensor cores read: 128 features x 64 k fp16, K-major, 128-byte swizzle.
//
// The sub-stage's work list holds group entries (one 8x8 leaf group, 4
// micro-blocks) and micro-block entries (split groups), each run sorted by
// decode class.  Warp dw (of kSubWarps) takes an equal contiguous slice of
// each run, so every warp does the same work: one pass over at most 16
// group entries, then one micro-block entry per lane pair per pass; lane
// pair (2e, 2e + 1) decodes the two column halves of its entry.  Sorted runs
// make most warps mode-uniform, so they take one specialised path; the
// others use the branch-free table decoder.
//   sl      staged sub-stage: [128 B descriptors][list (lbytes)][records]
//   cnt     group entries | micro-block entries << 16
//   part0   bytes of the row-0 records (the row-1 records follow)
//   tid_d   thread index among the kSubWarps warps; zero_row1: the stage's
//           second k-tile row lies beyond the matrix (zero it)
constexpr int kSubWarps = 8;
constexpr uint32_t kSubDescBytes = 128;
constexpr int kClassGeneric = 7;

// byte offset of element (row n, k) in a K-major SWIZZLE_128B tile of 64 fp16 per row
__device__ __forceinline__ uint32_t sw128_off(int n, int k) {
  return (uint32_t)n * 128u + ((((uint32_t)k >> 3) ^ ((uint32_t)n & 7u)) << 4) + (((uint32_t)k & 7u) << 1);
}

__device__ __forceinline__ void dequant_substage(uint8_t* Bt, const uint8_t* sl, uint32_t cnt, uint32_t lbytes,
                                                 uint32_t part0, bool zero_row1, const uint32_t* dtab,
                                                 int scale_words, float pow2e, int dw, int lane, int tid_d) {
  const int h = lane & 1;
  const uint64_t* list = reinterpret_cast<const uint64_t*>(sl + kSubDescBytes);
  const uint8_t* payload = sl + kSubDescBytes + lbytes;
  const mtc_tile_desc* descs = reinterpret_cast<const mtc_tile_desc*>(sl);
  // record of tile ti (row * 4 + column) inside the payload
  auto tile_record = [&](int ti) -> const uint8_t* {
    const mtc_tile_desc& d = descs[ti];
    return (ti >> 2) == 0 ? payload + (d.record_off - descs[0].record_off)
                          : payload + part0 + (d.record_off - descs[4].record_off);
  };
  const int n_group = (int)(cnt & 0xffffu), n_mb = (int)(cnt >> 16);
  const int pair = lane >> 1;
  // ---- group entries: each warp takes an equal contiguous slice (at most
  // 16) of the class-sorted run, one entry per lane pair ----
  {
    const int g0 = (dw * n_group) / kSubWarps, g1 = ((dw + 1) * n_group) / kSubWarps;
    const int u = g0 + pair;
    const bool valid = u < g1;
    const uint64_t ent = valid ? list[u] : 0ull;
    const int cls = valid ? (int)((ent >> 48) & 15u) : -1;
    const int cls0 = __shfl_sync(0xffffffffu, cls, 0);
    const uint8_t* prim = payload + (uint32_t)(ent & 0xffffu);
    const uint8_t* sec = payload + (uint32_t)((ent >> 16) & 0xffffu);
    const uint32_t s2 = h2const((uint16_t)((ent >> 32) & 0xffffu));
    const int ti = (int)((ent >> 52) & 15u), G = (int)((ent >> 56) & 15u);
    uint32_t R[4][4];
    const bool uniform = __all_sync(0xffffffffu, !valid || cls == cls0);
    if (uniform && cls0 != kClassGeneric) {
      switch (cls0) {  // warp-uniform branch
        case 1: decode_run4<2>(prim, sec, h, s2, R); break;
        case 2: decode_run4<3>(prim, sec, h, s2, R); break;
        case 3: decode_run4<4>(prim, sec, h, s2, R); break;
        case 4: decode_run4<5>(prim, sec, h, s2, R); break;
        case 5: decode_run4<6>(prim, sec, h, s2, R); break;
        case 6: decode_run4<8>(prim, sec, h, s2, R); break;
        default:
#pragma unroll
          for (int k = 0; k < 4; ++k) R[k][0] = R[k][1] = R[k][2] = R[k][3] = 0u;
      }
    } else {
      // class boundary inside the warp: table decoder for P0..P8 (one
      // instruction sequence), per-lane generic path for the rest
      if (valid && cls != kClassGeneric) decode_run4_class(dtab, cls, prim, sec, h, s2, R);
      if (valid && cls == kClassGeneric)
        decode_group_generic(reinterpret_cast<const uint32_t*>(tile_record(ti)), descs[ti].leaf_start, G, prim,
                             sec, scale_words, h, pow2e, R);
    }
    if (valid) {
      // R[2 di + dj] = micro-block (2t + di, 2jj + dj) of group G: pairs 0,1
      // feature 2h (k rows 0..3), pairs 2,3 feature 2h + 1; di selects k 0..3 / 4..7
      const int r = ti >> 2, col = ti & 3;
      const int t = ((G >> 3) & 1) << 1 | ((G >> 1) & 1);
      const int jj = ((G >> 2) & 1) << 1 | (G & 1);
#pragma unroll
      for (int dj = 0; dj < 2; ++dj) {
        const int f = 32 * col + 4 * (2 * jj + dj) + 2 * h;
        *reinterpret_cast<uint4*>(Bt + sw128_off(f, 32 * r + 8 * t)) =
            make_uint4(R[dj][0], R[dj][1], R[2 + dj][0], R[2 + dj][1]);
        *reinterpret_cast<uint4*>(Bt + sw128_off(f + 1, 32 * r + 8 * t)) =
            make_uint4(R[dj][2], R[dj][3], R[2 + dj][2], R[2 + dj][3]);
      }
    }
  }
  // ---- micro-block entries (split groups): each warp takes an equal
  // contiguous slice, one entry per lane pair per pass.  P0..P8 go through
  // the branch-free table decoder; generic entries (P16, inexact fp16
  // scales) through a per-lane path when present ----
  {
    const int m0 = (dw * n_mb) / kSubWarps, m1 = ((dw + 1) * n_mb) / kSubWarps;
#pragma unroll 1
    for (int base = m0; base < m1; base += 16) {  // warp-uniform
      const int j = base + pair;
      const bool ok = j < m1;
      const uint64_t e = ok ? list[n_group + j] : 0ull;
      const int cls = (int)((e >> 48) & 15u);
      const bool dec = ok && cls != kClassGeneric;
      const uint64_t ed = dec ? e : 0ull;
      uint32_t r[4];
      decode_half_class(dtab, dec ? cls : 0, payload + (uint32_t)(ed & 0xffffu),
                        payload + (uint32_t)((ed >> 16) & 0xffffu), h, h2const((uint16_t)((ed >> 32) & 0xffffu)), r);
      const bool gen = ok && cls == kClassGeneric;
      if (__any_sync(0xffffffffu, gen) && gen) {
        const int ti = (int)((e >> 52) & 15u), G = (int)((e >> 56) & 15u), mk = (int)((e >> 60) & 3u);
        const uint32_t* ltab = reinterpret_cast<const uint32_t*>(tile_record(ti));
        const int L = leaf_of(descs[ti].leaf_start, 4 * G + mk);
        decode_half_w16(lt_entry(ltab, L, scale_words), lt_scale_of(ltab, L, scale_words),
                        payload + (uint32_t)(e & 0xffffu), payload + (uint32_t)((e >> 16) & 0xffffu), h, pow2e, r);
      }
      if (ok) {
        // micro-block (2t + di, 2jj + dj) of group G, di = mk >> 1, dj = mk & 1
        const int ti = (int)((e >> 52) & 15u), G = (int)((e >> 56) & 15u), mk = (int)((e >> 60) & 3u);
        const int rr = ti >> 2, col = ti & 3;
        const int t = ((G >> 3) & 1) << 1 | ((G >> 1) & 1);
        const int jj = ((G >> 2) & 1) << 1 | (G & 1);
        const int f = 32 * col + 4 * (2 * jj + (mk & 1)) + 2 * h;
        const int k0 = 32 * rr + 8 * t + 4 * (mk >> 1);
        *reinterpret_cast<uint2*>(Bt + sw128_off(f, k0)) = make_uint2(r[0], r[1]);
        *reinterpret_cast<uint2*>(Bt + sw128_off(f + 1, k0)) = make_uint2(r[2], r[3]);
      }
    }
  }
  if (zero_row1) {
    // odd number of k-tile rows: the stage's second row is zero padding
    for (int c = tid_d; c < 128 * 4; c += kSubWarps * 32) {
      const int f = c >> 2, ch = 4 + (c & 3);
      *reinterpret_cast<uint4*>(Bt + f * 128 + ((ch ^ (f & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

}  // namespace mtc
