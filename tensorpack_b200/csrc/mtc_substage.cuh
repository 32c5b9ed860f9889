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
// the group run: one pass over at most 16 group entries, lane pair
// (2e, 2e + 1) decoding the two column halves of its entry.  Sorted runs
// make most warps mode-uniform, so they take one specialised path; the
// others use the branch-free table decoder.  Micro-block entries go one per
// lane, 32 to a pass, to rotating warps.
//   sl      staged sub-stage: [128 B descriptors][list (lbytes)][records]
//   cnt     group entries | micro-block entries << 16
//   part0   bytes of the row-0 records (the row-1 records follow)
//   tid_d   thread index among the kSubWarps warps; zero_row1: the stage's
//           second k-tile row lies beyond the matrix (zero it)
//   rot     rotation of the micro-block chunks over the warps (any value
//           that advances from one sub-stage to the next, the same for all
//           warps of the group)
constexpr int kSubWarps = 8;
constexpr uint32_t kSubDescBytes = 128;
constexpr int kClassGeneric = 7;

// byte offset of element (row n, k) in a K-major SWIZZLE_128B tile of 64 fp16 per row
__device__ __forceinline__ uint32_t sw128_off(int n, int k) {
  return (uint32_t)n * 128u + ((((uint32_t)k >> 3) ^ ((uint32_t)n & 7u)) << 4) + (((uint32_t)k & 7u) << 1);
}

__device__ __forceinline__ void dequant_substage(uint8_t* Bt, const uint8_t* sl, uint32_t cnt, uint32_t lbytes,
                                                 uint32_t part0, bool zero_row1, const uint32_t* dtab,
                                                 int scale_words, float pow2e, int dw, int lane, int tid_d,
                                                 int rot) {
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
  // ---- micro-block entries (split groups): one entry (both column halves)
  // per lane, in chunks of 32.  Chunk c goes to warp (c + rot) mod 8: most
  // sub-stages have one or two chunks, so only those warps make a pass, and
  // the rotation spreads the passes evenly over the warps across
  // consecutive sub-stages.  P0..P8 go through the branch-free table
  // decoder; generic entries (P16, inexact fp16 scales) through a per-lane
  // path when present ----
  {
    const int n_chunks = (n_mb + 31) >> 5;
#pragma unroll 1
    for (int c = (dw - rot) & (kSubWarps - 1); c < n_chunks; c += kSubWarps) {  // warp-uniform
      const int j = 32 * c + lane;
      const bool ok = j < n_mb;
      const uint64_t e = ok ? list[n_group + j] : 0ull;
      const int cls = (int)((e >> 48) & 15u);
      const bool dec = ok && cls != kClassGeneric;
      const uint64_t ed = dec ? e : 0ull;
      const uint8_t* prim = payload + (uint32_t)(ed & 0xffffu);
      const uint8_t* sec = payload + (uint32_t)((ed >> 16) & 0xffffu);
      const uint32_t s2 = h2const((uint16_t)((ed >> 32) & 0xffffu));
      uint32_t r0[4], r1[4];
      decode_half_class(dtab, dec ? cls : 0, prim, sec, 0, s2, r0);
      decode_half_class(dtab, dec ? cls : 0, prim, sec, 1, s2, r1);
      const bool gen = ok && cls == kClassGeneric;
      const int ti = (int)((e >> 52) & 15u), G = (int)((e >> 56) & 15u), mk = (int)((e >> 60) & 3u);
      if (__any_sync(0xffffffffu, gen) && gen) {
        const uint32_t* ltab = reinterpret_cast<const uint32_t*>(tile_record(ti));
        const int L = leaf_of(descs[ti].leaf_start, 4 * G + mk);
        const uint32_t le = lt_entry(ltab, L, scale_words);
        const float ls = lt_scale_of(ltab, L, scale_words);
        const uint8_t* gp = payload + (uint32_t)(e & 0xffffu);
        const uint8_t* gs = payload + (uint32_t)((e >> 16) & 0xffffu);
        decode_half_w16(le, ls, gp, gs, 0, pow2e, r0);
        decode_half_w16(le, ls, gp, gs, 1, pow2e, r1);
      }
      if (ok) {
        // micro-block (2t + di, 2jj + dj) of group G, di = mk >> 1, dj = mk & 1;
        // half 0 holds features f, f + 1, half 1 features f + 2, f + 3
        const int rr = ti >> 2, col = ti & 3;
        const int t = ((G >> 3) & 1) << 1 | ((G >> 1) & 1);
        const int jj = ((G >> 2) & 1) << 1 | (G & 1);
        const int f = 32 * col + 4 * (2 * jj + (mk & 1));
        const int k0 = 32 * rr + 8 * t + 4 * (mk >> 1);
        *reinterpret_cast<uint2*>(Bt + sw128_off(f, k0)) = make_uint2(r0[0], r0[1]);
        *reinterpret_cast<uint2*>(Bt + sw128_off(f + 1, k0)) = make_uint2(r0[2], r0[3]);
        *reinterpret_cast<uint2*>(Bt + sw128_off(f + 2, k0)) = make_uint2(r1[0], r1[1]);
        *reinterpret_cast<uint2*>(Bt + sw128_off(f + 3, k0)) = make_uint2(r1[2], r1[3]);
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
