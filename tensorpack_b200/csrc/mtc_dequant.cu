// Exact dequantisation of a device tile stream: out = q * scale in fp32.
// Reproduces MTCMatrix.to_array (mtc/kernels/gemm.py:510-538) and
// qt_dequant / permuted_qt_dequant (mtc/core/quadtree.py:157-171,
// mtc/core/permutation.py:76-79) bit for bit: the reference computes the
// fp32 product of the integer code and the fp32 (bf16-exact) scale, and so
// does __fmul_rn here.  Zero codes give +0.0 like the reference's `deq +=`.
#include "mtc_common.cuh"
#include "mtc_internal.h"

namespace mtc {
namespace {

// One warp per tile.  Lane (g, t) = (lane >> 2, lane & 3) owns the aligned
// 2x2 micro-block group (t, jj = g >> 1) and its column half h = g & 1.
__global__ void __launch_bounds__(256) dequant_tiles(mtc_stream_desc s, const int32_t* __restrict__ row_perm,
                                                     const int32_t* __restrict__ col_perm, float* __restrict__ out,
                                                     long long ldo) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x * 8 + warp;
  if (tile >= s.tk * s.tn) return;
  const int kt = tile / s.tn, nt = tile % s.tn;
  const mtc_tile_desc d = s.tiles[tile];
  const uint8_t* rec = s.records + d.record_off;
  const uint32_t* ltab = reinterpret_cast<const uint32_t*>(rec);
  const int sw = s.scale_words;
  const uint8_t* prim_base = rec + pad16(4 * sw * d.n_leaves);

  // Z-order prefix sums of the per-mb plane sizes (z = lane, lane + 32).
  uint32_t pk[2];
  for (int k = 0; k < 2; ++k) {
    const uint32_t e = lt_entry(ltab, leaf_of(d.leaf_start, lane + 32 * k), sw);
    pk[k] = (uint32_t)lt_prim(e) | ((uint32_t)lt_sec(e) << 16);
  }
  uint32_t inc0 = pk[0], inc1 = pk[1];
#pragma unroll
  for (int dd = 1; dd < 32; dd <<= 1) {
    const uint32_t u0 = __shfl_up_sync(0xffffffffu, inc0, dd);
    const uint32_t u1 = __shfl_up_sync(0xffffffffu, inc1, dd);
    if (lane >= dd) { inc0 += u0; inc1 += u1; }
  }
  const uint32_t tot0 = __shfl_sync(0xffffffffu, inc0, 31);
  inc1 += tot0;
  const uint8_t* sec_base = prim_base + pad16(d.prim_bytes);

  const int g = lane >> 2, t = lane & 3;
  const int jj = g >> 1, h = g & 1;
  for (int q4 = 0; q4 < 4; ++q4) {
    const int di = q4 >> 1, dj = q4 & 1;
    const int mi = 2 * t + di, mj = 2 * jj + dj;
    const int z = z_of(mi, mj);
    // fetch the inclusive offsets of micro-block z from its owner lane
    const uint32_t incz0 = __shfl_sync(0xffffffffu, inc0, z & 31);
    const uint32_t incz1 = __shfl_sync(0xffffffffu, inc1, z & 31);
    const uint32_t incl = (z < 32) ? incz0 : incz1;
    const int L = leaf_of(d.leaf_start, z);
    const uint32_t e = lt_entry(ltab, L, sw);
    const uint32_t mine = (uint32_t)lt_prim(e) | ((uint32_t)lt_sec(e) << 16);
    const uint32_t ex = incl - mine;
    const uint8_t* prim = prim_base + (ex & 0xffffu);
    const uint8_t* sec = sec_base + (ex >> 16);
    int code[8];
    decode_half_int(lt_mode(e), prim, sec, h, code);
    const float sc = lt_scale_of(ltab, L, sw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int k = kt * kTile + 4 * mi + 2 * (j & 1) + hi;
        const int n = nt * kTile + 4 * mj + 2 * h + (j >> 1);
        if (k < s.K && n < s.N) {
          const float v = __fadd_rn(__fmul_rn((float)code[2 * j + hi], sc), 0.0f);
          const long long ko = row_perm ? row_perm[k] : k;
          const long long no = col_perm ? col_perm[n] : n;
          out[ko * ldo + no] = v;
        }
      }
    }
  }
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" int mtc_dequant(const mtc_stream_desc* s, const int32_t* row_perm, const int32_t* col_perm, float* out,
                           int64_t ldo, void* stream) {
  clear_error();
  MTC_REQUIRE(s && out && s->records && s->tiles, "mtc_dequant: null pointer argument");
  MTC_REQUIRE(s->K > 0 && s->N > 0 && ldo >= s->N, "mtc_dequant: bad shape K=%d N=%d ldo=%lld", s->K, s->N,
              (long long)ldo);
  const int T = s->tk * s->tn;
  dequant_tiles<<<(T + 7) / 8, 256, 0, as_stream(stream)>>>(*s, row_perm, col_perm, out, (long long)ldo);
  MTC_CHECK_LAUNCH("mtc_dequant");
  return MTC_OK;
}
