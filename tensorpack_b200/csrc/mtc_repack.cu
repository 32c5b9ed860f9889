// GPU repack: reference-layout MTCMatrix (per-leaf payloads in an arena,
// mtc/kernels/gemm.py:432-488 extended to quadtree leaves) -> tile-major
// device stream (format described in mtc_common.cuh).
//
//   plan:  one thread per 32x32 tile measures its record (leaf table +
//          primary + secondary planes), validates the leaf tiling, then a
//          single-CTA scan lays the records out band-major and fills the
//          16-byte tile descriptors and the per-band k-row offsets.
//   fill:  one warp per tile writes the leaf table and transcodes every
//          4x4 micro-block from the LSB-first m-bit codes of its leaf into
//          the bit-plane-split, fragment-ordered planes.
#include "mtc_common.cuh"
#include "mtc_internal.h"

namespace mtc {
namespace {

constexpr uint32_t kErrCoverage = 1u;   // leaves do not tile the 64 micro-blocks in Z order
constexpr uint32_t kErrLeafCount = 2u;  // 0 or > 64 leaves in a tile
constexpr uint32_t kErrLeaf = 4u;       // bad mode / size / z0

__device__ __forceinline__ int stream_index(int kt, int nt, int tk, int tn, int bt) {
  const int b = nt / bt;
  const int w = min(bt, tn - b * bt);
  return b * bt * tk + kt * w + (nt - b * bt);
}

__device__ __forceinline__ bool valid_mode(int m) {
  return m == 0 || m == 2 || m == 3 || m == 4 || m == 5 || m == 6 || m == 8 || m == 16;
}

__global__ void plan_tiles(const mtc_leaf_in* __restrict__ leaves, const uint32_t* __restrict__ begin,
                           int tk, int tn, int bt, int sw, mtc_tile_desc* __restrict__ tiles,
                           uint32_t* __restrict__ rec_bytes, uint32_t* __restrict__ err) {
  const int T = tk * tn;
  const int tile = blockIdx.x * blockDim.x + threadIdx.x;
  if (tile >= T) return;
  const uint32_t b0 = begin[tile], b1 = begin[tile + 1];
  const int n = (int)(b1 - b0);
  uint32_t bad = 0;
  if (n <= 0 || n > kMbPerTile) bad |= kErrLeafCount;
  uint64_t mask = 0;
  int prim = 0, sec = 0, zrun = 0;
  if (!bad) {
    for (uint32_t l = b0; l < b1; ++l) {
      const mtc_leaf_in L = leaves[l];
      const int s = L.size;
      if (!valid_mode(L.mode) || (s != 4 && s != 8 && s != 16 && s != 32) || L.z0 >= 64) {
        bad |= kErrLeaf;
        break;
      }
      const int nmb = (s / 4) * (s / 4);
      if (L.z0 != zrun || (L.z0 % nmb) != 0) {
        bad |= kErrCoverage;
        break;
      }
      mask |= 1ull << L.z0;
      prim += mb_prim_bytes(L.mode) * nmb;
      sec += mb_sec_bytes(L.mode) * nmb;
      zrun += nmb;
    }
    if (!bad && zrun != kMbPerTile) bad |= kErrCoverage;
  }
  if (bad) {
    atomicOr(err, bad);
    return;
  }
  mtc_tile_desc d;
  d.record_off = 0;
  d.n_leaves = (uint16_t)n;
  d.prim_bytes = (uint16_t)prim;
  d.leaf_start = mask;
  tiles[tile] = d;
  const int kt = tile / tn, nt = tile % tn;
  rec_bytes[stream_index(kt, nt, tk, tn, bt)] = pad16(4 * sw * n) + pad16(prim) + pad16(sec);
}

// Single CTA: exclusive scan of record sizes in stream order.
__global__ void __launch_bounds__(1024) plan_scan(const uint32_t* __restrict__ rec_bytes, int tk, int tn,
                                                  int bt, mtc_tile_desc* __restrict__ tiles,
                                                  uint32_t* __restrict__ row_off,
                                                  unsigned long long* __restrict__ total,
                                                  uint32_t* __restrict__ max_row) {
  __shared__ unsigned long long part[1024];
  const int T = tk * tn;
  const int per = (T + blockDim.x - 1) / blockDim.x;
  const int lo = min(T, (int)threadIdx.x * per), hi = min(T, lo + per);
  unsigned long long s = 0;
  for (int i = lo; i < hi; ++i) s += rec_bytes[i];
  part[threadIdx.x] = s;
  __syncthreads();
  for (int d = 1; d < (int)blockDim.x; d <<= 1) {
    unsigned long long v = threadIdx.x >= (unsigned)d ? part[threadIdx.x - d] : 0ull;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  unsigned long long off = part[threadIdx.x] - s;
  const int nb = (tn + bt - 1) / bt;
  for (int si = lo; si < hi; ++si) {
    const int b = si / (bt * tk);
    const int w = min(bt, tn - b * bt);
    const int rem = si - b * bt * tk;
    const int kt = rem / w, i = rem % w;
    const int nt = b * bt + i;
    tiles[kt * tn + nt].record_off = (uint32_t)off;
    if (i == 0) row_off[b * (tk + 1) + kt] = (uint32_t)off;
    off += rec_bytes[si];
    if (si == b * bt * tk + tk * w - 1) row_off[b * (tk + 1) + tk] = (uint32_t)off;
  }
  __syncthreads();
  if (threadIdx.x == blockDim.x - 1) *total = part[blockDim.x - 1];
  // largest k-row of any band (bulk-copy stage size)
  uint32_t mx = 0;
  for (int r = threadIdx.x; r < nb * tk; r += blockDim.x) {
    const int b = r / tk, kt = r % tk;
    mx = max(mx, row_off[b * (tk + 1) + kt + 1] - row_off[b * (tk + 1) + kt]);
  }
  __shared__ uint32_t red[1024];
  red[threadIdx.x] = mx;
  __syncthreads();
  for (int d = blockDim.x / 2; d > 0; d >>= 1) {
    if (threadIdx.x < (unsigned)d) red[threadIdx.x] = max(red[threadIdx.x], red[threadIdx.x + d]);
    __syncthreads();
  }
  if (threadIdx.x == 0) *max_row = red[0];
}

__device__ __forceinline__ int read_code(const uint8_t* __restrict__ src, int e, int m) {
  const long bit = (long)e * m;
  const uint8_t* p = src + (bit >> 3);
  const int sh = (int)(bit & 7);
  uint32_t w = p[0];
  if (sh + m > 8) w |= (uint32_t)p[1] << 8;
  if (sh + m > 16) w |= (uint32_t)p[2] << 16;
  const uint32_t u = (w >> sh) & ((1u << m) - 1u);
  return (u >= (1u << (m - 1))) ? (int)u - (1 << m) : (int)u;
}

__device__ __forceinline__ bool scale_fp16_exact(float s) {
  const __half h = __float2half_rn(s);
  return __half2float(h) == s;
}

// Warp-inclusive scan of a u32 (sum).
__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += u;
  }
  return v;
}

__global__ void __launch_bounds__(256) fill_tiles(const uint8_t* __restrict__ arena, unsigned long long arena_bytes,
                                                  const mtc_leaf_in* __restrict__ leaves,
                                                  const uint32_t* __restrict__ begin, int tk, int tn,
                                                  const mtc_tile_desc* __restrict__ tiles, int exp2, int sw,
                                                  uint8_t* __restrict__ records, uint32_t* __restrict__ err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x * 8 + warp;
  if (tile >= tk * tn) return;
  const mtc_tile_desc d = tiles[tile];
  const uint32_t b0 = begin[tile];
  const int n = d.n_leaves;
  uint8_t* rec = records + d.record_off;
  const float pow2e = ldexpf(1.0f, exp2);

  // Leaf table (+ zero padding to 16 bytes).
  for (int w = lane; w < pad16(4 * sw * n) / 4; w += 32) {
    uint32_t e = 0;
    const int l = w / sw;
    if (l < n) {
      const mtc_leaf_in L = leaves[b0 + l];
      const int m = L.mode;
      const float s = __uint_as_float(L.scale_bits);
      if (w % sw == 1) {
        e = L.scale_bits;
      } else {
        const bool slow = (m != 0) && !scale_fp16_exact(s * pow2e);
        e = (uint32_t)m | ((uint32_t)(mb_prim_bytes(m) / 4) << 8) | ((uint32_t)(mb_sec_bytes(m) / 2) << 12) |
            ((slow ? 1u : 0u) << 14) | (L.scale_bits & 0xffff0000u);
      }
    }
    reinterpret_cast<uint32_t*>(rec)[w] = e;
  }

  // Per micro-block sizes and Z-order prefix sums (z = lane, lane + 32).
  int mode[2], lidx[2];
  uint32_t packed[2];
  for (int k = 0; k < 2; ++k) {
    const int z = lane + 32 * k;
    lidx[k] = leaf_of(d.leaf_start, z);
    mode[k] = leaves[b0 + lidx[k]].mode;
    packed[k] = (uint32_t)mb_prim_bytes(mode[k]) | ((uint32_t)mb_sec_bytes(mode[k]) << 16);
  }
  const uint32_t inc0 = warp_incl_scan(packed[0]);
  const uint32_t tot0 = __shfl_sync(0xffffffffu, inc0, 31);
  const uint32_t inc1 = warp_incl_scan(packed[1]) + tot0;
  const uint32_t excl[2] = {inc0 - packed[0], inc1 - packed[1]};

  uint8_t* prim_base = rec + pad16(4 * sw * n);
  uint8_t* sec_base = prim_base + pad16(d.prim_bytes);
  const uint32_t tot_all = __shfl_sync(0xffffffffu, inc1, 31);
  const int sec_bytes = (int)(tot_all >> 16);
  // zero the padding tails
  for (int i = d.prim_bytes + lane; i < pad16(d.prim_bytes); i += 32) prim_base[i] = 0;
  for (int i = sec_bytes + lane; i < pad16(sec_bytes); i += 32) sec_base[i] = 0;

  for (int k = 0; k < 2; ++k) {
    const int z = lane + 32 * k;
    const int m = mode[k];
    if (m == 0) continue;
    const mtc_leaf_in L = leaves[b0 + lidx[k]];
    const int s = L.size;
    const int li = z_row(L.z0), lj = z_col(L.z0);
    const int mi = z_row(z), mj = z_col(z);
    const unsigned long long leaf_bytes = (unsigned long long)m * s * s / 8;
    if ((unsigned long long)L.arena_off + leaf_bytes > arena_bytes) {
      atomicOr(err, kErrLeaf);
      continue;
    }
    const uint8_t* src = arena + L.arena_off;
    int q[4][4];  // [row r][col c] of this micro-block
    for (int r = 0; r < 4; ++r)
      for (int c = 0; c < 4; ++c) q[r][c] = read_code(src, (4 * (mi - li) + r) * s + 4 * (mj - lj) + c, m);
    uint8_t* pp = prim_base + (excl[k] & 0xffffu);
    uint8_t* sp = sec_base + (excl[k] >> 16);
    if (m == 16) {
      uint32_t* w = reinterpret_cast<uint32_t*>(pp);
      for (int h = 0; h < 2; ++h)
        for (int j = 0; j < 4; ++j) {
          const int c = 2 * h + (j >> 1), r = 2 * (j & 1);
          w[4 * h + j] = ((uint32_t)q[r][c] & 0xffffu) | (((uint32_t)q[r + 1][c] & 0xffffu) << 16);
        }
      continue;
    }
    const int wp = prim_width(m);
    const int bias = 1 << (m - 1);
    uint32_t pw[4] = {0, 0, 0, 0};
    uint32_t sv = 0;
    for (int h = 0; h < 2; ++h)
      for (int j = 0; j < 4; ++j)
        for (int hi = 0; hi < 2; ++hi) {
          const int c = 2 * h + (j >> 1), r = 2 * (j & 1) + hi;
          const uint32_t u = (uint32_t)(q[r][c] + bias);
          const uint32_t lo = u & ((1u << wp) - 1u), up = u >> wp;
          if (wp == 2) pw[0] |= lo << (8 * h + 2 * j + 16 * hi);
          if (wp == 4) pw[h] |= lo << (4 * (j & 1) + 8 * (j >> 1) + 16 * hi);
          if (wp == 8) pw[2 * h + (j >> 1)] |= lo << (8 * ((j & 1) + 2 * hi));
          if (m == 3 || m == 5) sv |= up << (4 * h + j + 8 * hi);
          if (m == 6) sv |= up << (8 * h + 2 * j + 16 * hi);
        }
    uint32_t* w = reinterpret_cast<uint32_t*>(pp);
    for (int i = 0; i < mb_prim_bytes(m) / 4; ++i) w[i] = pw[i];
    uint16_t* sw = reinterpret_cast<uint16_t*>(sp);
    if (m == 3 || m == 5) sw[0] = (uint16_t)sv;
    if (m == 6) {
      sw[0] = (uint16_t)(sv & 0xffffu);
      sw[1] = (uint16_t)(sv >> 16);
    }
  }
}

// Classes of the prefill work lists: decode path of an 8x8 group.
constexpr int kClassZero = 0;     // P0 leaf: writes zeros
constexpr int kClassGeneric = 7;  // four 4x4 leaves, P16 or inexact fp16 scale

__device__ __forceinline__ int class_of_mode(int m) {
  switch (m) {
    case 0: return kClassZero;
    case 2: return 1;
    case 3: return 2;
    case 4: return 3;
    case 5: return 4;
    case 6: return 5;
    case 8: return 6;
    default: return kClassGeneric;
  }
}

__device__ __forceinline__ uint32_t fp16_scale_bits(float sc, bool* exact) {
  const __half hs = __float2half_rn(sc);
  *exact = __half2float(hs) == sc;
  return *reinterpret_cast<const uint16_t*>(&hs);
}

// Record range of the four tiles 4 * half .. 4 * half + 3 of band `band` in
// k-tile row kt: {byte offset, bytes} (empty beyond the matrix).
__device__ __forceinline__ uint2 half_row_range(const mtc_stream_desc& s, int band, int half, int kt) {
  const int width = min(s.band_tiles, s.tn - band * s.band_tiles);
  const int c0 = 4 * half;
  if (kt >= s.tk || c0 >= width) return make_uint2(0u, 0u);
  const uint32_t start = s.tiles[(size_t)kt * s.tn + band * s.band_tiles + c0].record_off;
  const uint32_t end = (c0 + 4 < width) ? s.tiles[(size_t)kt * s.tn + band * s.band_tiles + c0 + 4].record_off
                                        : s.row_off[(size_t)band * (s.tk + 1) + kt + 1];
  return make_uint2(start, end - start);
}

// One CTA of 128 threads per sub-stage q = 2 * (band * nkb + kb) + half:
// thread i owns group G = i & 15 of tile (row i >> 6, column 4 * half +
// ((i >> 4) & 3)).  A group covered by one leaf becomes one group entry; a
// group of four 4x4 leaves becomes four micro-block entries (each with its own
// mode), so every entry decodes with one mode.  Group entries come first,
// sorted by class, then micro-block entries, sorted by class.  Pass 1
// (FILL = false) counts the entries and measures the two record parts; pass
// 2 writes the image: descriptors, entries, a copy of the records.
constexpr uint32_t kImgDescBytes = 128;

template <bool FILL>
__global__ void __launch_bounds__(128) stage_lists_kernel(mtc_stream_desc s, int nkb, const uint32_t* __restrict__ offs,
                                                          uint32_t* __restrict__ counts, uint32_t* __restrict__ totals,
                                                          uint32_t* __restrict__ ranges,
                                                          uint8_t* __restrict__ images) {
  __shared__ uint32_t cnt[16];   // [0, 8) group classes, [8, 16) micro-block classes
  __shared__ uint32_t base[16];
  const int q = blockIdx.x;  // half-band major: q = (2 band + half) nkb + kb
  const int hb = q / nkb, kb = q % nkb;
  const int band = hb >> 1, half = hb & 1;
  const int i = threadIdx.x;
  const int t8 = i >> 4, G = i & 15;
  const int r = t8 >> 2, colh = t8 & 3;
  const int kt = 2 * kb + r, nt = band * s.band_tiles + 4 * half + colh;
  const bool valid = kt < s.tk && nt < s.tn && 4 * half + colh < s.band_tiles;
  if (i < 16) cnt[i] = 0;
  __syncthreads();
  const uint2 p0 = half_row_range(s, band, half, 2 * kb);
  const uint2 p1 = half_row_range(s, band, half, 2 * kb + 1);
  const float pow2e = ldexpf(1.0f, s.exp2);
  const int sw = s.scale_words;
  uint32_t v = 0, e0 = 0;
  int l0 = 0;
  bool single = true;
  mtc_tile_desc d{};
  if (valid) {
    d = s.tiles[(size_t)kt * s.tn + nt];
    const uint32_t* ltab = reinterpret_cast<const uint32_t*>(s.records + d.record_off);
    l0 = leaf_of(d.leaf_start, 4 * G);
    single = ((d.leaf_start >> (4 * G + 1)) & 7ull) == 0ull;
    e0 = lt_entry(ltab, l0, sw);
    if (single) {
      v = 4u * ((uint32_t)lt_prim(e0) | ((uint32_t)lt_sec(e0) << 16));
    } else {
      for (int k = 0; k < 4; ++k) {
        const uint32_t e = lt_entry(ltab, l0 + k, sw);
        v += (uint32_t)lt_prim(e) | ((uint32_t)lt_sec(e) << 16);
      }
    }
  }
  // exclusive scan over the 16 groups of the tile (16 consecutive lanes)
  const int lane = i & 31;
  uint32_t incl = v;
#pragma unroll
  for (int dl = 1; dl < 16; dl <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, incl, dl);
    if ((lane & 15) >= dl) incl += u;
  }
  const uint32_t ex = incl - v;
  uint64_t entry[4] = {0, 0, 0, 0};
  int cls[4] = {-1, -1, -1, -1};  // slot < 8: group class; slot 8 + c: micro-block class c
  if (valid) {
    const uint32_t* ltab = reinterpret_cast<const uint32_t*>(s.records + d.record_off);
    // position of this tile's record in the sub-stage payload (row-0 part, then row-1 part)
    const uint32_t rec = r == 0 ? d.record_off - p0.x : d.record_off - p1.x + p0.y;
    uint32_t prim = rec + pad16(4 * sw * d.n_leaves) + (ex & 0xffffu);
    uint32_t sec = rec + pad16(4 * sw * d.n_leaves) + pad16(d.prim_bytes) + (ex >> 16);
    const uint64_t where = ((uint64_t)t8 << 52) | ((uint64_t)G << 56);
    if (single) {
      const int m = lt_mode(e0);
      bool exact;
      const uint32_t s16 = fp16_scale_bits(lt_scale_of(ltab, l0, sw) * pow2e, &exact);
      int c = class_of_mode(m);
      if (m != 0 && (lt_slow(e0) || !exact)) c = kClassGeneric;
      cls[0] = c;
      entry[0] = (uint64_t)(prim & 0xffffu) | ((uint64_t)(sec & 0xffffu) << 16) | ((uint64_t)s16 << 32) |
                 ((uint64_t)c << 48) | where;
    } else {
      for (int k = 0; k < 4; ++k) {
        const uint32_t e = lt_entry(ltab, l0 + k, sw);
        const int m = lt_mode(e);
        bool exact;
        const uint32_t s16 = fp16_scale_bits(lt_scale_of(ltab, l0 + k, sw) * pow2e, &exact);
        int c = class_of_mode(m);
        if (m != 0 && (lt_slow(e) || !exact)) c = kClassGeneric;
        cls[k] = 8 + c;
        entry[k] = (uint64_t)(prim & 0xffffu) | ((uint64_t)(sec & 0xffffu) << 16) | ((uint64_t)s16 << 32) |
                   ((uint64_t)c << 48) | where | ((uint64_t)k << 60) | (1ull << 62);
        prim += lt_prim(e);
        sec += lt_sec(e);
      }
    }
  }
  uint32_t rank[4] = {0, 0, 0, 0};
  for (int k = 0; k < 4; ++k)
    if (cls[k] >= 0) rank[k] = atomicAdd(&cnt[cls[k]], 1u);
  __syncthreads();
  if (i == 0) {
    uint32_t acc = 0;
    for (int c = 0; c < 16; ++c) {
      base[c] = acc;
      acc += cnt[c];
    }
    uint32_t ng = 0;
    for (int c = 0; c < 8; ++c) ng += cnt[c];
    if (!FILL) {
      counts[q] = ng | ((acc - ng) << 16);
      totals[q] = acc;
      ranges[4 * (size_t)q + 2] = p0.y;
      ranges[4 * (size_t)q + 3] = p1.y;
    }
  }
  __syncthreads();
  if (FILL) {
    uint8_t* img = images + offs[q];
    uint64_t* list = reinterpret_cast<uint64_t*>(img + kImgDescBytes);
    for (int k = 0; k < 4; ++k)
      if (cls[k] >= 0) list[base[cls[k]] + rank[k]] = entry[k];
    // descriptors of the 4 x 2 tiles (zero where the tile lies beyond the matrix)
    if (i < 8) {
      const int rr = i >> 2, cc = i & 3;
      const int kt2 = 2 * kb + rr, nt2 = band * s.band_tiles + 4 * half + cc;
      uint4 dsc = make_uint4(0u, 0u, 0u, 0u);
      if (kt2 < s.tk && nt2 < s.tn && 4 * half + cc < s.band_tiles)
        dsc = *reinterpret_cast<const uint4*>(s.tiles + (size_t)kt2 * s.tn + nt2);
      reinterpret_cast<uint4*>(img)[i] = dsc;
    }
    // the records of the two row parts, 16 bytes per thread-step
    const uint32_t lbytes = (8u * (base[15] + cnt[15]) + 15u) & ~15u;
    uint4* dst = reinterpret_cast<uint4*>(img + kImgDescBytes + lbytes);
    const uint4* src0 = reinterpret_cast<const uint4*>(s.records + p0.x);
    const uint4* src1 = reinterpret_cast<const uint4*>(s.records + p1.x);
    for (uint32_t c = i; c < p0.y / 16u; c += blockDim.x) dst[c] = src0[c];
    for (uint32_t c = i; c < p1.y / 16u; c += blockDim.x) dst[p0.y / 16u + c] = src1[c];
  }
}

// Image sizes (descriptors + list + records, 16-byte multiples) and their
// exclusive scan into byte offsets (single CTA); ranges[q] = {image bytes,
// list bytes, row-0 record bytes, row-1 record bytes}; out = {total, largest}.
__global__ void __launch_bounds__(1024) stage_scan_kernel(const uint32_t* __restrict__ totals, int n_sub,
                                                          uint32_t* __restrict__ ranges, uint32_t* __restrict__ offs,
                                                          unsigned long long* __restrict__ out) {
  __shared__ unsigned long long part[1024];
  __shared__ uint32_t red[1024];
  const int per = (n_sub + blockDim.x - 1) / blockDim.x;
  const int lo = min(n_sub, (int)threadIdx.x * per), hi = min(n_sub, lo + per);
  unsigned long long sum = 0;
  uint32_t mx = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t lbytes = (8u * totals[i] + 15u) & ~15u;
    const uint32_t size = kImgDescBytes + lbytes + ranges[4 * (size_t)i + 2] + ranges[4 * (size_t)i + 3];
    ranges[4 * (size_t)i + 0] = size;
    ranges[4 * (size_t)i + 1] = lbytes;
    sum += size;
    mx = max(mx, size);
  }
  part[threadIdx.x] = sum;
  red[threadIdx.x] = mx;
  __syncthreads();
  for (int dl = 1; dl < (int)blockDim.x; dl <<= 1) {
    const unsigned long long v = threadIdx.x >= (unsigned)dl ? part[threadIdx.x - dl] : 0ull;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  unsigned long long off = part[threadIdx.x] - sum;
  for (int i = lo; i < hi; ++i) {
    offs[i] = (uint32_t)off;
    off += ranges[4 * (size_t)i + 0];
  }
  for (int dl = blockDim.x / 2; dl > 0; dl >>= 1) {
    if (threadIdx.x < (unsigned)dl) red[threadIdx.x] = max(red[threadIdx.x], red[threadIdx.x + dl]);
    __syncthreads();
  }
  if (threadIdx.x == blockDim.x - 1) {
    offs[n_sub] = (uint32_t)part[blockDim.x - 1];
    out[0] = part[blockDim.x - 1];
  }
  if (threadIdx.x == 0) out[1] = red[0];
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" int mtc_repack_stage_plan(const mtc_stream_desc* s, uint32_t* counts, uint32_t* offsets,
                                     uint32_t* ranges, uint32_t* scratch_u32, uint64_t* out_host, void* stream) {
  clear_error();
  MTC_REQUIRE(s && counts && offsets && ranges && scratch_u32 && out_host && s->tiles && s->row_off && s->records,
              "mtc_repack_stage_plan: null pointer");
  MTC_REQUIRE(s->band_tiles == 8, "mtc_repack_stage_plan: band width %d (needs 8)", s->band_tiles);
  MTC_REQUIRE(2ull * s->max_row_bytes < 65536ull, "mtc_repack_stage_plan: stage of %u bytes exceeds 16-bit offsets",
              2 * s->max_row_bytes);
  const int nkb = (s->tk + 1) / 2;
  const int nb = (s->tn + s->band_tiles - 1) / s->band_tiles;
  const int n_sub = 2 * nb * nkb;
  cudaStream_t st = as_stream(stream);
  uint32_t* totals = scratch_u32;
  unsigned long long* out = reinterpret_cast<unsigned long long*>(scratch_u32 + ((n_sub + 1) & ~1));
  stage_lists_kernel<false><<<n_sub, 128, 0, st>>>(*s, nkb, nullptr, counts, totals, ranges, nullptr);
  MTC_CHECK_LAUNCH("mtc_repack_stage_plan: count");
  stage_scan_kernel<<<1, 1024, 0, st>>>(totals, n_sub, ranges, offsets, out);
  MTC_CHECK_LAUNCH("mtc_repack_stage_plan: scan");
  unsigned long long back[2];
  MTC_CHECK_CUDA(cudaMemcpyAsync(back, out, 16, cudaMemcpyDeviceToHost, st), "mtc_repack_stage_plan: copy back");
  MTC_CHECK_CUDA(cudaStreamSynchronize(st), "mtc_repack_stage_plan: sync");
  MTC_REQUIRE(back[0] < (1ull << 32), "mtc_repack_stage_plan: %llu bytes of sub-stage images exceed 32-bit offsets",
              back[0]);
  out_host[0] = back[0];
  out_host[1] = back[1];
  return MTC_OK;
}

extern "C" int mtc_repack_stage_fill(const mtc_stream_desc* s, const uint32_t* offsets, uint8_t* images,
                                     void* stream) {
  clear_error();
  MTC_REQUIRE(s && offsets && images && s->tiles && s->row_off && s->records, "mtc_repack_stage_fill: null pointer");
  MTC_REQUIRE((reinterpret_cast<uintptr_t>(images) & 15) == 0, "mtc_repack_stage_fill: images not 16-byte aligned");
  const int nkb = (s->tk + 1) / 2;
  const int nb = (s->tn + s->band_tiles - 1) / s->band_tiles;
  stage_lists_kernel<true><<<2 * nb * nkb, 128, 0, as_stream(stream)>>>(*s, nkb, offsets, nullptr, nullptr, nullptr,
                                                                        images);
  MTC_CHECK_LAUNCH("mtc_repack_stage_fill");
  return MTC_OK;
}

extern "C" int mtc_repack_plan(const mtc_leaf_in* leaves, const uint32_t* tile_leaf_begin, int32_t tk, int32_t tn,
                               int32_t band_tiles, int32_t scale_words, mtc_tile_desc* tiles, uint32_t* row_off,
                               uint32_t* scratch_u32, uint64_t* out_host, void* stream) {
  clear_error();
  MTC_REQUIRE(leaves && tile_leaf_begin && tiles && row_off && scratch_u32 && out_host,
              "mtc_repack_plan: null pointer argument");
  MTC_REQUIRE(tk > 0 && tn > 0 && band_tiles > 0, "mtc_repack_plan: bad grid %d x %d (band %d)", tk, tn,
              band_tiles);
  MTC_REQUIRE((long long)tk * tn < (1ll << 30), "mtc_repack_plan: too many tiles");
  MTC_REQUIRE(scale_words == 1 || scale_words == 2, "mtc_repack_plan: scale_words must be 1 or 2");
  cudaStream_t st = as_stream(stream);
  const int T = tk * tn;
  // scratch layout: [T] record bytes | u64 total | u32 err | u32 max row
  uint32_t* rec = scratch_u32;
  unsigned long long* total = reinterpret_cast<unsigned long long*>(scratch_u32 + ((T + 1) & ~1));
  uint32_t* err = reinterpret_cast<uint32_t*>(total + 1);
  uint32_t* max_row = err + 1;
  MTC_CHECK_CUDA(cudaMemsetAsync(total, 0, 16, st), "mtc_repack_plan: memset");
  plan_tiles<<<(T + 255) / 256, 256, 0, st>>>(leaves, tile_leaf_begin, tk, tn, band_tiles, scale_words, tiles,
                                              rec, err);
  MTC_CHECK_LAUNCH("mtc_repack_plan: plan_tiles");
  plan_scan<<<1, 1024, 0, st>>>(rec, tk, tn, band_tiles, tiles, row_off, total, max_row);
  MTC_CHECK_LAUNCH("mtc_repack_plan: plan_scan");
  uint32_t back[4];
  MTC_CHECK_CUDA(cudaMemcpyAsync(back, total, 16, cudaMemcpyDeviceToHost, st), "mtc_repack_plan: copy back");
  MTC_CHECK_CUDA(cudaStreamSynchronize(st), "mtc_repack_plan: sync");
  if (back[2] != 0) {
    set_error("mtc_repack_plan: leaf list does not tile the matrix (code %u: %s%s%s)", back[2],
              (back[2] & kErrCoverage) ? "coverage/order " : "", (back[2] & kErrLeafCount) ? "leaf-count " : "",
              (back[2] & kErrLeaf) ? "leaf-fields" : "");
    return MTC_ERR_INVALID;
  }
  out_host[0] = (uint64_t)back[0] | ((uint64_t)back[1] << 32);
  out_host[1] = back[3];
  return MTC_OK;
}

extern "C" int mtc_repack_fill(const uint8_t* arena, uint64_t arena_bytes, const mtc_leaf_in* leaves,
                               const uint32_t* tile_leaf_begin, const mtc_stream_desc* s, uint8_t* records,
                               uint32_t* scratch_u32, void* stream) {
  clear_error();
  MTC_REQUIRE(s && leaves && tile_leaf_begin && records && s->tiles && scratch_u32,
              "mtc_repack_fill: null pointer argument");
  MTC_REQUIRE(arena || arena_bytes == 0, "mtc_repack_fill: null arena");
  MTC_REQUIRE((reinterpret_cast<uintptr_t>(records) & 15) == 0, "mtc_repack_fill: records not 16-byte aligned");
  MTC_REQUIRE(s->scale_words == 1 || s->scale_words == 2, "mtc_repack_fill: scale_words must be 1 or 2");
  cudaStream_t st = as_stream(stream);
  const int T = s->tk * s->tn;
  uint32_t* err = scratch_u32;
  MTC_CHECK_CUDA(cudaMemsetAsync(err, 0, 4, st), "mtc_repack_fill: memset");
  fill_tiles<<<(T + 7) / 8, 256, 0, st>>>(arena, arena_bytes, leaves, tile_leaf_begin, s->tk, s->tn, s->tiles,
                                          s->exp2, s->scale_words, records, err);
  cudaError_t le = cudaGetLastError();
  uint32_t hb = 0;
  cudaError_t ce = cudaMemcpyAsync(&hb, err, 4, cudaMemcpyDeviceToHost, st);
  cudaError_t se = cudaStreamSynchronize(st);
  if (le != cudaSuccess) return cuda_fail(le, "mtc_repack_fill: fill_tiles");
  if (ce != cudaSuccess) return cuda_fail(ce, "mtc_repack_fill: copy back");
  if (se != cudaSuccess) return cuda_fail(se, "mtc_repack_fill: sync");
  MTC_REQUIRE(hb == 0, "mtc_repack_fill: a leaf payload lies outside the arena");
  return MTC_OK;
}
