// Tensor-core decode GEMM for M <= 16 tokens: Y[:, pc] = X[:, pr] @ Wp.
//
// Replaces the reference's packed GEMM (mtc/kernels/gemm.py:124-210, 541-574)
// and the MTC-QT-P gather / scatter (mtc/core/permutation.py:15-21) for
// decode-sized M.  The packed weights are read from HBM once; the product is
// computed swap-AB on the tensor cores: D (128 features x 16 tokens, fp32
// in TMEM) += W^T tile (128 features x 64 k, dequantised into shared memory)
// x X^T tile (16 tokens x 64 k, fp16, TMA).  The SMs' issue slots go to the
// dequantisation alone.
//
//  * work unit = (half band: 4 tiles = 128 features, range of k stages of
//    64); persistent CTAs, one per SM, take units u = blockIdx.x, + grid, ...
//    The stages of a unit go in pairs (2p, 2p + 1) to the two dequant
//    groups in turn: pair p to group p mod 2.
//  * warp roles:
//      warps 0-3  epilogue: TMEM -> partial sums of the unit -> workspace;
//                 the last unit of a half band (atomic ticket) reduces the
//                 partials in a fixed order and scatters Y[:, pc]
//      warp  4    X producer: one TMA per stage pair (a 3-d box of two
//                 64-k blocks of Xp) into a ring of pair slots
//      warp  5    packed producer: the two images of a stage pair (adjacent
//                 in the half-band-major image order) with one cp.async.bulk
//                 into a shared-memory byte ring
//      warps 6-7  MMA issuers, one per dequant group: when the group's
//                 eight warps have written the two W tiles of a pair
//                 (mbarrier), one thread issues the pair's eight MMAs into
//                 the group's own accumulator and commits them to the W
//                 buffer's release barrier
//      warps 8-23 dequant, two groups of eight (dequant_substage, shared
//                 with the prefill).  A warp never waits for the other
//                 warps of its group except through the W buffers (two
//                 pairs per group), and it pays the waits, proxy fence and
//                 arrivals once per pair of sub-stages.
//  * accumulators: 2 units in flight x 2 groups x 16 columns; the epilogue
//    adds the two groups' partial products of a unit.
// Every mbarrier wait is bounded; a timeout sets MTC_STATUS_TIMEOUT.
#include "mtc_common.cuh"
#include "mtc_internal.h"
#include "mtc_substage.cuh"
#include "mtc_tc.cuh"

namespace mtc {
namespace {

constexpr int kTok = 16;        // token columns of the MMA (N); M <= 16
constexpr int BK = 64;          // K per stage (two k-tile rows)
constexpr int kFeat = 128;      // features per unit (MMA M)
constexpr int kEpiWarps = 4;
constexpr int kXWarp = 4;
constexpr int kPackWarp = 5;
constexpr int kIssWarp0 = 6;
constexpr int kDeqWarp0 = 8;
constexpr int kDeqWarps = kSubWarps;
constexpr int kDeqGroups = 2;
constexpr int kThreads = (kDeqWarp0 + kDeqGroups * kDeqWarps) * 32;
constexpr uint32_t kXBytes = kTok * BK * 2;     // 2 KB
constexpr uint32_t kWBytes = kFeat * BK * 2;    // 16 KB
constexpr int kXPairs = 8;                      // X ring slots, one stage pair each
constexpr uint32_t kXPair = 2 * kXBytes;
constexpr int kWBufs = 2;                       // W buffers (two tiles each) per group
constexpr uint32_t kWPair = 2 * kWBytes;
constexpr int kRingSlots = 8;                   // stage pairs in the byte ring at most
constexpr int kMetaChunk = 32;
constexpr uint32_t kTmemCols = 64;              // [unit buffer d][group g] -> column 32 d + 16 g
constexpr int kEpiBar = 1;                      // named barrier of the epilogue warps

struct DecodeParams {
  mtc_stream_desc s;
  int M;
  float* Y;
  long long ldy;
  const int32_t* pc;   // column permutation (Y[:, pc[n]] = Yp[:, n]) or null
  float* part;         // [units][kTok][kFeat] partial sums
  uint32_t* counters;  // [half bands] tickets, zero between calls
  uint32_t* status;
  int n_hb, nkb, n_kr, R, n_units;
  uint32_t ring_bytes;
  float pow2e, inv_pow2e;
  unsigned long long timeout_ns;
  Epi ep;              // bias / activation applied to Y
};

__device__ __forceinline__ void flag(uint32_t* st, uint32_t bits) {
  if (st) atomicOr(st, bits);
}

// AND of `v` over the `n` threads meeting at named barrier `id` (all of them
// take part, so the group decides together whether to go on).
__device__ __forceinline__ bool bar_and(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmap_x, const DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sX = smem;                                         // [kXPairs][2][2 KB], 1024-byte aligned
  uint8_t* sW = sX + kXPairs * kXPair;                        // [2 groups][kWBufs][2][16 KB]
  uint8_t* sP = sW + kDeqGroups * kWBufs * kWPair;            // packed byte ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + p.ring_bytes);
  uint64_t* x_full = bars;                                    // [kXPairs]
  uint64_t* x_empty = x_full + kXPairs;                       // [kXPairs]
  uint64_t* w_empty = x_empty + kXPairs;                      // [groups * kWBufs]
  uint64_t* w_full = w_empty + kDeqGroups * kWBufs;           // [groups * kWBufs]
  uint64_t* pfull = w_full + kDeqGroups * kWBufs;             // [kRingSlots]
  uint64_t* pempty = pfull + kRingSlots;
  uint64_t* acc_full = pempty + kRingSlots;                   // [2]
  uint64_t* acc_empty = acc_full + 2;                         // [2]
  uint64_t* drain = acc_empty + 2;                            // [groups]
  volatile uint32_t* flags = reinterpret_cast<volatile uint32_t*>(drain + kDeqGroups);  // [0] abort, [1] last unit
  uint32_t* tmem_slot = const_cast<uint32_t*>(flags) + 4;
  uint32_t* pmeta = tmem_slot + 4;                            // [kRingSlots][2 stages][4]
  uint32_t* dtab = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(bars) + 1280);
  uint4* smeta = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(bars) + 1792);  // [2][kMetaChunk][2]
  static_assert((2 * kXPairs + 2 * kDeqGroups * kWBufs + 2 * kRingSlots + 4 + kDeqGroups) * 8 + 32 + 32 * kRingSlots <=
                    1280,
                "barrier region");

  const mtc_stream_desc& s = p.s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < kXPairs; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], kDeqGroups);  // one commit (or arrive) per group
      mbar_init(&acc_empty[i], kEpiWarps);
    }
    for (int i = 0; i < kDeqGroups * kWBufs; ++i) {
      mbar_init(&w_empty[i], 1);
      mbar_init(&w_full[i], kDeqWarps);
    }
    for (int i = 0; i < kRingSlots; ++i) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], kDeqWarps);
    }
    for (int i = 0; i < kDeqGroups; ++i) mbar_init(&drain[i], 1);
    flags[0] = 0;
    fence_barrier_init();
  }
  if (warp == 1) load_dec_table(dtab, lane);
  if (warp == 0) tc::tmem_alloc(tmem_slot, kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;

  // unit u -> half band hb = u / n_kr, stages [kb0, kb1)
  auto unit_range = [&](int u, int& hb, int& kb0, int& kb1) {
    hb = u / p.n_kr;
    kb0 = (u % p.n_kr) * p.R;
    kb1 = min(p.nkb, kb0 + p.R);
  };

  if (warp == kXWarp) {
    // ---------------------------------------------------------------- X producer
    // One TMA per stage pair (16 rows of Xp x two 64-k blocks) into a ring
    // of kXPairs slots, released by the MMAs' commits.
    if (lane == 0) {
      uint32_t ip = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.n_units && ok; u += gridDim.x) {
        int hb, kb0, kb1;
        unit_range(u, hb, kb0, kb1);
        const int P = (kb1 - kb0 + 1) / 2;
        for (int pr = 0; pr < P; ++pr, ++ip) {
          const int sx = ip % kXPairs;
          if (ip >= (uint32_t)kXPairs && !mbar_wait(&x_empty[sx], ((ip / kXPairs) & 1) ^ 1, p.timeout_ns)) {
            ok = false;
            break;
          }
          if (flags[0]) {
            ok = false;
            break;
          }
          mbar_expect_tx(&x_full[sx], kXPair);
          tc::tma_load_3d(sX + sx * kXPair, &tmap_x, 0, 0, kb0 + 2 * pr, &x_full[sx]);
        }
      }
      if (!ok) {
        flags[0] = 1;
        flag(p.status, MTC_STATUS_TIMEOUT);
      }
      // let the loads in flight land before the CTA can exit
      for (uint32_t q = ip > (uint32_t)kXPairs ? ip - kXPairs : 0u; q < ip; ++q)
        (void)mbar_wait(&x_full[q % kXPairs], (q / kXPairs) & 1, 10000000ull);
    }
  } else if (warp == kPackWarp) {
    // ---------------------------------------------------------------- packed producer
    // Metadata of up to 32 consecutive sub-stages of a unit, loaded by the
    // whole warp one chunk ahead of lane 0, which issues the bulk copies.
    const int n_my_units = (int)blockIdx.x < p.n_units ? (p.n_units - 1 - (int)blockIdx.x) / gridDim.x + 1 : 0;
    const int chunks_per_unit = (p.R + kMetaChunk - 1) / kMetaChunk;
    const int n_chunks = n_my_units * chunks_per_unit;
    uint4 nxt0, nxt1;
    auto load_chunk = [&](int q) {
      nxt0 = make_uint4(0u, 0u, 0u, 0u);
      nxt1 = make_uint4(0u, 0u, 0u, 0u);
      if (q >= n_chunks) return;
      int hb, kb0, kb1;
      unit_range(blockIdx.x + (q / chunks_per_unit) * gridDim.x, hb, kb0, kb1);
      const int kb = kb0 + (q % chunks_per_unit) * kMetaChunk + lane;
      if (kb < kb1) {
        const size_t sub = (size_t)hb * p.nkb + kb;
        nxt0 = *reinterpret_cast<const uint4*>(s.stage_ranges + 4 * sub);
        nxt1 = make_uint4(s.stage_counts[sub], s.stage_offsets[sub], 0u, 0u);
      }
    };
    auto store_chunk = [&](int buf) {
      smeta[2 * (buf * kMetaChunk + lane)] = nxt0;
      smeta[2 * (buf * kMetaChunk + lane) + 1] = nxt1;
    };
    load_chunk(0);
    store_chunk(0);
    __syncwarp();
    uint32_t it = 0, oldest = 0;
    unsigned long long ring_head = 0;
    uint32_t head_off = 0;
    unsigned long long ring_start[kRingSlots];
    for (int q = 0; q < n_chunks; ++q) {
      load_chunk(q + 1);
      if (lane == 0) {
        int hb, kb0, kb1;
        unit_range(blockIdx.x + (q / chunks_per_unit) * gridDim.x, hb, kb0, kb1);
        const int c0 = kb0 + (q % chunks_per_unit) * kMetaChunk;
        const int c1 = min(kb1, c0 + kMetaChunk);
        // stage pairs (c0 - kb0 is even): the two images are adjacent
        for (int kb = c0; kb < c1 && !flags[0]; kb += 2, ++it) {
          const bool two = kb + 1 < c1;
          const uint4 rg = smeta[2 * ((q & 1) * kMetaChunk + (kb - c0))];  // bytes: image, list, row 0, row 1
          const uint4 mc = smeta[2 * ((q & 1) * kMetaChunk + (kb - c0)) + 1];  // counts, image offset
          const uint4 rg1 = two ? smeta[2 * ((q & 1) * kMetaChunk + (kb + 1 - c0))] : make_uint4(0u, 0u, 0u, 0u);
          const uint4 mc1 = two ? smeta[2 * ((q & 1) * kMetaChunk + (kb + 1 - c0)) + 1] : make_uint4(0u, 0u, 0u, 0u);
          const uint32_t need = rg.x + rg1.x;
          if (need > p.ring_bytes || ((need | mc.y) & 15u) || (two && mc1.y != mc.y + rg.x)) {
            flag(p.status, MTC_STATUS_BAD_STREAM);
            flags[0] = 1;
            break;
          }
          // (positions advance without division: a piece that would cross
          // the end of the ring starts at the next lap instead)
          unsigned long long pos = ring_head;
          uint32_t start = head_off;
          if (start + need > p.ring_bytes) {
            pos += p.ring_bytes - start;
            start = 0;
          }
          // live bytes are [ring_start[oldest], ring_head): the new piece must
          // end within one ring length of the oldest live sub-stage's start
          bool ok = true;
          while (it - oldest >= (uint32_t)kRingSlots ||
                 (oldest != it && ring_start[oldest % kRingSlots] + p.ring_bytes < pos + need)) {
            if (!mbar_wait(&pempty[oldest % kRingSlots], (oldest / kRingSlots) & 1, p.timeout_ns)) {
              ok = false;
              break;
            }
            ++oldest;
          }
          if (!ok) {
            flags[0] = 1;
            break;
          }
          const int ps = it % kRingSlots;
          ring_start[ps] = pos;
          ring_head = pos + need;
          head_off = start + need;
          pmeta[8 * ps + 0] = start;
          pmeta[8 * ps + 1] = mc.x;
          pmeta[8 * ps + 2] = rg.y;
          pmeta[8 * ps + 3] = rg.z;
          pmeta[8 * ps + 4] = start + rg.x;
          pmeta[8 * ps + 5] = mc1.x;
          pmeta[8 * ps + 6] = rg1.y;
          pmeta[8 * ps + 7] = rg1.z;
          // both images of the pair in one bulk copy
          mbar_expect_tx(&pfull[ps], need);
          bulk_g2s(sP + start, s.stage_images + mc.y, need, &pfull[ps]);
        }
      }
      __syncwarp();
      store_chunk((q + 1) & 1);
      __syncwarp();
      if (flags[0]) break;
    }
    if (lane == 0 && flags[0]) {
      for (uint32_t j = it > (uint32_t)kRingSlots ? it - kRingSlots : 0u; j < it; ++j)
        (void)mbar_wait(&pfull[j % kRingSlots], (j / kRingSlots) & 1, 10000000ull);
      flag(p.status, MTC_STATUS_TIMEOUT);
    }
  } else if (warp >= kDeqWarp0) {
    // ---------------------------------------------------------------- dequant
    const int grp = (warp - kDeqWarp0) / kDeqWarps;
    const int dw = (warp - kDeqWarp0) % kDeqWarps;
    uint32_t ip = 0, sp = 0;
    bool go = true;
    for (int u = blockIdx.x; u < p.n_units && go; u += gridDim.x) {
      int hb, kb0, kb1;
      unit_range(u, hb, kb0, kb1);
      const int L = kb1 - kb0, P = (L + 1) / 2;
      for (int pr = 0; pr < P && go; ++pr, ++ip) {
        if ((pr & 1) != grp) continue;
        const int b = grp * kWBufs + (sp & 1);
        const int n = min(2, L - 2 * pr);
        const int ps = ip % kRingSlots;
        bool ok = !flags[0];
        if (ok && sp >= (uint32_t)kWBufs) ok = mbar_wait(&w_empty[b], ((sp >> 1) - 1) & 1, p.timeout_ns);
        ok = ok && mbar_wait(&pfull[ps], (ip / kRingSlots) & 1, p.timeout_ns);
        ok = __all_sync(0xffffffffu, ok);  // warp-uniform: the dequant uses whole-warp shuffles
        if (!ok) {
          flags[0] = 1;
          go = false;
          break;
        }
        for (int h = 0; h < n; ++h) {
          const int kb = kb0 + 2 * pr + h;
          const uint32_t* pm = pmeta + 8 * ps + 4 * h;
          dequant_substage(sW + b * kWPair + h * kWBytes, sP + pm[0], pm[1], pm[2], pm[3], 2 * kb + 1 >= s.tk, dtab,
                           s.scale_words, p.pow2e, dw, lane, tid - (kDeqWarp0 + grp * kDeqWarps) * 32,
                           (int)((2 * sp + h) * 3u));
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&pempty[ps]);
          mbar_arrive(&w_full[b]);
        }
        ++sp;
      }
    }
  } else if (warp >= kIssWarp0) {
    // ---------------------------------------------------------------- MMA issuers
    const int grp = warp - kIssWarp0;
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16_f32(kFeat, kTok);
      uint32_t sp = 0, ucount = 0, ip = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.n_units && ok; u += gridDim.x, ++ucount) {
        int hb, kb0, kb1;
        unit_range(u, hb, kb0, kb1);
        const int L = kb1 - kb0, P = (L + 1) / 2, d = ucount & 1;
        const uint32_t ipu = ip;
        ip += (uint32_t)P;
        // the accumulator of the unit two back must have been read out
        if (ucount >= 2 && !mbar_wait(&acc_empty[d], ((ucount >> 1) - 1) & 1, p.timeout_ns)) {
          ok = false;
          break;
        }
        if (P <= grp) {
          mbar_arrive(&acc_full[d]);  // no pair of this unit: the accumulator is not read
          continue;
        }
        const uint32_t acc = tmem + 32u * d + 16u * grp;
        for (int pr = grp; pr < P; pr += kDeqGroups, ++sp) {
          const int b = grp * kWBufs + (sp & 1);
          const int n = min(2, L - 2 * pr);
          const uint32_t ipp = ipu + pr;
          const int sx = ipp % kXPairs;
          if (flags[0] || !mbar_wait(&w_full[b], (sp >> 1) & 1, p.timeout_ns) ||
              !mbar_wait(&x_full[sx], (ipp / kXPairs) & 1, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc::fence_after();
          for (int h = 0; h < n; ++h) {
            const uint32_t w0 = smem_u32(sW + b * kWPair + h * kWBytes);
            const uint32_t x0 = smem_u32(sX + sx * kXPair + h * kXBytes);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              tc::mma_f16_ss(acc, tc::smem_desc_k_sw128(w0 + 32 * kk), tc::smem_desc_k_sw128(x0 + 32 * kk), idesc,
                             (pr > grp || h > 0 || kk > 0) ? 1u : 0u);
          }
          tc::commit(&x_empty[sx]);
          tc::commit(&w_empty[b]);
        }
        if (!ok) break;
        tc::commit(&acc_full[d]);
      }
      if (!ok) flags[0] = 1;
      tc::commit(&drain[grp]);
      (void)mbar_wait(&drain[grp], 0, 100000000ull);
      if (flags[0]) flag(p.status, MTC_STATUS_TIMEOUT);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 0-3)
    // Thread (warp w, lane l) owns feature 32 w + l of the unit.
    const int f = 32 * warp + lane;
    uint32_t ucount = 0;
    for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++ucount) {
      int hb, kb0, kb1;
      unit_range(u, hb, kb0, kb1);
      const int d = ucount & 1;
      const bool ok = !flags[0] && mbar_wait(&acc_full[d], (ucount >> 1) & 1, p.timeout_ns);
      if (!bar_and(kEpiBar, kEpiWarps * 32, ok)) {
        flags[0] = 1;
        break;
      }
      tc::fence_after();
      uint32_t v[16], w[16];
      const uint32_t row = tmem + ((uint32_t)(32 * warp) << 16) + 32u * d;
      tc::tmem_ld_32x32b_x16(row, v);
      if (kb1 - kb0 >= 3) {  // the second group has a pair in this unit
        tc::tmem_ld_32x32b_x16(row + 16u, w);
#pragma unroll
        for (int t = 0; t < kTok; ++t) v[t] = __float_as_uint(__uint_as_float(v[t]) + __uint_as_float(w[t]));
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[d]);
      float* part = p.part + (size_t)u * kTok * kFeat;
#pragma unroll
      for (int t = 0; t < kTok; ++t)
        if (t < p.M) part[t * kFeat + f] = __uint_as_float(v[t]);
      // ticket: the last unit of the half band reduces in a fixed order
      __threadfence();
      asm volatile("bar.sync %0, %1;" ::"r"(kEpiBar), "r"(kEpiWarps * 32) : "memory");
      if (tid == 0) flags[1] = atomicAdd(&p.counters[hb], 1u) == (uint32_t)(p.n_kr - 1) ? 1u : 0u;
      asm volatile("bar.sync %0, %1;" ::"r"(kEpiBar), "r"(kEpiWarps * 32) : "memory");
      if (flags[1]) {
        __threadfence();
        const int n = hb * kFeat + f;
        if (n < s.N) {
          const int col = p.pc ? p.pc[n] : n;
          // partials r = 0, 1, ... summed in that order for every token; the
          // loads of one partial are issued together
          float acc[kTok];
#pragma unroll
          for (int t = 0; t < kTok; ++t) acc[t] = 0.0f;
          for (int r = 0; r < p.n_kr; ++r) {
            const float* pr = p.part + (size_t)(hb * p.n_kr + r) * kTok * kFeat + f;
#pragma unroll
            for (int t = 0; t < kTok; ++t)
              if (t < p.M) acc[t] += __ldcg(pr + t * kFeat);
          }
#pragma unroll
          for (int t = 0; t < kTok; ++t)
            if (t < p.M) p.Y[(long long)t * p.ldy + col] = epi_apply(p.ep, acc[t] * p.inv_pow2e, col);
        }
        if (tid == 0) p.counters[hb] = 0u;
      }
      asm volatile("bar.sync %0, %1;" ::"r"(kEpiBar), "r"(kEpiWarps * 32) : "memory");
    }
    if (flags[0]) flag(p.status, MTC_STATUS_TIMEOUT);
  }

  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

struct DecodePlan {
  int Kp, nkb, n_hb, R, n_kr, n_units, grid;
  uint32_t ring_bytes;
  size_t smem, xp_bytes, part_bytes;
};

bool plan_decode(const mtc_stream_desc* s, int M, DecodePlan* pl) {
  if (M < 1 || M > kTok) return false;
  pl->Kp = (s->tk + 1) / 2 * BK;  // whole 64-k blocks: a block never runs into the next Xp row
  pl->nkb = (s->tk + 1) / 2;
  const int n_bands = (s->tn + s->band_tiles - 1) / s->band_tiles;
  pl->n_hb = 2 * n_bands;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // about four units per SM, at least four stages each
  const long long total = (long long)pl->n_hb * pl->nkb;
  long long R = (total + 4LL * sms - 1) / (4LL * sms);
  R = R < 4 ? 4 : R;
  pl->R = (int)(R < pl->nkb ? R : pl->nkb);
  pl->n_kr = (pl->nkb + pl->R - 1) / pl->R;
  pl->n_units = pl->n_hb * pl->n_kr;
  pl->grid = pl->n_units < sms ? pl->n_units : sms;
  const size_t cap = 227 * 1024;
  const size_t fixed = 1024 /*align*/ + 1792 /*barriers, flags, decoder table*/ + 64 * kMetaChunk;
  const size_t used = fixed + (size_t)kXPairs * kXPair + (size_t)kDeqGroups * kWBufs * kWPair;
  const size_t ring = (cap - used) & ~(size_t)127;
  if (s->max_stage_bytes == 0 || ring < s->max_stage_bytes) return false;
  pl->ring_bytes = (uint32_t)ring;
  pl->smem = used + ring;
  pl->xp_bytes = ((size_t)kTok * pl->Kp * 2 + 255) & ~(size_t)255;  // 16 rows (the MMA's N) x Kp
  pl->part_bytes = (size_t)pl->n_units * kTok * kFeat * sizeof(float);
  return true;
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" size_t mtc_decode_workspace_bytes(const mtc_stream_desc* s, int32_t M) {
  DecodePlan pl;
  if (!s || !plan_decode(s, M, &pl)) return 0;
  return pl.xp_bytes + pl.part_bytes;
}

extern "C" int mtc_decode(const mtc_stream_desc* s, const float* X, int32_t M, int64_t ldx, const int32_t* row_perm,
                          const int32_t* col_perm, float* Y, int64_t ldy, void* ws, size_t ws_bytes,
                          uint32_t* counters, uint32_t* status, const mtc_epilogue* ep, void* stream) {
  clear_error();
  EpiArg epa;
  {
    const int rc = read_epilogue(ep, &epa, "mtc_decode");
    if (rc != MTC_OK) return rc;
  }
  MTC_REQUIRE(s && X && Y && ws && counters && s->records && s->tiles && s->row_off,
              "mtc_decode: null pointer argument");
  MTC_REQUIRE(M >= 1 && M <= kTok, "mtc_decode: M=%d outside 1..%d (use mtc_gemm_prefill)", M, kTok);
  MTC_REQUIRE(ldx >= s->K && ldy >= s->N, "mtc_decode: bad leading dimensions");
  MTC_REQUIRE(s->band_tiles * kTile == 2 * kFeat, "mtc_decode: stream band width %d tiles, kernel needs %d",
              s->band_tiles, 2 * kFeat / kTile);
  MTC_REQUIRE(s->stage_images && s->stage_counts && s->stage_offsets && s->stage_ranges && s->max_stage_bytes,
              "mtc_decode: stage work lists missing (run mtc_repack_stage_plan and mtc_repack_stage_fill)");
  MTC_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 255) == 0, "mtc_decode: workspace not 256-byte aligned");
  DecodePlan pl;
  MTC_REQUIRE(plan_decode(s, M, &pl), "mtc_decode: a sub-stage of %u bytes does not fit shared memory",
              s->max_stage_bytes);
  if (ws_bytes < pl.xp_bytes + pl.part_bytes) {
    set_error("mtc_decode: workspace %zu bytes, need %zu", ws_bytes, pl.xp_bytes + pl.part_bytes);
    return MTC_ERR_WORKSPACE;
  }
  cudaStream_t st = as_stream(stream);
  __half* Xp = static_cast<__half*>(ws);
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + pl.xp_bytes);
  int rc = launch_gather_x(X, ldx, s->K, pl.Kp, row_perm, M, Xp, status, st);
  if (rc != MTC_OK) return rc;
  CUtensorMap tmap;
  rc = encode_xp_blocks_map(&tmap, Xp, pl.Kp, kTok, 2, "mtc_decode");
  if (rc != MTC_OK) return rc;
  DecodeParams p;
  p.s = *s;
  p.M = M;
  p.Y = Y;
  p.ldy = ldy;
  p.pc = col_perm;
  p.part = part;
  p.counters = counters;
  p.status = status;
  p.n_hb = pl.n_hb;
  p.nkb = pl.nkb;
  p.n_kr = pl.n_kr;
  p.R = pl.R;
  p.n_units = pl.n_units;
  p.ring_bytes = pl.ring_bytes;
  p.pow2e = ldexpf(1.0f, s->exp2);
  p.inv_pow2e = ldexpf(1.0f, -s->exp2);
  p.timeout_ns = wait_limit_ns();
  p.ep = Epi{epa.bias, epa.act};
  MTC_CHECK_CUDA(cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem),
                 "mtc_decode: smem attribute");
  decode_kernel<<<pl.grid, kThreads, pl.smem, st>>>(tmap, p);
  MTC_CHECK_LAUNCH("mtc_decode");
  return MTC_OK;
}
