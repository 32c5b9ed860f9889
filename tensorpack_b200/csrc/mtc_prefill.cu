// Fused dequant + tcgen05 GEMM for prefill-sized M: Y[:, pc] = X[:, pr] @ Wp.
//
// Replaces the reference's packed GEMM (mtc/kernels/gemm.py:124-210, 541-574)
// and the MTC-QT-P gather / scatter (mtc/core/permutation.py:15-21) for
// large M.  Three kernels on one stream:
//
//  1. gather_x:   Xp[m][k] = fp16(X[m][pr[k]]) (zero for k >= K); one CTA per
//                 row stages the row in shared memory so both the read and
//                 the write are coalesced.
//  2. prefill:    persistent, one CTA per SM, output tile 256 tokens x 256
//                 features, K step 64.  Warp roles:
//                   warps 0-3  epilogue: TMEM -> registers -> global
//                   warp  4    A producer: TMA of the Xp tile (SWIZZLE_128B)
//                   warp  5    TMEM allocator + single-thread tcgen05.mma issuer
//                   warp  6    packed producer: cp.async.bulk of each stage's
//                              descriptors, work list and records into a
//                              shared-memory byte ring, up to 8 stages ahead
//                   warps 7-22 dequant: the stage's work list, packed codes ->
//                              fp16 W tile in the K-major SWIZZLE_128B layout
//                              the MMA reads
//                 Two 128x256 fp32 accumulators (all 512 TMEM columns) share
//                 each dequantised W tile, so every weight is decoded once
//                 per 256 tokens.  A and W tiles have their own pipeline
//                 depths; mbarriers link the stages; every wait is bounded.
//  3. permute_y:  Y[m][j] = Yp[m][ipc[j]] for MTC-QT-P matrices (row staged in
//                 shared memory, coalesced in and out).
#include "mtc_common.cuh"
#include "mtc_internal.h"
#include "mtc_substage.cuh"
#include "mtc_tc.cuh"

namespace mtc {
namespace {

constexpr int CBM = 512;  // tokens per CTA pair tile (two M=256 pair MMAs)
constexpr int BM = 256;   // tokens whose A rows one CTA holds (128 per accumulator)
constexpr int BN = 256;   // features per pair tile (one column band)
constexpr int BNH = 128;  // features one CTA dequantises (its half of the band)
constexpr int BK = 64;    // K per pipeline stage (two k-tile rows)
constexpr int kEpiWarps = 4;
constexpr int kProdWarp = 4;   // A tiles
constexpr int kMmaWarp = 5;    // TMEM allocation (both CTAs), MMA issue (even CTA)
constexpr int kPackWarp = 6;   // packed sub-stages
constexpr int kDeqWarp0 = 7;
constexpr int kDeqWarps = kSubWarps;   // dequant warps per stage
// Dequant groups take alternate stages, so each group has two stage times
// for one stage: a stage's decode is latency-bound (dependent shared-memory
// loads, decode, stores), and a second group hides that latency.
#ifndef MTC_DEQ_GROUPS
#define MTC_DEQ_GROUPS 2
#endif
constexpr int kDeqGroups = MTC_DEQ_GROUPS;
constexpr int kThreads = (kDeqWarp0 + kDeqGroups * kDeqWarps) * 32;
constexpr uint32_t kAHalf = 128 * BK * 2;   // A rows of one accumulator
constexpr uint32_t kABytes = 2 * kAHalf;
constexpr uint32_t kBBytes = BNH * BK * 2;
constexpr int kMaxS = 4;
// Packed data of each sub-stage sits contiguously in a shared-memory byte
// ring: [128 B tile descriptors: 4 of k-row 2kb, 4 of k-row 2kb + 1][work
// list][records of the row-0 part][records of the row-1 part].  Sub-stage
// sizes vary (in MTC-QT-P allocations the largest is about twice the
// median), so a ring keeps several typical ones in flight where fixed slots
// sized for the largest would hold one or two.
constexpr int kRingSlots = 8;          // sub-stages in flight at most
constexpr int kMetaChunk = 32;         // sub-stages of metadata the packed producer stages at a time
constexpr uint32_t kDescBytes = kSubDescBytes;

struct PrefillParams {
  mtc_stream_desc s;
  int M;
  float* Y;           // Y (no column permutation) or Yp (permuted columns)
  long long ldy;
  uint32_t* status;
  int n_bands, n_tiles, nkb;
  // Split tail: tiles [t_main, n_tiles) (the last, partial wave) are cut
  // along K into `split` pieces each; piece j (cluster j < n_pieces) covers
  // k blocks [s nkb / split, (s + 1) nkb / split) of tile t_main + j / split,
  // s = j % split, and leaves its partial sums in part[j] (CBM x BN fp32,
  // row-major), which prefill_tail_reduce adds up.  n_pieces = 0: no split.
  int t_main, split, n_pieces;
  float* part;
  int SA, SB;         // A-tile and W-tile pipeline depths
  int vec2;           // Y rows 8-byte aligned: float2 stores
  uint32_t ring_bytes;
  float pow2e, inv_pow2e;
  unsigned long long timeout_ns;
  Epi ep;             // bias / activation applied to Y (direct output only)
};

__device__ __forceinline__ void flag(uint32_t* st, uint32_t bits) {
  if (st) atomicOr(st, bits);
}

// The work of one cluster, in the order every role walks it: its whole tiles
// t = cid, cid + G, ... below t_main, then at most one tail piece.
struct Item {
  int tile, kb0, kb1, piece;  // piece < 0: a whole tile
};
__device__ __forceinline__ int regular_items(const PrefillParams& p, int cid, int G) {
  return cid < p.t_main ? (p.t_main - 1 - cid) / G + 1 : 0;
}
__device__ __forceinline__ int item_count(const PrefillParams& p, int cid, int G) {
  return regular_items(p, cid, G) + (cid < p.n_pieces ? 1 : 0);
}
__device__ __forceinline__ Item item_of(const PrefillParams& p, int cid, int G, int i) {
  Item w;
  if (i < regular_items(p, cid, G)) {
    w.tile = cid + i * G;
    w.kb0 = 0;
    w.kb1 = p.nkb;
    w.piece = -1;
  } else {
    const int sp = cid % p.split;
    w.tile = p.t_main + cid / p.split;
    w.kb0 = sp * p.nkb / p.split;
    w.kb1 = (sp + 1) * p.nkb / p.split;
    w.piece = cid;
  }
  return w;
}


// Launched as clusters of two CTAs; cluster c takes pair tiles c, c + G, ...
// (G = number of clusters), each 512 tokens x one band of 256 features.
// EPI: the output epilogue (bias / activation) is applied in the store loop;
// the plain instance keeps the epilogue warps' registers for the main loop.
template <bool EPI>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmap_x, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base for the SWIZZLE_128B atoms (the same offset in
  // both CTAs, which the pair MMA requires); pointer arithmetic on the
  // __shared__ array keeps the shared address space visible to the compiler
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = sA + p.SA * kABytes;
  uint8_t* sP = sB + p.SB * kBBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + p.ring_bytes);
  uint64_t* full_a = bars;                    // [SA] even CTA: TMA bytes of both CTAs
  uint64_t* empty_a = full_a + kMaxS;         // [SA] MMA commit (both CTAs)
  uint64_t* full_b = empty_a + kMaxS;         // [SB] even CTA: dequant warps of both CTAs
  uint64_t* empty_b = full_b + kMaxS;         // [SB] MMA commit (both CTAs)
  uint64_t* pfull = empty_b + kMaxS;          // [kRingSlots] bulk-copy bytes
  uint64_t* pempty = pfull + kRingSlots;      // [kRingSlots] dequant warps
  uint64_t* acc_full = pempty + kRingSlots;   // MMA commit (both CTAs)
  uint64_t* acc_empty = acc_full + 1;         // even CTA: epilogue warps of both CTAs
  uint64_t* drain = acc_empty + 1;            // MMA commit (both CTAs)
  volatile uint32_t* flags = reinterpret_cast<volatile uint32_t*>(drain + 1);  // [0] abort
  uint32_t* tmem_slot = const_cast<uint32_t*>(flags) + 4;
  uint32_t* pmeta = tmem_slot + 4;            // [kRingSlots][4]: ring offset, counts, list bytes, part-0 bytes
  uint32_t* dtab = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(bars) + 512);  // decoder table
  uint4* smeta = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(bars) + 1024);      // [2][kMetaChunk][2]

  const mtc_stream_desc& s = p.s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = tc::cluster_rank();
  const int cid = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;

  if (tid == 0) {
    for (int i = 0; i < p.SA; ++i) {
      mbar_init(&full_a[i], 1);
      mbar_init(&empty_a[i], 1);
    }
    for (int i = 0; i < p.SB; ++i) {
      mbar_init(&full_b[i], 2 * kDeqWarps);
      mbar_init(&empty_b[i], 1);
    }
    for (int i = 0; i < kRingSlots; ++i) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], kDeqWarps);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * kEpiWarps);
    mbar_init(drain, 1);
    flags[0] = 0;
    tc::fence_mbarrier_init_cluster();
  }
  if (warp == 0) load_dec_table(dtab, lane);
  if (warp == kMmaWarp) tc::tmem_alloc_pair(tmem_slot, 512);
  tc::fence_before();
  tc::cluster_sync();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProdWarp) {
    // ---------------------------------------------------------------- A producer
    // This CTA's A rows are rows 256 * rank .. + 255 of the pair tile, one
    // box: the first 128 feed accumulator 0, the next 128 accumulator 1 (the
    // pair MMA takes accumulator rows 0-127 from the even CTA and 128-255
    // from the odd one); the bytes count on the even CTA's barrier.
    if (lane == 0) {
      uint32_t it = 0;
      const int n_items = item_count(p, cid, n_clusters);
      for (int ii = 0; ii < n_items && !flags[0]; ++ii) {
        const Item w = item_of(p, cid, n_clusters, ii);
        const int mblk = w.tile / p.n_bands;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int sa = it % p.SA;
          if (it >= (uint32_t)p.SA && !mbar_wait(&empty_a[sa], ((it / p.SA) & 1) ^ 1, p.timeout_ns)) {
            flags[0] = 1;
            break;
          }
          if (flags[0]) break;
          if (rank == 0) mbar_expect_tx(&full_a[sa], 2 * kABytes);
          const uint32_t bar = tc::mapa(&full_a[sa], 0);
          tc::tma_load_2d_pair(sA + sa * kABytes, &tmap_x, kb * BK, mblk * CBM + 256 * (int)rank, bar);
        }
      }
      if (flags[0]) flag(p.status, MTC_STATUS_TIMEOUT);
    }
  } else if (warp == kPackWarp) {
    // ---------------------------------------------------------------- packed producer
    // The whole warp loads the metadata (record ranges, entry counts, list
    // offset) of 32 sub-stages at a time into shared memory, one chunk ahead
    // of lane 0, which issues the bulk copies; so lane 0 never waits on a
    // global load.
    // chunks of kMetaChunk sub-stages: ceil(nkb / kMetaChunk) per whole
    // tile, then those of the tail piece
    const int n_reg = regular_items(p, cid, n_clusters);
    const int chunks_per_tile = (p.nkb + kMetaChunk - 1) / kMetaChunk;
    const Item tail = item_of(p, cid, n_clusters, n_reg);  // meaningful when cid < n_pieces
    const int tail_chunks = cid < p.n_pieces ? (tail.kb1 - tail.kb0 + kMetaChunk - 1) / kMetaChunk : 0;
    const int n_chunks = n_reg * chunks_per_tile + tail_chunks;
    // chunk q -> its item and k-block range [kb0, kb1)
    auto chunk_of = [&](int q, int& tile, int& kb0, int& kb1) {
      if (q < n_reg * chunks_per_tile) {
        tile = cid + (q / chunks_per_tile) * n_clusters;
        kb0 = (q % chunks_per_tile) * kMetaChunk;
        kb1 = min(p.nkb, kb0 + kMetaChunk);
      } else {
        tile = tail.tile;
        kb0 = tail.kb0 + (q - n_reg * chunks_per_tile) * kMetaChunk;
        kb1 = min(tail.kb1, kb0 + kMetaChunk);
      }
    };
    uint4 nxt0, nxt1;
    auto load_chunk = [&](int q) {
      int tile = 0, kc0 = 0, kc1 = 0;
      if (q < n_chunks) chunk_of(q, tile, kc0, kc1);
      const int band = tile % p.n_bands;
      const int kb = kc0 + lane;
      nxt0 = make_uint4(0u, 0u, 0u, 0u);
      nxt1 = make_uint4(0u, 0u, 0u, 0u);
      if (q < n_chunks && kb < kc1) {
        const size_t sub = (size_t)(2 * band + (int)rank) * p.nkb + kb;
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
    uint32_t it = 0;
    uint32_t oldest = 0;                              // oldest sub-stage not yet known to be released
    unsigned long long ring_head = 0;                 // monotonic byte position in the ring
    uint32_t head_off = 0;                            // ring_head modulo the ring size
    unsigned long long ring_start[kRingSlots];        // start position of each sub-stage in flight
    for (int q = 0; q < n_chunks; ++q) {
      load_chunk(q + 1);                              // in flight while lane 0 issues chunk q
      if (lane == 0) {
        int ctile, kb0, kb1;
        chunk_of(q, ctile, kb0, kb1);
        for (int kb = kb0; kb < kb1 && !flags[0]; ++kb, ++it) {
          // The sub-stage goes to the byte ring as one contiguous piece:
          // descriptors (128 B) | work list | row-0 records | row-1 records.
          // Its ring range must be free: release older sub-stages (FIFO)
          // until it is.
          const uint4 rg = smeta[2 * ((q & 1) * kMetaChunk + (kb - kb0))];  // bytes: image, list, row 0, row 1
          const uint4 mc = smeta[2 * ((q & 1) * kMetaChunk + (kb - kb0)) + 1];  // counts, image offset
          const uint32_t cnt = mc.x;
          const uint32_t need = rg.x;
          if (need > p.ring_bytes || ((need | mc.y) & 15u)) {
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
          pmeta[4 * ps + 0] = start;
          pmeta[4 * ps + 1] = cnt;
          pmeta[4 * ps + 2] = rg.y;
          pmeta[4 * ps + 3] = rg.z;
          // the whole sub-stage image in one bulk copy
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
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = tc::idesc_f16_f32(256, BN);
      uint32_t it = 0, tcount = 0;
      const int n_items = item_count(p, cid, n_clusters);
      for (int ii = 0; ii < n_items && !flags[0]; ++ii, ++tcount) {
        const Item w = item_of(p, cid, n_clusters, ii);
        if (tcount > 0 && !mbar_wait(acc_empty, (tcount - 1) & 1, p.timeout_ns)) {
          flags[0] = 1;
          break;
        }
        tc::fence_after();
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int sa = it % p.SA, sb = it % p.SB;
          if (!mbar_wait(&full_a[sa], (it / p.SA) & 1, p.timeout_ns) ||
              !mbar_wait(&full_b[sb], (it / p.SB) & 1, p.timeout_ns)) {
            flags[0] = 1;
            break;
          }
          tc::fence_after();
          const uint32_t a0 = smem_u32(sA + sa * kABytes);
          const uint32_t b0 = smem_u32(sB + sb * kBBytes);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j) {
            const uint64_t bd = tc::smem_desc_k_sw128(b0 + 32 * j);
            const uint32_t acc = (kb > w.kb0 || j > 0) ? 1u : 0u;
            tc::mma_f16_ss_pair(tmem, tc::smem_desc_k_sw128(a0 + 32 * j), bd, idesc, acc);
            tc::mma_f16_ss_pair(tmem + 256, tc::smem_desc_k_sw128(a0 + kAHalf + 32 * j), bd, idesc, acc);
          }
          tc::commit_pair(&empty_a[sa]);
          tc::commit_pair(&empty_b[sb]);
        }
        if (flags[0]) break;
        tc::commit_pair(acc_full);
      }
      // make sure no MMA is still reading shared memory or writing TMEM
      tc::commit_pair(drain);
      (void)mbar_wait(drain, 0, 100000000ull);
      if (flags[0]) flag(p.status, MTC_STATUS_TIMEOUT);
    }
  } else if (warp >= kDeqWarp0) {
    // ---------------------------------------------------------------- dequant
    // Two groups of eight warps take alternate sub-stages; each dequantises
    // its CTA's half band into a W tile (dequant_substage).
    const int grp = (warp - kDeqWarp0) / kDeqWarps;
    const int dw = (warp - kDeqWarp0) % kDeqWarps;
    const uint32_t full_b_remote = tc::mapa(full_b, 0);
    uint32_t it = 0;
    const int n_items = item_count(p, cid, n_clusters);
    for (int ii = 0; ii < n_items && !flags[0]; ++ii) {
      const Item w = item_of(p, cid, n_clusters, ii);
      for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
        if ((int)(it % kDeqGroups) != grp) continue;  // the other group's stage
        const int sb = it % p.SB, ps = it % kRingSlots;
        bool ok = mbar_wait(&pfull[ps], (it / kRingSlots) & 1, p.timeout_ns);
        if (ok && it >= (uint32_t)p.SB) ok = mbar_wait(&empty_b[sb], ((it / p.SB) & 1) ^ 1, p.timeout_ns);
        if (!__all_sync(0xffffffffu, ok)) {  // warp-uniform: the dequant uses whole-warp shuffles
          flags[0] = 1;
          break;
        }
        dequant_substage(sB + sb * kBBytes, sP + pmeta[4 * ps], pmeta[4 * ps + 1], pmeta[4 * ps + 2],
                         pmeta[4 * ps + 3], 2 * kb + 1 >= s.tk, dtab, s.scale_words, p.pow2e, dw, lane,
                         tid - (kDeqWarp0 + grp * kDeqWarps) * 32, (int)((it >> 1) * 3u));
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(&full_b[sb]);
          else tc::mbar_arrive_cluster(full_b_remote + 8u * sb);
          mbar_arrive(&pempty[ps]);
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 0-3)
    // This CTA's TMEM holds its pair-tile rows 256 * rank + 128 * half + lane
    // (half = accumulator).
    const uint32_t acc_empty_remote = tc::mapa(acc_empty, 0);
    uint32_t tcount = 0;
    const int n_items = item_count(p, cid, n_clusters);
    for (int ii = 0; ii < n_items && !flags[0]; ++ii, ++tcount) {
      const Item w = item_of(p, cid, n_clusters, ii);
      const int mblk = w.tile / p.n_bands, band = w.tile % p.n_bands;
      // a tail piece writes its partial sums (CBM x BN, row-major) instead
      const bool piece = w.piece >= 0;
      float* const ybase = piece ? p.part + (size_t)w.piece * CBM * BN - ((long long)mblk * CBM * BN + band * BN)
                                 : p.Y;
      const long long ld = piece ? BN : p.ldy;
      if (!mbar_wait(acc_full, tcount & 1, p.timeout_ns)) {
        flags[0] = 1;
        break;
      }
      tc::fence_after();
      // 16x256b loads give each lane quad 8 consecutive columns of one row,
      // so every float2 store instruction writes 8 full 32-byte sectors.
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
#pragma unroll 1
        for (int lb = 0; lb < 32; lb += 16) {
          const int m0 = mblk * CBM + 256 * (int)rank + 128 * half + 32 * warp + lb + (lane >> 2);
          // (the epilogue instance loads 32 columns at a time: fewer live
          // registers next to the activation's)
          constexpr int RW = EPI ? 4 : 8;
#pragma unroll 1
          for (int c = 0; c < BN; c += 8 * RW) {
            uint32_t v[4 * RW];
            if constexpr (EPI)
              tc::tmem_ld_16x256b_x4(tmem + ((uint32_t)(32 * warp + lb) << 16) + half * 256 + c, v);
            else
              tc::tmem_ld_16x256b_x8(tmem + ((uint32_t)(32 * warp + lb) << 16) + half * 256 + c, v);
            const int nb = band * BN + c + 2 * (lane & 3);
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
              const int m = m0 + 8 * hr;
              if (m >= p.M) continue;
              float* y = ybase + (long long)m * ld;
#pragma unroll
              for (int r = 0; r < RW; ++r) {
                const int n = nb + 8 * r;
                float a = __uint_as_float(v[4 * r + 2 * hr]) * p.inv_pow2e;
                float b = __uint_as_float(v[4 * r + 2 * hr + 1]) * p.inv_pow2e;
                if constexpr (EPI) {
                  if (!piece) {
                    if (n < s.N) a = epi_apply(p.ep, a, n);
                    if (n + 1 < s.N) b = epi_apply(p.ep, b, n + 1);
                  }
                }
                if ((p.vec2 || piece) && n + 1 < s.N) {
                  *reinterpret_cast<float2*>(y + n) = make_float2(a, b);
                } else {
                  if (n < s.N) y[n] = a;
                  if (n + 1 < s.N) y[n + 1] = b;
                }
              }
            }
          }
        }
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(acc_empty);
        else tc::mbar_arrive_cluster(acc_empty_remote);
      }
    }
    if (flags[0]) flag(p.status, MTC_STATUS_TIMEOUT);
  }

  // Both CTAs are done with each other's shared memory and TMEM only when
  // both reach this point (the even CTA's MMA thread has drained).
  tc::fence_before();
  tc::cluster_sync();
  if (warp == kMmaWarp) {
    tc::fence_after();
    tc::tmem_dealloc_pair(tmem, 512);
  }
}

// The split tail's partial sums: for the n_tail tiles t_main.., output
// Y[m][n] = epilogue(sum over s of part[t split + s][m - m0][n - n0]), the
// pieces added in order (deterministic).  One thread per four columns.
__global__ void __launch_bounds__(256) prefill_tail_reduce(const float* __restrict__ part, int t_main, int split,
                                                           int n_tail, int n_bands, int M, int N,
                                                           float* __restrict__ Y, long long ldy, int vec4, Epi ep) {
  constexpr int C4 = BN / 4;
  const long long total = (long long)n_tail * CBM * C4;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int c4 = (int)(idx % C4), r = (int)((idx / C4) % CBM), t = (int)(idx / ((long long)C4 * CBM));
    const int tile = t_main + t, mblk = tile / n_bands, band = tile % n_bands;
    const int m = mblk * CBM + r, n = band * BN + 4 * c4;
    if (m >= M || n >= N) continue;
    const float4* src = reinterpret_cast<const float4*>(part + ((size_t)t * split * CBM + r) * BN) + c4;
    float4 a = src[0];
    for (int sp = 1; sp < split; ++sp) {
      const float4 b = src[(size_t)sp * CBM * C4];
      a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
    }
    float v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (n + i < N) v[i] = epi_apply(ep, v[i], n + i);
    float* y = Y + (long long)m * ldy + n;
    if (vec4 && n + 3 < N) {
      *reinterpret_cast<float4*>(y) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      for (int i = 0; i < 4 && n + i < N; ++i) y[i] = v[i];
    }
  }
}

// Xp[m][k] = fp16(X[m][pr[k]]), k < K; zero up to Kp.  One CTA per row.
__global__ void __launch_bounds__(256) gather_x_kernel(const float* __restrict__ X, long long ldx, int K, int Kp,
                                                       const int32_t* __restrict__ pr, __half* __restrict__ Xp,
                                                       uint32_t* status) {
  extern __shared__ float row[];
  const int m = blockIdx.x;
  const float* x = X + (long long)m * ldx;
  for (int k = threadIdx.x; k < K; k += blockDim.x) row[k] = x[k];
  __syncthreads();
  uint32_t bad = 0;
  __half* out = Xp + (long long)m * Kp;
  for (int k = 2 * threadIdx.x; k < Kp; k += 2 * blockDim.x) {
    float a = 0.f, b = 0.f;
    if (k < K) a = row[pr ? pr[k] : k];
    if (k + 1 < K) b = row[pr ? pr[k + 1] : k + 1];
    if (!(fabsf(a) <= 65504.0f) || !(fabsf(b) <= 65504.0f)) bad = 1;
    *reinterpret_cast<__half2*>(out + k) = __floats2half2_rn(a, b);
  }
  if (bad) flag(status, MTC_STATUS_X_RANGE);
}

// Y[m][j] = row_m[pos[j]], where row_m is the concatenation of nseg segments
// src[g * seg_stride + m * ldp + (0 .. seg_len)].  One CTA per row; the row
// is staged in shared memory so reads and writes are both coalesced.  With
// one segment and pos = inverse column permutation this is Y[:, pc] = Yp;
// with one segment per rank it assembles all-gathered column shards.
__global__ void __launch_bounds__(512) permute_rows_kernel(const float* __restrict__ src, long long seg_stride,
                                                           long long ldp, int nseg, int seg_len,
                                                           const int32_t* __restrict__ pos, int N,
                                                           float* __restrict__ Y, long long ldy, const Epi ep) {
  extern __shared__ float row[];
  const int m = blockIdx.x;
  for (int g = 0; g < nseg; ++g) {
    const float* sg = src + g * seg_stride + (long long)m * ldp;
    for (int c = threadIdx.x; c < seg_len; c += blockDim.x) row[g * seg_len + c] = sg[c];
  }
  __syncthreads();
  float* dst = Y + (long long)m * ldy;
  for (int j = threadIdx.x; j < N; j += blockDim.x) dst[j] = epi_apply(ep, row[pos[j]], j);
}

// Persistent row kernels for the HBM-bound gather / scatter around the GEMM:
// each CTA takes rows blockIdx.x, + gridDim.x, ...; a row arrives by bulk
// copy into one of two shared-memory buffers while the previous row is
// written out, and every thread keeps the source index of its output
// elements in registers (the permutation is the same for every row).
constexpr int kRowThreads = 512;
constexpr int kRowNJ = 32;  // most output elements (permute) or pairs (gather) per thread per row

__device__ __forceinline__ bool row_wait_all(uint64_t* bar, uint32_t parity) {
  const bool ok = mbar_wait(bar, parity, 2000000000ull);
  return __syncthreads_and(ok) != 0;
}

template <int NJ>
__global__ void __launch_bounds__(kRowThreads)
    permute_rows_bulk_kernel(const float* __restrict__ src, long long seg_stride, long long ldp, int nseg,
                             int seg_len, const int32_t* __restrict__ pos, int N, int M, float* __restrict__ Y,
                             long long ldy, int buf_floats, const Epi ep, uint32_t* status) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  float* buf = reinterpret_cast<float*>(smem_raw);  // [2][buf_floats]
  uint64_t* bars = reinterpret_cast<uint64_t*>(buf + 2 * buf_floats);
  const int tid = threadIdx.x;
  int pj[NJ];
#pragma unroll
  for (int i = 0; i < NJ; ++i) {
    const int j = tid + i * kRowThreads;
    pj[i] = j < N ? pos[j] : 0;
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  const uint32_t row_bytes = (uint32_t)nseg * (uint32_t)seg_len * 4u;
  auto issue = [&](int m, int b) {
    mbar_expect_tx(&bars[b], row_bytes);
    for (int g = 0; g < nseg; ++g)
      bulk_g2s(buf + b * buf_floats + g * seg_len, src + g * seg_stride + (long long)m * ldp, (uint32_t)seg_len * 4u,
               &bars[b]);
  };
  if (tid == 0 && (int)blockIdx.x < M) issue(blockIdx.x, 0);
  uint32_t r = 0;
  int issued = (int)blockIdx.x < M ? 1 : 0;
  for (int m = blockIdx.x; m < M; m += gridDim.x, ++r) {
    const int b = r & 1;
    if (m + (int)gridDim.x < M) {
      if (tid == 0) issue(m + gridDim.x, b ^ 1);  // buffer b ^ 1 was released by the last __syncthreads
      ++issued;
    }
    if (!row_wait_all(&bars[b], (r >> 1) & 1)) {
      if (tid == 0) {
        flag(status, MTC_STATUS_TIMEOUT);
        // let copies still in flight land before the CTA exits
        for (uint32_t q = r; q < (uint32_t)issued; ++q) (void)mbar_wait(&bars[q & 1], (q >> 1) & 1, 10000000ull);
      }
      return;
    }
    const float* row = buf + b * buf_floats;
    float* dst = Y + (long long)m * ldy;
    if (ep.bias || ep.act) {
#pragma unroll
      for (int i = 0; i < NJ; ++i) {
        const int j = tid + i * kRowThreads;
        if (j < N) dst[j] = epi_apply(ep, row[pj[i]], j);
      }
    } else {
#pragma unroll
      for (int i = 0; i < NJ; ++i) {
        const int j = tid + i * kRowThreads;
        if (j < N) dst[j] = row[pj[i]];
      }
    }
    __syncthreads();
  }
}

// Xp[m][k] = fp16(X[m][pr[k]]) for k < K, zero up to Kp; pairs of k per thread.
template <int NJ>
__global__ void __launch_bounds__(kRowThreads)
    gather_x_bulk_kernel(const float* __restrict__ X, long long ldx, int K, int Kp, const int32_t* __restrict__ pr,
                         int M, __half* __restrict__ Xp, int buf_floats, uint32_t* status) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  float* buf = reinterpret_cast<float*>(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(buf + 2 * buf_floats);
  const int tid = threadIdx.x;
  int p0[NJ], p1[NJ];
#pragma unroll
  for (int i = 0; i < NJ; ++i) {
    const int k = 2 * (tid + i * kRowThreads);
    p0[i] = k < K ? (pr ? pr[k] : k) : -1;
    p1[i] = k + 1 < K ? (pr ? pr[k + 1] : k + 1) : -1;
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int m, int b) {
    mbar_expect_tx(&bars[b], (uint32_t)K * 4u);
    bulk_g2s(buf + b * buf_floats, X + (long long)m * ldx, (uint32_t)K * 4u, &bars[b]);
  };
  if (tid == 0 && (int)blockIdx.x < M) issue(blockIdx.x, 0);
  uint32_t r = 0, bad = 0;
  int issued = (int)blockIdx.x < M ? 1 : 0;
  for (int m = blockIdx.x; m < M; m += gridDim.x, ++r) {
    const int b = r & 1;
    if (m + (int)gridDim.x < M) {
      if (tid == 0) issue(m + gridDim.x, b ^ 1);
      ++issued;
    }
    if (!row_wait_all(&bars[b], (r >> 1) & 1)) {
      if (tid == 0) {
        flag(status, MTC_STATUS_TIMEOUT);
        for (uint32_t q = r; q < (uint32_t)issued; ++q) (void)mbar_wait(&bars[q & 1], (q >> 1) & 1, 10000000ull);
      }
      return;
    }
    const float* row = buf + b * buf_floats;
    __half* out = Xp + (long long)m * Kp;
#pragma unroll
    for (int i = 0; i < NJ; ++i) {
      const int k = 2 * (tid + i * kRowThreads);
      if (k < Kp) {
        const float a = p0[i] >= 0 ? row[p0[i]] : 0.f;
        const float c = p1[i] >= 0 ? row[p1[i]] : 0.f;
        if (!(fabsf(a) <= 65504.0f) || !(fabsf(c) <= 65504.0f)) bad = 1;
        *reinterpret_cast<__half2*>(out + k) = __floats2half2_rn(a, c);
      }
    }
    __syncthreads();
  }
  if (bad) flag(status, MTC_STATUS_X_RANGE);
}

int row_grid(const void* kernel, size_t smem, int M) {
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kRowThreads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const long long g = (long long)sms * per_sm;
  return (int)(M < g ? M : g);
}

int launch_permute_rows(const float* src, long long seg_stride, long long ldp, int nseg, int seg_len,
                        const int32_t* pos, int N, int M, float* Y, long long ldy, const EpiArg& epa,
                        uint32_t* status, cudaStream_t st) {
  const Epi ep{epa.bias, epa.act};
  const size_t row = (size_t)nseg * seg_len * 4;
  const size_t buf_floats = ((size_t)nseg * seg_len + 31) & ~(size_t)31;
  const size_t sm2 = 2 * buf_floats * 4 + 64;
  const bool bulk = N <= kRowThreads * kRowNJ && sm2 <= 227 * 1024 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                    (seg_stride & 3) == 0 && (ldp & 3) == 0 && (seg_len & 3) == 0;
  if (bulk) {
    auto go = [&](auto kernel) -> int {
      MTC_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2),
                     "permute: smem attribute");
      const int grid = row_grid(reinterpret_cast<const void*>(kernel), sm2, M);
      kernel<<<grid, kRowThreads, sm2, st>>>(src, seg_stride, ldp, nseg, seg_len, pos, N, M, Y, ldy, (int)buf_floats,
                                             ep, status);
      MTC_CHECK_LAUNCH("permute_rows");
      return MTC_OK;
    };
    if (N <= kRowThreads * 4) return go(permute_rows_bulk_kernel<4>);
    if (N <= kRowThreads * 8) return go(permute_rows_bulk_kernel<8>);
    if (N <= kRowThreads * 16) return go(permute_rows_bulk_kernel<16>);
    return go(permute_rows_bulk_kernel<32>);
  }
  MTC_REQUIRE(row <= 227 * 1024, "permute: a staged row of %zu bytes exceeds shared memory", row);
  if (row > 48 * 1024)
    MTC_CHECK_CUDA(cudaFuncSetAttribute(permute_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)row),
                   "permute: smem attribute");
  permute_rows_kernel<<<M, 512, row, st>>>(src, seg_stride, ldp, nseg, seg_len, pos, N, Y, ldy, ep);
  MTC_CHECK_LAUNCH("permute_rows");
  return MTC_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

struct PrefillPlan {
  int Kp, Np, nkb, n_mblk, n_bands, n_tiles, SA, SB;
  uint32_t ring_bytes;
  size_t smem, xp_bytes, yp_bytes;
  size_t part_bytes;  // partial sums of a split tail: one CBM x BN fp32 block per CTA pair of this device
};

// Compile-time overrides of the pipeline depths (tuning builds only).
#ifndef MTC_PREFILL_SA
#define MTC_PREFILL_SA 0
#endif
#ifndef MTC_PREFILL_SB
#define MTC_PREFILL_SB 0
#endif

bool plan_prefill(const mtc_stream_desc* s, int M, bool permuted, PrefillPlan* pl) {
  pl->Kp = s->tk * kTile;
  pl->Np = s->tn * kTile;
  pl->nkb = (s->tk + 1) / 2;
  pl->n_mblk = (M + CBM - 1) / CBM;
  pl->n_bands = (s->tn + s->band_tiles - 1) / s->band_tiles;
  pl->n_tiles = pl->n_mblk * pl->n_bands;
  const size_t cap = 227 * 1024;
  const size_t fixed = 1024 /*align*/ + 1024 /*barriers, flags, decoder table*/ + 64 * kMetaChunk /*stage metadata*/;
  // Deep A and W pipelines cover the TMA latency and let dequant run ahead
  // of the MMA; the packed byte ring takes the rest and should hold at least
  // two of the largest sub-stages, so the deepest pipelines that leave that
  // much are used.
  const size_t biggest = s->max_stage_bytes ? s->max_stage_bytes : s->max_row_bytes + 4 * 1024 + kDescBytes;
  static const int cand[5][2] = {{4, 4}, {4, 3}, {3, 3}, {3, 2}, {2, 2}};
  int SA = 2, SB = 2;
  for (int c = 0; c < 5; ++c) {
    const size_t used = fixed + (size_t)cand[c][0] * kABytes + (size_t)cand[c][1] * kBBytes;
    if (used + 2 * biggest <= cap || c == 4) {
      SA = cand[c][0];
      SB = cand[c][1];
      break;
    }
  }
  if (MTC_PREFILL_SA > 0) SA = MTC_PREFILL_SA;
  if (MTC_PREFILL_SB > 0) SB = MTC_PREFILL_SB;
  const size_t used = fixed + (size_t)SA * kABytes + (size_t)SB * kBBytes;
  if (used >= cap || SA > kMaxS || SB > kMaxS) return false;
  const size_t ring = (cap - used) & ~(size_t)127;
  if (ring < biggest) return false;
  pl->SA = SA;
  pl->SB = SB;
  pl->ring_bytes = (uint32_t)ring;
  pl->smem = used + ring;
  pl->xp_bytes = ((size_t)M * pl->Kp * 2 + 255) & ~(size_t)255;
  pl->yp_bytes = permuted ? (size_t)M * pl->Np * 4 : 0;
  pl->part_bytes = 0;
  int dev = 0, sms = 0;
  if (pl->nkb >= 4) {
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms >= 4)
      pl->part_bytes = (size_t)(sms / 2) * CBM * BN * 4;
    else
      (void)cudaGetLastError();  // no device here: no split tail, and no error left behind
  }
  return true;
}

}  // namespace

// Xp[m][k] = fp16(X[m][pr[k]]) (zero for K <= k < Kp), m < M: the persistent
// bulk-copy kernel when rows are 16-byte aligned, else one CTA per row.
int launch_gather_x(const float* X, long long ldx, int K, int Kp, const int32_t* row_perm, int M, __half* Xp,
                    uint32_t* status, cudaStream_t st) {
  MTC_REQUIRE((size_t)K * 4 <= 200 * 1024, "gather: K=%d above the 51200 row-staged limit", K);
  const size_t buf_floats = ((size_t)K + 31) & ~(size_t)31;
  const size_t sm2 = 2 * buf_floats * 4 + 64;
  if (Kp <= 2 * kRowThreads * kRowNJ && sm2 <= 227 * 1024 && (reinterpret_cast<uintptr_t>(X) & 15) == 0 &&
      (ldx & 3) == 0 && (K & 3) == 0) {
    auto go = [&](auto kernel) -> int {
      MTC_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2),
                     "gather: smem attribute");
      const int grid = row_grid(reinterpret_cast<const void*>(kernel), sm2, M);
      kernel<<<grid, kRowThreads, sm2, st>>>(X, ldx, K, Kp, row_perm, M, Xp, (int)buf_floats, status);
      MTC_CHECK_LAUNCH("gather_x");
      return MTC_OK;
    };
    if (Kp <= 2 * kRowThreads * 4) return go(gather_x_bulk_kernel<4>);
    if (Kp <= 2 * kRowThreads * 8) return go(gather_x_bulk_kernel<8>);
    if (Kp <= 2 * kRowThreads * 16) return go(gather_x_bulk_kernel<16>);
    return go(gather_x_bulk_kernel<32>);
  }
  const size_t sm = (size_t)K * 4;
  if (sm > 48 * 1024)
    MTC_CHECK_CUDA(cudaFuncSetAttribute(gather_x_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                   "gather: smem attribute");
  gather_x_kernel<<<M, 256, sm, st>>>(X, ldx, K, Kp, row_perm, Xp, status);
  MTC_CHECK_LAUNCH("gather_x");
  return MTC_OK;
}

// TMA descriptor of Xp (fp16 [M][Kp]): box 64 (k) x box_rows, 128-byte swizzle.
int encode_xp_map(CUtensorMap* map, const __half* Xp, int Kp, int M, int box_rows, const char* who) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) {
    set_error("%s: cuTensorMapEncodeTiled unavailable from the driver", who);
    return MTC_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)Kp * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(Xp), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d)", who, (int)r);
    return MTC_ERR_CUDA;
  }
  return MTC_OK;
}

// TMA descriptor of Xp (fp16 [rows][Kp], Kp a multiple of 64) as 64-k blocks:
// dims (k in block, row, k block); a box of (64, rows, nblk) lands as nblk
// consecutive (rows x 128 B) SWIZZLE_128B tiles.
int encode_xp_blocks_map(CUtensorMap* map, const __half* Xp, int Kp, int rows, int nblk, const char* who) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) {
    set_error("%s: cuTensorMapEncodeTiled unavailable from the driver", who);
    return MTC_ERR_CUDA;
  }
  if (Kp % 64) {
    set_error("%s: Xp row length %d is not a multiple of 64", who, Kp);
    return MTC_ERR_INVALID;
  }
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(Kp / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)Kp * 2, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)rows, (cuuint32_t)nblk};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(Xp), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled (3-d) failed (%d)", who, (int)r);
    return MTC_ERR_CUDA;
  }
  return MTC_OK;
}
}  // namespace mtc

using namespace mtc;

extern "C" size_t mtc_prefill_workspace_bytes(const mtc_stream_desc* s, int32_t M, int32_t permuted) {
  PrefillPlan pl;
  if (!s || M <= 0 || !plan_prefill(s, M, permuted != 0, &pl)) return 0;
  return pl.xp_bytes + pl.yp_bytes + pl.part_bytes;
}

namespace {

int check_prefill(const mtc_stream_desc* s, int32_t M, bool permuted, void* ws, size_t ws_bytes, PrefillPlan* pl,
                  const char* who) {
  MTC_REQUIRE(s && ws && s->records && s->tiles && s->row_off, "%s: null pointer argument", who);
  MTC_REQUIRE(M >= 1, "%s: M=%d", who, M);
  MTC_REQUIRE(s->band_tiles * kTile == BN, "%s: stream band width %d tiles, kernel needs %d", who, s->band_tiles,
              BN / kTile);
  MTC_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 255) == 0, "%s: workspace not 256-byte aligned", who);
  MTC_REQUIRE(plan_prefill(s, M, permuted, pl), "%s: a stage of %u bytes does not fit shared memory", who,
              s->max_stage_bytes);
  if (ws_bytes < pl->xp_bytes + pl->yp_bytes) {
    set_error("%s: workspace %zu bytes, need %zu", who, ws_bytes, pl->xp_bytes + pl->yp_bytes);
    return MTC_ERR_WORKSPACE;
  }
  return MTC_OK;
}

}  // namespace

extern "C" int mtc_prefill_gather(const mtc_stream_desc* s, const float* X, int32_t M, int64_t ldx,
                                  const int32_t* row_perm, void* ws, size_t ws_bytes, uint32_t* status,
                                  void* stream) {
  clear_error();
  PrefillPlan pl;
  int rc = check_prefill(s, M, false, ws, ws_bytes, &pl, "mtc_prefill_gather");
  if (rc != MTC_OK) return rc;
  MTC_REQUIRE(X && ldx >= s->K, "mtc_prefill_gather: bad activations");
  return launch_gather_x(X, ldx, s->K, pl.Kp, row_perm, M, static_cast<__half*>(ws), status, as_stream(stream));
}

extern "C" int mtc_prefill_scatter(const mtc_stream_desc* s, int32_t M, const int32_t* col_perm_inv, float* Y,
                                   int64_t ldy, void* ws, size_t ws_bytes, const mtc_epilogue* ep, void* stream) {
  clear_error();
  PrefillPlan pl;
  int rc = check_prefill(s, M, true, ws, ws_bytes, &pl, "mtc_prefill_scatter");
  if (rc != MTC_OK) return rc;
  MTC_REQUIRE(Y && col_perm_inv && ldy >= s->N, "mtc_prefill_scatter: bad output");
  EpiArg epa;
  rc = read_epilogue(ep, &epa, "mtc_prefill_scatter");
  if (rc != MTC_OK) return rc;
  const float* Yp = reinterpret_cast<const float*>(static_cast<const uint8_t*>(ws) + pl.xp_bytes);
  return launch_permute_rows(Yp, 0, pl.Np, 1, s->N, col_perm_inv, s->N, M, Y, ldy, epa, nullptr, as_stream(stream));
}

extern "C" int mtc_permute_rows(const float* src, int64_t seg_stride, int64_t ldp, int32_t nseg, int32_t seg_len,
                                const int32_t* pos, int32_t N, int32_t M, float* Y, int64_t ldy,
                                const mtc_epilogue* ep, void* stream) {
  clear_error();
  MTC_REQUIRE(src && pos && Y && nseg >= 1 && seg_len >= 1 && N >= 1 && M >= 1 && ldy >= N,
              "mtc_permute_rows: bad arguments");
  EpiArg epa;
  const int rc = read_epilogue(ep, &epa, "mtc_permute_rows");
  if (rc != MTC_OK) return rc;
  return launch_permute_rows(src, seg_stride, ldp, nseg, seg_len, pos, N, M, Y, ldy, epa, nullptr, as_stream(stream));
}

extern "C" int mtc_gemm_prefill(const mtc_stream_desc* s, const float* X, int32_t M, int64_t ldx,
                                const int32_t* row_perm, const int32_t* col_perm_inv, float* Y, int64_t ldy,
                                void* ws, size_t ws_bytes, uint32_t* status, const mtc_epilogue* ep, void* stream) {
  clear_error();
  EpiArg epa;
  int rc = read_epilogue(ep, &epa, "mtc_gemm_prefill");
  if (rc != MTC_OK) return rc;
  rc = mtc_prefill_gather(s, X, M, ldx, row_perm, ws, ws_bytes, status, stream);
  if (rc != MTC_OK) return rc;
  rc = mtc_prefill_gemm(s, M, Y, ldy, col_perm_inv != nullptr ? 1 : 0, ws, ws_bytes, status,
                        col_perm_inv != nullptr ? nullptr : ep, stream);
  if (rc != MTC_OK) return rc;
  if (col_perm_inv) return mtc_prefill_scatter(s, M, col_perm_inv, Y, ldy, ws, ws_bytes, ep, stream);
  return MTC_OK;
}

extern "C" int mtc_prefill_gemm(const mtc_stream_desc* s, int32_t M, float* Y, int64_t ldy, int32_t permuted_output,
                                void* ws, size_t ws_bytes, uint32_t* status, const mtc_epilogue* ep, void* stream) {
  clear_error();
  PrefillPlan pl;
  int rc = check_prefill(s, M, permuted_output != 0, ws, ws_bytes, &pl, "mtc_prefill_gemm");
  if (rc != MTC_OK) return rc;
  EpiArg epa;
  rc = read_epilogue(ep, &epa, "mtc_prefill_gemm");
  if (rc != MTC_OK) return rc;
  MTC_REQUIRE(!(permuted_output && ep), "mtc_prefill_gemm: the epilogue of a permuted output goes to the scatter");
  MTC_REQUIRE(s->stage_images && s->stage_counts && s->stage_offsets && s->stage_ranges && s->max_stage_bytes,
              "mtc_prefill_gemm: stage work lists missing (run mtc_repack_stage_plan and mtc_repack_stage_fill)");
  MTC_REQUIRE(permuted_output || (Y && ldy >= s->N), "mtc_prefill_gemm: bad output");
  const bool col_perm_inv = permuted_output != 0;
  cudaStream_t st = as_stream(stream);
  __half* Xp = static_cast<__half*>(ws);
  float* Yp = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + pl.xp_bytes);
  CUtensorMap tmap;
  rc = encode_xp_map(&tmap, Xp, pl.Kp, M, 256, "mtc_prefill_gemm");
  if (rc != MTC_OK) return rc;
  PrefillParams p;
  p.s = *s;
  p.M = M;
  p.Y = col_perm_inv ? Yp : Y;
  p.ldy = col_perm_inv ? pl.Np : ldy;
  p.status = status;
  p.n_bands = pl.n_bands;
  p.n_tiles = pl.n_tiles;
  p.nkb = pl.nkb;
  p.vec2 = ((p.ldy & 1) == 0 && (reinterpret_cast<uintptr_t>(p.Y) & 7) == 0) ? 1 : 0;
  p.SA = pl.SA;
  p.SB = pl.SB;
  p.ring_bytes = pl.ring_bytes;
  p.pow2e = ldexpf(1.0f, s->exp2);
  p.inv_pow2e = ldexpf(1.0f, -s->exp2);
  p.timeout_ns = wait_limit_ns();
  p.ep = Epi{epa.bias, epa.act};
  const bool with_ep = epa.bias || epa.act;
  auto kernel = with_ep ? prefill_kernel<true> : prefill_kernel<false>;
  MTC_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem),
                 "mtc_prefill_gemm: smem attribute");
  // CTA pairs: one cluster of two CTAs per pair tile, as many clusters as
  // can be resident at once (persistent; each loops over tiles)
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int max_clusters = 0;
  cfg.gridDim = dim3(2, 1, 1);
  MTC_CHECK_CUDA(cudaOccupancyMaxActiveClusters(&max_clusters, kernel, &cfg),
                 "mtc_prefill_gemm: cluster occupancy");
  MTC_REQUIRE(max_clusters >= 1, "mtc_prefill_gemm: no CTA pair of %zu bytes of shared memory fits", pl.smem);
  int P = max_clusters;
  if (s->max_sms >= 2 && P > (int)(s->max_sms / 2)) P = (int)(s->max_sms / 2);
  // Wave quantisation: the tiles beyond the last whole wave of P pairs
  // would leave most pairs idle for a whole tile time.  When they fill at
  // most half a wave they are cut along K into pieces spread over the pairs
  // (at least two k blocks each), and prefill_tail_reduce adds the pieces.
  const int R = pl.n_tiles >= P ? pl.n_tiles % P : pl.n_tiles;
  int S = R > 0 ? P / R : 0;
  if (S > pl.nkb / 2) S = pl.nkb / 2;
  if (S > 16) S = 16;
  const size_t avail = ws_bytes - pl.xp_bytes - pl.yp_bytes;
  const size_t piece_bytes = (size_t)CBM * BN * 4;
  if (S >= 2 && (size_t)R * S * piece_bytes <= avail) {
    p.t_main = pl.n_tiles - R;
    p.split = S;
    p.n_pieces = R * S;
    p.part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + pl.xp_bytes + pl.yp_bytes);
  } else {
    p.t_main = pl.n_tiles;
    p.split = 1;
    p.n_pieces = 0;
    p.part = nullptr;
  }
  int clusters = p.t_main > 0 ? (p.t_main < P ? p.t_main : P) : 0;
  if (p.n_pieces > clusters) clusters = p.n_pieces;
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  MTC_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kernel, tmap, p), "mtc_prefill_gemm: launch");
  MTC_CHECK_LAUNCH("mtc_prefill_gemm");
  if (p.n_pieces > 0) {
    const int n_tail = p.n_pieces / p.split;
    const long long threads = (long long)n_tail * CBM * (BN / 4);
    const int grid = (int)((threads + 255) / 256);
    const int vec4 = ((p.ldy & 3) == 0 && (reinterpret_cast<uintptr_t>(p.Y) & 15) == 0) ? 1 : 0;
    prefill_tail_reduce<<<grid, 256, 0, st>>>(p.part, p.t_main, p.split, n_tail, p.n_bands, M, s->N, p.Y, p.ldy,
                                              vec4, with_ep ? p.ep : Epi{nullptr, 0});
    MTC_CHECK_LAUNCH("mtc_prefill_gemm: tail reduce");
  }
  return MTC_OK;
}
