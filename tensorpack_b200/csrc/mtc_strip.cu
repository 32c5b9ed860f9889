// Strip-stream decode GEMM for M <= 4: Y[:, pc] = X[:, pr] @ Wp.
//
// Replaces, for decode-sized M, the reference's packed GEMM
// (mtc/kernels/gemm.py:124-210, 541-574) and the gather / scatter of MTC-QT-P
// inference (mtc/core/permutation.py:15-21).  The stream layout and the lane
// arithmetic are in mtc_strip.cuh.
//
// Execution follows a static schedule built on the host
// (mtc_strip_schedule): strips are dealt to CTAs by estimated decode cost,
// and each CTA's batch records are cut into one contiguous range per warp.
// A warp streams its range through a ring of shared-memory slots (lane 0
// issues one cp.async.bulk per batch record, completion on an mbarrier; the
// first copies go out before the activations are gathered), keeps its mma
// accumulators in registers across the batches of a strip, and flushes the
// strip's partial sums into a shared-memory slot when its part of the strip
// ends.  After a CTA barrier the CTA adds each strip's slots in slot order,
// applies the epilogue and writes Y[:, pc].  No global scratch, counters or
// atomics; the result is deterministic.
//
// Every mbarrier wait is bounded (globaltimer); a timeout sets
// MTC_STATUS_TIMEOUT, the warp waits (bounded) for its own copies in flight,
// and the CTA skips its output.
#include "mtc_common.cuh"
#include "mtc_internal.h"
#include "mtc_strip.cuh"

namespace mtc {
namespace {

using namespace strip;

constexpr int kMaxSlots = 3;

struct StripParams {
  const uint8_t* stream;
  unsigned long long stream_bytes;
  const uint32_t* work;       // [2 n_work]: {byte offset, (bytes / 16) | slot << 12 | flush << 31}
  const uint32_t* warp_work;  // [n_cta n_warps + 1]
  const uint32_t* red;        // [3 n_red]: {strip, first slot, slot count}
  const uint32_t* cta_red;    // [n_cta + 1]
  int n_strips, K, N, kpad;
  float inv_pow2e;
  const float* X;
  long long ldx;
  int M;
  const int32_t* pr;
  const int32_t* pc;
  float* Y;
  long long ldy;
  uint32_t* status;
  Epi ep;
  unsigned long long timeout_ns;
  uint32_t withhold;      // diagnostic: bytes expected but never copied on each warp's first batch
  int staged;             // X rows and pr arrive by bulk copy and are permuted in shared memory
  int nw, ns, max_slots;  // warps, slots per warp, partial-sum slots per CTA
  uint32_t slot_bytes;
  uint32_t off_x, off_scr, off_part, off_slots;  // shared-memory layout
};

__device__ __forceinline__ void mma_f16(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// A run of `run` identical full steps (the count sits in the run's first
// descriptor): the step size and every lane offset are constants, so the loop
// body is the decode and the two MMAs.
template <int C, bool GROUP, int MT>
__device__ __forceinline__ void full_run(int run, const uint8_t*& st, int lane, const uint16_t* x16, int kpad,
                                         float acc1[MT][4], float acc2[MT][4]) {
  constexpr int BYTES = GROUP ? strip::pad16(strip::pad16(32) + 32 * (prim_bytes(C) + sec_bytes(C)))
                              : strip::pad16(strip::pad16(128) + 32 * (prim_bytes(C) + sec_bytes(C)));
#pragma unroll 2
  for (int r = 0; r < run; ++r) {
    uint32_t a[8], b[MT][2];
    lane_fast<C, GROUP, true, MT>(st, 0, 0, lane, x16, kpad, a, b);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      mma_f16(acc1[m], a[0], a[1], a[2], a[3], b[m][0], b[m][1]);
      mma_f16(acc2[m], a[4], a[5], a[6], a[7], b[m][0], b[m][1]);
    }
    st += BYTES;
  }
}

template <int C, bool GROUP, int MT>
__device__ __forceinline__ void partial_step(const uint8_t* st, int n0, int n1, int lane, const uint16_t* x16,
                                             int kpad, float acc1[MT][4], float acc2[MT][4]) {
  uint32_t a[8], b[MT][2];
  lane_fast<C, GROUP, false, MT>(st, n0, n1, lane, x16, kpad, a, b);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    mma_f16(acc1[m], a[0], a[1], a[2], a[3], b[m][0], b[m][1]);
    mma_f16(acc2[m], a[4], a[5], a[6], a[7], b[m][0], b[m][1]);
  }
}

// Wide group steps (streams built with kWide): lane = (group, k half), both
// quartets; four MMAs share the B fragment.  acc[j] holds columns 2j, 2j + 1
// of the strip on every quad's diagonal.
template <int C, bool FULL, int MT>
__device__ __forceinline__ void wide_step(const uint8_t* st, int n, int lane, const uint16_t* x16, int kpad,
                                          float accw[4][MT][4]) {
  uint32_t a0[8], a1[8], b[MT][2];
  lane_wide<C, FULL, MT>(st, n, lane, x16, kpad, a0, a1, b);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    mma_f16(accw[0][m], a0[0], a0[1], a0[2], a0[3], b[m][0], b[m][1]);
    mma_f16(accw[1][m], a0[4], a0[5], a0[6], a0[7], b[m][0], b[m][1]);
    mma_f16(accw[2][m], a1[0], a1[1], a1[2], a1[3], b[m][0], b[m][1]);
    mma_f16(accw[3][m], a1[4], a1[5], a1[6], a1[7], b[m][0], b[m][1]);
  }
}
template <int C, int MT>
__device__ __forceinline__ void wide_run(int run, const uint8_t*& st, int lane, const uint16_t* x16, int kpad,
                                         float accw[4][MT][4]) {
  constexpr int BYTES = strip::pad16(64 + 64 * (prim_bytes(C) + sec_bytes(C)));
#pragma unroll 2
  for (int r = 0; r < run; ++r) {
    wide_step<C, true, MT>(st, 16, lane, x16, kpad, accw);
    st += BYTES;
  }
}

// Accumulators of one warp: acc1 / acc2 hold columns (0, 1) / (2, 3) of the
// lane's quartet on every quad's diagonal (narrow steps), accw[j] columns
// 2j, 2j + 1 of the strip (wide group steps), gacc the generic lanes' fp32
// products by column of the lane's quartet.
template <int MT, bool WIDE>
struct Acc {
  float acc1[MT][4], acc2[MT][4], gacc[MT][4];
  float accw[WIDE ? 4 : 1][MT][4];
  bool gen;
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc1[m][r] = acc2[m][r] = gacc[m][r] = 0.0f;
    if constexpr (WIDE) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int r = 0; r < 4; ++r) accw[j][m][r] = 0.0f;
    }
    gen = false;
  }
};

// The steps of one batch record in shared memory, added to the warp's
// accumulators.
template <int MT, bool WIDE>
__device__ __forceinline__ void process_batch(const uint8_t* base, int lane, const uint16_t* x16, int kpad,
                                              Acc<MT, WIDE>& A) {
  const uint32_t nst = ldu32(base + 4);
  const uint8_t* dsc = base + 8;
  const uint8_t* st = base + strip::pad16(8 + 4 * (int)nst);
  uint32_t i = 0;
  while (i < nst) {
    const uint32_t d = ldu32(dsc + 4 * i);
    const int n0 = desc_n0(d), n1 = desc_n1(d), run = desc_run(d);
    if constexpr (WIDE) {
      if (desc_kind(d) < kU2) {
        switch (d & 31u) {
          case 16 + kG2: wide_run<0, MT>(run, st, lane, x16, kpad, A.accw); i += run; continue;
          case 16 + kG3: wide_run<1, MT>(run, st, lane, x16, kpad, A.accw); i += run; continue;
          case 16 + kG4: wide_run<2, MT>(run, st, lane, x16, kpad, A.accw); i += run; continue;
          case 16 + kG5: wide_run<3, MT>(run, st, lane, x16, kpad, A.accw); i += run; continue;
          case 16 + kG6: wide_run<4, MT>(run, st, lane, x16, kpad, A.accw); i += run; continue;
          case 16 + kG8: wide_run<5, MT>(run, st, lane, x16, kpad, A.accw); i += run; continue;
          case kG2: wide_step<0, false, MT>(st, n0, lane, x16, kpad, A.accw); break;
          case kG3: wide_step<1, false, MT>(st, n0, lane, x16, kpad, A.accw); break;
          case kG4: wide_step<2, false, MT>(st, n0, lane, x16, kpad, A.accw); break;
          case kG5: wide_step<3, false, MT>(st, n0, lane, x16, kpad, A.accw); break;
          case kG6: wide_step<4, false, MT>(st, n0, lane, x16, kpad, A.accw); break;
          default: wide_step<5, false, MT>(st, n0, lane, x16, kpad, A.accw); break;
        }
        st += desc_bytes(d);
        ++i;
        continue;
      }
    }
    switch (d & 31u) {  // kind, plus 16 for a full step
      case 16 + kG2: full_run<0, true, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kG3: full_run<1, true, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kG4: full_run<2, true, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kG5: full_run<3, true, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kG6: full_run<4, true, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kG8: full_run<5, true, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kU2: full_run<0, false, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kU3: full_run<1, false, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kU4: full_run<2, false, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kU5: full_run<3, false, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kU6: full_run<4, false, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case 16 + kU8: full_run<5, false, MT>(run, st, lane, x16, kpad, A.acc1, A.acc2); i += run; continue;
      case kG2: partial_step<0, true, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kG3: partial_step<1, true, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kG4: partial_step<2, true, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kG5: partial_step<3, true, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kG6: partial_step<4, true, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kG8: partial_step<5, true, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kU2: partial_step<0, false, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kU3: partial_step<1, false, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kU4: partial_step<2, false, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kU5: partial_step<3, false, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kU6: partial_step<4, false, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      case kU8: partial_step<5, false, MT>(st, n0, n1, lane, x16, kpad, A.acc1, A.acc2); break;
      default:  // generic (fp32) steps, full or not
        lane_generic<MT>(st, n0, n1, lane, x16, kpad, A.gacc);
        A.gen = true;
        break;
    }
    st += desc_bytes(d);
    ++i;
  }
}

// The warp's sums for one strip -> out[m * 8 + f] (token m, feature f of
// the strip), then zero accumulators.  Quad g's sums sit on the diagonal:
// lane 4g + g/2 holds D[g][g] (element g & 1) and D[g+8][g] (element
// 2 + (g & 1)) of each accumulator; quads 4h..4h+3 cover columns 4h..4h+3.
// (Selects, not indexing, keep the accumulators in registers.)
template <int MT, bool WIDE>
__device__ __forceinline__ void flush(Acc<MT, WIDE>& A, int lane, float* scr, float* out) {
  const int g = lane >> 2, t = lane & 3;
  const bool odd = g & 1;
  if (t == (g >> 1)) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float* o = scr + (m * 8 + g) * 4;
      o[0] = odd ? A.acc1[m][1] : A.acc1[m][0];
      o[1] = odd ? A.acc1[m][3] : A.acc1[m][2];
      o[2] = odd ? A.acc2[m][1] : A.acc2[m][0];
      o[3] = odd ? A.acc2[m][3] : A.acc2[m][2];
    }
    if constexpr (WIDE) {  // wide accumulators: every quad holds all 8 columns
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float* o = scr + MT * 40 + (m * 8 + g) * 8;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o[2 * j] = odd ? A.accw[j][m][1] : A.accw[j][m][0];
          o[2 * j + 1] = odd ? A.accw[j][m][3] : A.accw[j][m][2];
        }
      }
    }
  }
  const bool gen = __any_sync(0xffffffffu, A.gen);
  if (gen) {  // generic lanes: column c of quartet lane >> 4 -> sum over each half warp
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v = A.gacc[m][c];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        if ((lane & 15) == 0) scr[MT * 32 + (m * 2 + (lane >> 4)) * 4 + c] = v;
      }
  }
  __syncwarp();
  if (lane < 8 * MT) {
    const int m = lane >> 3, f = lane & 7, h = f >> 2, c = f & 3;
    const float* s = scr + m * 32 + 16 * h + c;
    float v = s[0] + s[4] + s[8] + s[12];
    if (gen) v += scr[MT * 32 + (m * 2 + h) * 4 + c];
    if constexpr (WIDE) {
      const float* w = scr + MT * 40 + m * 64 + f;
#pragma unroll
      for (int q = 0; q < 8; ++q) v += w[8 * q];
    }
    out[lane] = v;
  }
  __syncwarp();
  A.zero();
}

template <int MT, bool WIDE>
__global__ void __launch_bounds__(MT == 1 ? (WIDE ? 768 : 1024) : 512, 1) strip_kernel(const StripParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nw = p.nw, ns = p.ns;
  const int c = blockIdx.x;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem) + warp * ns;
  uint16_t* x16 = reinterpret_cast<uint16_t*>(smem + p.off_x);
  float* scr = reinterpret_cast<float*>(smem + p.off_scr) + warp * (MT * (WIDE ? 104 : 40));
  float* part = reinterpret_cast<float*>(smem + p.off_part);  // [max_slots][MT][8]
  // slot k of warp w at off_slots + (k nw + w) slot_bytes: slot 1 of every
  // warp is one contiguous region, the staging area of the activations
  uint8_t* slots = smem + p.off_slots + (size_t)warp * p.slot_bytes;
  const size_t slot_stride = (size_t)nw * p.slot_bytes;
  __shared__ int cta_abort;
  __shared__ __align__(8) uint64_t xbar;

  const uint32_t w0 = __ldg(p.warp_work + c * nw + warp), w1 = __ldg(p.warp_work + c * nw + warp + 1);
  // lane 0 keeps the work entries of the slots: word 1 of item w0 + k in slot k
  uint32_t ent[kMaxSlots];
  uint32_t issued = 0;  // lane 0: slots with a copy in flight
  bool bad = false;     // lane 0: a work item failed its bounds check
  auto issue = [&](int s, uint32_t off, uint32_t e1, uint32_t extra) {
    const uint32_t bytes = (e1 & 0xFFFu) << 4;
    if (bytes < 16u || bytes > p.slot_bytes || (off & 15u) || (unsigned long long)off + bytes > p.stream_bytes ||
        (int)((e1 >> 12) & 0x7FFFFu) >= p.max_slots) {
      atomicOr(p.status, MTC_STATUS_BAD_STREAM);
      bad = true;
      return;
    }
    // `extra` > 0 only under mtc_debug_withhold_bytes: the phase then never
    // completes and the bounded wait on it runs out
    mbar_expect_tx(&bar[s], bytes + extra);
    bulk_g2s(slots + (size_t)s * slot_stride, p.stream + off, bytes, &bar[s]);
    issued |= 1u << s;
  };
  if (tid == 0) cta_abort = 0;
  float* xs = reinterpret_cast<float*>(smem + p.off_slots + slot_stride);  // staging: the slot-1 region
  const int32_t* prs = reinterpret_cast<const int32_t*>(xs + (size_t)p.M * p.K);
  if (p.staged && tid == 0) {
    // X rows and pr go out before any weight copy: they are L2 hits and
    // must not queue behind the first batches of every SM
    const uint32_t row = (uint32_t)p.K * 4u;
    mbar_init(&xbar, 1);
    fence_barrier_init();
    mbar_expect_tx(&xbar, row * (uint32_t)(p.M + (p.pr ? 1 : 0)));
    for (int m = 0; m < p.M; ++m) bulk_g2s(xs + (size_t)m * p.K, p.X + (long long)m * p.ldx, row, &xbar);
    if (p.pr) bulk_g2s(const_cast<int32_t*>(prs), p.pr, row, &xbar);
  }
  __syncthreads();
  uint32_t off0[kMaxSlots];
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < kMaxSlots; ++k) {
      off0[k] = ent[k] = 0u;
      if (k < ns && w0 + k < w1) {
        off0[k] = __ldg(p.work + 2 * (w0 + k));
        ent[k] = __ldg(p.work + 2 * (w0 + k) + 1);
      }
    }
    for (int k = 0; k < ns; ++k) mbar_init(&bar[k], 1);
    fence_barrier_init();
    // every warp's first batch goes out at once, ahead of the rest
    if (w0 < w1) issue(0, off0[0], ent[0], p.withhold);
  }

  if (p.staged) {
    // the activations were staged by bulk copy into the slot-1 region (not
    // yet in use); the permutation runs in shared memory, so 148 CTAs do not
    // each pull the scattered sectors of X[:, pr] from L2
    if (tid == 0) {
      if (!mbar_wait(&xbar, 0u, p.timeout_ns)) {
        atomicOr(p.status, MTC_STATUS_TIMEOUT);
        cta_abort = 1;
        (void)mbar_wait(&xbar, 0u, 10000000ull);  // let the copy land before the CTA exits
      }
    }
    __syncthreads();
    if (!cta_abort) {
      uint32_t xbad = 0;
      for (int k = tid; k < p.kpad; k += blockDim.x) {
        const int src = k < p.K ? (p.pr ? prs[k] : k) : -1;
        const bool ok = src >= 0 && src < p.K;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const float v = (m < p.M && ok) ? xs[(size_t)m * p.K + src] : 0.0f;
          if (!(fabsf(v) <= 65504.0f)) xbad = 1;
          x16[(size_t)m * p.kpad + k] = f2h(v);
        }
      }
      if (xbad) atomicOr(p.status, MTC_STATUS_X_RANGE);
    }
    __syncthreads();  // the staging area is read: slot 1 may be filled
    if (lane == 0 && !cta_abort) {
#pragma unroll
      for (int k = 1; k < kMaxSlots; ++k)
        if (k < ns && w0 + k < w1) issue(k, off0[k], ent[k], 0u);
    }
  } else {
  // X[:, pr] as fp16 for every token row (zero beyond M and K).  A thread's
  // source indices, then its activations, are loaded for all of its columns
  // of a pass before anything is stored, and the remaining weight copies are
  // issued only after the first pass's activation loads: these few
  // latency-bound loads then queue behind the first batches only, not
  // behind the bulk traffic of every SM.
  {
    constexpr int G = MT == 1 ? 4 : MT == 2 ? 2 : 1;  // column quads per thread and pass
    uint32_t xbad = 0;
    bool copies_out = false;
    const int step = 4 * (int)blockDim.x;
    for (int k00 = 4 * tid; k00 < p.kpad || !copies_out; k00 += step * G) {
      int src[G][4];
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k = k00 + g * step + j;
          src[g][j] = k < p.K ? (p.pr ? __ldg(p.pr + k) : k) : -1;
        }
      float v[G][MT][4];
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            v[g][m][j] = (m < p.M && src[g][j] >= 0) ? __ldg(p.X + (long long)m * p.ldx + src[g][j]) : 0.0f;
      if (!copies_out) {
        copies_out = true;
        if (lane == 0) {
#pragma unroll
          for (int k = 1; k < kMaxSlots; ++k)
            if (k < ns && w0 + k < w1) issue(k, off0[k], ent[k], 0u);
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int k0 = k00 + g * step;
        if (k0 >= p.kpad) continue;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          uint32_t h[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            if (!(fabsf(v[g][m][2 * j]) <= 65504.0f) || !(fabsf(v[g][m][2 * j + 1]) <= 65504.0f)) xbad = 1;
            h[j] = (uint32_t)f2h(v[g][m][2 * j]) | ((uint32_t)f2h(v[g][m][2 * j + 1]) << 16);
          }
          *reinterpret_cast<uint2*>(x16 + (size_t)m * p.kpad + k0) = make_uint2(h[0], h[1]);
        }
      }
    }
    if (xbad) atomicOr(p.status, MTC_STATUS_X_RANGE);
  }
  __syncthreads();
  }

  Acc<MT, WIDE> A;
  A.zero();
  uint32_t parity = 0;
  int slot = 0;
  bool abort = cta_abort != 0;
  for (uint32_t i = w0; i < w1 && !abort; ++i) {
    // the slot's next item, fetched now and used after this batch
    uint32_t noff = 0, nent = 0;
    const uint32_t ni = i + (uint32_t)ns;
    if (lane == 0 && ni < w1) {
      noff = __ldg(p.work + 2 * ni);
      nent = __ldg(p.work + 2 * ni + 1);
    }
    uint32_t e1 = 0;
#pragma unroll
    for (int k = 0; k < kMaxSlots; ++k)
      if (k == slot) e1 = ent[k];
    int ok = 1;
    if (lane == 0) {
      ok = !bad && mbar_wait(&bar[slot], (parity >> slot) & 1u, p.timeout_ns);
      if (ok) issued &= ~(1u << slot);
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) {
      if (lane == 0 && !bad) atomicOr(p.status, MTC_STATUS_TIMEOUT);
      abort = true;
      break;
    }
    e1 = __shfl_sync(0xffffffffu, e1, 0);
    parity ^= 1u << slot;
    const uint8_t* base = slots + (size_t)slot * slot_stride;
    // records are validated on the host before upload; this check keeps a
    // damaged record from reading beyond its slot
    if (strip::pad16(8 + 4 * (int)ldu32(base + 4)) > (int)((e1 & 0xFFFu) << 4)) {
      if (lane == 0) atomicOr(p.status, MTC_STATUS_BAD_STREAM);
      abort = true;
      break;
    }
    process_batch<MT, WIDE>(base, lane, x16, p.kpad, A);
    // refill the slot (its bytes are consumed)
    if (lane == 0 && ni < w1) {
      fence_proxy_async();
      issue(slot, noff, nent, 0u);
    }
#pragma unroll
    for (int k = 0; k < kMaxSlots; ++k)
      if (k == slot) ent[k] = nent;
    if (e1 & 0x80000000u) flush<MT, WIDE>(A, lane, scr, part + (size_t)((e1 >> 12) & 0x7FFFFu) * MT * 8);
    slot = (slot + 1 == ns) ? 0 : slot + 1;
  }
  if (abort) {
    if (lane == 0) {
      cta_abort = 1;
      // let this warp's copies still in flight land before the CTA exits
      for (int k = 0; k < ns; ++k)
        if (issued & (1u << k)) (void)mbar_wait(&bar[k], (parity >> k) & 1u, 10000000ull);
    }
  }
  __syncthreads();
  if (cta_abort) return;
  // each strip of this CTA: its slots in order, the epilogue, Y[:, pc]
  const uint32_t r0 = __ldg(p.cta_red + c), r1 = __ldg(p.cta_red + c + 1);
  for (uint32_t e = tid; e < (r1 - r0) * MT * 8; e += blockDim.x) {
    const uint32_t j = r0 + e / (MT * 8), q = e % (MT * 8);
    const int m = (int)(q >> 3), f = (int)(q & 7);
    const int strip = (int)__ldg(p.red + 3 * j);
    const uint32_t first = __ldg(p.red + 3 * j + 1), cnt = __ldg(p.red + 3 * j + 2);
    const int n = strip * 8 + f;
    if (m >= p.M || n >= p.N || strip >= p.n_strips) continue;
    if (first + cnt > (uint32_t)p.max_slots) {
      atomicOr(p.status, MTC_STATUS_BAD_STREAM);
      continue;
    }
    float sum = 0.0f;
    for (uint32_t s = first; s < first + cnt; ++s) sum += part[(size_t)s * MT * 8 + q];
    const int jcol = p.pc ? __ldg(p.pc + n) : n;
    p.Y[(long long)m * p.ldy + jcol] = epi_apply(p.ep, sum * p.inv_pow2e, jcol);
  }
}

struct Plan {
  int mt, nw, ns;
  uint32_t slot_bytes, off_x, off_scr, off_part, off_slots;
  size_t smem;
};

// Tokens per launch: 1, 2 or 4 (wide streams at most 2: four accumulators
// per token).  The warp count is the schedule's; two or three slots per warp.
bool make_plan(const mtc_strip_desc* s, int M, bool wide, Plan* pl) {
  if (M < 1 || M > (wide ? 2 : kMaxM)) return false;
  pl->mt = M == 1 ? 1 : M == 2 ? 2 : 4;
  const int max_nw = pl->mt == 1 ? (wide ? 24 : 32) : 16;
  if (s->n_warps < 1 || s->n_warps > max_nw) return false;
  pl->nw = s->n_warps;
  pl->slot_bytes = (s->max_batch_bytes + 127u) & ~127u;
  const int kpad = s->tk * 32;
  auto up = [](size_t x) { return (x + 127) & ~(size_t)127; };
  const size_t xb = up((size_t)pl->mt * kpad * 2);
  const size_t partb = up((size_t)s->max_cta_slots * pl->mt * 8 * 4);
  const size_t budget = 227 * 1024 - 128;  // static shared memory: the abort flag
  for (int ns = kMaxSlots; ns >= 2; --ns) {
    const size_t bars = up((size_t)pl->nw * ns * 8);
    const size_t scr = up((size_t)pl->nw * pl->mt * (wide ? 104 : 40) * 4);
    const size_t need = bars + xb + scr + partb + (size_t)pl->nw * ns * pl->slot_bytes;
    if (need <= budget) {
      pl->ns = ns;
      pl->off_x = (uint32_t)bars;
      pl->off_scr = (uint32_t)(bars + xb);
      pl->off_part = (uint32_t)(bars + xb + scr);
      pl->off_slots = (uint32_t)(bars + xb + scr + partb);
      pl->smem = need;
      return true;
    }
  }
  return false;
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" int mtc_strip_fits(const mtc_strip_desc* s, int32_t M) {
  if (!s || M < 1 || M > strip::kMaxM) return 0;
  const bool wide = (s->flags & MTC_STRIP_WIDE) != 0;
  const int per = wide ? 2 : strip::kMaxM;
  Plan pl;
  return make_plan(s, M < per ? M : per, wide, &pl) ? 1 : 0;
}

extern "C" int mtc_strip_decode(const mtc_strip_desc* s, const float* X, int32_t M, int64_t ldx,
                                const int32_t* row_perm, const int32_t* col_perm, float* Y, int64_t ldy,
                                uint32_t* status, const mtc_epilogue* ep, void* stream) {
  clear_error();
  MTC_REQUIRE(s && X && Y && s->stream && s->work && s->warp_work && s->red && s->cta_red,
              "mtc_strip_decode: null pointer argument");
  MTC_REQUIRE(M >= 1 && M <= strip::kMaxM, "mtc_strip_decode: M=%d outside 1..%d", M, strip::kMaxM);
  MTC_REQUIRE(ldx >= s->K && ldy >= s->N, "mtc_strip_decode: bad leading dimensions");
  MTC_REQUIRE(s->n_strips == s->tn * 4 && s->n_batches >= s->n_strips && s->tk >= 1,
              "mtc_strip_decode: inconsistent strip descriptor");
  MTC_REQUIRE(s->n_cta >= 1 && s->n_cta <= s->n_strips && s->n_warps >= 1 && s->n_warps <= 32,
              "mtc_strip_decode: schedule of %d CTAs x %d warps", s->n_cta, s->n_warps);
  MTC_REQUIRE(s->max_cta_slots >= 1 && s->max_cta_slots <= (uint32_t)s->n_batches,
              "mtc_strip_decode: bad max_cta_slots %u", s->max_cta_slots);
  MTC_REQUIRE((s->flags & ~MTC_STRIP_WIDE) == 0, "mtc_strip_decode: unknown stream flags 0x%x", s->flags);
  MTC_REQUIRE((reinterpret_cast<uintptr_t>(s->stream) & 15) == 0, "mtc_strip_decode: stream not 16-byte aligned");
  MTC_REQUIRE(s->max_batch_bytes >= 16 && s->max_batch_bytes <= 65520 && (s->max_batch_bytes & 15) == 0,
              "mtc_strip_decode: bad max_batch_bytes %u", s->max_batch_bytes);
  EpiArg e;
  int rc = read_epilogue(ep, &e, "mtc_strip_decode");
  if (rc) return rc;
  const bool wide = (s->flags & MTC_STRIP_WIDE) != 0;
  const int per = wide ? 2 : strip::kMaxM;  // tokens per launch
  cudaStream_t st = as_stream(stream);
  for (int m0 = 0; m0 < M; m0 += per) {
    const int Mi = M - m0 < per ? M - m0 : per;
    Plan pl;
    MTC_REQUIRE(make_plan(s, Mi, wide, &pl),
                "mtc_strip_decode: K=%d, %d warps and %u partial slots per CTA do not fit shared memory at M=%d",
                s->K, s->n_warps, s->max_cta_slots, Mi);
    StripParams p;
    p.stream = s->stream;
    p.stream_bytes = s->stream_bytes;
    p.work = s->work;
    p.warp_work = s->warp_work;
    p.red = s->red;
    p.cta_red = s->cta_red;
    p.n_strips = s->n_strips;
    p.K = s->K;
    p.N = s->N;
    p.kpad = s->tk * 32;
    p.inv_pow2e = ldexpf(1.0f, -s->exp2);
    p.X = X + (long long)m0 * ldx;
    p.ldx = ldx;
    p.M = Mi;
    p.pr = row_perm;
    p.pc = col_perm;
    p.Y = Y + (long long)m0 * ldy;
    p.ldy = ldy;
    p.status = status;
    p.ep = Epi{e.bias, e.act};
    p.timeout_ns = wait_limit_ns();
    p.withhold = m0 == 0 ? take_withheld_bytes() : 0u;
    // activations by bulk copy when rows and permutation are 16-byte
    // aligned and they fit the slot-1 region of every warp
    const uintptr_t xa = reinterpret_cast<uintptr_t>(p.X), pa = reinterpret_cast<uintptr_t>(row_perm);
    const size_t stage = (size_t)(Mi + (row_perm ? 1 : 0)) * (size_t)s->K * 4;
    p.staged = (xa & 15) == 0 && (ldx & 3) == 0 && (pa & 15) == 0 && (s->K & 3) == 0 &&
               stage <= (size_t)pl.nw * pl.slot_bytes && stage < (1u << 20);
    p.nw = pl.nw;
    p.ns = pl.ns;
    p.max_slots = (int)s->max_cta_slots;
    p.slot_bytes = pl.slot_bytes;
    p.off_x = pl.off_x;
    p.off_scr = pl.off_scr;
    p.off_part = pl.off_part;
    p.off_slots = pl.off_slots;
    const int which = (pl.mt == 1 ? 0 : pl.mt == 2 ? 1 : 2) + (wide ? 3 : 0);
    const void* fns[6] = {(const void*)strip_kernel<1, false>, (const void*)strip_kernel<2, false>,
                          (const void*)strip_kernel<4, false>, (const void*)strip_kernel<1, true>,
                          (const void*)strip_kernel<2, true>,  (const void*)strip_kernel<2, true>};
    // per-device attribute: set on every call (a process may use several GPUs)
    MTC_CHECK_CUDA(cudaFuncSetAttribute(fns[which], cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem),
                   "mtc_strip_decode: smem attribute");
    const dim3 grid(s->n_cta), block(pl.nw * 32);
    switch (which) {
      case 0: strip_kernel<1, false><<<grid, block, pl.smem, st>>>(p); break;
      case 1: strip_kernel<2, false><<<grid, block, pl.smem, st>>>(p); break;
      case 2: strip_kernel<4, false><<<grid, block, pl.smem, st>>>(p); break;
      case 3: strip_kernel<1, true><<<grid, block, pl.smem, st>>>(p); break;
      default: strip_kernel<2, true><<<grid, block, pl.smem, st>>>(p); break;
    }
    MTC_CHECK_LAUNCH("mtc_strip_decode");
  }
  return MTC_OK;
}
