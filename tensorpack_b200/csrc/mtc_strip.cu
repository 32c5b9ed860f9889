// Strip-stream decode GEMM for M <= 4: Y[:, pc] = X[:, pr] @ Wp.
//
// Replaces, for decode-sized M, the reference's packed GEMM
// (mtc/kernels/gemm.py:124-210, 541-574) and the gather / scatter of MTC-QT-P
// inference (mtc/core/permutation.py:15-21).  The stream layout and the lane
// arithmetic are in mtc_strip.cuh.
//
// Execution: one CTA per range of whole strips (mtc_strip_partition: ranges
// balanced by record bytes, one per SM), every warp an independent worker.
// A worker owns a ring of shared-memory slots; lane 0 copies whole batch
// records into them with cp.async.bulk (one copy per batch, completion on an
// mbarrier).  Each warp's first slots are filled by a static assignment
// before the activations are gathered, so the first HBM reads overlap the
// gather; later batches come from a shared-memory counter, so the warps of a
// CTA balance among themselves.  Partial sums stay in shared memory, one slot
// per batch; the warp that completes a strip's last batch (shared-memory
// ticket) adds the strip's slots in batch order, applies the epilogue and
// writes Y[:, pc].  The result is deterministic, and the kernel needs no
// global scratch, counters or atomics.
//
// Every mbarrier wait is bounded (globaltimer); a timeout sets
// MTC_STATUS_TIMEOUT, the warp waits (bounded) for its own copies in flight
// and stops.
#include "mtc_common.cuh"
#include "mtc_internal.h"
#include "mtc_strip.cuh"

namespace mtc {
namespace {

using namespace strip;

constexpr int kMaxSlots = 3;
constexpr int kMaxCta = MTC_STRIP_MAX_CTA;

struct StripParams {
  const uint8_t* stream;
  const uint32_t* batch_off;    // [n_batches + 1]
  const uint32_t* strip_batch;  // [n_strips + 1]
  int n_batches, n_strips, K, N, kpad;
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
  int nw, ns, cap;  // warps, slots per warp, batches per CTA range
  uint32_t slot_bytes;
  uint32_t off_x, off_scr, off_part, off_meta, off_slots;  // shared-memory layout
  uint32_t part[2 * (kMaxCta + 1)];                      // (first strip, first batch) per CTA range
};
static_assert(sizeof(StripParams) <= 4096, "kernel parameters must fit the 4 KB parameter space");

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

// One batch record in shared memory -> its partial sums (lanes 0 .. 8 MT - 1
// return the sum of column lane & 7 of token lane >> 3; other lanes 0).
template <int MT, bool WIDE>
__device__ __forceinline__ float process_batch(const uint8_t* base, int lane, const uint16_t* x16, int kpad,
                                               float* scr) {
  const uint32_t nst = ldu32(base + 4);
  const uint8_t* dsc = base + 8;
  const uint8_t* st = base + strip::pad16(8 + 4 * (int)nst);
  float acc1[MT][4], acc2[MT][4], gacc[MT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc1[m][r] = acc2[m][r] = gacc[m][r] = 0.0f;
  float accw[WIDE ? 4 : 1][MT][4];
  if constexpr (WIDE) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int r = 0; r < 4; ++r) accw[j][m][r] = 0.0f;
  }
  bool gen = false;
  uint32_t i = 0;
  while (i < nst) {
    const uint32_t d = ldu32(dsc + 4 * i);
    const int n0 = desc_n0(d), n1 = desc_n1(d), run = desc_run(d);
    if constexpr (WIDE) {
      if (desc_kind(d) < kU2) {
        switch (d & 31u) {
          case 16 + kG2: wide_run<0, MT>(run, st, lane, x16, kpad, accw); i += run; continue;
          case 16 + kG3: wide_run<1, MT>(run, st, lane, x16, kpad, accw); i += run; continue;
          case 16 + kG4: wide_run<2, MT>(run, st, lane, x16, kpad, accw); i += run; continue;
          case 16 + kG5: wide_run<3, MT>(run, st, lane, x16, kpad, accw); i += run; continue;
          case 16 + kG6: wide_run<4, MT>(run, st, lane, x16, kpad, accw); i += run; continue;
          case 16 + kG8: wide_run<5, MT>(run, st, lane, x16, kpad, accw); i += run; continue;
          case kG2: wide_step<0, false, MT>(st, n0, lane, x16, kpad, accw); break;
          case kG3: wide_step<1, false, MT>(st, n0, lane, x16, kpad, accw); break;
          case kG4: wide_step<2, false, MT>(st, n0, lane, x16, kpad, accw); break;
          case kG5: wide_step<3, false, MT>(st, n0, lane, x16, kpad, accw); break;
          case kG6: wide_step<4, false, MT>(st, n0, lane, x16, kpad, accw); break;
          default: wide_step<5, false, MT>(st, n0, lane, x16, kpad, accw); break;
        }
        st += desc_bytes(d);
        ++i;
        continue;
      }
    }
    switch (d & 31u) {  // kind, plus 16 for a full step
      case 16 + kG2: full_run<0, true, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kG3: full_run<1, true, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kG4: full_run<2, true, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kG5: full_run<3, true, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kG6: full_run<4, true, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kG8: full_run<5, true, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kU2: full_run<0, false, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kU3: full_run<1, false, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kU4: full_run<2, false, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kU5: full_run<3, false, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kU6: full_run<4, false, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case 16 + kU8: full_run<5, false, MT>(run, st, lane, x16, kpad, acc1, acc2); i += run; continue;
      case kG2: partial_step<0, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kG3: partial_step<1, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kG4: partial_step<2, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kG5: partial_step<3, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kG6: partial_step<4, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kG8: partial_step<5, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU2: partial_step<0, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU3: partial_step<1, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU4: partial_step<2, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU5: partial_step<3, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU6: partial_step<4, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU8: partial_step<5, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      default:  // generic (fp32) steps, full or not
        lane_generic<MT>(st, n0, n1, lane, x16, kpad, gacc);
        gen = true;
        break;
    }
    st += desc_bytes(d);
    ++i;
  }
  // Quad g's sums sit on the diagonal: lane 4g + g/2 holds D[g][g] (element
  // g & 1) and D[g+8][g] (element 2 + (g & 1)) of each accumulator; quads
  // 4h..4h+3 cover columns 4h..4h+3 of the strip.  (Selects, not indexing,
  // keep the accumulators in registers.)
  const int g = lane >> 2, t = lane & 3;
  const bool odd = g & 1;
  if (t == (g >> 1)) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float* o = scr + (m * 8 + g) * 4;
      o[0] = odd ? acc1[m][1] : acc1[m][0];
      o[1] = odd ? acc1[m][3] : acc1[m][2];
      o[2] = odd ? acc2[m][1] : acc2[m][0];
      o[3] = odd ? acc2[m][3] : acc2[m][2];
    }
  }
  if constexpr (WIDE) {  // wide accumulators: every quad holds all 8 columns
    if (t == (g >> 1)) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float* o = scr + MT * 40 + (m * 8 + g) * 8;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o[2 * j] = odd ? accw[j][m][1] : accw[j][m][0];
          o[2 * j + 1] = odd ? accw[j][m][3] : accw[j][m][2];
        }
      }
    }
  }
  if (gen) {  // generic lanes: column c of quartet lane >> 4 -> sum over each half warp
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v = gacc[m][c];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        if ((lane & 15) == 0) scr[MT * 32 + (m * 2 + (lane >> 4)) * 4 + c] = v;
      }
  }
  __syncwarp();
  float v = 0.0f;
  if (lane < 8 * MT) {
    const int m = lane >> 3, f = lane & 7, h = f >> 2, c = f & 3;
    const float* s = scr + m * 32 + 16 * h + c;
    v = s[0] + s[4] + s[8] + s[12];
    if (gen) v += scr[MT * 32 + (m * 2 + h) * 4 + c];
    if constexpr (WIDE) {
      const float* w = scr + MT * 40 + m * 64 + f;
#pragma unroll
      for (int q = 0; q < 8; ++q) v += w[8 * q];
    }
  }
  __syncwarp();
  return v;
}

template <int MT, bool WIDE>
__global__ void __launch_bounds__((MT == 4 || (WIDE && MT == 2)) ? 512 : 768, 1) strip_kernel(const StripParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nw = p.nw, ns = p.ns;
  const int c = blockIdx.x;
  const int s0 = (int)p.part[2 * c], s1 = (int)p.part[2 * c + 2];
  const int b0 = (int)p.part[2 * c + 1], b1 = (int)p.part[2 * c + 3];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [nw][ns]
  uint16_t* x16 = reinterpret_cast<uint16_t*>(smem + p.off_x);
  float* scr = reinterpret_cast<float*>(smem + p.off_scr) + warp * (MT * (WIDE ? 104 : 40));
  float* part = reinterpret_cast<float*>(smem + p.off_part);         // [cap][MT][8]
  uint32_t* meta = reinterpret_cast<uint32_t*>(smem + p.off_meta);   // tickets [cap], first batch [cap + 1], queue
  uint32_t* tick = meta;
  uint32_t* sfirst = meta + p.cap;
  uint32_t* queue = meta + 2 * p.cap + 1;
  uint8_t* slots = smem + p.off_slots + (size_t)warp * ns * p.slot_bytes;
  uint64_t* bar = full + warp * ns;

  // the first slots of every warp: batches b0 + warp + k nw (k < ns)
  uint32_t pre_off[kMaxSlots], pre_end[kMaxSlots];
#pragma unroll
  for (int k = 0; k < kMaxSlots; ++k) {
    const int b = b0 + warp + k * nw;
    pre_off[k] = pre_end[k] = 0u;
    if (lane == 0 && k < ns && b < b1) {
      pre_off[k] = __ldg(p.batch_off + b);
      pre_end[k] = __ldg(p.batch_off + b + 1);
    }
  }
  if (tid == 0) {
    for (int i = 0; i < nw * ns; ++i) mbar_init(&full[i], 1);
    fence_barrier_init();
    *queue = (uint32_t)(nw * ns);
  }
  for (int i = tid; i < s1 - s0; i += blockDim.x) tick[i] = 0u;
  for (int i = tid; i <= s1 - s0; i += blockDim.x) sfirst[i] = __ldg(p.strip_batch + s0 + i) - (uint32_t)b0;
  __syncthreads();

  uint32_t issued = 0;  // lane 0: slots with a copy in flight
  bool fail = false;    // lane 0: a batch record failed its bounds check
  auto issue = [&](int s, uint32_t off, uint32_t end) {
    const uint32_t bytes = end - off;
    if (end < off || bytes > p.slot_bytes || (off & 15u) || (bytes & 15u) || bytes < 16u) {
      atomicOr(p.status, MTC_STATUS_BAD_STREAM);
      fail = true;
      return;
    }
    mbar_expect_tx(&bar[s], bytes);
    bulk_g2s(slots + (size_t)s * p.slot_bytes, p.stream + off, bytes, &bar[s]);
    issued |= 1u << s;
  };
  int bq[kMaxSlots];
#pragma unroll
  for (int k = 0; k < kMaxSlots; ++k) {
    bq[k] = (k < ns && b0 + warp + k * nw < b1) ? b0 + warp + k * nw : 0x7fffffff;
    if (lane == 0 && bq[k] < b1) issue(k, pre_off[k], pre_end[k]);
  }

  // X[:, pr] as fp16 for every token row (zero beyond M and K); four columns
  // per thread and iteration, their loads issued together
  {
    uint32_t bad = 0;
    for (int k0 = 4 * tid; k0 < p.kpad; k0 += 4 * blockDim.x) {
      int src[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = k0 + j;
        src[j] = k < p.K ? (p.pr ? __ldg(p.pr + k) : k) : -1;
      }
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = (m < p.M && src[j] >= 0) ? __ldg(p.X + (long long)m * p.ldx + src[j]) : 0.0f;
        uint32_t h[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          if (!(fabsf(v[2 * j]) <= 65504.0f) || !(fabsf(v[2 * j + 1]) <= 65504.0f)) bad = 1;
          h[j] = (uint32_t)f2h(v[2 * j]) | ((uint32_t)f2h(v[2 * j + 1]) << 16);
        }
        *reinterpret_cast<uint2*>(x16 + (size_t)m * p.kpad + k0) = make_uint2(h[0], h[1]);
      }
    }
    if (bad) atomicOr(p.status, MTC_STATUS_X_RANGE);
  }
  __syncthreads();

  uint32_t parity = 0;
  int slot = 0, live = 0;
#pragma unroll
  for (int k = 0; k < kMaxSlots; ++k) live += (bq[k] < b1) ? 1 : 0;
  bool abort = false;
  while (live > 0) {
    int b = 0;
#pragma unroll
    for (int k = 0; k < kMaxSlots; ++k)
      if (k == slot) b = bq[k];
    if (b >= b1) {
      slot = (slot + 1 == ns) ? 0 : slot + 1;
      continue;
    }
    // the slot's next batch: index and record offsets fetched now, used after
    // this batch, so their latency hides behind the decode
    int nb = 0x7fffffff;
    uint32_t noff = 0, nend = 0;
    if (lane == 0) {
      const int j = (int)atomicAdd(queue, 1u);
      if (b0 + j < b1) {
        nb = b0 + j;
        noff = __ldg(p.batch_off + nb);
        nend = __ldg(p.batch_off + nb + 1);
      }
    }
    int ok = 1;
    if (lane == 0) {
      ok = !fail && mbar_wait(&bar[slot], (parity >> slot) & 1u, p.timeout_ns);
      if (ok) issued &= ~(1u << slot);
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) {
      if (lane == 0 && !fail) atomicOr(p.status, MTC_STATUS_TIMEOUT);
      abort = true;
      break;
    }
    parity ^= 1u << slot;
    const uint8_t* base = slots + (size_t)slot * p.slot_bytes;
    const int strip = (int)ldu32(base);
    // records are validated on the host before upload; these checks keep a
    // damaged record from indexing outside the CTA's tables or the slot
    if (strip < s0 || strip >= s1 || strip::pad16(8 + 4 * (int)ldu32(base + 4)) > (int)p.slot_bytes) {
      if (lane == 0) atomicOr(p.status, MTC_STATUS_BAD_STREAM);
      abort = true;
      break;
    }
    const float v = process_batch<MT, WIDE>(base, lane, x16, p.kpad, scr);
    // refill the slot (its bytes are consumed)
    if (lane == 0 && nb < b1) {
      fence_proxy_async();
      issue(slot, noff, nend);
    }
    nb = __shfl_sync(0xffffffffu, nb, 0);
#pragma unroll
    for (int k = 0; k < kMaxSlots; ++k)
      if (k == slot) bq[k] = nb;
    if (nb >= b1) --live;
    // partial sums of this batch, then the strip's ticket
    if (lane < 8 * MT) part[(b - b0) * MT * 8 + lane] = v;
    __syncwarp();
    const int ls = strip - s0;
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = (atomicAdd(&tick[ls], 1u) == sfirst[ls + 1] - sfirst[ls] - 1u) ? 1 : 0;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence_block();
      if (lane < 8 * MT) {
        const int m = lane >> 3, f = lane & 7;
        const int n = strip * 8 + f;
        if (m < p.M && n < p.N) {
          float sum = 0.0f;
          for (uint32_t bb = sfirst[ls]; bb < sfirst[ls + 1]; ++bb) sum += part[bb * MT * 8 + lane];
          const int jcol = p.pc ? __ldg(p.pc + n) : n;
          p.Y[(long long)m * p.ldy + jcol] = epi_apply(p.ep, sum * p.inv_pow2e, jcol);
        }
      }
    }
    slot = (slot + 1 == ns) ? 0 : slot + 1;
  }
  if (abort && lane == 0) {
    // let this warp's copies still in flight land before the CTA exits
    for (int k = 0; k < ns; ++k)
      if (issued & (1u << k)) (void)mbar_wait(&bar[k], (parity >> k) & 1u, 10000000ull);
  }
}

struct Plan {
  int mt, nw, ns, cap;
  uint32_t slot_bytes, off_x, off_scr, off_part, off_meta, off_slots;
  size_t smem;
};

// Tokens per launch: 1, 2 or 4 (wide streams at most 2: four accumulators
// per token).
bool make_plan(const mtc_strip_desc* s, int M, bool wide, Plan* pl) {
  if (M < 1 || M > (wide ? 2 : kMaxM)) return false;
  pl->mt = M == 1 ? 1 : M == 2 ? 2 : 4;
  pl->slot_bytes = (s->max_batch_bytes + 127u) & ~127u;
  pl->cap = (int)s->max_cta_batches;
  const int kpad = s->tk * 32;
  auto up = [](size_t x) { return (x + 127) & ~(size_t)127; };
  const size_t xb = up((size_t)pl->mt * kpad * 2);
  const size_t partb = up((size_t)pl->cap * pl->mt * 8 * 4);
  const size_t metab = up(((size_t)2 * pl->cap + 2) * 4);
  const size_t budget = 227 * 1024;
  const int max_nw = (pl->mt == 4 || (wide && pl->mt == 2)) ? 16 : 24;
  // three slots per warp while at least 16 warps fit, else two
  for (int ns = kMaxSlots; ns >= 2; --ns)
    for (int nw = max_nw; nw >= 4; --nw) {
      const size_t bars = up((size_t)nw * ns * 8);
      const size_t scr = up((size_t)nw * pl->mt * (wide ? 104 : 40) * 4);
      const size_t need = bars + xb + scr + partb + metab + (size_t)nw * ns * pl->slot_bytes;
      if (need <= budget && (ns == 2 || nw >= 16)) {
        pl->nw = nw;
        pl->ns = ns;
        pl->off_x = (uint32_t)bars;
        pl->off_scr = (uint32_t)(bars + xb);
        pl->off_part = (uint32_t)(bars + xb + scr);
        pl->off_meta = (uint32_t)(bars + xb + scr + partb);
        pl->off_slots = (uint32_t)(bars + xb + scr + partb + metab);
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
  MTC_REQUIRE(s && X && Y && s->stream && s->batch_off && s->strip_batch && s->cta_part,
              "mtc_strip_decode: null pointer argument");
  MTC_REQUIRE(M >= 1 && M <= strip::kMaxM, "mtc_strip_decode: M=%d outside 1..%d", M, strip::kMaxM);
  MTC_REQUIRE(ldx >= s->K && ldy >= s->N, "mtc_strip_decode: bad leading dimensions");
  MTC_REQUIRE(s->n_strips == s->tn * 4 && s->n_batches >= s->n_strips && s->tk >= 1,
              "mtc_strip_decode: inconsistent strip descriptor");
  MTC_REQUIRE(s->n_cta >= 1 && s->n_cta <= kMaxCta, "mtc_strip_decode: %d CTA ranges (1..%d)", s->n_cta, kMaxCta);
  MTC_REQUIRE(s->cta_part[0] == 0 && s->cta_part[1] == 0 && (int)s->cta_part[2 * s->n_cta] == s->n_strips &&
                  (int)s->cta_part[2 * s->n_cta + 1] == s->n_batches,
              "mtc_strip_decode: CTA partition does not cover the stream");
  for (int c = 0; c < s->n_cta; ++c)
    MTC_REQUIRE(s->cta_part[2 * c + 2] > s->cta_part[2 * c] && s->cta_part[2 * c + 3] > s->cta_part[2 * c + 1] &&
                    s->cta_part[2 * c + 3] - s->cta_part[2 * c + 1] <= s->max_cta_batches,
                "mtc_strip_decode: CTA range %d is empty or exceeds max_cta_batches", c);
  MTC_REQUIRE((s->flags & ~MTC_STRIP_WIDE) == 0, "mtc_strip_decode: unknown stream flags 0x%x", s->flags);
  MTC_REQUIRE((reinterpret_cast<uintptr_t>(s->stream) & 15) == 0, "mtc_strip_decode: stream not 16-byte aligned");
  MTC_REQUIRE(s->max_batch_bytes >= 16 && s->max_batch_bytes <= 65536 && (s->max_batch_bytes & 15) == 0,
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
                "mtc_strip_decode: K=%d / %u batches per CTA do not fit shared memory at M=%d", s->K,
                s->max_cta_batches, Mi);
    StripParams p;
    p.stream = s->stream;
    p.batch_off = s->batch_off;
    p.strip_batch = s->strip_batch;
    p.n_batches = s->n_batches;
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
    p.timeout_ns = 2000000000ull;
    p.nw = pl.nw;
    p.ns = pl.ns;
    p.cap = pl.cap;
    p.slot_bytes = pl.slot_bytes;
    p.off_x = pl.off_x;
    p.off_scr = pl.off_scr;
    p.off_part = pl.off_part;
    p.off_meta = pl.off_meta;
    p.off_slots = pl.off_slots;
    for (int i = 0; i < 2 * (s->n_cta + 1); ++i) p.part[i] = s->cta_part[i];
    const int which = (pl.mt == 1 ? 0 : pl.mt == 2 ? 1 : 2) + (wide ? 3 : 0);
    const void* fns[6] = {(const void*)strip_kernel<1, false>, (const void*)strip_kernel<2, false>,
                          (const void*)strip_kernel<4, false>, (const void*)strip_kernel<1, true>,
                          (const void*)strip_kernel<2, true>,  (const void*)strip_kernel<2, true>};
    // per-device attribute: set on every call (a process may use several GPUs)
    MTC_CHECK_CUDA(cudaFuncSetAttribute(fns[which], cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
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
