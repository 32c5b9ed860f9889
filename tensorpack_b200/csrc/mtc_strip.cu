// Strip-stream decode GEMM for M <= 4: Y[:, pc] = X[:, pr] @ Wp.
//
// Replaces, for decode-sized M, the reference's packed GEMM
// (mtc/kernels/gemm.py:124-210, 541-574) and the gather / scatter of MTC-QT-P
// inference (mtc/core/permutation.py:15-21).  The stream layout and the lane
// arithmetic are in mtc_strip.cuh.
//
// Execution: persistent CTAs (one per SM), every warp an independent worker.
// A worker owns a ring of shared-memory slots; lane 0 copies whole batch
// records into them with cp.async.bulk (one copy per batch, completion on an
// mbarrier) and takes the next batch index from a global counter, so work is
// balanced dynamically.  The first slots of every warp are filled by a
// static assignment before the activations are gathered, so the first HBM
// reads overlap the gather.  Each batch belongs to one strip; its partial
// sums go to a workspace slot per batch, and the warp that completes a
// strip's last batch (atomic ticket) adds the strip's slots in batch order,
// applies the epilogue and writes Y[:, pc] (deterministic result).
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

constexpr int kMaxSlots = 4;
constexpr int kMaxWarps = 16;

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
  float* ws;          // [n_batches][MT][8]
  uint32_t* tickets;  // [n_strips] then the schedule words [2]
  uint32_t* status;
  Epi ep;
  unsigned long long timeout_ns;
  int nw, ns;
  uint32_t slot_bytes;
  uint32_t off_x, off_scr, off_slots;  // shared-memory layout
};

__device__ __forceinline__ void mma_f16(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int C, bool GROUP, int MT>
__device__ __forceinline__ void fast_step(const uint8_t* st, int n0, int n1, int lane, const uint16_t* x16,
                                          int kpad, float acc1[MT][4], float acc2[MT][4]) {
  uint32_t a[8], b[MT][2];
  lane_fast<C, GROUP, MT>(st, n0, n1, lane, x16, kpad, a, b);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    mma_f16(acc1[m], a[0], a[1], a[2], a[3], b[m][0], b[m][1]);
    mma_f16(acc2[m], a[4], a[5], a[6], a[7], b[m][0], b[m][1]);
  }
}

// One batch record in shared memory -> partial sums of its strip in ws[b].
template <int MT>
__device__ __forceinline__ void process_batch(const uint8_t* base, int lane, const uint16_t* x16, int kpad,
                                              float* scr, float* out) {
  const uint32_t nst = ldu32(base + 4);
  const uint8_t* dsc = base + 8;
  const uint8_t* st = base + strip::pad16(8 + 4 * (int)nst);
  float acc1[MT][4], acc2[MT][4], gacc[MT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc1[m][r] = acc2[m][r] = gacc[m][r] = 0.0f;
  bool gen = false;
  for (uint32_t i = 0; i < nst; ++i) {
    const uint32_t d = ldu32(dsc + 4 * i);
    const int n0 = desc_n0(d), n1 = desc_n1(d);
    switch (desc_kind(d)) {
      case kG2: fast_step<0, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kG3: fast_step<1, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kG4: fast_step<2, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kG5: fast_step<3, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kG6: fast_step<4, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kG8: fast_step<5, true, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU2: fast_step<0, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU3: fast_step<1, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU4: fast_step<2, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU5: fast_step<3, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU6: fast_step<4, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      case kU8: fast_step<5, false, MT>(st, n0, n1, lane, x16, kpad, acc1, acc2); break;
      default:
        lane_generic<MT>(st, n0, n1, lane, x16, kpad, gacc);
        gen = true;
        break;
    }
    st += desc_bytes(d);
  }
  // Quad g's sums sit on the diagonal: lane 4g + g/2 holds D[g][g] (element
  // g & 1) and D[g+8][g] (element 2 + (g & 1)) of each accumulator; quads
  // 4h..4h+3 cover columns 4h..4h+3 of the strip.
  const int g = lane >> 2, t = lane & 3, sel = g & 1;
  if (t == (g >> 1)) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float* o = scr + (m * 8 + g) * 4;
      o[0] = acc1[m][sel];
      o[1] = acc1[m][2 + sel];
      o[2] = acc2[m][sel];
      o[3] = acc2[m][2 + sel];
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
  if (lane < 8 * MT) {
    const int m = lane >> 3, f = lane & 7, h = f >> 2, c = f & 3;
    const float* s = scr + m * 32 + 16 * h + c;
    float v = s[0] + s[4] + s[8] + s[12];
    if (gen) v += scr[MT * 32 + (m * 2 + h) * 4 + c];
    out[m * 8 + f] = v;
    __threadfence();
  }
  __syncwarp();
}

template <int MT>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) strip_kernel(const StripParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nw = p.nw, ns = p.ns;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [nw][ns]
  uint16_t* x16 = reinterpret_cast<uint16_t*>(smem + p.off_x);
  float* scr = reinterpret_cast<float*>(smem + p.off_scr) + warp * (MT * 40);
  uint8_t* slots = smem + p.off_slots + (size_t)warp * ns * p.slot_bytes;
  uint64_t* bar = full + warp * ns;
  uint32_t* sched = p.tickets + p.n_strips;

  if (tid == 0) {
    for (int i = 0; i < nw * ns; ++i) mbar_init(&full[i], 1);
    fence_barrier_init();
  }
  __syncthreads();

  const int W = gridDim.x * nw, wg = blockIdx.x * nw + warp;
  int bq[kMaxSlots];
  uint32_t issued = 0;  // lane 0: slots with a copy in flight
  bool fail = false;    // lane 0: a batch record failed its bounds check
  auto issue = [&](int s, int b) {
    const uint32_t off = p.batch_off[b], bytes = p.batch_off[b + 1] - off;
    if (bytes > p.slot_bytes || (off & 15u) || (bytes & 15u) || bytes < 16u) {
      atomicOr(p.status, MTC_STATUS_BAD_STREAM);
      fail = true;
      return;
    }
    mbar_expect_tx(&bar[s], bytes);
    bulk_g2s(slots + (size_t)s * p.slot_bytes, p.stream + off, bytes, &bar[s]);
    issued |= 1u << s;
  };
#pragma unroll
  for (int s = 0; s < kMaxSlots; ++s) {
    bq[s] = (s < ns) ? wg + s * W : 0x7fffffff;
    if (lane == 0 && bq[s] < p.n_batches) issue(s, bq[s]);
  }

  // X[:, pr] as fp16 for every token row (zero beyond M and K)
  {
    uint32_t bad = 0;
    for (int k = tid; k < p.kpad; k += blockDim.x) {
      const int src = k < p.K ? (p.pr ? p.pr[k] : k) : -1;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const float v = (m < p.M && src >= 0) ? p.X[(long long)m * p.ldx + src] : 0.0f;
        if (!(fabsf(v) <= 65504.0f)) bad = 1;
        x16[(size_t)m * p.kpad + k] = f2h(v);
      }
    }
    if (bad) atomicOr(p.status, MTC_STATUS_X_RANGE);
  }
  __syncthreads();

  uint32_t parity = 0;
  int slot = 0, live = 0;
#pragma unroll
  for (int s = 0; s < kMaxSlots; ++s) live += (bq[s] < p.n_batches) ? 1 : 0;
  bool abort = false;
  while (live > 0) {
    int b = 0;
#pragma unroll
    for (int s = 0; s < kMaxSlots; ++s)
      if (s == slot) b = bq[s];
    if (b >= p.n_batches) {
      slot = (slot + 1 == ns) ? 0 : slot + 1;
      continue;
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
    // records are validated on the host before upload; these two checks keep
    // a damaged record from indexing outside the tables or the slot
    if ((unsigned)strip >= (unsigned)p.n_strips || strip::pad16(8 + 4 * (int)ldu32(base + 4)) > (int)p.slot_bytes) {
      if (lane == 0) atomicOr(p.status, MTC_STATUS_BAD_STREAM);
      abort = true;
      break;
    }
    process_batch<MT>(base, lane, x16, p.kpad, scr, p.ws + (size_t)b * MT * 8);
    // refill the slot (its bytes are consumed) with the next dynamic batch
    int nb = 0x7fffffff;
    if (lane == 0) {
      nb = ns * W + (int)atomicAdd(&sched[0], 1u);
      if (nb < p.n_batches) {
        fence_proxy_async();
        issue(slot, nb);
      }
    }
    nb = __shfl_sync(0xffffffffu, nb, 0);
#pragma unroll
    for (int s = 0; s < kMaxSlots; ++s)
      if (s == slot) bq[s] = nb;
    if (nb >= p.n_batches) --live;
    // strip ticket: the warp that completes the strip's last batch writes Y
    int last = 0;
    const uint32_t b0 = p.strip_batch[strip], b1 = p.strip_batch[strip + 1];
    if (lane == 0) {
      __threadfence();
      last = (atomicAdd(&p.tickets[strip], 1u) == b1 - b0 - 1u) ? 1 : 0;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence();
      if (lane < 8 * MT) {
        const int m = lane >> 3, f = lane & 7;
        const int n = strip * 8 + f;
        if (m < p.M && n < p.N) {
          float sum = 0.0f;
          for (uint32_t bb = b0; bb < b1; ++bb) sum += __ldcg(p.ws + ((size_t)bb * MT + m) * 8 + f);
          const int j = p.pc ? p.pc[n] : n;
          p.Y[(long long)m * p.ldy + j] = epi_apply(p.ep, sum * p.inv_pow2e, j);
        }
      }
      if (lane == 0) p.tickets[strip] = 0u;
    }
    slot = (slot + 1 == ns) ? 0 : slot + 1;
  }
  if (abort && lane == 0) {
    // let this warp's copies still in flight land before the CTA exits
    for (int s = 0; s < ns; ++s)
      if (issued & (1u << s)) (void)mbar_wait(&bar[s], (parity >> s) & 1u, 10000000ull);
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&sched[1], 1u) == gridDim.x - 1) {  // last CTA: reset the schedule for the next call
      sched[0] = 0u;
      sched[1] = 0u;
      __threadfence();
    }
  }
}

struct Plan {
  int mt, nw, ns, grid;
  uint32_t slot_bytes, off_x, off_scr, off_slots;
  size_t smem;
};

bool make_plan(const mtc_strip_desc* s, int M, int sms, Plan* pl) {
  if (M < 1 || M > kMaxM) return false;
  pl->mt = M == 1 ? 1 : M == 2 ? 2 : 4;
  pl->slot_bytes = (s->max_batch_bytes + 127u) & ~127u;
  const int kpad = s->tk * 32;
  const size_t xb = ((size_t)pl->mt * kpad * 2 + 127) & ~(size_t)127;
  const size_t budget = 227 * 1024;
  pl->grid = sms;
  for (int ns = 3; ns >= 2; --ns)
    for (int nw = kMaxWarps; nw >= 4; --nw) {
      const size_t bars = ((size_t)nw * ns * 8 + 127) & ~(size_t)127;
      const size_t scr = ((size_t)nw * pl->mt * 40 * 4 + 127) & ~(size_t)127;
      const size_t need = bars + xb + scr + (size_t)nw * ns * pl->slot_bytes;
      if (need <= budget && (ns == 2 || nw >= 12)) {
        pl->nw = nw;
        pl->ns = ns;
        pl->off_x = (uint32_t)bars;
        pl->off_scr = (uint32_t)(bars + xb);
        pl->off_slots = (uint32_t)(bars + xb + scr);
        pl->smem = need;
        return true;
      }
    }
  return false;
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" size_t mtc_strip_workspace_bytes(const mtc_strip_desc* s, int32_t M) {
  if (!s || M < 1 || M > strip::kMaxM) return 0;
  const int mt = M == 1 ? 1 : M == 2 ? 2 : 4;
  return (size_t)s->n_batches * mt * 8 * sizeof(float);
}

extern "C" int mtc_strip_decode(const mtc_strip_desc* s, const float* X, int32_t M, int64_t ldx,
                                const int32_t* row_perm, const int32_t* col_perm, float* Y, int64_t ldy, void* ws,
                                size_t ws_bytes, uint32_t* counters, uint32_t* status, const mtc_epilogue* ep,
                                void* stream) {
  clear_error();
  MTC_REQUIRE(s && X && Y && ws && counters && s->stream && s->batch_off && s->strip_batch,
              "mtc_strip_decode: null pointer argument");
  MTC_REQUIRE(M >= 1 && M <= strip::kMaxM, "mtc_strip_decode: M=%d outside 1..%d", M, strip::kMaxM);
  MTC_REQUIRE(ldx >= s->K && ldy >= s->N, "mtc_strip_decode: bad leading dimensions");
  MTC_REQUIRE(s->n_strips == s->tn * 4 && s->n_batches >= s->n_strips && s->tk >= 1,
              "mtc_strip_decode: inconsistent strip descriptor");
  MTC_REQUIRE((reinterpret_cast<uintptr_t>(s->stream) & 15) == 0, "mtc_strip_decode: stream not 16-byte aligned");
  MTC_REQUIRE(s->max_batch_bytes >= 16 && s->max_batch_bytes <= 65536 && (s->max_batch_bytes & 15) == 0,
              "mtc_strip_decode: bad max_batch_bytes %u", s->max_batch_bytes);
  EpiArg e;
  int rc = read_epilogue(ep, &e, "mtc_strip_decode");
  if (rc) return rc;
  int dev = 0, sms = 148;
  MTC_CHECK_CUDA(cudaGetDevice(&dev), "mtc_strip_decode: cudaGetDevice");
  MTC_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "mtc_strip_decode: SM count");
  Plan pl;
  MTC_REQUIRE(make_plan(s, M, sms, &pl), "mtc_strip_decode: K=%d does not fit shared memory at M=%d", s->K, M);
  const size_t need = (size_t)s->n_batches * pl.mt * 8 * sizeof(float);
  if (ws_bytes < need) {
    set_error("mtc_strip_decode: workspace %zu bytes, need %zu", ws_bytes, need);
    return MTC_ERR_WORKSPACE;
  }
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
  p.X = X;
  p.ldx = ldx;
  p.M = M;
  p.pr = row_perm;
  p.pc = col_perm;
  p.Y = Y;
  p.ldy = ldy;
  p.ws = static_cast<float*>(ws);
  p.tickets = counters;
  p.status = status;
  p.ep = Epi{e.bias, e.act};
  p.timeout_ns = 2000000000ull;
  p.nw = pl.nw;
  p.ns = pl.ns;
  p.slot_bytes = pl.slot_bytes;
  p.off_x = pl.off_x;
  p.off_scr = pl.off_scr;
  p.off_slots = pl.off_slots;
  cudaStream_t st = as_stream(stream);
  static bool opted[3] = {false, false, false};
  const int which = pl.mt == 1 ? 0 : pl.mt == 2 ? 1 : 2;
  const void* fn = which == 0 ? (const void*)strip_kernel<1> : which == 1 ? (const void*)strip_kernel<2>
                                                                          : (const void*)strip_kernel<4>;
  if (!opted[which]) {
    MTC_CHECK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
                   "mtc_strip_decode: smem attribute");
    opted[which] = true;
  }
  const dim3 grid(pl.grid), block(pl.nw * 32);
  if (which == 0)
    strip_kernel<1><<<grid, block, pl.smem, st>>>(p);
  else if (which == 1)
    strip_kernel<2><<<grid, block, pl.smem, st>>>(p);
  else
    strip_kernel<4><<<grid, block, pl.smem, st>>>(p);
  MTC_CHECK_LAUNCH("mtc_strip_decode");
  return MTC_OK;
}
