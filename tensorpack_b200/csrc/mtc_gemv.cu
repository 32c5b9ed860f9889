// Split-K streaming GEMM for decode-sized M (<= 16): Y[:, pc] = X[:, pr] @ Wp.
//
// Replaces the reference's packed GEMM (mtc/kernels/gemm.py:124-210, 541-574)
// and the gather / scatter of MTC-QT-P inference (mtc/core/permutation.py:
// 15-21) for M <= 16.  The packed bits are read from HBM exactly once:
//
//  * work unit = (column band of 8 tiles = 256 features, range of k-tile
//    rows); one CTA per unit, 8 consumer warps (one tile column each) and
//    one producer warp.
//  * the producer streams each k-tile row of the band (8 contiguous tile
//    records) into a shared-memory ring with cp.async.bulk + mbarrier
//    transaction counts;
//  * each consumer lane decodes half of an aligned 2x2 micro-block group
//    straight into mma.sync A fragments (weights as the 16-row operand,
//    the M <= 16 tokens as the 8-column operand, fp32 accumulation); the
//    row permutation is applied when X is staged in shared memory as fp16;
//  * partial sums of a unit go to the workspace, and the last unit of a band
//    (atomic ticket) reduces them in a fixed order and scatters Y[:, pc].
//
// Every mbarrier wait is bounded (globaltimer); a timeout sets
// MTC_STATUS_TIMEOUT and the CTA leaves without completing its band.
#include "mtc_common.cuh"
#include "mtc_internal.h"

namespace mtc {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxStages = 8;
constexpr uint32_t kDescBytes = 128;  // tile descriptors at the head of each stage slot
constexpr int kHeadBytes = 1024;      // barriers, flags, decoder table

struct GemvParams {
  mtc_stream_desc s;
  const float* X;
  long long ldx;
  int M;
  const int32_t* pr;
  const int32_t* pc;
  float* Y;
  long long ldy;
  float* ws;
  uint32_t* counters;
  uint32_t* status;
  int rpu;          // k-tile rows per unit
  int upb;          // units per band
  int nst;          // pipeline stages
  uint32_t slot_bytes;
  int x_stride;     // halves per token row in shared memory
  float pow2e;
  float inv_pow2e;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void flag_status(uint32_t* st, uint32_t bits) {
  if (st) atomicOr(st, bits);
}

template <int TG>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  volatile uint32_t* flags = reinterpret_cast<volatile uint32_t*>(empty + kMaxStages);  // [0] abort, [1] last
  uint32_t* dtab = reinterpret_cast<uint32_t*>(smem + 256);  // two-plane decoder table (480 B)
  __half* xs = reinterpret_cast<__half*>(smem + kHeadBytes);
  const int xs_bytes = TG * 8 * p.x_stride * 2;
  uint8_t* slots = smem + kHeadBytes + ((xs_bytes + 127) & ~127);

  const mtc_stream_desc& s = p.s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int unit = blockIdx.x;
  const int b = unit / p.upb, part = unit % p.upb;
  const int r0 = part * p.rpu;
  const int r1 = min(s.tk, r0 + p.rpu);
  const int nrows = r1 - r0;
  const uint32_t* row_off = s.row_off + (size_t)b * (s.tk + 1);

  if (tid == 0) {
    for (int i = 0; i < p.nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_barrier_init();
  }
  if (warp == 0) load_dec_table(dtab, lane);
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer: starts streaming at once ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nrows; ++i) {
        const int slot = i % p.nst, round = i / p.nst;
        if (round > 0 && !mbar_wait(&empty[slot], (round - 1) & 1, p.timeout_ns)) {
          flags[0] = 1;
          flag_status(p.status, MTC_STATUS_TIMEOUT);
          break;
        }
        if (flags[0]) break;
        const uint32_t off = row_off[r0 + i];
        const uint32_t bytes = row_off[r0 + i + 1] - off;
        if (bytes + kDescBytes > p.slot_bytes || (off & 15u) || (bytes & 15u)) {
          flags[0] = 1;
          flag_status(p.status, MTC_STATUS_BAD_STREAM);
          break;
        }
        uint8_t* dst = slots + (size_t)slot * p.slot_bytes;
        // the 16-byte descriptors of the band's tiles in this row, then the records
        const int width = min(s.band_tiles, s.tn - b * s.band_tiles);
        mbar_expect_tx(&full[slot], bytes + 16u * width);
        bulk_g2s(dst, s.tiles + (size_t)(r0 + i) * s.tn + b * s.band_tiles, 16u * width, &full[slot]);
        bulk_g2s(dst + kDescBytes, s.records + off, bytes, &full[slot]);
        ++issued;
      }
      if (flags[0]) {
        // aborting: let every copy still in flight land before the CTA exits
        for (int i = max(0, issued - p.nst); i < issued; ++i)
          (void)mbar_wait(&full[i % p.nst], (i / p.nst) & 1, 10000000ull);
      }
    }
  } else {
    // ---------------- consumers ----------------
    // Stage X[:, pr] for this unit's k range as fp16 (zero beyond M and K)
    // while the first tile rows are in flight.
    {
      const int kr = nrows * kTile;
      uint32_t bad = 0;
      for (int m = 0; m < TG * 8; ++m) {
        __half* xr = xs + m * p.x_stride;
        if (m < p.M) {
          const float* x = p.X + (long long)m * p.ldx;
          for (int kk = tid; kk < kr; kk += kConsumerWarps * 32) {
            const int k = r0 * kTile + kk;
            float v = 0.0f;
            if (k < s.K) v = x[p.pr ? p.pr[k] : k];
            if (!(fabsf(v) <= 65504.0f)) bad = 1;
            xr[kk] = __float2half_rn(v);
          }
        } else {
          for (int kk = tid; kk < kr; kk += kConsumerWarps * 32) xr[kk] = __float2half_rn(0.0f);
        }
      }
      if (bad) flag_status(p.status, MTC_STATUS_X_RANGE);
      asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
    }
    const int nt = b * s.band_tiles + warp;
    const bool active = (warp < s.band_tiles) && (nt < s.tn);
    const int g = lane >> 2, t = lane & 3;
    const GroupLane gl = make_group_lane(lane);
    const int jj = g >> 1, h = g & 1;
    float acc[2][TG][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int c = 0; c < TG; ++c)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[a][c][r] = 0.0f;

    for (int i = 0; i < nrows; ++i) {
      const int slot = i % p.nst, round = i / p.nst;
      if (flags[0]) break;
      if (!mbar_wait(&full[slot], round & 1, p.timeout_ns)) {
        flags[0] = 1;
        flag_status(p.status, MTC_STATUS_TIMEOUT);
        break;
      }
      if (active) {
        const int kt = r0 + i;
        const uint8_t* sl = slots + (size_t)slot * p.slot_bytes;
        const mtc_tile_desc d = reinterpret_cast<const mtc_tile_desc*>(sl)[warp];
        const uint32_t base = reinterpret_cast<const mtc_tile_desc*>(sl)[0].record_off;
        const uint8_t* rec = sl + kDescBytes + (d.record_off - base);
        uint32_t R[4][4];
        decode_group_w16(rec, d.n_leaves, d.prim_bytes, d.leaf_start, s.scale_words, gl, p.pow2e, dtab, R);
#pragma unroll
        for (int di = 0; di < 2; ++di) {
          const int kl = i * kTile + 4 * (2 * t + di);
#pragma unroll
          for (int tg = 0; tg < TG; ++tg) {
            const uint2 bx = *reinterpret_cast<const uint2*>(xs + (g + 8 * tg) * p.x_stride + kl);
#pragma unroll
            for (int dj = 0; dj < 2; ++dj) {
              const uint32_t* r = R[2 * di + dj];
              const uint32_t A[4] = {r[0], r[2], r[1], r[3]};
              mma_16816(acc[dj][tg], A, bx.x, bx.y);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    // partial sums of this unit -> workspace [unit][token][band col]
    if (active && !flags[0]) {
      const int bandcols = s.band_tiles * kTile;
#pragma unroll
      for (int dj = 0; dj < 2; ++dj) {
        const int fa = kTile * warp + 4 * (2 * jj + dj) + 2 * h;
#pragma unroll
        for (int tg = 0; tg < TG; ++tg) {
          const int t0 = 2 * t + 8 * tg;
          float* w0 = p.ws + ((size_t)unit * TG * 8 + t0) * bandcols;
          float* w1 = w0 + bandcols;
          w0[fa] = acc[dj][tg][0];
          w1[fa] = acc[dj][tg][1];
          w0[fa + 1] = acc[dj][tg][2];
          w1[fa + 1] = acc[dj][tg][3];
        }
      }
    }
  }
  __syncthreads();
  if (flags[0]) return;
  if (tid == 0) {
    __threadfence();
    const uint32_t old = atomicAdd(&p.counters[b], 1u);
    flags[1] = (old == (uint32_t)(p.upb - 1)) ? 1u : 0u;
  }
  __syncthreads();
  if (!flags[1]) return;
  __threadfence();
  const int bandcols = s.band_tiles * kTile;
  const int total = p.M * bandcols;
  for (int idx = tid; idx < total; idx += kThreads) {
    const int m = idx / bandcols, c = idx - m * bandcols;
    const int n = b * bandcols + c;
    if (n >= s.N) continue;
    float sum = 0.0f;
    for (int q = 0; q < p.upb; ++q)
      sum += __ldcg(p.ws + ((size_t)(b * p.upb + q) * TG * 8 + m) * bandcols + c);
    p.Y[(long long)m * p.ldy + (p.pc ? p.pc[n] : n)] = sum * p.inv_pow2e;
  }
  if (tid == 0) p.counters[b] = 0u;
}

struct Plan {
  int tg, rpu, upb, units, nst, x_stride;
  uint32_t slot_bytes;
  size_t smem, ws_bytes;
};

bool make_plan(const mtc_stream_desc* s, int M, int rows_per_unit, Plan* pl) {
  if (M < 1 || M > 16) return false;
  pl->tg = (M <= 8) ? 1 : 2;
  const int nb = (s->tn + s->band_tiles - 1) / s->band_tiles;
  int rpu = rows_per_unit;
  if (rpu <= 0) {
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long target = 4LL * sms;  // about four units per SM
    const long long rows = (long long)nb * s->tk;
    rpu = (int)((rows + target - 1) / target);
    rpu = max(1, min(rpu, 32));
  }
  rpu = min(rpu, s->tk);
  pl->rpu = rpu;
  pl->upb = (s->tk + rpu - 1) / rpu;
  pl->units = nb * pl->upb;
  pl->slot_bytes = (kDescBytes + s->max_row_bytes + 127u) & ~127u;
  pl->x_stride = rpu * kTile + 8;
  const size_t xs = ((size_t)pl->tg * 8 * pl->x_stride * 2 + 127) & ~(size_t)127;
  const size_t budget = 96 * 1024;  // leaves room for two CTAs per SM
  const size_t slot = pl->slot_bytes ? pl->slot_bytes : 1;
  int nst = (int)((budget > xs + kHeadBytes ? budget - xs - kHeadBytes : 0) / slot);
  nst = max(2, min(nst, kMaxStages));
  pl->nst = nst;
  pl->smem = kHeadBytes + xs + (size_t)nst * pl->slot_bytes;
  pl->ws_bytes = (size_t)pl->units * pl->tg * 8 * s->band_tiles * kTile * sizeof(float);
  return true;
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" size_t mtc_gemv_workspace_bytes(const mtc_stream_desc* s, int32_t M, int32_t rows_per_unit) {
  Plan pl;
  if (!s || !make_plan(s, M, rows_per_unit, &pl)) return 0;
  return pl.ws_bytes;
}

extern "C" int mtc_gemv(const mtc_stream_desc* s, const float* X, int32_t M, int64_t ldx, const int32_t* row_perm,
                        const int32_t* col_perm, float* Y, int64_t ldy, int32_t rows_per_unit, void* ws,
                        size_t ws_bytes, uint32_t* counters, uint32_t* status, void* stream) {
  clear_error();
  MTC_REQUIRE(s && X && Y && ws && counters && s->records && s->tiles && s->row_off,
              "mtc_gemv: null pointer argument");
  MTC_REQUIRE(M >= 1 && M <= 16, "mtc_gemv: M=%d outside 1..16 (use mtc_gemm_prefill)", M);
  MTC_REQUIRE(ldx >= s->K && ldy >= s->N, "mtc_gemv: bad leading dimensions");
  MTC_REQUIRE(s->band_tiles == kConsumerWarps, "mtc_gemv: stream band width %d, kernel needs %d", s->band_tiles,
              kConsumerWarps);
  MTC_REQUIRE((reinterpret_cast<uintptr_t>(s->records) & 15) == 0, "mtc_gemv: records not 16-byte aligned");
  Plan pl;
  make_plan(s, M, rows_per_unit, &pl);
  if (ws_bytes < pl.ws_bytes) {
    set_error("mtc_gemv: workspace %zu bytes, need %zu", ws_bytes, pl.ws_bytes);
    return MTC_ERR_WORKSPACE;
  }
  MTC_REQUIRE(pl.smem <= 227 * 1024, "mtc_gemv: a k-tile row of %u bytes does not fit shared memory",
              s->max_row_bytes);
  GemvParams p;
  p.s = *s;
  p.X = X;
  p.ldx = ldx;
  p.M = M;
  p.pr = row_perm;
  p.pc = col_perm;
  p.Y = Y;
  p.ldy = ldy;
  p.ws = static_cast<float*>(ws);
  p.counters = counters;
  p.status = status;
  p.rpu = pl.rpu;
  p.upb = pl.upb;
  p.nst = pl.nst;
  p.slot_bytes = pl.slot_bytes;
  p.x_stride = pl.x_stride;
  p.pow2e = ldexpf(1.0f, s->exp2);
  p.inv_pow2e = ldexpf(1.0f, -s->exp2);
  p.timeout_ns = wait_limit_ns();
  cudaStream_t st = as_stream(stream);
  // The opt-in to large dynamic shared memory is a per-device attribute:
  // set it on every call, so every device a process uses gets it.
  MTC_CHECK_CUDA(cudaFuncSetAttribute(pl.tg == 2 ? (const void*)gemv_kernel<2> : (const void*)gemv_kernel<1>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
                 "mtc_gemv: smem attribute");
  if (pl.tg == 1)
    gemv_kernel<1><<<pl.units, kThreads, pl.smem, st>>>(p);
  else
    gemv_kernel<2><<<pl.units, kThreads, pl.smem, st>>>(p);
  MTC_CHECK_LAUNCH("mtc_gemv");
  return MTC_OK;
}

// ---------------------------------------------------------------------------
// Decode GEMM without caller-provided scratch.
//
// Some callers cannot allocate device memory at the point where they run a
// decode step: code inside an allocator hook, a plugin whose host framework
// owns the device heap and hands it only input and output buffers, or a
// real-time loop that must not take the allocator's lock.  mtc_gemv_static serves them: it runs the same split-K kernel as
// mtc_gemv, with its scratch (the partial sums of the split-K units and the
// per-band tickets) taken from the fixed array below instead of from a
// workspace argument.  It calls no cudaMalloc / cudaFree.
//
// Limits and sharing:
//   * kStaticScratchBytes (8 MiB) of device memory per GPU that loads this
//     library, held until the process exits;
//   * band tickets for up to kStaticMaxBands column bands (N <= 1,048,576);
//   * the split-K row count per unit is raised until the partial sums fit;
//     a matrix whose partials cannot fit even then is rejected;
//   * every call on a device shares the array: calls that overlap on the GPU
//     (different streams, no ordering between them) race and corrupt each
//     other's results.  Calls on one stream, or otherwise ordered, are safe.
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress); make that first call before any stream capture.
// ---------------------------------------------------------------------------
namespace mtc {
namespace {
constexpr size_t kStaticScratchBytes = 8u << 20;
constexpr int kStaticMaxBands = 4096;
constexpr size_t kStaticTicketBytes = kStaticMaxBands * sizeof(uint32_t);
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];
}  // namespace
}  // namespace mtc

#include <mutex>

extern "C" int mtc_gemv_static(const mtc_stream_desc* s, const float* X, int32_t M, int64_t ldx,
                               const int32_t* row_perm, const int32_t* col_perm, float* Y, int64_t ldy,
                               uint32_t* status, void* stream) {
  clear_error();
  MTC_REQUIRE(s && X && Y && s->records && s->tiles && s->row_off, "mtc_gemv_static: null pointer argument");
  MTC_REQUIRE(M >= 1 && M <= 16, "mtc_gemv_static: M=%d outside 1..16", M);
  MTC_REQUIRE(ldx >= s->K && ldy >= s->N, "mtc_gemv_static: bad leading dimensions");
  MTC_REQUIRE(s->band_tiles == kConsumerWarps, "mtc_gemv_static: stream band width %d, kernel needs %d",
              s->band_tiles, kConsumerWarps);
  const int nb = (s->tn + s->band_tiles - 1) / s->band_tiles;
  MTC_REQUIRE(nb <= kStaticMaxBands, "mtc_gemv_static: %d column bands exceed the static limit of %d (N <= %d)", nb,
              kStaticMaxBands, kStaticMaxBands * 256);

  // Device address of the static array, looked up once per device.
  static std::mutex mu;
  static void* addr[256] = {nullptr};
  int dev = 0;
  MTC_CHECK_CUDA(cudaGetDevice(&dev), "mtc_gemv_static: cudaGetDevice");
  MTC_REQUIRE(dev >= 0 && dev < 256, "mtc_gemv_static: device index %d", dev);
  uint8_t* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "mtc_gemv_static: cudaGetSymbolAddress");
      addr[dev] = p;
    }
    base = static_cast<uint8_t*>(addr[dev]);
  }
  uint32_t* tickets = reinterpret_cast<uint32_t*>(base);
  void* partials = base + kStaticTicketBytes;
  const size_t cap = kStaticScratchBytes - kStaticTicketBytes;

  // Fewest rows per unit whose partial sums fit the array.
  Plan pl;
  make_plan(s, M, 0, &pl);
  int rpu = pl.rpu;
  while (pl.ws_bytes > cap && rpu < s->tk) {
    rpu = rpu * 2 < s->tk ? rpu * 2 : s->tk;
    make_plan(s, M, rpu, &pl);
  }
  if (pl.ws_bytes > cap) {
    set_error("mtc_gemv_static: partial sums need %zu bytes, static scratch holds %zu", pl.ws_bytes, cap);
    return MTC_ERR_WORKSPACE;
  }
  // Tickets must start at zero; a call that failed may have left some set.
  cudaStream_t st = as_stream(stream);
  MTC_CHECK_CUDA(cudaMemsetAsync(tickets, 0, nb * sizeof(uint32_t), st), "mtc_gemv_static: clear tickets");
  return mtc_gemv(s, X, M, ldx, row_perm, col_perm, Y, ldy, rpu, partials, cap, tickets, status, stream);
}
