// Host builder of the strip stream (layout in mtc_strip.cuh).
//
// Input is the same leaf list the GPU repack reads (struct mtc_leaf_in, tile
// CSR, reference-layout arena: mtc/kernels/gemm.py:449-478); the output is a
// host byte stream the caller uploads.  The build is pure host code, so the
// format can be produced and checked without a GPU.  Strips are independent
// and built on all host threads: a plan pass sizes every strip, a fill pass
// writes them at their prefix-sum offsets.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <thread>
#include <vector>

#include "mtc_internal.h"
#include "mtc_strip.cuh"

namespace mtc {
namespace {

using namespace strip;

__host__ inline int zidx(int i, int j) {
  return (((i >> 2) & 1) << 5) | (((j >> 2) & 1) << 4) | (((i >> 1) & 1) << 3) | (((j >> 1) & 1) << 2) |
         ((i & 1) << 1) | (j & 1);
}
__host__ inline int zrow(int z) { return (((z >> 5) & 1) << 2) | (((z >> 3) & 1) << 1) | ((z >> 1) & 1); }
__host__ inline int zcol(int z) { return (((z >> 4) & 1) << 2) | (((z >> 2) & 1) << 1) | (z & 1); }

struct Ctx {
  const mtc_leaf_in* leaves;
  const uint32_t* begin;  // [tk * tn + 1]
  int tk, tn, exp2;
  const uint8_t* arena;
  uint64_t arena_bytes;
  uint32_t batch_bytes, batch_steps;
  bool wide;   // group steps of 16 groups, two micro-blocks per lane
  bool merge;  // P2 items packed as P3 and P6 items as P8 (fewer step kinds)
};

// Decoder class of a leaf mode, after the optional merge of P2 into P3 and
// P6 into P8 (their codes lie inside the wider ranges, so they are exact).
__host__ inline int packed_class(const Ctx& c, int mode) {
  const int cls = class_of_mode(mode);
  if (!c.merge) return cls;
  return cls == 0 ? 1 : cls == 4 ? 5 : cls;
}

// One item of a strip: a group (8 k x 8 features) or a micro-block (4 x 4).
struct Item {
  uint32_t leaf;  // global leaf index
  int row;        // group: group row (8 k); micro / generic: micro-block row (4 k)
  int kt;         // tile row of the item
};

struct Step {
  int kind, n0, n1;
  int first0, first1;  // first item of each list (group steps: first0 only)
};

struct StripPlan {
  std::vector<Item> grp[6], mic[6][2], gen[2];
  std::vector<Step> steps;
  std::vector<int> batch_first;  // first step of each batch (+ end)
  std::vector<uint32_t> batch_size;
  bool bad = false;
};

// fp16 bits of scale * 2^exp2 when that value is exact in fp16, else -1.
__host__ inline int exact_f16(float scale, int exp2) {
  const float f = ldexpf(scale, exp2);
  if (!isfinite(f)) return -1;
  const uint16_t h = f2h(f);
  if (h2f(h) != f) return -1;
  return (int)h;
}

__host__ bool plan_strip(const Ctx& c, int strip, StripPlan* P) {
  const int nt = strip >> 2, gj = strip & 3;
  int leaf_of_z[64];
  for (int kt = 0; kt < c.tk; ++kt) {
    const int tile = kt * c.tn + nt;
    const uint32_t l0 = c.begin[tile], l1 = c.begin[tile + 1];
    for (int z = 0; z < 64; ++z) leaf_of_z[z] = -1;
    for (uint32_t l = l0; l < l1; ++l) {
      const mtc_leaf_in& L = c.leaves[l];
      const int nmb = (L.size / 4) * (L.size / 4);
      if (L.size % 4 || L.z0 + nmb > 64) return false;
      for (int z = L.z0; z < L.z0 + nmb; ++z) leaf_of_z[z] = (int)l;
    }
    for (int gi = 0; gi < 4; ++gi) {
      int mb[2][2];  // [kr][h]
      for (int a = 0; a < 2; ++a)
        for (int h = 0; h < 2; ++h) {
          mb[a][h] = leaf_of_z[zidx(2 * gi + a, 2 * gj + h)];
          if (mb[a][h] < 0) return false;
        }
      const int grow = kt * 4 + gi;
      const bool uniform = mb[0][0] == mb[0][1] && mb[0][0] == mb[1][0] && mb[0][0] == mb[1][1];
      if (uniform) {
        const mtc_leaf_in& L = c.leaves[mb[0][0]];
        if (L.mode == 0) continue;
        float sc;
        memcpy(&sc, &L.scale_bits, 4);
        const int cls = packed_class(c, L.mode);
        if (cls >= 0 && exact_f16(sc, c.exp2) >= 0) {
          P->grp[cls].push_back(Item{(uint32_t)mb[0][0], grow, kt});
        } else {
          for (int a = 0; a < 2; ++a)
            for (int h = 0; h < 2; ++h) P->gen[h].push_back(Item{(uint32_t)mb[a][h], 2 * grow + a, kt});
        }
        continue;
      }
      for (int a = 0; a < 2; ++a)
        for (int h = 0; h < 2; ++h) {
          const mtc_leaf_in& L = c.leaves[mb[a][h]];
          if (L.mode == 0) continue;
          float sc;
          memcpy(&sc, &L.scale_bits, 4);
          const int cls = packed_class(c, L.mode);
          const Item it{(uint32_t)mb[a][h], 2 * grow + a, kt};
          if (cls >= 0 && exact_f16(sc, c.exp2) >= 0)
            P->mic[cls][h].push_back(it);
          else
            P->gen[h].push_back(it);
        }
    }
  }
  // steps in kind order
  const int gmax = group_step_max(c.wide);
  for (int cls = 0; cls < 6; ++cls) {
    const int n = (int)P->grp[cls].size();
    for (int i = 0; i < n; i += gmax) P->steps.push_back(Step{kG2 + cls, std::min(gmax, n - i), 0, i, 0});
  }
  auto split_steps = [&](int kind, const std::vector<Item>& L0, const std::vector<Item>& L1) {
    const int a = (int)L0.size(), b = (int)L1.size();
    for (int i = 0; i < std::max(a, b); i += 16)
      P->steps.push_back(Step{kind, std::max(0, std::min(16, a - i)), std::max(0, std::min(16, b - i)), i, i});
  };
  for (int cls = 0; cls < 6; ++cls) split_steps(kU2 + cls, P->mic[cls][0], P->mic[cls][1]);
  split_steps(kGeneric, P->gen[0], P->gen[1]);
  // batches: consecutive steps while the record fits batch_bytes / batch_steps
  const int ns = (int)P->steps.size();
  int i = 0;
  do {
    P->batch_first.push_back(i);
    int cnt = 0;
    uint32_t body = 0;
    while (i < ns) {
      const Step& s = P->steps[i];
      const uint32_t sb = (uint32_t)step_bytes(s.kind, s.n0, s.n1);
      const uint32_t hdr = (uint32_t)pad16(8 + 4 * (cnt + 1));
      if (cnt > 0 && (hdr + body + sb > c.batch_bytes || (uint32_t)cnt + 1 > c.batch_steps)) break;
      if (hdr + body + sb > c.batch_bytes) P->bad = true;  // one step larger than a batch
      body += sb;
      ++cnt;
      ++i;
    }
    P->batch_size.push_back((uint32_t)pad16(8 + 4 * cnt) + body);
  } while (i < ns);
  P->batch_first.push_back(ns);
  return true;
}

// Signed m-bit code of element (r, col) of leaf L (stored-matrix coordinates).
__host__ inline int leaf_code(const Ctx& c, const mtc_leaf_in& L, int kt, int nt, int r, int col) {
  const int zr = zrow(L.z0), zc = zcol(L.z0);
  const int lr = r - (kt * 32 + zr * 4), lc = col - (nt * 32 + zc * 4);
  const uint64_t idx = (uint64_t)lr * L.size + lc;
  const int m = L.mode;
  const uint64_t bit = (uint64_t)L.arena_off * 8 + idx * m;
  uint32_t u = 0;
  for (int i = 0; i < m; ++i) {
    const uint64_t b = bit + i;
    u |= (uint32_t)((c.arena[b >> 3] >> (b & 7)) & 1u) << i;
  }
  return (int)(u << (32 - m)) >> (32 - m);
}

// Codes q[r][cc] of the micro-block at micro row `mrow` and micro column
// `mcol` (global), taken from leaf L of tile row kt.
__host__ inline void micro_codes(const Ctx& c, const mtc_leaf_in& L, int kt, int mrow, int mcol, int q[4][4]) {
  const int nt = mcol >> 3;
  for (int r = 0; r < 4; ++r)
    for (int cc = 0; cc < 4; ++cc) q[r][cc] = leaf_code(c, L, kt, nt, mrow * 4 + r, mcol * 4 + cc);
}

}  // namespace


namespace {

__host__ bool fill_strip(const Ctx& c, int strip, const StripPlan& P, uint8_t* out, uint32_t base,
                         uint32_t* batch_off, uint32_t batch_base) {
  uint32_t off = base;
  const int nb = (int)P.batch_size.size();
  for (int bi = 0; bi < nb; ++bi) {
    batch_off[batch_base + bi] = off;
    uint8_t* rec = out + off;
    const int s0 = P.batch_first[bi], s1 = P.batch_first[bi + 1];
    const int cnt = s1 - s0;
    memset(rec, 0, P.batch_size[bi]);
    const uint32_t hdr[2] = {(uint32_t)strip, (uint32_t)cnt};
    memcpy(rec, hdr, 8);
    uint8_t* st = rec + pad16(8 + 4 * cnt);
    for (int si = s0; si < s1; ++si) {
      const Step& S = P.steps[si];
      const int sb = step_bytes(S.kind, S.n0, S.n1);
      // run of identical full steps starting here (only its first descriptor is read)
      int run = 1;
      if (full_counts(S.kind, S.n0, S.n1, c.wide)) {
        const bool head = si == s0 || P.steps[si - 1].kind != S.kind ||
                          !full_counts(P.steps[si - 1].kind, P.steps[si - 1].n0, P.steps[si - 1].n1, c.wide);
        if (head)
          while (si + run < s1 && run < kMaxRun && P.steps[si + run].kind == S.kind &&
                 full_counts(S.kind, P.steps[si + run].n0, P.steps[si + run].n1, c.wide))
            ++run;
      }
      const uint32_t d = make_desc(S.kind, S.n0, S.n1, sb, run, c.wide);
      memcpy(rec + 8 + 4 * (si - s0), &d, 4);
      int q[4][4];
      if (S.kind < kU2 && c.wide) {
        // wide group step: lane 2 gs + kr holds quartets 0 and 1 of group gs, k half kr
        const int cls = S.kind, n = S.n0, PB = prim_bytes(cls), SB = sec_bytes(cls), lanes = 2 * n;
        uint8_t* planes = st + pad16(4 * n);
        for (int gs = 0; gs < n; ++gs) {
          const Item& it = P.grp[cls][S.first0 + gs];
          const mtc_leaf_in& L = c.leaves[it.leaf];
          float sc;
          memcpy(&sc, &L.scale_bits, 4);
          const uint32_t e = (uint32_t)exact_f16(sc, c.exp2) | ((uint32_t)it.row << 16);
          memcpy(st + 4 * gs, &e, 4);
          for (int kr = 0; kr < 2; ++kr) {
            const int lane = 2 * gs + kr;
            for (int h = 0; h < 2; ++h) {
              micro_codes(c, L, it.kt, 2 * it.row + kr, 2 * strip + h, q);
              uint32_t A[4], B;
              if (!pack_lane(cls, q, A, &B)) return false;
              memcpy(planes + lane * 2 * PB + h * PB, A, PB);
              if (SB == 2) {
                const uint16_t b16 = (uint16_t)((B & 0xFFu) | ((B >> 8) & 0xFF00u));
                memcpy(planes + lanes * 2 * PB + lane * 4 + h * 2, &b16, 2);
              } else if (SB == 4) {
                memcpy(planes + lanes * 2 * PB + lane * 8 + h * 4, &B, 4);
              }
            }
          }
        }
      } else if (S.kind < kU2) {
        const int cls = S.kind, n = S.n0, PB = prim_bytes(cls), SB = sec_bytes(cls);
        uint8_t* planes = st + pad16(4 * n);
        for (int gs = 0; gs < n; ++gs) {
          const Item& it = P.grp[cls][S.first0 + gs];
          const mtc_leaf_in& L = c.leaves[it.leaf];
          float sc;
          memcpy(&sc, &L.scale_bits, 4);
          const uint32_t e = (uint32_t)exact_f16(sc, c.exp2) | ((uint32_t)it.row << 16);
          memcpy(st + 4 * gs, &e, 4);
          for (int h = 0; h < 2; ++h)
            for (int kr = 0; kr < 2; ++kr) {
              const int idx = 2 * gs + kr + h * 2 * n;
              micro_codes(c, L, it.kt, 2 * it.row + kr, 2 * strip + h, q);
              uint32_t A[4], B;
              if (!pack_lane(cls, q, A, &B)) return false;
              memcpy(planes + idx * PB, A, PB);
              if (SB == 2) {
                const uint16_t b16 = (uint16_t)((B & 0xFFu) | ((B >> 8) & 0xFF00u));
                memcpy(planes + 4 * n * PB + idx * 2, &b16, 2);
              } else if (SB == 4) {
                memcpy(planes + 4 * n * PB + idx * 4, &B, 4);
              }
            }
        }
      } else {
        const int nl = S.n0 + S.n1;
        for (int j = 0; j < nl; ++j) {
          const int h = j < S.n0 ? 0 : 1;
          const int li = h ? S.first1 + (j - S.n0) : S.first0 + j;
          const Item& it = (S.kind == kGeneric) ? P.gen[h][li] : P.mic[S.kind - kU2][h][li];
          const mtc_leaf_in& L = c.leaves[it.leaf];
          micro_codes(c, L, it.kt, it.row, 2 * strip + h, q);
          float sc;
          memcpy(&sc, &L.scale_bits, 4);
          if (S.kind == kGeneric) {
            const float f = ldexpf(sc, c.exp2);
            uint32_t e[2];
            memcpy(&e[0], &f, 4);
            e[1] = (uint32_t)it.row | ((uint32_t)L.mode << 16);
            memcpy(st + 8 * j, e, 8);
            uint8_t* slot = st + pad16(8 * nl) + kGenericSlot * j;
            const int m = L.mode;
            for (int r = 0; r < 4; ++r)
              for (int cc = 0; cc < 4; ++cc) {
                const uint32_t u = (uint32_t)q[r][cc] & ((1u << m) - 1u);
                const int bit0 = (4 * r + cc) * m;
                for (int i = 0; i < m; ++i)
                  if ((u >> i) & 1u) slot[(bit0 + i) >> 3] |= (uint8_t)(1u << ((bit0 + i) & 7));
              }
          } else {
            const int cls = S.kind - kU2, PB = prim_bytes(cls), SB = sec_bytes(cls);
            const uint32_t e = (uint32_t)exact_f16(sc, c.exp2) | ((uint32_t)it.row << 16);
            memcpy(st + 4 * j, &e, 4);
            uint8_t* planes = st + pad16(4 * nl);
            uint32_t A[4], B;
            if (!pack_lane(cls, q, A, &B)) return false;
            memcpy(planes + j * PB, A, PB);
            if (SB == 2) {
              const uint16_t b16 = (uint16_t)((B & 0xFFu) | ((B >> 8) & 0xFF00u));
              memcpy(planes + nl * PB + j * 2, &b16, 2);
            } else if (SB == 4) {
              memcpy(planes + nl * PB + j * 4, &B, 4);
            }
          }
        }
      }
      st += sb;
    }
    off += P.batch_size[bi];
  }
  return true;
}

template <class F>
void parallel_for(int n, F f) {
  const int nth = std::max(1, std::min((int)std::thread::hardware_concurrency(), 32));
  std::atomic<int> next(0);
  auto work = [&]() {
    for (int i; (i = next.fetch_add(1)) < n;) f(i);
  };
  std::vector<std::thread> th;
  for (int t = 1; t < nth; ++t) th.emplace_back(work);
  work();
  for (auto& t : th) t.join();
}

int check_args(const mtc_leaf_in* leaves, const uint32_t* begin, int32_t tk, int32_t tn, uint32_t batch_bytes,
               uint32_t batch_steps, uint32_t flags, const char* who) {
  MTC_REQUIRE((flags & ~(kWide | kMergeModes)) == 0, "%s: unknown stream flags 0x%x", who, flags);
  MTC_REQUIRE(leaves && begin, "%s: null pointer argument", who);
  MTC_REQUIRE(tk >= 1 && tn >= 1, "%s: bad tile grid %d x %d", who, tk, tn);
  MTC_REQUIRE(tk * 8 <= 65535, "%s: K of %d tiles exceeds the 16-bit micro-block row", who, tk);
  MTC_REQUIRE(batch_bytes >= 2048 && batch_bytes % 16 == 0 && batch_bytes <= 65536,
              "%s: batch_bytes %u must be a multiple of 16 in 2048..65536", who, batch_bytes);
  MTC_REQUIRE(batch_steps >= 1 && batch_steps <= 1024, "%s: batch_steps %u outside 1..1024", who, batch_steps);
  return MTC_OK;
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" int mtc_strip_plan(const mtc_leaf_in* leaves, const uint32_t* tile_leaf_begin, int32_t tk, int32_t tn,
                              int32_t exp2, uint32_t batch_bytes, uint32_t batch_steps, uint32_t flags,
                              uint64_t* out4) {
  clear_error();
  int rc = check_args(leaves, tile_leaf_begin, tk, tn, batch_bytes, batch_steps, flags, "mtc_strip_plan");
  if (rc) return rc;
  MTC_REQUIRE(out4, "mtc_strip_plan: null out4");
  const Ctx c{leaves, tile_leaf_begin, tk, tn, exp2, nullptr, 0, batch_bytes, batch_steps, (flags & kWide) != 0,
              (flags & kMergeModes) != 0};
  const int n_strips = tn * 4;
  std::vector<uint64_t> bytes(n_strips), nb(n_strips), mx(n_strips);
  std::atomic<int> bad(0);
  parallel_for(n_strips, [&](int s) {
    StripPlan P;
    if (!plan_strip(c, s, &P) || P.bad) {
      bad = 1;
      return;
    }
    uint64_t t = 0, m = 0;
    for (uint32_t b : P.batch_size) t += b, m = std::max<uint64_t>(m, b);
    bytes[s] = t, nb[s] = P.batch_size.size(), mx[s] = m;
  });
  MTC_REQUIRE(!bad, "mtc_strip_plan: leaves do not tile every 32x32 tile, or a step exceeds batch_bytes");
  uint64_t tb = 0, tnb = 0, tmx = 0;
  for (int s = 0; s < n_strips; ++s) tb += bytes[s], tnb += nb[s], tmx = std::max(tmx, mx[s]);
  MTC_REQUIRE(tb < (1ull << 32), "mtc_strip_plan: stream of %llu bytes exceeds 4 GiB", (unsigned long long)tb);
  out4[0] = tb;
  out4[1] = tnb;
  out4[2] = (uint64_t)n_strips;
  out4[3] = tmx;
  return MTC_OK;
}

extern "C" int mtc_strip_fill(const uint8_t* arena, uint64_t arena_bytes, const mtc_leaf_in* leaves,
                              const uint32_t* tile_leaf_begin, int32_t tk, int32_t tn, int32_t exp2,
                              uint32_t batch_bytes, uint32_t batch_steps, uint32_t flags, uint8_t* stream,
                              uint32_t* batch_off, uint32_t* strip_batch) {
  clear_error();
  int rc = check_args(leaves, tile_leaf_begin, tk, tn, batch_bytes, batch_steps, flags, "mtc_strip_fill");
  if (rc) return rc;
  MTC_REQUIRE(arena && stream && batch_off && strip_batch, "mtc_strip_fill: null pointer argument");
  const int n_strips = tn * 4;
  // payloads inside the arena
  const uint32_t nleaves = tile_leaf_begin[tk * tn];
  for (uint32_t l = 0; l < nleaves; ++l) {
    const mtc_leaf_in& L = leaves[l];
    const uint64_t need = (uint64_t)L.arena_off + (uint64_t)L.mode * L.size * L.size / 8;
    MTC_REQUIRE(L.mode == 0 || need <= arena_bytes, "mtc_strip_fill: leaf %u payload beyond the arena", l);
    MTC_REQUIRE(L.mode == 0 || L.mode == 2 || L.mode == 3 || L.mode == 4 || L.mode == 5 || L.mode == 6 ||
                    L.mode == 8 || L.mode == 16,
                "mtc_strip_fill: leaf %u has mode %d", l, (int)L.mode);
  }
  const Ctx c{leaves, tile_leaf_begin, tk, tn, exp2, arena, arena_bytes, batch_bytes, batch_steps,
              (flags & kWide) != 0, (flags & kMergeModes) != 0};
  std::vector<StripPlan> plans(n_strips);
  std::atomic<int> bad(0);
  parallel_for(n_strips, [&](int s) {
    if (!plan_strip(c, s, &plans[s]) || plans[s].bad) bad = 1;
  });
  MTC_REQUIRE(!bad, "mtc_strip_fill: leaves do not tile every 32x32 tile, or a step exceeds batch_bytes");
  std::vector<uint32_t> base(n_strips + 1, 0);
  strip_batch[0] = 0;
  for (int s = 0; s < n_strips; ++s) {
    uint64_t t = 0;
    for (uint32_t b : plans[s].batch_size) t += b;
    base[s + 1] = base[s] + (uint32_t)t;
    strip_batch[s + 1] = strip_batch[s] + (uint32_t)plans[s].batch_size.size();
  }
  parallel_for(n_strips, [&](int s) {
    if (!fill_strip(c, s, plans[s], stream, base[s], batch_off, strip_batch[s])) bad = 1;
    plans[s] = StripPlan();  // release the item lists as strips finish
  });
  MTC_REQUIRE(!bad, "mtc_strip_fill: a code placement recipe collided (library bug)");
  batch_off[strip_batch[n_strips]] = base[n_strips];
  return MTC_OK;
}

// Host-side validation of a strip stream before it is uploaded: record
// offsets and sizes, strip ranges, every step descriptor against the layout,
// and every entry's k row against the matrix.  The kernel trusts what passes.
extern "C" int mtc_strip_check(const uint8_t* stream, uint64_t stream_bytes, const uint32_t* batch_off,
                               const uint32_t* strip_batch, int32_t n_batches, int32_t n_strips, int32_t tk,
                               uint32_t max_batch_bytes, uint32_t flags) {
  clear_error();
  MTC_REQUIRE((flags & ~kWide) == 0, "mtc_strip_check: unknown stream flags 0x%x", flags);
  const bool wide = (flags & kWide) != 0;
  MTC_REQUIRE(stream && batch_off && strip_batch, "mtc_strip_check: null pointer argument");
  MTC_REQUIRE(n_strips >= 1 && n_batches >= n_strips && tk >= 1, "mtc_strip_check: bad sizes");
  MTC_REQUIRE(strip_batch[0] == 0 && (int64_t)strip_batch[n_strips] == n_batches,
              "mtc_strip_check: strip ranges do not cover the batches");
  MTC_REQUIRE((uint64_t)batch_off[n_batches] <= stream_bytes, "mtc_strip_check: records beyond the stream");
  for (int s = 0; s < n_strips; ++s) {
    MTC_REQUIRE(strip_batch[s + 1] > strip_batch[s], "mtc_strip_check: strip %d has no batch record", s);
    for (uint32_t b = strip_batch[s]; b < strip_batch[s + 1]; ++b) {
      const uint32_t off = batch_off[b], end = batch_off[b + 1];
      MTC_REQUIRE(end > off && (off & 15u) == 0 && ((end - off) & 15u) == 0 && end - off <= max_batch_bytes,
                  "mtc_strip_check: batch %u has a bad offset or size", b);
      const uint8_t* rec = stream + off;
      const uint32_t size = end - off;
      MTC_REQUIRE(ldu32(rec) == (uint32_t)s, "mtc_strip_check: batch %u names strip %u, not %d", b, ldu32(rec), s);
      const uint32_t nst = ldu32(rec + 4);
      MTC_REQUIRE((uint64_t)pad16(8 + 4 * (int)std::min<uint32_t>(nst, 1u << 20)) <= size,
                  "mtc_strip_check: batch %u step table beyond the record", b);
      uint32_t pos = (uint32_t)pad16(8 + 4 * (int)nst);
      for (uint32_t i = 0; i < nst; ++i) {
        const uint32_t d = ldu32(rec + 8 + 4 * i);
        const int kind = desc_kind(d), n0 = desc_n0(d), n1 = desc_n1(d), sb = desc_bytes(d);
        MTC_REQUIRE(kind < kKinds, "mtc_strip_check: batch %u step %u kind %d", b, i, kind);
        if (kind < kU2)
          MTC_REQUIRE(n0 >= 1 && n0 <= group_step_max(wide) && n1 == 0, "mtc_strip_check: batch %u step %u group count",
                      b, i);
        else
          MTC_REQUIRE(n0 <= 16 && n1 <= 16 && n0 + n1 >= 1, "mtc_strip_check: batch %u step %u counts", b, i);
        MTC_REQUIRE(sb == step_bytes(kind, n0, n1) && pos + (uint32_t)sb <= size,
                    "mtc_strip_check: batch %u step %u size", b, i);
        MTC_REQUIRE(desc_full(d) == full_counts(kind, n0, n1, wide), "mtc_strip_check: batch %u step %u full flag", b,
                    i);
        const int run = desc_run(d);
        MTC_REQUIRE(run >= 1 && (run == 1 || desc_full(d)) && i + (uint32_t)run <= nst,
                    "mtc_strip_check: batch %u step %u run length %d", b, i, run);
        for (int r = 1; r < run; ++r)
          MTC_REQUIRE(((ldu32(rec + 8 + 4 * (i + r)) ^ d) & 0x3FFFFFu) == 0,
                      "mtc_strip_check: batch %u step %u run of unlike steps", b, i);
        const uint8_t* st = rec + pos;
        const int nent = kind < kU2 ? n0 : n0 + n1;
        for (int j = 0; j < nent; ++j) {
          if (kind == kGeneric) {
            const uint32_t e1 = ldu32(st + 8 * j + 4);
            const int md = (int)((e1 >> 16) & 31u);
            MTC_REQUIRE((int)(e1 & 0xFFFFu) < 8 * tk && (class_of_mode(md) >= 0 || md == 16),
                        "mtc_strip_check: batch %u step %u generic entry %d", b, i, j);
          } else {
            const int row = (int)(ldu32(st + 4 * j) >> 16);
            MTC_REQUIRE(row < (kind < kU2 ? 4 * tk : 8 * tk), "mtc_strip_check: batch %u step %u entry %d row", b,
                        i, j);
          }
        }
        pos += (uint32_t)sb;
      }
      MTC_REQUIRE(pos == size, "mtc_strip_check: batch %u steps do not fill the record", b);
    }
  }
  return MTC_OK;
}

// Static schedule of a strip stream for the decode kernel.
//
// Cost model, in units of about one warp instruction at full issue, fitted
// to per-batch clock counts of the kernel on the Llama-3-8B gate layer: a
// step costs its decode by class (more for the micro-block layout and for
// classes with a secondary plane), every dispatch (the head of a run of full
// steps, or a partial step) adds the latency of reading and branching on its
// descriptor, a generic step runs the fp32 path, and every batch record adds
// its header and loop.  Only ratios matter: the schedule balances estimated
// warp time, not bytes.
__host__ inline int sched_step_cost(uint32_t d, bool wide) {
  const int kind = desc_kind(d);
  if (kind == kGeneric) return 170;
  static const int group_cost[6] = {30, 50, 28, 42, 42, 30};  // P2, P3, P4, P5, P6, P8
  static const int micro_cost[6] = {32, 40, 32, 40, 40, 32};
  int body = kind < kU2 ? group_cost[kind] : micro_cost[kind - kU2];
  if (wide && kind < kU2) body = body * 3 / 2;  // two micro-blocks per lane, one x load
  return body;
}
constexpr int kSchedBatchCost = 50;
constexpr int kSchedDispatchCost = 83;

// Cut costs c[0..n) into `parts` contiguous ranges whose largest sum is as
// small as possible (binary search on that sum, greedy fill); cut[w] is the
// first element of range w, cut[parts] = n.
__host__ inline void optimal_cuts(const std::vector<uint64_t>& c, int parts, std::vector<size_t>* cut) {
  const size_t n = c.size();
  uint64_t lo = 0, hi = 0;
  for (uint64_t v : c) lo = std::max(lo, v), hi += v;
  auto fits = [&](uint64_t cap) {
    int used = 1;
    uint64_t acc = 0;
    for (uint64_t v : c) {
      if (acc + v > cap) {
        ++used;
        acc = 0;
      }
      acc += v;
    }
    return used <= parts;
  };
  while (lo < hi) {
    const uint64_t mid = lo + (hi - lo) / 2;
    if (fits(mid)) hi = mid;
    else lo = mid + 1;
  }
  cut->assign(parts + 1, n);
  (*cut)[0] = 0;
  int w = 1;
  uint64_t acc = 0;
  for (size_t i = 0; i < n && w < parts; ++i) {
    if (acc + c[i] > lo) {
      (*cut)[w++] = i;
      acc = 0;
    }
    acc += c[i];
  }
}

namespace {
int schedule_impl(const uint8_t* stream, const uint32_t* batch_off, const uint32_t* strip_batch, int n_strips,
                  int n_cta, int n_warps, bool wide, uint32_t* work, uint32_t* warp_work, uint32_t* red,
                  uint32_t* cta_red, uint32_t* max_slots_out) {
  const int n_batches = (int)strip_batch[n_strips];
  // estimated cost of every batch record
  std::vector<uint64_t> bcost(n_batches);
  for (int b = 0; b < n_batches; ++b) {
    const uint8_t* rec = stream + batch_off[b];
    const uint32_t nst = ldu32(rec + 4);
    uint64_t c = kSchedBatchCost;
    for (uint32_t i = 0; i < nst;) {
      const uint32_t d = ldu32(rec + 8 + 4 * i);
      const uint32_t run = (uint32_t)std::max(1, desc_run(d));
      c += kSchedDispatchCost + (uint64_t)run * sched_step_cost(d, wide);
      i += run;
    }
    bcost[b] = c;
  }
  // strips to CTAs: longest first, each to the least loaded CTA
  std::vector<uint64_t> scost(n_strips, 0);
  for (int s = 0; s < n_strips; ++s)
    for (uint32_t b = strip_batch[s]; b < strip_batch[s + 1]; ++b) scost[s] += bcost[b];
  std::vector<int> order(n_strips);
  for (int s = 0; s < n_strips; ++s) order[s] = s;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return scost[a] > scost[b]; });
  std::vector<uint64_t> load(n_cta, 0);
  std::vector<std::vector<int>> cta_strips(n_cta);
  for (int s : order) {
    int best = 0;
    for (int c = 1; c < n_cta; ++c)
      if (load[c] < load[best]) best = c;
    load[best] += scost[s];
    cta_strips[best].push_back(s);
  }
  uint32_t wi = 0, ri = 0, max_slots = 0;
  for (int c = 0; c < n_cta; ++c) {
    std::vector<int>& st = cta_strips[c];
    std::sort(st.begin(), st.end());
    std::vector<uint32_t> seq;  // batches of this CTA in order
    for (int s : st)
      for (uint32_t b = strip_batch[s]; b < strip_batch[s + 1]; ++b) seq.push_back(b);
    // cut seq into n_warps contiguous ranges, the costliest as cheap as possible
    std::vector<uint64_t> sc(seq.size());
    for (size_t i = 0; i < seq.size(); ++i) sc[i] = bcost[seq[i]];
    std::vector<size_t> cut;
    optimal_cuts(sc, n_warps, &cut);
    // work items and flush slots: a segment is one warp's run of one strip
    uint32_t slot = 0;
    std::vector<uint32_t> strip_first(st.size(), 0), strip_cnt(st.size(), 0);
    size_t sidx = 0;  // index into st of the strip at seq position
    std::vector<int> strip_at(seq.size());
    {
      size_t k = 0;
      for (size_t j = 0; j < st.size(); ++j)
        for (uint32_t b = strip_batch[st[j]]; b < strip_batch[st[j] + 1]; ++b) strip_at[k++] = (int)j;
    }
    (void)sidx;
    for (int w = 0; w < n_warps; ++w) {
      warp_work[c * n_warps + w] = wi;
      for (size_t i = cut[w]; i < cut[w + 1]; ++i) {
        const uint32_t b = seq[i];
        const int j = strip_at[i];
        const bool first_of_seg = i == cut[w] || strip_at[i - 1] != j;
        const bool last_of_seg = i + 1 == cut[w + 1] || strip_at[i + 1] != j;
        if (first_of_seg) {
          if (strip_cnt[j] == 0) strip_first[j] = slot;
          ++strip_cnt[j];
        }
        const uint32_t bytes = batch_off[b + 1] - batch_off[b];
        work[2 * wi] = batch_off[b];
        work[2 * wi + 1] = (bytes >> 4) | (slot << 12) | (last_of_seg ? 0x80000000u : 0u);
        ++wi;
        if (last_of_seg) ++slot;
      }
    }
    cta_red[c] = ri;
    for (size_t j = 0; j < st.size(); ++j) {
      red[3 * ri] = (uint32_t)st[j];
      red[3 * ri + 1] = strip_first[j];
      red[3 * ri + 2] = strip_cnt[j];
      ++ri;
    }
    max_slots = std::max(max_slots, slot);
  }
  warp_work[n_cta * n_warps] = wi;
  cta_red[n_cta] = ri;
  *max_slots_out = max_slots;
  return MTC_OK;
}
}  // namespace

extern "C" int mtc_strip_schedule(const uint8_t* stream, const uint32_t* batch_off, const uint32_t* strip_batch,
                                  int32_t n_strips, int32_t n_cta, int32_t n_warps, uint32_t flags, uint32_t* work,
                                  uint32_t* warp_work, uint32_t* red, uint32_t* cta_red, uint32_t* max_slots) {
  clear_error();
  MTC_REQUIRE(stream && batch_off && strip_batch && work && warp_work && red && cta_red && max_slots,
              "mtc_strip_schedule: null pointer argument");
  MTC_REQUIRE(n_strips >= 1 && n_cta >= 1 && n_cta <= n_strips && n_warps >= 1 && n_warps <= 32,
              "mtc_strip_schedule: bad sizes (%d strips, %d CTAs, %d warps)", n_strips, n_cta, n_warps);
  MTC_REQUIRE((flags & ~kWide) == 0, "mtc_strip_schedule: unknown stream flags 0x%x", flags);
  for (int s = 0; s < n_strips; ++s)
    MTC_REQUIRE(strip_batch[s + 1] > strip_batch[s], "mtc_strip_schedule: strip %d has no batch record", s);
  const uint32_t n_batches = strip_batch[n_strips];
  for (uint32_t b = 0; b < n_batches; ++b) {
    const uint32_t bytes = batch_off[b + 1] - batch_off[b];
    MTC_REQUIRE(batch_off[b + 1] > batch_off[b] && (bytes & 15u) == 0 && bytes <= 65520u && (batch_off[b] & 15u) == 0,
                "mtc_strip_schedule: batch %u has a bad offset or size", b);
  }
  MTC_REQUIRE(n_batches < (1u << 19), "mtc_strip_schedule: %u batch records exceed the slot field", n_batches);
  return schedule_impl(stream, batch_off, strip_batch, n_strips, n_cta, n_warps, (flags & kWide) != 0, work,
                       warp_work, red, cta_red, max_slots);
}
