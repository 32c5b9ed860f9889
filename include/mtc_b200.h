/*
 * mtc_b200.h -- C ABI of the B200 (sm_100a) packed-quadtree MTC GEMM library.
 *
 * The reference (Sharexi/TensorPack, "MTC") is a Python + Numba package; its
 * hot path is the packed GEMM `mtc.kernels.gemm.mtc_gemm` over an `MTCMatrix`
 * (mtc/kernels/gemm.py:217-574).  This header is the native boundary a
 * Python caller binds with ctypes: plain pointers, sizes
 * and a CUDA stream handle passed as `void*`; no C++ or torch types.
 *
 * Conventions
 *  - Every entry point returns MTC_OK (0) or a negative MTC_ERR_* code and
 *    never exits or aborts.  `mtc_last_error()` returns the message of the
 *    most recent failure on the calling thread.
 *  - All array arguments are device pointers unless noted "host".
 *  - W is the K x N weight (in_features x out_features, reduction along the
 *    rows, mtc/core/allocation.py:8-10).  The device stream stores the
 *    PERMUTED matrix Wp = W[row_perm][:, col_perm] (mtc/core/permutation.py:
 *    15-21); row_perm / col_perm may be NULL for an unpermuted matrix.
 *  - Calls enqueue work on `stream` and do not synchronise, except
 *    mtc_repack_plan which reads back one 8-byte total.
 *  - Apart from mtc_gemv_static, the library holds no global mutable state:
 *    concurrent calls on different streams with different buffers are
 *    independent.  mtc_gemv_static keeps its scratch in one array per device
 *    built into the library, so its calls must not overlap on the GPU.
 */
#ifndef MTC_B200_H
#define MTC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MTC_API __attribute__((visibility("default")))
#else
#define MTC_API
#endif

#define MTC_ABI_VERSION 2

enum {
  MTC_OK = 0,
  MTC_ERR_INVALID = -1,     /* bad argument (shape, pointer, alignment, size)  */
  MTC_ERR_CUDA = -2,        /* a CUDA runtime call failed                      */
  MTC_ERR_WORKSPACE = -3,   /* caller-provided workspace too small             */
  MTC_ERR_UNSUPPORTED = -4  /* valid request this build does not handle        */
};

/* Device status word bits (written by kernels, read by the host after sync). */
enum {
  MTC_STATUS_TIMEOUT = 1u,       /* a bounded pipeline wait gave up           */
  MTC_STATUS_X_RANGE = 2u,       /* |x| beyond the fp16 range of the tensor path */
  MTC_STATUS_BAD_STREAM = 4u     /* a tile record failed a bounds check       */
};

/* Output epilogue fused into the kernel that writes Y (pass NULL for none):
 *   Y[m][j] = act(acc[m][j] + bias[j])
 * where j is the column of Y as written (the original column for calls that
 * take a column permutation; the stored column when the output is left in
 * stored order) and acc the product.  bias may be NULL.  Replaces the
 * separate bias add of LinearMTCAdaptive.forward (mtc/nn/layers.py:146-151)
 * and the activation that follows the layer.
 *   MTC_ACT_RELU       max(x, 0)  (NaN stays NaN)
 *   MTC_ACT_SILU       x / (1 + exp(-x))
 *   MTC_ACT_GELU_TANH  0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) */
enum { MTC_ACT_NONE = 0, MTC_ACT_RELU = 1, MTC_ACT_SILU = 2, MTC_ACT_GELU_TANH = 3 };

typedef struct mtc_epilogue {
  const float* bias; /* device, one per output column, or NULL */
  int32_t act;       /* MTC_ACT_* */
  int32_t pad_;
} mtc_epilogue;

/* One quadtree leaf as handed to the GPU repack (host builds, device reads).
 * Leaves are grouped by 32x32 tile (tile-major, grid order kt*tn+nt) and
 * sorted by Z-order inside each tile; `z0` is the Z index of the leaf's first
 * 4x4 micro-block inside its tile (0..63), `size` its edge (4, 8, 16 or 32).
 * `arena_off` is the byte offset of the leaf payload in the reference-layout
 * arena: m*size*size/8 bytes, codes row-major in the leaf, LSB-first m-bit
 * two's-complement fields (mtc/kernels/gemm.py:457-478).  P0 leaves carry no
 * payload.  `scale_bits` holds the raw fp32 bits of the (signed) leaf scale;
 * quadtree allocations use bf16-exact scales (mtc/core/allocation.py:97-103,
 * mtc/core/quadtree.py:84), fixed-block ones may use any fp32 scale
 * (allocation.py:197). */
typedef struct mtc_leaf_in {
  uint32_t arena_off;
  uint32_t scale_bits;
  uint8_t mode;   /* 0, 2, 3, 4, 5, 6, 8 or 16 */
  uint8_t z0;
  uint8_t size;
  uint8_t pad_;
} mtc_leaf_in;

/* 16-byte tile descriptor of the device stream, one per 32x32 tile, indexed
 * kt*tn + nt.  The tile record at `record_off` is
 *   [leaf table: n_leaves x scale_words u32, padded to 16 B]
 *   [primary code planes: prim_bytes, padded to 16 B]
 *   [secondary code planes, padded to 16 B]
 * Leaf-table entry: bits 0-4 mode, 8-11 primary bytes per micro-block / 4,
 * 12-13 secondary bytes per micro-block / 2, 14 fp32-conversion flag,
 * 16-31 bf16 scale bits; with scale_words == 2 a second word holds the fp32
 * scale (matrices whose scales are not all bf16-exact).  `leaf_start` has
 * bit z set when a leaf starts at
 * micro-block z (Z order), so popc(leaf_start & ((2<<z)-1)) - 1 is the leaf
 * of micro-block z. */
typedef struct mtc_tile_desc {
  uint32_t record_off;
  uint16_t n_leaves;
  uint16_t prim_bytes;
  uint64_t leaf_start;
} mtc_tile_desc;

/* Device-resident tile stream of one packed matrix (all pointers device). */
typedef struct mtc_stream_desc {
  const uint8_t* records;        /* tile records, band-major: [band][kt][tile in band] */
  const mtc_tile_desc* tiles;    /* [tk * tn] */
  const uint32_t* row_off;       /* [n_bands * (tk + 1)] byte offset of each k-tile row of a band */
  int32_t K, N;                  /* logical shape of W */
  int32_t tk, tn;                /* 32x32 tiles along K and N (padded up) */
  int32_t band_tiles;            /* tiles per column band (8 = 256 output features) */
  int32_t exp2;                  /* fp16 tensor path computes with W * 2^exp2 */
  uint64_t record_bytes;         /* total bytes of `records` */
  uint32_t max_row_bytes;        /* largest k-tile row of any band */
  int32_t scale_words;           /* 1: bf16 scale in the entry, 2: extra fp32 scale word */
  /* Sub-stage images for the tensor-core kernels (NULL until
   * mtc_repack_stage_plan / _fill build them), one per sub-stage q =
   * (2 * band + half) * n_kb + kb: the four tiles 4 * half .. 4 * half + 3
   * of a band in k-tile rows 2 kb and 2 kb + 1 (n_kb = (tk + 1) / 2).  The
   * images of one half band are consecutive, so neighbouring k stages can be
   * read with one copy.  An image is what the kernels stage in shared
   * memory: [128 B tile descriptors (4 of row 2 kb, 4 of row 2 kb + 1)][work
   * list][records of row 2 kb][records of row 2 kb + 1]. */
  const uint8_t* stage_images;   /* all images, each 16-byte aligned */
  const uint32_t* stage_counts;  /* [n_sub]: group entries | micro-block entries << 16 */
  const uint32_t* stage_offsets; /* [n_sub + 1]: byte offset of each image (last = total) */
  const uint32_t* stage_ranges;  /* [n_sub][4]: image bytes, work-list bytes, row-0 record bytes, row-1 record bytes */
  uint32_t max_stage_bytes;      /* largest image */
  uint32_t max_sms;              /* at most this many SMs for the prefill kernel (0: all); leaves SMs free for
                                    work that overlaps it, such as a collective on another stream */
} mtc_stream_desc;

MTC_API int mtc_abi_version(void);
MTC_API const char* mtc_last_error(void);
MTC_API int mtc_device_sm_count(int device);

/* Limit, in ns, of every bounded pipeline wait (mbarrier, ticket) in the
 * kernels launched after this call by any thread of the process; 0 restores
 * the default of 2 s.  A wait that runs out sets MTC_STATUS_TIMEOUT, the
 * kernel drains its own copies in flight (bounded) and returns without
 * writing its output.  No counterpart in the reference (it has no GPU
 * pipeline): a diagnostic of this library, also used by its tests. */
MTC_API int mtc_set_wait_limit_ns(uint64_t ns);

/* Diagnostic for tests of the timeout path: the NEXT mtc_strip_decode call
 * (this process, any thread) makes every warp's first batch expect `bytes`
 * (a multiple of 16, at most 4096) more than it copies, so that wait can
 * never complete and runs out at the wait limit; the call after it is
 * unaffected.  0 cancels a pending hold.  No counterpart in the reference. */
MTC_API int mtc_debug_withhold_bytes(uint32_t bytes);

/* Byte copy by the copy engines (cudaMemcpyAsync, device to device) on
 * `stream`; dst or src may be a peer GPU's memory mapped into this process
 * (symmetric memory), in which case the bytes cross NVLink without using
 * SMs.  Used to move column shards of a multi-GPU GEMM into the peers'
 * buffers while the GEMM runs.  Both pointers 16-byte aligned. */
MTC_API int mtc_copy_async(void* dst, const void* src, size_t bytes, void* stream);

/* Repack step 1 (replaces the per-block offset computation of
 * MTCMatrix.from_allocation, mtc/kernels/gemm.py:449-454): measures every
 * tile record, lays the records out band-major, fills `tiles`
 * (all fields) and `row_off`, and writes out_host[0] = total record bytes and
 * out_host[1] = the largest k-tile row of any band (host array of two;
 * synchronises `stream`).  `tile_leaf_begin` is the [tk*tn + 1] CSR of
 * `leaves`; `scratch_u32` is device scratch of at least tk*tn + 6 words.
 * Fails with MTC_ERR_INVALID when the leaves of a tile do not cover its 64
 * micro-blocks exactly once in Z order. */
MTC_API int mtc_repack_plan(const mtc_leaf_in* leaves, const uint32_t* tile_leaf_begin, int32_t tk,
                    int32_t tn, int32_t band_tiles, int32_t scale_words, mtc_tile_desc* tiles,
                    uint32_t* row_off, uint32_t* scratch_u32, uint64_t* out_host, void* stream);

/* Repack step 2: transcodes every leaf's reference-layout codes
 * (mtc/kernels/gemm.py:457-478) from `arena` into the tile records
 * (4x4 micro-blocks in Z order, bit-plane split, fragment order).
 * `s` must carry the tiles / row_off filled by mtc_repack_plan and the
 * chosen exp2; `scratch_u32` is one device word.  Synchronises `stream`. */
MTC_API int mtc_repack_fill(const uint8_t* arena, uint64_t arena_bytes, const mtc_leaf_in* leaves,
                    const uint32_t* tile_leaf_begin, const mtc_stream_desc* s, uint8_t* records,
                    uint32_t* scratch_u32, void* stream);

/* Repack step 3 (tensor-core kernels): per sub-stage (half a band: four
 * tiles, in a pair of k-tile rows) an image holding the tile descriptors, a
 * work list of 64-bit entries and a copy of the records.  An 8x8 group covered by one leaf is one "group"
 * entry; a group of four 4x4 leaves becomes four "micro-block" entries.  Group
 * entries come first, then micro-block entries, each sorted by decode class
 * (0 = P0, 1..6 = P2, P3, P4, P5, P6, P8, 7 = generic: P16 or a scale not
 * exact in fp16), so prefill dequant warps take mode-uniform work.  Entry
 * bits: 0-15 primary-plane and 16-31 secondary-plane byte offsets into the
 * image's records (its row-0 part, then its row-1 part), 32-47 fp16 bits
 * of scale * 2^exp2, 48-51 class, 52-55 tile in the sub-stage (row * 4 +
 * column), 56-59 group (Z order), 60-61 micro-block in the group, 62
 * micro-block entry.
 * plan: writes `counts` (group | micro-block << 16 per sub-stage), image
 *       `offsets` (n_sub + 1 byte offsets) and `ranges` (n_sub x 4 words:
 *       image, list, row-0 record and row-1 record bytes), returns out_host =
 *       {total image bytes, largest image}; `scratch_u32` holds 5 n_sub + 2
 *       words; syncs.
 * fill: writes the images into `images` (total image bytes). */
MTC_API int mtc_repack_stage_plan(const mtc_stream_desc* s, uint32_t* counts, uint32_t* offsets,
                                  uint32_t* ranges, uint32_t* scratch_u32, uint64_t* out_host, void* stream);
MTC_API int mtc_repack_stage_fill(const mtc_stream_desc* s, const uint32_t* offsets, uint8_t* images,
                                  void* stream);

/* Exact dequantisation (replaces MTCMatrix.to_array, gemm.py:510-538, and
 * qt_dequant / permuted_qt_dequant, quadtree.py:157-171, permutation.py:
 * 76-79): out = q * scale in fp32 (__fmul_rn), bit-identical to the
 * reference.  With row_perm/col_perm non-NULL, element (k, n) of the stored
 * matrix lands at out[row_perm[k]][col_perm[n]] (original order).  `ldo` is
 * the row stride of `out` in elements. */
MTC_API int mtc_dequant(const mtc_stream_desc* s, const int32_t* row_perm, const int32_t* col_perm,
                float* out, int64_t ldo, void* stream);

/* Split-K streaming GEMM for M <= 16 (decode): Y[:, col_perm] =
 * X[:, row_perm] @ Wp (replaces mtc_gemm, gemm.py:541-574, and the
 * gather/GEMM/scatter of permutation.py:15-21).  X is M x K fp32 (row
 * stride ldx), Y is M x N fp32 (row stride ldy).  fp16 operands on the
 * tensor cores, fp32 accumulation.  `ws` / `ws_bytes` is scratch for the
 * split-K partial sums (size from mtc_gemv_workspace_bytes); `counters`
 * points at n_bands u32 that are zero before the first call and are left
 * zero by every successful call; after a call that set a status bit the
 * caller zeroes them again.  `status` (nullable) receives MTC_STATUS_*
 * bits. */
MTC_API size_t mtc_gemv_workspace_bytes(const mtc_stream_desc* s, int32_t M, int32_t rows_per_unit);
MTC_API int mtc_gemv(const mtc_stream_desc* s, const float* X, int32_t M, int64_t ldx,
             const int32_t* row_perm, const int32_t* col_perm, float* Y, int64_t ldy,
             int32_t rows_per_unit, void* ws, size_t ws_bytes, uint32_t* counters,
             uint32_t* status, void* stream);

/* Decode GEMM (M <= 16) that allocates nothing and takes no workspace.  No
 * counterpart in the reference: it exists for callers that cannot allocate
 * device memory when they run a step (an allocator hook, a real-time loop
 * that must not take the allocator's lock, or a plugin whose host framework
 * owns the device heap and only hands over inputs and outputs).  Same arguments and result as mtc_gemv minus the scratch; the
 * split-K partial sums and band tickets live in an 8 MiB array built into
 * the library (held on every GPU that loads it until process exit), which
 * limits the matrix to 4096 column bands (N <= 1,048,576) and to partial
 * sums that fit after raising the rows per split-K unit; larger requests
 * fail with MTC_ERR_WORKSPACE.  All calls on a device share that array, so
 * calls that overlap on the GPU race; calls ordered on one stream are safe.
 * The first call on each device looks up the array's address: make it
 * before any stream capture. */
MTC_API int mtc_gemv_static(const mtc_stream_desc* s, const float* X, int32_t M, int64_t ldx,
                            const int32_t* row_perm, const int32_t* col_perm, float* Y, int64_t ldy,
                            uint32_t* status, void* stream);

/* Tensor-core decode GEMM for M <= 16: Y[:, col_perm] = X[:, row_perm] @ Wp
 * (replaces mtc_gemm, gemm.py:541-574, and the gather/GEMM/scatter of
 * permutation.py:15-21).  Same product as mtc_gemv, computed swap-AB with
 * tcgen05 (D = 128 features x 16 tokens in TMEM) from the prefill's
 * class-sorted work lists (needs mtc_repack_stage_plan / _fill).  `ws`
 * (256-byte aligned, size from mtc_decode_workspace_bytes) holds the fp16
 * gathered activations and the split-K partial sums; `counters` points at
 * 2 * n_bands u32 that are zero before the first call and are left zero by
 * every successful call; after a call that set a status bit the caller
 * zeroes them again.  `status` (nullable) receives MTC_STATUS_* bits. */
MTC_API size_t mtc_decode_workspace_bytes(const mtc_stream_desc* s, int32_t M);
MTC_API int mtc_decode(const mtc_stream_desc* s, const float* X, int32_t M, int64_t ldx,
                       const int32_t* row_perm, const int32_t* col_perm, float* Y, int64_t ldy, void* ws,
                       size_t ws_bytes, uint32_t* counters, uint32_t* status, const mtc_epilogue* ep,
                       void* stream);

/* Strip stream: the decode-sized layout of a packed matrix.  A strip is 8
 * output features (stored order) over all of K; its 8x8 groups and 4x4
 * micro-blocks are sorted by precision into steps that one warp consumes
 * with straight-line code, and consecutive steps of a strip form batch
 * records that one bulk copy moves.  See tensorpack_b200/csrc/mtc_strip.cuh
 * for the byte layout.  The kernel runs a static schedule
 * (mtc_strip_schedule) that deals strips to CTAs and cuts each CTA's batch
 * records into one contiguous range per warp.  All pointers are device
 * pointers for mtc_strip_decode. */
#define MTC_STRIP_WIDE 1u         /* stream flag: group steps of 16 groups, each lane both column quartets
                                     of one group's k half (four MMAs per B fragment) */
#define MTC_STRIP_MERGE_MODES 2u  /* build flag (mtc_strip_plan / _fill only): P2 items packed with the P3
                                     decoder and P6 items with the P8 one, exactly, for fewer step kinds */

typedef struct mtc_strip_desc {
  const uint8_t* stream;        /* batch records, 16-byte aligned */
  const uint32_t* batch_off;    /* [n_batches + 1] byte offset of each batch record (last = total) */
  const uint32_t* strip_batch;  /* [n_strips + 1] first batch of each strip (last = n_batches) */
  const uint32_t* work;         /* [2 n_batches] schedule: per batch record in warp order {byte offset,
                                   (bytes / 16) | slot << 12 | flush << 31} (mtc_strip_schedule) */
  const uint32_t* warp_work;    /* [n_cta n_warps + 1] first work item of each warp */
  const uint32_t* red;          /* [3 n_strips] {strip, first slot, slot count}, grouped by CTA */
  const uint32_t* cta_red;      /* [n_cta + 1] first `red` entry of each CTA */
  int32_t K, N;                 /* logical shape of W */
  int32_t tk, tn;               /* 32x32 tiles along K and N (padded up) */
  int32_t n_strips, n_batches;  /* n_strips = 4 tn */
  int32_t exp2;                 /* the stream's scales are scale * 2^exp2 */
  uint32_t max_batch_bytes;     /* largest batch record */
  int32_t n_cta, n_warps;       /* schedule grid: CTAs (1..n_strips) x warps per CTA */
  uint32_t max_cta_slots;       /* most partial-sum slots (strip segments) of one CTA */
  uint32_t flags;               /* MTC_STRIP_* flags the stream was built with */
  uint64_t stream_bytes;
} mtc_strip_desc;

/* Build the strip stream on the HOST from the leaf list the repack reads
 * (mtc_leaf_in, tile CSR and the reference-layout arena of
 * MTCMatrix.from_allocation, mtc/kernels/gemm.py:449-478).  All pointers are
 * host pointers; no CUDA call is made.  `exp2` pre-scales every scale by
 * 2^exp2 (choose it so the largest |scale| * 2^exp2 is at most 1); leaves of
 * P16 or whose pre-scaled scale is not exact in fp16 take the fp32 path.
 * Batch records hold at most `batch_bytes` bytes (2048..65536, multiple of
 * 16) and `batch_steps` steps.  `flags`: MTC_STRIP_WIDE and / or
 * MTC_STRIP_MERGE_MODES (the latter is not a stream flag: the descriptor and
 * the validator take only MTC_STRIP_WIDE).
 * plan: out4 = {stream bytes, n_batches, n_strips, largest batch record}.
 * fill: writes `stream` (stream bytes), `batch_off` (n_batches + 1) and
 *       `strip_batch` (n_strips + 1). */
MTC_API int mtc_strip_plan(const mtc_leaf_in* leaves, const uint32_t* tile_leaf_begin, int32_t tk, int32_t tn,
                           int32_t exp2, uint32_t batch_bytes, uint32_t batch_steps, uint32_t flags,
                           uint64_t* out4);
MTC_API int mtc_strip_fill(const uint8_t* arena, uint64_t arena_bytes, const mtc_leaf_in* leaves,
                           const uint32_t* tile_leaf_begin, int32_t tk, int32_t tn, int32_t exp2,
                           uint32_t batch_bytes, uint32_t batch_steps, uint32_t flags, uint8_t* stream,
                           uint32_t* batch_off, uint32_t* strip_batch);

/* Validate a host strip stream (record offsets and sizes, strip ranges,
 * every step descriptor and entry row) before it is uploaded; the decode
 * kernel relies on it.  Host pointers; returns MTC_ERR_INVALID with a
 * message naming the first bad record. */
MTC_API int mtc_strip_check(const uint8_t* stream, uint64_t stream_bytes, const uint32_t* batch_off,
                            const uint32_t* strip_batch, int32_t n_batches, int32_t n_strips, int32_t tk,
                            uint32_t max_batch_bytes, uint32_t flags);

/* Static schedule of a strip stream for mtc_strip_decode on `n_cta` CTAs
 * (1..n_strips, normally the SM count) of `n_warps` warps (host pointers, no
 * CUDA call).  Strips go to CTAs by estimated decode cost (longest first,
 * each to the least loaded CTA); each CTA's batch records, in strip order,
 * are cut into n_warps contiguous ranges of equal estimated cost.  The part
 * of a strip that one warp holds is a segment with its own partial-sum slot;
 * the last work item of a segment carries the flush bit.  Outputs (host
 * arrays sized by the caller): work [2 n_batches], warp_work
 * [n_cta n_warps + 1], red [3 n_strips], cta_red [n_cta + 1] and the most
 * slots of one CTA.  The stream must have passed mtc_strip_check. */
MTC_API int mtc_strip_schedule(const uint8_t* stream, const uint32_t* batch_off, const uint32_t* strip_batch,
                               int32_t n_strips, int32_t n_cta, int32_t n_warps, uint32_t flags, uint32_t* work,
                               uint32_t* warp_work, uint32_t* red, uint32_t* cta_red, uint32_t* max_slots);

/* 1 when mtc_strip_decode can run this stream at M tokens (the gathered
 * activations, M x K fp16, the partial-sum slots and the batch slots of the
 * schedule's warps fit shared memory), else 0.
 * Host-only query, no CUDA call. */
MTC_API int mtc_strip_fits(const mtc_strip_desc* s, int32_t M);

/* Decode GEMM over the strip stream for M <= 4: Y[:, col_perm] =
 * X[:, row_perm] @ Wp (replaces mtc_gemm, gemm.py:541-574, and the
 * gather/GEMM/scatter of permutation.py:15-21).  X is M x K fp32, Y is
 * M x N fp32.  Products are q * fp16(fp16(x) * fp16(scale * 2^exp2)) on
 * the tensor cores (mma.sync, fp32 accumulation); the fp32 path computes
 * q * (fp16(x) * scale * 2^exp2) in fp32.  The launch is s->n_cta CTAs of
 * s->n_warps warps running the descriptor's schedule; partial sums live in
 * shared memory, so the call takes no workspace and leaves no state behind.
 * `status` (nullable) receives MTC_STATUS_* bits. */
MTC_API int mtc_strip_decode(const mtc_strip_desc* s, const float* X, int32_t M, int64_t ldx,
                             const int32_t* row_perm, const int32_t* col_perm, float* Y, int64_t ldy,
                             uint32_t* status, const mtc_epilogue* ep, void* stream);

/* Fused dequant + tcgen05 GEMM for prefill-sized M (any M >= 1; used for
 * M > 16): Y[:, col_perm] = X[:, row_perm] @ Wp (replaces mtc_gemm,
 * gemm.py:541-574, and permutation.py:15-21).  Takes the INVERSE column
 * permutation (col_perm_inv[col_perm[n]] = n, NULL when unpermuted).  fp16
 * operands, fp32 TMEM accumulation.  `ws` (256-byte aligned) holds the fp16
 * gathered activations and, for permuted matrices, the permuted output; its
 * size comes from mtc_prefill_workspace_bytes(s, M, col_perm_inv != NULL).
 * Requires K, N <= 51200. */
MTC_API size_t mtc_prefill_workspace_bytes(const mtc_stream_desc* s, int32_t M, int32_t permuted);
MTC_API int mtc_gemm_prefill(const mtc_stream_desc* s, const float* X, int32_t M, int64_t ldx,
                             const int32_t* row_perm, const int32_t* col_perm_inv, float* Y,
                             int64_t ldy, void* ws, size_t ws_bytes, uint32_t* status,
                             const mtc_epilogue* ep, void* stream);

/* The three stages mtc_gemm_prefill runs, for callers that fuse or time them
 * separately (same workspace):
 *   gather:  ws <- fp16 X[:, row_perm] (padded to tk*32 columns)
 *   gemm:    fused dequant + tcgen05 GEMM of that; writes Y directly
 *            (permuted_output = 0; the epilogue `ep` is applied there) or the
 *            permuted-column product into ws (permuted_output = 1; `ep` must
 *            then be NULL and is given to the scatter instead)
 *   scatter: Y[:, col_perm] <- epilogue of the permuted-column product in ws */
MTC_API int mtc_prefill_gather(const mtc_stream_desc* s, const float* X, int32_t M, int64_t ldx,
                               const int32_t* row_perm, void* ws, size_t ws_bytes, uint32_t* status,
                               void* stream);
MTC_API int mtc_prefill_gemm(const mtc_stream_desc* s, int32_t M, float* Y, int64_t ldy,
                             int32_t permuted_output, void* ws, size_t ws_bytes, uint32_t* status,
                             const mtc_epilogue* ep, void* stream);
MTC_API int mtc_prefill_scatter(const mtc_stream_desc* s, int32_t M, const int32_t* col_perm_inv,
                                float* Y, int64_t ldy, void* ws, size_t ws_bytes, const mtc_epilogue* ep,
                                void* stream);

/* Row-wise column gather: Y[m][j] = row_m[pos[j]] with row_m the
 * concatenation of nseg segments src[g*seg_stride + m*ldp + (0..seg_len-1)]
 * (M rows, N output columns).  Used to assemble all-gathered column shards
 * of a multi-GPU GEMM in original column order. */
MTC_API int mtc_permute_rows(const float* src, int64_t seg_stride, int64_t ldp, int32_t nseg,
                             int32_t seg_len, const int32_t* pos, int32_t N, int32_t M, float* Y,
                             int64_t ldy, const mtc_epilogue* ep, void* stream);

/* GPU candidate search of the rate-distortion allocators (replaces the Numba
 * _search_kernel / _search_mode, mtc/core/allocation.py:106-160, used by
 * rd_candidates and QuadtreeRD): for every block_size x block_size block of
 * the K x N fp32 matrix W (row-major) and precision `mode`, the scale among
 * sign x alpha * amax / qmax (bf16-rounded when bf16_scales) minimising
 * sum_r h_norm[r] * sum_c (w - q s)^2.  Writes (K/bs) x (N/bs) fp64
 * distortions and fp32 scales; bit-identical to the reference. */
MTC_API int mtc_rd_search(const float* W, int32_t K, int32_t N, int32_t block_size, const double* h_norm,
                          int32_t mode, const float* alphas, int32_t n_alpha, int32_t bf16_scales,
                          double* out_dist, float* out_scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MTC_B200_H */
