/* C ABI of libhtrc_flat.so: the flat (tree-free) HTRC attention operator for NVIDIA B200 (sm_100a).
 *
 * Every pointer is a device pointer on the current CUDA device unless stated otherwise; the caller
 * owns all memory.  No entry point allocates device memory or synchronises the stream, so a whole
 * forward call can be captured in a CUDA graph once the library has been initialised on the device
 * (the first call of any entry point on a device sets kernel attributes; make it before capture).
 * Return value: HTRC_OK (0) or one of the HTRC_ERR_* codes; htrc_strerror() names them.  Errors
 * detected on the device (a bounded wait that gave up, an out-of-range leaf index, a non-finite
 * log-partition) are OR-ed into a status word that htrc_flat_status() reads back.
 *
 * Layouts (row-major, contiguous unless a pitch is given):
 *   q [N, D] f32 or bf16;  k, v [M, D] bf16;  D = 128;  M a multiple of `leaf`.
 *   Tiles of `tile` = 64 (or 32) query rows; nt = ceil(N / tile); the last tile is padded with repeats
 *   of the last query row.  Every tile is held as 64 rows (q8/dq8/sq/sdq [nt*64, ...]); a 32-row tile's
 *   rows 32..63 repeat its row 31.  nb = M / leaf leaves.  Per-(tile, leaf) scalars use the leaf pitch
 *   P = htrc_leaf_pitch(nb) (nb rounded up to 16).
 *   Groups: G consecutive tiles share one expansion centre, one far-field state row and one routing
 *   (G = 1 by default); ng = ceil(nt / G) state rows.  The per-(tile, leaf) arrays below are then
 *   per-(group, leaf).
 *   Order: with HTRC_ORDER_KMEANS the query rows are first reordered by a k-means permutation perm
 *   (tile row i holds query perm[i]) and the output is written back in the caller's row order.
 */
#ifndef HTRC_FLAT_H_
#define HTRC_FLAT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* htrc_stream_t; /* a cudaStream_t; NULL is the legacy default stream */

enum {
  HTRC_OK = 0,
  HTRC_ERR_ARG = 1,         /* invalid argument (shape, dtype, null pointer, range) */
  HTRC_ERR_UNSUPPORTED = 2, /* valid for the reference but not implemented by this library */
  HTRC_ERR_WORKSPACE = 3,   /* workspace missing or smaller than htrc_flat_workspace_size() */
  HTRC_ERR_CUDA = 4,        /* a CUDA runtime call failed (launch, attribute, tensor map) */
  HTRC_ERR_DEVICE = 5,      /* no sm_100 device, or the device status word reported a failure */
  HTRC_ERR_TOO_LARGE = 6    /* htrc_flat_forward_static_ws: the problem needs more than its 64 MiB */
};

enum { HTRC_DTYPE_F32 = 0, HTRC_DTYPE_BF16 = 1 };
enum { HTRC_ORDER_SEQ = 0, HTRC_ORDER_KMEANS = 1 };
enum { HTRC_CURV_LIN = 0, HTRC_CURV_ISO = 1 };
enum { HTRC_ROUND_HALF_EVEN = 0, HTRC_ROUND_HALF_AWAY = 1 };
enum { HTRC_FQ_INT8 = 1, HTRC_FQ_INT4 = 2, HTRC_FQ_FP8 = 3, HTRC_FQ_FP4 = 4 }; /* htrc_fake_quant formats */
enum { HTRC_STORE_INT8 = 0, HTRC_STORE_FP8 = 1, HTRC_STORE_BF16 = 2 };       /* far-field state format */
/* Arithmetic flags (HtrcFlatArgs.precision and the stage entry points' `precision`), OR-ed:
 * the leaf-statistics dots (the reference's precision= argument, h3/htrc_flat.py:101, :126-130):
 *   HTRC_PREC_FP32 ("fp32", the reference's PREC "ieee"): float32-accurate products (bf16 hi + lo splits of
 *   the float32 centre and softmax weights); HTRC_PREC_TF32 ("tf32", PROD's setting, h3/htrc_flat.py:391): the
 *   float32 operands enter as tf32, their low 13 mantissa bits cleared, the way the reference's tensor-core
 *   dots (h3/htrc_flat_triton.py:57, :62-63) read them on sm_100;
 * the division that forms the query and offset codes (x / s, h3/htrc_flat_triton.py:110-117) and the INT8
 * slope factor 127 / am (:75-77) or the fp8 state values g / sg, vbar / sv (:65-72):
 *   IEEE division without HTRC_PREC_TRITON_DIV (the reference's formula as written; its CPU-recorded
 *   fixtures); with HTRC_PREC_TRITON_DIV, PTX div.full.f32, what the reference's Triton kernels compute for
 *   `/` on the GPU (so the codes match its GPU operator's).  The key codes (a torch division,
 *   h3/htrc_flat.py:213-219) are IEEE in both. */
enum { HTRC_PREC_FP32 = 0, HTRC_PREC_TF32 = 1, HTRC_PREC_TRITON_DIV = 2 };

/* Device status bits (htrc_flat_status). */
enum { HTRC_STATUS_WAIT_TIMEOUT = 1, HTRC_STATUS_BAD_INDEX = 2, HTRC_STATUS_NONFINITE = 4 };

/* Arguments of one head of the operator. */
typedef struct HtrcFlatArgs {
  const void* q;           /* [n_queries, dim], q_dtype */
  int32_t q_dtype;         /* HTRC_DTYPE_F32 or HTRC_DTYPE_BF16 */
  const uint16_t* k;       /* [n_keys, dim] bf16 */
  const uint16_t* v;       /* [n_keys, dim] bf16 */
  int64_t n_queries;       /* N >= 1 */
  int64_t n_keys;          /* M, a positive multiple of leaf */
  int32_t dim;             /* D, must be 128 */
  int32_t tile;            /* query tile rows: 64, or 32 (the "max" mode; held as 64 rows, rows 32..63
                              repeating row 31) */
  int32_t leaf;            /* key leaf tokens: 64, or 32 / 16 with store INT8 and curvature LIN */
  int32_t exact_leaves;    /* E >= 0: leaves evaluated exactly per tile (clamped to nb) */
  int32_t sink_leaves;     /* leading leaves always exact (clamped to nb) */
  int32_t tile_chunk;      /* tiles per chunk of the far-field state (<= 0: all tiles at once) */
  float scale;             /* logit scale; <= 0 selects 1/sqrt(dim) */
  const float* tail_k;     /* [n_tail, dim] f32 keys past the last full leaf, or NULL */
  const float* tail_v;     /* [n_tail, dim] f32 */
  int32_t n_tail;          /* >= 0 */
  void* workspace;         /* device workspace, 256-byte aligned; its first 256 bytes (the status word)
                              must be zero when first used -- htrc_flat_status() clears them */
  size_t workspace_bytes;  /* >= htrc_flat_workspace_size(args) */
  float* out;              /* [n_queries, dim] f32 output */
  float* lse;              /* [n_queries] f32 log-partition (logit units), or NULL */
  /* Optional stage timing: cudaEvent_t handles recorded on the stream at fixed points (NULL = none):
   * [0] start, [1] after key pack + tile prep + tail, then per tile chunk c:
   * [2+4c] after leaf stats, [3+4c] after row-max, [4+4c] after routing, [5+4c] after the tile kernel.
   * Points past n_stage_events are not recorded. */
  void* const* stage_events;
  int32_t n_stage_events;
  int32_t group;           /* G consecutive tiles share one centre, state and routing (<= 1: one tile;
                              the reference's kern["group"], h3/htrc_flat.py:223-231) */
  int32_t order;           /* HTRC_ORDER_SEQ, or HTRC_ORDER_KMEANS: query rows grouped by a k-means
                              permutation first (order="kmeans", h3/htrc_flat.py:47-65, :146-147) */
  int32_t curvature;       /* HTRC_CURV_LIN (the production far field lz + g.dq), or HTRC_CURV_ISO: plus
                              the isotropic second-order term 0.5/D max(tr, 0) |q - mu|^2 with
                              tr = scale^2 (sum w |k|^2 - |sum w k|^2) per (centre, leaf) -- the torch
                              backend's curvature="iso" (h3/htrc_flat.py:331-333) on the INT8 path */
  int32_t store;           /* HTRC_STORE_INT8 (store="int8": INT8 state and INT8 query/key codes), or
                              HTRC_STORE_FP8 (store="fp8", h3/htrc_flat_triton.py FP8=1: e4m3 state codes with
                              row scales, fp16 far-field dots, bf16 near field; needs HTRC_CURV_LIN), or
                              HTRC_STORE_BF16 (store="bf16", :82-84: bf16 state without scales, bf16 far- and
                              near-field dots; needs HTRC_CURV_LIN and leaf 64) */
  int32_t qk_scale_block;  /* 0: the reference's INT8 scales (per key, per query row); 64: an extension with no
                              reference counterpart, one scale per 64 keys (a leaf) and per query tile
                              (one absmax scale per 64-token block); HTRC_STORE_INT8 only */
  uint8_t* route_mask;     /* optional debug export (NULL = none): [ceil(nt / group), P] uint8 routing masks, the
                              rows htrc_route writes (1 = the leaf is evaluated exactly for that centre row) */
  int32_t precision;       /* HTRC_PREC_* flags: tf32 statistics operands, Triton (div.full.f32) code division */
} HtrcFlatArgs;

/* nb rounded up to a multiple of 16: the row pitch of the per-(tile, leaf) scalar arrays. */
int64_t htrc_leaf_pitch(int64_t nb);

/* Workspace bytes one htrc_flat_forward call with these arguments needs (pointers are ignored). */
int htrc_flat_workspace_size(const HtrcFlatArgs* args, size_t* bytes);

/* The whole operator for one head: INT8 key pack, tile centres and query codes, leaf statistics,
 * row-max selection, top-E routing, far field + near field + tail, normalised output and log-Z
 * (store HTRC_STORE_FP8: the fp8 stage entry points below instead of the INT8 ones, no key pack).
 * Replaces flat_attention(q, k, v, backend="triton", store="int8"|"fp8", dot="bf16", select="max",
 * tile=64|32, leaf=64|32|16, exact_leaves=E, sink_leaves=S, tail=(tk, tv), order="seq"|"kmeans",
 * kern={"group": G}) of the reference (h3/htrc_flat.py:99-124 -> _flat_triton :181-276), plus the
 * log-Z output the reference lacks. */
int htrc_flat_forward(const HtrcFlatArgs* args, htrc_stream_t stream);

/* Read back (synchronously) and clear the device status word inside `workspace`. */
int htrc_flat_status(void* workspace, int32_t* status_out, htrc_stream_t stream);

/* ---- stage entry points (the same kernels htrc_flat_forward launches), for parity tests ---- */

/* Per-row INT8 pack of x [rows, dim]: scale = max(amax_row|x| * (1/127), 1e-20).
 * HTRC_ROUND_HALF_EVEN: x8 = clamp(rint(x / scale), -127, 127)   (h3/htrc_flat.py:216-218, keys)
 * HTRC_ROUND_HALF_AWAY: x8 = trunc(x / scale +- 0.5)              (h3/htrc_flat_triton.py:110-117) */
int htrc_pack_int8(const void* x, int32_t dtype, int64_t rows, int32_t dim, int32_t rounding, int8_t* x8,
                   float* scale, float* sqnorm, htrc_stream_t stream);   /* sqnorm: NULL or [rows] |x_row|^2 */

/* Tile centres and query codes (h3/htrc_flat.py:142-156 `_tiles`, :223-231 groups;
 * h3/htrc_flat_triton.py:103-117):
 * mu [ng, dim] f32; group 1: the mean of the tile's real rows; group G > 1: the mean of all G*tile rows of
 * the group, the last tile's padding rows and the repeats of the last tile that fill the last group
 * included (float64 sum rounded once); mu_hi/mu_lo [ng, dim] bf16 with mu_hi = bf16(mu),
 * mu_lo = bf16(mu - mu_hi);
 * q8/dq8 [nt*64, dim] int8 and sq/sdq [nt*64] f32: half-away codes of q and of q - mu[tile / G].
 * tile: 64 or 32; perm: NULL, or [n_queries] int32 (query i in tile order is row perm[i] of q). */
int htrc_tile_prep(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, int32_t tile, const int32_t* perm,
                   int32_t group, float* mu, uint16_t* mu_hi, uint16_t* mu_lo, int8_t* q8, float* sq, int8_t* dq8,
                   float* sdq, float* dd, htrc_stream_t stream);   /* dd: NULL or [nt*64] |q - mu|^2 (f32) */

/* k-means query order (h3/htrc_flat.py:47-65 `kmeans_order`: 32 clusters, Lloyd's iterations x 8 on
 * the rows round(linspace(0, N-1, min(4096, N))) seeded with sample rows round(linspace(0, S-1, 32)),
 * then the nearest centre of every row and a stable sort of the rows by centre): perm [n_queries]
 * int32.  Distances are exact float32 sums of squared differences (the reference's torch.cdist expands
 * |x|^2 - 2 x.c + |c|^2), ties go to the lower centre.  scratch: htrc_kmeans_scratch_size() bytes,
 * 256-byte aligned. */
int htrc_kmeans_scratch_size(int64_t n_queries, size_t* bytes);
int htrc_kmeans_order(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, int32_t* perm, void* scratch,
                      size_t scratch_bytes, htrc_stream_t stream);

/* Leaf statistics of centre rows [t0, t0 + tc) (h3/htrc_flat_triton.py:41-85 `_stats_kernel`, I8 store):
 * g8 [tc, nb, dim] int8 and sg/lz [tc, P] f32, vb [tc, nb, dim] bf16.  mu_hi/mu_lo as written by
 * htrc_tile_prep / htrc_tile_prep_ex (all nt centre rows: tiles, or groups of tiles); precision: HTRC_PREC_*
 * for the softmax weights of the second dot (the centres' precision is set where mu_hi/mu_lo are written);
 * leaf: 64, 32 or 16 (kn2 / cv only with 64); status: device int32 word or NULL. */
int htrc_leaf_stats(const uint16_t* mu_hi, const uint16_t* mu_lo, int64_t nt, int64_t t0, int64_t tc,
                    const uint16_t* k, const uint16_t* v, int64_t n_keys, int32_t dim, int32_t leaf, float scale,
                    int8_t* g8, float* sg, float* lz, uint16_t* vb, const float* kn2, float* cv, int32_t precision,
                    int32_t* status, htrc_stream_t stream);
/* kn2 / cv: both NULL, or the key norms |k|^2 [n_keys] (htrc_pack_int8's sqnorm) and the iso curvature
 * coefficients cv [tc, P] f32 = 0.5/D max(tr, 0) to write. */

/* Row-max selection sel [tc, P] f32 of tiles [t0, t0 + tc) (h3/htrc_flat_triton.py:214-254
 * `_rowmax_kernel`, I8): sel[t, l] = max_r (dq8_r . g8_l) * (sdq_r * sg_l) + lz_l over the tile's 64
 * rows, with the state row (t - t0) / group of g8/sg/lz (t0 a multiple of group).  The maximum over a
 * group's tiles is taken by htrc_route. */
int htrc_rowmax_select(const int8_t* dq8, const float* sdq, const float* dd, int64_t t0, int64_t tc, int32_t group,
                       const int8_t* g8, const float* sg, const float* lz, const float* cv, int64_t nb, int32_t dim,
                       float* sel, int32_t* status, htrc_stream_t stream);
/* dd / cv: both NULL, or the iso curvature inputs: each logit gains cv_l * dd_r before the maximum. */

/* Top-E routing of the groups of tiles [0, tc) (h3/htrc_flat.py:250-265): a group's selection is the
 * maximum of its tiles' sel rows (the reference's row-max over all G*64 rows); the first sink_leaves
 * leaves are forced, then the largest; kx = min(exact_leaves + sink_leaves, nb).  idx [ceil(tc/G), kx]
 * int32 in ascending leaf order (ties broken towards the lower leaf index); excl [ceil(tc/G), P] uint8
 * (1 = routed). */
int htrc_route(const float* sel, int64_t tc, int64_t nb, int32_t exact_leaves, int32_t sink_leaves, int32_t group,
               int32_t* idx, uint8_t* excl, htrc_stream_t stream);

/* Far field + near field (+ tail partial) of tiles [t0, t0 + tc) merged into out/lse rows
 * [t0*64, min(n_queries, (t0+tc)*64)) (h3/htrc_flat_triton.py:88-211 `_tile_kernel` with I8=1,
 * merged as :257-273).  State arrays as produced by the stages above (state row (t - t0) / group; t0 a
 * multiple of group); k8/ks from htrc_pack_int8 (half-even) of k; tail_part: NULL or
 * [n_queries, dim + 2] f32 rows (acc, m, l) from the tail, in the caller's row order; perm: NULL, or the
 * permutation given to htrc_tile_prep (query i in tile order is written to out/lse row perm[i]); tile: the
 * tile rows given to htrc_tile_prep; leaf: 64, 32 or 16 (cv / dd only with 64). */
int htrc_tile_attention(const int8_t* q8, const float* sq, const int8_t* dq8, const float* sdq, int64_t n_queries,
                        int32_t tile, int64_t t0, int64_t tc, int32_t group, const int8_t* g8, const float* sg,
                        const float* lz,
                        const uint16_t* vb, const uint8_t* excl, const int32_t* idx, int32_t kx, int64_t nb,
                        const int8_t* k8, const float* ks, const uint16_t* v, int64_t n_keys, int32_t dim,
                        int32_t leaf, float scale, const float* tail_part, const int32_t* perm, const float* cv,
                        const float* dd, float* out, float* lse, int32_t* status, htrc_stream_t stream);
/* cv / dd: both NULL, or the iso curvature inputs (each far logit gains cv_l * dd_r). */

/* Exact softmax partial of every query row against the tail keys (h3/htrc_flat_triton.py:187-207 for
 * n_tail <= 16 with bf16 operands; :381-388 float32 for longer tails): tail_part [N, dim + 2]. */
int htrc_tail_partial(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, const float* tail_k,
                      const float* tail_v, int32_t n_tail, float scale, float* tail_part, htrc_stream_t stream);

/* Per-block INT8 pack (extension, no reference counterpart): as htrc_pack_int8, with one scale per block of
 * block_rows (= 64) consecutive rows, s = max(amax_block|x| * (1/127), 1e-20), written for every row. */
int htrc_pack_int8_blocks(const void* x, int32_t dtype, int64_t rows, int32_t dim, int32_t rounding,
                          int32_t block_rows, int8_t* x8, float* scale, float* sqnorm, htrc_stream_t stream);

/* htrc_tile_prep with q_scale_block = 0 (the same codes) or 64 (extension): the codes q8 of a tile's rows
 * share one scale from the tile's abs-max (sq holds it for every row); dq8 / sdq stay per row.  precision
 * HTRC_PREC_TF32: mu_hi + mu_lo = mu with its low 13 mantissa bits cleared, exactly (HTRC_PREC_FP32: as
 * htrc_tile_prep); mu itself and the codes are the same for both. */
int htrc_tile_prep_ex(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, int32_t tile,
                      const int32_t* perm, int32_t group, float* mu, uint16_t* mu_hi, uint16_t* mu_lo, int8_t* q8,
                      float* sq, int8_t* dq8, float* sdq, float* dd, int32_t q_scale_block, int32_t precision,
                      htrc_stream_t stream);

/* ---- stage entry points of the fp8 state path (HTRC_STORE_FP8) ---- */

/* Tile centres as htrc_tile_prep, with the fp8 path's query operands (h3/htrc_flat_triton.py:103-109):
 * qb [nt*64, dim] bf16 rows of q and dqh [nt*64, dim] fp16 = fp16(q - mu[tile / G]) (float32 offsets
 * rounded once). */
int htrc_tile_prep_fp8(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, int32_t tile,
                       const int32_t* perm, int32_t group, float* mu, uint16_t* mu_hi, uint16_t* mu_lo, uint16_t* qb,
                       uint16_t* dqh, int32_t precision, htrc_stream_t stream);   /* precision: as htrc_tile_prep_ex */

/* Leaf statistics of centre rows [t0, t0 + tc) with the fp8 state (h3/htrc_flat_triton.py:41-85, FP8=1):
 * g8 [tc, nb, dim] e4m3 codes of g / sg, sg = max(amax|g| * (1/448), 1e-30); vb8 [tc, nb, dim] e4m3 codes
 * of vbar / sv with sv likewise; lz, sg, sv [tc, P] f32.  Codes are nearest even, saturated at 448. */
int htrc_leaf_stats_fp8(const uint16_t* mu_hi, const uint16_t* mu_lo, int64_t nt, int64_t t0, int64_t tc,
                        const uint16_t* k, const uint16_t* v, int64_t n_keys, int32_t dim, int32_t leaf, float scale,
                        uint8_t* g8, float* sg, float* lz, uint8_t* vb8, float* sv, int32_t precision,
                        int32_t* status, htrc_stream_t stream);   /* precision: as htrc_leaf_stats */

/* Row-max selection with the fp8 state (h3/htrc_flat_triton.py:214-254, FP8=1):
 * sel[t, l] = max_r (dqh_r . g_l) * sg_l + lz_l over the tile's 64 rows (fp16 operands, float32 sums);
 * state row (t - t0) / group as htrc_rowmax_select. */
int htrc_rowmax_select_fp8(const uint16_t* dqh, int64_t t0, int64_t tc, int32_t group, const uint8_t* g8,
                           const float* sg, const float* lz, int64_t nb, int32_t dim, float* sel, int32_t* status,
                           htrc_stream_t stream);

/* Far field + near field (+ tail partial) with the fp8 state (h3/htrc_flat_triton.py:88-211, FP8=1, DOT=1,
 * merged as :257-273): far logit (dqh . g) * sg + lz with value weight fp16(p * sv) on the vbar codes,
 * near logit (qb . bf16 k) * scale with weight bf16(p) on v.  Two launches: the far field writes one
 * partial row (acc, m, l) per query into far_part [n_queries, dim + 2] f32 (scratch; NULL only when
 * kx == nb), the near field merges it with the tail partial into out/lse.  Other arguments as
 * htrc_tile_attention (k, v: the bf16 keys and values). */
int htrc_tile_attention_fp8(const uint16_t* qb, const uint16_t* dqh, int64_t n_queries, int32_t tile, int64_t t0,
                            int64_t tc, int32_t group, const uint8_t* g8, const float* sg, const float* lz,
                            const uint8_t* vb8, const float* sv, const uint8_t* excl, const int32_t* idx, int32_t kx,
                            int64_t nb, const uint16_t* k, const uint16_t* v, int64_t n_keys, int32_t dim,
                            int32_t leaf, float scale, const float* tail_part, const int32_t* perm,
                            float* far_part, float* out, float* lse, int32_t* status, htrc_stream_t stream);

/* ---- stage entry points of the bf16 state path (HTRC_STORE_BF16) ---- */

/* Tile centres as htrc_tile_prep, with the bf16 state's query operands (h3/htrc_flat_triton.py:106-107):
 * qb [nt*64, dim] bf16 rows of q and dqb [nt*64, dim] bf16 = bf16(q - mu[tile / G]) (float32 offsets rounded
 * once). */
int htrc_tile_prep_bf16(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, int32_t tile,
                        const int32_t* perm, int32_t group, float* mu, uint16_t* mu_hi, uint16_t* mu_lo, uint16_t* qb,
                        uint16_t* dqb, int32_t precision, htrc_stream_t stream);   /* precision: as htrc_tile_prep_ex */

/* Leaf statistics of centre rows [t0, t0 + tc) with the bf16 state (h3/htrc_flat_triton.py:41-85, :82-84):
 * gb [tc, nb, dim] bf16 = bf16(scale * sum w k), vbb [tc, nb, dim] bf16 = bf16(sum w v), lz [tc, P] f32; leaf
 * 64. */
int htrc_leaf_stats_bf16(const uint16_t* mu_hi, const uint16_t* mu_lo, int64_t nt, int64_t t0, int64_t tc,
                         const uint16_t* k, const uint16_t* v, int64_t n_keys, int32_t dim, int32_t leaf, float scale,
                         uint16_t* gb, float* lz, uint16_t* vbb, int32_t precision, int32_t* status,
                         htrc_stream_t stream);   /* precision: as htrc_leaf_stats */

/* Row-max selection with the bf16 state (h3/htrc_flat_triton.py:214-254, DOT=1):
 * sel[t, l] = max_r (dqb_r . g_l) + lz_l over the tile's 64 rows (bf16 operands, float32 sums); state row
 * (t - t0) / group as htrc_rowmax_select. */
int htrc_rowmax_select_bf16(const uint16_t* dqb, int64_t t0, int64_t tc, int32_t group, const uint16_t* gb,
                            const float* lz, int64_t nb, int32_t dim, float* sel, int32_t* status,
                            htrc_stream_t stream);

/* Far field + near field (+ tail partial) with the bf16 state (h3/htrc_flat_triton.py:88-211, DOT=1, merged
 * as :257-273): far logit (dqb . g) + lz with weight bf16(p) on vbar, near logit (qb . bf16 k) * scale with
 * weight bf16(p) on v; two launches with far_part as htrc_tile_attention_fp8. */
int htrc_tile_attention_bf16(const uint16_t* qb, const uint16_t* dqb, int64_t n_queries, int32_t tile, int64_t t0,
                             int64_t tc, int32_t group, const uint16_t* gb, const float* lz, const uint16_t* vbb,
                             const uint8_t* excl, const int32_t* idx, int32_t kx, int64_t nb, const uint16_t* k,
                             const uint16_t* v, int64_t n_keys, int32_t dim, int32_t leaf, float scale,
                             const float* tail_part, const int32_t* perm, float* far_part, float* out, float* lse,
                             int32_t* status, htrc_stream_t stream);

/* The forward pass for callers that cannot allocate device memory (a plugin host that owns all device
 * allocations and lends only input and output buffers, or an embedding whose device footprint must not
 * grow after start-up).  Same arguments and results as htrc_flat_forward, except that args->workspace
 * and args->workspace_bytes are ignored: the scratch lives in a 64 MiB array declared in the library
 * (held on every GPU that uses this entry point until the process exits).  Problems whose
 * htrc_flat_workspace_size() exceeds 64 MiB are rejected with HTRC_ERR_TOO_LARGE (about 16k queries
 * and keys at the default routing; a smaller tile_chunk admits more).  All calls share the array: calls
 * that overlap on the GPU race, so issue them in order on one stream.  The status word is cleared at
 * the start of every call; read it after a call with htrc_flat_static_ws_status.  The first call on a
 * device looks up the array's address and caches it; make it before any stream capture, and do not use
 * this entry point across cudaDeviceReset.  Allocates nothing.
 * This entry point has no counterpart in the reference. */
int htrc_flat_forward_static_ws(const HtrcFlatArgs* args, htrc_stream_t stream);

/* The device status word of htrc_flat_forward_static_ws's array, read and cleared like htrc_flat_status
 * (synchronises `stream`; *status_out receives the HTRC_STATUS_* bits of the calls since the last read).
 * Like its forward entry point it has no counterpart in the reference and allocates nothing. */
int htrc_flat_static_ws_status(int32_t* status_out, htrc_stream_t stream);

/* Low-bit round trip of x [rows, dim] (h3/htrc_flat.py:68-97 `fake_quant`, a simulation of quantised
 * inputs): every group of `group` consecutive values of a row (0: the whole row; HTRC_FQ_FP4 with 0:
 * 16; else a power of two dividing dim) is rounded through the format with the symmetric scale
 * s = max(amax, 1e-20) / qmax and written back as s * code: INT8 / INT4 clamp(rint(x / s), +-qmax),
 * qmax 127 / 7; FP8 nearest-even e4m3 of clamp(x / s, +-448); FP4 the e2m1 grid value of |x / s|
 * chosen by the reference's thresholds, times sign(x).  x f32 or bf16; out f32 or bf16 (rounded
 * to nearest even). */
int htrc_fake_quant(const void* x, int32_t x_dtype, int64_t rows, int32_t dim, int32_t fmt, int32_t group, void* out,
                    int32_t out_dtype, htrc_stream_t stream);

/* out[r, :] = bf16(float(x8[r, :]) * scale[r]) for e4m3 codes x8 (h3/htrc_flat_triton.py:276-294
 * `dequant_rows`, the fp8 cache read path); row strides in elements (x8: multiple of 4, so rows stay
 * 4-byte aligned), out [rows, dim] contiguous. */
int htrc_dequant_rows(const uint8_t* x8, int64_t stride_x, const float* scale, int64_t stride_s, int64_t rows,
                      int32_t dim, uint16_t* out, htrc_stream_t stream);

/* Self-test of the device failure path (no reference counterpart): one CTA waits on a barrier nothing
 * arrives at, with the kernels' bounded wait given `limit_cycles` (at most 2^34) clock cycles; the wait
 * gives up and ORs HTRC_STATUS_WAIT_TIMEOUT into *status (a device int32 word), then the kernel returns.
 * Nothing faults or traps and the context stays usable. */
int htrc_selftest_wait_timeout(int32_t* status, int64_t limit_cycles, htrc_stream_t stream);

/* Human-readable name of a return code. */
const char* htrc_strerror(int code);

#ifdef __cplusplus
}
#endif

#endif /* HTRC_FLAT_H_ */
