/* C ABI of the hierarchical HTRC operator on B200 (sm_100a): the law of the reference's NumPy teaching
 * model, src/htrc_reference/model.py (exact_stats :35-49, merge_stats :51-66, build_forest :68-86,
 * predict :91-96, evaluate :98-137), for many queries and several query centres at once.
 *
 * The reference binds this path as Python functions (`build_forest(keys, values, center, leaf_size=16,
 * fanout=4)` and `evaluate(keys, values, query, center, forest, opening_threshold=0.01)`); the package
 * `htrc_b200.tree` keeps those names over this ABI, and a ctypes binding of the same entry points is
 * what a C, Go or Rust caller would write (INTEGRATION.md shows it).
 *
 * Rows are 128 wide: keys [n_keys, 128], values [n_keys, 128], queries [n_queries, 128], centres
 * [n_centres, 128] float32.  A narrower model pads its rows with zeros (no dot product changes; padded
 * output columns are zero).  Queries enter as scale * q; the centres are in that scaled space, as the
 * reference's `center`.  Query i is evaluated against the forest of centres[assign[i]].
 *
 * Sequence: htrc_tree_build (forest) -> htrc_tree_walk (opening decisions; synchronises the stream and
 * returns the number of partial records) -> htrc_tree_values (records, then out / lse / exact).
 * Every buffer is caller-allocated device memory, 256-byte aligned; sizes come from the *_size calls.
 * Results are bitwise deterministic (fixed reduction orders, no floating-point atomics).
 * Return values are the HTRC_OK / HTRC_ERR_* codes of htrc_flat.h. */
#ifndef HTRC_TREE_H
#define HTRC_TREE_H

#include "htrc_flat.h"

#ifdef __cplusplus
extern "C" {
#endif

enum { HTRC_TREE_MAX_LEVELS = 16, HTRC_TREE_MAX_CENTRES = 256, HTRC_TREE_KMEANS_CENTRES = 32 };
/* htrc_tree_values stages (OR-ed; run in this order): records of accepted internal nodes, records of the
 * opened level-1 nodes' leaf blocks, and the per-query merge into out / lse / exact_leaves */
enum { HTRC_TREE_STAGE_ACCEPT = 1, HTRC_TREE_STAGE_LEAVES = 2, HTRC_TREE_STAGE_FINAL = 4, HTRC_TREE_STAGE_ALL = 7 };

typedef struct {
  int64_t n_keys;      /* >= 1 */
  int64_t n_queries;   /* >= 0 */
  int32_t n_centres;   /* 1 .. HTRC_TREE_MAX_CENTRES */
  int32_t leaf_size;   /* 1 .. 64 keys per leaf (the last leaf may hold fewer), model.py:68 */
  int32_t fanout;      /* 2 .. 64 children per node, model.py:68 */
  int32_t kv_dtype;    /* HTRC_DTYPE_F32 or HTRC_DTYPE_BF16: keys and values */
  int32_t q_dtype;     /* HTRC_DTYPE_F32 or HTRC_DTYPE_BF16: queries */
  float scale;         /* the query scale (1 for queries already scaled, as model.py's evaluate takes) */
  float threshold;     /* opening threshold >= 0 (model.py:100) */
} HtrcTreeDims;

/* Levels of the forest (model.py:80-85): n_levels and nodes[l] per centre, level 0 = leaves. */
int htrc_tree_levels(const HtrcTreeDims* dims, int32_t* n_levels, int32_t nodes[HTRC_TREE_MAX_LEVELS]);

/* Forest of every centre: leaf log-masses and key logits a = k . c, and for each level >= 1 the node
 * log-mass L, mean key g, mean value u, Hessian H and transposed value Jacobian J^T (float32). */
int htrc_tree_forest_size(const HtrcTreeDims* dims, size_t* bytes);
int htrc_tree_build(const HtrcTreeDims* dims, const void* keys, const void* values, const float* centres,
                    void* forest, size_t forest_bytes, htrc_stream_t stream);
/* Device pointers into a built forest, for inspection: a [C, n_keys]; level 0: L [C, n0]; level l >= 1:
 * L [C, n], g and u [C, n, 128], H and JT [C, n, 128, 128].  Unused outputs may be NULL. */
int htrc_tree_forest_view(const HtrcTreeDims* dims, const void* forest, int32_t level, const float** a,
                          const float** L, const float** g, const float** u, const float** H, const float** JT);

/* Walk (model.py:104-127): per query the opened / accepted nodes of every level, and the reference's
 * counters visited_nodes and accepted_nodes [n_queries] int32 (leaves: NULL or [n_queries] int32, the leaves
 * each query visits).  Synchronises the stream and returns the number of partial records in *n_records.
 * HTRC_ERR_ARG if an assign entry is out of range. */
int htrc_tree_walk_size(const HtrcTreeDims* dims, size_t* bytes);
int htrc_tree_walk(const HtrcTreeDims* dims, const void* queries, const int32_t* assign, const float* centres,
                   const void* forest, void* walk, size_t walk_bytes, int32_t* visited, int32_t* accepted,
                   int32_t* leaves, int64_t* n_records, htrc_stream_t stream);

/* Values (model.py:91-96, :122-137): out [n_queries, 128] float32, lse [n_queries] float32 (log-sum-exp
 * of the accepted log-masses, the operator's log-Z; the reference does not return it) and exact_leaves
 * [n_queries] int32.  records: htrc_tree_records_size(n_records) bytes, n_records as htrc_tree_walk
 * returned it; stages: HTRC_TREE_STAGE_* bits (HTRC_TREE_STAGE_ALL for the whole evaluation; a subset lets a
 * caller time the stages).  keys, values and queries share one dtype. */
int htrc_tree_records_size(int64_t n_records, size_t* bytes);
int htrc_tree_values(const HtrcTreeDims* dims, const void* keys, const void* values, const void* queries,
                     const float* centres, const void* forest, void* walk, void* records, int64_t n_records,
                     size_t records_bytes, float* out, float* lse, int32_t* exact_leaves, int32_t stages,
                     htrc_stream_t stream);

/* Query centres for the operator: the k-means of htrc_kmeans_order (32 clusters, Lloyd x 8 on an even
 * sample of at most 4096 rows), scaled by `scale` -> centres [32, 128] float32, and the nearest centre
 * of every row -> assign [n_queries] int32.  scratch: htrc_tree_centres_scratch_size() bytes. */
int htrc_tree_centres_scratch_size(int64_t n_queries, size_t* bytes);
int htrc_tree_centres(const void* queries, int32_t q_dtype, int64_t n_queries, float scale, float* centres,
                      int32_t* assign, void* scratch, size_t scratch_bytes, htrc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* HTRC_TREE_H */
