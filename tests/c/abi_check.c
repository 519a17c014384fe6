/* A C host of libhtrc_flat.so that needs no GPU: argument validation, workspace sizing and error names
 * through include/htrc_flat.h, compiled by a plain C compiler (the drop-in boundary for non-Python hosts). */
#include <stdio.h>
#include <string.h>

#include "htrc_flat.h"

static int fail(const char* what) {
  fprintf(stderr, "FAIL: %s\n", what);
  return 1;
}

int main(void) {
  HtrcFlatArgs a;
  size_t need = 0, need_chunked = 0, need_iso = 0, need_fp8 = 0;
  memset(&a, 0, sizeof(a));
  a.q_dtype = HTRC_DTYPE_BF16;
  a.n_queries = 129024;
  a.n_keys = 129024;
  a.dim = 128;
  a.tile = 64;
  a.leaf = 64;
  a.exact_leaves = 256;
  a.group = 1;
  a.order = HTRC_ORDER_SEQ;
  a.curvature = HTRC_CURV_LIN;
  if (htrc_flat_workspace_size(&a, &need) != HTRC_OK || need == 0) return fail("workspace size");
  a.tile_chunk = 128;
  if (htrc_flat_workspace_size(&a, &need_chunked) != HTRC_OK || need_chunked >= need) return fail("chunked size");
  a.tile_chunk = 0;
  a.curvature = HTRC_CURV_ISO;
  if (htrc_flat_workspace_size(&a, &need_iso) != HTRC_OK || need_iso <= need) return fail("iso size");
  a.store = HTRC_STORE_FP8;
  if (htrc_flat_workspace_size(&a, &need_iso) != HTRC_ERR_UNSUPPORTED) return fail("fp8 state with iso curvature");
  a.curvature = HTRC_CURV_LIN;
  if (htrc_flat_workspace_size(&a, &need_fp8) != HTRC_OK || need_fp8 >= need) return fail("fp8 size");
  a.store = 5;
  if (htrc_flat_workspace_size(&a, &need_fp8) != HTRC_ERR_ARG) return fail("bad store");
  a.store = HTRC_STORE_INT8;
  a.curvature = 7;
  if (htrc_flat_workspace_size(&a, &need) != HTRC_ERR_ARG) return fail("bad curvature");
  a.curvature = HTRC_CURV_LIN;
  a.n_keys = 129024 + 1;
  if (htrc_flat_workspace_size(&a, &need) != HTRC_ERR_ARG) return fail("keys not a multiple of the leaf");
  a.n_keys = 129024;
  {
    size_t need16 = 0, need32 = 0;
    a.leaf = 32;
    if (htrc_flat_workspace_size(&a, &need32) != HTRC_OK || need32 <= need) return fail("leaf 32 size");
    a.leaf = 16;
    if (htrc_flat_workspace_size(&a, &need16) != HTRC_OK || need16 <= need32) return fail("leaf 16 size");
    a.curvature = HTRC_CURV_ISO;
    if (htrc_flat_workspace_size(&a, &need16) != HTRC_ERR_UNSUPPORTED) return fail("leaf 16 with iso curvature");
    a.curvature = HTRC_CURV_LIN;
    a.store = HTRC_STORE_FP8;
    if (htrc_flat_workspace_size(&a, &need16) != HTRC_ERR_UNSUPPORTED) return fail("leaf 16 with the fp8 state");
    a.store = HTRC_STORE_INT8;
    a.leaf = 8;
    if (htrc_flat_workspace_size(&a, &need16) != HTRC_ERR_UNSUPPORTED) return fail("leaf 8");
  }
  a.leaf = 64;
  if (htrc_flat_forward(&a, NULL) != HTRC_ERR_ARG) return fail("forward without pointers");
  if (htrc_leaf_pitch(2016) != 2016 || htrc_leaf_pitch(2017) != 2032) return fail("leaf pitch");
  if (strcmp(htrc_strerror(HTRC_OK), "ok") != 0) return fail("strerror");
  printf("ok %zu %zu %zu %zu\n", need_chunked, need, need_iso, sizeof(HtrcFlatArgs));
  return 0;
}
