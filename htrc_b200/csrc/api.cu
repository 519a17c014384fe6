// extern "C" entry points of libhtrc_flat.so (include/htrc_flat.h): argument checks, workspace
// layout, TMA tensor maps and the launch sequence of one head of the flat HTRC operator.
#include <cmath>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"

using namespace htrc;

namespace {

constexpr int kDim = 128;
constexpr int kTile = 64;        // rows of a tile as the kernels hold it (a 32-row tile is padded to 64)
constexpr int kLeaf = 64;          // the leaf every configuration supports
// other leaves (32, 16 keys) run with the INT8 state and the linear far field
bool leaf_ok(int64_t leaf) { return leaf == 64 || leaf == 32 || leaf == 16; }
constexpr int64_t kMaxLeaves = 8192;
constexpr int64_t kMaxRouted = 1024;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}

struct DeviceInfo {
  bool ok = false;
  int sms = 148;
};

DeviceInfo device_info() {
  static DeviceInfo cache[64];
  static bool probed[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DeviceInfo{};
  if (!probed[dev]) {
    int major = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cache[dev].ok = (major == 10);
    cache[dev].sms = sms > 0 ? sms : 148;
    probed[dev] = true;
  }
  return cache[dev];
}

// rank-2..4 tiled map; dims innermost first, strides in bytes for dims 1..rank-1
bool make_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides, const uint32_t* box, bool swizzle128) {
  if (!encoder() || base == nullptr || rank < 2 || rank > 4) return false;
  cuuint64_t gd[4], gs[3];
  cuuint32_t bx[4], es[4] = {1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    if (dims[i] == 0) return false;
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides[i];
  CUresult r = g_encode(m, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), gd, gs, bx, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// [rows, 128] matrix of 1- or 2-byte elements, box of `box_rows` rows x (128 B)
bool map_rows(CUtensorMap* m, const void* base, int64_t rows, bool bf16, int box_rows) {
  const uint64_t dims[2] = {128, static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {bf16 ? 256u : 128u};
  const uint32_t box[2] = {bf16 ? 64u : 128u, static_cast<uint32_t>(box_rows)};
  return make_map(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides,
                  box, true);
}

// [rows, 128] bf16 matrix seen as [2 halves][rows][64]: one box of `box_rows` rows lands in shared memory as
// the 64-column half 0 followed by half 1, each a 128-byte-swizzled [box_rows][64] tile (one TMA load for a
// whole leaf instead of one per half)
bool map_rows_halves(CUtensorMap* m, const void* base, int64_t rows, int box_rows) {
  const uint64_t dims[3] = {64, static_cast<uint64_t>(rows), 2};
  const uint64_t strides[2] = {256, 128};
  const uint32_t box[3] = {64, static_cast<uint32_t>(box_rows), 2};
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, true);
}

// [tc, nb, 128] bf16 state seen as [tc][2 halves][nb][64], box (64, box_leaves, 2, 1): the same split per tile
bool map_state_halves(CUtensorMap* m, const void* base, int64_t tc, int64_t nb, int box_leaves) {
  const uint64_t dims[4] = {64, static_cast<uint64_t>(nb), 2, static_cast<uint64_t>(tc)};
  const uint64_t strides[3] = {256, 128, static_cast<uint64_t>(nb) * 256};
  const uint32_t box[4] = {64, static_cast<uint32_t>(box_leaves), 2, 1};
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box, true);
}

// [tc, nb, 128] state of 1- or 2-byte elements, box (inner, box_leaves, box_tiles)
bool map_state(CUtensorMap* m, const void* base, int64_t tc, int64_t nb, bool bf16, int box_leaves, int box_tiles) {
  const uint64_t es = bf16 ? 2 : 1;
  const uint64_t dims[3] = {128, static_cast<uint64_t>(nb), static_cast<uint64_t>(tc)};
  const uint64_t strides[2] = {128 * es, static_cast<uint64_t>(nb) * 128 * es};
  const uint32_t box[3] = {bf16 ? 64u : 128u, static_cast<uint32_t>(box_leaves), static_cast<uint32_t>(box_tiles)};
  return make_map(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides,
                  box, true);
}

// [tc, nb, 128] one-byte codes staged as 128-byte rows (plain, or 128-byte swizzled), box (128, box_leaves, 1)
bool map_codes(CUtensorMap* m, const void* base, int64_t tc, int64_t nb, int box_leaves, bool swizzle) {
  const uint64_t dims[3] = {128, static_cast<uint64_t>(nb), static_cast<uint64_t>(tc)};
  const uint64_t strides[2] = {128, static_cast<uint64_t>(nb) * 128};
  const uint32_t box[3] = {128u, static_cast<uint32_t>(box_leaves), 1u};
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box, swizzle);
}

// [tc, nb] scalars (f32 or u8) with row pitch `pitch` elements, box (box_cols, 1)
bool map_scalars(CUtensorMap* m, const void* base, int64_t tc, int64_t nb, int64_t pitch, bool f32, int box_cols) {
  const uint64_t es = f32 ? 4 : 1;
  const uint64_t dims[2] = {static_cast<uint64_t>(nb), static_cast<uint64_t>(tc)};
  const uint64_t strides[1] = {static_cast<uint64_t>(pitch) * es};
  const uint32_t box[2] = {static_cast<uint32_t>(box_cols), 1u};
  return make_map(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides,
                  box, false);
}

int64_t pitch_of(int64_t nb) { return (nb + 15) / 16 * 16; }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace of one forward call.  Centre rows (mu, and the far-field state, routing and exclusion
// rows) are per group of `group` tiles; a chunk holds gcm groups = gcm * group tiles.
struct Layout {
  int64_t n = 0, m = 0, nt = 0, nb = 0, pitch = 0, kx = 0, group = 1, ng = 0, gcm = 0, tcm = 0, trows = 64;
  int64_t leaf = 64;
  bool kmeans = false;
  size_t status = 0, k8 = 0, ks = 0, mu = 0, mu_hi = 0, mu_lo = 0, q8 = 0, sq = 0, dq8 = 0, sdq = 0, tail = 0;
  size_t g8 = 0, vb = 0, sg = 0, lz = 0, sel = 0, excl = 0, idx = 0, perm = 0, km = 0, total = 0;
  bool iso = false;
  size_t kn2 = 0, dd = 0, cv = 0;           // iso curvature: key norms, row offsets, coefficients
  bool fp8 = false;                         // fp8 state: q8 / dq8 hold bf16 / fp16 rows, vb the vbar codes
  bool bf = false;                          // bf16 state: q8 / dq8 hold bf16 rows, g8 / vb bf16 values
  bool opf = false;                         // fp8 or bf16 state: the operand-form kernels of fp8.cu
  size_t sv = 0, fpart = 0;
};

constexpr int kMaxGroup = 65536;

int validate(const HtrcFlatArgs* a, bool need_ptrs) {
  if (a == nullptr) return HTRC_ERR_ARG;
  if (a->dim != kDim || (a->tile != kTile && a->tile != kTile / 2) || !leaf_ok(a->leaf)) return HTRC_ERR_UNSUPPORTED;
  if (a->n_queries < 1 || a->n_keys < a->leaf || a->n_keys % a->leaf) return HTRC_ERR_ARG;
  if (a->q_dtype != HTRC_DTYPE_F32 && a->q_dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (a->exact_leaves < 0 || a->sink_leaves < 0 || a->n_tail < 0) return HTRC_ERR_ARG;
  if (a->group > kMaxGroup) return HTRC_ERR_ARG;
  if (a->order != HTRC_ORDER_SEQ && a->order != HTRC_ORDER_KMEANS) return HTRC_ERR_ARG;
  if (a->curvature != HTRC_CURV_LIN && a->curvature != HTRC_CURV_ISO) return HTRC_ERR_ARG;
  if (a->store != HTRC_STORE_INT8 && a->store != HTRC_STORE_FP8 && a->store != HTRC_STORE_BF16) return HTRC_ERR_ARG;
  if (a->store != HTRC_STORE_INT8 && a->curvature != HTRC_CURV_LIN) return HTRC_ERR_UNSUPPORTED;
  if (a->qk_scale_block != 0 && a->qk_scale_block != 64) return HTRC_ERR_ARG;
  if (a->qk_scale_block != 0 && a->store != HTRC_STORE_INT8) return HTRC_ERR_UNSUPPORTED;
  if (a->leaf != kLeaf &&
      (a->store != HTRC_STORE_INT8 || a->curvature != HTRC_CURV_LIN || a->qk_scale_block != 0))
    return HTRC_ERR_UNSUPPORTED;
  if ((a->precision & ~(HTRC_PREC_TF32 | HTRC_PREC_TRITON_DIV)) != 0) return HTRC_ERR_ARG;
  if (a->n_queries > (int64_t(1) << 31) - 1) return HTRC_ERR_UNSUPPORTED;
  const int64_t nb = a->n_keys / a->leaf;
  if (nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  const int64_t sink = std::min<int64_t>(a->sink_leaves, nb);
  const int64_t kx = std::min<int64_t>(static_cast<int64_t>(a->exact_leaves) + sink, nb);
  if (kx > kMaxRouted) return HTRC_ERR_UNSUPPORTED;
  if (need_ptrs) {
    if (!a->q || !a->k || !a->v || !a->out) return HTRC_ERR_ARG;
    if (a->n_tail > 0 && (!a->tail_k || !a->tail_v)) return HTRC_ERR_ARG;
  }
  return HTRC_OK;
}

Layout layout_of(const HtrcFlatArgs* a) {
  Layout L;
  L.n = a->n_queries;
  L.m = a->n_keys;
  L.trows = a->tile;
  L.nt = (L.n + L.trows - 1) / L.trows;
  L.leaf = a->leaf;
  L.nb = L.m / L.leaf;
  L.pitch = pitch_of(L.nb);
  const int64_t sink = std::min<int64_t>(a->sink_leaves, L.nb);
  L.kx = std::min<int64_t>(static_cast<int64_t>(a->exact_leaves) + sink, L.nb);
  L.group = a->group > 1 ? a->group : 1;
  L.ng = (L.nt + L.group - 1) / L.group;
  L.kmeans = a->order == HTRC_ORDER_KMEANS;
  // groups per chunk: tile_chunk // group (the reference's gstep, h3/htrc_flat.py:238), made even in
  // tiles when the state is chunked so that no tile pair of the tile kernel straddles two chunks
  int64_t gcm = a->tile_chunk > 0 ? std::max<int64_t>(1, a->tile_chunk / L.group) : L.ng;
  gcm = std::min<int64_t>(gcm, L.ng);
  if (gcm < L.ng && (gcm * L.group) % 2) gcm = std::min<int64_t>(gcm + 1, L.ng);
  L.gcm = gcm;
  L.tcm = std::min<int64_t>(gcm * L.group, L.nt);
  const int64_t gcm_rows = gcm;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align256(o + bytes);
    return at;
  };
  L.fp8 = a->store == HTRC_STORE_FP8;
  L.bf = a->store == HTRC_STORE_BF16;
  L.opf = L.fp8 || L.bf;
  const size_t qes = L.opf ? 2 : 1;         // bytes per value of the query operands
  L.status = take(256);
  if (!L.opf) {
    L.k8 = take(static_cast<size_t>(L.m) * 128);
    L.ks = take(static_cast<size_t>(L.m) * 4);
  }
  L.mu = take(static_cast<size_t>(L.ng) * 128 * 4);
  L.mu_hi = take(static_cast<size_t>(L.ng) * 128 * 2);
  L.mu_lo = take(static_cast<size_t>(L.ng) * 128 * 2);
  L.q8 = take(static_cast<size_t>(L.nt) * 64 * 128 * qes);
  L.dq8 = take(static_cast<size_t>(L.nt) * 64 * 128 * qes);
  if (!L.opf) {
    L.sq = take(static_cast<size_t>(L.nt) * 64 * 4);
    L.sdq = take(static_cast<size_t>(L.nt) * 64 * 4);
  }
  L.tail = a->n_tail > 0 ? take(static_cast<size_t>(L.n) * 130 * 4) : 0;
  L.g8 = take(static_cast<size_t>(gcm_rows) * L.nb * (L.bf ? 256 : 128));
  L.vb = take(static_cast<size_t>(gcm_rows) * L.nb * (L.fp8 ? 128 : 256));
  if (L.fp8) L.sv = take(static_cast<size_t>(gcm_rows) * L.pitch * 4);
  if (L.opf && L.kx < L.nb) L.fpart = take(static_cast<size_t>(L.n) * 130 * 4);   // far-field partial rows
  L.sg = take(static_cast<size_t>(gcm_rows) * L.pitch * 4);
  L.lz = take(static_cast<size_t>(gcm_rows) * L.pitch * 4);
  L.sel = take(static_cast<size_t>(L.tcm) * L.pitch * 4);
  L.excl = take(static_cast<size_t>(gcm_rows) * L.pitch);
  L.idx = take(static_cast<size_t>(gcm_rows) * std::max<int64_t>(L.kx, 1) * 4);
  L.iso = a->curvature == HTRC_CURV_ISO;
  if (L.iso) {
    L.kn2 = take(static_cast<size_t>(L.m) * 4);
    L.dd = take(static_cast<size_t>(L.nt) * 64 * 4);
    L.cv = take(static_cast<size_t>(gcm_rows) * L.pitch * 4);
  }
  if (L.kmeans) {
    L.perm = take(static_cast<size_t>(L.n) * 4);
    L.km = take(kmeans_scratch_bytes(L.n));
  }
  L.total = o;
  return L;
}

template <typename T>
T* at(void* base, size_t off) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(base) + off);
}

int check_device() { return device_info().ok ? HTRC_OK : HTRC_ERR_DEVICE; }

// store: HTRC_STORE_INT8 / FP8 / BF16 (the g rows' element type: byte codes, or bf16 values)
int stats_maps(LeafStatsMaps* mp, const uint16_t* mu_hi, const uint16_t* mu_lo, int64_t nt, const uint16_t* k,
               const uint16_t* v, int64_t m, const void* g8, const void* vb, int64_t tc, int64_t nb, int store) {
  mp->mu_hi = mu_hi;
  mp->mu_lo = mu_lo;
  mp->nt = nt;
  bool ok = map_rows_halves(&mp->k, k, m, 64) && map_rows_halves(&mp->v, v, m, 64) &&
            map_state(&mp->g8, g8, tc, nb, store == HTRC_STORE_BF16, 1, 128) &&
            map_state(&mp->vb, vb, tc, nb, store != HTRC_STORE_FP8, 1, 128);
  return ok ? HTRC_OK : HTRC_ERR_CUDA;
}

// the bf16 state's row-max operands: bf16 offsets and g as [2][rows][64] halves (box of 128 leaves)
int rowmax_bf16_maps(RowmaxMaps* mp, const uint16_t* dqb, int64_t rows, const uint16_t* gb, const float* lz, int64_t tc,
                     int64_t nb, int64_t pitch) {
  bool ok = map_rows_halves(&mp->dq8, dqb, rows, 64) && map_state_halves(&mp->g8, gb, tc, nb, 128) &&
            map_scalars(&mp->lz, lz, tc, nb, pitch, true, 128) && map_scalars(&mp->sg, lz, tc, nb, pitch, true, 128) &&
            map_scalars(&mp->cv, lz, tc, nb, pitch, true, 128);
  return ok ? HTRC_OK : HTRC_ERR_CUDA;
}

// the bf16 state's tile maps: g and vbar as [2][nb][64] halves per state row (box of 64 leaves); the scale maps
// the kernel does not read point at lz
int tile_bf16_maps(TileFp8Maps* mp, const uint16_t* qb, const uint16_t* dqb, int64_t rows, const uint16_t* gb,
                   const uint16_t* vbb, const float* lz, const uint8_t* excl, int64_t tc, int64_t nb, int64_t pitch,
                   const uint16_t* k, const uint16_t* v, int64_t m) {
  bool ok = map_rows_halves(&mp->qb, qb, rows, 64) && map_rows_halves(&mp->dqh, dqb, rows, 64) &&
            map_state_halves(&mp->graw, gb, tc, nb, 64) && map_state_halves(&mp->vraw, vbb, tc, nb, 64) &&
            map_scalars(&mp->lz, lz, tc, nb, pitch, true, 64) && map_scalars(&mp->sg, lz, tc, nb, pitch, true, 64) &&
            map_scalars(&mp->sv, lz, tc, nb, pitch, true, 64) &&
            map_scalars(&mp->excl, excl, tc, nb, pitch, false, 64) && map_rows_halves(&mp->k, k, m, 64) &&
            map_rows_halves(&mp->v, v, m, 64);
  return ok ? HTRC_OK : HTRC_ERR_CUDA;
}

int rowmax_fp8_maps(RowmaxFp8Maps* mp, const uint16_t* dqh, int64_t rows, const uint8_t* g8, const float* sg,
                    const float* lz, int64_t tc, int64_t nb, int64_t pitch) {
  bool ok = map_rows_halves(&mp->dqh, dqh, rows, 64) && map_codes(&mp->graw, g8, tc, nb, 128, false) &&
            map_scalars(&mp->sg, sg, tc, nb, pitch, true, 128) && map_scalars(&mp->lz, lz, tc, nb, pitch, true, 128);
  return ok ? HTRC_OK : HTRC_ERR_CUDA;
}

int tile_fp8_maps(TileFp8Maps* mp, const uint16_t* qb, const uint16_t* dqh, int64_t rows, const uint8_t* g8,
                  const uint8_t* vb8, const float* lz, const float* sg, const float* sv, const uint8_t* excl, int64_t tc,
                  int64_t nb, int64_t pitch, const uint16_t* k, const uint16_t* v, int64_t m) {
  bool ok = map_rows_halves(&mp->qb, qb, rows, 64) && map_rows_halves(&mp->dqh, dqh, rows, 64) &&
            map_codes(&mp->graw, g8, tc, nb, 64, true) && map_codes(&mp->vraw, vb8, tc, nb, 64, true) &&
            map_scalars(&mp->lz, lz, tc, nb, pitch, true, 64) && map_scalars(&mp->sg, sg, tc, nb, pitch, true, 64) &&
            map_scalars(&mp->sv, sv, tc, nb, pitch, true, 64) &&
            map_scalars(&mp->excl, excl, tc, nb, pitch, false, 64) && map_rows_halves(&mp->k, k, m, 64) &&
            map_rows_halves(&mp->v, v, m, 64);
  return ok ? HTRC_OK : HTRC_ERR_CUDA;
}

int rowmax_maps(RowmaxMaps* mp, const int8_t* dq8, int64_t rows, const int8_t* g8, const float* sg, const float* lz,
                const float* cv, int64_t tc, int64_t nb, int64_t pitch) {
  bool ok = map_rows(&mp->dq8, dq8, rows, false, 64) && map_state(&mp->g8, g8, tc, nb, false, 128, 1) &&
            map_scalars(&mp->sg, sg, tc, nb, pitch, true, 128) && map_scalars(&mp->lz, lz, tc, nb, pitch, true, 128) &&
            map_scalars(&mp->cv, cv ? cv : sg, tc, nb, pitch, true, 128);
  return ok ? HTRC_OK : HTRC_ERR_CUDA;
}

int tile_maps(TileMaps* mp, const int8_t* q8, const int8_t* dq8, int64_t rows, const int8_t* g8, const uint16_t* vb,
              const float* lz, const float* sg, const float* cv, const uint8_t* excl, int64_t tc, int64_t nb,
              int64_t pitch, const int8_t* k8, const uint16_t* v, int64_t m, int leaf) {
  bool ok = map_rows(&mp->q8, q8, rows, false, 64) && map_rows(&mp->dq8, dq8, rows, false, 64) &&
            map_state(&mp->g8, g8, tc, nb, false, 64, 1) && map_state_halves(&mp->vb, vb, tc, nb, 64) &&
            map_scalars(&mp->lz, lz, tc, nb, pitch, true, 64) && map_scalars(&mp->sg, sg, tc, nb, pitch, true, 64) &&
            map_scalars(&mp->excl, excl, tc, nb, pitch, false, 64) && map_rows(&mp->k8, k8, m, false, leaf) &&
            map_rows_halves(&mp->v, v, m, leaf) && map_scalars(&mp->cv, cv ? cv : sg, tc, nb, pitch, true, 64);
  return ok ? HTRC_OK : HTRC_ERR_CUDA;
}

float scale_of(float s) { return s > 0.f ? s : 1.0f / std::sqrt(static_cast<float>(kDim)); }

}  // namespace

// Self-test of the failure path every kernel shares: a CTA waits on an mbarrier nothing arrives at, with
// the kernels' own bounded wait given a short limit; the wait gives up, flags the status word and the
// kernel returns (no trap, no fault; the context stays usable).
__global__ void __launch_bounds__(32) wait_selftest_kernel(int* status, long long limit) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_for(&bar, 0, status, &abort_flag, limit);   // no arrival: runs out
  __syncthreads();
}

extern "C" {

int64_t htrc_leaf_pitch(int64_t nb) { return pitch_of(nb); }

int htrc_flat_workspace_size(const HtrcFlatArgs* args, size_t* bytes) {
  const int rc = validate(args, false);
  if (rc != HTRC_OK) return rc;
  if (bytes == nullptr) return HTRC_ERR_ARG;
  *bytes = layout_of(args).total;
  return HTRC_OK;
}

int htrc_flat_forward(const HtrcFlatArgs* a, htrc_stream_t stream) {
  int rc = validate(a, true);
  if (rc != HTRC_OK) return rc;
  if ((rc = check_device()) != HTRC_OK) return rc;
  const Layout L = layout_of(a);
  if (a->workspace == nullptr || a->workspace_bytes < L.total ||
      (reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0)
    return HTRC_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  void* ws = a->workspace;
  int* status = at<int>(ws, L.status);
  const float scale = scale_of(a->scale);
  const int nb = static_cast<int>(L.nb), kx = static_cast<int>(L.kx);
  const int sink = static_cast<int>(std::min<int64_t>(a->sink_leaves, L.nb));
  int8_t* k8 = at<int8_t>(ws, L.k8);
  float* ks = at<float>(ws, L.ks);
  int8_t* q8 = at<int8_t>(ws, L.q8);
  int8_t* dq8 = at<int8_t>(ws, L.dq8);
  float* sq = at<float>(ws, L.sq);
  float* sdq = at<float>(ws, L.sdq);
  uint16_t* mu_hi = at<uint16_t>(ws, L.mu_hi);
  uint16_t* mu_lo = at<uint16_t>(ws, L.mu_lo);
  int8_t* g8 = at<int8_t>(ws, L.g8);
  uint16_t* vb = at<uint16_t>(ws, L.vb);
  float* sg = at<float>(ws, L.sg);
  float* lz = at<float>(ws, L.lz);
  float* sel = at<float>(ws, L.sel);
  uint8_t* excl = at<uint8_t>(ws, L.excl);
  int32_t* idx = at<int32_t>(ws, L.idx);
  float* tail = a->n_tail > 0 ? at<float>(ws, L.tail) : nullptr;
  int32_t* perm = L.kmeans ? at<int32_t>(ws, L.perm) : nullptr;
  const int group = static_cast<int>(L.group);

  auto mark = [&](int i) {
    if (a->stage_events && i < a->n_stage_events && a->stage_events[i])
      cudaEventRecord(static_cast<cudaEvent_t>(a->stage_events[i]), st);
  };
  mark(0);
  float* kn2 = L.iso ? at<float>(ws, L.kn2) : nullptr;
  float* dd = L.iso ? at<float>(ws, L.dd) : nullptr;
  float* cv = L.iso ? at<float>(ws, L.cv) : nullptr;
  float* sv = L.fp8 ? at<float>(ws, L.sv) : nullptr;
  if (!L.opf && a->qk_scale_block)
    launch_pack_blocks(a->k, HTRC_DTYPE_BF16, L.m, HTRC_ROUND_HALF_EVEN, k8, ks, kn2, st);
  else if (!L.opf)
    launch_pack_rows(a->k, HTRC_DTYPE_BF16, L.m, HTRC_ROUND_HALF_EVEN, k8, ks, kn2, st);
  if (perm && (rc = launch_kmeans_order(a->q, a->q_dtype, L.n, perm, at<void>(ws, L.km), st)) != HTRC_OK) return rc;
  const int trows = static_cast<int>(L.trows);
  launch_tile_prep(a->q, a->q_dtype, L.n, trows, perm, group, at<float>(ws, L.mu), mu_hi, mu_lo, q8, sq, dq8, sdq, dd,
                   L.opf, a->qk_scale_block != 0, (a->precision & HTRC_PREC_TF32) != 0,
                   (a->precision & HTRC_PREC_TRITON_DIV) != 0, st, L.bf);
  if (tail) launch_tail_partial(a->q, a->q_dtype, L.n, a->tail_k, a->tail_v, a->n_tail, scale, tail, st);
  if (cudaGetLastError() != cudaSuccess) return HTRC_ERR_CUDA;
  mark(1);
  const bool far = kx < nb;
  int chunk = 0;
  for (int64_t g0 = 0; g0 < L.ng; g0 += L.gcm, ++chunk) {
    const int64_t gc = std::min<int64_t>(L.gcm, L.ng - g0);     // centre rows of this chunk
    const int64_t t0 = g0 * L.group;
    const int64_t tc = std::min<int64_t>(gc * L.group, L.nt - t0);
    if (far) {
      LeafStatsMaps smp;
      if ((rc = stats_maps(&smp, mu_hi, mu_lo, L.ng, a->k, a->v, L.m, g8, vb, gc, L.nb, a->store)) != HTRC_OK)
        return rc;
      if ((rc = launch_leaf_stats(smp, sg, lz, L.pitch, g0, gc, nb, static_cast<int>(L.leaf), scale, kn2, cv, sv,
                                  status, device_info().sms,
                                  (a->precision & HTRC_PREC_TF32) != 0, (a->precision & HTRC_PREC_TRITON_DIV) != 0,
                                  st, L.bf)) != HTRC_OK)
        return rc;
    }
    mark(2 + 4 * chunk);
    if (far && L.fp8) {
      if (kx > 0) {
        RowmaxFp8Maps rmp;
        if ((rc = rowmax_fp8_maps(&rmp, reinterpret_cast<const uint16_t*>(dq8), L.nt * 64,
                                  reinterpret_cast<const uint8_t*>(g8), sg, lz, gc, L.nb, L.pitch)) != HTRC_OK)
          return rc;
        if ((rc = launch_rowmax_fp8(rmp, sel, L.pitch, t0, tc, nb, group, status, st)) != HTRC_OK) return rc;
      }
    } else if (far && L.bf) {
      if (kx > 0) {
        RowmaxMaps rmp;
        if ((rc = rowmax_bf16_maps(&rmp, reinterpret_cast<const uint16_t*>(dq8), L.nt * 64,
                                   reinterpret_cast<const uint16_t*>(g8), lz, gc, L.nb, L.pitch)) != HTRC_OK)
          return rc;
        if ((rc = launch_rowmax(rmp, nullptr, nullptr, sel, L.pitch, t0, tc, nb, group, status, st, true)) != HTRC_OK)
          return rc;
      }
    } else if (far) {
      if (kx > 0) {
        RowmaxMaps rmp;
        if ((rc = rowmax_maps(&rmp, dq8, L.nt * 64, g8, sg, lz, cv, gc, L.nb, L.pitch)) != HTRC_OK) return rc;
        if ((rc = launch_rowmax(rmp, sdq, dd, sel, L.pitch, t0, tc, nb, group, status, st)) != HTRC_OK) return rc;
      }
    }
    mark(3 + 4 * chunk);
    if ((rc = launch_route(sel, L.pitch, tc, group, nb, kx, sink, idx, excl, st)) != HTRC_OK) return rc;
    if (a->route_mask != nullptr &&
        cudaMemcpyAsync(a->route_mask + g0 * L.pitch, excl, static_cast<size_t>(gc) * L.pitch,
                        cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return HTRC_ERR_CUDA;
    mark(4 + 4 * chunk);
    if (L.opf) {
      TileFp8Maps tmp;
      rc = L.bf ? tile_bf16_maps(&tmp, reinterpret_cast<const uint16_t*>(q8), reinterpret_cast<const uint16_t*>(dq8),
                                 L.nt * 64, reinterpret_cast<const uint16_t*>(g8), reinterpret_cast<const uint16_t*>(vb),
                                 lz, excl, gc, L.nb, L.pitch, a->k, a->v, L.m)
                : tile_fp8_maps(&tmp, reinterpret_cast<const uint16_t*>(q8), reinterpret_cast<const uint16_t*>(dq8),
                                L.nt * 64, reinterpret_cast<const uint8_t*>(g8), reinterpret_cast<const uint8_t*>(vb), lz,
                                sg, sv, excl, gc, L.nb, L.pitch, a->k, a->v, L.m);
      if (rc != HTRC_OK) return rc;
      float* fpart = L.fpart ? at<float>(ws, L.fpart) : nullptr;
      if ((rc = launch_tile_fp8(tmp, idx, kx, nb, L.n, trows, t0, tc, group, scale, tail, perm, fpart, a->out, a->lse,
                                status, st, L.bf)) != HTRC_OK)
        return rc;
      mark(5 + 4 * chunk);
      continue;
    }
    TileMaps tmp;
    if ((rc = tile_maps(&tmp, q8, dq8, L.nt * 64, g8, vb, lz, sg, cv, excl, gc, L.nb, L.pitch, k8, a->v, L.m,
                        static_cast<int>(L.leaf))) != HTRC_OK)
      return rc;
    if ((rc = launch_tile_attention(tmp, sq, sdq, ks, idx, kx, nb, static_cast<int>(L.leaf), L.n, trows, t0, tc,
                                    group, scale, tail, perm,
                                    dd, a->out, a->lse, status, st)) != HTRC_OK)
      return rc;
    mark(5 + 4 * chunk);
  }
  return HTRC_OK;
}

int htrc_flat_status(void* workspace, int32_t* status_out, htrc_stream_t stream) {
  if (workspace == nullptr || status_out == nullptr) return HTRC_ERR_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int32_t* dev = static_cast<int32_t*>(workspace);   // the status word is the first field of the layout
  if (cudaMemcpyAsync(status_out, dev, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return HTRC_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return HTRC_ERR_CUDA;
  if (cudaMemsetAsync(dev, 0, 4, st) != cudaSuccess) return HTRC_ERR_CUDA;
  return HTRC_OK;
}

int htrc_pack_int8(const void* x, int32_t dtype, int64_t rows, int32_t dim, int32_t rounding, int8_t* x8,
                   float* scale, float* sqnorm, htrc_stream_t stream) {
  if (!x || !x8 || !scale || rows < 1) return HTRC_ERR_ARG;
  if (dim != kDim) return HTRC_ERR_UNSUPPORTED;
  if (dtype != HTRC_DTYPE_F32 && dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (rounding != HTRC_ROUND_HALF_EVEN && rounding != HTRC_ROUND_HALF_AWAY) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  launch_pack_rows(x, dtype, rows, rounding, x8, scale, sqnorm, reinterpret_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

int htrc_tile_prep(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, int32_t tile, const int32_t* perm,
                   int32_t group, float* mu, uint16_t* mu_hi, uint16_t* mu_lo, int8_t* q8, float* sq, int8_t* dq8,
                   float* sdq, float* dd, htrc_stream_t stream) {
  if (!q || !mu || !mu_hi || !mu_lo || !q8 || !sq || !dq8 || !sdq || n_queries < 1) return HTRC_ERR_ARG;
  if (dim != kDim || (tile != kTile && tile != kTile / 2)) return HTRC_ERR_UNSUPPORTED;
  if (q_dtype != HTRC_DTYPE_F32 && q_dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (group > kMaxGroup) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  launch_tile_prep(q, q_dtype, n_queries, tile, perm, group, mu, mu_hi, mu_lo, q8, sq, dq8, sdq, dd, false, false,
                   false, false, reinterpret_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

int htrc_tile_prep_ex(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, int32_t tile,
                      const int32_t* perm, int32_t group, float* mu, uint16_t* mu_hi, uint16_t* mu_lo, int8_t* q8,
                      float* sq, int8_t* dq8, float* sdq, float* dd, int32_t q_scale_block, int32_t precision,
                      htrc_stream_t stream) {
  if (q_scale_block != 0 && q_scale_block != 64) return HTRC_ERR_ARG;
  if ((precision & ~(HTRC_PREC_TF32 | HTRC_PREC_TRITON_DIV)) != 0) return HTRC_ERR_ARG;
  if (!q || !mu || !mu_hi || !mu_lo || !q8 || !sq || !dq8 || !sdq || n_queries < 1) return HTRC_ERR_ARG;
  if (dim != kDim || (tile != kTile && tile != kTile / 2)) return HTRC_ERR_UNSUPPORTED;
  if (q_dtype != HTRC_DTYPE_F32 && q_dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (group > kMaxGroup) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  launch_tile_prep(q, q_dtype, n_queries, tile, perm, group, mu, mu_hi, mu_lo, q8, sq, dq8, sdq, dd, false,
                   q_scale_block != 0, (precision & HTRC_PREC_TF32) != 0, (precision & HTRC_PREC_TRITON_DIV) != 0,
                   reinterpret_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

int htrc_pack_int8_blocks(const void* x, int32_t dtype, int64_t rows, int32_t dim, int32_t rounding,
                          int32_t block_rows, int8_t* x8, float* scale, float* sqnorm, htrc_stream_t stream) {
  if (!x || !x8 || !scale || rows < 1) return HTRC_ERR_ARG;
  if (dim != kDim || block_rows != 64) return HTRC_ERR_UNSUPPORTED;
  if (dtype != HTRC_DTYPE_F32 && dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (rounding != HTRC_ROUND_HALF_EVEN && rounding != HTRC_ROUND_HALF_AWAY) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  launch_pack_blocks(x, dtype, rows, rounding, x8, scale, sqnorm, reinterpret_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

int htrc_kmeans_scratch_size(int64_t n_queries, size_t* bytes) {
  if (n_queries < 1 || bytes == nullptr) return HTRC_ERR_ARG;
  *bytes = kmeans_scratch_bytes(n_queries);
  return HTRC_OK;
}

int htrc_kmeans_order(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, int32_t* perm, void* scratch,
                      size_t scratch_bytes, htrc_stream_t stream) {
  if (!q || !perm || n_queries < 1) return HTRC_ERR_ARG;
  if (dim != kDim) return HTRC_ERR_UNSUPPORTED;
  if (q_dtype != HTRC_DTYPE_F32 && q_dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (n_queries > (int64_t(1) << 31) - 1) return HTRC_ERR_UNSUPPORTED;
  if (scratch == nullptr || scratch_bytes < kmeans_scratch_bytes(n_queries) ||
      (reinterpret_cast<uintptr_t>(scratch) & 255u) != 0)
    return HTRC_ERR_WORKSPACE;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  return launch_kmeans_order(q, q_dtype, n_queries, perm, scratch, reinterpret_cast<cudaStream_t>(stream));
}

int htrc_leaf_stats(const uint16_t* mu_hi, const uint16_t* mu_lo, int64_t nt, int64_t t0, int64_t tc, const uint16_t* k,
                    const uint16_t* v, int64_t n_keys, int32_t dim, int32_t leaf, float scale, int8_t* g8, float* sg,
                    float* lz, uint16_t* vb, const float* kn2, float* cv, int32_t precision, int32_t* status,
                    htrc_stream_t stream) {
  if (!mu_hi || !mu_lo || !k || !v || !g8 || !sg || !lz || !vb) return HTRC_ERR_ARG;
  if ((precision & ~(HTRC_PREC_TF32 | HTRC_PREC_TRITON_DIV)) != 0) return HTRC_ERR_ARG;
  if ((kn2 == nullptr) != (cv == nullptr)) return HTRC_ERR_ARG;
  if (dim != kDim || !leaf_ok(leaf) || (leaf != kLeaf && cv != nullptr)) return HTRC_ERR_UNSUPPORTED;
  if (nt < 1 || t0 < 0 || tc < 1 || t0 + tc > nt || n_keys < leaf || n_keys % leaf) return HTRC_ERR_ARG;
  const int64_t nb = n_keys / leaf;
  if (nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  LeafStatsMaps mp;
  if ((rc = stats_maps(&mp, mu_hi, mu_lo, nt, k, v, n_keys, g8, vb, tc, nb, HTRC_STORE_INT8)) != HTRC_OK) return rc;
  return launch_leaf_stats(mp, sg, lz, pitch_of(nb), t0, tc, static_cast<int>(nb), leaf, scale_of(scale), kn2, cv,
                           nullptr,
                           status, device_info().sms, (precision & HTRC_PREC_TF32) != 0,
                           (precision & HTRC_PREC_TRITON_DIV) != 0, reinterpret_cast<cudaStream_t>(stream));
}

int htrc_tile_prep_fp8(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, int32_t tile,
                       const int32_t* perm, int32_t group, float* mu, uint16_t* mu_hi, uint16_t* mu_lo, uint16_t* qb,
                       uint16_t* dqh, int32_t precision, htrc_stream_t stream) {
  if (!q || !mu || !mu_hi || !mu_lo || !qb || !dqh || n_queries < 1) return HTRC_ERR_ARG;
  if ((precision & ~(HTRC_PREC_TF32 | HTRC_PREC_TRITON_DIV)) != 0) return HTRC_ERR_ARG;
  if (dim != kDim || (tile != kTile && tile != kTile / 2)) return HTRC_ERR_UNSUPPORTED;
  if (q_dtype != HTRC_DTYPE_F32 && q_dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (group > kMaxGroup) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  launch_tile_prep(q, q_dtype, n_queries, tile, perm, group, mu, mu_hi, mu_lo, reinterpret_cast<int8_t*>(qb), nullptr,
                   reinterpret_cast<int8_t*>(dqh), nullptr, nullptr, true, false, (precision & HTRC_PREC_TF32) != 0,
                   (precision & HTRC_PREC_TRITON_DIV) != 0, reinterpret_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

int htrc_leaf_stats_fp8(const uint16_t* mu_hi, const uint16_t* mu_lo, int64_t nt, int64_t t0, int64_t tc,
                        const uint16_t* k, const uint16_t* v, int64_t n_keys, int32_t dim, int32_t leaf, float scale,
                        uint8_t* g8, float* sg, float* lz, uint8_t* vb8, float* sv, int32_t precision,
                        int32_t* status, htrc_stream_t stream) {
  if (!mu_hi || !mu_lo || !k || !v || !g8 || !sg || !lz || !vb8 || !sv) return HTRC_ERR_ARG;
  if ((precision & ~(HTRC_PREC_TF32 | HTRC_PREC_TRITON_DIV)) != 0) return HTRC_ERR_ARG;
  if (dim != kDim || leaf != kLeaf) return HTRC_ERR_UNSUPPORTED;
  if (nt < 1 || t0 < 0 || tc < 1 || t0 + tc > nt || n_keys < leaf || n_keys % leaf) return HTRC_ERR_ARG;
  const int64_t nb = n_keys / leaf;
  if (nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  LeafStatsMaps mp;
  if ((rc = stats_maps(&mp, mu_hi, mu_lo, nt, k, v, n_keys, g8, vb8, tc, nb, HTRC_STORE_FP8)) != HTRC_OK) return rc;
  return launch_leaf_stats(mp, sg, lz, pitch_of(nb), t0, tc, static_cast<int>(nb), kLeaf, scale_of(scale), nullptr,
                           nullptr,
                           sv, status, device_info().sms, (precision & HTRC_PREC_TF32) != 0,
                           (precision & HTRC_PREC_TRITON_DIV) != 0, reinterpret_cast<cudaStream_t>(stream));
}

int htrc_rowmax_select_fp8(const uint16_t* dqh, int64_t t0, int64_t tc, int32_t group, const uint8_t* g8,
                           const float* sg, const float* lz, int64_t nb, int32_t dim, float* sel, int32_t* status,
                           htrc_stream_t stream) {
  if (!dqh || !g8 || !sg || !lz || !sel || t0 < 0 || tc < 1 || nb < 1) return HTRC_ERR_ARG;
  const int64_t g = group > 1 ? group : 1;
  if (g > kMaxGroup || t0 % g) return HTRC_ERR_ARG;
  if (dim != kDim) return HTRC_ERR_UNSUPPORTED;
  if (nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  RowmaxFp8Maps mp;
  if ((rc = rowmax_fp8_maps(&mp, dqh, (t0 + tc) * 64, g8, sg, lz, (tc + g - 1) / g, nb, pitch_of(nb))) != HTRC_OK)
    return rc;
  return launch_rowmax_fp8(mp, sel, pitch_of(nb), t0, tc, static_cast<int>(nb), static_cast<int>(g), status,
                           reinterpret_cast<cudaStream_t>(stream));
}

int htrc_tile_attention_fp8(const uint16_t* qb, const uint16_t* dqh, int64_t n_queries, int32_t tile, int64_t t0,
                            int64_t tc, int32_t group, const uint8_t* g8, const float* sg, const float* lz,
                            const uint8_t* vb8, const float* sv, const uint8_t* excl, const int32_t* idx, int32_t kx,
                            int64_t nb, const uint16_t* k, const uint16_t* v, int64_t n_keys, int32_t dim,
                            int32_t leaf, float scale, const float* tail_part, const int32_t* perm,
                            float* far_part, float* out, float* lse, int32_t* status, htrc_stream_t stream) {
  if (!qb || !dqh || !k || !v || !out || n_queries < 1 || t0 < 0 || tc < 1) return HTRC_ERR_ARG;
  const int64_t g = group > 1 ? group : 1;
  if (g > kMaxGroup || t0 % g) return HTRC_ERR_ARG;
  if (dim != kDim || leaf != kLeaf || (tile != kTile && tile != kTile / 2)) return HTRC_ERR_UNSUPPORTED;
  if (nb < 1 || n_keys != nb * leaf || kx < 0 || kx > nb) return HTRC_ERR_ARG;
  if (kx > kMaxRouted || nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  if (kx < nb && (!g8 || !sg || !lz || !vb8 || !sv || !excl || !far_part)) return HTRC_ERR_ARG;
  if (kx > 0 && !idx) return HTRC_ERR_ARG;
  const int64_t nt = (n_queries + tile - 1) / tile;
  if (t0 + tc > nt) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  // unused state maps (everything routed) still need a valid address: point them at the keys
  const void* kp = static_cast<const void*>(k);
  TileFp8Maps mp;
  if ((rc = tile_fp8_maps(&mp, qb, dqh, nt * 64, static_cast<const uint8_t*>(g8 ? g8 : kp),
                          static_cast<const uint8_t*>(vb8 ? vb8 : kp), lz ? lz : static_cast<const float*>(kp),
                          sg ? sg : static_cast<const float*>(kp), sv ? sv : static_cast<const float*>(kp),
                          excl ? excl : static_cast<const uint8_t*>(kp), (tc + g - 1) / g, nb, pitch_of(nb), k, v,
                          n_keys)) != HTRC_OK)
    return rc;
  return launch_tile_fp8(mp, idx, kx, static_cast<int>(nb), n_queries, tile, t0, tc, static_cast<int>(g),
                         scale_of(scale), tail_part, perm, far_part, out, lse, status,
                         reinterpret_cast<cudaStream_t>(stream));
}

int htrc_tile_prep_bf16(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, int32_t tile,
                        const int32_t* perm, int32_t group, float* mu, uint16_t* mu_hi, uint16_t* mu_lo, uint16_t* qb,
                        uint16_t* dqb, int32_t precision, htrc_stream_t stream) {
  if (!q || !mu || !mu_hi || !mu_lo || !qb || !dqb || n_queries < 1) return HTRC_ERR_ARG;
  if ((precision & ~(HTRC_PREC_TF32 | HTRC_PREC_TRITON_DIV)) != 0) return HTRC_ERR_ARG;
  if (dim != kDim || (tile != kTile && tile != kTile / 2)) return HTRC_ERR_UNSUPPORTED;
  if (q_dtype != HTRC_DTYPE_F32 && q_dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (group > kMaxGroup) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  launch_tile_prep(q, q_dtype, n_queries, tile, perm, group, mu, mu_hi, mu_lo, reinterpret_cast<int8_t*>(qb), nullptr,
                   reinterpret_cast<int8_t*>(dqb), nullptr, nullptr, true, false, (precision & HTRC_PREC_TF32) != 0,
                   (precision & HTRC_PREC_TRITON_DIV) != 0, reinterpret_cast<cudaStream_t>(stream), true);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

int htrc_leaf_stats_bf16(const uint16_t* mu_hi, const uint16_t* mu_lo, int64_t nt, int64_t t0, int64_t tc,
                         const uint16_t* k, const uint16_t* v, int64_t n_keys, int32_t dim, int32_t leaf, float scale,
                         uint16_t* gb, float* lz, uint16_t* vbb, int32_t precision, int32_t* status,
                         htrc_stream_t stream) {
  if (!mu_hi || !mu_lo || !k || !v || !gb || !lz || !vbb) return HTRC_ERR_ARG;
  if ((precision & ~(HTRC_PREC_TF32 | HTRC_PREC_TRITON_DIV)) != 0) return HTRC_ERR_ARG;
  if (dim != kDim || leaf != kLeaf) return HTRC_ERR_UNSUPPORTED;
  if (nt < 1 || t0 < 0 || tc < 1 || t0 + tc > nt || n_keys < leaf || n_keys % leaf) return HTRC_ERR_ARG;
  const int64_t nb = n_keys / leaf;
  if (nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  LeafStatsMaps mp;
  if ((rc = stats_maps(&mp, mu_hi, mu_lo, nt, k, v, n_keys, gb, vbb, tc, nb, HTRC_STORE_BF16)) != HTRC_OK) return rc;
  return launch_leaf_stats(mp, nullptr, lz, pitch_of(nb), t0, tc, static_cast<int>(nb), kLeaf, scale_of(scale),
                           nullptr, nullptr, nullptr, status, device_info().sms, (precision & HTRC_PREC_TF32) != 0,
                           false, reinterpret_cast<cudaStream_t>(stream), true);
}

int htrc_rowmax_select_bf16(const uint16_t* dqb, int64_t t0, int64_t tc, int32_t group, const uint16_t* gb,
                            const float* lz, int64_t nb, int32_t dim, float* sel, int32_t* status,
                            htrc_stream_t stream) {
  if (!dqb || !gb || !lz || !sel || t0 < 0 || tc < 1 || nb < 1) return HTRC_ERR_ARG;
  const int64_t g = group > 1 ? group : 1;
  if (g > kMaxGroup || t0 % g) return HTRC_ERR_ARG;
  if (dim != kDim) return HTRC_ERR_UNSUPPORTED;
  if (nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  RowmaxMaps mp;
  if ((rc = rowmax_bf16_maps(&mp, dqb, (t0 + tc) * 64, gb, lz, (tc + g - 1) / g, nb, pitch_of(nb))) != HTRC_OK)
    return rc;
  return launch_rowmax(mp, nullptr, nullptr, sel, pitch_of(nb), t0, tc, static_cast<int>(nb), static_cast<int>(g),
                       status, reinterpret_cast<cudaStream_t>(stream), true);
}

int htrc_tile_attention_bf16(const uint16_t* qb, const uint16_t* dqb, int64_t n_queries, int32_t tile, int64_t t0,
                             int64_t tc, int32_t group, const uint16_t* gb, const float* lz, const uint16_t* vbb,
                             const uint8_t* excl, const int32_t* idx, int32_t kx, int64_t nb, const uint16_t* k,
                             const uint16_t* v, int64_t n_keys, int32_t dim, int32_t leaf, float scale,
                             const float* tail_part, const int32_t* perm, float* far_part, float* out, float* lse,
                             int32_t* status, htrc_stream_t stream) {
  if (!qb || !dqb || !k || !v || !out || n_queries < 1 || t0 < 0 || tc < 1) return HTRC_ERR_ARG;
  const int64_t g = group > 1 ? group : 1;
  if (g > kMaxGroup || t0 % g) return HTRC_ERR_ARG;
  if (dim != kDim || leaf != kLeaf || (tile != kTile && tile != kTile / 2)) return HTRC_ERR_UNSUPPORTED;
  if (nb < 1 || n_keys != nb * leaf || kx < 0 || kx > nb) return HTRC_ERR_ARG;
  if (kx > kMaxRouted || nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  if (kx < nb && (!gb || !lz || !vbb || !excl || !far_part)) return HTRC_ERR_ARG;
  if (kx > 0 && !idx) return HTRC_ERR_ARG;
  const int64_t nt = (n_queries + tile - 1) / tile;
  if (t0 + tc > nt) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  // unused state maps (everything routed) still need a valid address: point them at the keys
  TileFp8Maps mp;
  if ((rc = tile_bf16_maps(&mp, qb, dqb, nt * 64, gb ? gb : k, vbb ? vbb : v, lz ? lz : reinterpret_cast<const float*>(k),
                           excl ? excl : reinterpret_cast<const uint8_t*>(k), (tc + g - 1) / g, nb, pitch_of(nb), k, v,
                           n_keys)) != HTRC_OK)
    return rc;
  return launch_tile_fp8(mp, idx, kx, static_cast<int>(nb), n_queries, tile, t0, tc, static_cast<int>(g),
                         scale_of(scale), tail_part, perm, far_part, out, lse, status,
                         reinterpret_cast<cudaStream_t>(stream), true);
}

int htrc_rowmax_select(const int8_t* dq8, const float* sdq, const float* dd, int64_t t0, int64_t tc, int32_t group,
                       const int8_t* g8, const float* sg, const float* lz, const float* cv, int64_t nb, int32_t dim,
                       float* sel, int32_t* status, htrc_stream_t stream) {
  if (!dq8 || !sdq || !g8 || !sg || !lz || !sel || t0 < 0 || tc < 1 || nb < 1) return HTRC_ERR_ARG;
  if ((dd == nullptr) != (cv == nullptr)) return HTRC_ERR_ARG;
  const int64_t g = group > 1 ? group : 1;
  if (g > kMaxGroup || t0 % g) return HTRC_ERR_ARG;
  if (dim != kDim) return HTRC_ERR_UNSUPPORTED;
  if (nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  RowmaxMaps mp;
  if ((rc = rowmax_maps(&mp, dq8, (t0 + tc) * 64, g8, sg, lz, cv, (tc + g - 1) / g, nb, pitch_of(nb))) != HTRC_OK)
    return rc;
  return launch_rowmax(mp, sdq, dd, sel, pitch_of(nb), t0, tc, static_cast<int>(nb), static_cast<int>(g), status,
                       reinterpret_cast<cudaStream_t>(stream));
}

int htrc_route(const float* sel, int64_t tc, int64_t nb, int32_t exact_leaves, int32_t sink_leaves, int32_t group,
               int32_t* idx, uint8_t* excl, htrc_stream_t stream) {
  if (!excl || tc < 1 || nb < 1 || exact_leaves < 0 || sink_leaves < 0 || group > kMaxGroup) return HTRC_ERR_ARG;
  if (nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  const int64_t sink = std::min<int64_t>(sink_leaves, nb);
  const int64_t kx = std::min<int64_t>(static_cast<int64_t>(exact_leaves) + sink, nb);
  if (kx > 0 && kx < nb && !sel) return HTRC_ERR_ARG;
  if (kx > 0 && !idx) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  return launch_route(sel, pitch_of(nb), tc, group, static_cast<int>(nb), static_cast<int>(kx), static_cast<int>(sink),
                      idx, excl, reinterpret_cast<cudaStream_t>(stream));
}

int htrc_tile_attention(const int8_t* q8, const float* sq, const int8_t* dq8, const float* sdq, int64_t n_queries,
                        int32_t tile, int64_t t0, int64_t tc, int32_t group, const int8_t* g8, const float* sg,
                        const float* lz, const uint16_t* vb, const uint8_t* excl, const int32_t* idx, int32_t kx,
                        int64_t nb, const int8_t* k8, const float* ks, const uint16_t* v, int64_t n_keys, int32_t dim,
                        int32_t leaf, float scale, const float* tail_part, const int32_t* perm, const float* cv,
                        const float* dd, float* out, float* lse, int32_t* status, htrc_stream_t stream) {
  if (!q8 || !sq || !dq8 || !sdq || !k8 || !ks || !v || !out || n_queries < 1 || t0 < 0 || tc < 1) return HTRC_ERR_ARG;
  if ((dd == nullptr) != (cv == nullptr)) return HTRC_ERR_ARG;
  const int64_t g = group > 1 ? group : 1;
  if (g > kMaxGroup || t0 % g) return HTRC_ERR_ARG;
  if (dim != kDim || !leaf_ok(leaf) || (leaf != kLeaf && cv != nullptr) || (tile != kTile && tile != kTile / 2))
    return HTRC_ERR_UNSUPPORTED;
  if (nb < 1 || n_keys != nb * leaf || kx < 0 || kx > nb) return HTRC_ERR_ARG;
  if (kx > kMaxRouted || nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  if (kx < nb && (!g8 || !sg || !lz || !vb || !excl)) return HTRC_ERR_ARG;
  if (kx > 0 && !idx) return HTRC_ERR_ARG;
  const int64_t nt = (n_queries + tile - 1) / tile;
  if (t0 + tc > nt) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  // unused state maps (everything routed) still need a valid address: point them at the keys
  const void* g8p = g8 ? static_cast<const void*>(g8) : static_cast<const void*>(k8);
  const void* vbp = vb ? static_cast<const void*>(vb) : static_cast<const void*>(v);
  const void* lzp = lz ? static_cast<const void*>(lz) : static_cast<const void*>(ks);
  const void* sgp = sg ? static_cast<const void*>(sg) : static_cast<const void*>(ks);
  const void* exp_ = excl ? static_cast<const void*>(excl) : static_cast<const void*>(k8);
  TileMaps mp;
  if ((rc = tile_maps(&mp, q8, dq8, nt * 64, static_cast<const int8_t*>(g8p), static_cast<const uint16_t*>(vbp),
                      static_cast<const float*>(lzp), static_cast<const float*>(sgp), cv,
                      static_cast<const uint8_t*>(exp_), (tc + g - 1) / g, nb, pitch_of(nb), k8, v, n_keys, leaf)) !=
      HTRC_OK)
    return rc;
  return launch_tile_attention(mp, sq, sdq, ks, idx, kx, static_cast<int>(nb), leaf, n_queries, tile, t0, tc,
                               static_cast<int>(g), scale_of(scale), tail_part, perm, cv ? dd : nullptr, out, lse, status,
                               reinterpret_cast<cudaStream_t>(stream));
}

int htrc_tail_partial(const void* q, int32_t q_dtype, int64_t n_queries, int32_t dim, const float* tail_k,
                      const float* tail_v, int32_t n_tail, float scale, float* tail_part, htrc_stream_t stream) {
  if (!q || !tail_k || !tail_v || !tail_part || n_queries < 1 || n_tail < 1) return HTRC_ERR_ARG;
  if (dim != kDim) return HTRC_ERR_UNSUPPORTED;
  if (q_dtype != HTRC_DTYPE_F32 && q_dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  launch_tail_partial(q, q_dtype, n_queries, tail_k, tail_v, n_tail, scale_of(scale), tail_part,
                      reinterpret_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

int htrc_fake_quant(const void* x, int32_t x_dtype, int64_t rows, int32_t dim, int32_t fmt, int32_t group, void* out,
                    int32_t out_dtype, htrc_stream_t stream) {
  if (!x || !out || rows < 1 || group < 0) return HTRC_ERR_ARG;
  if (fmt < HTRC_FQ_INT8 || fmt > HTRC_FQ_FP4) return HTRC_ERR_ARG;
  if (x_dtype != HTRC_DTYPE_F32 && x_dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (out_dtype != HTRC_DTYPE_F32 && out_dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (dim != kDim) return HTRC_ERR_UNSUPPORTED;
  const int gsz = group == 0 ? (fmt == HTRC_FQ_FP4 ? 16 : dim) : group;
  if (gsz > dim || dim % gsz || (gsz & (gsz - 1))) return HTRC_ERR_ARG;   // the reference: group divides D
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  launch_fake_quant(x, x_dtype, rows, fmt, gsz, out, out_dtype, reinterpret_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

int htrc_dequant_rows(const uint8_t* x8, int64_t stride_x, const float* scale, int64_t stride_s, int64_t rows,
                      int32_t dim, uint16_t* out, htrc_stream_t stream) {
  if (!x8 || !scale || !out || rows < 1 || stride_x < dim || stride_s < 0) return HTRC_ERR_ARG;
  if (dim != kDim) return HTRC_ERR_UNSUPPORTED;
  if ((stride_x & 3) || (reinterpret_cast<uintptr_t>(x8) & 3)) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  launch_dequant_rows(x8, stride_x, scale, stride_s, rows, out, reinterpret_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

int htrc_selftest_wait_timeout(int32_t* status, int64_t limit_cycles, htrc_stream_t stream) {
  if (!status || limit_cycles < 1 || limit_cycles > (int64_t(1) << 34)) return HTRC_ERR_ARG;
  int rc = check_device();
  if (rc != HTRC_OK) return rc;
  wait_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(status, limit_cycles);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

const char* htrc_strerror(int code) {
  switch (code) {
    case HTRC_OK: return "ok";
    case HTRC_ERR_ARG: return "invalid argument";
    case HTRC_ERR_UNSUPPORTED: return "unsupported configuration (needs dim 128, tile 64 or 32, leaf 64, <= 8192 leaves, <= 1024 routed leaves)";
    case HTRC_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case HTRC_ERR_CUDA: return "CUDA runtime error";
    case HTRC_ERR_DEVICE: return "no sm_100 device or device-side failure";
    case HTRC_ERR_TOO_LARGE: return "problem needs more scratch than the 64 MiB static workspace of htrc_flat_forward_static_ws";
    default: return "unknown error";
  }
}

}  // extern "C"
