// Hierarchical HTRC (the reference's NumPy teaching law, src/htrc_reference/model.py:35-137) on the GPU:
// one forest of leaf statistics per query centre, merged up a contiguous tree of `fanout` children, and a
// per-query walk that accepts a node's second-order prediction (log-mass L + g.d + d.H.d / 2, value
// u + J.d) or opens it (exact softmax attention over an opened leaf's keys).
//
// Everything is float32 with fixed reduction orders (bitwise deterministic); rows are 128 wide (the
// host pads narrower keys, values and queries with zeros, which changes no dot product).  The work is
// node-major: a CTA owns one (centre, node) and gathers the queries that reach it from per-query
// bitmasks, so a query pays only for the nodes it visits (a 64-query tile of one centre reaches most
// leaves between its queries while each query reaches few).
//
// Build (per centre c):
//   tree_leaf_kernel    (leaf, c):  a_s = k_s . c for every key, leaf log-mass L = logsumexp a
//   tree_gram_kernel    (node, c):  level-1 nodes from their keys: L, g = sum W k, u = sum W v,
//                                   H = sum W (k - g)(k - g)^T, J^T = (sum W (v - u)(k - g)^T)^T, W = e^(a - L)
//   tree_merge_kernel   (node, c):  levels >= 2 by the merge law (model.py:51-66)
// The leaves keep no H or J: for a leaf, d.H.d and J.d follow from its keys (x_s = k_s . d):
//   g.d = sum w x,  d.H.d = sum w (x - xbar)^2,  u + J.d = sum w (1 + x - xbar) v     (sum w = 1)
// so a visited leaf costs one pass over its keys whether it is accepted or opened.
// Evaluation:
//   tree_group_kernels                 queries grouped by centre (stable)
//   tree_walk_kernel   (parent, c, z): internal levels top-down: lm and d.H.d of the parent's children
//                                      for the queries that opened the parent (all queries at the roots,
//                                      whose predictions give norm); open / accept bits per query
//   tree_count_kernel + tree_scan:     partial records per query (one per accepted internal node, one per
//                                      opened level-1 node) and their offsets; the host reads the total
//   tree_accept_kernel (node, c, z):   u + J.d of accepted internal nodes -> partial records
//   tree_leafblock_kernel (p, c, z):   the leaves of an opened level-1 node: accepted (second order from
//                                      the keys) or opened (exact), merged online -> one partial record
//   tree_final_kernel:                 per query, the partial records merged in record order -> out, lse
#include "common.cuh"
#include "kernels.cuh"
#include "../../include/htrc_tree.h"

#include <cstdlib>
#include <type_traits>

namespace htrc {

namespace {
constexpr int kD = 128;          // row width (keys, queries, values, centres)
constexpr int kMaxLevels = 16;
constexpr int kChunkQ = 64;      // queries per compute chunk
constexpr int kWindow = 1024;    // candidate queries scanned per gather window
constexpr int kStr = 129;        // shared row stride (floats) of scalar-read operand tiles: conflict-free

template <typename T>
__device__ __forceinline__ float4 ld_row4(const T* p, int64_t row, int c4);
template <>
__device__ __forceinline__ float4 ld_row4<float>(const float* p, int64_t row, int c4) {
  return __ldg(reinterpret_cast<const float4*>(p + row * kD) + c4);
}
template <>
__device__ __forceinline__ float4 ld_row4<uint16_t>(const uint16_t* p, int64_t row, int c4) {
  const uint2 x = __ldg(reinterpret_cast<const uint2*>(p + row * kD) + c4);
  return make_float4(__uint_as_float(x.x << 16), __uint_as_float(x.x & 0xFFFF0000u), __uint_as_float(x.y << 16),
                     __uint_as_float(x.y & 0xFFFF0000u));
}

__device__ __forceinline__ float score_of(float lm, float quad, float norm) {
  // model.py:119-120: frac * expm1(min(|quad| / 2, 80)), frac = exp(min(0, lm - norm))
  return expf(fminf(0.f, lm - norm)) * expm1f(fminf(0.5f * fabsf(quad), 80.f));
}

// Gather the queries of centre c in [lo, hi) of the grouped order (hi - lo <= kWindow) whose bit `bit` is
// set in mask[q * words + bit / 32] (mask == nullptr: every query) into list[0 .. return), in candidate order.
// NT threads; thread t owns candidates lo + t * (kWindow / NT) + j: all of its loads go out first (the grouped
// order, then the mask words it names), then one block-wide scan of the per-thread counts places them.
template <int NT>
__device__ int gather_window_n(const int32_t* __restrict__ perm, int64_t lo, int64_t hi,
                               const uint32_t* __restrict__ mask, int words, int bit, int* list, int* wsum) {
  constexpr int kPer = kWindow / NT;
  constexpr int kWarps = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t i0 = lo + static_cast<int64_t>(tid) * kPer;
  int qv[kPer];
  bool tk[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) qv[j] = i0 + j < hi ? perm[i0 + j] : 0;
  int cnt = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    bool t = i0 + j < hi;
    if (t && mask != nullptr) t = (mask[static_cast<int64_t>(qv[j]) * words + (bit >> 5)] >> (bit & 31)) & 1u;
    tk[j] = t;
    cnt += t;
  }
  int x = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  int before = x - cnt, total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const int ws = wsum[w];
    if (w < warp) before += ws;
    total += ws;
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (tk[j]) list[before++] = qv[j];
  __syncthreads();
  return total;
}

__device__ __forceinline__ int gather_window(const int32_t* __restrict__ perm, int64_t lo, int64_t hi,
                                             const uint32_t* __restrict__ mask, int words, int bit, int* list,
                                             int* wsum) {
  return gather_window_n<256>(perm, lo, hi, mask, words, bit, list, wsum);
}

// number of children of node p of a level with n_parent nodes over a child level of n_child nodes
__device__ __forceinline__ int n_children(int p, int fanout, int n_child) {
  const int a = p * fanout;
  return min(n_child, a + fanout) - a;
}

__device__ __forceinline__ int popc_below(const uint32_t* m, int bit) {
  int s = 0;
  for (int w = 0; w < (bit >> 5); ++w) s += __popc(m[w]);
  if (bit & 31) s += __popc(m[bit >> 5] & ((1u << (bit & 31)) - 1u));
  return s;
}

__device__ __forceinline__ int popc_all(const uint32_t* m, int words) {
  int s = 0;
  for (int w = 0; w < words; ++w) s += __popc(m[w]);
  return s;
}
}  // namespace

// ---------------------------------------------------------------------------------------------------
// grouping of the queries by centre: count per centre, then one CTA per centre writes its queries in
// index order (a stable counting sort).  Out-of-range centre indices flag ST_BAD_INDEX.
__global__ void __launch_bounds__(256) tree_count_centres_kernel(const int32_t* __restrict__ assign, int64_t n,
                                                                 int ncen, int* __restrict__ count,
                                                                 int* __restrict__ status) {
  __shared__ int wsum[8];
  const int c = blockIdx.x, tid = threadIdx.x;
  int mine = 0;
  for (int64_t i = tid; i < n; i += 256) {
    const int a = assign[i];
    mine += a == c;
    if (c == 0 && (a < 0 || a >= ncen)) flag_status(status, ST_BAD_INDEX);
  }
  for (int o = 16; o; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
  if ((tid & 31) == 0) wsum[tid >> 5] = mine;
  __syncthreads();
  if (tid == 0) {
    int s = 0;
    for (int w = 0; w < 8; ++w) s += wsum[w];
    count[c] = s;
  }
}

__global__ void __launch_bounds__(256) tree_perm_kernel(const int32_t* __restrict__ assign, int64_t n, int ncen,
                                                        const int* __restrict__ count, int32_t* __restrict__ perm,
                                                        int64_t* __restrict__ coff) {
  __shared__ int wsum[8];
  const int c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int64_t off = 0;
  for (int j = 0; j < c; ++j) off += count[j];
  if (tid == 0) {
    coff[c] = off;
    if (c == ncen - 1) coff[ncen] = off + count[c];
  }
  for (int64_t base = 0; base < n; base += 256) {
    const int64_t i = base + tid;
    const bool take = i < n && assign[i] == c;
    const uint32_t b = __ballot_sync(0xffffffffu, take);
    if (lane == 0) wsum[warp] = __popc(b);
    __syncthreads();
    int before = 0, add = 0;
    for (int w = 0; w < 8; ++w) {
      if (w < warp) before += wsum[w];
      add += wsum[w];
    }
    if (take) perm[off + before + __popc(b & ((1u << lane) - 1u))] = static_cast<int32_t>(i);
    off += add;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------------------
// Leaves (model.py:35-49, :75-76): a_s = k_s . c for the leaf's keys and L = max a + log sum e^(a - max).
// One CTA of 64 threads per (leaf, centre); leaf_size <= 64.
template <typename T>
__global__ void __launch_bounds__(64) tree_leaf_kernel(const T* __restrict__ k, int64_t m, int leaf,
                                                       const float* __restrict__ centres, int nl,
                                                       float* __restrict__ a_out, float* __restrict__ leaf_l,
                                                       float* __restrict__ w_out) {
  __shared__ __align__(16) float ks[64][132];
  __shared__ __align__(16) float cs[kD];
  __shared__ float red[64];
  const int l = blockIdx.x, c = blockIdx.y, tid = threadIdx.x;
  const int64_t s0 = static_cast<int64_t>(l) * leaf;
  const int cnt = static_cast<int>(m - s0 < leaf ? m - s0 : leaf);
  for (int i = tid; i < kD; i += 64) cs[i] = centres[static_cast<int64_t>(c) * kD + i];
  for (int i = tid; i < cnt * 32; i += 64) {
    const int r = i >> 5, c4 = i & 31;
    *reinterpret_cast<float4*>(&ks[r][4 * c4]) = ld_row4<T>(k, s0 + r, c4);
  }
  __syncthreads();
  float a = -INFINITY;
  if (tid < cnt) {
    a = 0.f;
#pragma unroll 8
    for (int d = 0; d < kD; d += 4) {
      const float4 x = *reinterpret_cast<const float4*>(&ks[tid][d]);
      a = fmaf(x.x, cs[d], a);
      a = fmaf(x.y, cs[d + 1], a);
      a = fmaf(x.z, cs[d + 2], a);
      a = fmaf(x.w, cs[d + 3], a);
    }
    a_out[static_cast<int64_t>(c) * m + s0 + tid] = a;
  }
  red[tid] = a;
  __syncthreads();
  for (int o = 32; o; o >>= 1) {
    if (tid < o) red[tid] = fmaxf(red[tid], red[tid + o]);
    __syncthreads();
  }
  const float mx = red[0];
  __syncthreads();
  red[tid] = tid < cnt ? expf(a - mx) : 0.f;
  __syncthreads();
  for (int o = 32; o; o >>= 1) {
    if (tid < o) red[tid] += red[tid + o];
    __syncthreads();
  }
  __syncthreads();
  const float ll = mx + logf(red[0]);
  if (tid == 0) leaf_l[static_cast<int64_t>(c) * nl + l] = ll;
  if (tid < cnt) w_out[static_cast<int64_t>(c) * m + s0 + tid] = expf(a - ll);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Element offset of (row r, column e) of one 128 x 128 bf16 operand part stored as its shared-memory image:
// two K-blocks of 64 columns, each [128 rows][128 B] with the 128-byte swizzle (16-byte chunk c of row r at
// chunk c ^ (r & 7)), so that one bulk copy lands a node's operand ready for the MMA descriptors.
__host__ __device__ __forceinline__ int img_elem(int r, int e) {
  return (e >> 6) * (128 * 64) + r * 64 + ((((e & 63) >> 3) ^ (r & 7)) << 3) + (e & 7);
}

// 8 floats -> their bf16 parts: hi = bf16(x), lo = bf16(x - hi) (16 bytes each)
__device__ __forceinline__ void split_bf16x8(const float* x, uint4* hi, uint4* lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 hb = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    const float2 hf = __bfloat1622float2(hb);
    h[i] = *reinterpret_cast<const uint32_t*>(&hb);
    const __nv_bfloat162 lb = __floats2bfloat162_rn(x[2 * i] - hf.x, x[2 * i + 1] - hf.y);
    l[i] = *reinterpret_cast<const uint32_t*>(&lb);
  }
  *hi = make_uint4(h[0], h[1], h[2], h[3]);
  *lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// ---------------------------------------------------------------------------------------------------
// Level-1 nodes from their keys (model.py:35-49 over the node's keys, equal by the merge identity of
// model.py:51-66 to merging its leaves).  One CTA of 256 threads per (node, centre); the node's keys
// are staged 32 at a time; thread t owns the 8 x 8 blocks (t / 16, t % 16) of H and of J.
constexpr int kGramRows = 32;
struct GramSmem {
  float a[kGramRows][132];     // W_s (k_s - g)          (pass 1: raw keys)
  float b[kGramRows][132];     // k_s - g
  float cv[kGramRows][132];    // W_s (v_s - u)          (pass 1: raw values)
  float g[kD], u[kD];
  float w[kGramRows];
  float ln;
};

template <typename T>
__global__ void __launch_bounds__(256, 1) tree_gram_kernel(const T* __restrict__ k, const T* __restrict__ v, int64_t m,
                                                           int leaf, int fanout, int nl, const float* __restrict__ a,
                                                           const float* __restrict__ leaf_l, int n1,
                                                           float* __restrict__ L1, float* __restrict__ g1,
                                                           float* __restrict__ u1, float* __restrict__ H1,
                                                           float* __restrict__ JT1, uint16_t* __restrict__ Hb1,
                                                           uint16_t* __restrict__ Jb1) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  GramSmem& sh = *reinterpret_cast<GramSmem*>(smem_raw);
  const int i = blockIdx.x, c = blockIdx.y, tid = threadIdx.x;
  const int l0 = i * fanout, l1 = min(nl, l0 + fanout);
  const int64_t k0 = static_cast<int64_t>(l0) * leaf;
  const int64_t k1 = min(m, static_cast<int64_t>(l1) * leaf);
  const float* ac = a + static_cast<int64_t>(c) * m;
  if (tid == 0) {
    float mx = -INFINITY;
    for (int l = l0; l < l1; ++l) mx = fmaxf(mx, leaf_l[static_cast<int64_t>(c) * nl + l]);
    float s = 0.f;
    for (int l = l0; l < l1; ++l) s += expf(leaf_l[static_cast<int64_t>(c) * nl + l] - mx);
    sh.ln = mx + logf(s);
  }
  __syncthreads();
  const float ln = sh.ln;
  // pass 1: g = sum W k (threads 0..127), u = sum W v (threads 128..255), keys in order
  float acc1 = 0.f;
  for (int64_t base = k0; base < k1; base += kGramRows) {
    const int cnt = static_cast<int>(k1 - base < kGramRows ? k1 - base : kGramRows);
    for (int x = tid; x < cnt * 32; x += 256) {
      const int r = x >> 5, c4 = x & 31;
      *reinterpret_cast<float4*>(&sh.a[r][4 * c4]) = ld_row4<T>(k, base + r, c4);
      *reinterpret_cast<float4*>(&sh.cv[r][4 * c4]) = ld_row4<T>(v, base + r, c4);
    }
    if (tid < cnt) sh.w[tid] = expf(ac[base + tid] - ln);
    __syncthreads();
    if (tid < kD) {
      for (int s = 0; s < cnt; ++s) acc1 = fmaf(sh.w[s], sh.a[s][tid], acc1);
    } else {
      for (int s = 0; s < cnt; ++s) acc1 = fmaf(sh.w[s], sh.cv[s][tid - kD], acc1);
    }
    __syncthreads();
  }
  if (tid < kD) sh.g[tid] = acc1; else sh.u[tid - kD] = acc1;
  __syncthreads();
  const int64_t node = static_cast<int64_t>(c) * n1 + i;
  if (tid < kD) g1[node * kD + tid] = sh.g[tid]; else u1[node * kD + tid - kD] = sh.u[tid - kD];
  if (tid == 0) L1[node] = ln;
  // pass 2: H = sum W (k - g)(k - g)^T, J = sum W (v - u)(k - g)^T
  const int rb = tid >> 4, cb = tid & 15;
  float h[8][8], j[8][8];
#pragma unroll
  for (int x = 0; x < 8; ++x)
#pragma unroll
    for (int y = 0; y < 8; ++y) h[x][y] = j[x][y] = 0.f;
  for (int64_t base = k0; base < k1; base += kGramRows) {
    const int cnt = static_cast<int>(k1 - base < kGramRows ? k1 - base : kGramRows);
    if (tid < cnt) sh.w[tid] = expf(ac[base + tid] - ln);
    __syncthreads();
    for (int x = tid; x < cnt * 32; x += 256) {
      const int r = x >> 5, c4 = x & 31;
      const float4 kk = ld_row4<T>(k, base + r, c4);
      const float4 vv = ld_row4<T>(v, base + r, c4);
      const float w = sh.w[r];
      const float g0 = sh.g[4 * c4], g1_ = sh.g[4 * c4 + 1], g2 = sh.g[4 * c4 + 2], g3 = sh.g[4 * c4 + 3];
      const float4 bk = make_float4(kk.x - g0, kk.y - g1_, kk.z - g2, kk.w - g3);
      *reinterpret_cast<float4*>(&sh.b[r][4 * c4]) = bk;
      *reinterpret_cast<float4*>(&sh.a[r][4 * c4]) = make_float4(w * bk.x, w * bk.y, w * bk.z, w * bk.w);
      *reinterpret_cast<float4*>(&sh.cv[r][4 * c4]) =
          make_float4(w * (vv.x - sh.u[4 * c4]), w * (vv.y - sh.u[4 * c4 + 1]), w * (vv.z - sh.u[4 * c4 + 2]),
                      w * (vv.w - sh.u[4 * c4 + 3]));
    }
    __syncthreads();
    for (int s = 0; s < cnt; ++s) {
      float av[8], cvv[8], bv[8];
      *reinterpret_cast<float4*>(&av[0]) = *reinterpret_cast<const float4*>(&sh.a[s][rb * 8]);
      *reinterpret_cast<float4*>(&av[4]) = *reinterpret_cast<const float4*>(&sh.a[s][rb * 8 + 4]);
      *reinterpret_cast<float4*>(&cvv[0]) = *reinterpret_cast<const float4*>(&sh.cv[s][rb * 8]);
      *reinterpret_cast<float4*>(&cvv[4]) = *reinterpret_cast<const float4*>(&sh.cv[s][rb * 8 + 4]);
      *reinterpret_cast<float4*>(&bv[0]) = *reinterpret_cast<const float4*>(&sh.b[s][cb * 8]);
      *reinterpret_cast<float4*>(&bv[4]) = *reinterpret_cast<const float4*>(&sh.b[s][cb * 8 + 4]);
#pragma unroll
      for (int x = 0; x < 8; ++x)
#pragma unroll
        for (int y = 0; y < 8; ++y) {
          h[x][y] = fmaf(av[x], bv[y], h[x][y]);
          j[x][y] = fmaf(cvv[x], bv[y], j[x][y]);
        }
    }
    __syncthreads();
  }
  float* hn = H1 + node * kD * kD;
  float* jn = JT1 + node * kD * kD;
#pragma unroll
  for (int x = 0; x < 8; ++x) {
    *reinterpret_cast<float4*>(hn + (rb * 8 + x) * kD + cb * 8) = make_float4(h[x][0], h[x][1], h[x][2], h[x][3]);
    *reinterpret_cast<float4*>(hn + (rb * 8 + x) * kD + cb * 8 + 4) = make_float4(h[x][4], h[x][5], h[x][6], h[x][7]);
  }
#pragma unroll
  for (int y = 0; y < 8; ++y) {      // J^T[e][d] = J[d][e]
    *reinterpret_cast<float4*>(jn + (cb * 8 + y) * kD + rb * 8) = make_float4(j[0][y], j[1][y], j[2][y], j[3][y]);
    *reinterpret_cast<float4*>(jn + (cb * 8 + y) * kD + rb * 8 + 4) = make_float4(j[4][y], j[5][y], j[6][y], j[7][y]);
  }
  // bf16 hi / lo operand copies for the tensor-core walk: H rows and J rows (J[d][e], d = value dim)
  uint16_t* hb = Hb1 + node * 2 * kD * kD;
  uint16_t* jb = Jb1 + node * 2 * kD * kD;
#pragma unroll
  for (int x = 0; x < 8; ++x) {
    uint4 hi, lo;
    const int e = img_elem(rb * 8 + x, cb * 8);
    split_bf16x8(h[x], &hi, &lo);
    *reinterpret_cast<uint4*>(hb + e) = hi;
    *reinterpret_cast<uint4*>(hb + kD * kD + e) = lo;
    split_bf16x8(j[x], &hi, &lo);
    *reinterpret_cast<uint4*>(jb + e) = hi;
    *reinterpret_cast<uint4*>(jb + kD * kD + e) = lo;
  }
}

// Level-1 nodes on the tensor cores: pass 1 as tree_gram_kernel (L, g, u on the CUDA cores), then
//   H = (W ck)^T ck,  J = (W cv)^T ck    (ck = k - g, cv = v - u, W = e^(a - L) over the node's keys)
// as tcgen05 kind::f16 MMAs (M 128 dims x N 128 dims x K 32 keys per stage) with every operand split into three
// bf16 parts (x = h + m + l, 24 significant bits) and the six products of order up to 2^-16 (hh, hm, mh, hl,
// lh, mm): float32-level sums over the node's 1024 keys.  The operands are written by the CTA's threads in the
// 128-byte-swizzled MN-major layout (a key's 128 dims contiguous); H in TMEM columns 0..127, J in 128..255.
// One CTA of 256 threads per (node, centre), two per SM.
constexpr int kGtKeys = 32;                             // keys per stage
constexpr uint32_t kGtTile = 2 * kGtKeys * 128;         // one operand part: two 64-dim chunks of [32 key rows][128 B]
struct __align__(1024) GramTcSmem {
  uint8_t t[9][kGtTile];      // W ck h, m, l | W cv h, m, l | ck h, m, l   (pass 1 reuses the space as float rows)
  float g[kD], u[kD];
  float w[64];
  float ln;
  uint64_t bar;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t kGramTcSmemBytes = 80 * 1024;          // > 228 KB / 3: at most two CTAs (512 TMEM columns) per SM
static_assert(sizeof(GramTcSmem) + 1024 <= kGramTcSmemBytes, "tree build shared layout");

// 8 floats -> three bf16 parts each (x = h + m + l to 24 significant bits), 16 bytes per part
__device__ __forceinline__ void split3_bf16x8(const float* x, uint4* h, uint4* mm, uint4* l) {
  float r[8];
  uint4 t;
  split_bf16x8(x, h, &t);
  const uint32_t hw[4] = {h->x, h->y, h->z, h->w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 hf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hw[i]));
    r[2 * i] = x[2 * i] - hf.x;
    r[2 * i + 1] = x[2 * i + 1] - hf.y;
  }
  split_bf16x8(r, mm, l);
}

template <typename T>
__global__ void __launch_bounds__(256, 1) tree_gram_tc_kernel(
    const T* __restrict__ k, const T* __restrict__ v, int64_t m, int leaf, int fanout, int nl,
    const float* __restrict__ a, const float* __restrict__ leaf_l, int n1, float* __restrict__ L1,
    float* __restrict__ g1, float* __restrict__ u1, float* __restrict__ H1, float* __restrict__ JT1,
    uint16_t* __restrict__ Hb1, uint16_t* __restrict__ Jb1, int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  GramTcSmem& sh = *reinterpret_cast<GramTcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int i = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, warp = tid >> 5;
  const int l0 = i * fanout, l1 = min(nl, l0 + fanout);
  const int64_t k0 = static_cast<int64_t>(l0) * leaf;
  const int64_t k1 = min(m, static_cast<int64_t>(l1) * leaf);
  const float* ac = a + static_cast<int64_t>(c) * m;
  if (tid == 0) {
    float mx = -INFINITY;
    for (int l = l0; l < l1; ++l) mx = fmaxf(mx, leaf_l[static_cast<int64_t>(c) * nl + l]);
    float s = 0.f;
    for (int l = l0; l < l1; ++l) s += expf(leaf_l[static_cast<int64_t>(c) * nl + l] - mx);
    sh.ln = mx + logf(s);
    mbar_init(&sh.bar, 1);
    sh.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&sh.tmem_base, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const float ln = sh.ln;
  const uint32_t tmem = sh.tmem_base;
  // pass 1: g = sum W k (threads 0..127), u = sum W v (threads 128..255), keys in order
  {
    float (*kr)[132] = reinterpret_cast<float (*)[132]>(sh.t[0]);
    float (*vr)[132] = reinterpret_cast<float (*)[132]>(sh.t[0] + 32 * 132 * 4);
    float acc1 = 0.f;
    for (int64_t base = k0; base < k1; base += 32) {
      const int cnt = static_cast<int>(k1 - base < 32 ? k1 - base : 32);
      for (int x = tid; x < cnt * 32; x += 256) {
        const int r = x >> 5, c4 = x & 31;
        *reinterpret_cast<float4*>(&kr[r][4 * c4]) = ld_row4<T>(k, base + r, c4);
        *reinterpret_cast<float4*>(&vr[r][4 * c4]) = ld_row4<T>(v, base + r, c4);
      }
      if (tid < cnt) sh.w[tid] = expf(ac[base + tid] - ln);
      __syncthreads();
      if (tid < kD) {
        for (int s = 0; s < cnt; ++s) acc1 = fmaf(sh.w[s], kr[s][tid], acc1);
      } else {
        for (int s = 0; s < cnt; ++s) acc1 = fmaf(sh.w[s], vr[s][tid - kD], acc1);
      }
      __syncthreads();
    }
    if (tid < kD) sh.g[tid] = acc1; else sh.u[tid - kD] = acc1;
  }
  __syncthreads();
  const int64_t node = static_cast<int64_t>(c) * n1 + i;
  if (tid < kD) g1[node * kD + tid] = sh.g[tid]; else u1[node * kD + tid - kD] = sh.u[tid - kD];
  if (tid == 0) L1[node] = ln;
  // pass 2 on the tensor cores, 32 keys per stage; warps 0..3 own the H rows (TMEM lane d = row d), warps 4..7
  // the J rows (value dim dv = lane)
  const int d = tid & 127;
  const uint32_t lane_off = static_cast<uint32_t>(d & ~31) << 16;
  const bool isj = tid >= 128;
  float racc[kD];
#pragma unroll
  for (int j = 0; j < kD; ++j) racc[j] = 0.f;
  const uint32_t idesc = idesc_bf16(128, 128, true, true);
  const uint32_t t0 = smem_u32(sh.t[0]);
  uint32_t phase = 0;
  bool ok = true;
  for (int64_t base = k0; base < k1 && ok; base += kGtKeys) {
    const int cnt = static_cast<int>(k1 - base < kGtKeys ? k1 - base : kGtKeys);
    if (tid < kGtKeys) sh.w[tid] = tid < cnt ? expf(ac[base + tid] - ln) : 0.f;
    __syncthreads();
    for (int x = tid; x < kGtKeys * 16; x += 256) {
      const int r = x >> 4, cc = x & 15;
      float ck[8], aw[8], jw[8];
      if (r < cnt) {
        const float4 k0v = ld_row4<T>(k, base + r, 2 * cc), k1v = ld_row4<T>(k, base + r, 2 * cc + 1);
        const float4 v0v = ld_row4<T>(v, base + r, 2 * cc), v1v = ld_row4<T>(v, base + r, 2 * cc + 1);
        const float kk[8] = {k0v.x, k0v.y, k0v.z, k0v.w, k1v.x, k1v.y, k1v.z, k1v.w};
        const float vv[8] = {v0v.x, v0v.y, v0v.z, v0v.w, v1v.x, v1v.y, v1v.z, v1v.w};
        const float w = sh.w[r];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ck[e] = kk[e] - sh.g[8 * cc + e];
          aw[e] = w * ck[e];
          jw[e] = w * (vv[e] - sh.u[8 * cc + e]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) ck[e] = aw[e] = jw[e] = 0.f;
      }
      const uint32_t off = (cc >> 3) * (kGtKeys * 128) + sw128_off(r, cc & 7);
      uint4 p0, p1, p2;
      split3_bf16x8(aw, &p0, &p1, &p2);
      st_shared_v4(t0 + 0 * kGtTile + off, p0);
      st_shared_v4(t0 + 1 * kGtTile + off, p1);
      st_shared_v4(t0 + 2 * kGtTile + off, p2);
      split3_bf16x8(jw, &p0, &p1, &p2);
      st_shared_v4(t0 + 3 * kGtTile + off, p0);
      st_shared_v4(t0 + 4 * kGtTile + off, p1);
      st_shared_v4(t0 + 5 * kGtTile + off, p2);
      split3_bf16x8(ck, &p0, &p1, &p2);
      st_shared_v4(t0 + 6 * kGtTile + off, p0);
      st_shared_v4(t0 + 7 * kGtTile + off, p1);
      st_shared_v4(t0 + 8 * kGtTile + off, p2);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      // (A part, B part): h.h, h.m, m.h, h.l, l.h, m.m; each stage's sum starts afresh in TMEM
      const int ap[6] = {0, 0, 1, 0, 2, 1}, bp[6] = {0, 1, 0, 2, 0, 1};
#pragma unroll
      for (int kk = 0; kk < kGtKeys / 16; ++kk)
#pragma unroll
        for (int pr = 0; pr < 6; ++pr) {
          const uint64_t bd = sw128_desc(t0 + (6 + bp[pr]) * kGtTile + kk * 2048, kGtKeys * 128, 1024);
          const uint32_t acc = (kk || pr) ? 1u : 0u;
          mma_bf16(tmem, sw128_desc(t0 + (0 + ap[pr]) * kGtTile + kk * 2048, kGtKeys * 128, 1024), bd, idesc, acc);
          mma_bf16(tmem + 128, sw128_desc(t0 + (3 + ap[pr]) * kGtTile + kk * 2048, kGtKeys * 128, 1024), bd, idesc,
                   acc);
        }
      mma_commit(&sh.bar);
    }
    ok = mbar_wait(&sh.bar, phase, status, &sh.abort_flag);
    phase ^= 1u;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    // fold this stage's 32-key sums into the row's float32 accumulators (IEEE adds across stages: the tensor
    // core's own accumulation covers 32 keys only)
    tc_fence_after();
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      uint32_t y[32];
      tmem_ld32(tmem + lane_off + (isj ? 128 : 0) + 32 * cb, y);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) racc[32 * cb + j] += __uint_as_float(y[j]);
    }
    tc_fence_before();
    __syncthreads();
  }
  if (ok) {
    float* hn = H1 + node * kD * kD;
    float* jt = JT1 + node * kD * kD;
    uint16_t* bn = (isj ? Jb1 : Hb1) + node * 2 * kD * kD;
    if (!isj) {
#pragma unroll
      for (int j = 0; j < kD; j += 4)
        *reinterpret_cast<float4*>(hn + d * kD + j) = make_float4(racc[j], racc[j + 1], racc[j + 2], racc[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < kD; ++j) jt[j * kD + d] = racc[j];          // J^T[e][dv]
    }
#pragma unroll
    for (int j = 0; j < kD; j += 8) {
      uint4 h, l;
      split_bf16x8(racc + j, &h, &l);
      *reinterpret_cast<uint4*>(bn + img_elem(d, j)) = h;
      *reinterpret_cast<uint4*>(bn + kD * kD + img_elem(d, j)) = l;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// Levels >= 2 (model.py:51-66): w = softmax of the children's log-masses, g = sum w g_c, u = sum w u_c,
// H = sum w (H_c + dg dg^T), J = sum w (J_c + du dg^T).  One CTA of 256 threads per (node, centre);
// fanout <= 64.
struct MergeSmem {
  float dg[64][kD];
  float du[64][kD];
  float w[64];
  float g[kD], u[kD];
  float ln;
};

__global__ void __launch_bounds__(256) tree_merge_kernel(int fanout, int nch, const float* __restrict__ Lc,
                                                         const float* __restrict__ gc, const float* __restrict__ uc,
                                                         const float* __restrict__ Hc, const float* __restrict__ JTc,
                                                         int np, float* __restrict__ Lp, float* __restrict__ gp,
                                                         float* __restrict__ up, float* __restrict__ Hp,
                                                         float* __restrict__ JTp, uint16_t* __restrict__ Hbp,
                                                         uint16_t* __restrict__ Jbp) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  MergeSmem& sh = *reinterpret_cast<MergeSmem*>(smem_raw);
  const int i = blockIdx.x, c = blockIdx.y, tid = threadIdx.x;
  const int j0 = i * fanout, nc = min(nch, j0 + fanout) - j0;
  const int64_t cb0 = static_cast<int64_t>(c) * nch + j0;     // first child's node index
  if (tid == 0) {
    float mx = -INFINITY;
    for (int x = 0; x < nc; ++x) mx = fmaxf(mx, Lc[cb0 + x]);
    float s = 0.f;
    for (int x = 0; x < nc; ++x) s += expf(Lc[cb0 + x] - mx);
    const float ln = mx + logf(s);
    sh.ln = ln;
    for (int x = 0; x < nc; ++x) sh.w[x] = expf(Lc[cb0 + x] - ln);
  }
  __syncthreads();
  {
    const bool isg = tid < kD;
    const int d = isg ? tid : tid - kD;
    const float* src = isg ? gc : uc;
    float s = 0.f;
    for (int x = 0; x < nc; ++x) s = fmaf(sh.w[x], src[(cb0 + x) * kD + d], s);
    (isg ? sh.g : sh.u)[d] = s;
  }
  __syncthreads();
  for (int e = tid; e < nc * kD; e += 256) {
    const int x = e / kD, d = e % kD;
    sh.dg[x][d] = gc[(cb0 + x) * kD + d] - sh.g[d];
    sh.du[x][d] = uc[(cb0 + x) * kD + d] - sh.u[d];
  }
  const int64_t node = static_cast<int64_t>(c) * np + i;
  if (tid < kD) gp[node * kD + tid] = sh.g[tid]; else up[node * kD + tid - kD] = sh.u[tid - kD];
  if (tid == 0) Lp[node] = sh.ln;
  __syncthreads();
  for (int e = tid; e < kD * kD; e += 256) {
    const int r = e / kD, f = e % kD;
    float hs = 0.f, js = 0.f;
    for (int x = 0; x < nc; ++x) {
      const float w = sh.w[x];
      hs = fmaf(w, Hc[(cb0 + x) * kD * kD + e] + sh.dg[x][r] * sh.dg[x][f], hs);
      js = fmaf(w, JTc[(cb0 + x) * kD * kD + e] + sh.du[x][f] * sh.dg[x][r], js);   // J^T[r][f] = J[f][r]
    }
    Hp[node * kD * kD + e] = hs;
    JTp[node * kD * kD + e] = js;
    const __nv_bfloat16 hh = __float2bfloat16_rn(hs), jh = __float2bfloat16_rn(js);
    uint16_t* hb = Hbp + node * 2 * kD * kD;
    uint16_t* jb = Jbp + node * 2 * kD * kD;
    hb[img_elem(r, f)] = __bfloat16_as_ushort(hh);
    hb[kD * kD + img_elem(r, f)] = __bfloat16_as_ushort(__float2bfloat16_rn(hs - __bfloat162float(hh)));
    jb[img_elem(f, r)] = __bfloat16_as_ushort(jh);                   // J[f][r] = J^T[r][f]
    jb[kD * kD + img_elem(f, r)] = __bfloat16_as_ushort(__float2bfloat16_rn(js - __bfloat162float(jh)));
  }
}

// ---------------------------------------------------------------------------------------------------
// Evaluation.  TreeLevels describes the forest and the walk state; level 0 is the leaves, `top` the roots.
struct TreeLevels {
  int top, fanout, leaf;
  int n[kMaxLevels];          // nodes per level (per centre)
  int words[kMaxLevels];      // 32-bit words per query of the level's open / accept bitmasks
  uint32_t* open[kMaxLevels]; // [N][words] opened nodes of level l (l >= 1)
  uint32_t* acc[kMaxLevels];  // [N][words] accepted nodes of level l (l >= 1)
  float* lm[kMaxLevels];      // [N][n] predicted log-mass of the visited nodes of level l (l >= 1)
  const float* L[kMaxLevels]; // [C][n]          node log-mass (level 0: leaf log-mass)
  const float* g[kMaxLevels]; // [C][n][128]     (l >= 1)
  const float* u[kMaxLevels]; // [C][n][128]     (l >= 1)
  const float* H[kMaxLevels]; // [C][n][128][128] (l >= 1)
  const float* JT[kMaxLevels];// [C][n][128][128] (l >= 1), J transposed
  const uint16_t* Hb[kMaxLevels];  // [C][n][hi, lo] bf16 parts of H as shared-memory images (img_elem)
  const uint16_t* Jb[kMaxLevels];  // [C][n][hi, lo] bf16 parts of J (rows: value dims) as images
};

// Stage delta rows (scale * q - c) of list[0 .. nq) into ds[64][kStr]; rows nq..63 are zero.
template <typename T>
__device__ __forceinline__ void stage_delta(const T* __restrict__ q, float scale, const float* cs, const int* list,
                                            int nq, float (*ds)[kStr]) {
  for (int x = threadIdx.x; x < kChunkQ * 32; x += 256) {
    const int r = x >> 5, c4 = x & 31;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nq) {
      const float4 y = ld_row4<T>(q, list[r], c4);
      v = make_float4(fmaf(scale, y.x, -cs[4 * c4]), fmaf(scale, y.y, -cs[4 * c4 + 1]),
                      fmaf(scale, y.z, -cs[4 * c4 + 2]), fmaf(scale, y.w, -cs[4 * c4 + 3]));
    }
    ds[r][4 * c4] = v.x;
    ds[r][4 * c4 + 1] = v.y;
    ds[r][4 * c4 + 2] = v.z;
    ds[r][4 * c4 + 3] = v.w;
  }
}

// acc[i][j] = sum_k ds[qb * 4 + i][k] * M[k][cb * 8 + j]   (M row-major 128 x 128 in global memory)
__device__ __forceinline__ void delta_gemm(const float (*ds)[kStr], const float* __restrict__ M, int qb, int cb,
                                           float acc[4][8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  const float4* mp = reinterpret_cast<const float4*>(M) + cb * 2;
#pragma unroll 4
  for (int k = 0; k < kD; ++k) {
    const float4 m0 = __ldg(mp + k * 32), m1 = __ldg(mp + k * 32 + 1);
    const float mv[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float d = ds[qb * 4 + i][k];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(d, mv[j], acc[i][j]);
    }
  }
}

struct WalkSmem {
  float ds[kChunkQ][kStr];
  float lms[kChunkQ][65];
  float qds[kChunkQ][65];
  float cs[kD];
  float nrm[kChunkQ];
  int list[kWindow];
  int wsum[8];
};

// One internal level: the children (level lev) of parent p (level lev + 1) for the queries that opened p,
// or, with p < 0, the roots (level lev = top) for every query of centre c, whose predicted log-masses
// give norm (model.py:108-110).  Per (query, child): lm, |d.H.d|, then open or accept (model.py:112-127).
template <typename T>
__global__ void __launch_bounds__(256) tree_walk_kernel(const T* __restrict__ q, float scale,
                                                        const float* __restrict__ centres,
                                                        const int32_t* __restrict__ perm,
                                                        const int64_t* __restrict__ coff, int64_t slice,
                                                        TreeLevels lv, int lev, int root_mode, float thr,
                                                        float* __restrict__ norm) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  WalkSmem& sh = *reinterpret_cast<WalkSmem*>(smem_raw);
  const int c = blockIdx.y, tid = threadIdx.x, qb = tid >> 4, cb = tid & 15;
  const int p = root_mode ? -1 : static_cast<int>(blockIdx.x);
  const int64_t lo = coff[c] + static_cast<int64_t>(blockIdx.z) * slice;
  const int64_t hi = min(coff[c + 1], lo + slice);
  if (lo >= hi) return;
  const int n_lev = lv.n[lev];
  const int ch0 = root_mode ? 0 : p * lv.fanout;
  const int ch1 = root_mode ? n_lev : min(n_lev, ch0 + lv.fanout);
  for (int x = tid; x < kD; x += 256) sh.cs[x] = centres[static_cast<int64_t>(c) * kD + x];
  const uint32_t* pmask = root_mode ? nullptr : lv.open[lev + 1];
  const int pwords = root_mode ? 0 : lv.words[lev + 1];
  const int64_t nodes0 = static_cast<int64_t>(c) * n_lev;
  __syncthreads();
  for (int64_t win = lo; win < hi; win += kWindow) {
    const int cnt = gather_window(perm, win, min(hi, win + kWindow), pmask, pwords, p, sh.list, sh.wsum);
    for (int b0 = 0; b0 < cnt; b0 += kChunkQ) {
      const int nq = min(kChunkQ, cnt - b0);
      const int* lst = sh.list + b0;
      stage_delta<T>(q, scale, sh.cs, lst, nq, sh.ds);
      if (!root_mode && tid < nq) sh.nrm[tid] = norm[lst[tid]];
      __syncthreads();
      for (int n = ch0; n < ch1; ++n) {
        const int64_t node = nodes0 + n;
        float acc[4][8];
        delta_gemm(sh.ds, lv.H[lev] + node * kD * kD, qb, cb, acc);
        const float* gn = lv.g[lev] + node * kD + cb * 8;
        float r[4], qd[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          r[i] = 0.f;
          qd[i] = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float d = sh.ds[qb * 4 + i][cb * 8 + j];
            qd[i] = fmaf(d, acc[i][j], qd[i]);
            r[i] = fmaf(d, __ldg(gn + j), r[i]);
          }
        }
#pragma unroll
        for (int o = 8; o; o >>= 1)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            qd[i] += __shfl_xor_sync(0xffffffffu, qd[i], o);
            r[i] += __shfl_xor_sync(0xffffffffu, r[i], o);
          }
        if (cb == 0) {
          const float ln = lv.L[lev][node];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int jq = qb * 4 + i;
            if (jq >= nq) continue;
            const float lm = ln + r[i] + 0.5f * qd[i];
            if (root_mode) {
              sh.lms[jq][n] = lm;
              sh.qds[jq][n] = qd[i];
            } else {
              const int qq = lst[jq];
              lv.lm[lev][static_cast<int64_t>(qq) * n_lev + n] = lm;
              uint32_t* dst = score_of(lm, qd[i], sh.nrm[jq]) > thr ? lv.open[lev] : lv.acc[lev];
              atomicOr(dst + static_cast<int64_t>(qq) * lv.words[lev] + (n >> 5), 1u << (n & 31));
            }
          }
        }
      }
      if (root_mode) {
        __syncthreads();
        if (tid < nq) {
          const int qq = lst[tid];
          float mx = -INFINITY;
          for (int n = 0; n < n_lev; ++n) mx = fmaxf(mx, sh.lms[tid][n]);
          float s = 0.f;
          for (int n = 0; n < n_lev; ++n) s += expf(sh.lms[tid][n] - mx);
          const float nr = mx + logf(s);
          norm[qq] = nr;
          uint32_t ob[2] = {0u, 0u}, ab[2] = {0u, 0u};
          for (int n = 0; n < n_lev; ++n) {
            const float lm = sh.lms[tid][n];
            lv.lm[lev][static_cast<int64_t>(qq) * n_lev + n] = lm;
            if (score_of(lm, sh.qds[tid][n], nr) > thr) ob[n >> 5] |= 1u << (n & 31);
            else ab[n >> 5] |= 1u << (n & 31);
          }
          for (int w = 0; w < lv.words[lev]; ++w) {
            lv.open[lev][static_cast<int64_t>(qq) * lv.words[lev] + w] = ob[w];
            lv.acc[lev][static_cast<int64_t>(qq) * lv.words[lev] + w] = ab[w];
          }
        }
      }
      __syncthreads();
    }
  }
}

// Per query: the number of partial records (accepted internal nodes + opened level-1 nodes, or one for a
// forest whose roots are its leaves) and the reference's counters visited_nodes / accepted_nodes without
// the exact leaves' share (model.py:113-127: every visited node is traversed once; an accepted internal
// node and every visited leaf add one accepted entry).
__global__ void __launch_bounds__(256) tree_count_kernel(TreeLevels lv, int64_t nq, int64_t* __restrict__ count,
                                                         int32_t* __restrict__ visited,
                                                         int32_t* __restrict__ accepted,
                                                         int32_t* __restrict__ leaves_out) {
  const int64_t qq = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (qq >= nq) return;
  const int top = lv.top, F = lv.fanout;
  if (top == 0) {
    count[qq] = 1;
    visited[qq] = lv.n[0];
    accepted[qq] = lv.n[0];
    if (leaves_out) leaves_out[qq] = lv.n[0];
    return;
  }
  int vis = lv.n[top], acc_int = 0;
  int64_t cnt = 0;
  for (int l = top; l >= 1; --l) acc_int += popc_all(lv.acc[l] + qq * lv.words[l], lv.words[l]);
  cnt += acc_int;
  int leaves = 0;
  for (int l = top; l >= 1; --l) {
    const uint32_t* om = lv.open[l] + qq * lv.words[l];
    const int o = popc_all(om, lv.words[l]);
    const int last = lv.n[l] - 1;
    const bool last_open = (om[last >> 5] >> (last & 31)) & 1u;
    const int ch = o * F - (last_open ? F - n_children(last, F, lv.n[l - 1]) : 0);
    if (l >= 2) vis += ch; else leaves = ch;
    if (l == 1) cnt += o;
  }
  count[qq] = cnt;
  visited[qq] = vis + leaves;
  accepted[qq] = acc_int + leaves;
  if (leaves_out) leaves_out[qq] = leaves;
}

// Exclusive prefix sum of count[0 .. n) into base[0 .. n] (base[n] = total).  One CTA of 1024 threads,
// each a contiguous range.
__global__ void __launch_bounds__(1024) tree_scan_kernel(const int64_t* __restrict__ count, int64_t n,
                                                         int64_t* __restrict__ base) {
  __shared__ int64_t ws[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t per = (n + 1023) / 1024;
  const int64_t a = min(n, tid * per), b = min(n, a + per);
  int64_t s = 0;
  for (int64_t i = a; i < b; ++i) s += count[i];
  int64_t x = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) ws[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t w = ws[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    ws[lane] = w;
  }
  __syncthreads();
  int64_t run = (warp ? ws[warp - 1] : 0) + x - s;
  for (int64_t i = a; i < b; ++i) {
    base[i] = run;
    run += count[i];
  }
  if (tid == 1023) base[n] = ws[31];
}

// Records of the accepted nodes of one internal level: value u + J.d (model.py:91-96) and the predicted
// log-mass from the walk.  Record order per query: levels top..1, nodes in index order within a level,
// then the opened level-1 nodes' leaf blocks.
__device__ __forceinline__ int64_t record_of_internal(const TreeLevels& lv, const int64_t* base, int64_t qq,
                                                      int lev, int node) {
  int64_t r = base[qq];
  for (int l = lv.top; l > lev; --l) r += popc_all(lv.acc[l] + qq * lv.words[l], lv.words[l]);
  return r + popc_below(lv.acc[lev] + qq * lv.words[lev], node);
}

__device__ __forceinline__ int64_t record_of_block(const TreeLevels& lv, const int64_t* base, int64_t qq, int p) {
  if (lv.top == 0) return base[qq];
  int64_t r = base[qq];
  for (int l = lv.top; l >= 1; --l) r += popc_all(lv.acc[l] + qq * lv.words[l], lv.words[l]);
  return r + popc_below(lv.open[1] + qq * lv.words[1], p);
}

struct AcceptSmem {
  float ds[kChunkQ][kStr];
  float cs[kD];
  int64_t rec[kChunkQ];
  float lmv[kChunkQ];
  int list[kWindow];
  int wsum[8];
};

template <typename T>
__global__ void __launch_bounds__(256) tree_accept_kernel(const T* __restrict__ q, float scale,
                                                          const float* __restrict__ centres,
                                                          const int32_t* __restrict__ perm,
                                                          const int64_t* __restrict__ coff, int64_t slice,
                                                          TreeLevels lv, int lev, const int64_t* __restrict__ base,
                                                          int64_t nrec, float* __restrict__ rec_val,
                                                          float* __restrict__ rec_lm, int32_t* __restrict__ rec_ex,
                                                          int* __restrict__ status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  AcceptSmem& sh = *reinterpret_cast<AcceptSmem*>(smem_raw);
  const int n = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, qb = tid >> 4, cb = tid & 15;
  const int64_t lo = coff[c] + static_cast<int64_t>(blockIdx.z) * slice;
  const int64_t hi = min(coff[c + 1], lo + slice);
  if (lo >= hi) return;
  const int n_lev = lv.n[lev];
  const int64_t node = static_cast<int64_t>(c) * n_lev + n;
  for (int x = tid; x < kD; x += 256) sh.cs[x] = centres[static_cast<int64_t>(c) * kD + x];
  __syncthreads();
  for (int64_t win = lo; win < hi; win += kWindow) {
    const int cnt = gather_window(perm, win, min(hi, win + kWindow), lv.acc[lev], lv.words[lev], n, sh.list,
                                  sh.wsum);
    for (int b0 = 0; b0 < cnt; b0 += kChunkQ) {
      const int nq = min(kChunkQ, cnt - b0);
      const int* lst = sh.list + b0;
      stage_delta<T>(q, scale, sh.cs, lst, nq, sh.ds);
      if (tid < nq) {
        const int64_t qq = lst[tid];
        int64_t r = record_of_internal(lv, base, qq, lev, n);
        if (r < 0 || r >= nrec) {           // inconsistent walk state: write nothing, report
          flag_status(status, ST_BAD_INDEX);
          r = -1;
        }
        sh.rec[tid] = r;
        sh.lmv[tid] = lv.lm[lev][qq * n_lev + n];
      }
      __syncthreads();
      float acc[4][8];
      delta_gemm(sh.ds, lv.JT[lev] + node * kD * kD, qb, cb, acc);
      const float* un = lv.u[lev] + node * kD + cb * 8;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int jq = qb * 4 + i;
        if (jq >= nq || sh.rec[jq] < 0) continue;
        float* dst = rec_val + sh.rec[jq] * kD + cb * 8;
        *reinterpret_cast<float4*>(dst) = make_float4(__ldg(un) + acc[i][0], __ldg(un + 1) + acc[i][1],
                                                      __ldg(un + 2) + acc[i][2], __ldg(un + 3) + acc[i][3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(__ldg(un + 4) + acc[i][4], __ldg(un + 5) + acc[i][5],
                                                          __ldg(un + 6) + acc[i][6], __ldg(un + 7) + acc[i][7]);
      }
      if (tid < nq && sh.rec[tid] >= 0) {
        rec_lm[sh.rec[tid]] = sh.lmv[tid];
        rec_ex[sh.rec[tid]] = 0;
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// Leaf blocks: the leaves of opened level-1 node p for the queries that opened it (or, for a forest whose
// roots are its leaves, all leaves for every query of the centre, norm first).  Per (query, leaf), from
// S_s = q.k_s and x_s = S_s - a_s (= k_s . d):
//   predicted (model.py:91-96): lm = L + xbar + quad / 2, xbar = sum w x, quad = sum w (x - xbar)^2,
//                               value = sum w (1 + x - xbar) v,  w = e^(a - L)
//   opened (model.py:122-126):  log-mass logsumexp S, value softmax(S) . v
// merged online into one record (log-mass, value, opened-leaf count) per (query, block).
struct BlockSmem {
  float qs[kChunkQ][kStr];     // scaled queries
  float ks[64][kStr];          // the leaf's keys
  float vs[64][kD];            // the leaf's values
  float ss[kChunkQ][65];       // S, then the PV coefficients
  float as[64], ws[64];
  float cs[kD];
  float m[kChunkQ], s[kChunkQ], alpha[kChunkQ], nrm[kChunkQ];
  int nex[kChunkQ];
  int64_t rec[kChunkQ];
  int list[kWindow];
  int wsum[8];
};

template <typename T>
__device__ __forceinline__ void stage_leaf(const T* __restrict__ k, const T* __restrict__ v, int64_t s0, int cnt,
                                           const float* __restrict__ ac, float ll, BlockSmem& sh, bool values) {
  for (int x = threadIdx.x; x < 64 * 32; x += 256) {
    const int r = x >> 5, c4 = x & 31;
    float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), vv = kk;
    if (r < cnt) {
      kk = ld_row4<T>(k, s0 + r, c4);
      if (values) vv = ld_row4<T>(v, s0 + r, c4);
    }
    sh.ks[r][4 * c4] = kk.x;
    sh.ks[r][4 * c4 + 1] = kk.y;
    sh.ks[r][4 * c4 + 2] = kk.z;
    sh.ks[r][4 * c4 + 3] = kk.w;
    if (values) *reinterpret_cast<float4*>(&sh.vs[r][4 * c4]) = vv;
  }
  if (threadIdx.x < 64) {
    const int r = threadIdx.x;
    const float a = r < cnt ? ac[s0 + r] : 0.f;
    sh.as[r] = a;
    sh.ws[r] = r < cnt ? expf(a - ll) : 0.f;
  }
}

// S[qb * 4 + i][sb + 16 j] = qs[qb * 4 + i] . ks[sb + 16 j]  -> sh.ss
__device__ __forceinline__ void leaf_scores(BlockSmem& sh, int qb, int sb) {
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 4
  for (int k = 0; k < kD; ++k) {
    float qv[4], kv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) qv[i] = sh.qs[qb * 4 + i][k];
#pragma unroll
    for (int j = 0; j < 4; ++j) kv[j] = sh.ks[sb + 16 * j][k];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(qv[i], kv[j], acc[i][j]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) sh.ss[qb * 4 + i][sb + 16 * j] = acc[i][j];
}

// Per-(query, leaf) second-order prediction from the scores: 4 threads per query, keys sub * 16 .. + 16.
struct LeafPred {
  float xbar, quad, lm;
};
__device__ __forceinline__ LeafPred leaf_predict(const BlockSmem& sh, int jq, int sub, int cnt, float ll) {
  float sx = 0.f;
  for (int t = 0; t < 16; ++t) {
    const int s = sub * 16 + t;
    if (s < cnt) sx = fmaf(sh.ws[s], sh.ss[jq][s] - sh.as[s], sx);
  }
  sx += __shfl_xor_sync(0xffffffffu, sx, 1);
  sx += __shfl_xor_sync(0xffffffffu, sx, 2);
  float sq = 0.f;
  for (int t = 0; t < 16; ++t) {
    const int s = sub * 16 + t;
    if (s < cnt) {
      const float e = sh.ss[jq][s] - sh.as[s] - sx;
      sq = fmaf(sh.ws[s] * e, e, sq);
    }
  }
  sq += __shfl_xor_sync(0xffffffffu, sq, 1);
  sq += __shfl_xor_sync(0xffffffffu, sq, 2);
  return {sx, sq, ll + sx + 0.5f * sq};
}

template <typename T>
__global__ void __launch_bounds__(256, 1) tree_leafblock_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                                const T* __restrict__ v, int64_t m, float scale,
                                                                const float* __restrict__ centres,
                                                                const float* __restrict__ a,
                                                                const int32_t* __restrict__ perm,
                                                                const int64_t* __restrict__ coff, int64_t slice,
                                                                TreeLevels lv, float thr,
                                                                const float* __restrict__ norm,
                                                                const int64_t* __restrict__ base, int64_t nrec,
                                                                float* __restrict__ rec_val,
                                                                float* __restrict__ rec_lm,
                                                                int32_t* __restrict__ rec_ex,
                                                                int* __restrict__ status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BlockSmem& sh = *reinterpret_cast<BlockSmem*>(smem_raw);
  const int c = blockIdx.y, tid = threadIdx.x, qb = tid >> 4, sb = tid & 15;
  const bool all = lv.top == 0;
  const int p = all ? 0 : static_cast<int>(blockIdx.x);
  const int64_t lo = coff[c] + static_cast<int64_t>(blockIdx.z) * slice;
  const int64_t hi = min(coff[c + 1], lo + slice);
  if (lo >= hi) return;
  const int nl = lv.n[0], F = lv.fanout, leaf = lv.leaf;
  const int l0 = all ? 0 : p * F, l1 = all ? nl : min(nl, l0 + F);
  const float* ac = a + static_cast<int64_t>(c) * m;
  const float* lL = lv.L[0] + static_cast<int64_t>(c) * nl;
  for (int x = tid; x < kD; x += 256) sh.cs[x] = centres[static_cast<int64_t>(c) * kD + x];
  __syncthreads();
  const int jq = tid >> 2, sub = tid & 3;             // row-math mapping
  for (int64_t win = lo; win < hi; win += kWindow) {
    const int cnt = gather_window(perm, win, min(hi, win + kWindow), all ? nullptr : lv.open[1],
                                  all ? 0 : lv.words[1], p, sh.list, sh.wsum);
    for (int b0 = 0; b0 < cnt; b0 += kChunkQ) {
      const int nq = min(kChunkQ, cnt - b0);
      const int* lst = sh.list + b0;
      for (int x = tid; x < kChunkQ * 32; x += 256) {
        const int r = x >> 5, c4 = x & 31;
        float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < nq) y = ld_row4<T>(q, lst[r], c4);
        sh.qs[r][4 * c4] = scale * y.x;
        sh.qs[r][4 * c4 + 1] = scale * y.y;
        sh.qs[r][4 * c4 + 2] = scale * y.z;
        sh.qs[r][4 * c4 + 3] = scale * y.w;
      }
      if (tid < kChunkQ) {
        sh.m[tid] = -INFINITY;
        sh.s[tid] = 0.f;
        sh.nex[tid] = 0;
        sh.alpha[tid] = 1.f;
        if (!all && tid < nq) sh.nrm[tid] = norm[lst[tid]];
      }
      if (all) {
        // the leaves are the roots: norm = log-sum-exp of their predicted log-masses (model.py:108-110)
        float nm = -INFINITY, ns = 0.f;
        for (int l = l0; l < l1; ++l) {
          __syncthreads();
          const int64_t s0 = static_cast<int64_t>(l) * leaf;
          const int kc = static_cast<int>(m - s0 < leaf ? m - s0 : leaf);
          stage_leaf<T>(k, v, s0, kc, ac, lL[l], sh, false);
          __syncthreads();
          leaf_scores(sh, qb, sb);
          __syncthreads();
          const LeafPred pr = leaf_predict(sh, jq, sub, kc, lL[l]);
          const float mn = fmaxf(nm, pr.lm);
          ns = ns * expf(nm - mn) + expf(pr.lm - mn);
          nm = mn;
        }
        if (sub == 0) sh.nrm[jq] = nm + logf(ns);
      }
      float o[4][8];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) o[i][j] = 0.f;
      for (int l = l0; l < l1; ++l) {
        __syncthreads();
        const int64_t s0 = static_cast<int64_t>(l) * leaf;
        const int kc = static_cast<int>(m - s0 < leaf ? m - s0 : leaf);
        const float ll = lL[l];
        stage_leaf<T>(k, v, s0, kc, ac, ll, sh, true);
        __syncthreads();
        leaf_scores(sh, qb, sb);
        __syncthreads();
        {
          const LeafPred pr = leaf_predict(sh, jq, sub, kc, ll);
          const bool live = jq < nq;
          const bool open = live && score_of(pr.lm, pr.quad, sh.nrm[jq]) > thr;
          float mass = pr.lm;
          if (open) {
            float mx = -INFINITY;
            for (int t = 0; t < 16; ++t) {
              const int s = sub * 16 + t;
              if (s < kc) mx = fmaxf(mx, sh.ss[jq][s]);
            }
            // `open` is the same in the 4 lanes of a query, not across the warp: shuffle within the 4
            const unsigned gm = 0xFu << (threadIdx.x & 28);
            mx = fmaxf(mx, __shfl_xor_sync(gm, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(gm, mx, 2));
            float se = 0.f;
            for (int t = 0; t < 16; ++t) {
              const int s = sub * 16 + t;
              if (s < kc) se += expf(sh.ss[jq][s] - mx);
            }
            se += __shfl_xor_sync(gm, se, 1);
            se += __shfl_xor_sync(gm, se, 2);
            mass = mx + logf(se);
          }
          const float mo = sh.m[jq];
          const float mn = fmaxf(mo, mass);
          const float al = live ? expf(mo - mn) : 1.f;
          const float fw = expf(pr.lm - mn);
          for (int t = 0; t < 16; ++t) {
            const int s = sub * 16 + t;
            float pc = 0.f;
            if (live && s < kc)
              pc = open ? expf(sh.ss[jq][s] - mn) : fw * sh.ws[s] * (1.f + (sh.ss[jq][s] - sh.as[s] - pr.xbar));
            sh.ss[jq][s] = pc;
          }
          __syncwarp();
          if (sub == 0 && live) {
            sh.s[jq] = sh.s[jq] * al + expf(mass - mn);
            sh.m[jq] = mn;
            sh.alpha[jq] = al;
            sh.nex[jq] += open;
          }
        }
        __syncthreads();
        // o[i][:] = o[i][:] * alpha + sum_s P[i][s] v_s   (thread: queries qb*4.., dims sb*8..)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float al = sh.alpha[qb * 4 + i];
#pragma unroll
          for (int j = 0; j < 8; ++j) o[i][j] *= al;
        }
        for (int s = 0; s < kc; ++s) {
          const float4 v0 = *reinterpret_cast<const float4*>(&sh.vs[s][sb * 8]);
          const float4 v1 = *reinterpret_cast<const float4*>(&sh.vs[s][sb * 8 + 4]);
          const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float pc = sh.ss[qb * 4 + i][s];
#pragma unroll
            for (int j = 0; j < 8; ++j) o[i][j] = fmaf(pc, vv[j], o[i][j]);
          }
        }
      }
      __syncthreads();
      if (tid < nq) {
        const int64_t qq = lst[tid];
        int64_t r = record_of_block(lv, base, qq, p);
        if (r < 0 || r >= nrec) {           // inconsistent walk state: write nothing, report
          flag_status(status, ST_BAD_INDEX);
          r = -1;
        } else {
          rec_lm[r] = sh.m[tid] + logf(sh.s[tid]);
          rec_ex[r] = sh.nex[tid];
        }
        sh.rec[tid] = r;
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = qb * 4 + i;
        if (j >= nq || sh.rec[j] < 0) continue;
        const float inv = 1.f / sh.s[j];
        float* dst = rec_val + sh.rec[j] * kD + sb * 8;
        *reinterpret_cast<float4*>(dst) = make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
        *reinterpret_cast<float4*>(dst + 4) =
            make_float4(o[i][4] * inv, o[i][5] * inv, o[i][6] * inv, o[i][7] * inv);
      }
      __syncthreads();                       // sh.s / sh.rec are read above before the next chunk resets them
    }
  }
}

// Per query (one warp): the records merged in record order (model.py:131-134) -> out, lse, exact count.
__global__ void __launch_bounds__(256) tree_final_kernel(int64_t nq, const int64_t* __restrict__ base,
                                                         const float* __restrict__ rec_val,
                                                         const float* __restrict__ rec_lm,
                                                         const int32_t* __restrict__ rec_ex, float* __restrict__ out,
                                                         float* __restrict__ lse, int32_t* __restrict__ exact) {
  const int lane = threadIdx.x & 31;
  const int64_t qq = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (qq >= nq) return;
  const int64_t b = base[qq], e = base[qq + 1];
  float mx = -INFINITY;
  int ex = 0;
  for (int64_t r = b + lane; r < e; r += 32) {
    mx = fmaxf(mx, rec_lm[r]);
    ex += rec_ex[r];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    ex += __shfl_xor_sync(0xffffffffu, ex, o);
  }
  float s = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t r = b; r < e; ++r) {
    const float w = expf(rec_lm[r] - mx);
    s += w;
    const float4 x = *reinterpret_cast<const float4*>(rec_val + r * kD + lane * 4);
    acc.x = fmaf(w, x.x, acc.x);
    acc.y = fmaf(w, x.y, acc.y);
    acc.z = fmaf(w, x.z, acc.z);
    acc.w = fmaf(w, x.w, acc.w);
  }
  const float inv = 1.f / s;
  *reinterpret_cast<float4*>(out + qq * kD + lane * 4) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  if (lane == 0) {
    lse[qq] = mx + logf(s);
    exact[qq] = ex;
  }
}

// ---------------------------------------------------------------------------------------------------
// Leaf blocks on the tensor cores (bfloat16 keys, values and queries; forests of two or more levels): the
// arithmetic of tree_leafblock_kernel with chunks of 128 queries and, per leaf,
//   S' = q . k_s    tcgen05.mma kind::f16, M 128 x N 64 x K 128 (bf16 products are exact; f32 sums) -> TMEM
//   row math        one thread per query row = TMEM lane: S = scale S', prediction, decision, coefficients P
//   O += P . v_s    tcgen05.mma kind::f16, M 128 x N 128 x K 64, P from TMEM as bf16 hi + lo parts
// Operands are staged by the CTA's threads into 128-byte-swizzled shared tiles (the queries are gathered
// rows); one thread issues the MMAs; every wait on an MMA completion is bounded.
constexpr int kTcQ = 128;
constexpr int kTcCols = 256;         // TMEM columns: S 0..63, P hi 64..95, P lo 96..127, O 128..255
struct __align__(1024) TcSmem {
  uint8_t qs[2 * kTcQ * 128];        // queries: two K-blocks of [128 rows][128 B]  (K-major A)
  uint8_t ks[2][2 * 64 * 128];       // keys, two leaves in flight: two K-blocks of [64 rows][128 B] (K-major B)
  uint8_t vs[2][2 * 64 * 128];       // values, two leaves: two N-chunks of [64 key rows][128 B]   (MN-major B)
  float as[2][64], ws[2][64];
  float xch[4][2][kTcQ];              // per-row partial sums of the two halves (xbar, quad, max, sum)
  int64_t rec[kTcQ];
  int list[kWindow];
  int wsum[8];
  uint64_t bar_s, bar_pv;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t kTcSmemBytes = 110 * 1024;   // > 228 KB / 3: at most two CTAs (512 TMEM columns) per SM
static_assert(sizeof(TcSmem) + 1024 <= kTcSmemBytes, "tree tensor-core shared layout");

// gather_window for 128 threads
__device__ __forceinline__ int gather_window128(const int32_t* __restrict__ perm, int64_t lo, int64_t hi,
                                                const uint32_t* __restrict__ mask, int words, int bit, int* list,
                                                int* wsum) {
  return gather_window_n<128>(perm, lo, hi, mask, words, bit, list, wsum);
}

// 4-byte asynchronous global -> shared copy; src_bytes 0 writes zeros (the source is not read)
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// 16-byte asynchronous global -> shared copy; src_bytes 0 writes zeros (the source is not read)
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }


__global__ void __launch_bounds__(256, 2) tree_leafblock_tc_kernel(
    const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v, int64_t m,
    float scale, const float* __restrict__ a, const float* __restrict__ wk, const int32_t* __restrict__ perm,
    const int64_t* __restrict__ coff,
    int64_t slice, TreeLevels lv, float thr, const float* __restrict__ norm, const int64_t* __restrict__ base,
    int64_t nrec, float* __restrict__ rec_val, float* __restrict__ rec_lm, int32_t* __restrict__ rec_ex,
    int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  TcSmem& sh = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int c = blockIdx.y, p = blockIdx.x, tid = threadIdx.x, warp = tid >> 5;
  // two threads per query row: row = TMEM lane (tid & 127), half hf = keys 32 hf .. + 31 and O columns
  // 64 hf .. + 63; the warps (w, w + 4) hold the same rows and exchange partial sums through shared memory
  const int row = tid & 127, hf = tid >> 7, pair_bar = 1 + ((tid & 127) >> 5);
  const int64_t lo = coff[c] + static_cast<int64_t>(blockIdx.z) * slice;
  const int64_t hi = min(coff[c + 1], lo + slice);
  if (lo >= hi) return;
  const int nl = lv.n[0], leaf = lv.leaf;
  const int l0 = p * lv.fanout, l1 = min(nl, l0 + lv.fanout);
  const float* ac = a + static_cast<int64_t>(c) * m;
  const float* wc = wk + static_cast<int64_t>(c) * m;
  const float* lL = lv.L[0] + static_cast<int64_t>(c) * nl;
  if (tid == 0) {
    mbar_init(&sh.bar_s, 1);
    mbar_init(&sh.bar_pv, 1);
    sh.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&sh.tmem_base, kTcCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const uint32_t lane_off = static_cast<uint32_t>(row & ~31) << 16;
  const uint32_t id_s = idesc_bf16(128, 64, false, false);
  const uint32_t id_pv = idesc_bf16(128, 128, false, true);
  const uint32_t qa = smem_u32(sh.qs);
  // leaf l's keys into K buffer b, and its values with its key logits a and weights w into V buffer b (one
  // cp.async group each; rows past the leaf's keys are zeros).  l >= l1 commits an empty group, which keeps the
  // group count of every step the same (the waits below count groups).
  auto stage_k = [&](int l, int b) {
    if (l < l1) {
      const int64_t s0 = static_cast<int64_t>(l) * leaf;
      const int kc = static_cast<int>(m - s0 < leaf ? m - s0 : leaf);
      const uint32_t kb = smem_u32(sh.ks[b]);
      for (int x = tid; x < 64 * 16; x += 256) {
        const int r = x >> 4, cc = x & 15;
        const int64_t kr = s0 + (r < kc ? r : 0);
        cp_async16(kb + (cc >> 3) * (64 * 128) + sw128_off(r, cc & 7), k + kr * kD + cc * 8, r < kc ? 16u : 0u);
      }
    }
    cp_async_commit();
  };
  auto stage_v = [&](int l, int b) {
    if (l < l1) {
      const int64_t s0 = static_cast<int64_t>(l) * leaf;
      const int kc = static_cast<int>(m - s0 < leaf ? m - s0 : leaf);
      const uint32_t vb = smem_u32(sh.vs[b]);
      for (int x = tid; x < 64 * 16; x += 256) {
        const int r = x >> 4, cc = x & 15;
        const int64_t kr = s0 + (r < kc ? r : 0);
        cp_async16(vb + (cc >> 3) * (64 * 128) + sw128_off(r, cc & 7), v + kr * kD + cc * 8, r < kc ? 16u : 0u);
      }
      if (tid < 128) {
        const int r = tid & 63;
        const float* src = (tid < 64 ? ac : wc) + s0 + (r < kc ? r : 0);
        cp_async4(smem_u32(tid < 64 ? &sh.as[b][r] : &sh.ws[b][r]), src, r < kc ? 4u : 0u);
      }
    }
    cp_async_commit();
  };
  // S(l) = q . k of leaf l into TMEM columns 64 b .. 64 b + 63 (thread 0)
  auto issue_s = [&](int b) {
    tc_fence_after();
    const uint32_t ka = smem_u32(sh.ks[b]);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_bf16(tmem + 64 * b, sw128_desc(qa + kb * (kTcQ * 128) + ks * 32, 16, 1024),
                 sw128_desc(ka + kb * (64 * 128) + ks * 32, 16, 1024), id_s, (kb | ks) != 0);
    mma_commit(&sh.bar_s);
  };
  uint32_t ph_s = 0, ph_pv = 0;
  bool ok = true;
  for (int64_t win = lo; win < hi && ok; win += kWindow) {
    const int cnt = gather_window(perm, win, min(hi, win + kWindow), lv.open[1], lv.words[1], p, sh.list, sh.wsum);
    for (int b0 = 0; b0 < cnt && ok; b0 += kTcQ) {
      const int nq = min(kTcQ, cnt - b0);
      const int* lst = sh.list + b0;
      for (int x = tid; x < kTcQ * 16; x += 256) {
        const int r = x >> 4, cc = x & 15;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (r < nq) val = __ldg(reinterpret_cast<const uint4*>(q + static_cast<int64_t>(lst[r]) * kD) + cc);
        st_shared_v4(qa + (cc >> 3) * (kTcQ * 128) + sw128_off(r, cc & 7), val);
      }
      const bool live = row < nq;
      const float nrm = live ? norm[lst[row]] : 0.f;
      float m_run = -INFINITY, s_run = 0.f;
      int nex = 0;
      // pipeline over the block's leaves i = l - l0: S(i + 1) runs on the tensor cores during the row math of
      // leaf i, K(i + 2) and V(i + 1) load during leaf i; leaf i's S and then its P use TMEM columns 64 (i & 1)..,
      // O columns 128..255.  Prologue: K(0), (empty), K(1), V(0), then S(0).
      stage_k(l0, 0);
      cp_async_commit();
      stage_k(l0 + 1, 1);
      stage_v(l0, 0);
      cp_async_wait<2>();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) issue_s(0);
      for (int l = l0; l < l1; ++l) {
        const int b = (l - l0) & 1;
        const int64_t s0 = static_cast<int64_t>(l) * leaf;
        const int kc = static_cast<int>(m - s0 < leaf ? m - s0 : leaf);
        const float ll = lL[l];
        ok = mbar_wait(&sh.bar_s, ph_s, status, &sh.abort_flag);            // S(i)
        ph_s ^= 1u;
        if (!__syncthreads_and(ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        stage_k(l + 2, b);                         // K buffer b: its last reader S(i) has completed
        float S[32];
        {
          uint32_t r0[32];
          tmem_ld32(tmem + lane_off + 64 * b + 32 * hf, r0);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) S[j] = scale * __uint_as_float(r0[j]);
        }
        if (l > l0) {                              // PV(i - 1): frees V buffer b ^ 1, TMEM columns 64 (b ^ 1).., O
          ok = mbar_wait(&sh.bar_pv, ph_pv, status, &sh.abort_flag);
          ph_pv ^= 1u;
          if (!__syncthreads_and(ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        stage_v(l + 1, b ^ 1);
        cp_async_wait<2>();                        // K(i + 1), V(i), a(i), w(i) have landed
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0 && l + 1 < l1) issue_s(b ^ 1);
        const uint32_t va = smem_u32(sh.vs[b]);
        const float* as_ = sh.as[b] + 32 * hf;            // this half's keys
        const float* ws_ = sh.ws[b] + 32 * hf;
        const int kh = min(32, max(0, kc - 32 * hf));     // this half's valid keys
        const float4* w4p = reinterpret_cast<const float4*>(ws_);
        const float4* a4p = reinterpret_cast<const float4*>(as_);
        // prediction (model.py:91-96 from the keys): xbar = sum w x, quad = sum w (x - xbar)^2, x = S - a;
        // each half sums its 32 keys, the pair adds the two halves in a fixed order.  The first exchange also
        // carries the half's maximum score, which an opened leaf's logsumexp needs.
        {
          float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f, m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 w4 = w4p[j >> 2], a4 = a4p[j >> 2];
            p0 = fmaf(w4.x, S[j] - a4.x, p0);
            p1 = fmaf(w4.y, S[j + 1] - a4.y, p1);
            p2 = fmaf(w4.z, S[j + 2] - a4.z, p2);
            p3 = fmaf(w4.w, S[j + 3] - a4.w, p3);
            if (j < kh) m0 = fmaxf(m0, S[j]);
            if (j + 1 < kh) m1 = fmaxf(m1, S[j + 1]);
            if (j + 2 < kh) m0 = fmaxf(m0, S[j + 2]);
            if (j + 3 < kh) m1 = fmaxf(m1, S[j + 3]);
          }
          sh.xch[0][hf][row] = (p0 + p1) + (p2 + p3);
          sh.xch[2][hf][row] = fmaxf(m0, m1);
        }
        named_bar_sync(pair_bar, 64);
        const float xb = sh.xch[0][0][row] + sh.xch[0][1][row];
        const float mx = fmaxf(sh.xch[2][0][row], sh.xch[2][1][row]);
        {
          float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 w4 = w4p[j >> 2], a4 = a4p[j >> 2];
            const float e0 = S[j] - a4.x - xb, e1 = S[j + 1] - a4.y - xb;
            const float e2 = S[j + 2] - a4.z - xb, e3 = S[j + 3] - a4.w - xb;
            p0 = fmaf(w4.x * e0, e0, p0);
            p1 = fmaf(w4.y * e1, e1, p1);
            p2 = fmaf(w4.z * e2, e2, p2);
            p3 = fmaf(w4.w * e3, e3, p3);
          }
          sh.xch[1][hf][row] = (p0 + p1) + (p2 + p3);
        }
        named_bar_sync(pair_bar, 64);
        const float qd = sh.xch[1][0][row] + sh.xch[1][1][row];
        const float lmv = ll + xb + 0.5f * qd;
        const bool open = live && score_of(lmv, qd, nrm) > thr;
        // an opened leaf's log-mass: logsumexp of its scores (both halves, fixed order); its exponentials
        // e^(S - mx) replace the scores in S, and its P below is e^(S - mx) e^(mx - mn)
        {
          float e0 = 0.f, e1 = 0.f, e2 = 0.f, e3 = 0.f;
          if (open) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              S[j] = __expf(S[j] - mx);
              S[j + 1] = __expf(S[j + 1] - mx);
              S[j + 2] = __expf(S[j + 2] - mx);
              S[j + 3] = __expf(S[j + 3] - mx);
              if (j < kh) e0 += S[j];
              if (j + 1 < kh) e1 += S[j + 1];
              if (j + 2 < kh) e2 += S[j + 2];
              if (j + 3 < kh) e3 += S[j + 3];
            }
          }
          sh.xch[3][hf][row] = (e0 + e1) + (e2 + e3);
        }
        named_bar_sync(pair_bar, 64);
        const float mass = open ? mx + logf(sh.xch[3][0][row] + sh.xch[3][1][row]) : lmv;
        // lazy reference: the running maximum moves only when a leaf's mass exceeds it by more than 8 (so the
        // coefficients stay below e^8 and O is rescaled rarely); out and log-Z are relative to the same reference
        const bool bump = live && mass > m_run + 8.f;
        const float mn = live ? (bump ? mass : m_run) : 0.f;
        const float al = bump ? expf(m_run - mn) : 1.f;
        if (live) {
          s_run = s_run * al + expf(mass - mn);
          m_run = mn;
        }
        nex += open;
        const float fw = expf(lmv - mn);
        const float c0 = fw * (1.f - xb);          // far coefficient: w (fw (1 + x - xbar)) = w (fw x + c0)
        const float fo = open ? __expf(mx - mn) : 0.f;   // opened: P = e^(S - mx) e^(mx - mn)
        // rescale this half of O (its previous PV has completed).  tcgen05.ld / st are warp-collective
        // (.sync.aligned): the warp takes the branch as a whole, rows whose reference did not move scale by 1
        if (__any_sync(0xffffffffu, l > l0 && al != 1.f)) {
#pragma unroll 1
          for (int cb = 0; cb < 2; ++cb) {
            uint32_t o[32];
            const uint32_t col = 128 + 64 * hf + 32 * cb;
            tmem_ld32(tmem + lane_off + col, o);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * al);
            tmem_st32(tmem + lane_off + col, o);
          }
        }
        {                                          // P as bf16 hi and lo parts for this half's 32 keys
          uint32_t ph[16], pl[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float pc[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int jj = j + t;
              pc[t] = 0.f;
              if (live && jj < kh) pc[t] = open ? S[jj] * fo : ws_[jj] * fmaf(fw, S[jj] - as_[jj], c0);
            }
            const __nv_bfloat162 hb = __floats2bfloat162_rn(pc[0], pc[1]);
            const float2 hf2 = __bfloat1622float2(hb);
            ph[j >> 1] = *reinterpret_cast<const uint32_t*>(&hb);
            pl[j >> 1] = pack_bf16x2(pc[0] - hf2.x, pc[1] - hf2.y);
          }
          tmem_st16(tmem + lane_off + 64 * b + 16 * hf, ph);
          tmem_st16(tmem + lane_off + 64 * b + 32 + 16 * hf, pl);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {                            // PV(i): O += P(i) . V(i), P from TMEM columns 64 b..
          tc_fence_after();
#pragma unroll
          for (int part = 0; part < 2; ++part)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16_ts_by(1u, tmem + 128, tmem + 64 * b + 32 * part + 8 * kk,
                             sw128_desc(va + kk * 2048, 64 * 128, 1024), id_pv, (l > l0 || part || kk) ? 1u : 0u);
          mma_commit(&sh.bar_pv);
        }
      }
      if (ok) {                                    // PV of the block's last leaf
        ok = mbar_wait(&sh.bar_pv, ph_pv, status, &sh.abort_flag);
        ph_pv ^= 1u;
        ok = __syncthreads_and(ok);
        tc_fence_after();
      }
      if (!ok) break;
      if (hf == 0) {
        int64_t r = -1;
        if (live) {
          const int64_t qq = lst[row];
          r = record_of_block(lv, base, qq, p);
          if (r < 0 || r >= nrec) {
            flag_status(status, ST_BAD_INDEX);
            r = -1;
          } else {
            rec_lm[r] = m_run + logf(s_run);
            rec_ex[r] = nex;
          }
        }
        sh.rec[row] = r;
      }
      __syncthreads();
      const int64_t r = sh.rec[row];
      const float inv = 1.f / s_run;
#pragma unroll
      for (int cb = 0; cb < 2; ++cb) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_off + 128 + 64 * hf + 32 * cb, o);
        tmem_ld_wait();
        if (live && r >= 0) {
          float4* dst = reinterpret_cast<float4*>(rec_val + r * kD + 64 * hf + 32 * cb);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            dst[j] = make_float4(__uint_as_float(o[4 * j]) * inv, __uint_as_float(o[4 * j + 1]) * inv,
                                 __uint_as_float(o[4 * j + 2]) * inv, __uint_as_float(o[4 * j + 3]) * inv);
        }
      }
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
    }
  }
  cp_async_wait<0>();                       // no copy may land after the CTA leaves (an aborted chunk)
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTcCols);
}

// ---------------------------------------------------------------------------------------------------
// Internal nodes on the tensor cores: for a chunk of 128 gathered queries, Y = D . M with D = scale q - c
// (float32, split into bf16 hi + lo parts) and M a node's H (walk) or J (accept) as bf16 hi + lo rows:
// Y = Dh Mh + Dh Ml + Dl Mh, three chains of kind::f16 MMAs (M 128 x N 128 x K 128) into TMEM.
//   walk   (ACCEPT = false): one CTA per (parent, centre, slice) over the queries that opened the parent; the
//          parent's children one after another, their operands double-buffered by cp.async and Y
//          double-buffered in TMEM so that the next child's MMAs run during this child's epilogue; per row
//          lm = L + g.d + d.Y / 2, the decision (model.py:112-127), the bits (the roots stay on
//          tree_walk_kernel, whose decisions need every root's prediction first)
//   accept (ACCEPT = true):  one CTA per (node, centre, slice) over the queries that accepted the node;
//          val = u + Y (model.py:91-96) -> the query's record
// One thread per query row (= TMEM lane); every MMA completion wait is bounded.
struct __align__(1024) NodeSmem {
  uint8_t a[2][2][kTcQ * 128];       // D: [hi, lo][K-block][128 rows x 128 B]  (K-major A)
  uint8_t b[2][2][2][kTcQ * 128];    // M: [buffer][hi, lo][K-block][128 rows x 128 B] (K-major B)
  int64_t rec[kTcQ];
  int list[kWindow];
  int wsum[4];
  uint64_t bar[2];
  uint64_t bar_b[2];                 // operand buffer b[i] landed (bulk copy)
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t kNodeSmemBytes = sizeof(NodeSmem) + 1024;

template <typename T>
__device__ __forceinline__ void load_row128(const T* q, int64_t row, float scale, const float* __restrict__ c,
                                            float (&d)[kD]) {
  if constexpr (std::is_same<T, uint16_t>::value) {     // bf16 rows: 16-byte loads of 8 values, all issued first
    const uint4* src = reinterpret_cast<const uint4*>(q + row * kD);
    uint4 raw[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) raw[i] = __ldg(src + i);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const int e = 8 * i + 2 * h;
        d[e] = fmaf(scale, __uint_as_float(w[h] << 16), -__ldg(c + e));
        d[e + 1] = fmaf(scale, __uint_as_float(w[h] & 0xFFFF0000u), -__ldg(c + e + 1));
      }
    }
  } else {
#pragma unroll
    for (int c4 = 0; c4 < 32; ++c4) {
      const float4 x = ld_row4<T>(q, row, c4);
      const float4 cc = __ldg(reinterpret_cast<const float4*>(c) + c4);
      d[4 * c4] = fmaf(scale, x.x, -cc.x);
      d[4 * c4 + 1] = fmaf(scale, x.y, -cc.y);
      d[4 * c4 + 2] = fmaf(scale, x.z, -cc.z);
      d[4 * c4 + 3] = fmaf(scale, x.w, -cc.w);
    }
  }
}

template <typename T, bool ACCEPT>
__global__ void __launch_bounds__(128, 1) tree_node_tc_kernel(
    const T* __restrict__ q, float scale, const float* __restrict__ centres, const int32_t* __restrict__ perm,
    const int64_t* __restrict__ coff, int64_t slice, TreeLevels lv, int lev, float thr,
    const float* __restrict__ norm, const int64_t* __restrict__ base, int64_t nrec, float* __restrict__ rec_val,
    float* __restrict__ rec_lm, int32_t* __restrict__ rec_ex, int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  NodeSmem& sh = *reinterpret_cast<NodeSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int c = blockIdx.y, tid = threadIdx.x, warp = tid >> 5;
  const int64_t lo = coff[c] + static_cast<int64_t>(blockIdx.z) * slice;
  const int64_t hi = min(coff[c + 1], lo + slice);
  if (lo >= hi) return;
  const int n_lev = lv.n[lev];
  // walk: the children of parent blockIdx.x (level lev + 1); accept: node blockIdx.x of level lev
  const int ch0 = ACCEPT ? static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x) * lv.fanout;
  const int ch1 = ACCEPT ? ch0 + 1 : min(n_lev, ch0 + lv.fanout);
  const int nc = ch1 - ch0;
  const uint32_t* mask = ACCEPT ? lv.acc[lev] : lv.open[lev + 1];
  const int mwords = ACCEPT ? lv.words[lev] : lv.words[lev + 1];
  const int mbit = static_cast<int>(blockIdx.x);
  const float* cen = centres + static_cast<int64_t>(c) * kD;
  const int64_t nodes0 = static_cast<int64_t>(c) * n_lev;
  const uint16_t* Mb = ACCEPT ? lv.Jb[lev] : lv.Hb[lev];
  if (tid == 0) {
    mbar_init(&sh.bar[0], 1);
    mbar_init(&sh.bar[1], 1);
    mbar_init(&sh.bar_b[0], 1);
    mbar_init(&sh.bar_b[1], 1);
    sh.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&sh.tmem_base, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t idesc = idesc_bf16(128, 128, false, false);
  const uint32_t a0 = smem_u32(sh.a);
  // node's M hi + lo images (64 KB, the forest stores them in this shared-memory layout) -> b[buf] by one
  // bulk copy (thread 0); the MMA issuer waits for bar_b[buf] before it reads them
  uint32_t loads_b[2] = {0u, 0u}, issued_b[2] = {0u, 0u};
  auto stage_b = [&](int node, int buf) {
    ++issued_b[buf];
    mbar_arrive_expect_tx(&sh.bar_b[buf], 2 * kD * kD * 2);
    bulk_load(sh.b[buf], Mb + (nodes0 + node) * 2 * kD * kD, 2 * kD * kD * 2, &sh.bar_b[buf], policy_evict_normal());
  };
  auto wait_b = [&](int buf) {                    // thread 0, before the MMAs that read b[buf]
    const bool w = mbar_wait(&sh.bar_b[buf], loads_b[buf] & 1u, status, &sh.abort_flag);
    ++loads_b[buf];
    return w;
  };
  auto issue = [&](int buf, uint32_t ycol) {      // Y[ycol] = Dh Mh + Dh Ml + Dl Mh (thread 0)
    tc_fence_after();
    const uint32_t b0 = smem_u32(sh.b[buf]);
#pragma unroll
    for (int pr = 0; pr < 3; ++pr) {
      const int ap = pr == 2 ? 1 : 0, bp = pr == 1 ? 1 : 0;
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_bf16(tmem + ycol, sw128_desc(a0 + (ap * 2 + kb) * (kTcQ * 128) + ks * 32, 16, 1024),
                   sw128_desc(b0 + (bp * 2 + kb) * (kTcQ * 128) + ks * 32, 16, 1024), idesc, (pr | kb | ks) != 0);
    }
  };
  uint32_t uses[2] = {0u, 0u};                     // completed phases per barrier
  bool ok = true;
  bool b_ready = false;                            // accept: the one node's J has landed
  if (ACCEPT && tid == 0) stage_b(ch0, 0);         // the one node's J, for every chunk
  for (int64_t win = lo; win < hi && ok; win += kWindow) {
    const int cnt = gather_window128(perm, win, min(hi, win + kWindow), mask, mwords, mbit, sh.list, sh.wsum);
    for (int b0i = 0; b0i < cnt && ok; b0i += kTcQ) {
      const int nq = min(kTcQ, cnt - b0i);
      const int* lst = sh.list + b0i;
      const bool live = tid < nq;
      const int64_t qq = live ? lst[tid] : 0;
      if (!ACCEPT && tid == 0) stage_b(ch0, 0);
      // D = scale q - c of this thread's row, kept in registers (the walk's epilogue reads it), split into
      // the A operand's bf16 hi and lo parts
      float d[kD];
      if (live) {
        load_row128<T>(q, qq, scale, cen, d);
      } else {
#pragma unroll
        for (int j = 0; j < kD; ++j) d[j] = 0.f;
      }
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) {
        uint4 h, l;
        split_bf16x8(d + 8 * cc, &h, &l);
        const uint32_t off = (cc >> 3) * (kTcQ * 128) + sw128_off(tid, cc & 7);
        st_shared_v4(a0 + off, h);
        st_shared_v4(a0 + 2 * (kTcQ * 128) + off, l);
      }
      const float nrm = (!ACCEPT && live) ? norm[qq] : 0.f;
      float lm_acc = 0.f;                          // accept: the node's predicted log-mass, read early
      if (ACCEPT && live) {
        lm_acc = lv.lm[lev][qq * n_lev + ch0];
        int64_t r = record_of_internal(lv, base, qq, lev, ch0);
        if (r < 0 || r >= nrec) {
          flag_status(status, ST_BAD_INDEX);
          r = -1;
        }
        sh.rec[tid] = r;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        bool w = true;
        if (!ACCEPT || !b_ready) w = wait_b(0);
        b_ready = true;
        if (w) issue(0, 0);                       // (a failed wait leaves bar[0] incomplete: the wait below ends)
        mma_commit(&sh.bar[0]);
        if (!ACCEPT && nc > 1) stage_b(ch0 + 1, 1);
      }
      for (int i = 0; i < nc; ++i) {
        const int yb = i & 1;
        if (!ACCEPT && i + 1 < nc) {               // next child's MMAs, into the other Y buffer
          tc_fence_before();
          __syncthreads();                         // the epilogue of child i - 1 has read that Y buffer
          if (tid == 0) {
            if (wait_b(yb ^ 1)) issue(yb ^ 1, 128u * (yb ^ 1));
            mma_commit(&sh.bar[yb ^ 1]);
          }
        }
        ok = mbar_wait(&sh.bar[yb], uses[yb] & 1u, status, &sh.abort_flag);
        ++uses[yb];
        if (!__syncthreads_and(ok)) {
          ok = false;
          break;
        }
        if (!ACCEPT && i + 2 < nc && tid == 0) stage_b(ch0 + i + 2, yb);   // this buffer's MMAs completed
        tc_fence_after();
        const int n = ch0 + i;
        const int64_t node = nodes0 + n;
        if (ACCEPT) {
          const float* un = lv.u[lev] + node * kD;
          const int64_t r = live ? sh.rec[tid] : -1;
#pragma unroll 1
          for (int cb = 0; cb < 4; ++cb) {
            uint32_t y[32];
            tmem_ld32(tmem + lane_off + 128u * yb + 32 * cb, y);
            tmem_ld_wait();
            if (r >= 0) {
              float4* dst = reinterpret_cast<float4*>(rec_val + r * kD + 32 * cb);
              const float4* u4 = reinterpret_cast<const float4*>(un + 32 * cb);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float4 uu = __ldg(u4 + j);
                dst[j] = make_float4(uu.x + __uint_as_float(y[4 * j]), uu.y + __uint_as_float(y[4 * j + 1]),
                                     uu.z + __uint_as_float(y[4 * j + 2]), uu.w + __uint_as_float(y[4 * j + 3]));
              }
            }
          }
          if (r >= 0) {
            rec_lm[r] = lm_acc;
            rec_ex[r] = 0;
          }
        } else {
          const float* gn = lv.g[lev] + node * kD;
          float qd = 0.f, rg = 0.f;
#pragma unroll
          for (int cb = 0; cb < 4; ++cb) {
            uint32_t y[32];
            tmem_ld32(tmem + lane_off + 128u * yb + 32 * cb, y);
            tmem_ld_wait();
            float q0 = 0.f, q1 = 0.f, g0 = 0.f, g1 = 0.f;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float2 gg = __ldg(reinterpret_cast<const float2*>(gn + 32 * cb + j));
              q0 = fmaf(d[32 * cb + j], __uint_as_float(y[j]), q0);
              q1 = fmaf(d[32 * cb + j + 1], __uint_as_float(y[j + 1]), q1);
              g0 = fmaf(d[32 * cb + j], gg.x, g0);
              g1 = fmaf(d[32 * cb + j + 1], gg.y, g1);
            }
            qd += q0 + q1;
            rg += g0 + g1;
          }
          if (live) {
            const float lm = lv.L[lev][node] + rg + 0.5f * qd;
            lv.lm[lev][qq * n_lev + n] = lm;
            uint32_t* dstm = score_of(lm, qd, nrm) > thr ? lv.open[lev] : lv.acc[lev];
            atomicOr(dstm + qq * lv.words[lev] + (n >> 5), 1u << (n & 31));
          }
        }
        tc_fence_before();
      }
      if (!ok) break;
      __syncthreads();
    }
  }
  if (tid == 0) {                                  // no bulk copy may land after the CTA leaves
    volatile int none = 0;
    for (int bb = 0; bb < 2; ++bb)
      while (loads_b[bb] < issued_b[bb]) {
        mbar_wait_for(&sh.bar_b[bb], loads_b[bb] & 1u, status, &none, kWaitCycles);
        ++loads_b[bb];
      }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------------------------------------------
// centres for the operator from the k-means of the accurate mode: scaled centres and int32 assignment
__global__ void tree_centres_kernel(const float* __restrict__ km_centres, const uint8_t* __restrict__ km_assign,
                                    int64_t n, float scale, float* __restrict__ centres, int32_t* __restrict__ assign) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < HTRC_TREE_KMEANS_CENTRES * kD) centres[i] = scale * km_centres[i];
  if (i < n) assign[i] = km_assign[i];
}

namespace {
size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

struct Shape {
  int levels = 0;
  int n[kMaxLevels] = {};
  int words[kMaxLevels] = {};
};

int shape_of(const HtrcTreeDims* d, Shape* s) {
  if (d == nullptr) return HTRC_ERR_ARG;
  if (d->n_keys < 1 || d->n_queries < 0 || d->n_centres < 1 || d->n_centres > HTRC_TREE_MAX_CENTRES ||
      d->leaf_size < 1 || d->leaf_size > 64 || d->fanout < 2 || d->fanout > 64 || !(d->threshold >= 0.f) ||
      !(d->scale == d->scale))
    return HTRC_ERR_ARG;
  if ((d->kv_dtype != HTRC_DTYPE_F32 && d->kv_dtype != HTRC_DTYPE_BF16) ||
      (d->q_dtype != HTRC_DTYPE_F32 && d->q_dtype != HTRC_DTYPE_BF16))
    return HTRC_ERR_ARG;
  if (d->n_keys > (int64_t(1) << 31) - 1 || d->n_queries > (int64_t(1) << 31) - 1) return HTRC_ERR_UNSUPPORTED;
  int64_t n = (d->n_keys + d->leaf_size - 1) / d->leaf_size;
  s->levels = 0;
  for (;;) {
    if (s->levels == kMaxLevels) return HTRC_ERR_UNSUPPORTED;
    s->n[s->levels] = static_cast<int>(n);
    s->words[s->levels] = static_cast<int>((n + 31) / 32);
    ++s->levels;
    if (n <= d->fanout) break;
    n = (n + d->fanout - 1) / d->fanout;
  }
  return HTRC_OK;
}

struct ForestLayout {
  size_t status = 0, a = 0, w = 0, L[kMaxLevels] = {}, g[kMaxLevels] = {}, u[kMaxLevels] = {}, H[kMaxLevels] = {},
         JT[kMaxLevels] = {}, Hb[kMaxLevels] = {}, Jb[kMaxLevels] = {}, total = 0;
};
ForestLayout forest_layout(const HtrcTreeDims* d, const Shape& s) {
  ForestLayout f;
  const size_t C = d->n_centres;
  size_t o = 0;
  f.status = o;                               // the build's device status word
  o += 256;
  f.a = o;
  o += a256(C * d->n_keys * 4);
  f.w = o;                                    // w = e^(a - L) of every key within its leaf
  o += a256(C * d->n_keys * 4);
  f.L[0] = o;
  o += a256(C * s.n[0] * 4);
  for (int l = 1; l < s.levels; ++l) {
    const size_t nn = C * s.n[l];
    f.L[l] = o;
    o += a256(nn * 4);
    f.g[l] = o;
    o += a256(nn * kD * 4);
    f.u[l] = o;
    o += a256(nn * kD * 4);
    f.H[l] = o;
    o += a256(nn * kD * kD * 4);
    f.JT[l] = o;
    o += a256(nn * kD * kD * 4);
    f.Hb[l] = o;                              // [C][n][hi, lo] bf16 images (img_elem) of H
    o += a256(nn * 2 * kD * kD * 2);
    f.Jb[l] = o;                              // [C][n][hi, lo] bf16 images of J (rows: value dims)
    o += a256(nn * 2 * kD * kD * 2);
  }
  f.total = o;
  return f;
}

struct WalkLayout {
  size_t ccount = 0, perm = 0, coff = 0, status = 0, norm = 0, lm[kMaxLevels] = {}, open[kMaxLevels] = {},
         acc[kMaxLevels] = {}, count = 0, base = 0, total = 0;
};
WalkLayout walk_layout(const HtrcTreeDims* d, const Shape& s) {
  WalkLayout w;
  const size_t N = d->n_queries;
  size_t o = 0;
  w.ccount = o;
  o += a256(size_t(d->n_centres) * 4);
  w.perm = o;
  o += a256(N * 4);
  w.coff = o;
  o += a256((size_t(d->n_centres) + 1) * 8);
  w.status = o;
  o += 256;
  w.norm = o;
  o += a256(N * 4);
  for (int l = 1; l < s.levels; ++l) {
    w.lm[l] = o;
    o += a256(N * s.n[l] * 4);
    w.open[l] = o;
    o += a256(N * s.words[l] * 4);
    w.acc[l] = o;
    o += a256(N * s.words[l] * 4);
  }
  w.count = o;
  o += a256(N * 8);
  w.base = o;
  o += a256((N + 1) * 8);
  w.total = o;
  return w;
}

struct RecordLayout {
  size_t val = 0, lm = 0, ex = 0, total = 0;
};
RecordLayout record_layout(int64_t p) {
  RecordLayout r;
  const size_t n = p > 0 ? size_t(p) : 1;
  r.val = 0;
  r.lm = a256(n * kD * 4);
  r.ex = r.lm + a256(n * 4);
  r.total = r.ex + a256(n * 4);
  return r;
}

TreeLevels levels_of(const HtrcTreeDims* d, const Shape& s, const void* forest, void* walk) {
  TreeLevels lv{};
  const ForestLayout f = forest_layout(d, s);
  const uint8_t* fb = static_cast<const uint8_t*>(forest);
  uint8_t* wb = static_cast<uint8_t*>(walk);
  const WalkLayout w = walk_layout(d, s);
  lv.top = s.levels - 1;
  lv.fanout = d->fanout;
  lv.leaf = d->leaf_size;
  for (int l = 0; l < s.levels; ++l) {
    lv.n[l] = s.n[l];
    lv.words[l] = s.words[l];
    lv.L[l] = reinterpret_cast<const float*>(fb + f.L[l]);
    if (l >= 1) {
      lv.g[l] = reinterpret_cast<const float*>(fb + f.g[l]);
      lv.u[l] = reinterpret_cast<const float*>(fb + f.u[l]);
      lv.H[l] = reinterpret_cast<const float*>(fb + f.H[l]);
      lv.JT[l] = reinterpret_cast<const float*>(fb + f.JT[l]);
      lv.Hb[l] = reinterpret_cast<const uint16_t*>(fb + f.Hb[l]);
      lv.Jb[l] = reinterpret_cast<const uint16_t*>(fb + f.Jb[l]);
      if (wb) {
        lv.lm[l] = reinterpret_cast<float*>(wb + w.lm[l]);
        lv.open[l] = reinterpret_cast<uint32_t*>(wb + w.open[l]);
        lv.acc[l] = reinterpret_cast<uint32_t*>(wb + w.acc[l]);
      }
    }
  }
  return lv;
}

bool aligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 255u) == 0; }

int device_ok() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return HTRC_ERR_DEVICE;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return HTRC_ERR_DEVICE;
  return major == 10 ? HTRC_OK : HTRC_ERR_DEVICE;
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) ==
                 cudaSuccess
             ? HTRC_OK
             : HTRC_ERR_CUDA;
}

int launched() { return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA; }

// the bfloat16 leaf blocks run on the tensor cores unless HTRC_TREE_SIMT_LEAVES=1 selects the CUDA-core
// kernel (same arithmetic in float32 throughout; used by the tests to compare the two)
bool tc_leaves_enabled() {
  const char* e = getenv("HTRC_TREE_SIMT_LEAVES");
  return !(e && e[0] == '1');
}

// the internal nodes below the roots run on the tensor cores unless HTRC_TREE_SIMT_NODES=1 selects the
// float32 CUDA-core kernels (tree_walk_kernel / tree_accept_kernel)
bool tc_nodes_enabled() {
  const char* e = getenv("HTRC_TREE_SIMT_NODES");
  return !(e && e[0] == '1');
}

// largest per-centre query count (reads the grouped offsets back: one stream synchronisation)
int max_count(const int64_t* coff_dev, int ncen, cudaStream_t st, int64_t* mx) {
  int64_t host[HTRC_TREE_MAX_CENTRES + 1];
  if (cudaMemcpyAsync(host, coff_dev, (ncen + 1) * sizeof(int64_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return HTRC_ERR_CUDA;
  *mx = 0;
  for (int c = 0; c < ncen; ++c) *mx = host[c + 1] - host[c] > *mx ? host[c + 1] - host[c] : *mx;
  return HTRC_OK;
}

constexpr int64_t kRootSlice = 256;     // queries per root-walk CTA (every root for each of them)
constexpr int64_t kSlice = 4096;        // candidate queries per CTA of the node-major kernels

unsigned slices(int64_t mx, int64_t slice) { return static_cast<unsigned>(mx > 0 ? (mx + slice - 1) / slice : 1); }

template <typename T>
int build_impl(const HtrcTreeDims* d, const Shape& s, const T* k, const T* v, const float* centres, void* forest,
               cudaStream_t st) {
  const ForestLayout f = forest_layout(d, s);
  uint8_t* fb = static_cast<uint8_t*>(forest);
  float* a = reinterpret_cast<float*>(fb + f.a);
  int* status = reinterpret_cast<int*>(fb + f.status);
  const int C = d->n_centres;
  if (cudaMemsetAsync(status, 0, 4, st) != cudaSuccess) return HTRC_ERR_CUDA;
  tree_leaf_kernel<T><<<dim3(s.n[0], C), 64, 0, st>>>(k, d->n_keys, d->leaf_size, centres, s.n[0], a,
                                                       reinterpret_cast<float*>(fb + f.L[0]),
                                                       reinterpret_cast<float*>(fb + f.w));
  int rc = launched();
  if (rc != HTRC_OK || s.levels < 2) return rc;
  if (tc_nodes_enabled()) {
    if ((rc = set_smem(tree_gram_tc_kernel<T>, kGramTcSmemBytes)) != HTRC_OK) return rc;
    tree_gram_tc_kernel<T><<<dim3(s.n[1], C), 256, kGramTcSmemBytes, st>>>(
        k, v, d->n_keys, d->leaf_size, d->fanout, s.n[0], a, reinterpret_cast<const float*>(fb + f.L[0]), s.n[1],
        reinterpret_cast<float*>(fb + f.L[1]), reinterpret_cast<float*>(fb + f.g[1]),
        reinterpret_cast<float*>(fb + f.u[1]), reinterpret_cast<float*>(fb + f.H[1]),
        reinterpret_cast<float*>(fb + f.JT[1]), reinterpret_cast<uint16_t*>(fb + f.Hb[1]),
        reinterpret_cast<uint16_t*>(fb + f.Jb[1]), status);
  } else {
  if ((rc = set_smem(tree_gram_kernel<T>, sizeof(GramSmem))) != HTRC_OK) return rc;
  tree_gram_kernel<T><<<dim3(s.n[1], C), 256, sizeof(GramSmem), st>>>(
      k, v, d->n_keys, d->leaf_size, d->fanout, s.n[0], a, reinterpret_cast<const float*>(fb + f.L[0]), s.n[1],
      reinterpret_cast<float*>(fb + f.L[1]), reinterpret_cast<float*>(fb + f.g[1]),
      reinterpret_cast<float*>(fb + f.u[1]), reinterpret_cast<float*>(fb + f.H[1]),
      reinterpret_cast<float*>(fb + f.JT[1]), reinterpret_cast<uint16_t*>(fb + f.Hb[1]),
      reinterpret_cast<uint16_t*>(fb + f.Jb[1]));
  }
  if ((rc = launched()) != HTRC_OK) return rc;
  if ((rc = set_smem(tree_merge_kernel, sizeof(MergeSmem))) != HTRC_OK) return rc;
  for (int l = 2; l < s.levels; ++l) {
    tree_merge_kernel<<<dim3(s.n[l], C), 256, sizeof(MergeSmem), st>>>(
        d->fanout, s.n[l - 1], reinterpret_cast<const float*>(fb + f.L[l - 1]),
        reinterpret_cast<const float*>(fb + f.g[l - 1]), reinterpret_cast<const float*>(fb + f.u[l - 1]),
        reinterpret_cast<const float*>(fb + f.H[l - 1]), reinterpret_cast<const float*>(fb + f.JT[l - 1]), s.n[l],
        reinterpret_cast<float*>(fb + f.L[l]), reinterpret_cast<float*>(fb + f.g[l]),
        reinterpret_cast<float*>(fb + f.u[l]), reinterpret_cast<float*>(fb + f.H[l]),
        reinterpret_cast<float*>(fb + f.JT[l]), reinterpret_cast<uint16_t*>(fb + f.Hb[l]),
        reinterpret_cast<uint16_t*>(fb + f.Jb[l]));
    if ((rc = launched()) != HTRC_OK) return rc;
  }
  return HTRC_OK;
}

template <typename T>
int walk_impl(const HtrcTreeDims* d, const Shape& s, const T* q, const int32_t* assign, const float* centres,
              const void* forest, void* walk, int32_t* visited, int32_t* accepted, int32_t* leaves,
              int64_t* n_records, cudaStream_t st) {
  const WalkLayout w = walk_layout(d, s);
  uint8_t* wb = static_cast<uint8_t*>(walk);
  const int C = d->n_centres;
  const int64_t N = d->n_queries;
  int* ccount = reinterpret_cast<int*>(wb + w.ccount);
  int32_t* perm = reinterpret_cast<int32_t*>(wb + w.perm);
  int64_t* coff = reinterpret_cast<int64_t*>(wb + w.coff);
  int* status = reinterpret_cast<int*>(wb + w.status);
  float* norm = reinterpret_cast<float*>(wb + w.norm);
  int64_t* count = reinterpret_cast<int64_t*>(wb + w.count);
  int64_t* base = reinterpret_cast<int64_t*>(wb + w.base);
  if (cudaMemsetAsync(status, 0, 4, st) != cudaSuccess) return HTRC_ERR_CUDA;
  for (int l = 1; l < s.levels; ++l) {
    if (cudaMemsetAsync(wb + w.open[l], 0, size_t(N) * s.words[l] * 4, st) != cudaSuccess ||
        cudaMemsetAsync(wb + w.acc[l], 0, size_t(N) * s.words[l] * 4, st) != cudaSuccess)
      return HTRC_ERR_CUDA;
  }
  tree_count_centres_kernel<<<C, 256, 0, st>>>(assign, N, C, ccount, status);
  tree_perm_kernel<<<C, 256, 0, st>>>(assign, N, C, ccount, perm, coff);
  int rc = launched();
  if (rc != HTRC_OK) return rc;
  int64_t mx = 0;
  if ((rc = max_count(coff, C, st, &mx)) != HTRC_OK) return rc;
  const TreeLevels lv = levels_of(d, s, forest, walk);
  const int top = s.levels - 1;
  if (top >= 1) {
    if ((rc = set_smem(tree_walk_kernel<T>, sizeof(WalkSmem))) != HTRC_OK) return rc;
    tree_walk_kernel<T><<<dim3(1, C, slices(mx, kRootSlice)), 256, sizeof(WalkSmem), st>>>(
        q, d->scale, centres, perm, coff, kRootSlice, lv, top, 1, d->threshold, norm);
    if ((rc = launched()) != HTRC_OK) return rc;
    const bool tc = tc_nodes_enabled();
    if (tc && top >= 2 && (rc = set_smem(tree_node_tc_kernel<T, false>, kNodeSmemBytes)) != HTRC_OK) return rc;
    for (int l = top - 1; l >= 1; --l) {
      if (tc)
        tree_node_tc_kernel<T, false><<<dim3(s.n[l + 1], C, slices(mx, kSlice)), 128, kNodeSmemBytes, st>>>(
            q, d->scale, centres, perm, coff, kSlice, lv, l, d->threshold, norm, nullptr, 0, nullptr, nullptr,
            nullptr, status);
      else
        tree_walk_kernel<T><<<dim3(s.n[l + 1], C, slices(mx, kSlice)), 256, sizeof(WalkSmem), st>>>(
            q, d->scale, centres, perm, coff, kSlice, lv, l, 0, d->threshold, norm);
      if ((rc = launched()) != HTRC_OK) return rc;
    }
  }
  if (N > 0) {
    tree_count_kernel<<<static_cast<unsigned>((N + 255) / 256), 256, 0, st>>>(lv, N, count, visited, accepted,
                                                                              leaves);
    tree_scan_kernel<<<1, 1024, 0, st>>>(count, N, base);
    if ((rc = launched()) != HTRC_OK) return rc;
  }
  int64_t total = 0;
  int stat = 0, fstat = 0;
  const int* fstatus = reinterpret_cast<const int*>(static_cast<const uint8_t*>(forest) + forest_layout(d, s).status);
  if ((N > 0 && cudaMemcpyAsync(&total, base + N, 8, cudaMemcpyDeviceToHost, st) != cudaSuccess) ||
      cudaMemcpyAsync(&stat, status, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(&fstat, fstatus, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return HTRC_ERR_CUDA;
  *n_records = total;
  if (fstat) return HTRC_ERR_DEVICE;            // the build's MMA wait gave up
  return stat & ST_BAD_INDEX ? HTRC_ERR_ARG : stat ? HTRC_ERR_DEVICE : HTRC_OK;
}

template <typename T>
int values_impl(const HtrcTreeDims* d, const Shape& s, const T* k, const T* v, const T* q, const float* centres,
                const void* forest, void* walk, void* records, int64_t n_records, float* out, float* lse,
                int32_t* exact, cudaStream_t st, bool tc_leaves, int stages) {
  const WalkLayout w = walk_layout(d, s);
  const ForestLayout f = forest_layout(d, s);
  const RecordLayout r = record_layout(n_records);
  uint8_t* wb = static_cast<uint8_t*>(walk);
  uint8_t* rb = static_cast<uint8_t*>(records);
  const int C = d->n_centres;
  const int64_t N = d->n_queries;
  const int32_t* perm = reinterpret_cast<const int32_t*>(wb + w.perm);
  const int64_t* coff = reinterpret_cast<const int64_t*>(wb + w.coff);
  const float* norm = reinterpret_cast<const float*>(wb + w.norm);
  const int64_t* base = reinterpret_cast<const int64_t*>(wb + w.base);
  int* status = reinterpret_cast<int*>(wb + w.status);
  float* rec_val = reinterpret_cast<float*>(rb + r.val);
  float* rec_lm = reinterpret_cast<float*>(rb + r.lm);
  int32_t* rec_ex = reinterpret_cast<int32_t*>(rb + r.ex);
  const float* a = reinterpret_cast<const float*>(static_cast<const uint8_t*>(forest) + f.a);
  int64_t mx = 0;
  int rc = max_count(coff, C, st, &mx);
  if (rc != HTRC_OK) return rc;
  const TreeLevels lv = levels_of(d, s, forest, walk);
  const int top = s.levels - 1;
  if (top >= 1 && (stages & HTRC_TREE_STAGE_ACCEPT)) {
    const bool tc = tc_nodes_enabled();
    if ((rc = set_smem(tree_accept_kernel<T>, sizeof(AcceptSmem))) != HTRC_OK) return rc;
    if (tc && (rc = set_smem(tree_node_tc_kernel<T, true>, kNodeSmemBytes)) != HTRC_OK) return rc;
    for (int l = top; l >= 1; --l) {
      if (tc)
        tree_node_tc_kernel<T, true><<<dim3(s.n[l], C, slices(mx, kSlice)), 128, kNodeSmemBytes, st>>>(
            q, d->scale, centres, perm, coff, kSlice, lv, l, d->threshold, norm, base, n_records, rec_val, rec_lm,
            rec_ex, status);
      else
        tree_accept_kernel<T><<<dim3(s.n[l], C, slices(mx, kSlice)), 256, sizeof(AcceptSmem), st>>>(
            q, d->scale, centres, perm, coff, kSlice, lv, l, base, n_records, rec_val, rec_lm, rec_ex, status);
      if ((rc = launched()) != HTRC_OK) return rc;
    }
  }
  if (!(stages & HTRC_TREE_STAGE_LEAVES)) {
  } else if (std::is_same<T, uint16_t>::value && top >= 1 && tc_leaves) {
    if ((rc = set_smem(tree_leafblock_tc_kernel, kTcSmemBytes)) != HTRC_OK) return rc;
    tree_leafblock_tc_kernel<<<dim3(s.n[1], C, slices(mx, kSlice)), 256, kTcSmemBytes, st>>>(
        reinterpret_cast<const uint16_t*>(q), reinterpret_cast<const uint16_t*>(k),
        reinterpret_cast<const uint16_t*>(v), d->n_keys, d->scale, a,
        reinterpret_cast<const float*>(static_cast<const uint8_t*>(forest) + f.w), perm, coff, kSlice, lv,
        d->threshold, norm, base, n_records, rec_val, rec_lm, rec_ex, status);
  } else {
    if ((rc = set_smem(tree_leafblock_kernel<T>, sizeof(BlockSmem))) != HTRC_OK) return rc;
    tree_leafblock_kernel<T><<<dim3(top >= 1 ? s.n[1] : 1, C, slices(mx, kSlice)), 256, sizeof(BlockSmem), st>>>(
        q, k, v, d->n_keys, d->scale, centres, a, perm, coff, kSlice, lv, d->threshold, norm, base, n_records,
        rec_val, rec_lm, rec_ex, status);
  }
  if ((rc = launched()) != HTRC_OK) return rc;
  if (stages & HTRC_TREE_STAGE_FINAL) {
    tree_final_kernel<<<static_cast<unsigned>((N + 7) / 8), 256, 0, st>>>(N, base, rec_val, rec_lm, rec_ex, out, lse,
                                                                          exact);
    if ((rc = launched()) != HTRC_OK) return rc;
  }
  int stat = 0;
  if (cudaMemcpyAsync(&stat, status, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return HTRC_ERR_CUDA;
  return stat ? HTRC_ERR_DEVICE : HTRC_OK;
}
}  // namespace

}  // namespace htrc

using namespace htrc;

extern "C" {

int htrc_tree_levels(const HtrcTreeDims* dims, int32_t* n_levels, int32_t nodes[HTRC_TREE_MAX_LEVELS]) {
  Shape s;
  const int rc = shape_of(dims, &s);
  if (rc != HTRC_OK) return rc;
  if (n_levels) *n_levels = s.levels;
  if (nodes)
    for (int l = 0; l < HTRC_TREE_MAX_LEVELS; ++l) nodes[l] = l < s.levels ? s.n[l] : 0;
  return HTRC_OK;
}

int htrc_tree_forest_size(const HtrcTreeDims* dims, size_t* bytes) {
  Shape s;
  const int rc = shape_of(dims, &s);
  if (rc != HTRC_OK) return rc;
  if (!bytes) return HTRC_ERR_ARG;
  *bytes = forest_layout(dims, s).total;
  return HTRC_OK;
}

int htrc_tree_build(const HtrcTreeDims* dims, const void* keys, const void* values, const float* centres, void* forest,
                    size_t forest_bytes, htrc_stream_t stream) {
  Shape s;
  int rc = shape_of(dims, &s);
  if (rc != HTRC_OK) return rc;
  if (!keys || !values || !centres) return HTRC_ERR_ARG;
  if (!forest || !aligned(forest) || forest_bytes < forest_layout(dims, s).total) return HTRC_ERR_WORKSPACE;
  if ((rc = device_ok()) != HTRC_OK) return rc;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dims->kv_dtype == HTRC_DTYPE_BF16)
    return build_impl<uint16_t>(dims, s, static_cast<const uint16_t*>(keys), static_cast<const uint16_t*>(values),
                                centres, forest, st);
  return build_impl<float>(dims, s, static_cast<const float*>(keys), static_cast<const float*>(values), centres,
                           forest, st);
}

int htrc_tree_forest_view(const HtrcTreeDims* dims, const void* forest, int32_t level, const float** a,
                          const float** L, const float** g, const float** u, const float** H, const float** JT) {
  Shape s;
  const int rc = shape_of(dims, &s);
  if (rc != HTRC_OK) return rc;
  if (!forest || level < 0 || level >= s.levels) return HTRC_ERR_ARG;
  const ForestLayout f = forest_layout(dims, s);
  const uint8_t* fb = static_cast<const uint8_t*>(forest);
  auto at = [&](size_t off) { return reinterpret_cast<const float*>(fb + off); };
  if (a) *a = at(f.a);
  if (L) *L = at(f.L[level]);
  if (g) *g = level ? at(f.g[level]) : nullptr;
  if (u) *u = level ? at(f.u[level]) : nullptr;
  if (H) *H = level ? at(f.H[level]) : nullptr;
  if (JT) *JT = level ? at(f.JT[level]) : nullptr;
  return HTRC_OK;
}

int htrc_tree_walk_size(const HtrcTreeDims* dims, size_t* bytes) {
  Shape s;
  const int rc = shape_of(dims, &s);
  if (rc != HTRC_OK) return rc;
  if (!bytes) return HTRC_ERR_ARG;
  *bytes = walk_layout(dims, s).total;
  return HTRC_OK;
}

int htrc_tree_walk(const HtrcTreeDims* dims, const void* queries, const int32_t* assign, const float* centres,
                   const void* forest, void* walk, size_t walk_bytes, int32_t* visited, int32_t* accepted,
                   int32_t* leaves, int64_t* n_records, htrc_stream_t stream) {
  Shape s;
  int rc = shape_of(dims, &s);
  if (rc != HTRC_OK) return rc;
  if (!n_records) return HTRC_ERR_ARG;
  *n_records = 0;
  if (dims->n_queries == 0) return HTRC_OK;
  if (!queries || !assign || !centres || !forest || !visited || !accepted) return HTRC_ERR_ARG;
  if (dims->q_dtype != dims->kv_dtype) return HTRC_ERR_UNSUPPORTED;
  if (!walk || !aligned(walk) || walk_bytes < walk_layout(dims, s).total) return HTRC_ERR_WORKSPACE;
  if ((rc = device_ok()) != HTRC_OK) return rc;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dims->q_dtype == HTRC_DTYPE_BF16)
    return walk_impl<uint16_t>(dims, s, static_cast<const uint16_t*>(queries), assign, centres, forest, walk, visited,
                               accepted, leaves, n_records, st);
  return walk_impl<float>(dims, s, static_cast<const float*>(queries), assign, centres, forest, walk, visited,
                          accepted, leaves, n_records, st);
}

int htrc_tree_records_size(int64_t n_records, size_t* bytes) {
  if (n_records < 0 || !bytes) return HTRC_ERR_ARG;
  *bytes = record_layout(n_records).total;
  return HTRC_OK;
}

int htrc_tree_values(const HtrcTreeDims* dims, const void* keys, const void* values, const void* queries,
                     const float* centres, const void* forest, void* walk, void* records, int64_t n_records,
                     size_t records_bytes, float* out, float* lse, int32_t* exact_leaves, int32_t stages,
                     htrc_stream_t stream) {
  Shape s;
  int rc = shape_of(dims, &s);
  if (rc != HTRC_OK) return rc;
  if (dims->n_queries == 0) return HTRC_OK;
  if (!keys || !values || !queries || !centres || !forest || !out || !lse || !exact_leaves || n_records < 0 ||
      stages < 1 || stages > HTRC_TREE_STAGE_ALL)
    return HTRC_ERR_ARG;
  if (dims->q_dtype != dims->kv_dtype) return HTRC_ERR_UNSUPPORTED;
  if (!walk || !aligned(walk)) return HTRC_ERR_WORKSPACE;
  if (!records || !aligned(records) || records_bytes < record_layout(n_records).total) return HTRC_ERR_WORKSPACE;
  if ((rc = device_ok()) != HTRC_OK) return rc;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dims->kv_dtype == HTRC_DTYPE_BF16)
    return values_impl<uint16_t>(dims, s, static_cast<const uint16_t*>(keys), static_cast<const uint16_t*>(values),
                                 static_cast<const uint16_t*>(queries), centres, forest, walk, records, n_records,
                                 out, lse, exact_leaves, st, tc_leaves_enabled(), stages);
  return values_impl<float>(dims, s, static_cast<const float*>(keys), static_cast<const float*>(values),
                            static_cast<const float*>(queries), centres, forest, walk, records, n_records, out, lse,
                            exact_leaves, st, false, stages);
}

int htrc_tree_centres_scratch_size(int64_t n_queries, size_t* bytes) {
  if (n_queries < 1 || !bytes) return HTRC_ERR_ARG;
  *bytes = a256(kmeans_scratch_bytes(n_queries)) + a256(size_t(n_queries) * 4);
  return HTRC_OK;
}

int htrc_tree_centres(const void* queries, int32_t q_dtype, int64_t n_queries, float scale, float* centres,
                      int32_t* assign, void* scratch, size_t scratch_bytes, htrc_stream_t stream) {
  if (!queries || !centres || !assign || n_queries < 1) return HTRC_ERR_ARG;
  if (q_dtype != HTRC_DTYPE_F32 && q_dtype != HTRC_DTYPE_BF16) return HTRC_ERR_ARG;
  if (n_queries > (int64_t(1) << 31) - 1) return HTRC_ERR_UNSUPPORTED;
  size_t need = 0;
  htrc_tree_centres_scratch_size(n_queries, &need);
  if (!scratch || !aligned(scratch) || scratch_bytes < need) return HTRC_ERR_WORKSPACE;
  int rc = device_ok();
  if (rc != HTRC_OK) return rc;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* sb = static_cast<uint8_t*>(scratch);
  int32_t* perm = reinterpret_cast<int32_t*>(sb + a256(kmeans_scratch_bytes(n_queries)));
  if ((rc = launch_kmeans_order(queries, q_dtype, n_queries, perm, scratch, st)) != HTRC_OK) return rc;
  float* kc = nullptr;
  uint8_t* ka = nullptr;
  kmeans_views(scratch, n_queries, &kc, &ka);
  const int64_t cover = n_queries > HTRC_TREE_KMEANS_CENTRES * kD ? n_queries : HTRC_TREE_KMEANS_CENTRES * kD;
  tree_centres_kernel<<<static_cast<unsigned>((cover + 255) / 256), 256, 0, st>>>(kc, ka, n_queries, scale, centres,
                                                                                  assign);
  return launched();
}

}  // extern "C"
