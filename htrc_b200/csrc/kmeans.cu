// Query order of the accurate and max modes (h3/htrc_flat.py:47-65 `kmeans_order`): Lloyd's k-means
// with 32 clusters on an even sample of at most 4096 query rows, 8 iterations, then the nearest centre
// of every row and a stable counting sort of the rows by centre.  The result perm lists the query rows
// cluster by cluster, each cluster in row order; the tiles of 64 consecutive entries then hold queries
// that are close to each other.
//
// Launch sequence (no host synchronisation, no allocation):
//   8 x { km_sample_kernel  (one CTA per 32 sample rows: nearest centre, per-CTA cluster sums)
//         km_update_kernel  (one CTA per cluster: sums in CTA order -> new centre) }
//   km_assign_kernel        (one CTA per 32 query rows: nearest centre, per-1024-row cluster counts)
//   km_offsets_kernel       (one CTA: exclusive prefix of the counts over clusters, then row chunks)
//   km_scatter_kernel       (one CTA per 1024 rows: warp ranks by __match_any_sync -> perm)
// A nearest-centre search is one warp per 8 centres over the CTA's 32 rows (lane = row); distances are
// float32 sums of squared differences in dimension order, and the first minimum wins (torch.argmin).
#include "common.cuh"
#include "kernels.cuh"

namespace htrc {

namespace {
constexpr int kClusters = 32;
constexpr int kSample = 4096;
constexpr int kIters = 8;
constexpr int kRows = 32;             // rows per nearest-centre CTA
constexpr int kXStride = 132;         // shared row stride (floats): float4 reads conflict-free per phase
constexpr int kChunk = 1024;          // rows per counting-sort chunk
constexpr int kMaxBlocks = (kSample + kRows - 1) / kRows;

template <typename T>
__device__ __forceinline__ float4 load_row4(const T* q, int64_t row, int c4);
template <>
__device__ __forceinline__ float4 load_row4<float>(const float* q, int64_t row, int c4) {
  return __ldg(reinterpret_cast<const float4*>(q + row * 128) + c4);
}
template <>
__device__ __forceinline__ float4 load_row4<uint16_t>(const uint16_t* q, int64_t row, int c4) {
  const uint2 x = __ldg(reinterpret_cast<const uint2*>(q + row * 128) + c4);
  return make_float4(__uint_as_float(x.x << 16), __uint_as_float(x.x & 0xFFFF0000u), __uint_as_float(x.y << 16),
                     __uint_as_float(x.y & 0xFFFF0000u));
}

// torch.linspace(0, hi, steps)[i] in float32 -- the first half step * i, the second half
// hi - step * (steps - 1 - i) rounded once, step = hi / (steps - 1) -- rounded half-to-even to an index
// (the reference's `torch.linspace(...).round().long()`).
__device__ __forceinline__ int64_t lin_index(int64_t hi, int64_t steps, int64_t i) {
  if (steps <= 1) return 0;
  const float h = static_cast<float>(hi);
  const float step = __fdiv_rn(h, static_cast<float>(steps - 1));
  const float x = i < steps / 2 ? __fmul_rn(step, static_cast<float>(i))
                                : __fmaf_rn(-step, static_cast<float>(steps - 1 - i), h);
  return static_cast<int64_t>(rintf(x));
}

// Stage rows[0..nrows) of q (source rows given by row_of) into xs[32][kXStride] and the 32 centres
// into cs[32][128]; then the nearest centre of each staged row into best[32].  128 threads.
__device__ __forceinline__ void nearest_centres(const float* xs, const float* cs, int nrows, int* best, float* bd,
                                                int* bi) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float d[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) d[j] = 0.f;
  const float* xr = xs + lane * kXStride;
  const float* cw = cs + warp * 8 * 128;
#pragma unroll 2
  for (int k = 0; k < 128; k += 4) {
    const float4 x = *reinterpret_cast<const float4*>(xr + k);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 c = *reinterpret_cast<const float4*>(cw + j * 128 + k);
      float e = __fsub_rn(x.x, c.x);
      d[j] = __fmaf_rn(e, e, d[j]);
      e = __fsub_rn(x.y, c.y);
      d[j] = __fmaf_rn(e, e, d[j]);
      e = __fsub_rn(x.z, c.z);
      d[j] = __fmaf_rn(e, e, d[j]);
      e = __fsub_rn(x.w, c.w);
      d[j] = __fmaf_rn(e, e, d[j]);
    }
  }
  float m = d[0];
  int a = 0;
#pragma unroll
  for (int j = 1; j < 8; ++j)
    if (d[j] < m) { m = d[j]; a = j; }
  bd[warp * 32 + lane] = m;
  bi[warp * 32 + lane] = warp * 8 + a;
  __syncthreads();
  if (threadIdx.x < 32) {
    float mm = bd[lane];
    int aa = bi[lane];
#pragma unroll
    for (int w = 1; w < 4; ++w)
      if (bd[w * 32 + lane] < mm) { mm = bd[w * 32 + lane]; aa = bi[w * 32 + lane]; }
    best[lane] = lane < nrows ? aa : -1;
  }
  __syncthreads();
}

template <typename T>
__device__ __forceinline__ void stage_rows(const T* q, const int64_t* src, int nrows, float* xs) {
  // 128 threads: thread -> (row r = tid / 32 + 4 i, column group c4 = tid % 32)
  const int c4 = threadIdx.x & 31;
  for (int r = threadIdx.x >> 5; r < kRows; r += 4) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nrows) v = load_row4<T>(q, src[r], c4);
    *reinterpret_cast<float4*>(xs + r * kXStride + 4 * c4) = v;
  }
}

struct KmShared {
  float xs[kRows * kXStride];
  float cs[kClusters * 128];
  float bd[128];
  int bi[128];
  int best[kRows];
  int64_t src[kRows];
};
}  // namespace

// One Lloyd assignment step on the sample: nearest centre of 32 sample rows, their per-cluster sums
// (row order) and counts.  Iteration 0 takes the seed centres from the sample itself and CTA 0
// publishes them (they are the kept value of a cluster that receives no row).
template <typename T>
__global__ void __launch_bounds__(128) km_sample_kernel(const T* __restrict__ q, int64_t n, int64_t s, int iter,
                                                        float* __restrict__ centres, float* __restrict__ psum,
                                                        int* __restrict__ pcnt) {
  __shared__ __align__(16) KmShared sh;
  const int tid = threadIdx.x;
  const int b = blockIdx.x;
  const int64_t r0 = static_cast<int64_t>(b) * kRows;
  const int nrows = static_cast<int>(s - r0 < kRows ? s - r0 : kRows);
  if (tid < kRows) sh.src[tid] = tid < nrows ? lin_index(n - 1, s, r0 + tid) : 0;
  if (iter == 0) {
    // seed centre j = sample row round(linspace(0, s - 1, 32))[j]
    const int c4 = tid & 31;
    for (int j = tid >> 5; j < kClusters; j += 4) {
      const int64_t row = lin_index(n - 1, s, lin_index(s - 1, kClusters, j));
      const float4 v = load_row4<T>(q, row, c4);
      *reinterpret_cast<float4*>(sh.cs + j * 128 + 4 * c4) = v;
      if (b == 0) *reinterpret_cast<float4*>(centres + j * 128 + 4 * c4) = v;
    }
  } else {
    for (int i = tid; i < kClusters * 32; i += 128)
      reinterpret_cast<float4*>(sh.cs)[i] = reinterpret_cast<const float4*>(centres)[i];
  }
  __syncthreads();
  stage_rows<T>(q, sh.src, nrows, sh.xs);
  __syncthreads();
  nearest_centres(sh.xs, sh.cs, nrows, sh.best, sh.bd, sh.bi);
  // thread = column: per-cluster sums of this CTA's rows in row order
  float acc[kClusters];
#pragma unroll
  for (int j = 0; j < kClusters; ++j) acc[j] = 0.f;
  for (int r = 0; r < nrows; ++r) {
    const int a = sh.best[r];
    const float x = sh.xs[r * kXStride + tid];
#pragma unroll
    for (int j = 0; j < kClusters; ++j)
      if (j == a) acc[j] = __fadd_rn(acc[j], x);
  }
  float* ps = psum + static_cast<int64_t>(b) * kClusters * 128;
#pragma unroll
  for (int j = 0; j < kClusters; ++j) ps[j * 128 + tid] = acc[j];
  if (tid < kClusters) {
    int c = 0;
    for (int r = 0; r < nrows; ++r) c += sh.best[r] == tid;
    pcnt[b * kClusters + tid] = c;
  }
}

// New centres: one CTA per cluster, thread = column; the CTA partial sums are added in CTA order in
// float64 and divided once (a cluster that received no row keeps its centre).
__global__ void __launch_bounds__(128) km_update_kernel(const float* __restrict__ psum, const int* __restrict__ pcnt,
                                                        int nblk, float* __restrict__ centres) {
  const int j = blockIdx.x, tid = threadIdx.x;
  double sum = 0.0;
  int cnt = 0;
  for (int b = 0; b < nblk; ++b) {
    sum += static_cast<double>(psum[(static_cast<int64_t>(b) * kClusters + j) * 128 + tid]);
    cnt += pcnt[b * kClusters + j];
  }
  if (cnt > 0) centres[j * 128 + tid] = static_cast<float>(sum / static_cast<double>(cnt));
}

// Nearest centre of every query row; counts per (1024-row chunk, cluster) by integer atomics
// (order-independent).
template <typename T>
__global__ void __launch_bounds__(128) km_assign_kernel(const T* __restrict__ q, int64_t n,
                                                        const float* __restrict__ centres,
                                                        uint8_t* __restrict__ assign, int* __restrict__ counts) {
  __shared__ __align__(16) KmShared sh;
  const int tid = threadIdx.x;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int nrows = static_cast<int>(n - r0 < kRows ? n - r0 : kRows);
  if (tid < kRows) sh.src[tid] = r0 + (tid < nrows ? tid : 0);
  for (int i = tid; i < kClusters * 32; i += 128)
    reinterpret_cast<float4*>(sh.cs)[i] = reinterpret_cast<const float4*>(centres)[i];
  __syncthreads();
  stage_rows<T>(q, sh.src, nrows, sh.xs);
  __syncthreads();
  nearest_centres(sh.xs, sh.cs, nrows, sh.best, sh.bd, sh.bi);
  if (tid < nrows) {
    const int a = sh.best[tid];
    assign[r0 + tid] = static_cast<uint8_t>(a);
    atomicAdd(&counts[((r0 + tid) / kChunk) * kClusters + a], 1);
  }
}

// offsets[c][j] = (rows of clusters < j) + (rows of cluster j in chunks < c).  One CTA of 1024
// threads: warp j owns cluster j, lane l a contiguous range of chunks.
__global__ void __launch_bounds__(1024) km_offsets_kernel(const int* __restrict__ counts, int nchunk,
                                                          int* __restrict__ offsets) {
  __shared__ int tot[kClusters];
  const int j = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = (nchunk + 31) / 32;
  const int c0 = min(nchunk, lane * per), c1 = min(nchunk, c0 + per);
  int s = 0;
  for (int c = c0; c < c1; ++c) s += counts[c * kClusters + j];
  int x = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) tot[j] = x;
  __syncthreads();
  int base = 0;
  for (int i = 0; i < j; ++i) base += tot[i];
  int run = base + x - s;
  for (int c = c0; c < c1; ++c) {
    offsets[c * kClusters + j] = run;
    run += counts[c * kClusters + j];
  }
}

// perm[offsets[chunk][a] + (earlier rows of the chunk in cluster a)] = row.  One CTA of 1024 threads per
// chunk, warp w = rows 32 w .. 32 w + 31 of the chunk.
__global__ void __launch_bounds__(1024) km_scatter_kernel(const uint8_t* __restrict__ assign, int64_t n,
                                                          const int* __restrict__ offsets, int32_t* __restrict__ perm) {
  __shared__ int wcnt[32][kClusters];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kChunk + threadIdx.x;
  wcnt[w][lane] = 0;
  __syncthreads();
  const bool live = row < n;
  const int a = live ? assign[row] : kClusters;      // kClusters: no row
  const uint32_t same = __match_any_sync(0xffffffffu, a);
  const int rank = __popc(same & ((1u << lane) - 1u));
  if (live && rank == 0) wcnt[w][a] = __popc(same);
  __syncthreads();
  if (live) {
    int before = 0;
    for (int i = 0; i < w; ++i) before += wcnt[i][a];
    perm[offsets[blockIdx.x * kClusters + a] + before + rank] = static_cast<int32_t>(row);
  }
}

size_t kmeans_scratch_bytes(int64_t n) {
  const int64_t nchunk = (n + kChunk - 1) / kChunk;
  auto a256 = [](size_t x) { return (x + 255) & ~size_t(255); };
  return a256(kClusters * 128 * 4) + a256(size_t(kMaxBlocks) * kClusters * 128 * 4) +
         a256(size_t(kMaxBlocks) * kClusters * 4) + a256(size_t(n)) + 2 * a256(size_t(nchunk) * kClusters * 4);
}

// the scratch's centre rows [32][128] (unscaled query space) and per-row nearest centre [n] (uint8)
void kmeans_views(void* scratch, int64_t n, float** centres, uint8_t** assign) {
  auto a256 = [](size_t x) { return (x + 255) & ~size_t(255); };
  uint8_t* p = static_cast<uint8_t*>(scratch);
  *centres = reinterpret_cast<float*>(p);
  *assign = p + a256(kClusters * 128 * 4) + a256(size_t(kMaxBlocks) * kClusters * 128 * 4) +
            a256(size_t(kMaxBlocks) * kClusters * 4);
  (void)n;
}

int launch_kmeans_order(const void* q, int dtype, int64_t n, int32_t* perm, void* scratch, cudaStream_t st) {
  const int64_t nchunk = (n + kChunk - 1) / kChunk;
  auto a256 = [](size_t x) { return (x + 255) & ~size_t(255); };
  uint8_t* p = static_cast<uint8_t*>(scratch);
  float* centres = reinterpret_cast<float*>(p);
  p += a256(kClusters * 128 * 4);
  float* psum = reinterpret_cast<float*>(p);
  p += a256(size_t(kMaxBlocks) * kClusters * 128 * 4);
  int* pcnt = reinterpret_cast<int*>(p);
  p += a256(size_t(kMaxBlocks) * kClusters * 4);
  uint8_t* assign = p;
  p += a256(size_t(n));
  int* counts = reinterpret_cast<int*>(p);
  p += a256(size_t(nchunk) * kClusters * 4);
  int* offsets = reinterpret_cast<int*>(p);
  const int64_t s = n < kSample ? n : kSample;
  const int nblk = static_cast<int>((s + kRows - 1) / kRows);
  const bool bf = dtype == HTRC_DTYPE_BF16;
  for (int it = 0; it < kIters; ++it) {
    if (bf)
      km_sample_kernel<uint16_t><<<nblk, 128, 0, st>>>(static_cast<const uint16_t*>(q), n, s, it, centres, psum, pcnt);
    else
      km_sample_kernel<float><<<nblk, 128, 0, st>>>(static_cast<const float*>(q), n, s, it, centres, psum, pcnt);
    km_update_kernel<<<kClusters, 128, 0, st>>>(psum, pcnt, nblk, centres);
  }
  if (cudaMemsetAsync(counts, 0, size_t(nchunk) * kClusters * 4, st) != cudaSuccess) return HTRC_ERR_CUDA;
  const unsigned ga = static_cast<unsigned>((n + kRows - 1) / kRows);
  if (bf)
    km_assign_kernel<uint16_t><<<ga, 128, 0, st>>>(static_cast<const uint16_t*>(q), n, centres, assign, counts);
  else
    km_assign_kernel<float><<<ga, 128, 0, st>>>(static_cast<const float*>(q), n, centres, assign, counts);
  km_offsets_kernel<<<1, 1024, 0, st>>>(counts, static_cast<int>(nchunk), offsets);
  km_scatter_kernel<<<static_cast<unsigned>(nchunk), 1024, 0, st>>>(assign, n, offsets, perm);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

}  // namespace htrc
