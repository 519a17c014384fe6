// Per-tile top-E near-leaf routing (h3/htrc_flat.py:232-233, :250-265): the first `sink` leaves are
// forced (selection +inf), then the kx largest selections.  With groups of G tiles (:223-231) a group's
// selection is the maximum over its tiles' rows (the reference's row-max runs over all G * 64 rows of
// the group; the repeats of the last tile that pad the last group add nothing to a maximum) and one
// routing serves the whole group.  One CTA of 256 threads per group: an
// MSB-first 8-bit radix select of the kx-th largest order-preserving key, ties at the threshold
// broken towards the lower leaf index, then an order-preserving compaction, so idx comes out in
// ascending leaf order.  No host synchronisation (fixed-size output).
#include "common.cuh"
#include "kernels.cuh"

namespace htrc {

namespace {
constexpr int kThreads = 256;       // also the number of radix bins (one per thread)
constexpr int kMaxLeaves = 8192;

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// exclusive block-wide prefix sum of one int per thread; returns the total in *total
__device__ __forceinline__ int block_exclusive_scan(int v, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kThreads / 32 ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kThreads / 32) scratch[lane] = w;
  }
  __syncthreads();
  const int base = warp ? scratch[warp - 1] : 0;
  *total = scratch[kThreads / 32 - 1];
  __syncthreads();
  return base + x - v;
}
}  // namespace

__global__ void __launch_bounds__(kThreads)
    route_kernel(const float* __restrict__ sel, int64_t pitch, int64_t tc, int group, int nb, int kx, int sink,
                 int32_t* __restrict__ idx, uint8_t* __restrict__ excl) {
  __shared__ uint32_t keys[kMaxLeaves];
  __shared__ int hist[256];
  __shared__ int scratch[32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;
  const int t = blockIdx.x;
  const int tid = threadIdx.x;
  uint8_t* ex = excl + static_cast<int64_t>(t) * pitch;
  int32_t* ix = idx + static_cast<int64_t>(t) * kx;

  if (kx <= 0 || kx >= nb) {
    // nothing routed / everything routed: no selection needed
    for (int l = tid; l < static_cast<int>(pitch); l += kThreads) ex[l] = (kx > 0 && l < nb) ? 1 : 0;
    if (kx > 0)
      for (int l = tid; l < kx; l += kThreads) ix[l] = l;
    return;
  }
  const int64_t ta = static_cast<int64_t>(t) * group;
  const int64_t tb = ta + group < tc ? ta + group : tc;
  for (int l = tid; l < nb; l += kThreads) {
    float s = sel[ta * pitch + l];
    for (int64_t x = ta + 1; x < tb; ++x) s = fmaxf(s, sel[x * pitch + l]);
    keys[l] = l < sink ? 0xFFFFFFFFu : order_key(s);
  }
  if (tid == 0) {
    s_prefix = 0;
    s_remaining = kx;
  }
  __syncthreads();
  uint32_t mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    hist[tid] = 0;                                   // kThreads == 256 bins
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int l = tid; l < nb; l += kThreads) {
      const uint32_t k = keys[l];
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFF], 1);
    }
    __syncthreads();
    // thread t holds digit 255 - t: an inclusive scan gives the count of candidates with a digit >= it;
    // the digit of the kx-th largest is the one where that count first reaches the remaining rank
    const int rem = s_remaining;
    const int c = hist[255 - tid];
    int tot;
    const int above = block_exclusive_scan(c, scratch, &tot);      // candidates with a larger digit
    if (above < rem && above + c >= rem) {
      s_remaining = rem - above;
      s_prefix = prefix | (static_cast<uint32_t>(255 - tid) << shift);
    }
    mask |= 0xFFu << shift;
    __syncthreads();
  }
  const uint32_t thr = s_prefix;
  const int need_eq = s_remaining;   // keys equal to thr that are taken (lowest leaf indices first)
  // each thread owns a contiguous chunk of leaves so that the compaction keeps leaf order
  const int chunk = (nb + kThreads - 1) / kThreads;
  const int lo = min(nb, tid * chunk), hi = min(nb, lo + chunk);
  int n_eq = 0;
  for (int l = lo; l < hi; ++l) n_eq += keys[l] == thr;
  int tot;
  int eq_before = block_exclusive_scan(n_eq, scratch, &tot);
  int n_take = 0;
  {
    int e = eq_before;
    for (int l = lo; l < hi; ++l) {
      const uint32_t k = keys[l];
      const bool take = k > thr || (k == thr && e++ < need_eq);
      n_take += take;
    }
  }
  int pos = block_exclusive_scan(n_take, scratch, &tot);
  {
    int e = eq_before;
    for (int l = lo; l < hi; ++l) {
      const uint32_t k = keys[l];
      const bool take = k > thr || (k == thr && e++ < need_eq);
      ex[l] = take ? 1 : 0;
      if (take && pos < kx) ix[pos++] = l;
    }
  }
  for (int l = nb + tid; l < static_cast<int>(pitch); l += kThreads) ex[l] = 0;
}

int launch_route(const float* sel, int64_t pitch, int64_t tc, int group, int nb, int kx, int sink, int32_t* idx,
                 uint8_t* excl, cudaStream_t st) {
  if (nb > kMaxLeaves) return HTRC_ERR_UNSUPPORTED;
  if (tc <= 0) return HTRC_OK;
  const int g = group > 1 ? group : 1;
  const unsigned ng = static_cast<unsigned>((tc + g - 1) / g);
  route_kernel<<<ng, kThreads, 0, st>>>(sel, pitch, tc, g, nb, kx, sink, idx, excl);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

}  // namespace htrc
