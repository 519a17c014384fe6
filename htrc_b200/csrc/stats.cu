// Leaf statistics of the flat HTRC far field on tcgen05 tensor cores.
//
// One CTA owns 128 tile centres (the MMA M dimension) and a contiguous range of leaves.  Per leaf:
//   S  = mu . K_leaf^T            (M=128 centres, N=64 tokens, K=128; mu = mu_hi + mu_lo, two bf16 MMAs)
//   softmax over the 64 tokens of each centre row (one thread per row, in registers): lz, w
//   G  = W . K_leaf               (M=128, N=128, K=64; W = w_hi + w_lo, two bf16 MMAs, K_leaf MN-major)
//   VB = W_hi . V_leaf            (M=128, N=128, K=64)
//   epilogue: g = scale * G -> (g8, sg) half-away INT8 with the row abs-max scale; vbar -> bf16;
//   g8/vbar rows staged in shared memory and written by TMA stores, lz/sg by plain stores.
// This is the arithmetic of h3/htrc_flat_triton.py:41-85 (_stats_kernel, I8=1); the hi/lo splits keep
// the products at ~2^-16 relative precision (the reference uses tf32 dots).
//
// Warp roles (320 threads): warp 0 TMA producer, warp 1 MMA issuer (+ TMEM owner), warps 2-5 softmax
// (S -> lz, W), warps 6-9 epilogue (G, VB -> g8/sg, vbar), which drains G/VB into registers first so
// the next leaf's MMAs overlap its quantisation and stores.  A thread's row is 32 * (warp % 4) + lane,
// the TMEM lane it may access.
#include "common.cuh"
#include "kernels.cuh"

namespace htrc {

namespace {
constexpr int kStages = 2;
constexpr uint32_t kMuBytes = 128 * 128 * 2;        // one of mu_hi / mu_lo: 128 rows x 256 B
constexpr uint32_t kLeafBytes = 64 * 128 * 2;       // K (or V) of one 64-token leaf
constexpr uint32_t kStageBytes = 2 * kLeafBytes;    // K + V
constexpr uint32_t kWBytes = 128 * 128;             // W_hi or W_lo: 128 rows x 64 bf16
constexpr uint32_t kOffMuHi = 0;
constexpr uint32_t kOffMuLo = kOffMuHi + kMuBytes;
constexpr uint32_t kOffStage = kOffMuLo + kMuBytes;
constexpr uint32_t kOffWHi = kOffStage + kStages * kStageBytes;
constexpr uint32_t kOffWLo = kOffWHi + kWBytes;
constexpr uint32_t kOffStG = kOffWLo + kWBytes;     // g8 staging: 128 rows x 128 B
constexpr uint32_t kOffStV = kOffStG + 128 * 128;   // vbar staging: 2 x (128 rows x 128 B)
constexpr uint32_t kOffBar = kOffStV + 2 * 128 * 128;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + barriers, + alignment slack

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;      // two 64-column S buffers
constexpr uint32_t kColG = 128;    // 128 columns
constexpr uint32_t kColV = 256;    // 128 columns

struct Bars {
  uint64_t mu_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t s_empty[2];
  uint64_t w_full;
  uint64_t w_empty;
  uint64_t gv_full;
  uint64_t gv_empty;
  uint64_t stg_free;   // thread 0 of the epilogue: the previous TMA store has read the staging buffers
  uint64_t stg_full;   // the 128 epilogue threads: this leaf's rows are staged
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
}  // namespace

__global__ void __launch_bounds__(320, 1)
    leaf_stats_kernel(const __grid_constant__ CUtensorMap tm_mu_hi, const __grid_constant__ CUtensorMap tm_mu_lo,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_g8, const __grid_constant__ CUtensorMap tm_vb,
                      float* __restrict__ sg_out, float* __restrict__ lz_out, int64_t pitch, int64_t t0, int64_t tc,
                      int nb, int leaves_per_cta, float scale, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int blk = blockIdx.x;                       // block of 128 centres (local to the chunk)
  const int l_begin = blockIdx.y * leaves_per_cta;
  const int l_end = min(nb, l_begin + leaves_per_cta);
  const int nl = max(0, l_end - l_begin);
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->mu_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->s_empty[b], 128);
    }
    mbar_init(&bars->w_full, 128);
    mbar_init(&bars->w_empty, 1);
    mbar_init(&bars->gv_full, 1);
    mbar_init(&bars->gv_empty, 128);
    mbar_init(&bars->stg_free, 1);
    mbar_init(&bars->stg_full, 128);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0 && nl > 0) {
      tma_prefetch_desc(&tm_mu_hi);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const uint64_t pol_keep = policy_evict_last();
      const int trow = static_cast<int>(t0) + blk * 128;
      mbar_arrive_expect_tx(&bars->mu_full, 2 * kMuBytes);
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(smem + kOffMuHi + c * (kMuBytes / 2), &tm_mu_hi, &bars->mu_full, 64 * c, trow, pol_keep);
        tma_load_2d(smem + kOffMuLo + c * (kMuBytes / 2), &tm_mu_lo, &bars->mu_full, 64 * c, trow, pol_keep);
      }
      for (int j = 0; j < nl; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&bars->kv_empty[s], ((j / kStages) - 1) & 1, status, abort_flag)) break;
        uint8_t* st = smem + kOffStage + s * kStageBytes;
        const int row = (l_begin + j) * 64;
        mbar_arrive_expect_tx(&bars->kv_full[s], kStageBytes);
        tma_load_2d(st, &tm_k, &bars->kv_full[s], 0, row, pol_keep);
        tma_load_2d(st + kLeafBytes / 2, &tm_k, &bars->kv_full[s], 64, row, pol_keep);
        tma_load_2d(st + kLeafBytes, &tm_v, &bars->kv_full[s], 0, row, pol_keep);
        tma_load_2d(st + kLeafBytes + kLeafBytes / 2, &tm_v, &bars->kv_full[s], 64, row, pol_keep);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nl > 0) {
      const uint32_t id_s = idesc_bf16(128, 64, false, false);
      const uint32_t id_gv = idesc_bf16(128, 128, false, true);
      const uint32_t mu_hi = smem_u32(smem + kOffMuHi), mu_lo = smem_u32(smem + kOffMuLo);
      const uint32_t w_hi = smem_u32(smem + kOffWHi), w_lo = smem_u32(smem + kOffWLo);
      bool ok = mbar_wait(&bars->mu_full, 0, status, abort_flag);
      for (int j = 0; ok && j <= nl; ++j) {
        if (j < nl) {
          const int s = j % kStages, b = j & 1;
          if (!mbar_wait(&bars->kv_full[s], (j / kStages) & 1, status, abort_flag)) break;
          if (j >= 2 && !mbar_wait(&bars->s_empty[b], ((j >> 1) - 1) & 1, status, abort_flag)) break;
          tc_fence_after();
          const uint32_t kst = smem_u32(smem + kOffStage + s * kStageBytes);
          const uint32_t d = tmem + kColS + 64 * b;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint64_t a = sw128_desc((h ? mu_lo : mu_hi) + c * (kMuBytes / 2) + kk * 32, 16, 1024);
                const uint64_t bdesc = sw128_desc(kst + c * (kLeafBytes / 2) + kk * 32, 16, 1024);
                mma_bf16(d, a, bdesc, id_s, (h | c | kk) != 0);
              }
            }
          }
          mma_commit(&bars->s_full[b]);
        }
        if (j >= 1) {
          const int jj = j - 1, s = jj % kStages;
          if (!mbar_wait(&bars->w_full, jj & 1, status, abort_flag)) break;
          if (jj >= 1 && !mbar_wait(&bars->gv_empty, (jj - 1) & 1, status, abort_flag)) break;
          tc_fence_after();
          const uint32_t kst = smem_u32(smem + kOffStage + s * kStageBytes);
          const uint32_t vst = kst + kLeafBytes;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t a = sw128_desc((h ? w_lo : w_hi) + kk * 32, 16, 1024);
              const uint64_t bdesc = sw128_desc(kst + kk * 2048, kLeafBytes / 2, 1024);
              mma_bf16(tmem + kColG, a, bdesc, id_gv, (h | kk) != 0);
            }
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t a = sw128_desc(w_hi + kk * 32, 16, 1024);
            const uint64_t bdesc = sw128_desc(vst + kk * 2048, kLeafBytes / 2, 1024);
            mma_bf16(tmem + kColV, a, bdesc, id_gv, kk != 0);
          }
          mma_commit(&bars->gv_full);
          mma_commit(&bars->w_empty);
          mma_commit(&bars->kv_empty[s]);
        }
      }
    }
  } else if (warp < 6) {
    // softmax warpgroup: S -> (lz, W)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t tloc = static_cast<int64_t>(blk) * 128 + row;   // tile index within the chunk
    const bool valid = tloc < tc;
    const float kLog2e = 1.4426950408889634f;
    const uint32_t wh = smem_u32(smem + kOffWHi), wl = smem_u32(smem + kOffWLo);
    for (int j = 0; j < nl; ++j) {
      const int b = j & 1;
      const int leaf = l_begin + j;
      if (!mbar_wait(&bars->s_full[b], (j >> 1) & 1, status, abort_flag)) break;
      __syncwarp();
      tc_fence_after();
      float a[64];
      {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + kColS + 64 * b, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) a[i] = __uint_as_float(r[i]);
        tmem_ld32(tmem + lane_base + kColS + 64 * b + 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) a[32 + i] = __uint_as_float(r[i]);
      }
      tc_fence_before();
      mbar_arrive(&bars->s_empty[b]);
      float m = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        a[i] = __fmul_rn(a[i], scale);
        m = fmaxf(m, a[i]);
      }
      float z = 0.f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        a[i] = ex2(__fmul_rn(a[i] - m, kLog2e));
        z += a[i];
      }
      const float lz = m + logf(z);
      if (valid) {
        lz_out[tloc * pitch + leaf] = lz;
        if (!isfinite(lz)) flag_status(status, ST_NONFINITE);
      }
      const float rz = 1.0f / z;
      if (j >= 1 && !mbar_wait(&bars->w_empty, (j - 1) & 1, status, abort_flag)) break;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float w0 = a[c * 8 + 2 * e] * rz, w1 = a[c * 8 + 2 * e + 1] * rz;
          const __nv_bfloat16 h0 = __float2bfloat16_rn(w0), h1 = __float2bfloat16_rn(w1);
          const float l0 = w0 - __bfloat162float(h0), l1 = w1 - __bfloat162float(h1);
          hi[e] = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
          lo[e] = pack_bf16x2(l0, l1);
        }
        st_shared_v4(wh + sw128_off(row, c), hi[0], hi[1], hi[2], hi[3]);
        st_shared_v4(wl + sw128_off(row, c), lo[0], lo[1], lo[2], lo[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->w_full);
    }
  } else {
    // epilogue warpgroup: G, VB rows -> g8/sg, vbar (overlaps the softmax of the next leaf)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t tloc = static_cast<int64_t>(blk) * 128 + row;   // tile index within the chunk
    const bool valid = tloc < tc;
    const int tid_wg = threadIdx.x - 192;
    const uint32_t stg = smem_u32(smem + kOffStG), stv = smem_u32(smem + kOffStV);
    for (int j = 0; j < nl; ++j) {
      const int leaf = l_begin + j;
      if (!mbar_wait(&bars->gv_full, j & 1, status, abort_flag)) break;
      __syncwarp();
      tc_fence_after();
      // pass 1 over G: the row's abs-max of g = scale * G
      float am = 0.f;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + kColG + 32 * q4, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) am = fmaxf(am, fabsf(__fmul_rn(__uint_as_float(r[i]), scale)));
      }
      am = fmaxf(am, 1e-30f);
      const float sgv = __fmul_rn(am, 1.0f / 127.0f);
      const float rr = __fdiv_rn(127.0f, am);
      if (valid) sg_out[tloc * pitch + leaf] = sgv;
      // pass 2: INT8 codes; then the vbar row as bf16 pairs
      uint32_t gw[32];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + kColG + 32 * q4, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint32_t w = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float gv = __fmul_rn(__uint_as_float(r[4 * i + e]), scale);
            const int cq = round_half_away_i8(__fmul_rn(gv, rr));
            w |= (static_cast<uint32_t>(cq) & 0xFFu) << (8 * e);
          }
          gw[q4 * 8 + i] = w;
        }
      }
      uint32_t vbw[64];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + kColV + 32 * q4, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) vbw[q4 * 16 + i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
      }
      // G and VB are in registers: the next leaf's G/VB MMAs may start
      tc_fence_before();
      mbar_arrive(&bars->gv_empty);
      // previous TMA store must have finished reading the staging buffers
      if (tid_wg == 0) {
        bulk_wait_group_read0();
        mbar_arrive(&bars->stg_free);
      }
      if (!mbar_wait(&bars->stg_free, j & 1, status, abort_flag)) break;
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 8; ++c) st_shared_v4(stg + sw128_off(row, c), gw[4 * c], gw[4 * c + 1], gw[4 * c + 2], gw[4 * c + 3]);
      // vbar: 64 bf16 per 128-byte half row, 8 chunks of 16 B per half
#pragma unroll
      for (int c = 0; c < 16; ++c)
        st_shared_v4(stv + (c >> 3) * (128 * 128) + sw128_off(row, c & 7), vbw[4 * c], vbw[4 * c + 1], vbw[4 * c + 2],
                     vbw[4 * c + 3]);
      fence_proxy_async_smem();
      mbar_arrive(&bars->stg_full);
      if (tid_wg == 0) {
        if (!mbar_wait(&bars->stg_full, j & 1, status, abort_flag)) break;
        tma_store_3d(&tm_g8, smem + kOffStG, 0, leaf, blk * 128);
        tma_store_3d(&tm_vb, smem + kOffStV, 0, leaf, blk * 128);
        tma_store_3d(&tm_vb, smem + kOffStV + 128 * 128, 64, leaf, blk * 128);
        bulk_commit_group();
      }
    }
    if (tid_wg == 0) bulk_wait_group0();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

int launch_leaf_stats(const LeafStatsMaps& maps, float* sg, float* lz, int64_t pitch, int64_t t0, int64_t tc, int nb,
                      float scale, int* status, int num_sms, cudaStream_t st) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(leaf_stats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
      return HTRC_ERR_CUDA;
    attr_done[dev] = true;
  }
  const int bx = static_cast<int>((tc + 127) / 128);
  int by = max(1, (num_sms + bx - 1) / bx);
  by = min(by, nb);
  const int lpc = (nb + by - 1) / by;
  by = (nb + lpc - 1) / lpc;
  leaf_stats_kernel<<<dim3(bx, by), 320, kSmemBytes, st>>>(maps.mu_hi, maps.mu_lo, maps.k, maps.v, maps.g8, maps.vb,
                                                            sg, lz, pitch, t0, tc, nb, lpc, scale, status);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

}  // namespace htrc
