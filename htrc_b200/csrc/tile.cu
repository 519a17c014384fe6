// Far field + near field of the flat HTRC operator, fused into one online softmax per query row,
// on tcgen05 tensor cores (h3/htrc_flat_triton.py:88-211, `_tile_kernel` with I8=1, DOT=1; the split
// merge of :257-273 is unnecessary because one CTA walks all leaves of its tiles).
//
// One CTA per pair of 64-row tiles (A = 2p, B = 2p+1).  Each tile is an M=64 MMA; tile A's accumulators
// live in TMEM lanes {0..15} + 32k, tile B's at lane offset 16, so the 128 softmax threads each own one
// query row.  Steps (64 columns each):
//   far  (blocks of 64 leaves of the tile's own state): S = dq8 . g8^T (int8 -> int32),
//        logit = S * (sdq_r * sg_l) + lz_l, excluded / padding leaves masked, value vbar_l (bf16);
//   near (one routed 64-token leaf per step):           S = q8 . k8^T,
//        logit = S * (sq_r * ks_j) * scale, value v_j (bf16).
// P = exp(logit - m) goes to shared memory as bf16 and O += P . V runs as an M=64, N=128 bf16 MMA.
// The running maximum is updated lazily: O and l are rescaled only when the maximum grows by more
// than 2^8 (P <= 256 otherwise), so most steps never touch O.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer (+ TMEM owner), warps 2-5 softmax.
#include "common.cuh"
#include "kernels.cuh"

namespace htrc {

namespace {
constexpr int kStages = 3;
constexpr uint32_t kXBytes = 64 * 128;                        // g8 block / k8 leaf: 64 rows x 128 B
constexpr uint32_t kYBytes = 64 * 256;                        // vbar block / v leaf: 2 chunks of 64x64 bf16
constexpr uint32_t kParBytes = 1024;                          // far: lz[64], sg[64], excl[64]; near: ks[64]
constexpr uint32_t kTileStage = kXBytes + kYBytes + kParBytes;  // 25600
constexpr uint32_t kStageBytes = 2 * kTileStage;              // 51200 (a multiple of 1024)
constexpr uint32_t kOffQ8 = 0;                                // 2 tiles x 8 KB
constexpr uint32_t kOffDq8 = 16384;                           // 2 tiles x 8 KB
constexpr uint32_t kOffStage = 32768;
constexpr uint32_t kOffP = kOffStage + kStages * kStageBytes;  // 2 tiles x 8 KB
constexpr uint32_t kOffIdx = kOffP + 16384;                   // 2 tiles x kMaxKx int32
constexpr int kMaxKx = 1536;
constexpr uint32_t kOffBar = kOffIdx + 2 * kMaxKx * 4;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColO = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescale = 8.0f;   // lazy-rescale threshold (log2 units)

struct Bars {
  uint64_t qd_full;
  uint64_t st_full[kStages];
  uint64_t st_empty[kStages];
  uint64_t s_full[2];
  uint64_t s_empty[2];
  uint64_t p_full;
  uint64_t pv_done;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
}  // namespace

__global__ void __launch_bounds__(192, 1)
    tile_attention_kernel(const __grid_constant__ CUtensorMap tm_q8, const __grid_constant__ CUtensorMap tm_dq8,
                          const __grid_constant__ CUtensorMap tm_g8, const __grid_constant__ CUtensorMap tm_vb,
                          const __grid_constant__ CUtensorMap tm_lz, const __grid_constant__ CUtensorMap tm_sg,
                          const __grid_constant__ CUtensorMap tm_excl, const __grid_constant__ CUtensorMap tm_k8,
                          const __grid_constant__ CUtensorMap tm_v, const float* __restrict__ sq,
                          const float* __restrict__ sdq, const float* __restrict__ ks, const int32_t* __restrict__ idx,
                          int kx, int nb, int nf, int64_t n, int64_t t0, int64_t tc, float scale,
                          const float* __restrict__ tail_part, float* __restrict__ out, float* __restrict__ lse,
                          int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  int32_t* idx_s = reinterpret_cast<int32_t*>(smem + kOffIdx);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tlocA = 2 * blockIdx.x;
  const int ntiles = (tlocA + 1 < tc) ? 2 : 1;
  const int nn = kx;                 // near steps: one routed leaf per step
  const int total = nf + nn;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->qd_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->st_full[s], 1);
      mbar_init(&bars->st_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->s_empty[b], 128);
    }
    mbar_init(&bars->p_full, 128);
    mbar_init(&bars->pv_done, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    // routed leaves of both tiles -> shared memory, range-checked
    for (int x = 0; x < ntiles; ++x) {
      const int32_t* src = idx + static_cast<int64_t>(tlocA + x) * kx;
      for (int e = lane; e < nn; e += 32) {
        int leaf = __ldg(src + e);
        if (leaf < 0 || leaf >= nb) {
          flag_status(status, ST_BAD_INDEX);
          leaf = 0;
        }
        idx_s[x * kMaxKx + e] = leaf;
      }
    }
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_stream = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      mbar_arrive_expect_tx(&bars->qd_full, 2 * kXBytes * ntiles);
      for (int x = 0; x < ntiles; ++x) {
        const int row = static_cast<int>((t0 + tlocA + x) * 64);
        tma_load_2d(smem + kOffQ8 + x * kXBytes, &tm_q8, &bars->qd_full, 0, row, pol_stream);
        tma_load_2d(smem + kOffDq8 + x * kXBytes, &tm_dq8, &bars->qd_full, 0, row, pol_stream);
      }
      for (int j = 0; j < total; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&bars->st_empty[s], ((j / kStages) - 1) & 1, status, abort_flag)) break;
        uint8_t* st = smem + kOffStage + s * kStageBytes;
        if (j < nf) {
          mbar_arrive_expect_tx(&bars->st_full[s], (kXBytes + kYBytes + 256 + 256 + 64) * ntiles);
          for (int x = 0; x < ntiles; ++x) {
            uint8_t* tx = st + x * kTileStage;
            const int tl = tlocA + x;
            tma_load_3d(tx, &tm_g8, &bars->st_full[s], 0, j * 64, tl, pol_stream);
            tma_load_3d(tx + kXBytes, &tm_vb, &bars->st_full[s], 0, j * 64, tl, pol_stream);
            tma_load_3d(tx + kXBytes + kYBytes / 2, &tm_vb, &bars->st_full[s], 64, j * 64, tl, pol_stream);
            tma_load_2d(tx + kXBytes + kYBytes, &tm_lz, &bars->st_full[s], j * 64, tl, pol_stream);
            tma_load_2d(tx + kXBytes + kYBytes + 256, &tm_sg, &bars->st_full[s], j * 64, tl, pol_stream);
            tma_load_2d(tx + kXBytes + kYBytes + 512, &tm_excl, &bars->st_full[s], j * 64, tl, pol_stream);
          }
        } else {
          const int e = j - nf;
          mbar_arrive_expect_tx(&bars->st_full[s], (kXBytes + kYBytes + 256) * ntiles);
          for (int x = 0; x < ntiles; ++x) {
            uint8_t* tx = st + x * kTileStage;
            const int leaf = idx_s[x * kMaxKx + e];
            tma_load_2d(tx, &tm_k8, &bars->st_full[s], 0, leaf * 64, pol_keep);
            tma_load_2d(tx + kXBytes, &tm_v, &bars->st_full[s], 0, leaf * 64, pol_keep);
            tma_load_2d(tx + kXBytes + kYBytes / 2, &tm_v, &bars->st_full[s], 64, leaf * 64, pol_keep);
            bulk_load(tx + kXBytes + kYBytes, ks + static_cast<int64_t>(leaf) * 64, 256, &bars->st_full[s], pol_keep);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_qk = idesc_i8(64, 64);
      const uint32_t id_pv = idesc_bf16(64, 128, false, true);
      bool ok = mbar_wait(&bars->qd_full, 0, status, abort_flag);
      for (int j = 0; ok && j <= total; ++j) {
        if (j < total) {
          const int s = j % kStages, b = j & 1;
          if (!mbar_wait(&bars->st_full[s], (j / kStages) & 1, status, abort_flag)) break;
          if (j >= 2 && !mbar_wait(&bars->s_empty[b], ((j >> 1) - 1) & 1, status, abort_flag)) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + (j < nf ? kOffDq8 : kOffQ8));
          const uint32_t st = smem_u32(smem + kOffStage + s * kStageBytes);
          for (int x = 0; x < ntiles; ++x) {
            const uint32_t d = tmem + (static_cast<uint32_t>(16 * x) << 16) + 64 * b;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_i8(d, sw128_desc(a_base + x * kXBytes + kk * 32, 16, 1024),
                     sw128_desc(st + x * kTileStage + kk * 32, 16, 1024), id_qk, kk != 0);
          }
          mma_commit(&bars->s_full[b]);
        }
        if (j >= 1) {
          const int jj = j - 1, s = jj % kStages;
          if (!mbar_wait(&bars->p_full, jj & 1, status, abort_flag)) break;
          tc_fence_after();
          const uint32_t st = smem_u32(smem + kOffStage + s * kStageBytes);
          const uint32_t pb = smem_u32(smem + kOffP);
          for (int x = 0; x < ntiles; ++x) {
            const uint32_t d = tmem + (static_cast<uint32_t>(16 * x) << 16) + kColO;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16(d, sw128_desc(pb + x * kXBytes + kk * 32, 16, 1024),
                       sw128_desc(st + x * kTileStage + kXBytes + kk * 2048, kYBytes / 2, 1024), id_pv,
                       (jj | kk) != 0);
          }
          mma_commit(&bars->pv_done);
          mma_commit(&bars->st_empty[s]);
        }
      }
    }
  } else {
    // softmax warpgroup: thread -> (tile x, row r)
    const int quarter = warp & 3;
    const int x = lane >> 4;
    const int r = quarter * 16 + (lane & 15);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const bool has_tile = x < ntiles;
    const int64_t tl = tlocA + x;
    const int64_t gr = (t0 + tl) * 64 + r;
    const bool valid = has_tile && gr < n;
    const float sq_r = has_tile ? __ldg(sq + gr) : 0.f;
    const float sdq_r = has_tile ? __ldg(sdq + gr) : 0.f;
    const uint32_t p_row = smem_u32(smem + kOffP + x * kXBytes);
    float m_used = -INFINITY, l = 0.f;
    bool aborted = false;
    for (int j = 0; j < total; ++j) {
      const int b = j & 1, s = j % kStages;
      if (!mbar_wait(&bars->s_full[b], (j >> 1) & 1, status, abort_flag)) { aborted = true; break; }
      __syncwarp();
      tc_fence_after();
      uint32_t d0[32], d1[32];
      tmem_ld32(tmem + lane_base + 64 * b, d0);
      tmem_ld32(tmem + lane_base + 64 * b + 32, d1);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&bars->s_empty[b]);
      if (!mbar_wait(&bars->st_full[s], (j / kStages) & 1, status, abort_flag)) { aborted = true; break; }
      const uint8_t* par = smem + kOffStage + s * kStageBytes + x * kTileStage + kXBytes + kYBytes;
      float lg[64];
      if (j < nf) {
        const float* lz_s = reinterpret_cast<const float*>(par);
        const float* sg_s = reinterpret_cast<const float*>(par + 256);
        const uint8_t* ex_s = par + 512;
        const int lb = j * 64;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const int di = static_cast<int>(i < 32 ? d0[i] : d1[i - 32]);
          const float v = __fadd_rn(__fmul_rn(static_cast<float>(di), __fmul_rn(sdq_r, sg_s[i])), lz_s[i]);
          lg[i] = (ex_s[i] != 0 || lb + i >= nb) ? -INFINITY : v * kLog2e;
        }
      } else {
        const float* ks_s = reinterpret_cast<const float*>(par);
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const int di = static_cast<int>(i < 32 ? d0[i] : d1[i - 32]);
          lg[i] = __fmul_rn(static_cast<float>(di), __fmul_rn(__fmul_rn(sq_r, ks_s[i]), scale)) * kLog2e;
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) mx = fmaxf(mx, lg[i]);
      const float m_new = fmaxf(m_used, mx);
      if (j >= 1 && !mbar_wait(&bars->pv_done, (j - 1) & 1, status, abort_flag)) { aborted = true; break; }
      // lazy rescale; the TMEM access is warp-collective, so the whole warp joins when any lane needs it
      const bool need = m_new > m_used + kRescale;
      const float alpha = need ? ex2(m_used - m_new) : 1.0f;
      if (need) {
        l *= alpha;
        m_used = m_new;
      }
      __syncwarp();
      if (j >= 1 && __any_sync(0xffffffffu, need)) {
        tc_fence_after();
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + kColO + 32 * q4, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tmem + lane_base + kColO + 32 * q4, o);
        }
        tmem_st_wait();
      }
      const bool live = m_used != -INFINITY;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = live ? ex2(lg[c * 8 + 2 * e] - m_used) : 0.f;
          const float p1 = live ? ex2(lg[c * 8 + 2 * e + 1] - m_used) : 0.f;
          rs += p0 + p1;
          w[e] = pack_bf16x2(p0, p1);
        }
        st_shared_v4(p_row + sw128_off(r, c), w[0], w[1], w[2], w[3]);
      }
      l += rs;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_full);
    }
    if (!aborted && total > 0 && mbar_wait(&bars->pv_done, (total - 1) & 1, status, abort_flag)) {
      __syncwarp();
      tc_fence_after();
      // merge with the tail partial (natural-log units) and normalise
      const float m1 = m_used * kLn2;
      float wa = 1.f, wb = 0.f, den = l, mm = m1;
      const float* tp = (tail_part != nullptr && valid) ? tail_part + gr * 130 : nullptr;
      if (tp) {
        const float mt = tp[128], lt = tp[129];
        mm = fmaxf(m1, mt);
        wa = expf(m1 - mm);
        wb = expf(mt - mm);
        den = l * wa + lt * wb;
      }
      const float inv = 1.0f / fmaxf(den, 1e-30f);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + kColO + 32 * q4, o);
        tmem_ld_wait();
        if (valid) {
          float4* dst = reinterpret_cast<float4*>(out + gr * 128 + 32 * q4);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float a = __uint_as_float(o[4 * i + e]) * wa;
              if (tp) a = fmaf(tp[32 * q4 + 4 * i + e], wb, a);
              v[e] = a * inv;
            }
            dst[i] = make_float4(v[0], v[1], v[2], v[3]);
          }
        }
      }
      if (valid && lse != nullptr) lse[gr] = mm + logf(fmaxf(den, 1e-30f));
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

int launch_tile_attention(const TileMaps& maps, const float* sq, const float* sdq, const float* ks, const int32_t* idx,
                          int kx, int nb, int64_t n, int64_t t0, int64_t tc, float scale, const float* tail_part,
                          float* out, float* lse, int* status, cudaStream_t st) {
  if (kx > kMaxKx) return HTRC_ERR_UNSUPPORTED;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(tile_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
        cudaSuccess)
      return HTRC_ERR_CUDA;
    attr_done[dev] = true;
  }
  const int nf = kx >= nb ? 0 : (nb + 63) / 64;
  const unsigned grid = static_cast<unsigned>((tc + 1) / 2);
  tile_attention_kernel<<<grid, 192, kSmemBytes, st>>>(maps.q8, maps.dq8, maps.g8, maps.vb, maps.lz, maps.sg,
                                                        maps.excl, maps.k8, maps.v, sq, sdq, ks, idx, kx, nb, nf, n, t0,
                                                        tc, scale, tail_part, out, lse, status);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

}  // namespace htrc
