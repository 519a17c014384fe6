// Row-max near-leaf selection on tcgen05 INT8 tensor cores.
//
// SEL[t, l] = max_r (dq8_r . g8_{t,l}) * (sdq_r * sg_{t,l}) + lz_{t,l}     (h3/htrc_flat_triton.py:214-254)
//
// Computed transposed so the maximum over the 64 tile rows stays inside one thread: per block of 128
// leaves, C = G8_block (M=128 leaves, K=128) x DQ8_tile^T (N=64 rows) into TMEM (int32); the thread
// owning TMEM lane l reduces its 64 columns.  One CTA per tile; warp 0 loads (TMA), warp 1 issues
// MMAs, warps 2-5 reduce.  The state is streamed once (HBM-bound).  With groups of G tiles sharing one
// state row (h3/htrc_flat.py:223-231) the CTA of tile t reads state row t / G and writes its own sel row;
// the maximum over the group's tiles is taken by the routing kernel.  ISO adds the isotropic curvature
// term c_l * |q_r - mu|^2 to every logit before the maximum (h3/htrc_flat.py:331-333).
// BF: the bf16 state (store="bf16", h3/htrc_flat_triton.py:247-248 with DOT=1): SEL[t, l] = max_r (bf16(dq_r) . g_l)
// + lz_l with bf16 g and dq as the operands of kind::f16 MMAs (no scales); a stage is the block's two 64-column
// halves of g (32 KB), two stages, two CTAs per SM.
#include "common.cuh"
#include "kernels.cuh"

namespace htrc {

namespace {
constexpr int kMaxStages = 3;
constexpr uint32_t kTmemCols = 128;
template <bool BF>
struct RLay {
  static constexpr int kStages = BF ? 2 : 3;
  static constexpr uint32_t kBlkBytes = (BF ? 2 : 1) * 128 * 128;     // 128 leaves x 128 B of g8 (BF: 2 halves)
  static constexpr uint32_t kParBytes = 3 * 128 * 4;                 // sg[128], lz[128], cv[128] (ISO)
  static constexpr uint32_t kStageBytes = kBlkBytes + kParBytes;
  static constexpr uint32_t kOffDq = 0;                              // 64 rows x 128 B (BF: 2 halves)
  static constexpr uint32_t kOffSdq = kOffDq + (BF ? 2 : 1) * 64 * 128;   // 64 floats, then dd[64] (ISO)
  static constexpr uint32_t kOffStage = kOffSdq + 1024;              // 1024-aligned
  static constexpr uint32_t kStageStride = (kStageBytes + 1023) / 1024 * 1024;
  static constexpr uint32_t kOffBar = kOffStage + kStages * kStageStride;
  static constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;
};

struct Bars {
  uint64_t dq_full;
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};
}  // namespace

template <bool ISO, bool BF>
__global__ void __launch_bounds__(192)
    rowmax_kernel(const __grid_constant__ CUtensorMap tm_dq8, const __grid_constant__ CUtensorMap tm_g8,
                  const __grid_constant__ CUtensorMap tm_sg, const __grid_constant__ CUtensorMap tm_lz,
                  const __grid_constant__ CUtensorMap tm_cv, const float* __restrict__ sdq,
                  const float* __restrict__ dd, float* __restrict__ sel, int64_t pitch, int64_t t0, int nb,
                  int group, int* status) {
  using Y = RLay<BF>;
  constexpr int kStages = Y::kStages;
  constexpr uint32_t kBlkBytes = Y::kBlkBytes, kOffDq = Y::kOffDq, kOffSdq = Y::kOffSdq, kOffStage = Y::kOffStage;
  constexpr uint32_t kStageStride = Y::kStageStride;
  static_assert(!(ISO && BF), "the bf16 state has the linear far field");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + Y::kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tloc = blockIdx.x;
  const int srow = tloc / group;             // state row of this tile
  const int64_t tg = t0 + tloc;
  const int nblk = (nb + 127) / 128;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->dq_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1 + 128);   // MMA commit + the 128 reducing threads (they read sg/lz)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 128);
    }
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_stream = policy_evict_first();
      if constexpr (BF) {
        // bf16 offsets of the tile as two 64-column halves; no row scales
        mbar_arrive_expect_tx(&bars->dq_full, 2 * 64 * 128);
        tma_load_3d(smem + kOffDq, &tm_dq8, &bars->dq_full, 0, static_cast<int>(tg * 64), 0, pol_stream);
      } else {
        mbar_arrive_expect_tx(&bars->dq_full, 64 * 128 + 256 + (ISO ? 256 : 0));
        tma_load_2d(smem + kOffDq, &tm_dq8, &bars->dq_full, 0, static_cast<int>(tg * 64), pol_stream);
        bulk_load(smem + kOffSdq, sdq + tg * 64, 256, &bars->dq_full, pol_stream);
        if (ISO) bulk_load(smem + kOffSdq + 256, dd + tg * 64, 256, &bars->dq_full, pol_stream);
      }
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&bars->empty[s], ((j / kStages) - 1) & 1, status, abort_flag)) break;
        uint8_t* st = smem + kOffStage + s * kStageStride;
        if constexpr (BF) {
          mbar_arrive_expect_tx(&bars->full[s], kBlkBytes + 512);
          tma_load_4d(st, &tm_g8, &bars->full[s], 0, j * 128, 0, srow, pol_stream);     // both halves
          tma_load_2d(st + kBlkBytes + 512, &tm_lz, &bars->full[s], j * 128, srow, pol_stream);
          continue;
        }
        mbar_arrive_expect_tx(&bars->full[s], kBlkBytes + 1024 + (ISO ? 512 : 0));
        tma_load_3d(st, &tm_g8, &bars->full[s], 0, j * 128, srow, pol_stream);
        tma_load_2d(st + kBlkBytes, &tm_sg, &bars->full[s], j * 128, srow, pol_stream);
        tma_load_2d(st + kBlkBytes + 512, &tm_lz, &bars->full[s], j * 128, srow, pol_stream);
        if (ISO) tma_load_2d(st + kBlkBytes + 1024, &tm_cv, &bars->full[s], j * 128, srow, pol_stream);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = BF ? idesc_bf16(128, 64, false, false) : idesc_i8(128, 64);
      const uint32_t dq = smem_u32(smem + kOffDq);
      bool ok = mbar_wait(&bars->dq_full, 0, status, abort_flag);
      int nmma = 0;                   // blocks whose MMAs were issued (and committed)
      for (int j = 0; ok && j < nblk; ++j) {
        const int s = j % kStages, b = j & 1;
        if (!mbar_wait(&bars->full[s], (j / kStages) & 1, status, abort_flag)) break;
        if (j >= 2 && !mbar_wait(&bars->acc_empty[b], ((j >> 1) - 1) & 1, status, abort_flag)) break;
        tc_fence_after();
        const uint32_t gst = smem_u32(smem + kOffStage + s * kStageStride);
        if constexpr (BF) {
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16(tmem + 64 * b, sw128_desc(gst + h * 16384 + kk * 32, 16, 1024),
                       sw128_desc(dq + h * 8192 + kk * 32, 16, 1024), idesc, (h | kk) != 0);
        } else {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            mma_i8(tmem + 64 * b, sw128_desc(gst + kk * 32, 16, 1024), sw128_desc(dq + kk * 32, 16, 1024), idesc,
                   kk != 0);
          }
        }
        mma_commit(&bars->acc_full[b]);
        mma_commit(&bars->empty[s]);
        nmma = j + 1;
      }
      // the stage release signals of the last blocks have no waiter: let them land before the CTA leaves
      drain_ring<false>(bars->empty, kStages, nmma, status, abort_flag);
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;                 // leaf within the block
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float* sdq_s = reinterpret_cast<const float*>(smem + kOffSdq);
    const float* dd_s = sdq_s + 64;
    if (mbar_wait(&bars->dq_full, 0, status, abort_flag)) {
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kStages, b = j & 1;
        if (!mbar_wait(&bars->acc_full[b], (j >> 1) & 1, status, abort_flag)) break;
        if (!mbar_wait(&bars->full[s], (j / kStages) & 1, status, abort_flag)) break;
        __syncwarp();
        tc_fence_after();
        uint32_t d0[32], d1[32];
        tmem_ld32(tmem + lane_base + 64 * b, d0);
        tmem_ld32(tmem + lane_base + 64 * b + 32, d1);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&bars->acc_empty[b]);
        const uint8_t* st = smem + kOffStage + s * kStageStride;
        const float sgl = BF ? 1.0f : reinterpret_cast<const float*>(st + kBlkBytes)[r];
        const float lzl = reinterpret_cast<const float*>(st + kBlkBytes + 512)[r];
        const float cvl = ISO ? reinterpret_cast<const float*>(st + kBlkBytes + 1024)[r] : 0.f;
        // the stage is refilled by TMA (async proxy) once this arrival lands: without the proxy fence the
        // refill can overtake these generic reads (seen as the next block's sg or lz in about one warp-block
        // in 10^7)
        fence_proxy_async_smem();
        mbar_arrive(&bars->empty[s]);
        float best = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if constexpr (BF) {           // float32 accumulators: the logit is the dot itself
            best = fmaxf(best, fmaxf(__uint_as_float(d0[i]), __uint_as_float(d1[i])));
            continue;
          }
          float a = __fmul_rn(static_cast<float>(static_cast<int>(d0[i])), __fmul_rn(sdq_s[i], sgl));
          float b = __fmul_rn(static_cast<float>(static_cast<int>(d1[i])), __fmul_rn(sdq_s[32 + i], sgl));
          if (ISO) {
            a = __fadd_rn(a, __fmul_rn(cvl, dd_s[i]));
            b = __fadd_rn(b, __fmul_rn(cvl, dd_s[32 + i]));
          }
          best = fmaxf(best, fmaxf(a, b));
        }
        const int leaf = j * 128 + r;
        if (leaf < nb) sel[static_cast<int64_t>(tloc) * pitch + leaf] = __fadd_rn(best, lzl);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

int launch_rowmax(const RowmaxMaps& maps, const float* sdq, const float* dd, float* sel, int64_t pitch, int64_t t0,
                  int64_t tc, int nb, int group, int* status, cudaStream_t st, bool bf16_state) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(rowmax_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             RLay<false>::kSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(rowmax_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             RLay<false>::kSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(rowmax_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             RLay<true>::kSmemBytes) != cudaSuccess)
      return HTRC_ERR_CUDA;
    attr_done[dev] = true;
  }
  if (bf16_state && dd != nullptr) return HTRC_ERR_UNSUPPORTED;
  auto kernel = bf16_state ? rowmax_kernel<false, true> : dd != nullptr ? rowmax_kernel<true, false> : rowmax_kernel<false, false>;
  const uint32_t smem = bf16_state ? RLay<true>::kSmemBytes : RLay<false>::kSmemBytes;
  kernel<<<static_cast<unsigned>(tc), 192, smem, st>>>(maps.dq8, maps.g8, maps.sg, maps.lz, maps.cv, sdq, dd, sel,
                                                       pitch, t0, nb, group > 1 ? group : 1, status);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

}  // namespace htrc
