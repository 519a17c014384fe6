// Leaf statistics of the flat HTRC far field on tcgen05 tensor cores.
//
// One CTA owns 128 tile centres (the MMA M dimension) and a contiguous range of leaves.  Per leaf:
//   S  = mu . K_leaf^T            (M=128 centres, N=64 tokens, K=128; mu = mu_hi + mu_lo, two bf16 MMAs
//                                  with mu in TMEM as the A operand, which leaves shared memory to four
//                                  K/V stages)
//   softmax over the 64 tokens of each centre row (one thread per row, in registers): lz, w; W = w_hi + w_lo
//   (bf16) goes back into TMEM over the S buffer it came from, as the A operand of the next MMAs
//   [G | VB] = W . [K_leaf | V_leaf]  (M=128, N=256, K=64; two bf16 MMA chains (w_hi, w_lo) with A in TMEM,
//                                  K and V of a stage adjacent in shared memory as one MN-major operand)
//   epilogue: g = scale * G -> (g8, sg) half-away INT8 with the row abs-max scale; vbar -> bf16;
//   g8/vbar rows staged in shared memory and written by TMA stores, lz/sg by plain stores.
// This is the arithmetic of h3/htrc_flat_triton.py:41-85 (_stats_kernel, I8=1).  Precision "fp32" (the
// reference's PREC="ieee"): the hi/lo splits keep the products at ~2^-16 relative precision.  Precision "tf32"
// (PREC="tf32", the reference's production setting): the float32 operands of both dots, the centre and the
// softmax weights, enter with their low 13 mantissa bits cleared, as the reference's tensor-core dots read them
// on sm_100 (its log-partitions match that model to ~1e-5); hi + lo then represents each operand exactly.
// ISO adds the isotropic curvature of each (centre, leaf) (h3/htrc_flat.py:331-333, the torch
// backend's curvature="iso"): c = 0.5 / D * max(tr, 0), tr = scale^2 (sum_s w_s |k_s|^2 - |sum_s w_s k_s|^2);
// the softmax warps form sum_s w_s |k_s|^2 from the key norms staged with K/V, the epilogue |G|^2 from
// its G columns (the two halves exchange partial sums with their abs-maxima).
// LEAF (64, 32 or 16 keys; INT8 state, linear far field) sets the leaf: a K/V stage still holds 64 keys, i.e.
// 64 / LEAF leaves, and each leaf takes its own S (N = LEAF), softmax, [G | VB] (K = LEAF) and epilogue
// (h3/htrc_flat.py:99-103: the reference takes any leaf that divides the key count, default 16).
// BF stores the state as bf16 values without scales (store="bf16", h3/htrc_flat_triton.py:82-84): g = bf16(scale
// G), vbar = bf16(VB), each staged as two 64-column boxes; its staging needs 32 KB more, so it runs four K/V stages.
// FP8 stores the state as e4m3 codes with per-(centre, leaf) row scales instead (h3/htrc_flat_triton.py:65-72,
// store="fp8"): sg = max(amax|g| * (1/448), 1e-30), g codes = e4m3(g / sg) rounded to nearest even and
// saturated at 448, and the same for vbar with sv.
//
// Warp roles (512 threads, one role per warpgroup so that setmaxnreg can move registers from the
// issuing warps to the arithmetic): warpgroup 0 = warp 0 TMA producer, warp 1 S issuer (+ TMEM owner),
// warp 2 G/VB issuer, warp 3 idle; warpgroup 1 softmax (S -> lz, W); warpgroups 2 and 3 the epilogue,
// each for half of the 128 columns of G and VB (the two halves of a row exchange their abs-max through
// shared memory and a named barrier), so each leaf's quantisation is spread over eight warps.  A
// thread's row is 32 * (warp % 4) + lane, the TMEM lane it may access.  The producer and issuer warps
// run converged and let one elected lane issue.
#include "common.cuh"
#include "kernels.cuh"

namespace htrc {

namespace {
constexpr int kThreads = 512;
constexpr int kMaxStages = 5;
constexpr uint32_t kLeafBytes = 64 * 128 * 2;       // K (or V) of one 64-token leaf
constexpr uint32_t kStageBytes = 2 * kLeafBytes;    // K + V
constexpr uint32_t kOffStage = 0;
// shared-memory layout; BF (bf16 state) stages g as two boxes and runs one K/V stage fewer
template <bool BF>
struct SLay {
  static constexpr int kStages = BF ? 4 : 5;
  static constexpr uint32_t kOffStG = kOffStage + kStages * kStageBytes;   // g staging: 128 rows x 128 B (BF: x2)
  static constexpr uint32_t kOffStV = kOffStG + (BF ? 2 : 1) * 128 * 128;  // vbar staging: 2 x (128 rows x 128 B)
  static constexpr uint32_t kOffAm = kOffStV + 2 * 128 * 128;   // row abs-max halves [2 (leaf parity)][2 (half)][128]
  static constexpr uint32_t kOffB2 = kOffAm + 2 * 2 * 128 * 4;  // ISO: |G|^2 halves [2][2][128]
  static constexpr uint32_t kOffAw = kOffB2 + 2 * 2 * 128 * 4;  // ISO: sum_s w_s |k_s|^2 [4 (leaf % 4)][128]
  static constexpr uint32_t kOffKn = kOffAw + 4 * 128 * 4;      // ISO: key norms of each K/V stage [kStages][64]
  static constexpr uint32_t kOffBar = kOffKn + kStages * 64 * 4;
  static constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + barriers, + alignment slack
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;      // two 64-column S buffers; W_hi / W_lo of the leaf then in 32 columns each
constexpr uint32_t kColG = 128;    // 128 columns
constexpr uint32_t kColV = 256;    // 128 columns
constexpr uint32_t kColMu = 384;   // mu_hi (64 columns of bf16 pairs), then mu_lo

struct Bars {
  uint64_t mu_full;    // the 128 softmax threads stored their mu rows in TMEM
  uint64_t kv_full[kMaxStages];
  uint64_t kv_empty[kMaxStages];
  uint64_t s_full[2];
  uint64_t s_empty[2];  // G/VB of the leaf done: its W (over S in TMEM) is consumed
  uint64_t w_full[2];   // the 128 softmax threads wrote W into the S buffer
  uint64_t gv_full;
  uint64_t gv_empty;   // the 256 epilogue threads drained G and VB into registers
  uint64_t stg_free;   // thread 0 of the epilogue: the previous TMA stores have read the staging buffers
  uint64_t stg_full;   // the 256 epilogue threads: this leaf's rows are staged
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// INT8 codes of two values y (|y| <= 127 + rounding): trunc(y + copysign(0.5, y)) with the sum rounded to
// float first, the reference's round-half-away-from-zero codes.  z + copysign(2^23, z) rounded toward zero
// drops the fraction; subtracting the constant again gives trunc(z) exactly, and adding 1.5 * 2^23 puts
// the code in the low byte of the float's bits.  Returns those bits (only the low byte is used).
__device__ __forceinline__ uint2 half_away_codes2(float2 y) {
  const uint32_t s0 = __float_as_uint(y.x) & 0x80000000u, s1 = __float_as_uint(y.y) & 0x80000000u;
  const float2 z = add2(y, make_float2(__uint_as_float(s0 | 0x3F000000u), __uint_as_float(s1 | 0x3F000000u)));
  const float2 c23 = make_float2(__uint_as_float((__float_as_uint(z.x) & 0x80000000u) | 0x4B000000u),
                                 __uint_as_float((__float_as_uint(z.y) & 0x80000000u) | 0x4B000000u));
  const float2 t = sub2(add2_rz(z, c23), c23);
  const float2 b = add2(t, make_float2(12582912.0f, 12582912.0f));
  return make_uint2(__float_as_uint(b.x), __float_as_uint(b.y));
}
}  // namespace

template <bool ISO, bool FP8, bool TDIV, int LEAF, bool BF = false>
__global__ void __launch_bounds__(kThreads, 1)
    leaf_stats_kernel(const uint16_t* __restrict__ mu_hi_g, const uint16_t* __restrict__ mu_lo_g, int64_t nt,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_g8, const __grid_constant__ CUtensorMap tm_vb,
                      float* __restrict__ sg_out, float* __restrict__ lz_out, int64_t pitch, int64_t t0, int64_t tc,
                      int nb, int leaves_per_cta, float scale, const float* __restrict__ kn2,
                      float* __restrict__ cv_out, float* __restrict__ sv_out, int* status, uint32_t wmask) {
  constexpr int kStages = SLay<BF>::kStages;
  constexpr uint32_t kOffStG = SLay<BF>::kOffStG, kOffStV = SLay<BF>::kOffStV, kOffAm = SLay<BF>::kOffAm;
  constexpr uint32_t kOffB2 = SLay<BF>::kOffB2, kOffAw = SLay<BF>::kOffAw, kOffKn = SLay<BF>::kOffKn;
  static_assert(!BF || (!ISO && !FP8 && LEAF == 64), "the bf16 state: linear far field, leaf 64");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + SLay<BF>::kOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int blk = blockIdx.x;                       // block of 128 centres (local to the chunk)
  const int l_begin = blockIdx.y * leaves_per_cta;
  const int l_end = min(nb, l_begin + leaves_per_cta);
  const int nl = max(0, l_end - l_begin);
  static_assert(LEAF == 64 || LEAF == 32 || LEAF == 16, "leaf of 16, 32 or 64 keys");
  static_assert(LEAF == 64 || (!ISO && !FP8), "the iso and fp8 variants take leaf 64");
  constexpr int kPerStage = 64 / LEAF;            // leaves per K/V stage
  const int nst = (nl + kPerStage - 1) / kPerStage;   // K/V stages of this CTA
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->mu_full, 128);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->s_empty[b], 1);
      mbar_init(&bars->w_full[b], 128);
    }
    mbar_init(&bars->gv_full, 1);
    mbar_init(&bars->gv_empty, 256);
    mbar_init(&bars->stg_free, 1);
    mbar_init(&bars->stg_full, 256);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp < 4) {
    // one setmaxnreg per warpgroup, executed by all of its warps at the same instruction
    asm volatile("setmaxnreg.dec.sync.aligned.u32 64;");
    if (warp == 0) {
      // ------------------------------------------------------------------ TMA producer
      const uint32_t leader = elect_one();
      if (nl > 0) {
        const uint64_t pol_keep = policy_evict_last();
        if (leader) {
          tma_prefetch_desc(&tm_k);
          tma_prefetch_desc(&tm_v);
        }
        // one stage = the next 64 keys = kPerStage leaves
        for (int gi = 0; gi < nst; ++gi) {
          const int s = gi % kStages;
          if (gi >= kStages && !mbar_wait_warp(&bars->kv_empty[s], ((gi / kStages) - 1) & 1, status, abort_flag))
            break;
          if (leader) {
            uint8_t* st = smem + kOffStage + s * kStageBytes;
            const int row = l_begin * LEAF + gi * 64;
            mbar_arrive_expect_tx(&bars->kv_full[s], kStageBytes + (ISO ? 256 : 0));
            tma_load_3d(st, &tm_k, &bars->kv_full[s], 0, row, 0, pol_keep);        // both 64-column halves
            tma_load_3d(st + kLeafBytes, &tm_v, &bars->kv_full[s], 0, row, 0, pol_keep);
            if (ISO) bulk_load(smem + kOffKn + s * 256, kn2 + row, 256, &bars->kv_full[s], pol_keep);
          }
          __syncwarp();
        }
      }
    } else if (warp == 1) {
      // ------------------------------------------------------------------ S issuer
      // S(j) = mu . K_j^T into S buffer j % 2 once the K/V stage landed and the softmax released it
      const uint32_t leader = elect_one();
      if (nl > 0) {
        const uint32_t id_s = idesc_bf16(128, LEAF, false, false);
        bool ok = mbar_wait_warp(&bars->mu_full, 0, status, abort_flag);
        for (int j = 0; ok && j < nl; ++j) {
          const int gi = j / kPerStage, s = gi % kStages, b = j & 1;
          if (!mbar_wait_warp(&bars->kv_full[s], (gi / kStages) & 1, status, abort_flag)) break;
          if (j >= 2 && !mbar_wait_warp(&bars->s_empty[b], ((j >> 1) - 1) & 1, status, abort_flag)) break;
          tc_fence_after();
          // this leaf's keys are rows LEAF * (j % kPerStage) .. of the stage's 64 (whole 8-row swizzle atoms)
          const uint32_t kst = smem_u32(smem + kOffStage + s * kStageBytes) + (j % kPerStage) * LEAF * 128;
          const uint32_t d = tmem + kColS + 64 * b;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                // A: mu_hi / mu_lo dims 64 c + 16 kk .. + 15 = TMEM columns (64 h + 32 c + 8 kk) .. + 7
                const uint32_t a = tmem + kColMu + 64 * h + 32 * c + 8 * kk;
                const uint64_t bdesc = sw128_desc(kst + c * (kLeafBytes / 2) + kk * 32, 16, 1024);
                mma_bf16_ts_by(leader, d, a, bdesc, id_s, (h | c | kk) != 0);
              }
            }
          }
          mma_commit_by(leader, &bars->s_full[b]);
        }
      }
    } else if (warp == 2) {
      // ------------------------------------------------------------------ G/VB issuer
      // G(j) = W . K_j and VB(j) = W . V_j once the softmax wrote W (into S buffer j % 2) and the epilogue
      // drained the previous G/VB; their completion releases the S buffer for S(j + 2) and the K/V stage
      const uint32_t leader = elect_one();
      if (nl > 0) {
        const uint32_t id_gv = idesc_bf16(128, 256, false, true);
        static_assert(kColV == kColG + 128 && kStageBytes == 2 * kLeafBytes, "[G | VB] and [K | V] side by side");
        for (int j = 0; j < nl; ++j) {
          const int gi = j / kPerStage, s = gi % kStages, b = j & 1;
          if (!mbar_wait_warp(&bars->w_full[b], (j >> 1) & 1, status, abort_flag)) break;
          if (j >= 1 && !mbar_wait_warp(&bars->gv_empty, (j - 1) & 1, status, abort_flag)) break;
          tc_fence_after();
          // this leaf's keys: the 16-key K steps (j % kPerStage) * LEAF / 16 .. of the stage
          const uint32_t kst = smem_u32(smem + kOffStage + s * kStageBytes) + (j % kPerStage) * LEAF * 128;
          const uint32_t wt = tmem + kColS + 64 * b;      // W_hi at wt, W_lo at wt + 32 (keys in pairs)
          // [G | VB] = (W_hi + W_lo) . [K | V]: the stage's K and V are four 64-column chunks 8 KB apart, one
          // N = 256 operand, and TMEM holds G and VB side by side (kColV = kColG + 128)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int kk = 0; kk < LEAF / 16; ++kk) {
              const uint64_t bdesc = sw128_desc(kst + kk * 2048, kLeafBytes / 2, 1024);
              mma_bf16_ts_by(leader, tmem + kColG, wt + 32 * h + 8 * kk, bdesc, id_gv, (h | kk) != 0);
            }
          }
          mma_commit_by(leader, &bars->gv_full);
          // the S buffer and the K/V stage are released only for a later leaf that waits for them: every
          // commit issued is observed before the CTA leaves (an arrival nobody waits for could land after it
          // exited, in shared memory that already belongs to the next CTA on the SM)
          if (j + 2 < nl) mma_commit_by(leader, &bars->s_empty[b]);
          if ((j % kPerStage == kPerStage - 1 || j == nl - 1) && gi + kStages < nst)
            mma_commit_by(leader, &bars->kv_empty[s]);
        }
      }
    }
    // warp 3: nothing (it completes warpgroup 0 for setmaxnreg)
  } else if (warp < 8) {
    // ------------------------------------------------------------------ softmax warpgroup: S -> (lz, W)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 144;");
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t tloc = static_cast<int64_t>(blk) * 128 + row;   // tile index within the chunk
    const bool valid = tloc < tc;
    const float kLog2e = 1.4426950408889634f;
    if (nl > 0) {
      // this row's centre (hi and lo parts, 128 bf16 each) -> TMEM lane `row`; rows past the end are zero
      const int64_t grow = t0 + static_cast<int64_t>(blk) * 128 + row;
      for (int part = 0; part < 2; ++part) {
        const uint4* src = reinterpret_cast<const uint4*>((part ? mu_lo_g : mu_hi_g) + grow * 128);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t r[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 v = grow < nt ? __ldg(src + half * 8 + i) : make_uint4(0u, 0u, 0u, 0u);
            r[4 * i] = v.x;
            r[4 * i + 1] = v.y;
            r[4 * i + 2] = v.z;
            r[4 * i + 3] = v.w;
          }
          tmem_st32(tmem + lane_base + kColMu + 64 * part + 32 * half, r);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->mu_full);
    }
    for (int j = 0; j < nl; ++j) {
      const int b = j & 1;
      const int leaf = l_begin + j;
      if (!mbar_wait(&bars->s_full[b], (j >> 1) & 1, status, abort_flag)) break;
      __syncwarp();
      tc_fence_after();
      float a[LEAF];
      if constexpr (LEAF == 16) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + kColS + 64 * b, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) a[i] = __uint_as_float(r[i]);
      } else {
#pragma unroll
        for (int c = 0; c < LEAF / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + kColS + 64 * b + 32 * c, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) a[32 * c + i] = __uint_as_float(r[i]);
        }
      }
      float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      const float2 sc2 = make_float2(scale, scale);
#pragma unroll
      for (int i = 0; i < LEAF; i += 2) {
        const float2 v = mul2(make_float2(a[i], a[i + 1]), sc2);
        a[i] = v.x;
        a[i + 1] = v.y;
        mxa[(i >> 1) & 3] = max3(mxa[(i >> 1) & 3], v.x, v.y);
      }
      const float m = fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3]));
      float2 zs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 m2 = make_float2(m, m), l2e2 = make_float2(kLog2e, kLog2e);
#pragma unroll
      for (int i = 0; i < LEAF; i += 2) {
        const float2 e = mul2(sub2(make_float2(a[i], a[i + 1]), m2), l2e2);
        a[i] = ex2(e.x);
        a[i + 1] = ex2(e.y);
        zs[(i >> 1) & 3] = add2(zs[(i >> 1) & 3], make_float2(a[i], a[i + 1]));
      }
      const float2 zz = add2(add2(zs[0], zs[1]), add2(zs[2], zs[3]));
      const float z = zz.x + zz.y;
      const float lz = m + logf(z);
      float kw = 0.f;                           // ISO: sum_s e_s |k_s|^2 (divided by z below)
      if constexpr (ISO && LEAF == 64) {
        const float4* kn = reinterpret_cast<const float4*>(smem + kOffKn + (j % kStages) * 256);
        float2 acc2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 c = kn[i];
          acc2[i & 1] = fma2(make_float2(a[4 * i], a[4 * i + 1]), make_float2(c.x, c.y), acc2[i & 1]);
          acc2[i & 1] = fma2(make_float2(a[4 * i + 2], a[4 * i + 3]), make_float2(c.z, c.w), acc2[i & 1]);
        }
        const float2 t = add2(acc2[0], acc2[1]);
        kw = t.x + t.y;
      }
      if (valid) {
        lz_out[tloc * pitch + leaf] = lz;
        if (!isfinite(lz)) flag_status(status, ST_NONFINITE);
      }
      const float rz = 1.0f / z;
      // slot j % 4: the epilogue read slot j - 4 before G/VB(j - 3) began, and S(j) (so this softmax) came
      // after G/VB(j - 2) completed
      if (ISO) reinterpret_cast<float*>(smem + kOffAw)[(j & 3) * 128 + row] = kw * rz;
      // W = w_hi + w_lo as bf16 pairs over this row's S columns (already read): hi in 32 columns, lo in 32
      {
        uint32_t hi[LEAF / 2], lo[LEAF / 2];
#pragma unroll
        for (int i = 0; i < LEAF / 2; ++i) {
          float2 w = mul2(make_float2(a[2 * i], a[2 * i + 1]), make_float2(rz, rz));
          w.x = __uint_as_float(__float_as_uint(w.x) & wmask);     // precision "tf32": the operand value
          w.y = __uint_as_float(__float_as_uint(w.y) & wmask);
          hi[i] = pack_bf16x2(w.x, w.y);
          const float2 lw = sub2(w, make_float2(__uint_as_float(hi[i] << 16), __uint_as_float(hi[i] & 0xFFFF0000u)));
          lo[i] = pack_bf16x2(lw.x, lw.y);
        }
        tmem_st_cols<LEAF / 2>(tmem + lane_base + kColS + 64 * b, hi);
        tmem_st_cols<LEAF / 2>(tmem + lane_base + kColS + 64 * b + 32, lo);
      }
      tmem_st_wait();
      tc_fence_before();
      if (ISO) fence_proxy_async_smem();   // the key norms read above sit in a K/V stage that TMA refills
      mbar_arrive(&bars->w_full[b]);
    }
  } else {
    // ------------------------------------------------------------------ epilogue: G, VB -> g8/sg, vbar
    // warpgroup 2 takes columns 0-63 of G and VB, warpgroup 3 columns 64-127; it overlaps the softmax of
    // the next leaf
    asm volatile("setmaxnreg.inc.sync.aligned.u32 144;");
    const int half = (warp - 8) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t tloc = static_cast<int64_t>(blk) * 128 + row;   // tile index within the chunk
    const bool valid = tloc < tc;
    const bool lead = threadIdx.x == 256;             // issues the TMA stores
    const uint32_t stg = smem_u32(smem + kOffStG), stv = smem_u32(smem + kOffStV);
    float* amx = reinterpret_cast<float*>(smem + kOffAm);
    const uint32_t colg = kColG + 64 * half, colv = kColV + 64 * half;
    for (int j = 0; j < nl; ++j) {
      const int leaf = l_begin + j;
      if (!mbar_wait(&bars->gv_full, j & 1, status, abort_flag)) break;
      __syncwarp();
      tc_fence_after();
      if constexpr (BF) {
        // this half of G and VB (64 columns each) as bf16 pairs; TMEM is released at once
        uint32_t gw[32], vw[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + colg + 32 * c, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i)
            gw[16 * c + i] = pack_bf16x2(__fmul_rn(__uint_as_float(r[2 * i]), scale),
                                         __fmul_rn(__uint_as_float(r[2 * i + 1]), scale));
          tmem_ld32(tmem + lane_base + colv + 32 * c, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) vw[16 * c + i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
        }
        tc_fence_before();
        mbar_arrive(&bars->gv_empty);
        if (lead) {
          bulk_wait_group_read0();
          mbar_arrive(&bars->stg_free);
        }
        if (!mbar_wait(&bars->stg_free, j & 1, status, abort_flag)) break;
        __syncwarp();
        // this half is the 128-byte row of staging box `half` of g and of vbar
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          st_shared_v4(stg + half * (128 * 128) + sw128_off(row, c), gw[4 * c], gw[4 * c + 1], gw[4 * c + 2],
                       gw[4 * c + 3]);
          st_shared_v4(stv + half * (128 * 128) + sw128_off(row, c), vw[4 * c], vw[4 * c + 1], vw[4 * c + 2],
                       vw[4 * c + 3]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->stg_full);
        if (lead) {
          if (!mbar_wait(&bars->stg_full, j & 1, status, abort_flag)) break;
          tma_store_3d(&tm_g8, smem + kOffStG, 0, leaf, blk * 128);
          tma_store_3d(&tm_g8, smem + kOffStG + 128 * 128, 64, leaf, blk * 128);
          tma_store_3d(&tm_vb, smem + kOffStV, 0, leaf, blk * 128);
          tma_store_3d(&tm_vb, smem + kOffStV + 128 * 128, 64, leaf, blk * 128);
          bulk_commit_group();
        }
        continue;
      }
      if constexpr (FP8) {
        // this half of G and its abs-max, then the abs-max of this half of VB (read twice from TMEM, so that
        // only G stays in registers); the halves of a row exchange both through shared memory
        uint32_t gr[64];
        tmem_ld32(tmem + lane_base + colg, *reinterpret_cast<uint32_t(*)[32]>(gr));
        tmem_ld32(tmem + lane_base + colg + 32, *reinterpret_cast<uint32_t(*)[32]>(gr + 32));
        tmem_ld_wait();
        float ama[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 64; i += 2)
          ama[(i >> 1) & 3] = max3(ama[(i >> 1) & 3], fabsf(__uint_as_float(gr[i])), fabsf(__uint_as_float(gr[i + 1])));
        float am = __fmul_rn(fmaxf(fmaxf(ama[0], ama[1]), fmaxf(ama[2], ama[3])), scale);
        float vam = 0.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + colv + 32 * c, r);
          tmem_ld_wait();
          float vm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int i = 0; i < 32; i += 2)
            vm[(i >> 1) & 3] = max3(vm[(i >> 1) & 3], fabsf(__uint_as_float(r[i])), fabsf(__uint_as_float(r[i + 1])));
          vam = fmaxf(vam, fmaxf(fmaxf(vm[0], vm[1]), fmaxf(vm[2], vm[3])));
        }
        float* amv = reinterpret_cast<float*>(smem + kOffB2);
        amx[((j & 1) * 2 + half) * 128 + row] = am;
        amv[((j & 1) * 2 + half) * 128 + row] = vam;
        named_bar_sync(1 + quarter, 64);
        am = fmaxf(am, amx[((j & 1) * 2 + (half ^ 1)) * 128 + row]);
        vam = fmaxf(vam, amv[((j & 1) * 2 + (half ^ 1)) * 128 + row]);
        const float sgv = fmaxf(__fmul_rn(am, 1.0f / 448.0f), 1e-30f);
        const float svv = fmaxf(__fmul_rn(vam, 1.0f / 448.0f), 1e-30f);
        if (valid && half == 0) {
          sg_out[tloc * pitch + leaf] = sgv;
          sv_out[tloc * pitch + leaf] = svv;
        }
        const float2 sc2 = make_float2(scale, scale);
        const float rg = __frcp_rn(sgv), rv = __frcp_rn(svv);
        const float2 rg2 = make_float2(rg, rg), rv2 = make_float2(rv, rv);
        uint32_t gw[16], vw[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 ga = mul2(make_float2(__uint_as_float(gr[4 * i]), __uint_as_float(gr[4 * i + 1])), sc2);
          const float2 gb = mul2(make_float2(__uint_as_float(gr[4 * i + 2]), __uint_as_float(gr[4 * i + 3])), sc2);
          // g / sg: g * (1 / sg), or per value with div.full.f32 like the reference's Triton kernel (tdiv)
          const float2 a = TDIV ? make_float2(div_full(ga.x, sgv), div_full(ga.y, sgv)) : mul2(ga, rg2);
          const float2 b = TDIV ? make_float2(div_full(gb.x, sgv), div_full(gb.y, sgv)) : mul2(gb, rg2);
          gw[i] = f32x2_to_e4m3x2(a.x, a.y) | (f32x2_to_e4m3x2(b.x, b.y) << 16);
        }
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + colv + 32 * c, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 va = make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]));
            const float2 vb2 = make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
            const float2 a = TDIV ? make_float2(div_full(va.x, svv), div_full(va.y, svv)) : mul2(va, rv2);
            const float2 b = TDIV ? make_float2(div_full(vb2.x, svv), div_full(vb2.y, svv)) : mul2(vb2, rv2);
            vw[8 * c + i] = f32x2_to_e4m3x2(a.x, a.y) | (f32x2_to_e4m3x2(b.x, b.y) << 16);
          }
        }
        tc_fence_before();
        mbar_arrive(&bars->gv_empty);
        if (lead) {
          bulk_wait_group_read0();
          mbar_arrive(&bars->stg_free);
        }
        if (!mbar_wait(&bars->stg_free, j & 1, status, abort_flag)) break;
        __syncwarp();
        // this half is the 16-byte chunks 4 half .. 4 half + 3 of the 128-byte code rows of g and vbar
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          st_shared_v4(stg + sw128_off(row, 4 * half + c), gw[4 * c], gw[4 * c + 1], gw[4 * c + 2], gw[4 * c + 3]);
          st_shared_v4(stv + sw128_off(row, 4 * half + c), vw[4 * c], vw[4 * c + 1], vw[4 * c + 2], vw[4 * c + 3]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->stg_full);
        if (lead) {
          if (!mbar_wait(&bars->stg_full, j & 1, status, abort_flag)) break;
          tma_store_3d(&tm_g8, smem + kOffStG, 0, leaf, blk * 128);
          tma_store_3d(&tm_vb, smem + kOffStV, 0, leaf, blk * 128);
          bulk_commit_group();
        }
        continue;
      }
      // drain this half of G (raw) and VB (as bf16 pairs) into registers and release TMEM at once, so the
      // next leaf's G/VB MMAs overlap the quantisation below
      uint32_t gr[64];
      tmem_ld32(tmem + lane_base + colg, *reinterpret_cast<uint32_t(*)[32]>(gr));
      tmem_ld32(tmem + lane_base + colg + 32, *reinterpret_cast<uint32_t(*)[32]>(gr + 32));
      uint32_t vbw[32];
      {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + colv, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) vbw[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
        tmem_ld32(tmem + lane_base + colv + 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) vbw[16 + i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
      }
      float aw = 0.f, b2 = 0.f;                 // ISO: sum w |k|^2 of this row, this half's |G|^2
      if (ISO) {
        aw = reinterpret_cast<const float*>(smem + kOffAw)[(j & 3) * 128 + row];
        float2 s2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          const float2 gg = make_float2(__uint_as_float(gr[i]), __uint_as_float(gr[i + 1]));
          s2[(i >> 1) & 1] = fma2(gg, gg, s2[(i >> 1) & 1]);
        }
        const float2 t = add2(s2[0], s2[1]);
        b2 = t.x + t.y;
      }
      tc_fence_before();
      mbar_arrive(&bars->gv_empty);
      // abs-max of g = scale * G, as scale * max |G| (scale > 0 and rounding is monotonic, so this is the
      // maximum of the rounded products); the other half of the row comes through shared memory
      // (buffered by leaf parity)
      float ama[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 64; i += 2)
        ama[(i >> 1) & 3] = max3(ama[(i >> 1) & 3], fabsf(__uint_as_float(gr[i])), fabsf(__uint_as_float(gr[i + 1])));
      float am = __fmul_rn(fmaxf(fmaxf(ama[0], ama[1]), fmaxf(ama[2], ama[3])), scale);
      amx[((j & 1) * 2 + half) * 128 + row] = am;
      if (ISO) reinterpret_cast<float*>(smem + kOffB2)[((j & 1) * 2 + half) * 128 + row] = b2;
      named_bar_sync(1 + quarter, 64);
      am = fmaxf(am, amx[((j & 1) * 2 + (half ^ 1)) * 128 + row]);
      if (ISO && half == 0) {
        const float gg = b2 + reinterpret_cast<const float*>(smem + kOffB2)[((j & 1) * 2 + 1) * 128 + row];
        const float tr = __fmul_rn(__fmul_rn(scale, scale), __fsub_rn(aw, gg));
        if (valid) cv_out[tloc * pitch + leaf] = __fmul_rn(0.5f / 128.0f, fmaxf(tr, 0.f));
      }
      am = fmaxf(am, 1e-30f);
      const float sgv = __fmul_rn(am, 1.0f / 127.0f);
      // the factor 127 / am: IEEE, or div.full.f32 like the reference's Triton kernel (tdiv)
      const float rr = TDIV ? div_full(127.0f, am) : __fdiv_rn(127.0f, am);
      if (valid && half == 0) sg_out[tloc * pitch + leaf] = sgv;
      // INT8 codes
      uint32_t gw[16];
      const float2 sc2 = make_float2(scale, scale), rr2 = make_float2(rr, rr);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint2 c01 = half_away_codes2(mul2(mul2(make_float2(__uint_as_float(gr[4 * i]), __uint_as_float(gr[4 * i + 1])), sc2), rr2));
        const uint2 c23 = half_away_codes2(mul2(mul2(make_float2(__uint_as_float(gr[4 * i + 2]), __uint_as_float(gr[4 * i + 3])), sc2), rr2));
        gw[i] = __byte_perm(__byte_perm(c01.x, c01.y, 0x0040), __byte_perm(c23.x, c23.y, 0x0040), 0x5410);
      }
      // the previous TMA stores must have finished reading the staging buffers
      if (lead) {
        bulk_wait_group_read0();
        mbar_arrive(&bars->stg_free);
      }
      if (!mbar_wait(&bars->stg_free, j & 1, status, abort_flag)) break;
      __syncwarp();
      // g8: this half is the 16-byte chunks 4 half .. 4 half + 3 of the 128-byte row
#pragma unroll
      for (int c = 0; c < 4; ++c)
        st_shared_v4(stg + sw128_off(row, 4 * half + c), gw[4 * c], gw[4 * c + 1], gw[4 * c + 2], gw[4 * c + 3]);
      // vbar: this half is the 128-byte row of staging box `half`
#pragma unroll
      for (int c = 0; c < 8; ++c)
        st_shared_v4(stv + half * (128 * 128) + sw128_off(row, c), vbw[4 * c], vbw[4 * c + 1], vbw[4 * c + 2],
                     vbw[4 * c + 3]);
      fence_proxy_async_smem();
      mbar_arrive(&bars->stg_full);
      if (lead) {
        if (!mbar_wait(&bars->stg_full, j & 1, status, abort_flag)) break;
        tma_store_3d(&tm_g8, smem + kOffStG, 0, leaf, blk * 128);
        tma_store_3d(&tm_vb, smem + kOffStV, 0, leaf, blk * 128);
        tma_store_3d(&tm_vb, smem + kOffStV + 128 * 128, 64, leaf, blk * 128);
        bulk_commit_group();
      }
    }
    if (lead) bulk_wait_group0();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

int launch_leaf_stats(const LeafStatsMaps& maps, float* sg, float* lz, int64_t pitch, int64_t t0, int64_t tc, int nb,
                      int leaf, float scale, const float* kn2, float* cv, float* sv, int* status, int num_sms,
                      bool tf32, bool tdiv, cudaStream_t st, bool bf16_state) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    bool ok = true;
    for (auto k : {leaf_stats_kernel<false, false, false, 64>, leaf_stats_kernel<true, false, false, 64>,
                   leaf_stats_kernel<false, true, false, 64>, leaf_stats_kernel<false, false, true, 64>,
                   leaf_stats_kernel<true, false, true, 64>, leaf_stats_kernel<false, true, true, 64>,
                   leaf_stats_kernel<false, false, false, 32>, leaf_stats_kernel<false, false, true, 32>,
                   leaf_stats_kernel<false, false, false, 16>, leaf_stats_kernel<false, false, true, 16>})
      ok = ok && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SLay<false>::kSmemBytes) ==
                     cudaSuccess;
    ok = ok && cudaFuncSetAttribute(leaf_stats_kernel<false, false, false, 64, true>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, SLay<true>::kSmemBytes) == cudaSuccess;
    if (!ok) return HTRC_ERR_CUDA;
    attr_done[dev] = true;
  }
  if (sv != nullptr && cv != nullptr) return HTRC_ERR_UNSUPPORTED;
  if (leaf != 64 && leaf != 32 && leaf != 16) return HTRC_ERR_UNSUPPORTED;
  if (leaf != 64 && (sv != nullptr || cv != nullptr)) return HTRC_ERR_UNSUPPORTED;
  if (bf16_state && (leaf != 64 || sv != nullptr || cv != nullptr)) return HTRC_ERR_UNSUPPORTED;
  const int bx = static_cast<int>((tc + 127) / 128);
  int by = max(1, num_sms / bx);                    // one wave: bx * by <= SMs
  by = min(by, nb);
  const int per_stage = 64 / leaf;                  // a CTA's leaf range covers whole K/V stages
  int lpc = (nb + by - 1) / by;
  lpc = (lpc + per_stage - 1) / per_stage * per_stage;
  by = (nb + lpc - 1) / lpc;
  decltype(&leaf_stats_kernel<false, false, false, 64>) kernel;
  if (bf16_state)
    kernel = leaf_stats_kernel<false, false, false, 64, true>;     // no division in its epilogue
  else if (leaf == 32)
    kernel = tdiv ? leaf_stats_kernel<false, false, true, 32> : leaf_stats_kernel<false, false, false, 32>;
  else if (leaf == 16)
    kernel = tdiv ? leaf_stats_kernel<false, false, true, 16> : leaf_stats_kernel<false, false, false, 16>;
  else
    kernel = tdiv ? (sv != nullptr ? leaf_stats_kernel<false, true, true, 64>
                                   : (cv != nullptr ? leaf_stats_kernel<true, false, true, 64>
                                                    : leaf_stats_kernel<false, false, true, 64>))
                  : (sv != nullptr ? leaf_stats_kernel<false, true, false, 64>
                                   : (cv != nullptr ? leaf_stats_kernel<true, false, false, 64>
                                                    : leaf_stats_kernel<false, false, false, 64>));
  const uint32_t smem = bf16_state ? SLay<true>::kSmemBytes : SLay<false>::kSmemBytes;
  kernel<<<dim3(bx, by), kThreads, smem, st>>>(maps.mu_hi, maps.mu_lo, maps.nt, maps.k, maps.v, maps.g8, maps.vb,
                                                     sg, lz, pitch, t0, tc, nb, lpc, scale, kn2, cv, sv, status,
                                                     tf32 ? kTf32Mask : 0xFFFFFFFFu);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

}  // namespace htrc
