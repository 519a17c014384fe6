// The fp8 (e4m3) state path of the flat HTRC operator (h3/htrc_flat_triton.py with FP8=1, DOT=1: the
// reference's store="fp8", dot="bf16"): row-max near-leaf selection and the fused far + near tile attention.
//
// The far-field state is e4m3 codes with per-(centre, leaf) row scales: g codes with sg, vbar codes with sv
// (written by the leaf-statistics kernel).  e4m3 values are exact in fp16, so the kernels stage the codes
// by TMA, convert them on chip into fp16 operands in the 128-byte-swizzled UMMA layout (one cvt per pair
// of codes; measured faster here than placing the code bits into fp16 position with integer ops) and run
// kind::f16 MMAs with float32 accumulation:
//   selection (:214-254):  SEL[t, l] = max_r (fp16(q_r - mu) . g_l) * sg_l + lz_l
//   far field (:118-160):  logit = (fp16(q_r - mu) . g_l) * sg_l + lz_l, value weight fp16(p * sv_l) on g's
//                          vbar codes (the normaliser sums p, not p * sv)
//   near field (:161-186): logit = (bf16 q_r . bf16 k_j) * scale, weight bf16(p) on bf16 v_j
// with one float32 online softmax per query row.  The state stays in HBM as one byte per value.
#include "common.cuh"
#include "kernels.cuh"

namespace htrc {

namespace {
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// rows x 128 e4m3 codes (plain 128-byte rows at `raw`) -> fp16 values as two 128-byte-swizzled K-major
// halves [2][rows][64] at `dst` (half stride rows * 128 bytes).  The nthreads threads of the caller split
// the 8-byte chunks: consecutive threads read consecutive chunks; the 16-byte stores of eight consecutive
// threads fill one swizzled 128-byte row.
template <int ROWS, int NTHREADS>
__device__ __forceinline__ void codes_to_f16(const uint8_t* raw, uint32_t dst, int tid) {
#pragma unroll 4
  for (int k = 0; k < ROWS * 16 / NTHREADS; ++k) {
    const int i = tid + NTHREADS * k;
    const int row = i >> 4, c8 = i & 15;
    const uint2 w = *reinterpret_cast<const uint2*>(raw + row * 128 + c8 * 8);
    st_shared_v4(dst + (c8 >> 3) * (ROWS * 128) + sw128_off(row, c8 & 7), e4m3x2_to_f16x2(w.x),
                 e4m3x2_to_f16x2(w.x >> 16), e4m3x2_to_f16x2(w.y), e4m3x2_to_f16x2(w.y >> 16));
  }
}
// In place: 64 rows x 128 e4m3 codes landed by TMA with the 128-byte swizzle in the upper half of a 16 KB
// operand (row r's 16-byte chunk k at dst + 8192 + 128 r + 16 (k ^ (r & 7))) -> fp16 values as two
// 128-byte-swizzled halves [2][64][64] at dst.  Thread `row` converts its row: it reads the whole row of
// codes first, so its writes to half 1 (the same 128 bytes) cannot overwrite codes not yet read, and no
// other thread reads them.
__device__ __forceinline__ void codes_to_f16_in_place(uint32_t dst, int row) {
  const uint32_t sw = static_cast<uint32_t>(row & 7);
  const uint32_t raw = dst + 8192 + static_cast<uint32_t>(row) * 128;
  uint32_t c[8][4];
#pragma unroll
  for (int k = 0; k < 8; ++k)
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(c[k][0]), "=r"(c[k][1]), "=r"(c[k][2]), "=r"(c[k][3])
                 : "r"(raw + ((static_cast<uint32_t>(k) ^ sw) << 4))
                 : "memory");
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    // codes 16k .. 16k + 15 are dims 16k .. 16k + 15: half k / 4, 16-byte chunks 2 (k % 4) and 2 (k % 4) + 1
    const uint32_t base = dst + static_cast<uint32_t>(k >> 2) * 8192 + static_cast<uint32_t>(row) * 128;
    const uint32_t c0 = 2u * static_cast<uint32_t>(k & 3);
    st_shared_v4(base + ((c0 ^ sw) << 4), e4m3x2_to_f16x2(c[k][0]), e4m3x2_to_f16x2(c[k][0] >> 16),
                 e4m3x2_to_f16x2(c[k][1]), e4m3x2_to_f16x2(c[k][1] >> 16));
    st_shared_v4(base + (((c0 + 1) ^ sw) << 4), e4m3x2_to_f16x2(c[k][2]), e4m3x2_to_f16x2(c[k][2] >> 16),
                 e4m3x2_to_f16x2(c[k][3]), e4m3x2_to_f16x2(c[k][3] >> 16));
  }
}
}  // namespace

// ================================================================================================
// Row-max selection.  Per block of 128 leaves: C = G_block (M=128 leaves, K=128, fp16 from the codes) x
// DQ_tile^T (N=64 rows, fp16) into TMEM; the thread owning TMEM lane l reduces its 64 columns.  One CTA per
// tile, two CTAs per SM; warp 0 loads (TMA), warp 1 issues the MMAs, warps 2-5 reduce block j while eight
// warps convert the next block.
// Groups of G tiles read state row t / G (the routing kernel takes the maximum over the group's rows).
namespace {
namespace rmx {
constexpr int kStages = 3;                              // raw code stages: the HBM stream in flight
constexpr int kOpStages = 1;                            // converted fp16 blocks (two CTAs share an SM)
constexpr int kConv = 256;                              // converting threads (warps 6 ..)
constexpr int kThreads = 192 + kConv;
constexpr uint32_t kRawBytes = 128 * 128;               // 128 leaves x 128 codes
constexpr uint32_t kRawStage = kRawBytes + 1024;        // + sg[128], lz[128]
constexpr uint32_t kOpBytes = 2 * 128 * 128;            // fp16 g block: 2 halves x 128 rows x 128 B
constexpr uint32_t kOffDq = 0;                          // fp16 offsets of the tile: 2 halves x 64 rows x 128 B
constexpr uint32_t kOffRaw = 16384;
constexpr uint32_t kOffOp = kOffRaw + kStages * kRawStage;
constexpr uint32_t kOffBar = kOffOp + kOpStages * kOpBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;
constexpr uint32_t kTmemCols = 128;
static_assert(kOffOp % 1024 == 0, "swizzled operands need 1024-byte alignment");

struct Bars {
  uint64_t dq_full;
  uint64_t raw_full[kStages];    // TMA: codes, sg, lz
  uint64_t raw_empty[kStages];   // the converting threads read the codes, the 128 reducing threads sg / lz
  uint64_t op_full[kOpStages];   // the converting threads wrote the fp16 block
  uint64_t op_empty[kOpStages];  // MMA commit
  uint64_t acc_full[2];
  uint64_t acc_empty[2];         // the 128 reducing threads drained the accumulator
  uint32_t tmem_base;
  int abort_flag;
};
}  // namespace rmx
}  // namespace

__global__ void __launch_bounds__(rmx::kThreads, 2)
    rowmax_fp8_kernel(const __grid_constant__ CUtensorMap tm_dqh, const __grid_constant__ CUtensorMap tm_graw,
                      const __grid_constant__ CUtensorMap tm_sg, const __grid_constant__ CUtensorMap tm_lz,
                      float* __restrict__ sel, int64_t pitch, int64_t t0, int nb, int group, int* status) {
  using namespace rmx;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tloc = blockIdx.x;
  const int srow = tloc / group;
  const int64_t tg = t0 + tloc;
  const int nblk = (nb + 127) / 128;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->dq_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->raw_full[s], 1);
      mbar_init(&bars->raw_empty[s], kConv + 128);
    }
    for (int s = 0; s < kOpStages; ++s) {
      mbar_init(&bars->op_full[s], kConv);
      mbar_init(&bars->op_empty[s], 1);
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
      const uint64_t pol = policy_evict_first();
      mbar_arrive_expect_tx(&bars->dq_full, 2 * 64 * 128);
      tma_load_3d(smem + kOffDq, &tm_dqh, &bars->dq_full, 0, static_cast<int>(tg * 64), 0, pol);
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&bars->raw_empty[s], ((j / kStages) - 1) & 1, status, abort_flag)) break;
        uint8_t* st = smem + kOffRaw + s * kRawStage;
        mbar_arrive_expect_tx(&bars->raw_full[s], kRawBytes + 1024);
        tma_load_3d(st, &tm_graw, &bars->raw_full[s], 0, j * 128, srow, pol);
        tma_load_2d(st + kRawBytes, &tm_sg, &bars->raw_full[s], j * 128, srow, pol);
        tma_load_2d(st + kRawBytes + 512, &tm_lz, &bars->raw_full[s], j * 128, srow, pol);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, 64, false, false);
      const uint32_t dq = smem_u32(smem + kOffDq);
      bool ok = mbar_wait(&bars->dq_full, 0, status, abort_flag);
      int nmma = 0;                   // blocks whose MMAs were issued (and committed)
      for (int j = 0; ok && j < nblk; ++j) {
        const int s = j % kOpStages, b = j & 1;
        if (!mbar_wait(&bars->op_full[s], (j / kOpStages) & 1, status, abort_flag)) break;
        if (j >= 2 && !mbar_wait(&bars->acc_empty[b], ((j >> 1) - 1) & 1, status, abort_flag)) break;
        tc_fence_after();
        const uint32_t op = smem_u32(smem + kOffOp + s * kOpBytes);   // s: the op stage
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(tmem + 64 * b, sw128_desc(op + h * (kOpBytes / 2) + kk * 32, 16, 1024),
                     sw128_desc(dq + h * (64 * 128) + kk * 32, 16, 1024), idesc, (h | kk) != 0);
        mma_commit(&bars->acc_full[b]);
        mma_commit(&bars->op_empty[s]);
        nmma = j + 1;
      }
      // the operand-stage release signals of the last blocks have no waiter: let them land before the CTA leaves
      drain_ring<false>(bars->op_empty, kOpStages, nmma, status, abort_flag);
    }
  } else if (warp < 6) {
    // reduce block j: sel over the tile's 64 rows for the leaf of this thread's TMEM lane
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;                 // leaf within the block (TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    for (int j = 0; j < nblk; ++j) {
      const int s = j % kStages, b = j & 1;
      if (!mbar_wait_warp(&bars->raw_full[s], (j / kStages) & 1, status, abort_flag)) break;
      const uint8_t* st = smem + kOffRaw + s * kRawStage;
      const float sgl = reinterpret_cast<const float*>(st + kRawBytes)[r];
      const float lzl = reinterpret_cast<const float*>(st + kRawBytes + 512)[r];
      fence_proxy_async_smem();          // the TMA refill (async proxy) must not overtake these generic reads
      mbar_arrive(&bars->raw_empty[s]);
      if (!mbar_wait_warp(&bars->acc_full[b], (j >> 1) & 1, status, abort_flag)) break;
      __syncwarp();
      tc_fence_after();
      uint32_t d0[32], d1[32];
      tmem_ld32(tmem + lane_base + 64 * b, d0);
      tmem_ld32(tmem + lane_base + 64 * b + 32, d1);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&bars->acc_empty[b]);
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      const float2 s2 = make_float2(sgl, sgl);
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float2 a = mul2(make_float2(__uint_as_float(d0[i]), __uint_as_float(d0[i + 1])), s2);
        const float2 c = mul2(make_float2(__uint_as_float(d1[i]), __uint_as_float(d1[i + 1])), s2);
        mx[(i >> 1) & 1] = max3(mx[(i >> 1) & 1], a.x, a.y);
        mx[2 + ((i >> 1) & 1)] = max3(mx[2 + ((i >> 1) & 1)], c.x, c.y);
      }
      const int leaf = j * 128 + r;
      if (leaf < nb)
        sel[static_cast<int64_t>(tloc) * pitch + leaf] = __fadd_rn(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), lzl);
    }
  } else {
    // convert the codes of block j into the fp16 operand of stage j % kOpStages
    const int tid = threadIdx.x - 192;
    for (int j = 0; j < nblk; ++j) {
      const int s = j % kStages, o = j % kOpStages;
      if (!mbar_wait_warp(&bars->raw_full[s], (j / kStages) & 1, status, abort_flag)) break;
      if (j >= kOpStages && !mbar_wait_warp(&bars->op_empty[o], ((j / kOpStages) - 1) & 1, status, abort_flag))
        break;
      codes_to_f16<128, kConv>(smem + kOffRaw + s * kRawStage, smem_u32(smem + kOffOp + o * kOpBytes), tid);
      fence_proxy_async_smem();
      mbar_arrive(&bars->op_full[o]);
      mbar_arrive(&bars->raw_empty[s]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

int launch_rowmax_fp8(const RowmaxFp8Maps& maps, float* sel, int64_t pitch, int64_t t0, int64_t tc, int nb, int group,
                      int* status, cudaStream_t st) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(rowmax_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, rmx::kSmemBytes) !=
        cudaSuccess)
      return HTRC_ERR_CUDA;
    attr_done[dev] = true;
  }
  rowmax_fp8_kernel<<<static_cast<unsigned>(tc), rmx::kThreads, rmx::kSmemBytes, st>>>(maps.dqh, maps.graw, maps.sg, maps.lz, sel,
                                                                             pitch, t0, nb, group > 1 ? group : 1,
                                                                             status);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

// ================================================================================================
// Tile attention, in two passes over the tiles of a chunk that share one kernel body:
// (BF: the bf16 state, store="bf16", h3/htrc_flat_triton.py:139-140 and :154 with DOT=1 -- the far pass lands g and
// vbar as bf16 operands directly, logit = (bf16 dq . g) + lz and weights bf16(p); the converting warps only hand
// the landed blocks on.  The near pass is the same for both states.)
//   FAR:  the far field alone (blocks of 64 leaves of the tile's state, fp16 from the codes), written as one
//         partial (acc[128], m, l) per query row, like the tail partial;
//   NEAR: the routed leaves (bf16 keys and values, by TMA), merged in the epilogue with the far partial and
//         the tail partial into the normalised output and log-Z.
// Splitting keeps each pass's shared memory for its own rings: FAR lands the codes of a block in the upper
// half of its fp16 operand slot and converts them in place, three pairs of g and of vbar blocks in flight;
// NEAR holds three pairs of keys and of values in flight.  The merge is the exact
// (max, sum) combination the reference applies to its splits (:257-273).
//
// Within a pass: one CTA per 64-row tile; steps of 64 columns taken in pairs: the MMAs of steps 2p and
// 2p + 1 are M=64 each, step 2p in TMEM lanes {0..15} + 32k and step 2p + 1 at lane offset 16, so every
// softmax thread owns one (query row, step parity) of S, P and O and all 128 threads of a warpgroup work
// on every pair.  Two warpgroups take alternate pairs, each with its own O accumulator (two per row: one
// per step parity) and running (max, sum); the lazy maximum is rescaled only when it grew by more than 2^8.
// The FAR pass pads its steps to an even count (the extra block lies past nb and is masked).
//
// Warp roles.  Both passes: warp 0 X producer (tile rows; FAR: block parameters and g codes, NEAR:
// routed keys), warp 1 PV issuer (+ TMEM owner), warp 2 QK issuer, warps 4-7 and 8-11 the softmax
// warpgroups.  FAR: warp 3 per-column constants, warps 12-13 convert g codes, warps 14-15 load (two pairs
// ahead) and convert vbar codes (512 threads, warpgroup-aligned setmaxnreg).  NEAR: warp 3 loads the
// routed values (384 threads).
namespace {
namespace tfx {
constexpr uint32_t kOpBytes = 16384;                     // 2 halves x 64 rows x 128 B
constexpr uint32_t kRawBytes = 64 * 128;                 // 64 leaves x 128 codes
constexpr int kMaxKx = 1024;
constexpr float kRescale = 8.0f;
constexpr uint32_t kColS = 0;       // S/P buffer b (= pair % 4) at 64 b; P uses its first 32 columns
constexpr uint32_t kColO = 256;     // O[g] at 256 + 128 g (step parity by lane offset 0 / 16)
constexpr uint32_t kTmemCols = 512;

template <bool FAR>
struct Cfg {
  static constexpr int kThreads = FAR ? 512 : 384;
  static constexpr int kXP = 3;                          // X ring: pairs
  static constexpr int kYP = 3;                          // Y ring: pairs
  static constexpr uint32_t kXSub = kOpBytes + (FAR ? 1024 : 0);   // far: + lz[64], sg[64], sv[64], excl[64]
  static constexpr uint32_t kOffQ = 0;                   // FAR: fp16 offsets; NEAR: bf16 rows
  static constexpr uint32_t kOffX = kOpBytes;            // [pair slot][step parity] x kXSub
  static constexpr uint32_t kOffY = kOffX + 2 * kXP * kXSub;
  static constexpr uint32_t kOffCC = kOffY + 2 * kYP * kOpBytes;  // FAR: [warpgroup][parity][64] float2
  static constexpr uint32_t kOffCS = kOffCC + (FAR ? 4 * 64 * 8 : 0);   // FAR: sv
  static constexpr uint32_t kOffEpi = kOffCS + (FAR ? 4 * 64 * 4 : 0);  // m, l of warpgroup 1
  static constexpr uint32_t kOffIdx = kOffEpi + 2 * 128 * 4;           // NEAR: [kMaxKx] uint16
  static constexpr uint32_t kOffBar = kOffIdx + (FAR ? 0 : kMaxKx * 2);
  static constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;
  static_assert(kOffX % 1024 == 0 && kXSub % 1024 == 0 && kOffY % 1024 == 0, "swizzled operands: 1024-byte alignment");
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

struct Bars {
  uint64_t qd_full;
  uint64_t x_full[3];     // NEAR: X producer (arrive + bytes); FAR: 64 g converter threads
  uint64_t x_empty[3];    // QK commit [+ 32 constant lanes]
  uint64_t y_full[3];     // NEAR: Y producer (arrive + bytes); FAR: 64 vbar converter threads
  uint64_t xr_full[3];    // FAR: g codes and block parameters landed (X producer: arrive + bytes)
  uint64_t yr_full[3];    // FAR: vbar codes landed (vbar loader: arrive + bytes)
  uint64_t cc_full[2];    // 32 constant lanes
  uint64_t cc_empty[2];   // 128 softmax threads of the pair's warpgroup
  uint64_t s_full[4];     // QK of the pair done
  uint64_t p_full[4];     // 128 softmax threads wrote P (and rescaled O if needed)
  uint64_t pv_done[4];    // PV of the pair done
  uint64_t epi1;          // 128 threads of warpgroup 1 published (m, l)
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Bars) <= 512, "barrier block");
}  // namespace tfx
}  // namespace

template <int TROWS, bool FAR, bool BF = false>
__global__ void __launch_bounds__(tfx::Cfg<FAR>::kThreads, 1)
    tile_fp8_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_graw,
                    const __grid_constant__ CUtensorMap tm_vraw, const __grid_constant__ CUtensorMap tm_lz,
                    const __grid_constant__ CUtensorMap tm_sg, const __grid_constant__ CUtensorMap tm_sv,
                    const __grid_constant__ CUtensorMap tm_excl, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const int32_t* __restrict__ idx, int kx, int nb,
                    int64_t n, int64_t t0, int group, float scale, const float* __restrict__ tail_part,
                    const int32_t* __restrict__ perm, float* __restrict__ far_part, float* __restrict__ out,
                    float* __restrict__ lse, int* status) {
  using namespace tfx;
  using C = Cfg<FAR>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + C::kOffBar);
  uint16_t* idx_s = reinterpret_cast<uint16_t*>(smem + C::kOffIdx);
  float2* cc = reinterpret_cast<float2*>(smem + C::kOffCC);
  float* cs = reinterpret_cast<float*>(smem + C::kOffCS);
  float* epi = reinterpret_cast<float*>(smem + C::kOffEpi);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tloc = blockIdx.x;
  const int srow = tloc / group;            // state row of this tile
  // FAR: blocks of 64 leaves, padded to an even count; NEAR: the routed leaves
  const int total = FAR ? ((nb + 127) / 128) * 2 : kx;
  const int np = (total + 1) / 2;           // pairs of steps
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->qd_full, 1);
    for (int s = 0; s < C::kXP; ++s) {
      mbar_init(&bars->x_full[s], FAR ? 64 : 1);
      mbar_init(&bars->x_empty[s], FAR ? 1 + 32 : 1);
      mbar_init(&bars->xr_full[s], 1);
    }
    for (int s = 0; s < C::kYP; ++s) {
      mbar_init(&bars->y_full[s], FAR ? 64 : 1);
      mbar_init(&bars->yr_full[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->cc_full[s], 32);
      mbar_init(&bars->cc_empty[s], 128);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->p_full[b], 128);
      mbar_init(&bars->pv_done[b], 1);
    }
    mbar_init(&bars->epi1, 128);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (!FAR && warp == 0) {
    // routed leaves of the tile's state row -> shared memory, range-checked
    const int32_t* src = idx + static_cast<int64_t>(srow) * kx;
    for (int e = lane; e < kx; e += 32) {
      int leaf = __ldg(src + e);
      if (leaf < 0 || leaf >= nb) {
        flag_status(status, ST_BAD_INDEX);
        leaf = 0;
      }
      idx_s[e] = static_cast<uint16_t>(leaf);
    }
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  auto xsub = [&](int p, int x) { return smem + C::kOffX + ((p % C::kXP) * 2 + x) * C::kXSub; };
  auto ysub = [&](int p, int x) { return smem + C::kOffY + ((p % C::kYP) * 2 + x) * kOpBytes; };

  if (warp < 4) {
    if constexpr (FAR) asm volatile("setmaxnreg.dec.sync.aligned.u32 64;");
    const uint32_t leader = elect_one();
    if (warp == 0) {
      // ---------------------------------------------------------------- X producer
      const uint64_t pol_stream = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      if (leader) {
        mbar_arrive_expect_tx(&bars->qd_full, kOpBytes);
        tma_load_3d(smem + C::kOffQ, &tm_q, &bars->qd_full, 0, static_cast<int>((t0 + tloc) * 64), 0, pol_stream);
      }
      for (int p = 0; p < np; ++p) {
        const int xs = p % C::kXP;
        if (p >= C::kXP && !mbar_wait_warp(&bars->x_empty[xs], ((p / C::kXP) - 1) & 1, status, abort_flag)) break;
        if (leader) {
          uint32_t tx = 0;
          for (int x = 0; x < 2; ++x)
            if (2 * p + x < total) tx += FAR ? (BF ? kOpBytes + 256 + 64 : kRawBytes + 3 * 256 + 64) : kOpBytes;
          uint64_t* bar = FAR ? &bars->xr_full[xs] : &bars->x_full[xs];
          mbar_arrive_expect_tx(bar, tx);
          for (int x = 0; x < 2; ++x) {
            const int j = 2 * p + x;
            if (j >= total) continue;
            uint8_t* xp = xsub(p, x);
            if constexpr (FAR && BF) {
              // the block's bf16 g as its operand (both halves), lz and the exclusion bytes
              tma_load_4d(xp, &tm_graw, bar, 0, j * 64, 0, srow, pol_stream);
              tma_load_2d(xp + kOpBytes, &tm_lz, bar, j * 64, srow, pol_stream);
              tma_load_2d(xp + kOpBytes + 768, &tm_excl, bar, j * 64, srow, pol_stream);
            } else if constexpr (FAR) {
              // the block's g codes into the upper half of its operand slot (converted there in place)
              tma_load_3d(xp + kOpBytes / 2, &tm_graw, bar, 0, j * 64, srow, pol_stream);
              tma_load_2d(xp + kOpBytes, &tm_lz, bar, j * 64, srow, pol_stream);
              tma_load_2d(xp + kOpBytes + 256, &tm_sg, bar, j * 64, srow, pol_stream);
              tma_load_2d(xp + kOpBytes + 512, &tm_sv, bar, j * 64, srow, pol_stream);
              tma_load_2d(xp + kOpBytes + 768, &tm_excl, bar, j * 64, srow, pol_stream);
            } else {
              tma_load_3d(xp, &tm_k, &bars->x_full[xs], 0, idx_s[j] * 64, 0, pol_keep);
            }
          }
        }
        __syncwarp();
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------------- PV issuer
      const uint32_t idesc = (FAR && !BF) ? idesc_f16(64, 128, false, true) : idesc_bf16(64, 128, false, true);
      int npv = 0;                    // steps whose PV MMAs were issued (and committed)
      for (int p = 0; p < np; ++p) {
        const int b = p & 3, g = p & 1, ys = p % C::kYP;
        if (!mbar_wait_warp(&bars->p_full[b], (p >> 2) & 1, status, abort_flag)) break;
        if (!mbar_wait_warp(&bars->y_full[ys], (p / C::kYP) & 1, status, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (2 * p + x < total) {
            const uint32_t lane_off = static_cast<uint32_t>(16 * x) << 16;
            const uint32_t d = tmem + lane_off + kColO + 128 * g;
            const uint32_t a = tmem + lane_off + kColS + 64 * b;
            const uint32_t yb = smem_u32(ysub(p, x));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16_ts_by(leader, d, a + 8 * kk, sw128_desc(yb + kk * 2048, kOpBytes / 2, 1024), idesc,
                             ((p >> 1) | kk) != 0);
          }
        }
        mma_commit_by(leader, &bars->pv_done[b]);
        npv = p + 1;
      }
      // every PV completion signal has landed before the CTA leaves (the last ones have no other waiter)
      drain_ring<true>(bars->pv_done, 4, npv, status, abort_flag);
    } else if (warp == 2) {
      // ---------------------------------------------------------------- QK issuer
      // QK(p) into S/P buffer p % 4 once PV(p - 4) freed it and the pair's X slot landed
      const uint32_t idesc = (FAR && !BF) ? idesc_f16(64, 64, false, false) : idesc_bf16(64, 64, false, false);
      const uint32_t a0 = smem_u32(smem + C::kOffQ);
      bool ok = mbar_wait_warp(&bars->qd_full, 0, status, abort_flag);
      int nqk = 0;                    // steps whose QK MMAs were issued (and committed)
      for (int p = 0; ok && p < np; ++p) {
        const int xs = p % C::kXP;
        if (p >= 4 && !mbar_wait_warp(&bars->pv_done[p & 3], ((p - 4) >> 2) & 1, status, abort_flag)) break;
        if (!mbar_wait_warp(&bars->x_full[xs], (p / C::kXP) & 1, status, abort_flag)) break;
        tc_fence_after();
        const uint32_t b = p & 3;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (2 * p + x < total) {
            const uint32_t b0 = smem_u32(xsub(p, x));
            const uint32_t d = tmem + (static_cast<uint32_t>(16 * x) << 16) + kColS + 64 * b;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_bf16_by(leader, d, sw128_desc(a0 + h * (kOpBytes / 2) + kk * 32, 16, 1024),
                            sw128_desc(b0 + h * (kOpBytes / 2) + kk * 32, 16, 1024), idesc, (h | kk) != 0);
          }
        }
        mma_commit_by(leader, &bars->s_full[b]);
        mma_commit_by(leader, &bars->x_empty[xs]);
        nqk = p + 1;
      }
      // every X-slot release (the QK commit and, in the far pass, the constants warp's reads) has landed before
      // the CTA leaves
      drain_ring<true>(bars->x_empty, C::kXP, nqk, status, abort_flag);
    } else if constexpr (FAR) {
      // ---------------------------------------------------------------- per-column constants (FAR)
      // (sg * log2 e, lz * log2 e or -inf if routed / past nb) and sv
      for (int p = 0; p < np; ++p) {
        const int xs = p % C::kXP, cs_slot = p & 1;
        if (!mbar_wait_warp(&bars->xr_full[xs], (p / C::kXP) & 1, status, abort_flag)) break;
        if (p >= 2 && !mbar_wait_warp(&bars->cc_empty[cs_slot], ((p >> 1) - 1) & 1, status, abort_flag)) break;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int colq = q * 32 + lane;      // step parity x = colq / 64, column colq % 64
          const int x = colq >> 6, i = colq & 63;
          const int j = 2 * p + x;
          const uint8_t* par = xsub(p, x) + kOpBytes;
          const float* pf = reinterpret_cast<const float*>(par);
          const bool masked = j >= total || par[768 + i] != 0 || j * 64 + i >= nb;
          // the bf16 state has no row scales: sg = sv = 1
          cc[(cs_slot * 2 + x) * 64 + i] = make_float2(BF ? kLog2e : pf[64 + i] * kLog2e,
                                                       masked ? -INFINITY : pf[i] * kLog2e);
          cs[(cs_slot * 2 + x) * 64 + i] = masked ? 0.f : (BF ? 1.0f : pf[128 + i]);
        }
        fence_proxy_async_smem();             // generic reads of a slot that TMA refills
        mbar_arrive(&bars->x_empty[xs]);      // the raw parameters of this slot have been read
        mbar_arrive(&bars->cc_full[cs_slot]);
      }
    } else {
      // ---------------------------------------------------------------- Y producer (NEAR)
      // the values of the pair's routed leaves once PV(p - kYP) freed its Y slot
      const uint64_t pol_keep = policy_evict_last();
      for (int p = 0; p < np; ++p) {
        const int ys = p % C::kYP;
        if (p >= C::kYP &&
            !mbar_wait_warp(&bars->pv_done[(p - C::kYP) & 3], ((p - C::kYP) >> 2) & 1, status, abort_flag))
          break;
        if (leader) {
          mbar_arrive_expect_tx(&bars->y_full[ys], (2 * p + 1 < total ? 2 : 1) * kOpBytes);
          for (int x = 0; x < 2; ++x)
            if (2 * p + x < total)
              tma_load_3d(ysub(p, x), &tm_v, &bars->y_full[ys], 0, idx_s[2 * p + x] * 64, 0, pol_keep);
        }
        __syncwarp();
      }
    }
  } else if (warp < 12) {
    // ------------------------------------------------------------------ softmax warpgroups
    if constexpr (FAR) asm volatile("setmaxnreg.inc.sync.aligned.u32 184;");
    const int g = (warp - 4) >> 2;            // warpgroup: 0 takes even pairs, 1 odd pairs
    const int quarter = warp & 3;
    const int x = lane >> 4;                  // step parity of this thread
    const int r = quarter * 16 + (lane & 15); // query row
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const bool warp_rows = quarter * 16 < TROWS;   // warp-uniform: false for the held copies of row 31
    const float c_near = scale * kLog2e;
    float m_used = -INFINITY, l = 0.f;
    bool aborted = false;
    int kcount = 0;
    for (int p = g; p < np; p += 2, ++kcount) {
      const int b = p & 3;
      const bool has = 2 * p + x < total;
      if (!mbar_wait_warp(&bars->s_full[b], (p >> 2) & 1, status, abort_flag)) { aborted = true; break; }
      __syncwarp();
      tc_fence_after();
      if (TROWS < 64 && !warp_rows) {
        if (FAR) {
          if (!mbar_wait_warp(&bars->cc_full[g], (p >> 1) & 1, status, abort_flag)) { aborted = true; break; }
          mbar_arrive(&bars->cc_empty[g]);
        }
        uint32_t z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0u;
        tmem_st32(tmem + lane_base + kColS + 64 * b, z);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bars->p_full[b]);
        continue;
      }
      uint32_t d0[32], d1[32];
      tmem_ld32(tmem + lane_base + kColS + 64 * b, d0);
      tmem_ld32(tmem + lane_base + kColS + 64 * b + 32, d1);
      tmem_ld_wait();
      const float2* c = cc + (g * 2 + x) * 64;
      const float* sv = cs + (g * 2 + x) * 64;
      if (FAR && !mbar_wait_warp(&bars->cc_full[g], (p >> 1) & 1, status, abort_flag)) { aborted = true; break; }
      float lg[64];
      float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const uint32_t di0 = i < 32 ? d0[i] : d1[i - 32];
        const uint32_t di1 = i < 32 ? d0[i + 1] : d1[i - 31];
        float2 v;
        if constexpr (FAR) {
          const float4 cv = *reinterpret_cast<const float4*>(c + i);     // (c1_i, c2_i, c1_i+1, c2_i+1)
          v = fma2(make_float2(__uint_as_float(di0), __uint_as_float(di1)), make_float2(cv.x, cv.z),
                   make_float2(cv.y, cv.w));
        } else {
          v = make_float2(__uint_as_float(di0), __uint_as_float(di1));   // raw S; scaled in the exponent's FMA
        }
        lg[i] = v.x;
        lg[i + 1] = v.y;
        mxa[(i >> 1) & 3] = max3(mxa[(i >> 1) & 3], v.x, v.y);
      }
      // NEAR: logit = c_near * S with c_near = scale * log2 e > 0, so its maximum is c_near * max S
      const float esc = FAR ? 1.0f : c_near;
      const float mx = __fmul_rn(esc, fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])));
      // the half of an absent step (odd step count) holds stale TMEM: keep it inert
      const float m_new = has ? fmaxf(m_used, mx) : m_used;
      const bool need = m_new > m_used + kRescale;
      const float alpha = need ? ex2(m_used - m_new) : 1.0f;
      if (need) {
        l *= alpha;
        m_used = m_new;
      }
      const bool live = has && m_used != -INFINITY;
      const float2 negm2 = make_float2(live ? -m_used : 0.f, live ? -m_used : 0.f), esc2 = make_float2(esc, esc);
      uint32_t pw[32];
      float2 rs2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const float2 e = fma2(make_float2(lg[i], lg[i + 1]), esc2, negm2);
        const float2 pp = live ? make_float2(ex2(e.x), ex2(e.y)) : make_float2(0.f, 0.f);
        rs2[(i >> 1) & 3] = add2(rs2[(i >> 1) & 3], pp);
        if constexpr (FAR && !BF) {
          // far weights fp16(p * sv), as the reference's (p * sv).to(fp16) on the vbar codes
          const float2 w = mul2(pp, *reinterpret_cast<const float2*>(sv + i));
          pw[i >> 1] = pack_f16x2(w.x, w.y);
        } else {
          pw[i >> 1] = pack_bf16x2(pp.x, pp.y);
        }
      }
      if (FAR) mbar_arrive(&bars->cc_empty[g]);
      const float2 rsa = add2(add2(rs2[0], rs2[1]), add2(rs2[2], rs2[3]));
      l += rsa.x + rsa.y;
      // the O rows are rescaled only after this warpgroup's previous PV (pair p - 2) is done; the whole warp
      // takes part because TMEM loads and stores are warp-collective
      __syncwarp();
      const bool any_need = __any_sync(0xffffffffu, need);
      if (kcount >= 1 && any_need) {
        if (!mbar_wait_warp(&bars->pv_done[(p - 2) & 3], ((p - 2) >> 2) & 1, status, abort_flag)) {
          aborted = true;
          break;
        }
        __syncwarp();
        tc_fence_after();
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + kColO + 128 * g + 32 * q4, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tmem + lane_base + kColO + 128 * g + 32 * q4, o);
        }
      }
      tmem_st32(tmem + lane_base + kColS + 64 * b, pw);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->p_full[b]);
    }
    // ---------------------------------------------------------------- epilogue
    const int pl = g + 2 * (kcount - 1);     // this warpgroup's last pair
    const bool last_ok =
        !aborted && (kcount == 0 || mbar_wait_warp(&bars->pv_done[pl & 3], (pl >> 2) & 1, status, abort_flag));
    float* m1s = epi;
    float* l1s = epi + 128;
    const int slot = x * 64 + r;
    if (g == 1) {
      m1s[slot] = m_used;
      l1s[slot] = l;
      mbar_arrive(&bars->epi1);
    } else if (last_ok && mbar_wait_warp(&bars->epi1, 0, status, abort_flag)) {
      const float n0 = m_used * kLn2, n1 = m1s[slot] * kLn2;     // natural-log units
      const float l1 = l1s[slot];
      const int64_t li = (t0 + tloc) * TROWS + r;                // query index in tile order
      const bool valid = r < TROWS && li < n;
      const int64_t orow = (perm != nullptr && valid) ? static_cast<int64_t>(__ldg(perm + li)) : li;
      // NEAR: the far and tail partials of the row join the merge
      const float* fp = (!FAR && far_part != nullptr && valid) ? far_part + orow * 130 : nullptr;
      const float* tp = (!FAR && tail_part != nullptr && valid) ? tail_part + orow * 130 : nullptr;
      const float mf = fp ? fp[128] : -INFINITY, lf = fp ? fp[129] : 0.f;
      const float mt = tp ? tp[128] : -INFINITY, lt = tp ? tp[129] : 0.f;
      const float mh = fmaxf(n0, n1);
      const float mm = fmaxf(fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, 16)), fmaxf(mf, mt));
      const float a0 = n0 == -INFINITY ? 0.f : expf(n0 - mm);
      const float a1 = n1 == -INFINITY ? 0.f : expf(n1 - mm);
      const float af = mf == -INFINITY ? 0.f : expf(mf - mm);
      const float at = mt == -INFINITY ? 0.f : expf(mt - mm);
      const float dh = l * a0 + l1 * a1;
      const float den = dh + __shfl_xor_sync(0xffffffffu, dh, 16) + lf * af + lt * at;
      // FAR keeps the row unnormalised (acc relative to mm, with l = den) for the NEAR merge
      const float inv = FAR ? 1.0f : 1.0f / fmaxf(den, 1e-30f);
      const float c0 = a0 * inv, c1 = a1 * inv, cf = af * inv, ct = at * inv;
      if (valid && x == 0) {
        if (FAR) {
          far_part[orow * 130 + 128] = mm;
          far_part[orow * 130 + 129] = den;
        } else if (lse != nullptr) {
          lse[orow] = mm + logf(fmaxf(den, 1e-30f));
        }
      }
      __syncwarp();
      tc_fence_after();
      float* dst_row = FAR ? far_part + orow * 130 : out + orow * 128;
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t o0[32], o1[32];
        tmem_ld32(tmem + lane_base + kColO + 32 * q4, o0);
        tmem_ld32(tmem + lane_base + kColO + 128 + 32 * q4, o1);
        tmem_ld_wait();
        float a[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float v = 0.f;
          if (c0 != 0.f) v = __uint_as_float(o0[i]) * c0;
          if (c1 != 0.f) v = fmaf(__uint_as_float(o1[i]), c1, v);
          a[i] = v + __shfl_xor_sync(0xffffffffu, v, 16);      // + the other step parity of the row
        }
        if (valid && x == (q4 >> 1)) {
          float4* dst = reinterpret_cast<float4*>(dst_row + 32 * q4);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float t = a[4 * i + e];
              if (cf != 0.f) t = fmaf(fp[32 * q4 + 4 * i + e], cf, t);
              if (ct != 0.f) t = fmaf(tp[32 * q4 + 4 * i + e], ct, t);
              v[e] = t;
            }
            if (FAR) {      // 130-float rows are only 8-byte aligned
              reinterpret_cast<float2*>(dst_row + 32 * q4)[2 * i] = make_float2(v[0], v[1]);
              reinterpret_cast<float2*>(dst_row + 32 * q4)[2 * i + 1] = make_float2(v[2], v[3]);
            } else {
              dst[i] = make_float4(v[0], v[1], v[2], v[3]);
            }
          }
        }
      }
    }
  } else if constexpr (FAR) {
    // ------------------------------------------------------------------ code converters (FAR)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 72;");
    if (warp < 14) {
      // g codes -> fp16 X operand of each block, in place, once they landed
      const int row = threadIdx.x - 384;
      for (int p = 0; p < np; ++p) {
        const int xs = p % C::kXP;
        if (!mbar_wait_warp(&bars->xr_full[xs], (p / C::kXP) & 1, status, abort_flag)) break;
        if constexpr (!BF) {
          codes_to_f16_in_place(smem_u32(xsub(p, 0)), row);
          codes_to_f16_in_place(smem_u32(xsub(p, 1)), row);
          fence_proxy_async_smem();      // the fp16 operand is read by the tensor cores (async proxy)
        }
        mbar_arrive(&bars->x_full[xs]);
      }
    } else {
      // vbar codes into the upper halves of the pair's Y slots, issued two pairs ahead (the slot of pair
      // p + 2 is freed by PV(p - 1)), then converted in place
      const int row = threadIdx.x - 448;
      const uint32_t leader = elect_one() && warp == 14;      // one issuing lane for the two warps
      const uint64_t pol_stream = policy_evict_first();
      auto load = [&](int p) -> bool {
        if (p >= np) return true;
        const int ys = p % C::kYP;
        if (p >= C::kYP &&
            !mbar_wait_warp(&bars->pv_done[(p - C::kYP) & 3], ((p - C::kYP) >> 2) & 1, status, abort_flag))
          return false;
        if (leader) {
          mbar_arrive_expect_tx(&bars->yr_full[ys], 2 * (BF ? kOpBytes : kRawBytes));
          for (int x = 0; x < 2; ++x) {
            if constexpr (BF)     // the bf16 vbar block as its operand (both halves)
              tma_load_4d(ysub(p, x), &tm_vraw, &bars->yr_full[ys], 0, (2 * p + x) * 64, 0, srow, pol_stream);
            else
              tma_load_3d(ysub(p, x) + kOpBytes / 2, &tm_vraw, &bars->yr_full[ys], 0, (2 * p + x) * 64, srow,
                          pol_stream);
          }
        }
        __syncwarp();
        return true;
      };
      bool ok = load(0) && load(1);
      for (int p = 0; ok && p < np; ++p) {
        if (!load(p + 2)) break;
        const int ys = p % C::kYP;
        if (!mbar_wait_warp(&bars->yr_full[ys], (p / C::kYP) & 1, status, abort_flag)) break;
        if constexpr (!BF) {
          codes_to_f16_in_place(smem_u32(ysub(p, 0)), row);
          codes_to_f16_in_place(smem_u32(ysub(p, 1)), row);
          fence_proxy_async_smem();
        }
        mbar_arrive(&bars->y_full[ys]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

namespace {
template <bool FAR, bool BF>
int set_tile_attr() {
  using C = tfx::Cfg<FAR>;
  bool ok = cudaFuncSetAttribute(tile_fp8_kernel<64, FAR, BF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::kSmemBytes) == cudaSuccess &&
            cudaFuncSetAttribute(tile_fp8_kernel<32, FAR, BF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::kSmemBytes) == cudaSuccess;
  return ok ? HTRC_OK : HTRC_ERR_CUDA;
}
}  // namespace

int launch_tile_fp8(const TileFp8Maps& maps, const int32_t* idx, int kx, int nb, int64_t n, int tile_rows, int64_t t0,
                    int64_t tc, int group, float scale, const float* tail_part, const int32_t* perm, float* far_part,
                    float* out, float* lse, int* status, cudaStream_t st, bool bf16_state) {
  if (kx > tfx::kMaxKx || nb > 65535) return HTRC_ERR_UNSUPPORTED;
  if (kx < nb && far_part == nullptr) return HTRC_ERR_ARG;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    if (set_tile_attr<true, false>() != HTRC_OK || set_tile_attr<false, false>() != HTRC_OK ||
        set_tile_attr<true, true>() != HTRC_OK)
      return HTRC_ERR_CUDA;
    attr_done[dev] = true;
  }
  const int g = group > 1 ? group : 1;
  const unsigned grid = static_cast<unsigned>(tc);
  if (kx < nb) {
    // the far field (all leaves not routed) first, as per-row partials
    auto kf = bf16_state ? (tile_rows == 32 ? tile_fp8_kernel<32, true, true> : tile_fp8_kernel<64, true, true>)
                         : (tile_rows == 32 ? tile_fp8_kernel<32, true> : tile_fp8_kernel<64, true>);
    kf<<<grid, tfx::Cfg<true>::kThreads, tfx::Cfg<true>::kSmemBytes, st>>>(
        maps.dqh, maps.graw, maps.vraw, maps.lz, maps.sg, maps.sv, maps.excl, maps.k, maps.v, idx, kx, nb, n, t0, g,
        scale, nullptr, perm, far_part, nullptr, nullptr, status);
    if (cudaGetLastError() != cudaSuccess) return HTRC_ERR_CUDA;
  }
  auto kn = tile_rows == 32 ? tile_fp8_kernel<32, false> : tile_fp8_kernel<64, false>;
  kn<<<grid, tfx::Cfg<false>::kThreads, tfx::Cfg<false>::kSmemBytes, st>>>(
      maps.qb, maps.graw, maps.vraw, maps.lz, maps.sg, maps.sv, maps.excl, maps.k, maps.v, idx, kx, nb, n, t0, g, scale,
      tail_part, perm, kx < nb ? far_part : nullptr, out, lse, status);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

}  // namespace htrc
