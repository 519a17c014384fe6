// Far field + near field of the flat HTRC operator, fused into one online softmax per query row,
// on tcgen05 tensor cores (h3/htrc_flat_triton.py:88-211, `_tile_kernel` with I8=1, DOT=1, and the
// split merge of :257-273).
//
// One CTA per pair of 64-row tiles (A = 2p, B = 2p+1).  Steps of 64 columns:
//   far  (blocks of 64 leaves of the tile's own state): S = dq8 . g8^T (int8 -> int32),
//        logit = S * (sdq_r * sg_l) + lz_l, excluded / padding leaves masked, value vbar_l (bf16);
//   near (64 keys of routed leaves per step: one leaf of 64, two of 32 or four of 16 keys):
//        S = q8 . k8^T, logit = S * (sq_r * ks_j * scale), value v_j (bf16).  A last step with fewer
//        routed leaves than fit masks its empty columns and issues no PV MMA for them.
// Every MMA is M=64 per tile: tile A's rows live in TMEM lanes {0..15} + 32k, tile B's at lane offset
// 16, so each softmax thread owns one query row of S, P and O.  P (bf16) is written back into the
// TMEM columns of its S buffer and feeds O += P . V as the TMEM A operand; V comes from shared memory
// as an MN-major B operand.
//
// Two softmax warpgroups take alternate steps, each with its own running (max, sum) and O accumulator;
// the two partials (and the tail partial) are merged in the epilogue.  The running maximum is updated
// lazily: a thread rescales its O row only when its maximum grew by more than 2^8 (P <= 256 otherwise).
//
// Data movement: the QK operand of a step (g8 block or k8 leaf, plus its per-column parameters) goes
// through a 3-slot ring freed as soon as the QK MMA completes; the PV operand (vbar block or v leaf)
// through a 4-slot ring freed by the PV MMA (the value loads are the longer-lead ones: a step's V is
// requested four steps ahead).  The completion of PV(j) (one commit, pv_done[j % 4]) frees
// S/P buffer j % 4 for QK(j + 4), Y slot j % 4 for step j + 4, and lets the warpgroup of step j + 2
// rescale its O rows.  All waits block (a suspended thread takes no issue slots from the softmax warps).
// The producer and issuer warps run converged and let one elected lane issue: a warp whose lanes take
// different roles serialises them, since a lane suspended in an mbarrier wait holds up the others.
//
// Tiles of 32 rows (the "max" mode, h3/htrc_flat_runner.py:52) are held as 64 rows whose rows 32..63
// repeat row 31; only rows < 32 are written, and the softmax warps that own only such rows skip the
// arithmetic (they keep their place in the barrier protocol and leave P = 0).
//
// ISO adds the isotropic curvature term c_l * |q_r - mu|^2 to every far logit (h3/htrc_flat.py:331-333,
// the torch backend's curvature="iso"; c_l from the leaf statistics, |q_r - mu|^2 from the tile prep).
//
// Groups (h3/htrc_flat.py:223-231): G consecutive tiles share one far-field state row and one routing;
// tile t of the chunk reads state row t / G.  k-means order (:146-147, :159-165): tile row i is query
// perm[i], so the epilogue writes out/lse row perm[i] (and reads the tail partial of that row).
//
// Warp roles (384 threads): warp 0 X-ring producer; warp 1 PV issuer (+ TMEM owner); warp 11 QK issuer
// and Y-ring producer (both wait for the same PV completions); warps 2-5 and 6-9 the two softmax
// warpgroups; warp 10 per-column constants (scale * log2 e, lz * log2 e or -inf).
#include "common.cuh"
#include "kernels.cuh"

namespace htrc {

namespace {
constexpr int kThreads = 384;
constexpr int kXSlots = 3;
constexpr int kYSlots = 4;
constexpr int kSBufs = 4;
static_assert(kYSlots <= kSBufs, "the QK issuer's loop produces Y(j + kYSlots) for every QK(j + kSBufs)");
constexpr uint32_t kXBytes = 64 * 128;                          // g8 block / k8 leaf: 64 rows x 128 B
constexpr uint32_t kYBytes = 64 * 256;                          // vbar block / v leaf: 2 chunks of 64x64 bf16
constexpr uint32_t kParBytes = 1024;                            // far: lz[64], sg[64], excl[64], cv[64]; near: ks[64]
constexpr uint32_t kXTile = kXBytes + kParBytes;                // 9216 (a multiple of 1024)
constexpr uint32_t kXSlot = 2 * kXTile;
constexpr uint32_t kYSlot = 2 * kYBytes;
constexpr uint32_t kOffQ8 = 0;                                  // 2 tiles x 8 KB
constexpr uint32_t kOffDq8 = 16384;                             // 2 tiles x 8 KB
constexpr uint32_t kOffX = 32768;
constexpr uint32_t kOffY = kOffX + kXSlots * kXSlot;
constexpr uint32_t kOffCC = kOffY + kYSlots * kYSlot;           // [X slot][tile][64] float2 constants
constexpr uint32_t kOffEpi = kOffCC + kXSlots * 2 * 64 * 8;     // m1, l1 [128] each
constexpr uint32_t kOffIdx = kOffEpi + 2 * 128 * 4;             // [tile][kMaxKx] uint16
constexpr int kMaxKx = 1024;
constexpr uint32_t kOffCC3 = kOffIdx + 2 * kMaxKx * 2;          // ISO: [X slot][tile][64] c * log2 e (0 for near)
constexpr uint32_t kOffBar = kOffCC3 + kXSlots * 2 * 64 * 4;
constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;       // S/P buffer b (= step % 4) at 64 b; P uses its first 32 columns
constexpr uint32_t kColO = 256;     // O[g] at 256 + 128 g (tile A / B by lane offset 0 / 16)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescale = 8.0f;    // lazy-rescale threshold (log2 units)
constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23: int32 |x| < 2^22 -> float by an integer add
constexpr int kMagicBits = 0x4B400000;

struct Bars {
  uint64_t qd_full;
  uint64_t x_full[kXSlots];
  uint64_t x_empty[kXSlots];    // QK MMA done (commit) + constants read (32 helper lanes)
  uint64_t y_full[kYSlots];
  uint64_t cc_full[kXSlots];    // 32 helper lanes
  uint64_t cc_empty[kXSlots];   // 128 softmax threads of the step's warpgroup
  uint64_t s_full[kSBufs];      // QK done
  uint64_t p_full[kSBufs];      // 128 softmax threads wrote P into the buffer (and rescaled O if needed)
  uint64_t pv_done[kSBufs];     // PV of the step in this buffer done
  uint64_t epi1;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace

// ML: near steps of several routed leaves (leaf 32 or 16); the leaf-64 instantiation keeps the one-leaf step's
// straight-line producer code (the producers' per-leaf loops, even unexecuted, slowed the QK issuer's loop)
template <int TROWS, bool ISO, bool ML>
__global__ void __launch_bounds__(kThreads, 1)
    tile_attention_kernel(const __grid_constant__ CUtensorMap tm_q8, const __grid_constant__ CUtensorMap tm_dq8,
                          const __grid_constant__ CUtensorMap tm_g8, const __grid_constant__ CUtensorMap tm_vb,
                          const __grid_constant__ CUtensorMap tm_lz, const __grid_constant__ CUtensorMap tm_sg,
                          const __grid_constant__ CUtensorMap tm_excl, const __grid_constant__ CUtensorMap tm_k8,
                          const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_cv,
                          const float* __restrict__ dd, const float* __restrict__ sq,
                          const float* __restrict__ sdq, const float* __restrict__ ks, const int32_t* __restrict__ idx,
                          int kx, int nb, int nf, int leaf, int64_t n, int64_t t0, int64_t tc, int group,
                          float scale,
                          const float* __restrict__ tail_part, const int32_t* __restrict__ perm,
                          float* __restrict__ out, float* __restrict__ lse, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  uint16_t* idx_s = reinterpret_cast<uint16_t*>(smem + kOffIdx);
  float2* cc = reinterpret_cast<float2*>(smem + kOffCC);
  float* epi = reinterpret_cast<float*>(smem + kOffEpi);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tlocA = 2 * blockIdx.x;
  const int ntiles = (tlocA + 1 < tc) ? 2 : 1;
  const int srow[2] = {tlocA / group, (tlocA + 1) / group};     // state rows of tiles A and B
  const int rl = ML ? 64 / leaf : 1;                 // routed leaves per near step
  const int total = nf + (kx + rl - 1) / rl;          // far steps + near steps
  const int tail_cols = (ML && kx % rl) ? (kx % rl) * leaf : 64;   // key columns of the last near step
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->qd_full, 1);
    for (int s = 0; s < kXSlots; ++s) {
      mbar_init(&bars->x_full[s], 1);
      mbar_init(&bars->x_empty[s], 1 + 32);
      mbar_init(&bars->cc_full[s], 32);
      mbar_init(&bars->cc_empty[s], 128);
    }
    for (int s = 0; s < kYSlots; ++s) mbar_init(&bars->y_full[s], 1);
    for (int b = 0; b < kSBufs; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->p_full[b], 128);
      mbar_init(&bars->pv_done[b], 1);
    }
    mbar_init(&bars->epi1, 128);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    // routed leaves of both tiles -> shared memory, range-checked
    for (int x = 0; x < ntiles; ++x) {
      const int32_t* src = idx + static_cast<int64_t>(srow[x]) * kx;
      for (int e = lane; e < kx; e += 32) {
        int leaf = __ldg(src + e);
        if (leaf < 0 || leaf >= nb) {
          flag_status(status, ST_BAD_INDEX);
          leaf = 0;
        }
        idx_s[x * kMaxKx + e] = static_cast<uint16_t>(leaf);
      }
    }
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ X-ring producer
    // QK operands + per-column parameters, up to four steps ahead of the QK MMAs
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    const uint32_t leader = elect_one();
    {
      if (leader) {
        mbar_arrive_expect_tx(&bars->qd_full, 2 * kXBytes * ntiles);
        for (int x = 0; x < ntiles; ++x) {
          const int row = static_cast<int>((t0 + tlocA + x) * 64);
          tma_load_2d(smem + kOffQ8 + x * kXBytes, &tm_q8, &bars->qd_full, 0, row, pol_stream);
          tma_load_2d(smem + kOffDq8 + x * kXBytes, &tm_dq8, &bars->qd_full, 0, row, pol_stream);
        }
      }
      for (int nx = 0; nx < total; ++nx) {
        if (nx >= kXSlots && !mbar_wait_warp(&bars->x_empty[nx % kXSlots], ((nx / kXSlots) - 1) & 1, status, abort_flag))
          break;
        if (leader) {
          const int s = nx % kXSlots;
          uint8_t* st = smem + kOffX + s * kXSlot;
          if (nx < nf) {
            mbar_arrive_expect_tx(&bars->x_full[s], (kXBytes + 256 + 256 + 64 + (ISO ? 256 : 0)) * ntiles);
            for (int x = 0; x < ntiles; ++x) {
              uint8_t* tx = st + x * kXTile;
              const int tl = srow[x];
              tma_load_3d(tx, &tm_g8, &bars->x_full[s], 0, nx * 64, tl, pol_stream);
              tma_load_2d(tx + kXBytes, &tm_lz, &bars->x_full[s], nx * 64, tl, pol_stream);
              tma_load_2d(tx + kXBytes + 256, &tm_sg, &bars->x_full[s], nx * 64, tl, pol_stream);
              tma_load_2d(tx + kXBytes + 512, &tm_excl, &bars->x_full[s], nx * 64, tl, pol_stream);
              if (ISO) tma_load_2d(tx + kXBytes + 768, &tm_cv, &bars->x_full[s], nx * 64, tl, pol_stream);
            }
          } else {
            // the step's routed leaves: rows leaf * i .. of the k8 block, key scales at 4 leaf * i
            if constexpr (!ML) {
              mbar_arrive_expect_tx(&bars->x_full[s], (kXBytes + 256) * ntiles);
              for (int x = 0; x < ntiles; ++x) {
                uint8_t* tx = st + x * kXTile;
                const int lf = idx_s[x * kMaxKx + (nx - nf)];
                tma_load_2d(tx, &tm_k8, &bars->x_full[s], 0, lf * 64, pol_keep);
                bulk_load(tx + kXBytes, ks + static_cast<int64_t>(lf) * 64, 256, &bars->x_full[s], pol_keep);
              }
            } else {
              const int e0 = (nx - nf) * rl, cnt = min(rl, kx - e0);
              mbar_arrive_expect_tx(&bars->x_full[s], (128 + 4) * leaf * cnt * ntiles);
              for (int x = 0; x < ntiles; ++x) {
                uint8_t* tx = st + x * kXTile;
#pragma unroll 1
                for (int i = 0; i < cnt; ++i) {
                  const int lf = idx_s[x * kMaxKx + e0 + i];
                  tma_load_2d(tx + i * leaf * 128, &tm_k8, &bars->x_full[s], 0, lf * leaf, pol_keep);
                  bulk_load(tx + kXBytes + i * leaf * 4, ks + static_cast<int64_t>(lf) * leaf, leaf * 4,
                            &bars->x_full[s], pol_keep);
                }
              }
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ PV issuer
    // O[g] += P . V for step np once its warpgroup wrote P and its Y slot landed; one commit per step.
    // Descriptors are built from precomputed words: the start address is the low 14 bits.
    const uint32_t leader = elect_one();
    const uint32_t id_pv = idesc_bf16(64, 128, /*a_mn_major=*/false, /*b_mn_major=*/true);
    const uint32_t hi = (1024u >> 4) | (1u << 14) | (2u << 29);          // SBO 1024, version, SWIZZLE_128B
    const uint32_t lo0 = (smem_u32(smem + kOffY) >> 4) | ((kYBytes / 2) >> 4 << 16);   // + LBO (chunk stride)
    // near steps: the Y slot holds [leaf][half][leaf rows][64] (one load per routed leaf), so the 64-column
    // halves are leaf * 128 bytes apart and K step kk (keys 16 kk ..) starts in leaf 16 kk / leaf
    const uint32_t lo0n = (smem_u32(smem + kOffY) >> 4) | (static_cast<uint32_t>(leaf * 128) >> 4 << 16);
    uint32_t koff_near[4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      koff_near[kk] = static_cast<uint32_t>((16 * kk / leaf) * leaf * 256 + (16 * kk % leaf) * 128) >> 4;
    int ys = 0;
    uint32_t yph = 0;
    int npv = 0;
    for (int np = 0; np < total; ++np) {
      if (!mbar_wait_warp(&bars->p_full[np & 3], (np >> 2) & 1, status, abort_flag)) break;
      if (!mbar_wait_warp(&bars->y_full[ys], yph, status, abort_flag)) break;
      tc_fence_after();
      const uint32_t b = np & 3, g = np & 1, k = np >> 1;
      const bool near = ML && np >= nf;
      const uint32_t lo = (near ? lo0n : lo0) + ys * (kYSlot >> 4);
      const int kks = (ML && near && np == total - 1) ? tail_cols / 16 : 4;     // K steps with keys
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (x < ntiles) {
          const uint32_t lane_off = static_cast<uint32_t>(16 * x) << 16;
          const uint32_t d = tmem + lane_off + kColO + 128 * g;
          const uint32_t a = tmem + lane_off + kColS + 64 * b;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            if (kk < kks)
              mma_bf16_ts_by(leader, d, a + 8 * kk,
                             (static_cast<uint64_t>(hi) << 32) |
                                 (lo + ((x * kYBytes) >> 4) + (near ? koff_near[kk] : (kk * 2048) >> 4)),
                             id_pv, (k | kk) != 0);
        }
      }
      mma_commit_by(leader, &bars->pv_done[b]);
      if (++ys == kYSlots) { ys = 0; yph ^= 1; }
      npv = np + 1;
    }
    // every PV completion signal has landed before the CTA leaves (the last ones have no other waiter)
    drain_ring<true>(bars->pv_done, kSBufs, npv, status, abort_flag);
  } else if (warp == 11) {
    // ------------------------------------------------------------------ QK issuer + Y-ring producer
    // Both wait for PV(j): it frees S/P buffer j % 4 for QK(j + 4) and Y slot j % 4 for step j + 4.
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    const uint32_t leader = elect_one();
    const uint32_t id_qk = idesc_i8(64, 64);
    const uint32_t hi = (1024u >> 4) | (1u << 14) | (2u << 29);
    const uint32_t lo_q8 = (smem_u32(smem + kOffQ8) >> 4) | (1u << 16);      // LBO 16 (unused for SW128 K-major)
    const uint32_t lo_dq8 = (smem_u32(smem + kOffDq8) >> 4) | (1u << 16);
    const uint32_t lo_x = (smem_u32(smem + kOffX) >> 4) | (1u << 16);
    auto produce_y = [&](int ny) {
      if (leader) {
        const int s = ny % kYSlots;
        uint8_t* st = smem + kOffY + s * kYSlot;
        // both 64-column halves in one load: [half][rows][64]; a near step's leaves one after another
        if constexpr (!ML) {
          mbar_arrive_expect_tx(&bars->y_full[s], kYBytes * ntiles);
          for (int x = 0; x < ntiles; ++x) {
            uint8_t* ty = st + x * kYBytes;
            if (ny < nf)
              tma_load_4d(ty, &tm_vb, &bars->y_full[s], 0, ny * 64, 0, srow[x], pol_stream);
            else
              tma_load_3d(ty, &tm_v, &bars->y_full[s], 0, idx_s[x * kMaxKx + (ny - nf)] * 64, 0, pol_keep);
          }
        } else {
          const int e0 = (ny - nf) * rl, cnt = ny < nf ? 1 : min(rl, kx - e0);
          mbar_arrive_expect_tx(&bars->y_full[s], (ny < nf ? kYBytes : 256u * leaf * cnt) * ntiles);
          for (int x = 0; x < ntiles; ++x) {
            uint8_t* ty = st + x * kYBytes;
            if (ny < nf) {
              tma_load_4d(ty, &tm_vb, &bars->y_full[s], 0, ny * 64, 0, srow[x], pol_stream);
            } else {
#pragma unroll 1
              for (int i = 0; i < cnt; ++i)
                tma_load_3d(ty + i * leaf * 256, &tm_v, &bars->y_full[s], 0, idx_s[x * kMaxKx + e0 + i] * leaf, 0,
                            pol_keep);
            }
          }
        }
      }
      __syncwarp();
    };
    // QK of step nq into S/P buffer nq % 4, once its X slot landed
    int nqk = 0;                    // QK steps issued (and committed)
    auto issue_qk = [&](int nq) -> bool {
      const int s = nq % kXSlots;
      if (!mbar_wait_warp(&bars->x_full[s], (nq / kXSlots) & 1, status, abort_flag)) return false;
      tc_fence_after();
      const uint32_t b = nq & 3;
      const uint32_t la = nq < nf ? lo_dq8 : lo_q8;
      const uint32_t lb = lo_x + s * (kXSlot >> 4);
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (x < ntiles) {
          const uint32_t d = tmem + (static_cast<uint32_t>(16 * x) << 16) + kColS + 64 * b;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_i8_by(leader, d, (static_cast<uint64_t>(hi) << 32) | (la + ((x * kXBytes + kk * 32) >> 4)),
                      (static_cast<uint64_t>(hi) << 32) | (lb + ((x * kXTile + kk * 32) >> 4)), id_qk, kk != 0);
        }
      }
      mma_commit_by(leader, &bars->s_full[b]);
      mma_commit_by(leader, &bars->x_empty[s]);
      nqk = nq + 1;
      return true;
    };
    bool ok = mbar_wait_warp(&bars->qd_full, 0, status, abort_flag);
    for (int j = 0; j < total && j < kYSlots; ++j) produce_y(j);
    for (int j = 0; ok && j < total && j < kSBufs; ++j) ok = issue_qk(j);
    for (int j = 0; ok && j + kYSlots < total; ++j) {
      if (!mbar_wait_warp(&bars->pv_done[j & 3], (j >> 2) & 1, status, abort_flag)) break;
      if (j + kSBufs < total) ok = issue_qk(j + kSBufs);    // first: QK(j + 4) is on the step's critical chain
      produce_y(j + kYSlots);
    }
    // every QK-operand slot's release (the QK commit and the constants warp's reads) has landed before the
    // CTA leaves
    drain_ring<true>(bars->x_empty, kXSlots, nqk, status, abort_flag);
  } else if (warp == 10) {
    // ------------------------------------------------------------------ per-column constants
    // far: (sg * log2 e, lz * log2 e or -inf if routed / past nb) per column; near: ks * scale * log2 e per
    // column, packed
    const float near_scale = scale * kLog2e;
    for (int j = 0; j < total; ++j) {
      const int s = j % kXSlots;
      if (!mbar_wait_warp(&bars->x_full[s], (j / kXSlots) & 1, status, abort_flag)) break;
      if (j >= kXSlots && !mbar_wait_warp(&bars->cc_empty[s], ((j / kXSlots) - 1) & 1, status, abort_flag)) break;
      const uint8_t* st = smem + kOffX + s * kXSlot;
      float2* c = cc + s * 128;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int colq = q * 32 + lane;      // tile x = colq / 64, column colq % 64
        const int x = colq >> 6, i = colq & 63;
        const uint8_t* par = st + x * kXTile + kXBytes;
        if (j < nf) {
          const float lzv = reinterpret_cast<const float*>(par)[i];
          const float sgv = reinterpret_cast<const float*>(par + 256)[i];
          const bool masked = par[512 + i] != 0 || j * 64 + i >= nb;
          const float2 v = make_float2(sgv * kLog2e, masked ? -INFINITY : lzv * kLog2e);
          if (ISO) reinterpret_cast<float*>(smem + kOffCC3)[s * 128 + colq] =
              reinterpret_cast<const float*>(par + 768)[i] * kLog2e;
          c[colq] = v;
        } else if (j != total - 1 || tail_cols == 64) {
          // near: one constant per column, packed (tile x's 64 at x * 64 of the slot's float view)
          reinterpret_cast<float*>(c)[colq] = reinterpret_cast<const float*>(par)[i] * near_scale;
          if (ISO) reinterpret_cast<float*>(smem + kOffCC3)[s * 128 + colq] = 0.f;
        } else {
          // partial last near step: (key constant, 0) per column as the far steps lay them out, columns past
          // the routed leaves (stale key scales) (0, -inf)
          const bool key = i < tail_cols;
          c[colq] = make_float2(key ? reinterpret_cast<const float*>(par)[i] * near_scale : 0.f,
                                key ? 0.f : -INFINITY);
          if (ISO) reinterpret_cast<float*>(smem + kOffCC3)[s * 128 + colq] = 0.f;
        }
      }
      fence_proxy_async_smem();            // generic reads of a slot that TMA refills
      mbar_arrive(&bars->x_empty[s]);      // the raw parameters of this slot have been read
      mbar_arrive(&bars->cc_full[s]);
    }
  } else {
    // ------------------------------------------------------------------ softmax warpgroups
    const int g = (warp - 2) >> 2;            // warpgroup: 0 takes even steps, 1 odd steps
    const int quarter = warp & 3;
    const int x = lane >> 4;                  // tile of this thread's query row
    const int r = quarter * 16 + (lane & 15);
    const int col = x * 64 + r;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const bool has_tile = x < ntiles;
    const bool warp_rows = quarter * 16 < TROWS;   // warp-uniform: false for the held copies of row 31
    const int64_t tl = tlocA + x;
    const int64_t gr = (t0 + tl) * 64 + r;
    const float sq_r = has_tile ? __ldg(sq + gr) : 0.f;
    const float sdq_r = has_tile ? __ldg(sdq + gr) : 0.f;
    const float dd_r = (ISO && has_tile) ? __ldg(dd + gr) : 0.f;
    float m_used = -INFINITY, l = 0.f;
    bool aborted = false;
    int kcount = 0;
    for (int j = g; j < total; j += 2, ++kcount) {
      const int s = j % kXSlots, b = j & 3;
      if (!mbar_wait_warp(&bars->s_full[b], (j >> 2) & 1, status, abort_flag)) { aborted = true; break; }
      __syncwarp();
      tc_fence_after();
      if (TROWS < 64 && !warp_rows) {
        // held copies only: consume the step's constants in order and write P = 0 after QK(j)
        if (!mbar_wait_warp(&bars->cc_full[s], (j / kXSlots) & 1, status, abort_flag)) { aborted = true; break; }
        mbar_arrive(&bars->cc_empty[s]);
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
      if (!mbar_wait_warp(&bars->cc_full[s], (j / kXSlots) & 1, status, abort_flag)) { aborted = true; break; }
      const float2* c = cc + s * 128 + x * 64;
      const float2 magic2 = make_float2(kMagic, kMagic);
      float lg[64];
      float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};   // independent chains
      float esc;        // the exponent's argument is esc * lg - m (one FMA)
      if (j >= nf && (j != total - 1 || tail_cols == 64)) {
        // near step (warp-uniform): lg = S * (ks * scale * log2 e); the row's scale sq_r > 0 multiplies after
        // the maximum and inside the exponent's FMA.  The constants are packed one per column.
        const float* c1 = reinterpret_cast<const float*>(cc + s * 128) + x * 64;
#pragma unroll
        for (int i = 0; i < 64; i += 4) {
          const float4 cv = *reinterpret_cast<const float4*>(c1 + i);    // c1 of columns i .. i + 3
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int ii = i + 2 * h;
            const uint32_t di0 = ii < 32 ? d0[ii] : d1[ii - 32];
            const uint32_t di1 = ii < 32 ? d0[ii + 1] : d1[ii - 31];
            const float2 xm = make_float2(__int_as_float(static_cast<int>(di0) + kMagicBits),
                                          __int_as_float(static_cast<int>(di1) + kMagicBits));
            const float2 u = mul2(sub2(xm, magic2), h ? make_float2(cv.z, cv.w) : make_float2(cv.x, cv.y));
            lg[ii] = u.x;
            lg[ii + 1] = u.y;
            mxa[(ii >> 1) & 3] = max3(mxa[(ii >> 1) & 3], u.x, u.y);
          }
        }
        esc = sq_r;
      } else {
        // far step: lg = S * (sdq_r * sg * log2 e) + lz * log2 e (+ the iso term), masked columns -inf; a
        // partial last near step (fewer routed leaves than fit) the same way with sq_r and the key constants,
        // its columns past the routed leaves masked
        const float* c3 = reinterpret_cast<const float*>(smem + kOffCC3) + s * 128 + x * 64;
        const float2 dd2 = make_float2(dd_r, dd_r);
        const float sr = (!ML || j < nf) ? sdq_r : sq_r;
        const float2 srow2 = make_float2(sr, sr);
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          const float4 cv = *reinterpret_cast<const float4*>(c + i);     // (c1_i, c2_i, c1_i+1, c2_i+1)
          const uint32_t di0 = i < 32 ? d0[i] : d1[i - 32];
          const uint32_t di1 = i < 32 ? d0[i + 1] : d1[i - 31];
          const float2 xm = make_float2(__int_as_float(static_cast<int>(di0) + kMagicBits),
                                        __int_as_float(static_cast<int>(di1) + kMagicBits));
          const float2 fd = sub2(xm, magic2);
          const float2 t = mul2(srow2, make_float2(cv.x, cv.z));
          float2 v = fma2(fd, t, make_float2(cv.y, cv.w));
          if (ISO) v = fma2(*reinterpret_cast<const float2*>(c3 + i), dd2, v);
          lg[i] = v.x;
          lg[i + 1] = v.y;
          mxa[(i >> 1) & 3] = max3(mxa[(i >> 1) & 3], v.x, v.y);
        }
        esc = 1.0f;
      }
      const float mx = __fmul_rn(esc, fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])));
      mbar_arrive(&bars->cc_empty[s]);
      // rows of an absent tile B (odd tile count) hold stale TMEM: keep them inert
      const float m_new = has_tile ? fmaxf(m_used, mx) : m_used;
      const bool need = m_new > m_used + kRescale;
      const float alpha = need ? ex2(m_used - m_new) : 1.0f;
      if (need) {
        l *= alpha;
        m_used = m_new;
      }
      // a row whose maximum is still -inf has only -inf logits so far (P = 0 from ex2); rows of an absent
      // tile B get garbage P, which no MMA reads (PV runs for present tiles only)
      const float mref = m_used != -INFINITY ? m_used : 0.f;
      const float2 negm2 = make_float2(-mref, -mref), esc2 = make_float2(esc, esc);
      uint32_t pw[32];
      float2 rs2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const float2 e = fma2(make_float2(lg[i], lg[i + 1]), esc2, negm2);
        const float2 p = make_float2(ex2(e.x), ex2(e.y));
        rs2[(i >> 1) & 3] = add2(rs2[(i >> 1) & 3], p);
        pw[i >> 1] = pack_bf16x2(p.x, p.y);
      }
      const float2 rsa = add2(add2(rs2[0], rs2[1]), add2(rs2[2], rs2[3]));
      l += rsa.x + rsa.y;
      // the O row is rescaled only after this warpgroup's previous PV (step j - 2) is done; the whole
      // warp takes part because TMEM loads and stores are warp-collective.  pv_done[(j - 2) % 4] is then
      // at most one phase behind: QK(j - 2) was issued after PV(j - 6) completed.
      __syncwarp();
      const bool any_need = __any_sync(0xffffffffu, need);
      if (kcount >= 1 && any_need) {
        if (!mbar_wait_warp(&bars->pv_done[(j - 2) & 3], ((j - 2) >> 2) & 1, status, abort_flag)) {
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
    const int jl = g + 2 * (kcount - 1);     // this warpgroup's last step
    const bool last_ok =
        !aborted && (kcount == 0 || mbar_wait_warp(&bars->pv_done[jl & 3], (jl >> 2) & 1, status, abort_flag));
    float* m1s = epi;
    float* l1s = epi + 128;
    if (g == 1) {
      m1s[col] = kcount ? m_used : -INFINITY;
      l1s[col] = l;
      mbar_arrive(&bars->epi1);
    } else if (last_ok && mbar_wait_warp(&bars->epi1, 0, status, abort_flag)) {
      const float m1 = m1s[col], l1 = l1s[col];
      const float m0 = kcount ? m_used : -INFINITY;
      const float n0 = m0 * kLn2, n1 = m1 * kLn2;           // natural-log units
      const int64_t li = (t0 + tl) * TROWS + r;                  // query index in tile order
      const bool valid = has_tile && r < TROWS && li < n;
      const int64_t orow = (perm != nullptr && valid) ? static_cast<int64_t>(__ldg(perm + li)) : li;
      const float* tp = (tail_part != nullptr && valid) ? tail_part + orow * 130 : nullptr;
      const float mt = tp ? tp[128] : -INFINITY, lt = tp ? tp[129] : 0.f;
      const float mm = fmaxf(fmaxf(n0, n1), mt);
      const float a0 = n0 == -INFINITY ? 0.f : expf(n0 - mm);
      const float a1 = n1 == -INFINITY ? 0.f : expf(n1 - mm);
      const float at = mt == -INFINITY ? 0.f : expf(mt - mm);
      const float den = l * a0 + l1 * a1 + lt * at;
      const float inv = 1.0f / fmaxf(den, 1e-30f);
      const float c0 = a0 * inv, c1 = a1 * inv, ct = at * inv;
      if (valid && lse != nullptr) lse[orow] = mm + logf(fmaxf(den, 1e-30f));
      __syncwarp();
      tc_fence_after();
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t o0[32], o1[32];
        tmem_ld32(tmem + lane_base + kColO + 32 * q4, o0);
        tmem_ld32(tmem + lane_base + kColO + 128 + 32 * q4, o1);
        tmem_ld_wait();
        if (valid) {
          float4* dst = reinterpret_cast<float4*>(out + orow * 128 + 32 * q4);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float a = 0.f;
              if (c0 != 0.f) a = __uint_as_float(o0[4 * i + e]) * c0;
              if (c1 != 0.f) a = fmaf(__uint_as_float(o1[4 * i + e]), c1, a);
              if (ct != 0.f) a = fmaf(tp[32 * q4 + 4 * i + e], ct, a);
              v[e] = a;
            }
            dst[i] = make_float4(v[0], v[1], v[2], v[3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

int launch_tile_attention(const TileMaps& maps, const float* sq, const float* sdq, const float* ks, const int32_t* idx,
                          int kx, int nb, int leaf, int64_t n, int tile_rows, int64_t t0, int64_t tc, int group,
                          float scale, const float* tail_part, const int32_t* perm, const float* dd, float* out,
                          float* lse, int* status, cudaStream_t st) {
  if (kx > kMaxKx || nb > 65535) return HTRC_ERR_UNSUPPORTED;
  if (leaf != 64 && leaf != 32 && leaf != 16) return HTRC_ERR_UNSUPPORTED;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    bool ok = true;
    for (auto k : {tile_attention_kernel<64, false, false>, tile_attention_kernel<32, false, false>,
                   tile_attention_kernel<64, true, false>, tile_attention_kernel<32, true, false>,
                   tile_attention_kernel<64, false, true>, tile_attention_kernel<32, false, true>})
      ok = ok && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) == cudaSuccess;
    if (!ok) return HTRC_ERR_CUDA;
    attr_done[dev] = true;
  }
  const int nf = kx >= nb ? 0 : (nb + 63) / 64;
  const unsigned grid = static_cast<unsigned>((tc + 1) / 2);
  const bool iso = dd != nullptr;
  if (iso && leaf != 64) return HTRC_ERR_UNSUPPORTED;
  auto kernel = leaf != 64 ? (tile_rows == 32 ? tile_attention_kernel<32, false, true>
                                              : tile_attention_kernel<64, false, true>)
                           : tile_rows == 32 ? (iso ? tile_attention_kernel<32, true, false>
                                                    : tile_attention_kernel<32, false, false>)
                                             : (iso ? tile_attention_kernel<64, true, false>
                                                    : tile_attention_kernel<64, false, false>);
  kernel<<<grid, kThreads, kSmemBytes, st>>>(maps.q8, maps.dq8, maps.g8, maps.vb, maps.lz, maps.sg, maps.excl, maps.k8,
                                             maps.v, maps.cv, dd, sq, sdq, ks, idx, kx, nb, nf, leaf, n, t0, tc,
                                             group > 1 ? group : 1, scale, tail_part, perm, out, lse, status);
  return cudaGetLastError() == cudaSuccess ? HTRC_OK : HTRC_ERR_CUDA;
}

}  // namespace htrc
