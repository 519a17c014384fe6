// HBM-bound preparation kernels: INT8 row packing of keys (and of any [rows, 128] matrix), tile
// centres + query codes, and the exact tail-key partial.
#include "common.cuh"
#include "kernels.cuh"

namespace htrc {

namespace {
constexpr float kInv127 = 1.0f / 127.0f;  // float32 of the reference's (1.0 / 127.0)

template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&v)[4]) {
  float4 x = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
}
template <>
__device__ __forceinline__ void load4<uint16_t>(const uint16_t* p, float (&v)[4]) {
  uint2 x = __ldg(reinterpret_cast<const uint2*>(p));
  v[0] = __uint_as_float(x.x << 16); v[1] = __uint_as_float(x.x & 0xFFFF0000u);
  v[2] = __uint_as_float(x.y << 16); v[3] = __uint_as_float(x.y & 0xFFFF0000u);
}

// sum of squares of a 128-value row held four values per lane (fp32, lane products then a tree)
__device__ __forceinline__ float row_sqnorm(const float (&v)[4]) {
  float s = __fmaf_rn(v[3], v[3], __fmaf_rn(v[2], v[2], __fmaf_rn(v[1], v[1], __fmul_rn(v[0], v[0]))));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  return s;
}

__device__ __forceinline__ uint32_t pack_i8x4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

// INT8 code of v / s (s > 0, |v / s| <= 127 + rounding): ROUND 1 = the reference's half-away
// trunc(fl(fl(v / s) +- 0.5)), ROUND 0 = half-even rint(fl(v / s)) clamped to +-127.  The quotient is
// taken as v * r with r = 1/s correctly rounded (within 2^-22 relative of v / s, so within 4e-5 of it
// for |v / s| < 128) and the code is read from it, unless it lies within 2^-12 of a rounding boundary
// k + 1/2, where the correctly rounded quotient and the reference's formula decide.  Away from the
// boundaries both rounding modes give the nearest integer.  No transcendental-unit instruction on the
// fast path: floor and nearest integer come from adding 2^23 (toward zero / to nearest).
template <int ROUND, bool DIVF = false>
__device__ __forceinline__ int quant_code(float v, float s, float r) {
  const float ya = __fmul_rn(v, r);
  const float h = __fadd_rn(fabsf(ya), 0.5f);                          // boundaries -> integers
  const float n = __fsub_rn(__fadd_rn(h, 12582912.0f), 12582912.0f);   // nearest integer to h
  if (fabsf(__fsub_rn(h, n)) < 2.44140625e-4f) {
    const float y = DIVF ? div_full(v, s) : __fdiv_rn(v, s);
    if (ROUND == 0) return max(-127, min(127, static_cast<int>(rintf(y))));
    return round_half_away_i8(y);
  }
  const int k = min(127, __float_as_int(__fadd_rz(h, 8388608.0f)) - 0x4B000000);   // floor(h)
  return ya < 0.f ? -k : k;
}

// x8 codes of 4 values given the row scale s and its reciprocal r: the fast path of quant_code on pairs
// (paired fp32 arithmetic), the exact quotient only for the values near a rounding boundary (rare: the
// whole warp takes that branch only when one of its lanes needs it)
template <int ROUND, bool DIVF = false>
__device__ __forceinline__ uint32_t quant4(const float (&v)[4], float s, float r) {
  const float2 r2 = make_float2(r, r);
  const float2 m2 = make_float2(12582912.0f, 12582912.0f);
  int c[4];
  bool near = false;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const float2 ya = mul2(make_float2(v[2 * p], v[2 * p + 1]), r2);
    const float2 h = make_float2(__fadd_rn(fabsf(ya.x), 0.5f), __fadd_rn(fabsf(ya.y), 0.5f));
    const float2 t = add2(h, m2);                 // nearest integer of h in the low mantissa bits
    const float2 nn = sub2(t, m2);
    const float2 e = sub2(h, nn);
    near |= (fabsf(e.x) < 2.44140625e-4f) | (fabsf(e.y) < 2.44140625e-4f);
    const int k0 = (__float_as_int(t.x) - 0x4B400000) - (h.x < nn.x);      // floor(h)
    const int k1 = (__float_as_int(t.y) - 0x4B400000) - (h.y < nn.y);
    c[2 * p] = ya.x < 0.f ? -k0 : k0;
    c[2 * p + 1] = ya.y < 0.f ? -k1 : k1;
  }
  if (__any_sync(0xffffffffu, near)) {
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = quant_code<ROUND, DIVF>(v[i], s, r);
  }
  return pack_i8x4(c[0], c[1], c[2], c[3]);
}
}  // namespace

// One warp per kPackRows rows of 128 values (all of its loads issued first, for memory-level parallelism);
// each lane owns 4 consecutive values of a row.
constexpr int kPackRows = 4;
template <typename T, int ROUND>
__global__ void __launch_bounds__(256) pack_rows_kernel(const T* __restrict__ x, int64_t rows,
                                                        int8_t* __restrict__ x8, float* __restrict__ scale,
                                                        float* __restrict__ sqnorm) {
  const int lane = threadIdx.x & 31;
  const int64_t r0 = (static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * kPackRows;
  float v[kPackRows][4];
#pragma unroll
  for (int i = 0; i < kPackRows; ++i)
    if (r0 + i < rows) load4<T>(x + (r0 + i) * 128 + lane * 4, v[i]);
#pragma unroll
  for (int i = 0; i < kPackRows; ++i) {
    const int64_t row = r0 + i;
    if (row >= rows) break;                  // warp-uniform
    float am = fmaxf(fmaxf(fabsf(v[i][0]), fabsf(v[i][1])), fmaxf(fabsf(v[i][2]), fabsf(v[i][3])));
    am = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(am)));   // non-negative: uint order
    const float s = fmaxf(__fmul_rn(am, kInv127), 1e-20f);
    reinterpret_cast<uint32_t*>(x8 + row * 128)[lane] = quant4<ROUND>(v[i], s, __frcp_rn(s));
    if (lane == 0) scale[row] = s;
    if (sqnorm != nullptr) {               // |x_row|^2 (the iso curvature's key norms)
      const float n2 = row_sqnorm(v[i]);
      if (lane == 0) sqnorm[row] = n2;
    }
  }
}

// The same codes with one scale per block of 64 consecutive rows (an extension: one absmax scale per
// 64-token block; the reference's are per row): s = max(amax_block|x| * (1/127), 1e-20),
// written once per row.  One CTA per block; warp w holds rows 8w .. 8w + 7 in registers, the block maximum
// goes through shared memory.
template <typename T, int ROUND>
__global__ void __launch_bounds__(256) pack_blocks_kernel(const T* __restrict__ x, int64_t rows,
                                                          int8_t* __restrict__ x8, float* __restrict__ scale,
                                                          float* __restrict__ sqnorm) {
  __shared__ float bam[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * 64 + warp * 8;
  float v[8][4];
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (r0 + i < rows) {
      load4<T>(x + (r0 + i) * 128 + lane * 4, v[i]);
    } else {
      v[i][0] = v[i][1] = v[i][2] = v[i][3] = 0.f;
    }
    am = fmaxf(am, fmaxf(fmaxf(fabsf(v[i][0]), fabsf(v[i][1])), fmaxf(fabsf(v[i][2]), fabsf(v[i][3]))));
  }
  am = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(am)));
  if (lane == 0) bam[warp] = am;
  __syncthreads();
  float b = bam[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) b = fmaxf(b, bam[w]);
  const float s = fmaxf(__fmul_rn(b, kInv127), 1e-20f);
  const float r = __frcp_rn(s);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t row = r0 + i;
    if (row >= rows) break;                  // warp-uniform
    reinterpret_cast<uint32_t*>(x8 + row * 128)[lane] = quant4<ROUND>(v[i], s, r);
    if (lane == 0) scale[row] = s;
    if (sqnorm != nullptr) {
      const float n2 = row_sqnorm(v[i]);
      if (lane == 0) sqnorm[row] = n2;
    }
  }
}

void launch_pack_blocks(const void* x, int dtype, int64_t rows, int rounding, int8_t* x8, float* scale,
                        float* sqnorm, cudaStream_t st) {
  const unsigned grid = static_cast<unsigned>((rows + 63) / 64);
  if (dtype == HTRC_DTYPE_BF16) {
    if (rounding == HTRC_ROUND_HALF_EVEN)
      pack_blocks_kernel<uint16_t, 0><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(x), rows, x8, scale, sqnorm);
    else
      pack_blocks_kernel<uint16_t, 1><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(x), rows, x8, scale, sqnorm);
  } else {
    if (rounding == HTRC_ROUND_HALF_EVEN)
      pack_blocks_kernel<float, 0><<<grid, 256, 0, st>>>(static_cast<const float*>(x), rows, x8, scale, sqnorm);
    else
      pack_blocks_kernel<float, 1><<<grid, 256, 0, st>>>(static_cast<const float*>(x), rows, x8, scale, sqnorm);
  }
}

void launch_pack_rows(const void* x, int dtype, int64_t rows, int rounding, int8_t* x8, float* scale,
                      float* sqnorm, cudaStream_t st) {
  const unsigned grid = static_cast<unsigned>((rows + 8 * kPackRows - 1) / (8 * kPackRows));
  if (dtype == HTRC_DTYPE_BF16) {
    if (rounding == HTRC_ROUND_HALF_EVEN)
      pack_rows_kernel<uint16_t, 0><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(x), rows, x8, scale, sqnorm);
    else
      pack_rows_kernel<uint16_t, 1><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(x), rows, x8, scale, sqnorm);
  } else {
    if (rounding == HTRC_ROUND_HALF_EVEN)
      pack_rows_kernel<float, 0><<<grid, 256, 0, st>>>(static_cast<const float*>(x), rows, x8, scale, sqnorm);
    else
      pack_rows_kernel<float, 1><<<grid, 256, 0, st>>>(static_cast<const float*>(x), rows, x8, scale, sqnorm);
  }
}

// Row of q that row r of tile t holds.  Tiles of T = 64 or 32 query rows are held as 64 rows: a 32-row
// tile's rows 32..63 repeat its row 31, which changes no centre (taken over the real rows), no row
// maximum and no output (only rows < T are written).  Rows past n repeat the last row (the reference
// pads the last tile that way, h3/htrc_flat.py:150-152), after the optional k-means permutation
// (:146-147).
__device__ __forceinline__ int64_t source_row(const int32_t* perm, int64_t n, int trows, int64_t t, int r) {
  const int64_t li = t * trows + (r < trows ? r : trows - 1);
  const int64_t c = li < n - 1 ? li : n - 1;
  return perm ? static_cast<int64_t>(__ldg(perm + c)) : c;
}

// The centre in float32, and as the two bf16 parts the leaf statistics multiply with: hi + lo is the centre to
// ~2^-16 relative (precision "fp32"), or exactly its tf32 operand value, the low 13 mantissa bits cleared, when
// tmask = kTf32Mask (precision "tf32": the reference's tensor-core dots read float32 operands that way; an
// 11-bit significand splits exactly into bf16 hi + lo)
__device__ __forceinline__ void store_centre(int64_t c, int col, float m, float* mu, uint16_t* mu_hi,
                                             uint16_t* mu_lo, uint32_t tmask) {
  mu[c * 128 + col] = m;
  const float mt = __uint_as_float(__float_as_uint(m) & tmask);
  const __nv_bfloat16 hi = __float2bfloat16_rn(mt);
  const __nv_bfloat16 lo = __float2bfloat16_rn(__fsub_rn(mt, __bfloat162float(hi)));
  mu_hi[c * 128 + col] = __bfloat16_as_ushort(hi);
  mu_lo[c * 128 + col] = __bfloat16_as_ushort(lo);
}

// Centres of groups of G > 1 consecutive tiles (h3/htrc_flat.py:223-231): the mean of all G * T rows
// of the padded tiles -- the last tile's rows past n repeat the last row and the tiles that fill the
// last group repeat the last tile.  One CTA per group, thread = column; float64 sum rounded once.
template <typename T>
__global__ void __launch_bounds__(128) group_centre_kernel(const T* __restrict__ q, const int32_t* __restrict__ perm,
                                                           int64_t n, int trows, int64_t nt, int group,
                                                           float* __restrict__ mu, uint16_t* __restrict__ mu_hi,
                                                           uint16_t* __restrict__ mu_lo, uint32_t tmask) {
  const int64_t g = blockIdx.x;
  const int col = threadIdx.x;
  double s = 0.0;
  for (int x = 0; x < group; ++x) {
    const int64_t t = g * group + x < nt ? g * group + x : nt - 1;
#pragma unroll 8
    for (int r = 0; r < trows; ++r) {
      const int64_t src = source_row(perm, n, trows, t, r);
      if constexpr (sizeof(T) == 4)
        s += static_cast<double>(__ldg(reinterpret_cast<const float*>(q) + src * 128 + col));
      else
        s += static_cast<double>(__uint_as_float(static_cast<uint32_t>(__ldg(q + src * 128 + col)) << 16));
    }
  }
  store_centre(g, col, static_cast<float>(s / static_cast<double>(group * trows)), mu, mu_hi, mu_lo, tmask);
}

// One CTA (4 warps) per tile of T query rows (held as 64 rows): the tile's centre (group 1; else the
// group centre written by group_centre_kernel) and the codes of its rows and of their offsets from
// the centre.  qblock (an extension): one scale for the codes of all 64 held rows, from the tile's
// abs-max (the held rows repeat real rows, so it is the maximum over the tile's queries); the offsets'
// codes keep per-row scales.  FP8 (the fp8 state path, h3/htrc_flat_triton.py:103-109) writes instead the rows as bf16
// (q8 holds uint16 bf16 rows) and the float32 offsets rounded once to fp16 (dq8 holds uint16 fp16 rows), or, with
// dqbf (the bf16 state, :106-107), to bf16; sq / sdq are not written.
template <typename T, bool FP8>
__global__ void __launch_bounds__(128) tile_prep_kernel(const T* __restrict__ q, const int32_t* __restrict__ perm,
                                                        int64_t n, int trows, int group, float* __restrict__ mu,
                                                        uint16_t* __restrict__ mu_hi, uint16_t* __restrict__ mu_lo,
                                                        int8_t* __restrict__ q8, float* __restrict__ sq,
                                                        int8_t* __restrict__ dq8, float* __restrict__ sdq,
                                                        float* __restrict__ dd, int qblock, uint32_t tmask,
                                                        int tdiv, int dqbf) {
  // row pitch 132 floats: a lane's 4 values are one aligned 16-byte access (a warp's row read or write is
  // conflict-free), and the column walk of the centre (thread = column, one row at a time) hits 32 banks
  __shared__ __align__(16) float qs[64][132];
  __shared__ float mus[128];
  __shared__ float tmx[4];
  const int t = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t r0 = static_cast<int64_t>(t) * 64;              // first of the tile's 64 held rows
  const int64_t first = static_cast<int64_t>(t) * trows;         // its first query (in tile order)
  const int nreal = static_cast<int>(n - first < trows ? n - first : trows);
  // stage the tile: warp w loads rows w, w+4, ...; lane owns 4 columns; all 16 loads of a warp in flight
  const int warp = tid >> 5, lane = tid & 31;
  {
    int64_t src[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) src[i] = source_row(perm, n, trows, t, warp + 4 * i);
    float v[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) load4<T>(q + src[i] * 128 + lane * 4, v[i]);
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
      *reinterpret_cast<float4*>(&qs[warp + 4 * i][lane * 4]) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
  }
  __syncthreads();
  if (group <= 1) {
    // centre: float64 sum over the real rows, divided and rounded once
    double s = 0.0;
    for (int r = 0; r < nreal; ++r) s += static_cast<double>(qs[r][tid]);
    const float m = static_cast<float>(s / static_cast<double>(nreal));
    mus[tid] = m;
    store_centre(t, tid, m, mu, mu_hi, mu_lo, tmask);
  } else {
    mus[tid] = mu[static_cast<int64_t>(t / group) * 128 + tid];
  }
  __syncthreads();
  float m4[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) m4[i] = mus[lane * 4 + i];
  float tq = 0.f;                            // qblock: the tile's abs-max (thread = column, then CTA)
  if (qblock) {
    float cm = 0.f;
    for (int r = 0; r < 64; ++r) cm = fmaxf(cm, fabsf(qs[r][tid]));
    cm = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(cm)));
    if (lane == 0) tmx[warp] = cm;
    __syncthreads();
    tq = fmaxf(fmaxf(tmx[0], tmx[1]), fmaxf(tmx[2], tmx[3]));
  }
#pragma unroll 4
  for (int r = warp; r < 64; r += 4) {
    float v[4], d[4];
    {
      const float4 x = *reinterpret_cast<const float4*>(&qs[r][lane * 4]);
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = __fsub_rn(v[i], m4[i]);
    const int64_t gr = r0 + r;
    if constexpr (FP8) {
      reinterpret_cast<uint2*>(q8 + gr * 256)[lane] = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
      reinterpret_cast<uint2*>(dq8 + gr * 256)[lane] =
          dqbf ? make_uint2(pack_bf16x2(d[0], d[1]), pack_bf16x2(d[2], d[3]))
               : make_uint2(pack_f16x2(d[0], d[1]), pack_f16x2(d[2], d[3]));
      continue;
    }
    float aq = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    float ad = fmaxf(fmaxf(fabsf(d[0]), fabsf(d[1])), fmaxf(fabsf(d[2]), fabsf(d[3])));
    aq = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(aq)));
    ad = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(ad)));
    const float s_q = fmaxf(__fmul_rn(qblock ? tq : aq, kInv127), 1e-20f);
    const float s_d = fmaxf(__fmul_rn(ad, kInv127), 1e-20f);
    // the quotient x / s decides a code only near a rounding boundary: there it is the IEEE quotient (the
    // reference's formula as written), or div.full.f32 (tdiv: what its Triton kernels compute on the GPU)
    if (tdiv) {
      reinterpret_cast<uint32_t*>(q8 + gr * 128)[lane] = quant4<1, true>(v, s_q, __frcp_rn(s_q));
      reinterpret_cast<uint32_t*>(dq8 + gr * 128)[lane] = quant4<1, true>(d, s_d, __frcp_rn(s_d));
    } else {
      reinterpret_cast<uint32_t*>(q8 + gr * 128)[lane] = quant4<1>(v, s_q, __frcp_rn(s_q));
      reinterpret_cast<uint32_t*>(dq8 + gr * 128)[lane] = quant4<1>(d, s_d, __frcp_rn(s_d));
    }
    if (lane == 0) {
      sq[gr] = s_q;
      sdq[gr] = s_d;
    }
    if (dd != nullptr) {                     // |q - mu|^2 in float32 (the iso curvature's offsets)
      const float n2 = row_sqnorm(d);
      if (lane == 0) dd[gr] = n2;
    }
  }
}

void launch_tile_prep(const void* q, int dtype, int64_t n, int tile_rows, const int32_t* perm, int group, float* mu,
                      uint16_t* mu_hi, uint16_t* mu_lo, int8_t* q8, float* sq, int8_t* dq8, float* sdq, float* dd,
                      bool fp8, bool qblock, bool tf32, bool tdiv, cudaStream_t st, bool dq_bf16) {
  const int tr = tile_rows == 32 ? 32 : 64;
  const uint32_t tmask = tf32 ? kTf32Mask : 0xFFFFFFFFu;
  const int64_t nt = (n + tr - 1) / tr;
  const int g = group > 1 ? group : 1;
  const unsigned ng = static_cast<unsigned>((nt + g - 1) / g);
  if (dtype == HTRC_DTYPE_BF16) {
    const uint16_t* qb = static_cast<const uint16_t*>(q);
    if (g > 1) group_centre_kernel<uint16_t><<<ng, 128, 0, st>>>(qb, perm, n, tr, nt, g, mu, mu_hi, mu_lo, tmask);
    auto k = fp8 ? tile_prep_kernel<uint16_t, true> : tile_prep_kernel<uint16_t, false>;
    k<<<static_cast<unsigned>(nt), 128, 0, st>>>(qb, perm, n, tr, g, mu, mu_hi, mu_lo, q8, sq, dq8, sdq, dd,
                                                 qblock ? 1 : 0, tmask, tdiv ? 1 : 0, dq_bf16 ? 1 : 0);
  } else {
    const float* qf = static_cast<const float*>(q);
    if (g > 1) group_centre_kernel<float><<<ng, 128, 0, st>>>(qf, perm, n, tr, nt, g, mu, mu_hi, mu_lo, tmask);
    auto k = fp8 ? tile_prep_kernel<float, true> : tile_prep_kernel<float, false>;
    k<<<static_cast<unsigned>(nt), 128, 0, st>>>(qf, perm, n, tr, g, mu, mu_hi, mu_lo, q8, sq, dq8, sdq, dd,
                                                 qblock ? 1 : 0, tmask, tdiv ? 1 : 0, dq_bf16 ? 1 : 0);
  }
}

// Exact partial of each query row against the n_tail tail keys: one warp per row.
//   n_tail <= 16: logits from bf16-rounded q and keys, P rounded to bf16 for the value product
//                 (h3/htrc_flat_triton.py:187-207); otherwise float32 (h3/htrc_flat_triton.py:381-388).
// Output row: acc[128], m, l  (natural-log units).
template <typename T>
__global__ void __launch_bounds__(256) tail_partial_kernel(const T* __restrict__ q, int64_t n,
                                                           const float* __restrict__ tk, const float* __restrict__ tv,
                                                           int n_tail, float scale, float* __restrict__ part) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= n) return;
  const bool small = n_tail <= 16;
  float qv[4];
  load4<T>(q + row * 128 + lane * 4, qv);
  if (small) {
#pragma unroll
    for (int i = 0; i < 4; ++i) qv[i] = __bfloat162float(__float2bfloat16_rn(qv[i]));
  }
  float m = -INFINITY;
  for (int j = 0; j < n_tail; ++j) {
    float kv[4];
    load4<float>(tk + static_cast<int64_t>(j) * 128 + lane * 4, kv);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float kk = small ? __bfloat162float(__float2bfloat16_rn(kv[i])) : kv[i];
      s = fmaf(qv[i], kk, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    m = fmaxf(m, s * scale);
  }
  float l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < n_tail; ++j) {
    float kv[4], vv[4];
    load4<float>(tk + static_cast<int64_t>(j) * 128 + lane * 4, kv);
    load4<float>(tv + static_cast<int64_t>(j) * 128 + lane * 4, vv);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float kk = small ? __bfloat162float(__float2bfloat16_rn(kv[i])) : kv[i];
      s = fmaf(qv[i], kk, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float p = expf(s * scale - m);
    l += p;
    const float pv = small ? __bfloat162float(__float2bfloat16_rn(p)) : p;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float vvv = small ? __bfloat162float(__float2bfloat16_rn(vv[i])) : vv[i];
      acc[i] = fmaf(pv, vvv, acc[i]);
    }
  }
  float* o = part + row * 130;
#pragma unroll
  for (int i = 0; i < 4; ++i) o[lane * 4 + i] = acc[i];
  if (lane == 0) {
    o[128] = m;
    o[129] = l;
  }
}

void launch_tail_partial(const void* q, int dtype, int64_t n, const float* tk, const float* tv, int n_tail, float scale,
                         float* part, cudaStream_t st) {
  const unsigned grid = static_cast<unsigned>((n + 7) / 8);
  if (dtype == HTRC_DTYPE_BF16)
    tail_partial_kernel<uint16_t><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(q), n, tk, tv, n_tail, scale,
                                                        part);
  else
    tail_partial_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(q), n, tk, tv, n_tail, scale, part);
}

}  // namespace htrc
