// Low-bit simulation and fp8 row dequantisation (h3/htrc_flat.py:68-97 `fake_quant`,
// h3/htrc_flat_triton.py:276-294 `dequant_rows`).
//
// fake_quant rounds every group of `gsz` consecutive values of a row through a low-bit format with a
// symmetric per-group scale s = max(amax, 1e-20) / qmax and writes s * code back:
//   int8 / int4: code = clamp(rint(x / s), -qmax, qmax), qmax 127 / 7 (round half to even);
//   fp8 (e4m3):  code = e4m3(clamp(x / s, -448, 448)) rounded to nearest even, qmax 448;
//   fp4 (e2m1):  code = sign(x) * grid[#(thresholds < |x / s|)], grid {0, .5, 1, 1.5, 2, 3, 4, 6}, qmax 6.
// One warp per 128-value row, four values per lane; a group spans gsz / 4 lanes (segmented shuffle
// maximum) or lies inside one lane (gsz 1 or 2).
#include "common.cuh"
#include "kernels.cuh"

namespace htrc {

namespace {
template <typename T>
__device__ __forceinline__ void load4q(const T* p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4q<float>(const float* p, float (&v)[4]) {
  const float4 x = *reinterpret_cast<const float4*>(p);
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
}
template <>
__device__ __forceinline__ void load4q<uint16_t>(const uint16_t* p, float (&v)[4]) {
  const uint2 x = *reinterpret_cast<const uint2*>(p);
  v[0] = __uint_as_float(x.x << 16); v[1] = __uint_as_float(x.x & 0xFFFF0000u);
  v[2] = __uint_as_float(x.y << 16); v[3] = __uint_as_float(x.y & 0xFFFF0000u);
}

__device__ __forceinline__ float e4m3_round(float t) {
  // nearest-even e4m3 value of t (|t| <= 448), as float
  uint16_t b;
  asm("{\n\t.reg .b16 r;\n\tcvt.rn.satfinite.e4m3x2.f32 r, %1, %1;\n\tmov.b16 %0, r;\n\t}" : "=h"(b) : "f"(t));
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(b));
  return __half2float(__ushort_as_half(static_cast<uint16_t>(h2 & 0xFFFFu)));
}

template <int FMT>
__device__ __forceinline__ float fq_value(float x, float s) {
  if (FMT == HTRC_FQ_INT8 || FMT == HTRC_FQ_INT4) {
    const float qmax = FMT == HTRC_FQ_INT8 ? 127.0f : 7.0f;
    const float c = fminf(fmaxf(rintf(__fdiv_rn(x, s)), -qmax), qmax);
    return __fmul_rn(c, s);
  } else if (FMT == HTRC_FQ_FP8) {
    const float t = fminf(fmaxf(__fdiv_rn(x, s), -448.0f), 448.0f);
    return __fmul_rn(e4m3_round(t), s);
  } else {
    const float a = fabsf(__fdiv_rn(x, s));
    const int i = (a > 0.25f) + (a > 0.75f) + (a > 1.25f) + (a > 1.75f) + (a > 2.5f) + (a > 3.5f) + (a > 5.0f);
    const float g = i < 4 ? 0.5f * static_cast<float>(i) : (i == 4 ? 2.0f : (i == 5 ? 3.0f : (i == 6 ? 4.0f : 6.0f)));
    const float sg = x > 0.f ? 1.0f : (x < 0.f ? -1.0f : 0.0f);
    return __fmul_rn(__fmul_rn(sg, g), s);
  }
}

template <typename T, typename O, int FMT>
__global__ void __launch_bounds__(256) fake_quant_kernel(const T* __restrict__ x, int64_t rows, int gsz,
                                                         O* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float qmax = FMT == HTRC_FQ_INT8 ? 127.0f : (FMT == HTRC_FQ_INT4 ? 7.0f : (FMT == HTRC_FQ_FP8 ? 448.0f : 6.0f));
  float v[4];
  load4q<T>(x + row * 128 + lane * 4, v);
  float am[4];
  if (gsz == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) am[i] = fabsf(v[i]);
  } else if (gsz == 2) {
    am[0] = am[1] = fmaxf(fabsf(v[0]), fabsf(v[1]));
    am[2] = am[3] = fmaxf(fabsf(v[2]), fabsf(v[3]));
  } else {
    float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    for (int o = 1; o < gsz / 4; o <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    am[0] = am[1] = am[2] = am[3] = a;
  }
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) y[i] = fq_value<FMT>(v[i], __fdiv_rn(fmaxf(am[i], 1e-20f), qmax));
  if constexpr (sizeof(O) == 4) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + row * 128 + lane * 4) =
        make_float4(y[0], y[1], y[2], y[3]);
  } else {
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(out) + row * 128 + lane * 4) =
        make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
  }
}

// out[r, :] = bf16(float(x8[r, :]) * scale[r]); one warp per row, four values per lane
__global__ void __launch_bounds__(256) dequant_rows_kernel(const uint8_t* __restrict__ x8, int64_t stride_x,
                                                           const float* __restrict__ scale, int64_t stride_s,
                                                           int64_t rows, uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint32_t w = *reinterpret_cast<const uint32_t*>(x8 + row * stride_x + lane * 4);
  const float sc = scale[row * stride_s];
  uint32_t h01, h23;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h01) : "h"(static_cast<uint16_t>(w & 0xFFFFu)));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h23) : "h"(static_cast<uint16_t>(w >> 16)));
  const float f0 = __half2float(__ushort_as_half(static_cast<uint16_t>(h01 & 0xFFFFu)));
  const float f1 = __half2float(__ushort_as_half(static_cast<uint16_t>(h01 >> 16)));
  const float f2 = __half2float(__ushort_as_half(static_cast<uint16_t>(h23 & 0xFFFFu)));
  const float f3 = __half2float(__ushort_as_half(static_cast<uint16_t>(h23 >> 16)));
  *reinterpret_cast<uint2*>(out + row * 128 + lane * 4) =
      make_uint2(pack_bf16x2(__fmul_rn(f0, sc), __fmul_rn(f1, sc)), pack_bf16x2(__fmul_rn(f2, sc), __fmul_rn(f3, sc)));
}

template <typename T, typename O>
void launch_fq(const void* x, int64_t rows, int fmt, int gsz, void* out, cudaStream_t st) {
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  const T* xi = static_cast<const T*>(x);
  O* o = static_cast<O*>(out);
  switch (fmt) {
    case HTRC_FQ_INT8: fake_quant_kernel<T, O, HTRC_FQ_INT8><<<grid, 256, 0, st>>>(xi, rows, gsz, o); break;
    case HTRC_FQ_INT4: fake_quant_kernel<T, O, HTRC_FQ_INT4><<<grid, 256, 0, st>>>(xi, rows, gsz, o); break;
    case HTRC_FQ_FP8: fake_quant_kernel<T, O, HTRC_FQ_FP8><<<grid, 256, 0, st>>>(xi, rows, gsz, o); break;
    default: fake_quant_kernel<T, O, HTRC_FQ_FP4><<<grid, 256, 0, st>>>(xi, rows, gsz, o); break;
  }
}
}  // namespace

void launch_fake_quant(const void* x, int x_dtype, int64_t rows, int fmt, int gsz, void* out, int out_dtype,
                       cudaStream_t st) {
  const bool xb = x_dtype == HTRC_DTYPE_BF16, ob = out_dtype == HTRC_DTYPE_BF16;
  if (xb && ob) launch_fq<uint16_t, uint16_t>(x, rows, fmt, gsz, out, st);
  else if (xb) launch_fq<uint16_t, float>(x, rows, fmt, gsz, out, st);
  else if (ob) launch_fq<float, uint16_t>(x, rows, fmt, gsz, out, st);
  else launch_fq<float, float>(x, rows, fmt, gsz, out, st);
}

void launch_dequant_rows(const uint8_t* x8, int64_t stride_x, const float* scale, int64_t stride_s, int64_t rows,
                         uint16_t* out, cudaStream_t st) {
  dequant_rows_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(x8, stride_x, scale, stride_s, rows, out);
}

}  // namespace htrc
