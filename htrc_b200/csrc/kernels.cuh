// Internal launchers of the flat HTRC kernels (one translation unit per kernel family).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace htrc {

// precision "tf32": a float32 operand's value as the tensor cores read it in tf32 (low 13 mantissa bits cleared)
constexpr uint32_t kTf32Mask = 0xFFFFE000u;

struct LeafStatsMaps {
  const uint16_t* mu_hi;      // [nt, 128] bf16 rows (loaded into TMEM by the kernel)
  const uint16_t* mu_lo;
  int64_t nt;
  CUtensorMap k, v;           // [M, 128] bf16 as [2][M][64], box (64, 64, 2), 128B swizzle
  CUtensorMap g8;             // [tc, nb, 128] int8 (store), box (128, 1, 128), 128B swizzle; bf16 state: as vb
  CUtensorMap vb;             // [tc, nb, 128] bf16 (store), box (64, 1, 128), 128B swizzle; fp8: codes as g8
};

// state arrays hold one row per centre: per tile, or per group of tiles (rows [tc] below)
struct RowmaxMaps {
  CUtensorMap dq8;            // [nt*64, 128] int8, box (128, 64), 128B swizzle; bf16 state: bf16 dq as [2][rows][64]
  CUtensorMap g8;             // [tc, nb, 128] int8, box (128, 128, 1), 128B swizzle; bf16 state: [tc][2][nb][64]
  CUtensorMap sg, lz;         // [tc, nb] f32 (row pitch P), box (128, 1); sg unused with the bf16 state
  CUtensorMap cv;             // iso curvature coefficients, as sg (unused without ISO: any valid map)
};

struct TileMaps {
  CUtensorMap q8, dq8;        // [nt*64, 128] int8, box (128, 64), 128B swizzle
  CUtensorMap g8;             // [tc, nb, 128] int8, box (128, 64, 1), 128B swizzle
  CUtensorMap vb;             // [tc, nb, 128] bf16 as [tc][2][nb][64], box (64, 64, 2, 1), 128B swizzle
  CUtensorMap lz, sg;         // [tc, nb] f32 (row pitch P), box (64, 1)
  CUtensorMap excl;           // [tc, nb] u8 (row pitch P), box (64, 1)
  CUtensorMap k8;             // [M, 128] int8, box (128, 64), 128B swizzle
  CUtensorMap v;              // [M, 128] bf16 as [2][M][64], box (64, 64, 2), 128B swizzle
  CUtensorMap cv;             // iso curvature coefficients [tc, nb] f32 (row pitch P), box (64, 1); any valid map
};

// fp8 (e4m3) state path
struct RowmaxFp8Maps {
  CUtensorMap dqh;            // [nt*64, 128] fp16 as [2][rows][64], box (64, 64, 2), 128B swizzle
  CUtensorMap graw;           // [tc, nb, 128] e4m3 codes, box (128, 128, 1), no swizzle
  CUtensorMap sg, lz;         // [tc, nb] f32 (row pitch P), box (128, 1)
};

struct TileFp8Maps {
  CUtensorMap qb, dqh;        // [nt*64, 128] bf16 / fp16 as [2][rows][64], box (64, 64, 2), 128B swizzle
  CUtensorMap graw, vraw;     // [tc, nb, 128] e4m3 codes of g / vbar, box (128, 64, 1), 128B swizzle; bf16 state:
                              // bf16 g / vbar as [tc][2][nb][64], box (64, 64, 2, 1)
  CUtensorMap lz, sg, sv;     // [tc, nb] f32 (row pitch P), box (64, 1)
  CUtensorMap excl;           // [tc, nb] u8 (row pitch P), box (64, 1)
  CUtensorMap k, v;           // [M, 128] bf16 as [2][M][64], box (64, 64, 2), 128B swizzle
};

void launch_pack_rows(const void* x, int dtype, int64_t rows, int rounding, int8_t* x8, float* scale, float* sqnorm,
                      cudaStream_t st);
void launch_tile_prep(const void* q, int dtype, int64_t n, int tile_rows, const int32_t* perm, int group, float* mu,
                      uint16_t* mu_hi, uint16_t* mu_lo, int8_t* q8, float* sq, int8_t* dq8, float* sdq, float* dd,
                      bool fp8, bool qblock, bool tf32, bool tdiv, cudaStream_t st,
                      bool dq_bf16 = false);
void launch_pack_blocks(const void* x, int dtype, int64_t rows, int rounding, int8_t* x8, float* scale,
                        float* sqnorm, cudaStream_t st);
size_t kmeans_scratch_bytes(int64_t n);
int launch_kmeans_order(const void* q, int dtype, int64_t n, int32_t* perm, void* scratch, cudaStream_t st);
void kmeans_views(void* scratch, int64_t n, float** centres, uint8_t** assign);
void launch_fake_quant(const void* x, int x_dtype, int64_t rows, int fmt, int gsz, void* out, int out_dtype,
                       cudaStream_t st);
void launch_dequant_rows(const uint8_t* x8, int64_t stride_x, const float* scale, int64_t stride_s, int64_t rows,
                         uint16_t* out, cudaStream_t st);
void launch_tail_partial(const void* q, int dtype, int64_t n, const float* tk, const float* tv, int n_tail, float scale,
                         float* part, cudaStream_t st);
// leaf: 64, or 32 / 16 for the INT8 state with the linear far field
// bf16_state: g and vbar stored as bf16 without scales (sg, sv, kn2, cv unused; leaf 64)
int launch_leaf_stats(const LeafStatsMaps& maps, float* sg, float* lz, int64_t pitch, int64_t t0, int64_t tc, int nb,
                      int leaf, float scale, const float* kn2, float* cv, float* sv, int* status, int num_sms,
                      bool tf32, bool tdiv, cudaStream_t st, bool bf16_state = false);
int launch_rowmax(const RowmaxMaps& maps, const float* sdq, const float* dd, float* sel, int64_t pitch, int64_t t0,
                  int64_t tc, int nb, int group, int* status, cudaStream_t st, bool bf16_state = false);
int launch_route(const float* sel, int64_t pitch, int64_t tc, int group, int nb, int kx, int sink, int32_t* idx,
                 uint8_t* excl, cudaStream_t st);
// the maps' key-leaf boxes (k8, v) are `leaf` rows high
int launch_tile_attention(const TileMaps& maps, const float* sq, const float* sdq, const float* ks, const int32_t* idx,
                          int kx, int nb, int leaf, int64_t n, int tile_rows, int64_t t0, int64_t tc, int group, float scale,
                          const float* tail_part, const int32_t* perm, const float* dd, float* out, float* lse,
                          int* status, cudaStream_t st);
int launch_rowmax_fp8(const RowmaxFp8Maps& maps, float* sel, int64_t pitch, int64_t t0, int64_t tc, int nb, int group,
                      int* status, cudaStream_t st);
int launch_tile_fp8(const TileFp8Maps& maps, const int32_t* idx, int kx, int nb, int64_t n, int tile_rows, int64_t t0,
                    int64_t tc, int group, float scale, const float* tail_part, const int32_t* perm, float* far_part,
                    float* out, float* lse, int* status, cudaStream_t st, bool bf16_state = false);

}  // namespace htrc
