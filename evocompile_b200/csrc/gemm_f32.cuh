// fp32 GEMM with the same fused epilogues, for fp32 operands.
//
// tcgen05 has no full-precision fp32 kind (kind::tf32 rounds operands to 10
// mantissa bits), and the fp32 contract is "rel 1e-3 with TF32 disabled", so
// fp32 inputs run on the CUDA cores with exact fp32 FMA. Tile 64 x 64 outputs
// (SwiGLU: 64 gate + 64 up columns), K step 16, 256 threads, 4 x 4 outputs per
// thread; operands are read through arbitrary element strides.
#pragma once

#include "gemm_sm100.cuh"

namespace gko {
namespace gemm_f32 {

constexpr int kTile = 64;
constexpr int kBK = 16;

template <int EPI>
__global__ void __launch_bounds__(256) kernel(const float* __restrict__ A, int64_t sam, int64_t sak,
                                              const float* __restrict__ B, int64_t sbk,
                                              int64_t sbn, float* __restrict__ D, int64_t ldd,
                                              const GemmParams p) {
  constexpr bool kSwiglu = (EPI == kEpiSwiglu);
  __shared__ float As[kBK][kTile + 4];
  __shared__ float Bs[kBK][kTile + 4];
  __shared__ float Us[kSwiglu ? kBK : 1][kSwiglu ? kTile + 4 : 1];

  const int tx = threadIdx.x & 15;
  const int ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kTile;
  const int n0 = blockIdx.x * kTile;
  float acc[4][4] = {};
  float accu[kSwiglu ? 4 : 1][kSwiglu ? 4 : 1] = {};

  for (int k0 = 0; k0 < p.K; k0 += kBK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = threadIdx.x + i * 256;  // 0..1023
      // A tile: 64 rows x 16 k  (k fastest for row-major A)
      const int ar = idx >> 4, ak = idx & 15;
      const int gm = m0 + ar, gk = k0 + ak;
      As[ak][ar] = (gm < p.M && gk < p.K) ? A[gm * sam + gk * sak] : 0.f;
      // B tile: 16 k x 64 n  (n fastest)
      const int bk = idx >> 6, bn = idx & 63;
      const int gk2 = k0 + bk, gn = n0 + bn;
      const bool okb = (gk2 < p.K && gn < p.N_out);
      Bs[bk][bn] = okb ? B[gk2 * sbk + gn * sbn] : 0.f;
      if constexpr (kSwiglu)
        Us[bk][bn] = okb ? B[gk2 * sbk + (gn + p.up_offset) * sbn] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      if constexpr (kSwiglu) {
        float u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) u[j] = Us[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) accu[i][j] = fmaf(a[i], u[j], accu[i][j]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= p.N_out) continue;
      float x = acc[i][j];
      if constexpr (kSwiglu) {
        x = gemm::silu(x) * accu[i][j];
      } else {
        x += gemm::load_bias(p.bias, p.bias_kind, gn, p.N_out);
        if constexpr (EPI == kEpiGelu) x = gemm::gelu_erf(x);
        if constexpr (EPI == kEpiRelu) x = fmaxf(x, 0.f);
      }
      D[gm * ldd + gn] = x;
    }
  }
}

}  // namespace gemm_f32
}  // namespace gko
