// out = silu(x) * y, elementwise (gko::silu_mul), and the SwiGLU backward from saved
// pre-activations (gko_swiglu_bwd). HBM-bound: 16-byte vector loads/stores, grid sized to a
// multiple of the SM count, grid-stride loop.
#include "host_common.h"
#include "sm100_ptx.cuh"

namespace {

template <typename T>
__global__ void __launch_bounds__(256) silu_mul_vec(const T* __restrict__ x, const T* __restrict__ y,
                                                    T* __restrict__ out, int64_t n) {
  constexpr int kVec = 16 / sizeof(T);
  const int64_t nvec = n / kVec;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x) + i);
    const uint4 yv = __ldg(reinterpret_cast<const uint4*>(y) + i);
    uint4 ov;
    const T* xs = reinterpret_cast<const T*>(&xv);
    const T* ys = reinterpret_cast<const T*>(&yv);
    T* os = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const float a = static_cast<float>(xs[j]);
      const float b = static_cast<float>(ys[j]);
      os[j] = static_cast<T>(a / (1.f + __expf(-a)) * b);
    }
    reinterpret_cast<uint4*>(out)[i] = ov;
  }
  // tail
  for (int64_t i = nvec * kVec + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float a = static_cast<float>(x[i]);
    const float b = static_cast<float>(y[i]);
    out[i] = static_cast<T>(a / (1.f + __expf(-a)) * b);
  }
}

template <typename T>
int launch(const void* x, const void* y, void* out, int64_t n, cudaStream_t s) {
  const int64_t nvec = n / (16 / sizeof(T)) + 1;
  int64_t blocks = (nvec + 255) / 256;
  const int64_t cap = (int64_t)gko::host::sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  silu_mul_vec<T><<<(unsigned)blocks, 256, 0, s>>>(static_cast<const T*>(x), static_cast<const T*>(y),
                                                   static_cast<T*>(out), n);
  return gko::host::cuda_check(cudaGetLastError(), "silu_mul launch");
}

// SwiGLU backward: with s = sigmoid(g), y = g s u,
//   d_up = dy g s,   d_gate = dy u s (1 + g (1 - s)).
// One thread per 8 consecutive columns j of a row: reads dy[j], gate_up[j] and gate_up[h + j],
// writes d_gate_up[j] and d_gate_up[h + j]. The math matches the reference backward
// (eval/kernels/gemm_swiglu.py:177-200).
template <typename T>
__global__ void __launch_bounds__(256) swiglu_bwd_vec(const T* __restrict__ dy, int64_t ld_dy,
                                                      const T* __restrict__ gu, int64_t ld_gu, T* __restrict__ dgu,
                                                      int64_t ld_dgu, int64_t rows, int64_t h) {
  const int64_t per_row = h / 8;
  const int64_t n = rows * per_row;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t r = i / per_row, j = (i % per_row) * 8;
    const uint4 dv = __ldg(reinterpret_cast<const uint4*>(dy + r * ld_dy + j));
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gu + r * ld_gu + j));
    const uint4 uv = __ldg(reinterpret_cast<const uint4*>(gu + r * ld_gu + h + j));
    const T* ds = reinterpret_cast<const T*>(&dv);
    const T* gs = reinterpret_cast<const T*>(&gv);
    const T* us = reinterpret_cast<const T*>(&uv);
    uint4 og, ou;
    T* ogs = reinterpret_cast<T*>(&og);
    T* ous = reinterpret_cast<T*>(&ou);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float d = static_cast<float>(ds[e]), g = static_cast<float>(gs[e]), u = static_cast<float>(us[e]);
      const float sg = 1.f / (1.f + __expf(-g));
      ous[e] = static_cast<T>(d * g * sg);
      ogs[e] = static_cast<T>(d * u * sg * (1.f + g * (1.f - sg)));
    }
    *reinterpret_cast<uint4*>(dgu + r * ld_dgu + j) = og;
    *reinterpret_cast<uint4*>(dgu + r * ld_dgu + h + j) = ou;
  }
}

template <typename T>
int launch_swiglu_bwd(const void* dy, int64_t ld_dy, const void* gu, int64_t ld_gu, void* dgu, int64_t ld_dgu,
                      int64_t rows, int64_t h, cudaStream_t s) {
  const int64_t n = rows * (h / 8);
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = (int64_t)gko::host::sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  swiglu_bwd_vec<T><<<(unsigned)blocks, 256, 0, s>>>(static_cast<const T*>(dy), ld_dy, static_cast<const T*>(gu),
                                                     ld_gu, static_cast<T*>(dgu), ld_dgu, rows, h);
  return gko::host::cuda_check(cudaGetLastError(), "swiglu_bwd launch");
}

}  // namespace

extern "C" int gko_swiglu_bwd(int dtype, int64_t rows, int64_t h, const void* dy, int64_t ld_dy, const void* gate_up,
                              int64_t ld_gu, void* d_gate_up, int64_t ld_dgu, unsigned int* status, void* stream) {
  (void)status;
  using gko::host::fail;
  if (rows < 0 || h < 0) return fail(GKO_ERR_INVALID, "negative size");
  if (rows == 0 || h == 0) return GKO_OK;
  if (!dy || !gate_up || !d_gate_up) return fail(GKO_ERR_INVALID, "null operand pointer");
  if (h % 8 || ld_dy % 8 || ld_gu % 8 || ld_dgu % 8 || !gko::host::aligned16(dy) || !gko::host::aligned16(gate_up) ||
      !gko::host::aligned16(d_gate_up))
    return fail(GKO_ERR_UNSUPPORTED, "swiglu_bwd needs h and row strides that are multiples of 8 and 16-byte "
                                     "aligned buffers");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GKO_F16: return launch_swiglu_bwd<__half>(dy, ld_dy, gate_up, ld_gu, d_gate_up, ld_dgu, rows, h, s);
    case GKO_BF16: return launch_swiglu_bwd<__nv_bfloat16>(dy, ld_dy, gate_up, ld_gu, d_gate_up, ld_dgu, rows, h, s);
    default: return fail(GKO_ERR_UNSUPPORTED, "swiglu_bwd takes bf16 or f16 (dtype code %d)", dtype);
  }
}

extern "C" int gko_silu_mul(int dtype, int64_t n, const void* x, const void* y, void* out,
                            unsigned int* status, void* stream) {
  (void)status;
  using gko::host::fail;
  if (n < 0) return fail(GKO_ERR_INVALID, "negative element count");
  if (n == 0) return GKO_OK;
  if (!x || !y || !out) return fail(GKO_ERR_INVALID, "null operand pointer");
  if (!gko::host::aligned16(x) || !gko::host::aligned16(y) || !gko::host::aligned16(out))
    return fail(GKO_ERR_UNSUPPORTED, "silu_mul needs 16-byte aligned buffers");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GKO_F16: return launch<__half>(x, y, out, n, s);
    case GKO_BF16: return launch<__nv_bfloat16>(x, y, out, n, s);
    case GKO_F32: return launch<float>(x, y, out, n, s);
    default: return fail(GKO_ERR_INVALID, "unknown dtype code %d", dtype);
  }
}
