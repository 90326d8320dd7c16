// out = silu(x) * y, elementwise (gko::silu_mul). HBM-bound: 16-byte vector
// loads/stores, grid sized to a multiple of the SM count, grid-stride loop.
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

}  // namespace

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
