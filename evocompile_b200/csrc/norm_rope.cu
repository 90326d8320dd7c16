// Memory-bound pieces of the transformer block around the fused operators:
//   gko_rmsnorm  y = rmsnorm(x (+ r)) * w, optionally writing the residual sum x + r
//   gko_rms_stats  inv[row] = 1 / sqrt(mean((x + r)^2) + eps) only (optionally writing x + r): the
//                statistics a GEMM needs to apply RMSNorm as a per-row scale in its epilogue
//   gko_rope     rotary position embedding applied in place to q / k heads
// Both are HBM-bound: 16-byte vector loads/stores, fp32 arithmetic.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "host_common.h"

namespace {

template <typename T>
struct Vec8;  // 8 elements in 16 bytes
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const void* p, float (&f)[8]) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static __device__ __forceinline__ void store(void* p, const float (&f)[8]) {
    uint4 v;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = v;
  }
};
template <>
struct Vec8<__half> {
  static __device__ __forceinline__ void load(const void* p, float (&f)[8]) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static __device__ __forceinline__ void store(void* p, const float (&f)[8]) {
    uint4 v;
    __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = v;
  }
};

constexpr int kNormThreads = 256;
constexpr int kMaxVecPerThread = 8;  // cols <= 256 * 8 * 8 = 16384

// One CTA per row; VPT 16-byte vectors per thread, chosen on the host as the smallest
// power of two covering the row, so short rows keep few registers and many rows in flight.
// The row (x + r) stays in registers between the two passes.
template <typename T, int VPT>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ r,
                                                               const T* __restrict__ w, T* __restrict__ y,
                                                               T* __restrict__ sum_out, int cols, int64_t ld,
                                                               float eps, float* __restrict__ inv_out) {
  const int64_t row = blockIdx.x;
  const int nvec = cols / 8;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * kNormThreads;
    if (vi < nvec) Vec8<T>::load(x + row * ld + vi * 8, v[i]);
  }
  if (r) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = threadIdx.x + i * kNormThreads;
      if (vi < nvec) {
        float rr[8];
        Vec8<T>::load(r + row * ld + vi * 8, rr);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] += rr[e];
        if (sum_out) Vec8<T>::store(sum_out + row * ld + vi * 8, v[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * kNormThreads;
    if (vi < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[i][e], v[i][e], ss);
    }
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / (float)cols + eps);
  if (inv_out && threadIdx.x == 0) inv_out[row] = inv;
  if (!y) return;  // statistics only
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * kNormThreads;
    if (vi < nvec) {
      float ww[8];
      Vec8<T>::load(w + vi * 8, ww);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = v[i][e] * inv * ww[e];
      Vec8<T>::store(y + row * ld + vi * 8, v[i]);
    }
  }
}

// Rotate-half RoPE (the Llama / HF convention): for pair (i, i + D/2) of a head,
//   out_i = x_i cos(p f_i) - x_{i+D/2} sin(p f_i),  out_{i+D/2} = x_{i+D/2} cos(p f_i) + x_i sin(p f_i),
// f_i = theta^(-2i/D), p = token position. One thread per (token, 8 consecutive i): it evaluates
// its 8 angles once and applies them to every head of the token with 16-byte loads and stores
// (the 8 threads of a token cover a head's two 128-byte halves).
template <typename T>
__global__ void __launch_bounds__(256) rope_kernel(T* __restrict__ x, int64_t tokens, int heads, int d,
                                                   int64_t st_token, int64_t st_head,
                                                   const int* __restrict__ pos, int seq_len,
                                                   float log2_theta) {
  const int half = d / 2;
  const int chunks = half / 8;
  const int64_t n = tokens * chunks;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int i0 = (int)(idx % chunks) * 8;
    const int64_t t = idx / chunks;
    const int p = pos ? pos[t] : (int)(t % seq_len);
    float c[8], s[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float inv_freq = exp2f(-log2_theta * (2.f * (float)(i0 + e) / (float)d));
      sincosf((float)p * inv_freq, &s[e], &c[e]);
    }
    T* row = x + t * st_token + i0;
    for (int h = 0; h < heads; ++h) {
      T* base = row + (int64_t)h * st_head;
      float a[8], b[8];
      Vec8<T>::load(base, a);
      Vec8<T>::load(base + half, b);
      float oa[8], ob[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        oa[e] = a[e] * c[e] - b[e] * s[e];
        ob[e] = b[e] * c[e] + a[e] * s[e];
      }
      Vec8<T>::store(base, oa);
      Vec8<T>::store(base + half, ob);
    }
  }
}

}  // namespace

using gko::host::fail;

namespace {
template <typename T>
void launch_rmsnorm(int vpt, int64_t rows, const void* x, const void* r, const void* w, void* y, void* sum_out,
                    int cols, int64_t ld, float eps, cudaStream_t s, float* inv_out = nullptr) {
  const T* xp = static_cast<const T*>(x);
  const T* rp = static_cast<const T*>(r);
  const T* wp = static_cast<const T*>(w);
  T* yp = static_cast<T*>(y);
  T* sp = static_cast<T*>(sum_out);
  const unsigned g = (unsigned)rows;
  if (vpt == 1) rmsnorm_kernel<T, 1><<<g, kNormThreads, 0, s>>>(xp, rp, wp, yp, sp, cols, ld, eps, inv_out);
  else if (vpt == 2) rmsnorm_kernel<T, 2><<<g, kNormThreads, 0, s>>>(xp, rp, wp, yp, sp, cols, ld, eps, inv_out);
  else if (vpt == 4) rmsnorm_kernel<T, 4><<<g, kNormThreads, 0, s>>>(xp, rp, wp, yp, sp, cols, ld, eps, inv_out);
  else rmsnorm_kernel<T, 8><<<g, kNormThreads, 0, s>>>(xp, rp, wp, yp, sp, cols, ld, eps, inv_out);
}
}  // namespace

extern "C" int gko_rmsnorm(int dtype, int64_t rows, int64_t cols, const void* x, const void* residual,
                           const void* weight, float eps, void* out, void* sum_out, int64_t ld,
                           unsigned int* status, void* stream) {
  (void)status;
  if (dtype != GKO_BF16 && dtype != GKO_F16) return fail(GKO_ERR_UNSUPPORTED, "rmsnorm takes bf16 or f16");
  if (rows < 0 || cols <= 0) return fail(GKO_ERR_INVALID, "bad rmsnorm sizes");
  if (rows == 0) return GKO_OK;
  if (cols % 8 || ld % 8 || ld < cols)
    return fail(GKO_ERR_UNSUPPORTED, "rmsnorm needs cols and row stride multiples of 8 (ld >= cols)");
  if (cols > kNormThreads * kMaxVecPerThread * 8) return fail(GKO_ERR_UNSUPPORTED, "rmsnorm supports cols <= 16384");
  if (!x || !weight || !out) return fail(GKO_ERR_INVALID, "null pointer argument");
  if (!gko::host::aligned16(x) || !gko::host::aligned16(weight) || !gko::host::aligned16(out) ||
      (residual && !gko::host::aligned16(residual)) || (sum_out && !gko::host::aligned16(sum_out)))
    return fail(GKO_ERR_UNSUPPORTED, "rmsnorm needs 16-byte aligned buffers");
  if (rows > 0x7fffffffll) return fail(GKO_ERR_UNSUPPORTED, "too many rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t per = (cols / 8 + kNormThreads - 1) / kNormThreads;  // vectors per thread
  const int vpt = per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : 8;
  if (dtype == GKO_BF16)
    launch_rmsnorm<__nv_bfloat16>(vpt, rows, x, residual, weight, out, sum_out, (int)cols, ld, eps, s);
  else
    launch_rmsnorm<__half>(vpt, rows, x, residual, weight, out, sum_out, (int)cols, ld, eps, s);
  return gko::host::cuda_check(cudaGetLastError(), "rmsnorm launch");
}

extern "C" int gko_rope(int dtype, int64_t tokens, int64_t heads, int64_t head_dim, void* x, int64_t st_token,
                        int64_t st_head, const int32_t* positions, int64_t seq_len, float theta,
                        unsigned int* status, void* stream) {
  (void)status;
  if (dtype != GKO_BF16 && dtype != GKO_F16) return fail(GKO_ERR_UNSUPPORTED, "rope takes bf16 or f16");
  if (tokens < 0 || heads < 0 || head_dim <= 0 || head_dim % 2) return fail(GKO_ERR_INVALID, "bad rope sizes");
  if (tokens == 0 || heads == 0) return GKO_OK;
  if (!x) return fail(GKO_ERR_INVALID, "null pointer argument");
  if (!positions && seq_len <= 0) return fail(GKO_ERR_INVALID, "rope needs positions or seq_len > 0");
  if (!(theta > 1.f)) return fail(GKO_ERR_INVALID, "rope theta must be > 1");
  if (head_dim % 16 || st_token % 8 || st_head % 8 || !gko::host::aligned16(x))
    return fail(GKO_ERR_UNSUPPORTED, "rope needs head_dim a multiple of 16, token/head strides multiples of 8 "
                                     "elements and a 16-byte aligned buffer");
  const int64_t n = tokens * (head_dim / 16);
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = (int64_t)gko::host::sm_count() * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const float l2t = log2f(theta);
  if (dtype == GKO_BF16)
    rope_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(static_cast<__nv_bfloat16*>(x), tokens, (int)heads,
                                                                (int)head_dim, st_token, st_head, positions,
                                                                (int)seq_len, l2t);
  else
    rope_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(static_cast<__half*>(x), tokens, (int)heads, (int)head_dim,
                                                         st_token, st_head, positions, (int)seq_len, l2t);
  return gko::host::cuda_check(cudaGetLastError(), "rope launch");
}

extern "C" int gko_rms_stats(int dtype, int64_t rows, int64_t cols, const void* x, const void* residual, float eps,
                             void* sum_out, float* inv_out, int64_t ld, unsigned int* status, void* stream) {
  (void)status;
  if (dtype != GKO_BF16 && dtype != GKO_F16) return fail(GKO_ERR_UNSUPPORTED, "rms_stats takes bf16 or f16");
  if (rows < 0 || cols <= 0) return fail(GKO_ERR_INVALID, "bad rms_stats sizes");
  if (rows == 0) return GKO_OK;
  if (cols % 8 || ld % 8 || ld < cols)
    return fail(GKO_ERR_UNSUPPORTED, "rms_stats needs cols and row stride multiples of 8 (ld >= cols)");
  if (cols > kNormThreads * kMaxVecPerThread * 8) return fail(GKO_ERR_UNSUPPORTED, "rms_stats supports cols <= 16384");
  if (!x || !inv_out) return fail(GKO_ERR_INVALID, "null pointer argument");
  if (!gko::host::aligned16(x) || (residual && !gko::host::aligned16(residual)) ||
      (sum_out && !gko::host::aligned16(sum_out)))
    return fail(GKO_ERR_UNSUPPORTED, "rms_stats needs 16-byte aligned buffers");
  if (rows > 0x7fffffffll) return fail(GKO_ERR_UNSUPPORTED, "too many rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t per = (cols / 8 + kNormThreads - 1) / kNormThreads;
  const int vpt = per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : 8;
  if (dtype == GKO_BF16)
    launch_rmsnorm<__nv_bfloat16>(vpt, rows, x, residual, nullptr, nullptr, sum_out, (int)cols, ld, eps, s, inv_out);
  else
    launch_rmsnorm<__half>(vpt, rows, x, residual, nullptr, nullptr, sum_out, (int)cols, ld, eps, s, inv_out);
  return gko::host::cuda_check(cudaGetLastError(), "rms_stats launch");
}
