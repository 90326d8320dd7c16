// Row-slice all-reduce over NVLink multicast, fused with the residual add and the RMSNorm
// statistics that follow a row-parallel projection in the tensor-parallel block.
//
// Every rank has written its partial output P_r [rows, cols] into its copy of a symmetric buffer
// (and the group has passed a barrier). Rank r then owns rows [row0, row1): for each of them one
// CTA reads the sum over ranks of the row through the buffer's multicast address
// (multimem.ld_reduce: the NVSwitch reads every rank's copy and adds them, fp32 accumulation),
// adds the residual row from local memory, writes the result to every rank's copy of the output
// buffer through its multicast address (multimem.st), and, when asked, the row's
// 1 / sqrt(mean(v^2) + eps) to every rank's copy of an fp32 statistics buffer. After a second
// barrier every rank holds the whole summed output: per rank, NVLink carries the rank's own
// partial once out (read by the owners of its rows) and the whole output once in, which is what
// a ring all-reduce moves too, with the residual add and the statistics pass folded in.
#include "host_common.h"
#include "sm100_ptx.cuh"

namespace gko {
namespace nvls {

constexpr int kThreads = 256;
constexpr int kMaxChunks = 8;  // 16-byte chunks per thread per row: cols <= 256 * 8 * 8 = 16384

template <typename T>
__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
  Cvt<T>::unpack(v.x, f[0], f[1]);
  Cvt<T>::unpack(v.y, f[2], f[3]);
  Cvt<T>::unpack(v.z, f[4], f[5]);
  Cvt<T>::unpack(v.w, f[6], f[7]);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) allreduce_residual_kernel(const uint8_t* partial_mc, const T* resid,
                                                                      uint8_t* out_mc, uint8_t* inv_mc, int row0,
                                                                      int row1, int cols, int64_t ld, float eps) {
  const int chunks = cols / 8;
  __shared__ float red[kThreads / 32];
  for (int row = row0 + (int)blockIdx.x; row < row1; row += (int)gridDim.x) {
    // every switch reduction and residual load of the row is in flight before the first is used
    uint4 sum[kMaxChunks], res[kMaxChunks];
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int j = (int)threadIdx.x + c * kThreads;
      if (j < chunks) {
        const int64_t off = (int64_t)row * ld + (int64_t)j * 8;
        sum[c] = multimem_ld_reduce_add_x8<T>(partial_mc + off * (int64_t)sizeof(T));
        res[c] = resid ? __ldg(reinterpret_cast<const uint4*>(resid + off)) : make_uint4(0, 0, 0, 0);
      }
    }
    float sq = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int j = (int)threadIdx.x + c * kThreads;
      if (j < chunks) {
        const int64_t off = (int64_t)row * ld + (int64_t)j * 8;
        float v[8], r[8];
        unpack8<T>(sum[c], v);
        unpack8<T>(res[c], r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] += r[e];
        uint4 w;
        w.x = Cvt<T>::pack(v[0], v[1]);
        w.y = Cvt<T>::pack(v[2], v[3]);
        w.z = Cvt<T>::pack(v[4], v[5]);
        w.w = Cvt<T>::pack(v[6], v[7]);
        multimem_st_x8<T>(out_mc + off * (int64_t)sizeof(T), w);
        if (inv_mc) {
          // the statistics of the rounded row, as the next GEMM reads it
          float q[8];
          unpack8<T>(w, q);
#pragma unroll
          for (int e = 0; e < 8; ++e) sq = fmaf(q[e], q[e], sq);
        }
      }
    }
    if (inv_mc) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) t += red[w];
        multimem_st_f32(inv_mc + (int64_t)row * 4, rsqrtf(t / (float)cols + eps));
      }
      __syncthreads();
    }
  }
  // the stores reach every GPU at system scope before the kernel is seen as complete
  __threadfence_system();
}

}  // namespace nvls
}  // namespace gko

using gko::host::fail;

extern "C" int gko_allreduce_residual_nvls(int dtype, int64_t rows, int64_t cols, int64_t ld, int64_t row0,
                                           int64_t row1, const void* partial_mc, const void* resid, void* out_mc,
                                           void* inv_mc, float eps, unsigned int* status, void* stream) {
  (void)status;
  if (dtype != GKO_BF16 && dtype != GKO_F16)
    return fail(GKO_ERR_UNSUPPORTED, "allreduce_residual_nvls takes bf16 or f16");
  if (rows < 0 || cols <= 0 || row0 < 0 || row1 < row0 || row1 > rows || ld < cols)
    return fail(GKO_ERR_INVALID, "allreduce_residual_nvls: bad sizes (rows %lld cols %lld ld %lld rows [%lld, %lld))",
                (long long)rows, (long long)cols, (long long)ld, (long long)row0, (long long)row1);
  if (cols % 8 || ld % 8 || cols > gko::nvls::kThreads * 8 * gko::nvls::kMaxChunks)
    return fail(GKO_ERR_UNSUPPORTED, "allreduce_residual_nvls needs cols %% 8 == 0, ld %% 8 == 0 and cols <= %d",
                gko::nvls::kThreads * 8 * gko::nvls::kMaxChunks);
  if (rows >= (1ll << 31)) return fail(GKO_ERR_UNSUPPORTED, "too many rows");
  if (row1 == row0) return GKO_OK;
  if (!partial_mc || !out_mc) return fail(GKO_ERR_INVALID, "null multicast address");
  if (!gko::host::aligned16(partial_mc) || !gko::host::aligned16(out_mc) || (resid && !gko::host::aligned16(resid)) ||
      (inv_mc && (reinterpret_cast<uintptr_t>(inv_mc) & 3)))
    return fail(GKO_ERR_UNSUPPORTED, "allreduce_residual_nvls needs 16-byte aligned buffers");
  const int64_t n = row1 - row0;
  const int sms = gko::host::sm_count();
  const int grid = (int)(n < 4 * sms ? n : 4 * sms);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const auto* pm = static_cast<const uint8_t*>(partial_mc);
  auto* om = static_cast<uint8_t*>(out_mc);
  auto* im = static_cast<uint8_t*>(inv_mc);
  if (dtype == GKO_BF16)
    gko::nvls::allreduce_residual_kernel<__nv_bfloat16><<<grid, gko::nvls::kThreads, 0, s>>>(
        pm, static_cast<const __nv_bfloat16*>(resid), om, im, (int)row0, (int)row1, (int)cols, ld, eps);
  else
    gko::nvls::allreduce_residual_kernel<__half><<<grid, gko::nvls::kThreads, 0, s>>>(
        pm, static_cast<const __half*>(resid), om, im, (int)row0, (int)row1, (int)cols, ld, eps);
  return gko::host::cuda_check(cudaGetLastError(), "allreduce_residual_nvls launch");
}
