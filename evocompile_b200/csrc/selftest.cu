// Self-test of the bounded-wait failure path: a kernel waits on an mbarrier
// that nothing ever arrives on, with a short time limit, through the same
// wait_bounded used by every operator. It must record the timeout bit in the
// status word and return, leaving the context usable.
#include "host_common.h"
#include "sm100_ptx.cuh"

namespace {

__global__ void wait_never_kernel(unsigned* status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    gko::mbar_init(gko::smem_u32(&bar), 1);
    abort_flag = 0;
    gko::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // phase 0 of a fresh barrier with one expected arrival never completes
    gko::wait_bounded(gko::smem_u32(&bar), 0, &abort_flag, status, gko::kStatusTimeoutProducer, limit_ns);
  }
  __syncthreads();
}

}  // namespace

extern "C" int gko_selftest_wait_timeout(unsigned int* status, long long limit_ns, void* stream) {
  using gko::host::fail;
  if (!status) return fail(GKO_ERR_INVALID, "status word pointer is null");
  if (limit_ns <= 0 || limit_ns > 2000000000ll) return fail(GKO_ERR_INVALID, "limit must be in (0, 2e9] ns");
  wait_never_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(status, (unsigned long long)limit_ns);
  return gko::host::cuda_check(cudaGetLastError(), "selftest launch");
}
