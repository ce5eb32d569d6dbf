// selftest_sm100.cu -- a self-test of the kernels' bounded waits.
//
// Every pipeline wait in this library gives up after a time limit, records
// bit 0 of the device error word and lets its CTA wind down, so that a wait
// that is never satisfied (a lost TMA completion, a role that stopped early)
// surfaces as B2A_ERR_TIMEOUT on the host instead of a hung GPU.  The kernel
// here makes one such wait run out on purpose: a single thread waits on an
// mbarrier that nothing arrives at, with a short limit.  Nothing else is in
// flight in that CTA (no TMA, no UMMA, no TMEM), so giving up is clean and the
// context stays usable.  The reference has host checks only
// (cuda/flash_attn_fa3_db_full.cu:352-363) and a launch check (:399).
#include "sm100_ptx.cuh"
#include "b2a_host.h"

namespace b2a {
namespace selftest {

__global__ void wait_timeout_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  const uint32_t b = smem_u32(&bar);
  mbar_init(b, 1u);
  abort_flag = 0;
  fence_mbar_init();
  // phase 0 never completes: nothing arrives on the barrier
  mbar_wait_limit(b, 0u, &abort_flag, limit_ns);
}

}  // namespace selftest

B2A_DEFINE_ERROR_READER(selftest)

}  // namespace b2a

extern "C" int b2a_selftest_wait_timeout(int limit_us, void* stream) {
  using namespace b2a;
  if (limit_us <= 0 || limit_us > 1000000)
    return set_error(B2A_ERR_INVALID_ARG, "limit_us must be in [1, 1000000]");
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      major != 10) {
    cudaGetLastError();
    return set_error(B2A_ERR_NO_DEVICE, "b200attn requires a current sm_100 (B200) CUDA device");
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  selftest::wait_timeout_kernel<<<1, 32, 0, s>>>((uint64_t)limit_us * 1000ull);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "self-test kernel launch");
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return set_cuda_error(e, "self-test kernel");
  uint32_t flags = 0;
  int rc = take_error_flags_selftest(&flags);
  if (rc != B2A_OK) return rc;
  if (flags & kErrWaitTimeout)
    return set_error(B2A_ERR_TIMEOUT, "self-test: the bounded wait gave up as intended");
  return set_error(B2A_ERR_CUDA, "self-test: the wait returned without timing out");
}
