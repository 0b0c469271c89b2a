// Self-test of the bounded device waits (no reference counterpart): a kernel
// waits on an mbarrier that nothing ever arrives at, through the same
// mbar_wait_limit every tensor-core kernel of the library uses, but with a
// short limit.  The wait runs out, the kernel records
// PQ_DEVICE_ERR_WAIT_SELFTEST in the device error word and returns normally,
// so the context stays usable and pq_device_status() reports the code.  This
// is how a stalled pipeline (a copy or MMA that never completes) surfaces to
// the host without a trap or a hang.
#include "tc.cuh"

namespace pqb {

__global__ void wait_selftest_kernel(long long limit_cycles) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  const uint32_t b = tc::smem_u32(&bar);
  if (threadIdx.x == 0) {
    tc::mbar_init(b, 1);  // expects one arrival; none comes
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    tc::mbar_wait_limit(b, 0u, &abort_flag, tc::kErrWaitSelftest, limit_cycles);
  __syncthreads();
}

}  // namespace pqb

extern "C" int pq_selftest_wait_timeout(int64_t limit_cycles, void* stream) {
  using namespace pqb;
  PQ_CHECK_ARG(limit_cycles >= 1000 && limit_cycles <= 4000000000ll,
               "limit_cycles must be in [1e3, 4e9] (got %lld)", (long long)limit_cycles);
  wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((long long)limit_cycles);
  PQ_LAUNCH_CHECK("wait_selftest_kernel");
  return PQ_OK;
}
