// Failure-detection self test: runs the two bounded waits every kernel of the library
// relies on against conditions that never complete, so the timeout path (record
// MHMOE_ERR_TIMEOUT in the device status word, return, context stays usable) can be
// tested on a GPU without faulting or hanging it.
//
//   mode bit 0: wait on a shared-memory mbarrier that nothing arrives on (mbar_wait, the
//               wait of the TMA / tcgen05 pipelines);
//   mode bit 1: wait for the global flag *flag to reach `expected` (flag_wait_geq, the
//               wait of anything that polls memory another agent writes).
// elapsed_ns[0] receives the time spent waiting (globaltimer).
#include "kernels.cuh"

namespace mhmoe {

__global__ void wait_selftest_kernel(const int* flag, int expected, int mode, uint64_t timeout_ns, int* status,
                                     int64_t* elapsed_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(smem_u32(&bar), 1);
  fence_mbar_init();
  const uint64_t t0 = globaltimer_ns();
  if (mode & 1) mbar_wait(smem_u32(&bar), 0, status, MHMOE_ERR_TIMEOUT, timeout_ns);
  if ((mode & 2) && flag) flag_wait_geq(flag, expected, status, MHMOE_ERR_TIMEOUT, timeout_ns);
  if (elapsed_ns) *elapsed_ns = (int64_t)(globaltimer_ns() - t0);
  // complete the barrier's phase so it ends in a consistent state
  mbar_arrive(smem_u32(&bar));
}

cudaError_t launch_wait_selftest(const int* flag, int expected, int mode, uint64_t timeout_ns, int* status,
                                 int64_t* elapsed_ns, cudaStream_t st) {
  wait_selftest_kernel<<<1, 32, 0, st>>>(flag, expected, mode, timeout_ns, status, elapsed_ns);
  return cudaGetLastError();
}

}  // namespace mhmoe
