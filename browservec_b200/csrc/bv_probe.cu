// bv_probe.cu -- a self-test of the kernels' bounded waits.
//
// Every wait of the scan, tail and GEMM kernels is an mbarrier poll with a
// budget: when it runs out, the kernel raises kErrWaitTimeout in the index's
// error word and returns, and the host reports BV_ERR_TIMEOUT instead of
// hanging the GPU.  This kernel exercises exactly that path on a barrier that
// nothing will ever complete -- one thread, no copies in flight, no tensor
// memory -- so a test can check the status the host reads and that the
// context stays usable afterwards.
#include <cstdint>

#include "bv_device.cuh"
#include "bv_internal.h"

namespace bv {

namespace {

__global__ void __launch_bounds__(32) wait_probe_kernel(uint32_t* err, uint32_t polls) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival; none is ever made
    fence_mbar_init();
    mbar_wait_bounded(&bar, 0, err, polls);
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_addr(&bar)) : "memory");
  }
}

}  // namespace

cudaError_t launch_wait_probe(uint32_t* err, uint32_t polls, cudaStream_t s) {
  wait_probe_kernel<<<1, 32, 0, s>>>(err, polls);
  return cudaGetLastError();
}

}  // namespace bv
