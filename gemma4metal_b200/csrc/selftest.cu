// tq_wait_selftest: runs out the bounded shared-memory barrier wait that every
// pipeline of this library uses (mbar_wait_bounded), on purpose and with a
// caller-chosen bound, so the expiry path -- record kErrBarrierTimeout in the
// device error word, give up, return -- is exercised without any fault: the
// barrier expects two arrivals and gets one, no copy is in flight, and every
// thread leaves after the bound.
#include "../../include/turboquant_c.h"
#include "tq_common.cuh"
#include "tq_internal.h"

namespace tq {
namespace {

__global__ void wait_selftest_kernel(long long budget, uint32_t* err, uint32_t* gave_up) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 2);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_arrive(&bar);  // one arrival of two: the phase never completes
  const bool done = mbar_wait_bounded(&bar, 0, err, budget);
  if (!done) atomicAdd(gave_up, 1u);
}

}  // namespace
}  // namespace tq

extern "C" TQ_API int tq_wait_selftest(int timeout_us, uint32_t* gave_up, void* stream) {
  if (timeout_us < 1 || timeout_us > 10000000 || !gave_up) {
    tq::set_last_error("tq_wait_selftest: need 1 <= timeout_us <= 10^7 and a device counter");
    return TQ_ERR_INVALID;
  }
  int dev = 0, khz = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev);
  const long long budget = static_cast<long long>(timeout_us) * (khz > 0 ? khz : 2000000) / 1000;
  tq::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      budget, tq::device_error_word(), gave_up);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    tq::set_last_error("tq_wait_selftest: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}
