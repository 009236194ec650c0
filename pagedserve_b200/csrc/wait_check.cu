// Self-test of the library's bounded device-side waits.
//
// Every mbarrier wait in the tensor-core prefill and the greedy selection
// goes through mbar_wait (common.cuh): a poll bounded by a wall-clock limit,
// after which the kernel records PSB_DEVERR_TIMEOUT and unwinds instead of
// hanging.  psb_bounded_wait_check runs that same wait on an mbarrier that
// nothing arrives on, so the bound is the only way out: the call returns
// after the limit with the timeout bit set, and the context stays usable.
#include "common.cuh"
#include "host_util.h"

namespace psb {
namespace {

__global__ void __launch_bounds__(32) bounded_wait_check_kernel(int32_t* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  // phase 0 never completes: no thread arrives and no copy is in flight
  const bool done = mbar_wait(&bar, 0);
  if (!done && threadIdx.x == 0) flag_error(err, PSB_DEVERR_TIMEOUT);
}

}  // namespace
}  // namespace psb

extern "C" int psb_bounded_wait_check(int32_t* error_flag, psb_stream_t stream) {
  if (error_flag == nullptr) return PSB_ERR_INVALID;
  psb::discard_stale_error();
  psb::bounded_wait_check_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(error_flag);
  return psb::check_launch();
}
