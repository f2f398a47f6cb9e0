// Diagnostic entry point for the bounded-wait failure path.
//
// Every wait of the tensor-core kernels (TMA completion, MMA commit, a peer
// role's arrival) is bounded: after kWaitTimeoutNs the waiting role records
// TT_ERR_DEVICE_TIMEOUT in the caller's status word and the kernel unwinds
// instead of spinning.  This kernel exercises exactly that path on purpose: it
// waits, with the same bounded wait, for an mbarrier phase nothing will ever
// complete, then records the timeout.  It faults nothing and leaves the
// context usable, so a test can check that the status reaches the host and
// that the next launch runs normally.
#include "tt_sm100.cuh"

namespace tt {
namespace {

__global__ void bounded_wait_probe(int32_t* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);      // expects one arrival; none is ever made
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !sm100::mbar_wait(&bar, 0, nullptr))
    set_status(status, TT_ERR_DEVICE_TIMEOUT);
}

}  // namespace
}  // namespace tt

extern "C" int tt_diag_bounded_wait(int32_t* status, void* stream) {
  if (!status) return TT_ERR_INVALID_ARG;
  tt::bounded_wait_probe<<<1, 32, 0, (cudaStream_t)stream>>>(status);
  tt_count_launches(1);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}
