// Self-test of the bounded-wait mechanism every kernel of this library uses.
//
// One warp waits on an mbarrier that nothing ever arrives on, with the
// caller's limit instead of the production 2 s.  The wait must give up,
// record its code in the device status word and return, leaving the CUDA
// context usable - the same path an attention launch takes if one of its
// pipeline waits ever expires.  No fault, trap or unbounded loop is involved.
#include "ps_b200.h"
#include "internal.h"
#include "ptx.cuh"

namespace psb {
namespace {

__global__ void bounded_wait_probe(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Phase 0 of `bar` never completes: the bounded wait expires.
  mbar_wait_for(smem_u32(&bar), 0, &abort_flag, status, PS_B200_DEVICE_TIMEOUT_LAST, limit_ns);
}

}  // namespace
}  // namespace psb

extern "C" int ps_b200_selftest_bounded_wait(int* status, int limit_us, void* stream) {
  using namespace psb;
  if (!status || (reinterpret_cast<uintptr_t>(status) & 3u))
    return set_error(PS_B200_ERR_INVALID, "status must be a 4-byte aligned device pointer");
  if (limit_us < 1 || limit_us > 2000000) return set_error(PS_B200_ERR_INVALID, "limit_us must be in [1, 2e6]");
  bounded_wait_probe<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, uint64_t(limit_us) * 1000u);
  const cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? PS_B200_OK : set_cuda_error("selftest launch", err);
}
