// Self-test of the bounded mbarrier wait used by every kernel of the library
// (g4::mbar_wait): a one-CTA kernel whose waits are made to succeed, to run
// out of time, or to see an abort raised by another warp.  None of the cases
// faults or hangs: an expired wait records its code in the error word and
// returns, which is the behaviour the attention kernels rely on when a
// producer or a tensor-core commit never arrives.
#include <cuda_runtime.h>
#include <stdint.h>

#include "g4_kernels.h"
#include "g4_sm100.cuh"

namespace g4 {

// mode 0: warp 1 arrives, warp 0 waits (completes)
// mode 1: nothing arrives; warp 0's wait expires after kWaitLimitNs
// mode 2: warp 1 raises the CTA abort word (recording kDevTimeoutTma as a
//         role that timed out would); warp 0's wait returns false promptly
//         without recording its own code
// out[0]: 1 if the wait returned true; out[1]: elapsed ns of the wait
__global__ void __launch_bounds__(64, 1) selftest_wait_kernel(int mode, int* err,
                                                              unsigned long long* out) {
  __shared__ uint64_t bar;
  __shared__ int abort_word;
  const int warp = __shfl_sync(0xffffffffu, threadIdx.x >> 5, 0);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_word = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const CtaAbort ab{&abort_word, err};
  if (warp == 1 && threadIdx.x == 32) {
    if (mode == 0) mbar_arrive(&bar);
    if (mode == 2) wait_fail(ab, kDevTimeoutTma);
  } else if (warp == 0) {
    const uint64_t t0 = global_timer_ns();
    const bool ok = mbar_wait(&bar, 0, ab, kDevTimeoutPeer);
    const uint64_t t1 = global_timer_ns();
    if (threadIdx.x == 0) {
      out[0] = ok ? 1ull : 0ull;
      out[1] = t1 - t0;
    }
  }
}

int launch_selftest_wait(int mode, int* err, unsigned long long* out, cudaStream_t stream) {
  selftest_wait_kernel<<<1, 64, 0, stream>>>(mode, err, out);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace g4
