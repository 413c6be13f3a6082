// Diagnostic: the bounded waits of the library's kernels give up.
//
// Every pipeline wait of the attention, prefill and cascade kernels is
// mbar_wait (an mbarrier wait) and the end-of-launch merge of the split-K
// kernels waits on a grid counter with wait_count; both stop after a time
// limit, set NF_STATUS_WAIT_TIMEOUT and return false, so that no kernel can
// spin forever.  This kernel runs those same two functions, with a short
// limit, on a wait that nothing can satisfy: an mbarrier that no thread
// arrives on, or a counter that nothing increments.  The host then sees the
// kernel end, the status bit set and the wait's result false, with the
// context still usable.  No fault, trap or endless loop is involved.
#include "nf_common.cuh"
#include "nf_internal.h"

namespace nf {

__global__ void wait_selftest_kernel(int kind, long long limit, const int* counter, int target, int* status,
                                     int* result) {
  __shared__ __align__(8) unsigned long long bar;
  bool satisfied;
  if (kind == 0) {
    const uint32_t b = smem_u32(&bar);
    mbar_init(b, 1);
    fence_mbar_init();
    satisfied = mbar_wait(b, 0, status, limit);  // phase 0 completes only when one thread arrives
  } else {
    satisfied = wait_count(counter, target, status, limit);
  }
  *result = satisfied ? 1 : 0;
}

}  // namespace nf

extern "C" int nf_selftest_wait(int32_t kind, int64_t limit_cycles, const int32_t* counter, int32_t target,
                                int32_t* status, int32_t* result, void* stream) {
  using namespace nf;
  if (kind != 0 && kind != 1) return fail(NF_EINVAL, "nf_selftest_wait: kind %d (0 or 1)", kind);
  if (limit_cycles <= 0 || limit_cycles > kWaitLimitCycles)
    return fail(NF_EINVAL, "nf_selftest_wait: limit %lld cycles outside (0, %lld]", (long long)limit_cycles,
                (long long)kWaitLimitCycles);
  if (!status || !result || (kind == 1 && !counter)) return fail(NF_EINVAL, "nf_selftest_wait: null pointer argument");
  wait_selftest_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(kind, limit_cycles, counter, target, status,
                                                                        result);
  return check_launch("nf_selftest_wait");
}
