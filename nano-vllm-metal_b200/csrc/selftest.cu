// selftest.cu -- nvm_selftest_wait_expiry: drives the kernels' bounded mbarrier wait to
// expiry on purpose, so that failure detection can be tested without a GPU fault.
//
// One warp initialises an mbarrier that expects one arrival and never arrives on it;
// lane 0 waits for its first phase through mbar_wait_for, the same spin-and-timer loop
// (mbar_wait) every TMA / tensor-core wait of the library uses, with the caller's
// short limit instead of the kernels' 2 s.  When the limit passes, the kernel records
// kDevErrFullWait in the device error word and returns; no copy or MMA is in flight,
// so nothing needs draining and the context stays usable.
#include "nvm_common.cuh"
#include "nvm_internal.h"

namespace nvm {
namespace {

constexpr int64_t kMinLimitNs = 1000;        // 1 us
constexpr int64_t kMaxLimitNs = 100000000;   // 100 ms

__global__ void __launch_bounds__(32) wait_expiry_kernel(int* err, uint64_t limit_ns,
                                                         unsigned long long* waited_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();
    const bool completed = mbar_wait_for(&bar, 0, limit_ns);  // nobody arrives
    if (!completed) record_error(err, kDevErrFullWait);
    if (waited_ns != nullptr) *waited_ns = globaltimer_ns() - t0;
  }
}

}  // namespace
}  // namespace nvm

using namespace nvm;

extern "C" int nvm_selftest_wait_expiry(int64_t limit_ns, unsigned long long* waited_ns, void* stream) {
  if (limit_ns < kMinLimitNs || limit_ns > kMaxLimitNs)
    return fail(NVM_ERR_INVALID_ARGUMENT, "selftest_wait_expiry: limit %lld ns outside [%lld, %lld]",
                (long long)limit_ns, (long long)kMinLimitNs, (long long)kMaxLimitNs);
  int* err = device_error_word();
  if (err == nullptr) return fail(NVM_ERR_CUDA, "selftest_wait_expiry: no device error word");
  wait_expiry_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(err, (uint64_t)limit_ns, waited_ns);
  return check_cuda(cudaGetLastError(), "selftest_wait_expiry: launch");
}
