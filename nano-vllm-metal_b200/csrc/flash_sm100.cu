// flash_sm100.cu -- tcgen05 / TMEM causal prefill for 16-bit Q/K/V with D == 128.
// (Enabled once validated on B200; until then every call is served by the
// mma.sync kernel in paged_mma.cu.)
#include "nvm_common.cuh"
#include "nvm_internal.h"

namespace nvm {

bool sm100_prefill_eligible(const PagedArgs& a) {
  (void)a;
  return false;
}

int launch_sm100_prefill(const PagedArgs& a, cudaStream_t s) {
  (void)a;
  (void)s;
  return fail(NVM_ERR_UNSUPPORTED, "flash_attention: sm100 prefill kernel not built");
}

}  // namespace nvm
