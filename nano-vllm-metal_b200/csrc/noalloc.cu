// noalloc.cu -- nvm_paged_attention_noalloc: paged attention whose split-K scratch
// lives in a fixed array inside this library instead of a caller-provided workspace.
//
// Who needs it: callers that must not allocate device memory while serving --
// an engine that hands every free byte of HBM to its KV page pools at start-up and
// treats a later cudaMalloc as a failure, a decode loop that cannot pay for
// cudaMalloc's implicit device synchronisation between steps, or a foreign-language
// host with no device allocator of its own.  They pass only their inputs and the
// output buffer; the scratch this kernel needs for combining long-context chunks is
// the file-scope array below.
//
// Limits and rules:
//  * kNoAllocScratchBytes (32 MiB) of device memory backs the array on each device
//    the entry point is called on, for the life of the process.  The array is the
//    only object of its own CUDA module, and with lazy module loading (the CUDA 12
//    default) the runtime loads that module -- and takes the 32 MiB -- at the first
//    call on the device, not when the library is loaded.  An engine that sizes its
//    page pools from the free memory should therefore make one call (of any size)
//    on each device before it does so.  A call whose split-K plan needs more than
//    32 MiB returns NVM_ERR_WORKSPACE (nothing runs); use nvm_paged_attention with
//    a workspace then.
//  * Every call, whatever its size, looks up the array's device address with
//    cudaGetSymbolAddress the first time it runs on a device (host code cannot use
//    the symbol itself: in host code it names a host-side stand-in, not device
//    memory), so the first call on each device does the set-up.  Make that first
//    call before any stream capture.
//  * All calls share the one array and it keeps the previous call's contents.  The
//    ticket counters that must start at zero are cleared with cudaMemsetAsync on the
//    caller's stream before every launch; calls that overlap on the GPU (different
//    streams, no ordering between them) race on the array.
//  * Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <mutex>

#include "nvm_internal.h"

namespace nvm {
namespace {

constexpr size_t kNoAllocScratchBytes = 32u << 20;
static_assert(kTicketRegionBytes <= kNoAllocScratchBytes, "the ticket region must fit in the scratch array");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};

// Device address of the scratch array on the current device (set up once per device).
int scratch_address(void** out) {
  int dev = 0;
  int st = check_cuda(cudaGetDevice(&dev), "paged_attention_noalloc: cudaGetDevice");
  if (st != NVM_OK) return st;
  if (dev < 0 || dev >= 64) return fail(NVM_ERR_UNSUPPORTED, "paged_attention_noalloc: device index %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    st = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "paged_attention_noalloc: cudaGetSymbolAddress");
    if (st != NVM_OK) return st;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return NVM_OK;
}

}  // namespace
}  // namespace nvm

using namespace nvm;

extern "C" int nvm_paged_attention_noalloc(const void* q, int q_dtype, const void* k_pages, const void* v_pages,
                                           int kv_dtype, const void* k_scales, const void* v_scales,
                                           int scale_dtype, const int32_t* block_table,
                                           const int32_t* context_lens, void* out, int out_dtype, int64_t B,
                                           int64_t Hq, int64_t Hkv, int64_t L, int64_t D, int64_t P,
                                           int64_t page_size, int64_t max_pages, float scale, int is_causal,
                                           void* stream) {
  // Same plan as nvm_paged_attention; only the scratch source differs.
  size_t need = nvm_paged_attention_workspace_size(B, Hq, Hkv, L, D, page_size, max_pages, kv_dtype);
  if (need > kNoAllocScratchBytes)
    return fail(NVM_ERR_WORKSPACE,
                "paged_attention_noalloc: these sizes need %zu bytes of split-K scratch, the built-in limit is "
                "%zu bytes; call nvm_paged_attention with a workspace",
                need, kNoAllocScratchBytes);
  // resolved on every call (cached per device), so the first call of any size sets up
  // the device and a later call that needs scratch never does it inside a capture
  void* scratch = nullptr;
  int st = scratch_address(&scratch);
  if (st != NVM_OK) return st;
  if (need > 0) {
    // the tickets must start at zero; whatever the last call left elsewhere is overwritten
    const size_t tickets = need < kTicketRegionBytes ? need : kTicketRegionBytes;
    st = check_cuda(cudaMemsetAsync(scratch, 0, tickets, static_cast<cudaStream_t>(stream)),
                    "paged_attention_noalloc: cudaMemsetAsync");
    if (st != NVM_OK) return st;
  }
  return nvm_paged_attention(q, q_dtype, k_pages, v_pages, kv_dtype, k_scales, v_scales, scale_dtype, block_table,
                             context_lens, out, out_dtype, B, Hq, Hkv, L, D, P, page_size, max_pages, scale,
                             is_causal, need > 0 ? scratch : nullptr, need, stream);
}
