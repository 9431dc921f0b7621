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
//  * kNoAllocScratchBytes (32 MiB) is reserved on every GPU that loads the library,
//    for the life of the process.  A call whose split-K plan needs more returns
//    NVM_ERR_WORKSPACE (nothing runs); use nvm_paged_attention with a workspace then.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (host code cannot use the symbol itself: in host code it
//    names a host-side stand-in, not device memory).  Make that first call before
//    any stream capture.
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
// Bytes at the start of a split-K workspace that hold the tickets (see paged_mma.cu).
constexpr size_t kTicketBytes = 1u << 20;

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
  void* scratch = nullptr;
  if (need > 0) {
    int st = scratch_address(&scratch);
    if (st != NVM_OK) return st;
    // the tickets must start at zero; whatever the last call left elsewhere is overwritten
    const size_t tickets = need < kTicketBytes ? need : kTicketBytes;
    st = check_cuda(cudaMemsetAsync(scratch, 0, tickets, static_cast<cudaStream_t>(stream)),
                    "paged_attention_noalloc: cudaMemsetAsync");
    if (st != NVM_OK) return st;
  }
  return nvm_paged_attention(q, q_dtype, k_pages, v_pages, kv_dtype, k_scales, v_scales, scale_dtype, block_table,
                             context_lens, out, out_dtype, B, Hq, Hkv, L, D, P, page_size, max_pages, scale,
                             is_causal, scratch, need, stream);
}
