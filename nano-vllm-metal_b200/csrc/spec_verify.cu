// spec_verify.cu -- batched acceptance of speculative-decoding drafts on the device.
//
// The reference verifies one request at a time on the host (speculative_generate,
// src/nano_vllm_metal/engine/generate.py:130-169): the candidate row is the last
// accepted token followed by the k draft tokens, the target model's argmax at each of
// the k + 1 positions is the verified row, and the request walks the positions in
// order -- position 0 compares the last token with itself, position i > 0 compares
// draft token i - 1 with verified token i - 1.  A matching token is emitted (unless it
// is the end-of-sequence id, which finishes the request, or the request's token budget
// is used up after it, which also finishes it).  At the first mismatch, position i,
// the rejected suffix of k + 1 - i tokens is dropped from the target's KV cache
// (k - i from the draft's) and verified token i - 1 becomes the next token (an
// end-of-sequence next token finishes the request).  When every position matches the
// next token is the last verified token and nothing is dropped.
//
// Here one thread walks one request; the whole batch is one launch and the outputs
// stay on the device, where DevicePageTable's batched rewind consumes them.
#include "nvm_internal.h"

namespace nvm {
namespace {

__global__ void spec_accept_kernel(const int32_t* __restrict__ cand, const int32_t* __restrict__ ver, int64_t B,
                                   int64_t K1, int32_t eos, const int32_t* __restrict__ budget,
                                   const int32_t* __restrict__ active, int32_t* __restrict__ emitted,
                                   int32_t* __restrict__ n_emitted, int32_t* __restrict__ next_token,
                                   int32_t* __restrict__ rewind, int32_t* __restrict__ draft_rewind,
                                   int32_t* __restrict__ finished) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int32_t* c = cand + b * K1;
  const int32_t* v = ver + b * K1;
  int32_t* e = emitted + b * K1;
  int64_t n = 0;
  int32_t nxt = -1, rw = 0, drw = 0, fin = 0;
  if (active == nullptr || active[b] != 0) {
    const int64_t limit = budget != nullptr ? budget[b] : -1;  // < 0: no budget
    nxt = v[K1 - 1];                                             // every position accepted
    for (int64_t i = 0; i < K1; ++i) {
      const int32_t comp = i == 0 ? c[0] : v[i - 1];
      if (comp != c[i]) {  // first rejected position (never 0)
        rw = (int32_t)(K1 - i);
        drw = rw - 1;
        nxt = comp;
        fin = eos >= 0 && comp == eos;
        break;
      }
      if (eos >= 0 && comp == eos) {  // an end-of-sequence token finishes the request unemitted
        fin = 1;
        nxt = -1;
        break;
      }
      e[n++] = comp;
      if (limit >= 0 && n >= limit) {  // budget used up right after this token
        fin = 1;
        nxt = -1;
        break;
      }
    }
  }
  for (int64_t j = n; j < K1; ++j) e[j] = -1;
  n_emitted[b] = (int32_t)n;
  next_token[b] = nxt;
  rewind[b] = rw;
  draft_rewind[b] = drw;
  finished[b] = fin;
}

}  // namespace
}  // namespace nvm

using namespace nvm;

extern "C" int nvm_spec_verify_accept(const int32_t* candidates, const int32_t* verified, int64_t B, int64_t K1,
                                      int32_t eos_id, const int32_t* budget, const int32_t* active,
                                      int32_t* emitted, int32_t* n_emitted, int32_t* next_token, int32_t* rewind,
                                      int32_t* draft_rewind, int32_t* finished, void* stream) {
  const char* op = "spec_verify_accept";
  if (B < 0 || K1 < 1) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: need B >= 0 and at least one position", op);
  if (B == 0) return NVM_OK;
  if (!candidates || !verified || !emitted || !n_emitted || !next_token || !rewind || !draft_rewind || !finished)
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: a required pointer is NULL", op);
  if (K1 > (1 << 20)) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: %lld positions per request", op, (long long)K1);
  const int threads = 128;
  const int64_t blocks = (B + threads - 1) / threads;
  if (blocks > INT32_MAX) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: batch too large", op);
  spec_accept_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      candidates, verified, B, K1, eos_id, budget, active, emitted, n_emitted, next_token, rewind, draft_rewind,
      finished);
  return check_cuda(cudaGetLastError(), "spec_verify_accept: launch");
}
