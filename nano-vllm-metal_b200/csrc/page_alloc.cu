// page_alloc.cu -- device-side page allocation and slot mapping for one batched
// append, so a decode step needs no host round trip to extend block tables.
//
// Semantics are those of running, for b = 0..B-1 in order, the reference's
// TinyKvPagedCache._append_chunk (src/nano_vllm_metal/cache/paged.py:424-459) with
// TinyKvPagedPool.allocate_page (paged.py:60-70): the tail page is filled first,
// then fresh pages are taken LIFO from the free list (free_stack[top-1] first) and,
// once it is empty, new ids num_pages, num_pages+1, ... are minted.  Because the
// k-th page allocated in the whole batch is a pure function of k, the batch is
// resolved with two prefix sums instead of a serial loop.
#include "nvm_common.cuh"
#include "nvm_internal.h"

namespace nvm {
namespace {

constexpr int kThreads = 1024;
constexpr int kMaxB = 4096;

// Inclusive block-wide scan of one value per thread (kThreads threads).
__device__ int64_t block_inclusive_scan(int64_t v, int64_t* buf) {
  const int t = threadIdx.x;
  buf[t] = v;
  __syncthreads();
  for (int off = 1; off < kThreads; off <<= 1) {
    const int64_t add = t >= off ? buf[t - off] : 0;
    __syncthreads();
    buf[t] += add;
    __syncthreads();
  }
  const int64_t r = buf[t];
  __syncthreads();
  return r;
}

struct AppendParams {
  int32_t* block_table;
  int32_t* context_lens;
  const int32_t* new_tokens;
  int32_t* free_stack;
  int32_t* free_top;
  int32_t* num_pages;
  int32_t* refcount;
  int64_t* slot_mapping;
  int64_t slot_capacity;
  int32_t* status;
  int64_t B, mp, ps, capacity;
};

__global__ void __launch_bounds__(kThreads) paged_append_kernel(AppendParams p) {
  __shared__ int64_t scan_buf[kThreads];
  __shared__ int32_t page_start[kMaxB + 1];  // exclusive prefix of pages needed
  __shared__ int32_t tok_start[kMaxB + 1];   // exclusive prefix of new tokens
  __shared__ int s_bad;
  const int t = threadIdx.x;
  const int64_t per = (p.B + kThreads - 1) / kThreads;
  const int64_t b0 = t * per, b1 = min(p.B, b0 + per);
  if (t == 0) s_bad = 0;
  __syncthreads();

  // Per-thread segment sums of pages needed and tokens appended.
  int64_t seg_pages = 0, seg_toks = 0;
  for (int64_t b = b0; b < b1; ++b) {
    const int64_t len = p.context_lens[b];
    const int64_t add = p.new_tokens[b];
    const int64_t have = (len + p.ps - 1) / p.ps;
    const int64_t room = (len % p.ps != 0) ? (p.ps - len % p.ps) : 0;
    const int64_t rest = add > room ? add - room : 0;
    const int64_t need = (rest + p.ps - 1) / p.ps;
    if (add < 0 || len < 0 || have + need > p.mp) atomicExch(&s_bad, 1);
    seg_pages += need;
    seg_toks += add > 0 ? add : 0;
  }
  const int64_t incl_pages = block_inclusive_scan(seg_pages, scan_buf);
  const int64_t incl_toks = block_inclusive_scan(seg_toks, scan_buf);
  int64_t run_p = incl_pages - seg_pages, run_t = incl_toks - seg_toks;
  for (int64_t b = b0; b < b1; ++b) {
    page_start[b] = (int32_t)run_p;
    tok_start[b] = (int32_t)run_t;
    const int64_t len = p.context_lens[b];
    const int64_t add = p.new_tokens[b] > 0 ? p.new_tokens[b] : 0;
    const int64_t room = (len % p.ps != 0) ? (p.ps - len % p.ps) : 0;
    const int64_t rest = add > room ? add - room : 0;
    run_p += (rest + p.ps - 1) / p.ps;
    run_t += add;
  }
  if (t == kThreads - 1) {
    page_start[p.B] = (int32_t)incl_pages;
    tok_start[p.B] = (int32_t)incl_toks;
  }
  __syncthreads();
  const int64_t total_pages = page_start[p.B];
  const int64_t total_toks = tok_start[p.B];
  const int64_t top = *p.free_top;
  const int64_t minted0 = *p.num_pages;
  const int64_t fresh = total_pages > top ? total_pages - top : 0;
  if (s_bad || minted0 + fresh > p.capacity || total_toks > p.slot_capacity) {
    if (t == 0) *p.status = NVM_ERR_OUT_OF_PAGES;
    return;
  }

  // New page ids into the block table (+ refcount 1).
  for (int64_t b = 0; b < p.B; ++b) {
    const int64_t need = page_start[b + 1] - page_start[b];
    if (need == 0) continue;
    const int64_t have = (p.context_lens[b] + p.ps - 1) / p.ps;
    for (int64_t j = t; j < need; j += kThreads) {
      const int64_t k = page_start[b] + j;
      const int64_t pid = k < top ? (int64_t)p.free_stack[top - 1 - k] : minted0 + (k - top);
      p.block_table[b * p.mp + have + j] = (int32_t)pid;
      p.refcount[pid] = 1;
    }
  }
  __syncthreads();

  // Slot of every appended token.
  for (int64_t i = t; i < total_toks; i += kThreads) {
    int64_t lo = 0, hi = p.B - 1;  // last b with tok_start[b] <= i
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) >> 1;
      if (tok_start[mid] <= i) lo = mid; else hi = mid - 1;
    }
    const int64_t b = lo, ii = i - tok_start[b];
    const int64_t len = p.context_lens[b];
    const int64_t pos = len + ii;  // absolute position of this token
    const int64_t pid = p.block_table[b * p.mp + pos / p.ps];
    p.slot_mapping[i] = pid * p.ps + pos % p.ps;
  }
  __syncthreads();
  for (int64_t b = t; b < p.B; b += kThreads) p.context_lens[b] += p.new_tokens[b] > 0 ? p.new_tokens[b] : 0;
  if (t == 0) {
    *p.free_top = (int32_t)(top - (total_pages < top ? total_pages : top));
    *p.num_pages = (int32_t)(minted0 + fresh);
    *p.status = NVM_OK;
  }
}

}  // namespace

int launch_paged_append(int32_t* block_table, int32_t* context_lens, const int32_t* new_tokens, int32_t* free_stack,
                        int32_t* free_top, int32_t* num_pages, int32_t* page_refcount, int64_t* slot_mapping,
                        int64_t slot_capacity, int32_t* status, int64_t B, int64_t max_pages, int64_t page_size,
                        int64_t capacity, cudaStream_t s) {
  AppendParams p{block_table, context_lens, new_tokens, free_stack, free_top, num_pages, page_refcount,
                 slot_mapping, slot_capacity, status, B, max_pages, page_size, capacity};
  paged_append_kernel<<<1, kThreads, 0, s>>>(p);
  return check_cuda(cudaGetLastError(), "allocate_page: kernel launch");
}

}  // namespace nvm
