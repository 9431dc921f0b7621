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

// ---------------------------------------------------------------------------
// Rewind / release of a batch: for b = 0..B-1 in order, the reference's
// TinyKvPagedCache.rewind(n_b) (paged.py:530-550; n_b == offset is release(),
// paged.py:552-559) with TinyKvPagedPool.free_page (paged.py:197-210).  Every page a
// request gives up is one free_page call; calls are numbered in that sequential order
// (release walks a row forward, rewind pops it from the end).  A page returns to the
// free list at the call that drops its refcount to zero -- its last call in order, and
// only if the batch's calls reach zero -- so pushes are ordered by call number.
// last_call[capacity] is scratch kept at -1 between calls.

struct RewindParams {
  int32_t* block_table;
  int32_t* context_lens;
  const int32_t* rewind;
  int32_t* free_stack;
  int32_t* free_top;
  int32_t* refcount;
  int32_t* last_call;
  int32_t* status;
  int64_t B, mp, ps, capacity;
};

__device__ __forceinline__ void rewind_span(const RewindParams& p, int64_t b, int64_t& have, int64_t& first,
                                            int64_t& calls, bool& fwd, int64_t& new_len) {
  const int64_t len = p.context_lens[b];
  const int64_t n = p.rewind[b];
  new_len = len - n;
  have = (len + p.ps - 1) / p.ps;
  const int64_t target = new_len == 0 ? 0 : (new_len + p.ps - 1) / p.ps;
  calls = n == 0 ? 0 : have - target;
  fwd = new_len == 0;  // release: forward; rewind: from the last page back
  first = target;
}

// Last request b with start[b] <= i (start is an exclusive prefix over B requests).
__device__ __forceinline__ int64_t owner_of(const int32_t* start, int64_t B, int64_t i) {
  int64_t lo = 0, hi = B - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (start[mid] <= i) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kThreads) paged_rewind_kernel(RewindParams p) {
  __shared__ int64_t scan_buf[kThreads];
  __shared__ int32_t call_start[kMaxB + 1];
  __shared__ int s_bad;
  const int t = threadIdx.x;
  const int64_t per = (p.B + kThreads - 1) / kThreads;
  const int64_t b0 = t * per, b1 = min(p.B, b0 + per);
  if (t == 0) s_bad = 0;
  __syncthreads();
  int64_t seg = 0;
  for (int64_t b = b0; b < b1; ++b) {
    const int64_t len = p.context_lens[b], n = p.rewind[b];
    if (n < 0 || len < 0 || n > len || (len + p.ps - 1) / p.ps > p.mp) {
      atomicExch(&s_bad, 1);
      continue;
    }
    int64_t have, first, calls, nl;
    bool fwd;
    rewind_span(p, b, have, first, calls, fwd, nl);
    for (int64_t k = 0; k < calls; ++k) {
      const int64_t pid = p.block_table[b * p.mp + (fwd ? k : have - 1 - k)];
      if (pid < 0 || pid >= p.capacity || p.refcount[pid] <= 0) atomicExch(&s_bad, 1);
    }
    seg += calls;
  }
  const int64_t incl = block_inclusive_scan(seg, scan_buf);
  int64_t run = incl - seg;
  for (int64_t b = b0; b < b1; ++b) {
    call_start[b] = (int32_t)run;
    const int64_t len = p.context_lens[b], n = p.rewind[b];
    if (n < 0 || len < 0 || n > len || (len + p.ps - 1) / p.ps > p.mp) continue;
    int64_t have, first, calls, nl;
    bool fwd;
    rewind_span(p, b, have, first, calls, fwd, nl);
    run += calls;
  }
  if (t == kThreads - 1) call_start[p.B] = (int32_t)incl;
  __syncthreads();
  if (s_bad) {
    if (t == 0) *p.status = NVM_ERR_INVALID_ARGUMENT;
    return;
  }
  const int64_t total = call_start[p.B];
  auto call_page = [&](int64_t i, int64_t& b, int64_t& slot) -> int64_t {
    b = owner_of(call_start, p.B, i);
    int64_t have, first, calls, nl;
    bool fwd;
    rewind_span(p, b, have, first, calls, fwd, nl);
    const int64_t k = i - call_start[b];
    slot = fwd ? k : have - 1 - k;
    return p.block_table[b * p.mp + slot];
  };
  // every call drops one reference; the last call of each page in order is recorded
  for (int64_t i = t; i < total; i += kThreads) {
    int64_t b, slot;
    const int64_t pid = call_page(i, b, slot);
    atomicSub(&p.refcount[pid], 1);
    atomicMax(&p.last_call[pid], (int32_t)i);
  }
  __syncthreads();
  // pushes in call order: contiguous call ranges per thread, ranked by a block scan
  const int64_t cper = (total + kThreads - 1) / kThreads;
  const int64_t i0 = min(total, t * cper), i1 = min(total, i0 + cper);
  int64_t pushes = 0;
  for (int64_t i = i0; i < i1; ++i) {
    int64_t b, slot;
    const int64_t pid = call_page(i, b, slot);
    pushes += (p.refcount[pid] == 0 && p.last_call[pid] == i) ? 1 : 0;
  }
  const int64_t pincl = block_inclusive_scan(pushes, scan_buf);
  const int64_t top = *p.free_top;
  int64_t pos = top + pincl - pushes;
  for (int64_t i = i0; i < i1; ++i) {
    int64_t b, slot;
    const int64_t pid = call_page(i, b, slot);
    if (p.refcount[pid] == 0 && p.last_call[pid] == i) p.free_stack[pos++] = (int32_t)pid;
  }
  __syncthreads();
  // scratch back to -1, freed block-table entries to -1, new lengths
  for (int64_t i = t; i < total; i += kThreads) {
    int64_t b, slot;
    const int64_t pid = call_page(i, b, slot);
    p.last_call[pid] = -1;
  }
  __syncthreads();
  for (int64_t i = t; i < total; i += kThreads) {
    int64_t b, slot;
    call_page(i, b, slot);
    p.block_table[b * p.mp + slot] = -1;
  }
  __syncthreads();
  for (int64_t b = t; b < p.B; b += kThreads) p.context_lens[b] -= p.rewind[b];
  if (t == kThreads - 1) {
    *p.free_top = (int32_t)(top + pincl);
    *p.status = NVM_OK;
  }
}

// ---------------------------------------------------------------------------
// Prefix attach (PrefixCache.attach, paged.py:305-328, for one layer's pool): fresh
// requests take `count[b]` shared full pages; each page gains a reference.
struct AttachParams {
  int32_t* block_table;
  int32_t* context_lens;
  const int32_t* pages;
  const int32_t* count;
  int32_t* refcount;
  int32_t* status;
  int64_t B, mp, ps, max_prefix, capacity;
};

__global__ void __launch_bounds__(kThreads) paged_attach_kernel(AttachParams p) {
  __shared__ int s_bad;
  const int t = threadIdx.x;
  if (t == 0) s_bad = 0;
  __syncthreads();
  for (int64_t b = t; b < p.B; b += kThreads) {
    const int64_t c = p.count[b];
    if (c < 0 || c > p.mp || c > p.max_prefix) {
      atomicExch(&s_bad, 1);
      continue;
    }
    if (c > 0 && (p.context_lens[b] != 0 || p.block_table[b * p.mp] != -1)) atomicExch(&s_bad, 1);
    for (int64_t k = 0; k < c; ++k) {
      const int64_t pid = p.pages[b * p.max_prefix + k];
      if (pid < 0 || pid >= p.capacity || p.refcount[pid] <= 0) atomicExch(&s_bad, 1);
    }
  }
  __syncthreads();
  if (s_bad) {
    if (t == 0) *p.status = NVM_ERR_INVALID_ARGUMENT;
    return;
  }
  for (int64_t b = 0; b < p.B; ++b) {
    const int64_t c = p.count[b];
    for (int64_t k = t; k < c; k += kThreads) {
      const int32_t pid = p.pages[b * p.max_prefix + k];
      p.block_table[b * p.mp + k] = pid;
      atomicAdd(&p.refcount[pid], 1);
    }
  }
  __syncthreads();
  for (int64_t b = t; b < p.B; b += kThreads)
    if (p.count[b] > 0) p.context_lens[b] = (int32_t)(p.count[b] * p.ps);
  if (t == 0) *p.status = NVM_OK;
}

}  // namespace

int launch_paged_rewind(int32_t* block_table, int32_t* context_lens, const int32_t* rewind, int32_t* free_stack,
                        int32_t* free_top, int32_t* page_refcount, int32_t* last_call, int32_t* status, int64_t B,
                        int64_t max_pages, int64_t page_size, int64_t capacity, cudaStream_t s) {
  RewindParams p{block_table, context_lens, rewind, free_stack, free_top, page_refcount, last_call, status,
                 B, max_pages, page_size, capacity};
  paged_rewind_kernel<<<1, kThreads, 0, s>>>(p);
  return check_cuda(cudaGetLastError(), "rewind: kernel launch");
}

int launch_paged_attach(int32_t* block_table, int32_t* context_lens, const int32_t* pages, const int32_t* count,
                        int32_t* page_refcount, int32_t* status, int64_t B, int64_t max_pages, int64_t page_size,
                        int64_t max_prefix, int64_t capacity, cudaStream_t s) {
  AttachParams p{block_table, context_lens, pages, count, page_refcount, status, B, max_pages, page_size,
                 max_prefix, capacity};
  paged_attach_kernel<<<1, kThreads, 0, s>>>(p);
  return check_cuda(cudaGetLastError(), "attach: kernel launch");
}

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
