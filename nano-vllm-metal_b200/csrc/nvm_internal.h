// nvm_internal.h -- host-side declarations shared by the translation units of
// libnvm_attn.so (not part of the public ABI; see include/nvm_attn.h for that).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "nvm_attn.h"

namespace nvm {

// Records the message returned by nvm_last_error() for this thread; returns `status`.
int fail(int status, const char* fmt, ...);
// Maps a CUDA runtime error (after a launch or API call) to NVM_ERR_CUDA + message.
int check_cuda(cudaError_t e, const char* what);
// Device address of the calling device's error word (set up once per device).
int* device_error_word();

size_t dtype_size(int dtype);

// Bytes at the start of every split-K workspace that hold the ticket counters: zero
// before a call, zero again after a successful one.  paged_mma.cu and flash_sm100.cu
// lay their counters out inside this region; noalloc.cu clears exactly this much.
constexpr size_t kTicketRegionBytes = size_t(1) << 20;

// Arguments of one paged-attention call after validation.  block_table == nullptr
// selects the dense identity layout used by flash attention: sequence b owns
// "page" b of size page_size == S, and context_lens == nullptr means every
// sequence holds `dense_ctx` tokens.
struct PagedArgs {
  const void* q;
  int q_dtype;
  const void* k_pages;
  const void* v_pages;
  int kv_dtype;
  const void* k_scales;
  const void* v_scales;
  int scale_dtype;
  const int32_t* block_table;
  const int32_t* context_lens;
  void* out;
  int out_dtype;
  int64_t B, Hq, Hkv, L, D, P, page_size, max_pages;
  float scale;
  int is_causal;
  int dense;          // 1: dense K/V viewed as one page per sequence (no block table)
  int64_t dense_ctx;  // tokens per sequence when dense
};

// Generic CUDA-core kernel: any D <= 256, any page_size, F32/F16/BF16/I8 pages.
int launch_paged_generic(const PagedArgs& a, cudaStream_t s);

// Generic dense flash attention with the reference's additive-mask semantics.
struct FlashArgs {
  const void* q;
  const void* k;
  const void* v;
  int dtype;
  const float* mask;
  int64_t ms_n, ms_l, ms_s;
  void* out;
  int out_dtype;
  int64_t B, Hq, Hkv, L, S, D;
  float scale;
  int is_causal;
};
int launch_flash_generic(const FlashArgs& a, cudaStream_t s);

// Tensor-core (mma.sync m16n8k16) paged kernel fed by TMA tiles.
struct MmaPlan {
  bool eligible;   // shapes/dtypes/alignment served by the tensor-core kernel
  int nwm;         // 16-row m-tiles per CTA (warps along rows)
  int nwk;         // warps splitting the key tiles of one CTA
  int variant;     // decode kernel variant (consumer warps x stage depth)
  int rows_per_block;
  int64_t n_row_blocks;
  int64_t rows_real;      // rows of one (seq, kv head) unit actually stored per block
  int64_t chunk_tiles;    // 16-token tiles per CTA (split-K granularity)
  int64_t n_chunks;       // max chunks per unit
  int64_t n_units;
  size_t ws_bytes;        // workspace for the split-K combine (0 if n_chunks == 1 or cluster)
  int cluster;            // 1: a unit's n_chunks CTAs form one thread-block cluster and merge
                          // their partial results over distributed shared memory (no workspace)
};
MmaPlan plan_paged_mma(const PagedArgs& a);
int launch_paged_mma(const PagedArgs& a, const MmaPlan& plan, void* workspace, cudaStream_t s);

// tcgen05 / TMEM causal prefill (dense or paged) for 16-bit Q/K/V, D == 128.
// tcgen05/TMEM kernel (flash_sm100.cu): prefill (>= 64 query rows per head) and grouped
// few-token calls (a kv head's g*L query rows as one tile, split-K over keys when paged).
struct Sm100Plan {
  bool eligible;
  int grouped;
  int64_t M_rows, n_outer, n_row_tiles, n_units, rows_real, ct, n_chunks;
  size_t ws_bytes;
};
// sizing_only: plan from shapes alone (q dtype, pointers and scale unknown), for
// nvm_paged_attention_workspace_size.
Sm100Plan plan_sm100(const PagedArgs& a, bool sizing_only);
int launch_sm100(const PagedArgs& a, const Sm100Plan& plan, void* ws, cudaStream_t s);

// tcgen05 kernel with two 128-row query tiles per CTA (flash_2q.cu): prefill with at least
// 256 query rows per head, 16-bit, D == 128; no workspace.
bool flash2q_eligible(const PagedArgs& a);
int launch_flash2q(const PagedArgs& a, cudaStream_t s);

int launch_kv_write(const void* k, const void* v, int in_dtype, int64_t stride_t, int64_t stride_h,
                    void* k_pages, void* v_pages, int kv_dtype, void* k_scales, void* v_scales,
                    int scale_dtype, const int64_t* slot_mapping, int64_t T, int64_t Hkv, int64_t D,
                    int64_t P, int64_t page_size, cudaStream_t s);

int launch_paged_append(int32_t* block_table, int32_t* context_lens, const int32_t* new_tokens,
                        int32_t* free_stack, int32_t* free_top, int32_t* num_pages,
                        int32_t* page_refcount, int64_t* slot_mapping, int64_t slot_capacity, int32_t* status, int64_t B,
                        int64_t max_pages, int64_t page_size, int64_t capacity, cudaStream_t s);
int launch_paged_rewind(int32_t* block_table, int32_t* context_lens, const int32_t* rewind, int32_t* free_stack,
                        int32_t* free_top, int32_t* page_refcount, int32_t* last_call, int32_t* status, int64_t B,
                        int64_t max_pages, int64_t page_size, int64_t capacity, cudaStream_t s);
int launch_paged_attach(int32_t* block_table, int32_t* context_lens, const int32_t* pages, const int32_t* count,
                        int32_t* page_refcount, int32_t* status, int64_t B, int64_t max_pages, int64_t page_size,
                        int64_t max_prefix, int64_t capacity, cudaStream_t s);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle);

}  // namespace nvm
