/*
 * nvm_attn.h -- C ABI of libnvm_attn.so, the B200 (sm_100a) attention hot path of
 * nano-vllm-metal: paged-attention decode / multi-query, dense flash attention,
 * the paged KV scatter-write (with int8 quantise-on-write), device-side page
 * allocation for a batch of appends, and the fused per-layer q/k RMSNorm + RoPE +
 * K/V write that precedes every attention call, and the 4-bit (W4A16) matmul of the
 * projections around it.
 *
 * Conventions shared by every entry point
 *   - All tensor arguments are raw DEVICE pointers to row-major contiguous memory
 *     (strides are given explicitly where an argument may be a strided view).
 *   - Sizes are int64_t element counts.  Element types are `nvm_dtype` codes.
 *   - `stream` is a cudaStream_t passed as void*; every call is stream-ordered and
 *     never synchronises the device.  NULL means the legacy default stream.
 *   - Return value: NVM_OK (0) or a negative nvm_status.  No C++ exception crosses
 *     the ABI.  nvm_last_error() returns the message of the last failing call on
 *     the calling thread; messages start with the reference operator's name
 *     ("paged_attention: ...", "flash_attention: ...") so a Python wrapper can
 *     re-raise them verbatim.
 *   - The library holds no mutable global state apart from a per-device error word
 *     written by kernels whose bounded waits expire (nvm_device_error()).
 *
 * Reference interfaces replaced (paths inside PepperoniBlvd/nano-vllm-metal):
 *   src/nano_vllm_metal/metal/bindings.cpp:34-82           (nanobind _ext module)
 *   src/nano_vllm_metal/metal/src/kernels.h:37-75          (operator declarations)
 *   src/nano_vllm_metal/metal/src/paged_attention.cpp:19-120, 413-642
 *   src/nano_vllm_metal/metal/src/flash_attention.cpp:17-61, 251-352
 *   src/nano_vllm_metal/cache/paged.py:152-195             (page write + int8 quantiser)
 *   src/nano_vllm_metal/cache/paged.py:60-70, 424-459      (page allocation on append)
 *   src/nano_vllm_metal/cache/paged.py:197-210, 305-328, 530-559 (free, prefix attach,
 *                                                            rewind, release)
 *   src/nano_vllm_metal/models/qwen3.py:100-116            (q/k norm, RoPE, cache update)
 *   src/nano_vllm_metal/layers/layernorm.py:4-14, layers/rotary_embedding.py:74-124
 *   src/nano_vllm_metal/metal/src/quantized_matmul.cpp:7-270  (W4A16 matmul)
 *   src/nano_vllm_metal/engine/generate.py:130-169         (speculative acceptance)
 */
#ifndef NVM_ATTN_H_
#define NVM_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element type codes. */
typedef enum nvm_dtype {
  NVM_F32 = 0,
  NVM_F16 = 1,
  NVM_BF16 = 2,
  NVM_I8 = 3,
  NVM_I32 = 4,
  NVM_I64 = 5
} nvm_dtype;

/* Status codes (0 = success). */
typedef enum nvm_status {
  NVM_OK = 0,
  NVM_ERR_INVALID_ARGUMENT = -1, /* bad shape / dtype / pointer combination      */
  NVM_ERR_UNSUPPORTED = -2,      /* valid request this build cannot serve        */
  NVM_ERR_WORKSPACE = -3,        /* workspace missing or smaller than required   */
  NVM_ERR_CUDA = -4,             /* a CUDA runtime / driver call failed          */
  NVM_ERR_DEVICE_TIMEOUT = -5,   /* a kernel's bounded wait expired (see below)  */
  NVM_ERR_OUT_OF_PAGES = -6      /* page allocation exceeded the pool capacity   */
} nvm_status;

/* Human-readable name of a status code (static string). */
const char* nvm_status_string(int status);

/* Detailed message of the last failing call on this thread ("" if none). */
const char* nvm_last_error(void);

/* Library version string, e.g. "nvm_attn 0.1 sm_100a". */
const char* nvm_version(void);

/*
 * Device error word.  Kernels that spin on an mbarrier give every wait an
 * iteration/time limit; when one expires the kernel records a nonzero code here,
 * drains its own in-flight copies (bounded) and returns, leaving the context
 * usable.  nvm_device_error() synchronises `stream`, reads the word of the current
 * device, optionally clears it, and returns it (0 = no error).  The first code
 * recorded stays: 1 a wait for a tile to land expired, 2 a wait for a free stage,
 * 3 draining in-flight copies, 4 tensor-memory allocation, 5 tensor-core completion,
 * 6 dynamic shared memory was not 1024-byte aligned (that kernel computed nothing),
 * 7 a device-side index (a rope position or a slot) was outside its table (row skipped).
 */
int nvm_device_error(void* stream, int clear);

/*
 * Failure-detection self-test (no counterpart in the reference: the reference's Metal
 * kernels have no bounded waits).  Launches one warp on `stream` that waits on an
 * mbarrier nobody arrives on, through the same bounded wait the kernels use, but
 * with a limit of `limit_ns` (1e3 .. 1e8 ns) instead of 2 s.  When it expires the
 * kernel records code 1 in the device error word and returns, so that a following
 * nvm_device_error() returns 1 and the device keeps serving calls.  waited_ns, if
 * not NULL, is a device uint64 that receives the time the wait took.
 */
int nvm_selftest_wait_expiry(int64_t limit_ns, unsigned long long* waited_ns, void* stream);

/* ------------------------------------------------------------------------- */
/* Paged attention (decode, multi-token verify, chunked prefill)              */
/* ------------------------------------------------------------------------- */
/*
 * Replaces: _ext.paged_attention / _ext.paged_attention_int8_decode
 *   (src/nano_vllm_metal/metal/bindings.cpp:34-66,
 *    src/nano_vllm_metal/metal/src/paged_attention.cpp:19-120 validation,
 *    :413-574 and :576-642 GPU dispatch) and the dequantise-then-attend int8 L>1
 *    path of src/nano_vllm_metal/layers/attention.py:204-215 (done in-kernel here).
 *
 * q            [B*Hq, L, D] of q_dtype (F32/F16/BF16), row n = b*Hq + head.
 * k_pages,
 * v_pages      [P, Hkv, page_size, D] of kv_dtype (F32/F16/BF16/I8).
 * k_scales,
 * v_scales     [P, Hkv, page_size, 1] of scale_dtype (F32/F16/BF16); required iff
 *              kv_dtype == NVM_I8, else NULL.  value = int8 * scale.
 * block_table  [B, max_pages] int32 physical page ids; entries < 0 (or >= P) are
 *              holes whose positions are skipped, as in paged_attention.cpp:216-222.
 * context_lens [B] int32; context_len <= 0 gives a zero output row block.
 * out          [B*Hq, L, D] of out_dtype (F32/F16/BF16); the reference returns F32.
 * scale        softmax scale applied to q.k.
 * is_causal    row l of L may see key positions <= l + context_len - L.
 * workspace    device scratch of at least nvm_paged_attention_workspace_size(...)
 *              bytes.  Its first 1 MiB holds split-K tickets: it must be zero-
 *              filled before the first use and every successful call leaves it
 *              zero again, so one workspace serves calls of any shape; the rest
 *              is overwritten by every call.  May be NULL if the size is 0.
 *              Calls that share one workspace must not overlap on the GPU.
 */
int nvm_paged_attention(const void* q, int q_dtype, const void* k_pages, const void* v_pages,
                        int kv_dtype, const void* k_scales, const void* v_scales, int scale_dtype,
                        const int32_t* block_table, const int32_t* context_lens, void* out,
                        int out_dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t L, int64_t D,
                        int64_t P, int64_t page_size, int64_t max_pages, float scale,
                        int is_causal, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes nvm_paged_attention needs for these sizes (0 if none). */
size_t nvm_paged_attention_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t L,
                                          int64_t D, int64_t page_size, int64_t max_pages,
                                          int kv_dtype);

/*
 * nvm_paged_attention without a workspace argument.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory on their
 * hot path (an engine that gives all free HBM to its page pools up front, a decode
 * loop that cannot afford cudaMalloc's implicit device synchronisation, a host
 * without a device allocator).  Arguments and results are those of
 * nvm_paged_attention.  The split-K scratch is a 32 MiB array built into the
 * library; the runtime takes its device memory at the first call on each device
 * (lazy module loading) and holds it until the process exits, so make one call, of
 * any size, on each device before sizing page pools from the free memory and before
 * any stream capture (that first call also resolves the array's device address).
 * Sizes whose plan needs more than 32 MiB return NVM_ERR_WORKSPACE before any GPU
 * work.  Every call clears the scratch tickets on `stream` and shares the one
 * array: calls that overlap on the GPU race.  Allocates nothing.
 */
int nvm_paged_attention_noalloc(const void* q, int q_dtype, const void* k_pages,
                                const void* v_pages, int kv_dtype, const void* k_scales,
                                const void* v_scales, int scale_dtype, const int32_t* block_table,
                                const int32_t* context_lens, void* out, int out_dtype, int64_t B,
                                int64_t Hq, int64_t Hkv, int64_t L, int64_t D, int64_t P,
                                int64_t page_size, int64_t max_pages, float scale, int is_causal,
                                void* stream);

/* ------------------------------------------------------------------------- */
/* Dense flash attention (prefill)                                            */
/* ------------------------------------------------------------------------- */
/*
 * Replaces: _ext.flash_attention (src/nano_vllm_metal/metal/bindings.cpp:68-82,
 *   src/nano_vllm_metal/metal/src/flash_attention.cpp:17-61 validation, :251-352
 *   dispatch) and the MLX fast SDPA call of the initial-prefill branch
 *   (src/nano_vllm_metal/models/qwen3.py:137-144).
 *
 * q            [B*Hq, L, D], k/v [B*Hkv, S, D], all of `dtype` (F32/F16/BF16).
 * mask         optional additive F32 mask read as mask[n*ms_n + l*ms_l + s*ms_s]
 *              (strides in elements, 0 broadcasts), or NULL.  With is_causal the
 *              rows see keys s <= l + S - L (flash_attention.cpp:132-139) and the
 *              mask, when given, is added on the visible keys only for tiles that
 *              are not fully visible -- exactly the reference's block skip.
 * out          [B*Hq, L, D] of out_dtype.
 */
int nvm_flash_attention(const void* q, const void* k, const void* v, int dtype, const float* mask,
                        int64_t mask_stride_n, int64_t mask_stride_l, int64_t mask_stride_s,
                        void* out, int out_dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t L,
                        int64_t S, int64_t D, float scale, int is_causal, void* stream);

/* ------------------------------------------------------------------------- */
/* Paged KV scatter-write (+ int8 quantise-on-write)                          */
/* ------------------------------------------------------------------------- */
/*
 * Replaces: TinyKvPagedPool.write_page_slice / _quantize_page_slice
 *   (src/nano_vllm_metal/cache/paged.py:152-195) as driven by
 *   TinyKvPagedCache._append_chunk (paged.py:424-459) and
 *   BatchingKvCache.update_and_fetch_paged (src/nano_vllm_metal/cache/kv_cache.py:134-151).
 *
 * k, v         token t, head h element d at k[t*stride_t + h*stride_h + d]
 *              (element strides; d is contiguous), of in_dtype (F32/F16/BF16).
 * slot_mapping [T] int64: slot = page_id*page_size + offset, or < 0 to skip.
 * k_pages,
 * v_pages      [P, Hkv, page_size, D] of kv_dtype.  kv_dtype == in_dtype copies the
 *              bits; kv_dtype == NVM_I8 quantises each (token, head) row:
 *                amax = max|x| (fp32); s = amax > 0 ? amax/127 : 1;
 *                q = clip(round_half_even(x / s), -127, 127);
 *              and stores s rounded to scale_dtype in k_scales / v_scales
 *              [P, Hkv, page_size, 1] (paged.py:153-158).
 * Pages are mutated in place (the reference's buffer-donating slice-assign).
 */
int nvm_reshape_and_cache(const void* k, const void* v, int in_dtype, int64_t stride_t,
                          int64_t stride_h, void* k_pages, void* v_pages, int kv_dtype,
                          void* k_scales, void* v_scales, int scale_dtype,
                          const int64_t* slot_mapping, int64_t T, int64_t Hkv, int64_t D,
                          int64_t P, int64_t page_size, void* stream);

/* ------------------------------------------------------------------------- */
/* Fused per-layer preparation: q/k RMSNorm + RoPE + K/V scatter-write        */
/* ------------------------------------------------------------------------- */
/*
 * Replaces the steps of Qwen3Attention.__call__ between the QKV projection and the
 * attention call (src/nano_vllm_metal/models/qwen3.py:100-116): q_norm/k_norm
 * (layers/layernorm.py:4-14, RMSNorm over the head dim with weight, eps), RoPE on q and
 * k (layers/rotary_embedding.py:74-124; halves rotated, or interleaved pairs when
 * traditional != 0) and the pool write of cache.update_and_fetch_paged
 * (cache/paged.py:160-195, int8 through _quantize_page_slice, paged.py:152-158).
 *   q [T, Hq, D], k/v [T, Hkv, D] (dtype f16/bf16; q_stride_t / kv_stride_t elements
 *   between tokens, heads contiguous); q_norm_weight / k_norm_weight [D] (dtype);
 *   cos_table / sin_table [table_rows, D/2] fp32 (position p, angle index i);
 *   positions [T] int32 (the token's position = request offset + index in the chunk);
 *   q_out: the normalised, rotated q, [T, Hq, D], or [T/q_out_L, Hq, q_out_L, D] when
 *   q_out_L > 0 (the [B, Hq, L, D] layout paged_attention takes);
 *   K (normalised, rotated) and V (as given) go to the pages at slot_mapping[t]
 *   (page_id * page_size + offset; negative = skip), copied or int8-quantised as
 *   nvm_reshape_and_cache does.  D must be 64 or 128.  Rounding follows the reference:
 *   the norm result and the rotation result are each rounded to dtype, the rotation is
 *   computed in fp32 from the rounded norm result.
 */
int nvm_qk_norm_rope_write(const void* q, const void* k, const void* v, int dtype, int64_t q_stride_t,
                           int64_t kv_stride_t, const void* q_norm_weight, const void* k_norm_weight,
                           float eps, const float* cos_table, const float* sin_table, int64_t table_rows,
                           int traditional, const int32_t* positions, void* q_out, int64_t q_out_L,
                           void* k_pages, void* v_pages, int kv_dtype, void* k_scales, void* v_scales,
                           int scale_dtype, const int64_t* slot_mapping, int64_t T, int64_t Hq,
                           int64_t Hkv, int64_t D, int64_t P, int64_t page_size, void* stream);

/* ------------------------------------------------------------------------- */
/* Device-side page allocation for one batched append                         */
/* ------------------------------------------------------------------------- */
/*
 * Replaces, for a whole batch at once and on the device: the per-request loop of
 * BatchingKvCache.update_and_fetch_paged (src/nano_vllm_metal/cache/kv_cache.py:134-173)
 * over TinyKvPagedCache._append_chunk (src/nano_vllm_metal/cache/paged.py:424-459)
 * and TinyKvPagedPool.allocate_page (paged.py:60-70).
 *
 * Request b appends new_tokens[b] >= 0 tokens (0 for an idle slot) after its
 * context_lens[b] existing tokens.  The tail page is filled first, then fresh
 * pages are popped, in request order, from the free stack (LIFO: the page taken
 * next is free_stack[*free_top - 1]); when the stack is empty fresh ids
 * *num_pages, *num_pages+1, ... are minted -- the same ids, in the same order, as
 * the reference's sequential allocate_page calls.  On success:
 *   block_table[b, :] gains the new page ids (row width max_pages),
 *   page_refcount[id] = 1 for each new page,
 *   slot_mapping[tok_offsets[b] + i] = slot of new token i of request b
 *     (tok_offsets = exclusive prefix sum of new_tokens, computed in-kernel),
 *   context_lens[b] += new_tokens[b], *free_top and *num_pages are updated.
 * capacity bounds minted ids; exceeding it, a block-table row, or the
 * slot_capacity entries of slot_mapping sets *status = NVM_ERR_OUT_OF_PAGES
 * (checked on the device before anything is written; nothing is written then).
 * Single CTA; B <= 4096.  The device ints are int32.
 */
int nvm_paged_append(int32_t* block_table, int32_t* context_lens, const int32_t* new_tokens,
                     int32_t* free_stack, int32_t* free_top, int32_t* num_pages,
                     int32_t* page_refcount, int64_t* slot_mapping, int64_t slot_capacity,
                     int32_t* status, int64_t B, int64_t max_pages, int64_t page_size,
                     int64_t capacity, void* stream);

/*
 * Batched rewind / release on the device.  Replaces, for b = 0..B-1 in order,
 * TinyKvPagedCache.rewind(n) (src/nano_vllm_metal/cache/paged.py:530-550; n equal to
 * the request's length is release(), paged.py:552-559) with TinyKvPagedPool.free_page
 * (paged.py:197-210) -- e.g. dropping the rejected draft tokens of a batched
 * speculative verify (engine/generate.py:55-169), or finishing requests.
 *
 * Request b drops rewind[b] tokens (0 <= rewind[b] <= context_lens[b]).  Pages past
 * the new length lose one reference each (release walks the row forward, rewind pops
 * it from the end); a page whose count reaches zero is pushed on the free stack at the
 * position of the reference's sequential call that freed it.  Freed block-table
 * entries become -1, context_lens[b] -= rewind[b].  last_call is [capacity] int32
 * scratch holding -1 (and left so).  Invalid lengths or page ids set *status =
 * NVM_ERR_INVALID_ARGUMENT before anything is written.  Single CTA; B <= 4096.
 */
int nvm_paged_rewind(int32_t* block_table, int32_t* context_lens, const int32_t* rewind,
                     int32_t* free_stack, int32_t* free_top, int32_t* page_refcount,
                     int32_t* last_call, int32_t* status, int64_t B, int64_t max_pages,
                     int64_t page_size, int64_t capacity, void* stream);

/*
 * Prefix attach on the device: PrefixCache.attach (src/nano_vllm_metal/cache/paged.py:
 * 305-328) for one layer's pool.  Fresh request b (no pages, length 0) with
 * count[b] > 0 takes the shared full pages pages[b, 0:count[b]] (row width
 * max_prefix): block_table[b, k] = pages[b, k], each page gains one reference,
 * context_lens[b] = count[b] * page_size.  A non-fresh row or an invalid page sets
 * *status = NVM_ERR_INVALID_ARGUMENT before anything is written.
 */
int nvm_paged_attach(int32_t* block_table, int32_t* context_lens, const int32_t* pages,
                     const int32_t* count, int32_t* page_refcount, int32_t* status, int64_t B,
                     int64_t max_pages, int64_t page_size, int64_t max_prefix, int64_t capacity,
                     void* stream);

/*
 * Batched speculative-decoding acceptance on the device.  Replaces, for a whole batch
 * in one launch, the per-request acceptance loop of speculative_generate
 * (src/nano_vllm_metal/engine/generate.py:130-169), whose result drives the rewind of
 * cache/paged.py:530-550 (nvm_paged_rewind here).
 *
 * candidates [B, K1] int32: the request's last accepted token, then its K1 - 1 drafts.
 * verified   [B, K1] int32: the target model's argmax at each of the K1 positions.
 * Request b walks positions i = 0 .. K1-1, comparing (i == 0 ? candidates[b][0] :
 * verified[b][i-1]) with candidates[b][i]:
 *   match: the token is emitted, unless it equals eos_id (request finished, token not
 *     emitted); when budget[b] >= 0 tokens have been emitted the request is finished;
 *   first mismatch at i: rewind[b] = K1 - i tokens are dropped from the target cache,
 *     draft_rewind[b] = K1 - i - 1 from the draft cache, next_token[b] =
 *     verified[b][i-1] (finished if it equals eos_id);
 *   all matched: next_token[b] = verified[b][K1-1], rewind[b] = draft_rewind[b] = 0.
 * Outputs: emitted [B, K1] (-1 padded), n_emitted, next_token (-1 when finished by an
 * emitted eos or the budget), rewind, draft_rewind, finished (0/1), all [B] int32.
 * budget and active ([B] int32, active[b] == 0 marks an idle slot with zero outputs)
 * may be NULL; eos_id < 0 disables the end-of-sequence check.
 */
int nvm_spec_verify_accept(const int32_t* candidates, const int32_t* verified, int64_t B, int64_t K1,
                           int32_t eos_id, const int32_t* budget, const int32_t* active,
                           int32_t* emitted, int32_t* n_emitted, int32_t* next_token, int32_t* rewind,
                           int32_t* draft_rewind, int32_t* finished, void* stream);

/* ------------------------------------------------------------------------- */
/* W4A16 quantized matmul (4-bit weights, group 128)                          */
/* ------------------------------------------------------------------------- */
/*
 * Replaces QuantizedMatmul (src/nano_vllm_metal/metal/src/quantized_matmul.cpp:7-270;
 * Metal kernels quantized_matmul.metal:5-123; caller layers/linear.py:73-126):
 *   out[m, k] = sum_n a[m, n] * (q[k, n] * scales[k, n / 128] + biases[k, n / 128])
 * a [M, N] and out [M, K] in `dtype` (NVM_F16 / NVM_BF16, row-major), w [K, N / 8]
 * uint32 with element n of a word in bits 4 (n % 8) .. 4 (n % 8) + 3, scales and
 * biases [K, N / 128] in `dtype`; fp32 accumulation, the result rounded to `dtype`.
 * group_size must be 128 and bits 4 (as the reference), N a multiple of 128, a and w
 * 16-byte aligned.  Weights are read once per 16 rows of a.
 */
int nvm_w4a16_matmul(const void* a, int dtype, const uint32_t* w, const void* scales,
                     const void* biases, void* out, int64_t M, int64_t N, int64_t K,
                     int64_t group_size, int64_t bits, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NVM_ATTN_H_ */
