/*
 * nvm_oracle.c -- TEST INFRASTRUCTURE ONLY.  CPU restatement of the reference's
 * attention hot path, used by tests/ as the parity checker and by bench.py as the
 * CPU baseline.  It is never linked into, called by, or shipped as part of the
 * product library (libnvm_attn.so); the product path fails loudly without CUDA.
 *
 * Reference: PepperoniBlvd/nano-vllm-metal (pinned mlx 0.29.1, pdm.lock:785-786).
 * The reference's own CPU path is the MLX primitives' eval_cpu, plain C++ loops
 * inside one encoder.dispatch lambda.  MLX is not importable in this container and
 * the reference cannot be compiled without MLX headers, so those loops are restated
 * here in our own C, function by function, keeping the reference's tiling (Br=Bc=32)
 * and accumulation order so results match it to float rounding.
 *
 * Parity pin: the reference ships no golden vectors.  This restatement is pinned by
 * the reference's own differential tests and known-answer assertions, re-run in
 * tests/test_oracle.py (paged vs dense flash attention, batched decode with an empty
 * slot, int8 decode vs dequantised grouped SDPA, flash attention vs grouped SDPA),
 * and by the committed fixtures in tests/golden/ produced by tests/golden/make_golden.py.
 *
 * Float contraction is disabled at build time (-ffp-contract=off) so the products
 * and sums below are evaluated exactly as written.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2, OR_I8 = 3 };

static inline float bf16_to_f32(uint16_t h) {
  union { uint32_t u; float f; } v;
  v.u = ((uint32_t)h) << 16;
  return v.f;
}

static inline float f16_to_f32(uint16_t h) {
  _Float16 x;
  memcpy(&x, &h, 2);
  return (float)x;
}

/* fp32 -> bf16 bits, round to nearest even (NaN kept quiet). */
static inline uint16_t f32_to_bf16(float f) {
  union { uint32_t u; float f; } v;
  v.f = f;
  if ((v.u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((v.u >> 16) | 0x40u);
  uint32_t rounding = 0x7fffu + ((v.u >> 16) & 1u);
  return (uint16_t)((v.u + rounding) >> 16);
}

/* fp32 -> f16 bits, round to nearest even (compiler's IEEE conversion). */
static inline uint16_t f32_to_f16(float f) {
  _Float16 x = (_Float16)f;
  uint16_t h;
  memcpy(&h, &x, 2);
  return h;
}

static inline float load_elem(const void* base, int64_t idx, int dtype) {
  switch (dtype) {
    case OR_F32: return ((const float*)base)[idx];
    case OR_F16: return f16_to_f32(((const uint16_t*)base)[idx]);
    case OR_BF16: return bf16_to_f32(((const uint16_t*)base)[idx]);
    default: return (float)((const int8_t*)base)[idx];
  }
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
  omp_set_num_threads(nthreads > 0 ? nthreads : 1);
#else
  (void)nthreads;
#endif
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_num_procs();
#else
  return 1;
#endif
}

/*
 * PagedAttention::eval_cpu -- src/nano_vllm_metal/metal/src/paged_attention.cpp:148-287.
 * q [N, L, D] f32 (N = B*num_heads); pages [P, Hkv, page_size, D] of kv_dtype
 * (F32/F16/BF16); block_table [B, max_pages]; context_lens [B]; out [N, L, D] f32.
 * Rows are processed in Br=32 tiles against Bc=32 key tiles with an online softmax;
 * causal skips key > row + (ctx - L); holes (page id < 0) are skipped; ctx <= 0 -> 0.
 */
void oracle_paged_attention(const float* q, const void* key_pages, const void* value_pages,
                            int kv_dtype, const int32_t* block_table, const int32_t* context_lens,
                            float* out, int64_t N, int64_t L, int64_t D, int64_t num_kv_heads,
                            int64_t num_heads, int64_t page_size, int64_t max_pages, float scale,
                            int is_causal, int nthreads) {
  const int64_t q_kv_ratio = num_heads / num_kv_heads;
  const int64_t Br = 32, Bc = 32;
  const int64_t Tr = (L + Br - 1) / Br;
  const int64_t S_capacity = max_pages * page_size;
  const int64_t context_capacity = S_capacity > 0 ? S_capacity : 0;
  set_threads(nthreads);

#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t n = 0; n < N; n++) {
    const int64_t batch = n / num_heads;
    const int64_t q_head = n % num_heads;
    const int64_t kv_head = q_head / q_kv_ratio;
    const int64_t context_len = context_lens[batch];
    if (context_len <= 0) {
      for (int64_t x = 0; x < L * D; x++) out[n * L * D + x] = 0.0f;
      continue;
    }
    const int64_t context_limit = context_len < context_capacity ? context_len : context_capacity;
    const int64_t Tc = (context_limit + Bc - 1) / Bc;
    const int64_t causal_offset = context_len - L;

    float* q_i = (float*)malloc(sizeof(float) * Br * D);
    float* o_i = (float*)malloc(sizeof(float) * Br * D);
    float* s_i = (float*)malloc(sizeof(float) * Br * Bc);
    char* valid = (char*)malloc(Br * Bc);
    float l_i[32], m_i[32];

    for (int64_t i = 0; i < Tr; i++) {
      const int64_t br_upper = (L - i * Br) < Br ? (L - i * Br) : Br;
      for (int64_t x = 0; x < Br * D; x++) q_i[x] = 0.0f;
      for (int64_t a = 0; a < br_upper; a++)
        for (int64_t c = 0; c < D; c++) q_i[a * D + c] = q[n * L * D + (i * Br + a) * D + c];
      for (int64_t x = 0; x < Br * D; x++) o_i[x] = 0.0f;
      for (int64_t a = 0; a < Br; a++) {
        l_i[a] = 0.0f;
        m_i[a] = -INFINITY;
      }

      for (int64_t j = 0; j < Tc; j++) {
        const int64_t col_min = j * Bc;
        const int64_t row_max = i * Br + br_upper - 1;
        if (is_causal && col_min > row_max + causal_offset) continue;
        const int64_t bc_upper = (context_limit - col_min) < Bc ? (context_limit - col_min) : Bc;
        for (int64_t x = 0; x < Br * Bc; x++) {
          s_i[x] = -INFINITY;
          valid[x] = 0;
        }
        for (int64_t b = 0; b < bc_upper; b++) {
          const int64_t key_pos = col_min + b;
          const int64_t page_idx = key_pos / page_size;
          if (page_idx >= max_pages) continue;
          const int64_t page_id = block_table[batch * max_pages + page_idx];
          if (page_id < 0) continue;
          const int64_t slot = key_pos - page_idx * page_size;
          for (int64_t a = 0; a < br_upper; a++) {
            if (is_causal && key_pos > i * Br + a + causal_offset) continue;
            float score = 0.0f;
            for (int64_t c = 0; c < D; c++) {
              const int64_t k_idx = ((page_id * num_kv_heads + kv_head) * page_size + slot) * D + c;
              score += q_i[a * D + c] * load_elem(key_pages, k_idx, kv_dtype);
            }
            s_i[a * Bc + b] = score * scale;
            valid[a * Bc + b] = 1;
          }
        }
        for (int64_t a = 0; a < br_upper; a++) {
          float rowmax = -INFINITY;
          for (int64_t b = 0; b < bc_upper; b++)
            if (valid[a * Bc + b] && s_i[a * Bc + b] > rowmax) rowmax = s_i[a * Bc + b];
          if (rowmax == -INFINITY) continue;
          const float new_max = m_i[a] > rowmax ? m_i[a] : rowmax;
          const float old_scale = expf(m_i[a] - new_max);
          float rowsum = 0.0f;
          for (int64_t b = 0; b < bc_upper; b++)
            if (valid[a * Bc + b]) rowsum += expf(s_i[a * Bc + b] - new_max);
          for (int64_t c = 0; c < D; c++) {
            float res = 0.0f;
            for (int64_t b = 0; b < bc_upper; b++) {
              if (!valid[a * Bc + b]) continue;
              const int64_t key_pos = col_min + b;
              const int64_t page_idx = key_pos / page_size;
              const int64_t page_id = block_table[batch * max_pages + page_idx];
              const int64_t slot = key_pos - page_idx * page_size;
              const int64_t v_idx = ((page_id * num_kv_heads + kv_head) * page_size + slot) * D + c;
              res += expf(s_i[a * Bc + b] - new_max) * load_elem(value_pages, v_idx, kv_dtype);
            }
            o_i[a * D + c] = old_scale * o_i[a * D + c] + res;
          }
          l_i[a] = old_scale * l_i[a] + rowsum;
          m_i[a] = new_max;
        }
      }
      for (int64_t a = 0; a < br_upper; a++)
        for (int64_t c = 0; c < D; c++)
          out[n * L * D + (i * Br + a) * D + c] = l_i[a] > 0.0f ? o_i[a * D + c] / l_i[a] : 0.0f;
    }
    free(q_i);
    free(o_i);
    free(s_i);
    free(valid);
  }
}

/*
 * PagedAttentionInt8Decode::eval_cpu -- paged_attention.cpp:329-409.
 * Decode only (L == 1).  Two passes: scores with k = int8 * key_scale (fp32), then
 * softmax sum and the weighted value sum with v = int8 * value_scale.
 * key_scales / value_scales are fp32 [P, Hkv, page_size, 1] (the wrapper casts the
 * stored fp16/bf16 scales to fp32 before the call, attention.py:195-196).
 */
void oracle_paged_attention_int8_decode(const float* q, const int8_t* key_pages,
                                        const int8_t* value_pages, const float* key_scales,
                                        const float* value_scales, const int32_t* block_table,
                                        const int32_t* context_lens, float* out, int64_t N,
                                        int64_t D, int64_t num_kv_heads, int64_t num_heads,
                                        int64_t page_size, int64_t max_pages, float scale,
                                        int is_causal, int nthreads) {
  const int64_t q_kv_ratio = num_heads / num_kv_heads;
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t n = 0; n < N; n++) {
    const int64_t batch = n / num_heads;
    const int64_t q_head = n % num_heads;
    const int64_t kv_head = q_head / q_kv_ratio;
    const int64_t context_len = context_lens[batch];
    const int64_t context_capacity = max_pages * page_size;
    const int64_t context_limit = context_len < context_capacity ? context_len : context_capacity;
    if (context_limit <= 0) {
      for (int64_t c = 0; c < D; c++) out[n * D + c] = 0.0f;
      continue;
    }
    float* scores = (float*)malloc(sizeof(float) * context_limit);
    float rowmax = -INFINITY;
    for (int64_t pos = 0; pos < context_limit; pos++) {
      scores[pos] = -INFINITY;
      if (is_causal && pos > context_len - 1) continue;
      const int64_t page_idx = pos / page_size;
      const int64_t slot = pos - page_idx * page_size;
      const int64_t page_id = block_table[batch * max_pages + page_idx];
      if (page_id < 0) continue;
      const int64_t scale_idx = (page_id * num_kv_heads + kv_head) * page_size + slot;
      const float key_scale = key_scales[scale_idx];
      float score = 0.0f;
      for (int64_t c = 0; c < D; c++)
        score += q[n * D + c] * ((float)key_pages[scale_idx * D + c] * key_scale);
      scores[pos] = score * scale;
      if (scores[pos] > rowmax) rowmax = scores[pos];
    }
    float rowsum = 0.0f;
    for (int64_t pos = 0; pos < context_limit; pos++)
      if (scores[pos] != -INFINITY) rowsum += expf(scores[pos] - rowmax);
    for (int64_t c = 0; c < D; c++) {
      float acc = 0.0f;
      for (int64_t pos = 0; pos < context_limit; pos++) {
        if (scores[pos] == -INFINITY) continue;
        const int64_t page_idx = pos / page_size;
        const int64_t slot = pos - page_idx * page_size;
        const int64_t page_id = block_table[batch * max_pages + page_idx];
        const int64_t scale_idx = (page_id * num_kv_heads + kv_head) * page_size + slot;
        acc += expf(scores[pos] - rowmax) *
               ((float)value_pages[scale_idx * D + c] * value_scales[scale_idx]);
      }
      out[n * D + c] = rowsum > 0.0f ? acc / rowsum : 0.0f;
    }
    free(scores);
  }
}

/*
 * FlashAttention::eval_cpu -- src/nano_vllm_metal/metal/src/flash_attention.cpp:94-248.
 * q [N, L, E], k/v [N_kv, S, E] f32 (N_kv = N / (num_heads/num_kv_heads)); additive
 * f32 mask read at mask[n*ms_n + l*ms_l + s*ms_s] (the reference reads through
 * elem_to_loc, i.e. strides; broadcast dims have stride 0).  Causal skips key tiles
 * entirely above the diagonal (offset S - L) and skips the mask on tiles that are
 * entirely visible.  No l > 0 guard on the final division, as in the reference.
 */
void oracle_flash_attention(const float* q, const float* k, const float* v, const float* mask,
                            int64_t ms_n, int64_t ms_l, int64_t ms_s, float* out, int64_t N,
                            int64_t L, int64_t S, int64_t E, int64_t num_kv_heads,
                            int64_t num_heads, float scale, int is_causal, int nthreads) {
  const int64_t Br = 32, Bc = 32;
  const int64_t Tr = (L + Br - 1) / Br;
  const int64_t Tc = (S + Bc - 1) / Bc;
  const int64_t ratio = num_heads / num_kv_heads;
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t n = 0; n < N; n++) {
    const float* q_b = q + n * L * E;
    const float* k_b = k + (n / ratio) * S * E;
    const float* v_b = v + (n / ratio) * S * E;
    float* q_i = (float*)malloc(sizeof(float) * Br * E);
    float* o_i = (float*)malloc(sizeof(float) * Br * E);
    float* k_j = (float*)malloc(sizeof(float) * Bc * E);
    float* v_j = (float*)malloc(sizeof(float) * Bc * E);
    float s_i[32 * 32], p[32 * 32];
    float l_i[32], m_i[32], m_diff[32];
    for (int64_t i = 0; i < Tr; i++) {
      const int64_t br_upper = (L - i * Br) < Br ? (L - i * Br) : Br;
      for (int64_t x = 0; x < Br * E; x++) q_i[x] = 0.0f;
      for (int64_t a = 0; a < br_upper; a++)
        for (int64_t b = 0; b < E; b++) q_i[a * E + b] = q_b[(i * Br + a) * E + b];
      for (int64_t x = 0; x < Br * E; x++) o_i[x] = 0.0f;
      for (int64_t a = 0; a < Br; a++) {
        l_i[a] = 0.0f;
        m_i[a] = -INFINITY;
      }
      const int64_t causal_offset = S - L;
      for (int64_t j = 0; j < Tc; j++) {
        const int64_t row_max = i * Br + br_upper - 1;
        const int64_t col_min = j * Bc;
        if (is_causal && col_min > row_max + causal_offset) continue;
        const int64_t bc_upper = (S - j * Bc) < Bc ? (S - j * Bc) : Bc;
        for (int64_t x = 0; x < Bc * E; x++) {
          k_j[x] = 0.0f;
          v_j[x] = 0.0f;
        }
        for (int64_t a = 0; a < bc_upper; a++)
          for (int64_t b = 0; b < E; b++) {
            k_j[a * E + b] = k_b[(j * Bc + a) * E + b];
            v_j[a * E + b] = v_b[(j * Bc + a) * E + b];
          }
        for (int64_t x = 0; x < Br * Bc; x++) s_i[x] = 0.0f;
        for (int64_t a = 0; a < br_upper; a++)
          for (int64_t b = 0; b < bc_upper; b++)
            for (int64_t c = 0; c < E; c++) s_i[a * Bc + b] += q_i[a * E + c] * k_j[b * E + c];
        const int64_t row_min = i * Br;
        const int64_t col_max = j * Bc + bc_upper - 1;
        const int block_all_valid = is_causal && (col_max <= row_min + causal_offset);
        for (int64_t a = 0; a < br_upper; a++)
          for (int64_t b = 0; b < bc_upper; b++) {
            s_i[a * Bc + b] *= scale;
            if (!block_all_valid) {
              if (mask != NULL) {
                const int64_t off = n * ms_n + (i * Br + a) * ms_l + (j * Bc + b) * ms_s;
                s_i[a * Bc + b] += mask[off];
              } else if (is_causal && (j * Bc + b) > (i * Br + a) + causal_offset) {
                /* the wrapper's materialised causal_mask (attention.py:59-61,119-125) */
                s_i[a * Bc + b] += -INFINITY;
              }
            }
          }
        for (int64_t a = 0; a < br_upper; a++) {
          float rowmax = -INFINITY;
          for (int64_t b = 0; b < bc_upper; b++)
            if (s_i[a * Bc + b] > rowmax) rowmax = s_i[a * Bc + b];
          const float mx = m_i[a] > rowmax ? m_i[a] : rowmax;
          m_diff[a] = m_i[a] - mx;
          m_i[a] = mx;
        }
        for (int64_t a = 0; a < br_upper; a++)
          for (int64_t b = 0; b < bc_upper; b++) p[a * Bc + b] = expf(s_i[a * Bc + b] - m_i[a]);
        for (int64_t a = 0; a < br_upper; a++) {
          float rowsum = 0.0f;
          for (int64_t b = 0; b < bc_upper; b++) rowsum += p[a * Bc + b];
          l_i[a] = expf(m_diff[a]) * l_i[a] + rowsum;
        }
        for (int64_t a = 0; a < br_upper; a++)
          for (int64_t c = 0; c < E; c++) {
            float res = 0.0f;
            for (int64_t b = 0; b < bc_upper; b++) res += p[a * Bc + b] * v_j[b * E + c];
            o_i[a * E + c] = expf(m_diff[a]) * o_i[a * E + c] + res;
          }
      }
      for (int64_t a = 0; a < br_upper; a++)
        for (int64_t b = 0; b < E; b++) out[n * L * E + (i * Br + a) * E + b] = o_i[a * E + b] / l_i[a];
    }
    free(q_i);
    free(o_i);
    free(k_j);
    free(v_j);
  }
}

/*
 * TinyKvPagedPool._quantize_page_slice -- src/nano_vllm_metal/cache/paged.py:152-158.
 * x [rows, D] of in_dtype (F32/F16/BF16).  Per row: amax = max|x| in fp32,
 * s = amax > 0 ? amax / 127 : 1 (fp32), q = clip(round(x / s), -127, 127) with
 * round-half-to-even (numpy/MLX `round`), stored scale = s cast to in_dtype (RNE).
 * scale_out receives raw bits of in_dtype (4 bytes for F32, 2 for F16/BF16).
 */
void oracle_quantize_int8(const void* x, int in_dtype, int64_t rows, int64_t D, int8_t* q_out,
                          void* scale_out) {
  for (int64_t r = 0; r < rows; r++) {
    float amax = 0.0f;
    for (int64_t d = 0; d < D; d++) {
      const float a = fabsf(load_elem(x, r * D + d, in_dtype));
      if (a > amax) amax = a;
    }
    const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
    for (int64_t d = 0; d < D; d++) {
      float y = rintf(load_elem(x, r * D + d, in_dtype) / s);
      if (y < -127.0f) y = -127.0f;
      if (y > 127.0f) y = 127.0f;
      q_out[r * D + d] = (int8_t)y;
    }
    if (in_dtype == OR_F32)
      ((float*)scale_out)[r] = s;
    else if (in_dtype == OR_F16)
      ((uint16_t*)scale_out)[r] = f32_to_f16(s);
    else
      ((uint16_t*)scale_out)[r] = f32_to_bf16(s);
  }
}
