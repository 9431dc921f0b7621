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

/* raw store of one element of dtype (F32 / F16 bits / BF16 bits), RNE */
static inline void store_elem(void* base, int64_t idx, int dtype, float f) {
  if (dtype == OR_F32)
    ((float*)base)[idx] = f;
  else if (dtype == OR_F16)
    ((uint16_t*)base)[idx] = f32_to_f16(f);
  else
    ((uint16_t*)base)[idx] = f32_to_bf16(f);
}

/* value after a round trip through dtype (identity for F32) */
static inline float round_to(float f, int dtype) {
  if (dtype == OR_F16) return f16_to_f32(f32_to_f16(f));
  if (dtype == OR_BF16) return bf16_to_f32(f32_to_bf16(f));
  return f;
}

/* One row of _quantize_page_slice (paged.py:152-158): amax in fp32, s = amax / 127
 * (1 when amax == 0), q = clip(round_half_even(x / s), -127, 127); scale stored in
 * scale_dtype at index sidx. */
static void quantize_row(const float* x, int64_t D, int8_t* q_out, void* scale_out, int64_t sidx,
                         int scale_dtype) {
  float amax = 0.0f;
  for (int64_t d = 0; d < D; d++) {
    const float a = fabsf(x[d]);
    if (a > amax) amax = a;
  }
  const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
  for (int64_t d = 0; d < D; d++) {
    float y = rintf(x[d] / s);
    if (y < -127.0f) y = -127.0f;
    if (y > 127.0f) y = 127.0f;
    q_out[d] = (int8_t)y;
  }
  store_elem(scale_out, sidx, scale_dtype, s);
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
  float* row = (float*)malloc((size_t)D * sizeof(float));
  for (int64_t r = 0; r < rows; r++) {
    for (int64_t d = 0; d < D; d++) row[d] = load_elem(x, r * D + d, in_dtype);
    quantize_row(row, D, q_out + r * D, scale_out, r, in_dtype);
  }
  free(row);
}

/* sum of x[i]^2 in the order of a 32-lane tree: lane l holds EH = D/64 elements of each
 * half of the row (x[l*EH .. l*EH+EH-1] and x[D/2 + l*EH ..]) and sums their squares in
 * that order, then five butterfly steps (offsets 16, 8, 4, 2, 1) add the partner lane's
 * partial.  Every order is a valid evaluation of mean(x^2); this one is the order of the
 * product kernel, so the oracle agrees with it bit for bit.  D not a multiple of 64 sums
 * sequentially. */
static float sum_squares(const float* x, int64_t D) {
  if (D % 64 != 0) {
    float ss = 0.0f;
    for (int64_t d = 0; d < D; d++) ss = ss + x[d] * x[d];
    return ss;
  }
  const int64_t EH = D / 64, half = D / 2;
  float part[32];
  for (int l = 0; l < 32; l++) {
    float ss = 0.0f;
    for (int64_t e = 0; e < EH; e++) ss = ss + x[l * EH + e] * x[l * EH + e];
    for (int64_t e = 0; e < EH; e++) ss = ss + x[half + l * EH + e] * x[half + l * EH + e];
    part[l] = ss;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float nxt[32];
    for (int l = 0; l < 32; l++) nxt[l] = part[l] + part[l ^ off];
    memcpy(part, nxt, sizeof(part));
  }
  return part[0];
}

/*
 * The per-layer step between the QKV projection and attention in
 * Qwen3Attention.__call__ -- src/nano_vllm_metal/models/qwen3.py:100-116:
 *   1. q_norm / k_norm (layers/layernorm.py:4-14, mx.fast.rms_norm): per head row,
 *      x * (1 / sqrt(mean(x^2) + eps)) * weight in fp32, result rounded to dtype.
 *      wq == NULL skips the norm (RoPE alone, as the reference's RoPE tests run it).
 *   2. RoPE (layers/rotary_embedding.py:74-124, custom backend): cos/sin rows of the
 *      fp32 tables at the token's position; halves (x1 = x[:D/2], x2 = x[D/2:]) or,
 *      when traditional, interleaved pairs (x[2i], x[2i+1]); real = x1*c - x2*s,
 *      imag = x1*s + x2*c with every product and sum rounded to fp32 (dtype inputs
 *      promote to fp32), result rounded to dtype.
 *   3. cache.update_and_fetch_paged (cache/kv_cache.py:113-173 -> cache/paged.py:
 *      160-195): rotated K and raw V written at slot = page_id * page_size + offset
 *      of pools [P, Hkv, page_size, D]; int8 pools through _quantize_page_slice.
 * q, k, v [T, H, D] of dtype; q_out [T, Hq, D] of dtype.  Slots < 0 are skipped.
 * Returns 0, or 1 for a position outside the table / a page id >= P (that row is
 * skipped, as the product kernel does).
 */
int oracle_qk_norm_rope_write(const void* q, const void* k, const void* v, int dtype, const void* wq,
                              const void* wk, float eps, const float* cos_t, const float* sin_t,
                              int64_t table_rows, int traditional, const int32_t* pos, void* q_out,
                              void* k_pages, void* v_pages, int kv_dtype, void* k_scales, void* v_scales,
                              int scale_dtype, const int64_t* slots, int64_t T, int64_t Hq, int64_t Hkv,
                              int64_t D, int64_t P, int64_t page_size) {
  const int64_t half = D / 2;
  int err = 0;
  float* x = (float*)malloc((size_t)D * sizeof(float));
  float* y = (float*)malloc((size_t)D * sizeof(float));
  for (int64_t t = 0; t < T; t++) {
    for (int64_t r = 0; r < Hq + 2 * Hkv; r++) {
      const int is_q = r < Hq, is_k = !is_q && r < Hq + Hkv;
      const int64_t h = is_q ? r : (is_k ? r - Hq : r - Hq - Hkv);
      const void* src = is_q ? q : (is_k ? k : v);
      const int64_t base = (t * (is_q ? Hq : Hkv) + h) * D;
      for (int64_t d = 0; d < D; d++) x[d] = load_elem(src, base + d, dtype);
      if (is_q || is_k) {
        const void* w = is_q ? wq : wk;
        if (w != NULL) {
          const float inv = 1.0f / sqrtf(sum_squares(x, D) / (float)D + eps);
          for (int64_t d = 0; d < D; d++) x[d] = round_to(x[d] * inv * load_elem(w, d, dtype), dtype);
        }
        if (pos[t] < 0 || pos[t] >= table_rows) {
          err = 1;
          continue;
        }
        const float* c = cos_t + (int64_t)pos[t] * half;
        const float* s = sin_t + (int64_t)pos[t] * half;
        for (int64_t i = 0; i < half; i++) {
          const float x1 = traditional ? x[2 * i] : x[i];
          const float x2 = traditional ? x[2 * i + 1] : x[i + half];
          const float re = x1 * c[i] - x2 * s[i];
          const float im = x1 * s[i] + x2 * c[i];
          y[traditional ? 2 * i : i] = re;
          y[traditional ? 2 * i + 1 : i + half] = im;
        }
        for (int64_t d = 0; d < D; d++) x[d] = round_to(y[d], dtype);
      }
      if (is_q) {
        for (int64_t d = 0; d < D; d++) store_elem(q_out, (t * Hq + h) * D + d, dtype, x[d]);
        continue;
      }
      if (slots[t] < 0) continue;
      const int64_t pid = slots[t] / page_size, off = slots[t] % page_size;
      if (pid >= P) {
        err = 1;
        continue;
      }
      const int64_t prow = (pid * Hkv + h) * page_size + off;
      void* pool = is_k ? k_pages : v_pages;
      if (kv_dtype == OR_I8)
        quantize_row(x, D, (int8_t*)pool + prow * D, is_k ? k_scales : v_scales, prow, scale_dtype);
      else
        for (int64_t d = 0; d < D; d++) store_elem(pool, prow * D + d, kv_dtype, x[d]);
    }
  }
  free(x);
  free(y);
  return err;
}

/*
 * QuantizedMatmul::eval_cpu -- src/nano_vllm_metal/metal/src/quantized_matmul.cpp:80-148.
 * a [M, N] and out [M, K] of dtype (F16 / BF16), b [K, N / 8] uint32 (element n of a
 * word: bits 4 (n % 8) .. +3), scales / biases [K, N / 128] of dtype.  For every (i, k):
 * sum over groups in order, inside a group over the words in order and the 8 nibbles of
 * a word in order: w = nibble * scale + bias (fp32), sum += a * w (fp32); out rounded.
 */
void oracle_quantized_matmul(const void* a, int dtype, const uint32_t* b, const void* scales, const void* biases,
                             void* out, int64_t M, int64_t N, int64_t K, int nthreads) {
  const int64_t groups = N / 128;
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < M; i++) {
    for (int64_t k = 0; k < K; k++) {
      float sum = 0.0f;
      for (int64_t gi = 0; gi < groups; gi++) {
        const float scale = load_elem(scales, k * groups + gi, dtype);
        const float bias = load_elem(biases, k * groups + gi, dtype);
        for (int64_t wd = 0; wd < 16; wd++) {
          const uint32_t word = b[(k * N + gi * 128) / 8 + wd];
          for (int j = 0; j < 8; j++) {
            const float q = (float)((word >> (4 * j)) & 15u);
            const float w = q * scale + bias;
            const float av = load_elem(a, i * N + gi * 128 + wd * 8 + j, dtype);
            sum = sum + av * w;
          }
        }
      }
      store_elem(out, i * K + k, dtype, sum);
    }
  }
}

