// attn_generic.cu -- CUDA-core kernels that serve every shape the tensor-core
// kernels do not: any head dim <= 256, any page size, F32 pages (exact fp32 math,
// matching the reference's fp32 tolerance), masks with arbitrary strides.
//
// Paged kernel semantics follow PagedAttention (paged_attention.cpp:148-287 and the
// Metal kernels paged_attention.metal:6-128,134-238,417-525): key positions beyond
// min(ctx, max_pages*page_size), holes (page id < 0 or >= P) and, with causal, keys
// after row + ctx - L are skipped; a row that sees nothing is written as zeros.
// Flash kernel semantics follow FlashAttention (flash_attention.cpp:94-248): Bc=32
// key tiles, causal tile skip above the diagonal, additive mask only on tiles that
// are not entirely visible, no guard on the final division.
//
// One warp per query row: lane j scores key j of a 32-key chunk, the chunk's
// probabilities are broadcast by shuffle and every lane accumulates its slice of D.
#include "nvm_common.cuh"
#include "nvm_internal.h"

namespace nvm {
namespace {

constexpr int kWarps = 4;

struct GenericPagedParams {
  const void* q;
  const void* k;
  const void* v;
  const void* ks;
  const void* vs;
  const int32_t* block_table;
  const int32_t* context_lens;
  void* out;
  int q_dtype, kv_dtype, scale_dtype, out_dtype;
  int64_t B, Hq, Hkv, L, D, P, ps, mp, dense_ctx;
  float scale;
  int causal;
};

template <int DPL>
__global__ void __launch_bounds__(kWarps * 32) paged_generic_kernel(GenericPagedParams p) {
  __shared__ float qs[kWarps][32 * DPL];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + warp;
  if (row >= p.B * p.Hq * p.L) return;
  const int64_t n = row / p.L, l = row % p.L;
  const int64_t b = n / p.Hq, qh = n % p.Hq;
  const int64_t kvh = qh / (p.Hq / p.Hkv);
  const int64_t ctx = p.context_lens ? (int64_t)p.context_lens[b] : p.dense_ctx;
  const int64_t base_out = row * p.D;
  if (ctx <= 0) {
    for (int64_t d = lane; d < p.D; d += 32) store_dyn(p.out, base_out + d, p.out_dtype, 0.0f);
    return;
  }
  const int64_t cap = p.mp * p.ps;
  const int64_t ctx_limit = ctx < cap ? ctx : cap;
  int64_t n_keys = ctx_limit;
  if (p.causal) {
    const int64_t lim = l + ctx - p.L + 1;  // keys [0, lim) are visible
    if (lim < n_keys) n_keys = lim;
  }
  for (int64_t d = lane; d < 32 * DPL; d += 32) qs[warp][d] = d < p.D ? load_dyn(p.q, row * p.D + d, p.q_dtype) : 0.0f;
  __syncwarp();

  const bool is_i8 = p.kv_dtype == NVM_I8;
  float m = -INFINITY, lsum = 0.0f;
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.0f;

  for (int64_t j0 = 0; j0 < n_keys; j0 += 32) {
    const int64_t pos = j0 + lane;
    int64_t base = -1;  // element offset / D of this key's row inside the pool
    if (pos < n_keys) {
      const int64_t page_idx = pos / p.ps;
      const int64_t pid = p.block_table ? (int64_t)p.block_table[b * p.mp + page_idx] : b;
      if (pid >= 0 && pid < p.P) base = (pid * p.Hkv + kvh) * p.ps + (pos - page_idx * p.ps);
    }
    float s = -INFINITY;
    if (base >= 0) {
      float dot = 0.0f;
      for (int64_t d = 0; d < p.D; ++d) dot += qs[warp][d] * load_dyn(p.k, base * p.D + d, p.kv_dtype);
      if (is_i8) dot *= load_dyn(p.ks, base, p.scale_dtype);
      s = dot * p.scale;
    }
    const float mx = warp_max(s);
    const float m_new = fmaxf(m, mx);
    if (m_new == -INFINITY) continue;
    const float alpha = expf(m - m_new);
    const float pj = base >= 0 ? expf(s - m_new) : 0.0f;
    lsum = lsum * alpha + warp_sum(pj);
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] *= alpha;
    for (int jj = 0; jj < 32; ++jj) {
      const int64_t bj = __shfl_sync(0xffffffffu, base, jj);
      const float pjj = __shfl_sync(0xffffffffu, pj, jj);
      if (bj < 0) continue;
      const float sv = is_i8 ? load_dyn(p.vs, bj, p.scale_dtype) : 1.0f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int64_t d = lane + 32 * i;
        if (d < p.D) acc[i] += pjj * (load_dyn(p.v, bj * p.D + d, p.kv_dtype) * sv);
      }
    }
    m = m_new;
  }
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int64_t d = lane + 32 * i;
    if (d < p.D) store_dyn(p.out, base_out + d, p.out_dtype, lsum > 0.0f ? acc[i] / lsum : 0.0f);
  }
}

struct GenericFlashParams {
  const void* q;
  const void* k;
  const void* v;
  const float* mask;
  int64_t ms_n, ms_l, ms_s;
  void* out;
  int dtype, out_dtype;
  int64_t B, Hq, Hkv, L, S, D;
  float scale;
  int causal;
};

template <int DPL>
__global__ void __launch_bounds__(kWarps * 32) flash_generic_kernel(GenericFlashParams p) {
  __shared__ float qs[kWarps][32 * DPL];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + warp;
  if (row >= p.B * p.Hq * p.L) return;
  const int64_t n = row / p.L, l = row % p.L;
  const int64_t kv_row0 = (n / (p.Hq / p.Hkv)) * p.S;
  for (int64_t d = lane; d < 32 * DPL; d += 32) qs[warp][d] = d < p.D ? load_dyn(p.q, row * p.D + d, p.dtype) : 0.0f;
  __syncwarp();
  const int64_t off = p.S - p.L;  // causal offset
  const int64_t i_tile = l / 32;
  const int64_t row_max_tile = (i_tile * 32 + 31) < (p.L - 1) ? (i_tile * 32 + 31) : (p.L - 1);

  float m = -INFINITY, lsum = 0.0f;
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.0f;

  for (int64_t j0 = 0; j0 < p.S; j0 += 32) {
    if (p.causal && j0 > row_max_tile + off) break;  // this and every later tile is fully masked
    const int64_t pos = j0 + lane;
    const bool in_range = pos < p.S;
    float s = -INFINITY;
    if (in_range) {
      float dot = 0.0f;
      for (int64_t d = 0; d < p.D; ++d) dot += qs[warp][d] * load_dyn(p.k, (kv_row0 + pos) * p.D + d, p.dtype);
      s = dot * p.scale;
      const int64_t col_max = (j0 + 31) < (p.S - 1) ? (j0 + 31) : (p.S - 1);
      const bool all_valid = p.causal && (col_max <= i_tile * 32 + off);
      if (!all_valid) {
        if (p.mask != nullptr)
          s += p.mask[n * p.ms_n + l * p.ms_l + pos * p.ms_s];
        else if (p.causal && pos > l + off)
          s = -INFINITY;
      }
    }
    const float mx = warp_max(s);
    const float m_new = fmaxf(m, mx);
    const float alpha = expf(m - m_new);
    const float pj = in_range ? expf(s - m_new) : 0.0f;
    lsum = alpha * lsum + warp_sum(pj);
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] *= alpha;
    for (int jj = 0; jj < 32; ++jj) {
      if (j0 + jj >= p.S) break;
      const float pjj = __shfl_sync(0xffffffffu, pj, jj);
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int64_t d = lane + 32 * i;
        if (d < p.D) acc[i] += pjj * load_dyn(p.v, (kv_row0 + j0 + jj) * p.D + d, p.dtype);
      }
    }
    m = m_new;
  }
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int64_t d = lane + 32 * i;
    if (d < p.D) store_dyn(p.out, row * p.D + d, p.out_dtype, acc[i] / lsum);
  }
}

}  // namespace

int launch_paged_generic(const PagedArgs& a, cudaStream_t s) {
  GenericPagedParams p{};
  p.q = a.q; p.k = a.k_pages; p.v = a.v_pages; p.ks = a.k_scales; p.vs = a.v_scales;
  p.block_table = a.block_table; p.context_lens = a.context_lens; p.out = a.out;
  p.q_dtype = a.q_dtype; p.kv_dtype = a.kv_dtype; p.scale_dtype = a.scale_dtype; p.out_dtype = a.out_dtype;
  p.B = a.B; p.Hq = a.Hq; p.Hkv = a.Hkv; p.L = a.L; p.D = a.D; p.P = a.P; p.ps = a.page_size; p.mp = a.max_pages;
  p.dense_ctx = a.dense_ctx; p.scale = a.scale; p.causal = a.is_causal;
  const int64_t rows = a.B * a.Hq * a.L;
  const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps));
  const int dpl = (int)((a.D + 31) / 32);
  if (dpl <= 1) paged_generic_kernel<1><<<grid, kWarps * 32, 0, s>>>(p);
  else if (dpl <= 2) paged_generic_kernel<2><<<grid, kWarps * 32, 0, s>>>(p);
  else if (dpl <= 4) paged_generic_kernel<4><<<grid, kWarps * 32, 0, s>>>(p);
  else paged_generic_kernel<8><<<grid, kWarps * 32, 0, s>>>(p);
  return check_cuda(cudaGetLastError(), "paged_attention: generic kernel launch");
}

int launch_flash_generic(const FlashArgs& a, cudaStream_t s) {
  GenericFlashParams p{};
  p.q = a.q; p.k = a.k; p.v = a.v; p.mask = a.mask; p.ms_n = a.ms_n; p.ms_l = a.ms_l; p.ms_s = a.ms_s;
  p.out = a.out; p.dtype = a.dtype; p.out_dtype = a.out_dtype;
  p.B = a.B; p.Hq = a.Hq; p.Hkv = a.Hkv; p.L = a.L; p.S = a.S; p.D = a.D; p.scale = a.scale; p.causal = a.is_causal;
  const int64_t rows = a.B * a.Hq * a.L;
  const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps));
  const int dpl = (int)((a.D + 31) / 32);
  if (dpl <= 1) flash_generic_kernel<1><<<grid, kWarps * 32, 0, s>>>(p);
  else if (dpl <= 2) flash_generic_kernel<2><<<grid, kWarps * 32, 0, s>>>(p);
  else if (dpl <= 4) flash_generic_kernel<4><<<grid, kWarps * 32, 0, s>>>(p);
  else flash_generic_kernel<8><<<grid, kWarps * 32, 0, s>>>(p);
  return check_cuda(cudaGetLastError(), "flash_attention: generic kernel launch");
}

}  // namespace nvm
