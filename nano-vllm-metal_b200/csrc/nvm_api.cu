// nvm_api.cu -- the extern "C" entry points of libnvm_attn.so (include/nvm_attn.h):
// argument validation (messages keep the reference operators' prefixes, e.g.
// paged_attention.cpp:22-63 and flash_attention.cpp:20-56), kernel selection, the
// per-device error word and tensor-map encoding.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "nvm_internal.h"

__device__ int g_nvm_error_word;

namespace nvm {

namespace {
thread_local std::string t_last_error;
std::mutex g_mu;
int* g_err_ptr[64] = {nullptr};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

bool env_flag(const char* name) {
  const char* v = std::getenv(name);
  return v != nullptr && v[0] != '\0' && v[0] != '0';
}
}  // namespace

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return status;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return NVM_OK;
  return fail(NVM_ERR_CUDA, "%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
}

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_err_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_nvm_error_word) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

size_t dtype_size(int dtype) {
  switch (dtype) {
    case NVM_F32: case NVM_I32: return 4;
    case NVM_F16: case NVM_BF16: return 2;
    case NVM_I8: return 1;
    case NVM_I64: return 8;
    default: return 0;
  }
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
        return fail(NVM_ERR_CUDA, "nvm: cuTensorMapEncodeTiled entry point unavailable");
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  cuuint64_t gdim[5], gstride[4];
  cuuint32_t bdim[5], estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i + 1 < rank) gstride[i] = strides_bytes[i];
  }
  CUresult r = g_encode(map, dt, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstride, bdim, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NVM_ERR_CUDA, "nvm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NVM_OK;
}

}  // namespace nvm

using namespace nvm;

namespace {

bool is_float_dtype(int d) { return d == NVM_F32 || d == NVM_F16 || d == NVM_BF16; }

// Shared validation of nvm_paged_attention / nvm_paged_attention_workspace_size.
int validate_paged(const PagedArgs& a, bool check_ptrs) {
  const char* op = a.kv_dtype == NVM_I8 ? "paged_attention_int8_decode" : "paged_attention";
  if (!is_float_dtype(a.q_dtype)) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: q must be float32, float16 or bfloat16", op);
  if (!is_float_dtype(a.kv_dtype) && a.kv_dtype != NVM_I8)
    return fail(NVM_ERR_INVALID_ARGUMENT,
                "paged_attention: key_pages and value_pages must be float32, float16, bfloat16 or int8");
  if (!is_float_dtype(a.out_dtype)) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: output dtype must be floating point", op);
  if (a.B < 0 || a.Hq <= 0 || a.Hkv <= 0 || a.L <= 0 || a.D <= 0 || a.P < 0 || a.page_size <= 0 ||
      a.max_pages < 0)
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: sizes must be positive (B=%lld Hq=%lld Hkv=%lld L=%lld D=%lld)", op,
                (long long)a.B, (long long)a.Hq, (long long)a.Hkv, (long long)a.L, (long long)a.D);
  if (a.Hq % a.Hkv != 0) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: num_heads must be divisible by num_kv_heads", op);
  if (a.D > 256) return fail(NVM_ERR_UNSUPPORTED, "%s: head dimension must be <= 256 (got %lld)", op, (long long)a.D);
  if (a.kv_dtype == NVM_I8) {
    if (!is_float_dtype(a.scale_dtype))
      return fail(NVM_ERR_INVALID_ARGUMENT, "%s: key_scales and value_scales must be floating point", op);
    if (check_ptrs && (a.k_scales == nullptr || a.v_scales == nullptr))
      return fail(NVM_ERR_INVALID_ARGUMENT, "%s: int8 pages need key_scales and value_scales", op);
  }
  if (check_ptrs && a.B > 0) {
    if (a.q == nullptr || a.out == nullptr || a.context_lens == nullptr || a.block_table == nullptr)
      return fail(NVM_ERR_INVALID_ARGUMENT, "%s: null tensor pointer", op);
    if (a.max_pages > 0 && a.P > 0 && (a.k_pages == nullptr || a.v_pages == nullptr))
      return fail(NVM_ERR_INVALID_ARGUMENT, "%s: null page pointer", op);
  }
  if (a.B * a.Hq * a.L > (int64_t)INT32_MAX * 4)
    return fail(NVM_ERR_UNSUPPORTED, "%s: too many query rows", op);
  return NVM_OK;
}

}  // namespace

extern "C" {

const char* nvm_status_string(int status) {
  switch (status) {
    case NVM_OK: return "NVM_OK";
    case NVM_ERR_INVALID_ARGUMENT: return "NVM_ERR_INVALID_ARGUMENT";
    case NVM_ERR_UNSUPPORTED: return "NVM_ERR_UNSUPPORTED";
    case NVM_ERR_WORKSPACE: return "NVM_ERR_WORKSPACE";
    case NVM_ERR_CUDA: return "NVM_ERR_CUDA";
    case NVM_ERR_DEVICE_TIMEOUT: return "NVM_ERR_DEVICE_TIMEOUT";
    case NVM_ERR_OUT_OF_PAGES: return "NVM_ERR_OUT_OF_PAGES";
    default: return "NVM_ERR_UNKNOWN";
  }
}

const char* nvm_last_error(void) { return t_last_error.c_str(); }

const char* nvm_version(void) { return "nvm_attn 0.1 sm_100a"; }

int nvm_device_error(void* stream, int clear) {
  int* w = device_error_word();
  if (w == nullptr) return fail(NVM_ERR_CUDA, "nvm_device_error: no device error word");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = check_cuda(cudaStreamSynchronize(s), "nvm_device_error");
  if (st != NVM_OK) return st;
  int v = 0;
  st = check_cuda(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost), "nvm_device_error");
  if (st != NVM_OK) return st;
  if (clear && v != 0) {
    st = check_cuda(cudaMemset(w, 0, sizeof(int)), "nvm_device_error");
    if (st != NVM_OK) return st;
  }
  return v;
}

size_t nvm_paged_attention_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t L, int64_t D,
                                          int64_t page_size, int64_t max_pages, int kv_dtype) {
  PagedArgs a{};
  a.q_dtype = NVM_F32;
  a.kv_dtype = kv_dtype;
  a.scale_dtype = NVM_F16;
  a.out_dtype = NVM_F32;
  a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.L = L; a.D = D; a.P = 1; a.page_size = page_size; a.max_pages = max_pages;
  a.is_causal = 1;
  if (validate_paged(a, false) != NVM_OK) return 0;
  if (env_flag("NVM_ATTN_FORCE_GENERIC")) return 0;
  // q's dtype is not known here: cover the tcgen05 plan (taken when q matches the pages)
  // and the mma.sync plan (taken otherwise).
  MmaPlan plan = plan_paged_mma(a);
  size_t need = plan.eligible ? plan.ws_bytes : 0;
  if (!env_flag("NVM_ATTN_NO_SM100")) {
    const Sm100Plan sp = plan_sm100(a, true);
    if (sp.eligible && sp.ws_bytes > need) need = sp.ws_bytes;
  }
  return need;
}

int nvm_paged_attention(const void* q, int q_dtype, const void* k_pages, const void* v_pages, int kv_dtype,
                        const void* k_scales, const void* v_scales, int scale_dtype,
                        const int32_t* block_table, const int32_t* context_lens, void* out, int out_dtype,
                        int64_t B, int64_t Hq, int64_t Hkv, int64_t L, int64_t D, int64_t P, int64_t page_size,
                        int64_t max_pages, float scale, int is_causal, void* workspace, size_t workspace_bytes,
                        void* stream) {
  PagedArgs a{};
  a.q = q; a.q_dtype = q_dtype; a.k_pages = k_pages; a.v_pages = v_pages; a.kv_dtype = kv_dtype;
  a.k_scales = k_scales; a.v_scales = v_scales; a.scale_dtype = scale_dtype;
  a.block_table = block_table; a.context_lens = context_lens; a.out = out; a.out_dtype = out_dtype;
  a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.L = L; a.D = D; a.P = P; a.page_size = page_size; a.max_pages = max_pages;
  a.scale = scale; a.is_causal = is_causal ? 1 : 0; a.dense_ctx = 0;
  int st = validate_paged(a, true);
  if (st != NVM_OK) return st;
  if (B == 0) return NVM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!env_flag("NVM_ATTN_FORCE_GENERIC")) {
    if (!env_flag("NVM_ATTN_NO_SM100") && flash2q_eligible(a)) return launch_flash2q(a, s);
    if (!env_flag("NVM_ATTN_NO_SM100")) {
      const Sm100Plan sp = plan_sm100(a, false);
      if (sp.eligible) {
        if (sp.ws_bytes > 0 && (workspace == nullptr || workspace_bytes < sp.ws_bytes))
          return fail(NVM_ERR_WORKSPACE, "paged_attention: workspace of %zu bytes required, %zu given", sp.ws_bytes,
                      workspace_bytes);
        return launch_sm100(a, sp, workspace, s);
      }
    }
    MmaPlan plan = plan_paged_mma(a);
    if (plan.eligible) {
      if (plan.ws_bytes > 0 && (workspace == nullptr || workspace_bytes < plan.ws_bytes))
        return fail(NVM_ERR_WORKSPACE, "paged_attention: workspace of %zu bytes required, %zu given", plan.ws_bytes,
                    workspace_bytes);
      return launch_paged_mma(a, plan, workspace, s);
    }
  }
  return launch_paged_generic(a, s);
}

int nvm_flash_attention(const void* q, const void* k, const void* v, int dtype, const float* mask,
                        int64_t mask_stride_n, int64_t mask_stride_l, int64_t mask_stride_s, void* out,
                        int out_dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t L, int64_t S, int64_t D,
                        float scale, int is_causal, void* stream) {
  if (!is_float_dtype(dtype)) return fail(NVM_ERR_INVALID_ARGUMENT, "flash_attention: all input arrays must be float32, float16 or bfloat16");
  if (!is_float_dtype(out_dtype)) return fail(NVM_ERR_INVALID_ARGUMENT, "flash_attention: output dtype must be floating point");
  if (B < 0 || Hq <= 0 || Hkv <= 0 || L <= 0 || S <= 0 || D <= 0)
    return fail(NVM_ERR_INVALID_ARGUMENT, "flash_attention: sizes must be positive");
  if (Hq % Hkv != 0) return fail(NVM_ERR_INVALID_ARGUMENT, "flash_attention: num_heads must be divisible by num_kv_heads");
  if (D > 256) return fail(NVM_ERR_UNSUPPORTED, "flash_attention: E must be <= 256 (got %lld)", (long long)D);
  if (B == 0) return NVM_OK;
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(NVM_ERR_INVALID_ARGUMENT, "flash_attention: null tensor pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (mask == nullptr && dtype != NVM_F32 && !env_flag("NVM_ATTN_FORCE_GENERIC")) {
    // Dense K/V [B*Hkv, S, D] viewed as a pool of B pages of size S (page id = b).
    PagedArgs a{};
    a.q = q; a.q_dtype = dtype; a.k_pages = k; a.v_pages = v; a.kv_dtype = dtype;
    a.block_table = nullptr; a.context_lens = nullptr; a.out = out; a.out_dtype = out_dtype;
    a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.L = L; a.D = D; a.P = B; a.page_size = S; a.max_pages = 1;
    a.scale = scale; a.is_causal = is_causal ? 1 : 0; a.dense = 1; a.dense_ctx = S;
    if (!env_flag("NVM_ATTN_NO_SM100")) {
      if (flash2q_eligible(a)) return launch_flash2q(a, s);
      const Sm100Plan sp = plan_sm100(a, false);
      if (sp.eligible && sp.ws_bytes == 0) return launch_sm100(a, sp, nullptr, s);
    }
    MmaPlan plan = plan_paged_mma(a);
    if (plan.eligible && plan.ws_bytes == 0) return launch_paged_mma(a, plan, nullptr, s);
  }
  FlashArgs f{};
  f.q = q; f.k = k; f.v = v; f.dtype = dtype; f.mask = mask;
  f.ms_n = mask_stride_n; f.ms_l = mask_stride_l; f.ms_s = mask_stride_s;
  f.out = out; f.out_dtype = out_dtype;
  f.B = B; f.Hq = Hq; f.Hkv = Hkv; f.L = L; f.S = S; f.D = D; f.scale = scale; f.is_causal = is_causal ? 1 : 0;
  return launch_flash_generic(f, s);
}

int nvm_reshape_and_cache(const void* k, const void* v, int in_dtype, int64_t stride_t, int64_t stride_h,
                          void* k_pages, void* v_pages, int kv_dtype, void* k_scales, void* v_scales,
                          int scale_dtype, const int64_t* slot_mapping, int64_t T, int64_t Hkv, int64_t D,
                          int64_t P, int64_t page_size, void* stream) {
  if (!is_float_dtype(in_dtype)) return fail(NVM_ERR_INVALID_ARGUMENT, "write_page_slice: key/value must be floating point");
  if (kv_dtype != in_dtype && kv_dtype != NVM_I8)
    return fail(NVM_ERR_INVALID_ARGUMENT, "write_page_slice: page dtype must equal the input dtype or be int8");
  if (kv_dtype == NVM_I8 && (k_scales == nullptr || v_scales == nullptr || !is_float_dtype(scale_dtype)))
    return fail(NVM_ERR_INVALID_ARGUMENT, "write_page_slice: int8 pages need floating-point key/value scales");
  if (T < 0 || Hkv <= 0 || D <= 0 || P < 0 || page_size <= 0)
    return fail(NVM_ERR_INVALID_ARGUMENT, "write_page_slice: sizes must be positive");
  if (T == 0) return NVM_OK;
  if (k == nullptr || v == nullptr || k_pages == nullptr || v_pages == nullptr || slot_mapping == nullptr)
    return fail(NVM_ERR_INVALID_ARGUMENT, "write_page_slice: null tensor pointer");
  return launch_kv_write(k, v, in_dtype, stride_t, stride_h, k_pages, v_pages, kv_dtype, k_scales, v_scales,
                         scale_dtype, slot_mapping, T, Hkv, D, P, page_size, static_cast<cudaStream_t>(stream));
}

int nvm_paged_append(int32_t* block_table, int32_t* context_lens, const int32_t* new_tokens, int32_t* free_stack,
                     int32_t* free_top, int32_t* num_pages, int32_t* page_refcount, int64_t* slot_mapping,
                     int64_t slot_capacity, int32_t* status, int64_t B, int64_t max_pages, int64_t page_size,
                     int64_t capacity, void* stream) {
  if (B < 0 || B > 4096 || max_pages < 0 || page_size <= 0 || capacity < 0 || slot_capacity < 0)
    return fail(NVM_ERR_INVALID_ARGUMENT, "allocate_page: invalid sizes (B must be in [0, 4096])");
  if (B == 0) return NVM_OK;
  if (!block_table || !context_lens || !new_tokens || !free_stack || !free_top || !num_pages || !page_refcount ||
      !slot_mapping || !status)
    return fail(NVM_ERR_INVALID_ARGUMENT, "allocate_page: null tensor pointer");
  return launch_paged_append(block_table, context_lens, new_tokens, free_stack, free_top, num_pages, page_refcount,
                             slot_mapping, slot_capacity, status, B, max_pages, page_size, capacity,
                             static_cast<cudaStream_t>(stream));
}

int nvm_paged_rewind(int32_t* block_table, int32_t* context_lens, const int32_t* rewind, int32_t* free_stack,
                     int32_t* free_top, int32_t* page_refcount, int32_t* last_call, int32_t* status, int64_t B,
                     int64_t max_pages, int64_t page_size, int64_t capacity, void* stream) {
  if (B < 0 || B > 4096 || max_pages < 0 || page_size <= 0 || capacity < 0)
    return fail(NVM_ERR_INVALID_ARGUMENT, "rewind: invalid sizes (B must be in [0, 4096])");
  if (B == 0) return NVM_OK;
  if (!block_table || !context_lens || !rewind || !free_stack || !free_top || !page_refcount || !last_call || !status)
    return fail(NVM_ERR_INVALID_ARGUMENT, "rewind: null tensor pointer");
  return launch_paged_rewind(block_table, context_lens, rewind, free_stack, free_top, page_refcount, last_call, status,
                             B, max_pages, page_size, capacity, static_cast<cudaStream_t>(stream));
}

int nvm_paged_attach(int32_t* block_table, int32_t* context_lens, const int32_t* pages, const int32_t* count,
                     int32_t* page_refcount, int32_t* status, int64_t B, int64_t max_pages, int64_t page_size,
                     int64_t max_prefix, int64_t capacity, void* stream) {
  if (B < 0 || B > 4096 || max_pages < 0 || page_size <= 0 || max_prefix < 0 || capacity < 0)
    return fail(NVM_ERR_INVALID_ARGUMENT, "attach: invalid sizes (B must be in [0, 4096])");
  if (B == 0) return NVM_OK;
  if (!block_table || !context_lens || !count || !page_refcount || !status || (max_prefix > 0 && !pages))
    return fail(NVM_ERR_INVALID_ARGUMENT, "attach: null tensor pointer");
  return launch_paged_attach(block_table, context_lens, pages, count, page_refcount, status, B, max_pages, page_size,
                             max_prefix, capacity, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
