// kv_write.cu -- paged KV scatter-write (reshape_and_cache) for one batch of tokens.
//
// Replaces the per-page MLX slice-assign of TinyKvPagedPool.write_page_slice
// (src/nano_vllm_metal/cache/paged.py:160-195) and the int8 quantiser
// _quantize_page_slice (paged.py:152-158).  One warp handles one (token, kv head)
// row of K and the same row of V; the destination is the contiguous D-element row
// at ((page_id * Hkv + h) * page_size + offset) * D.  Copies are bit-exact; the
// int8 path reproduces the reference's fp32 arithmetic exactly (IEEE division,
// round-half-to-even, clip to [-127, 127], scale stored rounded to the scale dtype).
#include "nvm_common.cuh"
#include "nvm_internal.h"

namespace nvm {
namespace {

constexpr int kWarps = 8;

struct KvWriteParams {
  const void* k;
  const void* v;
  void* kp;
  void* vp;
  void* ks;
  void* vs;
  const int64_t* slots;
  int64_t st, sh, T, Hkv, D, P, ps;
  int in_dtype, kv_dtype, scale_dtype;
  int vec16;  // 1 if rows can be moved with 16-byte vectors
};

__device__ __forceinline__ void copy_row(const char* src, char* dst, int64_t bytes, bool vec16, int lane) {
  if (vec16) {
    const int64_t n = bytes >> 4;
    for (int64_t i = lane; i < n; i += 32)
      reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
  } else {
    for (int64_t i = lane; i < bytes; i += 32) dst[i] = src[i];
  }
}

__device__ __forceinline__ void quantize_row(const void* src, int64_t src_off, int in_dtype, int8_t* dst, int64_t D,
                                             void* scales, int64_t scale_idx, int scale_dtype, int lane) {
  float amax = 0.0f;
  for (int64_t d = lane; d < D; d += 32) amax = fmaxf(amax, fabsf(load_dyn(src, src_off + d, in_dtype)));
  amax = warp_max(amax);
  const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  const float r = __frcp_rn(s);
  for (int64_t d = lane; d < D; d += 32) dst[d] = (int8_t)quantize_i8(load_dyn(src, src_off + d, in_dtype), s, r);
  if (lane == 0) store_dyn(scales, scale_idx, scale_dtype, s);
}

__global__ void __launch_bounds__(kWarps * 32) kv_write_kernel(KvWriteParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * kWarps + warp;
  if (w >= p.T * p.Hkv) return;
  // 32-bit divisions where the values fit (a 64-bit division costs about as much as
  // copying the row)
  int64_t t, h;
  if (w <= 0x7fffffffLL && p.Hkv <= 0x7fffffffLL) {
    const uint32_t tu = (uint32_t)w / (uint32_t)p.Hkv;
    t = tu;
    h = (uint32_t)w - tu * (uint32_t)p.Hkv;
  } else {
    t = w / p.Hkv;
    h = w - t * p.Hkv;
  }
  const int64_t slot = p.slots[t];
  if (slot < 0) return;
  int64_t pid, off;
  if (slot <= 0x7fffffffLL && p.ps <= 0x7fffffffLL) {
    const uint32_t pu = (uint32_t)slot / (uint32_t)p.ps;
    pid = pu;
    off = (uint32_t)slot - pu * (uint32_t)p.ps;
  } else {
    pid = slot / p.ps;
    off = slot - pid * p.ps;
  }
  if (pid >= p.P) return;  // out-of-pool slot: skipped (the host validates before launch)
  const int64_t row = (pid * p.Hkv + h) * p.ps + off;  // destination row index
  const int64_t src_off = t * p.st + h * p.sh;          // element offset of the source row
  if (p.kv_dtype == NVM_I8) {
    quantize_row(p.k, src_off, p.in_dtype, reinterpret_cast<int8_t*>(p.kp) + row * p.D, p.D, p.ks, row,
                 p.scale_dtype, lane);
    quantize_row(p.v, src_off, p.in_dtype, reinterpret_cast<int8_t*>(p.vp) + row * p.D, p.D, p.vs, row,
                 p.scale_dtype, lane);
  } else {
    const int64_t e = p.in_dtype == NVM_F32 ? 4 : 2;
    const int64_t bytes = p.D * e;
    copy_row(reinterpret_cast<const char*>(p.k) + src_off * e, reinterpret_cast<char*>(p.kp) + row * bytes, bytes,
             p.vec16 != 0, lane);
    copy_row(reinterpret_cast<const char*>(p.v) + src_off * e, reinterpret_cast<char*>(p.vp) + row * bytes, bytes,
             p.vec16 != 0, lane);
  }
}

}  // namespace

int launch_kv_write(const void* k, const void* v, int in_dtype, int64_t stride_t, int64_t stride_h, void* k_pages,
                    void* v_pages, int kv_dtype, void* k_scales, void* v_scales, int scale_dtype,
                    const int64_t* slot_mapping, int64_t T, int64_t Hkv, int64_t D, int64_t P, int64_t page_size,
                    cudaStream_t s) {
  KvWriteParams p{};
  p.k = k; p.v = v; p.kp = k_pages; p.vp = v_pages; p.ks = k_scales; p.vs = v_scales; p.slots = slot_mapping;
  p.st = stride_t; p.sh = stride_h; p.T = T; p.Hkv = Hkv; p.D = D; p.P = P; p.ps = page_size;
  p.in_dtype = in_dtype; p.kv_dtype = kv_dtype; p.scale_dtype = scale_dtype;
  const int64_t e = (int64_t)dtype_size(in_dtype);
  const bool aligned = ((uintptr_t)k % 16 == 0) && ((uintptr_t)v % 16 == 0) && ((uintptr_t)k_pages % 16 == 0) &&
                       ((uintptr_t)v_pages % 16 == 0) && ((stride_t * e) % 16 == 0) && ((stride_h * e) % 16 == 0) &&
                       ((D * e) % 16 == 0);
  p.vec16 = aligned ? 1 : 0;
  const int64_t warps = T * Hkv;
  kv_write_kernel<<<(unsigned)((warps + kWarps - 1) / kWarps), kWarps * 32, 0, s>>>(p);
  return check_cuda(cudaGetLastError(), "write_page_slice: kernel launch");
}

}  // namespace nvm
