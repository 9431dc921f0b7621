// nvm_common.cuh -- device helpers shared by the sm_100a kernels of libnvm_attn.so:
// element conversion, mbarrier with bounded waits, TMA tensor loads (plain tile mode,
// each CTA loading into its own shared memory), ldmatrix / mma.sync fragments, and the launch-side
// parameter structs.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "nvm_attn.h"

namespace nvm {

// Codes written to the device error word when a bounded wait expires.
enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrFullWait = 1,    // consumer waited too long for a tile to land
  kDevErrEmptyWait = 2,   // producer waited too long for a stage to be released
  kDevErrDrainWait = 3,   // in-flight copies did not land while draining
  kDevErrTmemAlloc = 4,   // tensor-memory allocation wait expired
  kDevErrMmaWait = 5,     // tensor-core completion wait expired
  kDevErrSmemAlign = 6,   // dynamic shared memory not 1024-byte aligned (kernel did nothing)
  kDevErrBadIndex = 7,    // a device-side index (position, slot) outside its table; the row was skipped
};

// Every spin-wait gives up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

// ---------------------------------------------------------------------------
// element conversion
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<int8_t>(int8_t x) { return (float)x; }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Load element `i` of a buffer whose dtype is only known at run time.
__device__ __forceinline__ float load_dyn(const void* p, int64_t i, int dtype) {
  switch (dtype) {
    case NVM_F32: return reinterpret_cast<const float*>(p)[i];
    case NVM_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    case NVM_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    default: return (float)reinterpret_cast<const int8_t*>(p)[i];
  }
}

// Elements i and i + 1 (i even, the pointer aligned to two elements) as one load.
template <typename T>
__device__ __forceinline__ float2 load_pair(const void* p, int64_t i);
template <>
__device__ __forceinline__ float2 load_pair<float>(const void* p, int64_t i) {
  return __ldg(reinterpret_cast<const float2*>(p) + (i >> 1));
}
template <>
__device__ __forceinline__ float2 load_pair<__half>(const void* p, int64_t i) {
  return __half22float2(__ldg(reinterpret_cast<const __half2*>(p) + (i >> 1)));
}
template <>
__device__ __forceinline__ float2 load_pair<__nv_bfloat16>(const void* p, int64_t i) {
  return __bfloat1622float2(__ldg(reinterpret_cast<const __nv_bfloat162*>(p) + (i >> 1)));
}

__device__ __forceinline__ void store_dyn(void* p, int64_t i, int dtype, float v) {
  switch (dtype) {
    case NVM_F32: reinterpret_cast<float*>(p)[i] = v; break;
    case NVM_F16: reinterpret_cast<__half*>(p)[i] = __float2half_rn(v); break;
    default: reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
  }
}

// Pack two floats into a 16-bit pair (low = a, high = b) of the mma input type.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// int8 quantisation of x with row scale s = fl(amax / 127) (1 when amax == 0) and its
// reciprocal r = fl(1 / s): clip(rint(fl(x / s)), -127, 127), round half to even, as the
// reference's fp32 quotient.  |x| <= amax gives |x / s| <= 128, so t = fl(x * r) is within
// 2^-16 of x / s (two roundings of relative size 2^-24) and within 2^-15 of fl(x / s)
// (half an ulp below 128 is 2^-18).  If t lies at least 2^-14 from every half-integer, t
// and fl(x / s) are on the same side of it and round to the same integer.
//
// quantize_i8_fast rounds t through the 1.5 * 2^23 shifter (t + 1.5 * 2^23 is rounded to
// nearest even at unit spacing for |t| < 2^22) and reads the integer from the sum's low
// bits, so no conversion unit is involved; `amb` marks values within 2^-14 of a
// half-integer (and NaN), which the caller sends to quantize_i8_div.
__device__ __forceinline__ int quantize_i8_fast(float x, float r, bool& amb) {
  const float t = __fmul_rn(x, r);
  const float f = __fadd_rn(t, 12582912.0f);
  const float n = __fsub_rn(f, 12582912.0f);
  amb = !(fabsf(__fsub_rn(t, n)) < 0.5f - 0x1p-14f);
  const int q = __float_as_int(f) - 0x4B400000;
  return min(max(q, -127), 127);
}

__device__ __forceinline__ int quantize_i8_div(float x, float s) {
  const float y = rintf(__fdiv_rn(x, s));
  return (int)fminf(fmaxf(y, -127.0f), 127.0f);
}

__device__ __forceinline__ int quantize_i8(float x, float s, float r) {
  bool amb;
  const int q = quantize_i8_fast(x, r, amb);
  return amb ? quantize_i8_div(x, s) : q;
}

// ---------------------------------------------------------------------------
// shared memory, mbarrier, timers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with `parity` to complete; false once `limit_ns` of %globaltimer
// elapsed without it.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// The kernels' wait: false if kWaitTimeoutNs elapsed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  return mbar_wait_for(bar, parity, kWaitTimeoutNs);
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// Named barrier over `nthreads` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// TMA (tensor) loads into this CTA's shared memory, completing on an mbarrier.
// Plain tile mode only: every load fills the issuing CTA's own shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// L2 prefetch of one tensor box (no shared-memory destination, no completion signal).
__device__ __forceinline__ void tma_prefetch_4d(const CUtensorMap* map, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// ldmatrix / mma.sync fragments (m16n8k16, fp32 accumulate)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void lds128(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Two int8 values (bytes picked by `sel` out of x ^ 0x80808080) to an exact f16x2:
// the byte becomes the low mantissa of 1024.0h, then 1152.0h = 1024 + 128 is
// subtracted, giving the signed value exactly.
__device__ __forceinline__ uint32_t i8pair_to_f16x2(uint32_t x_flipped, uint32_t sel) {
  uint32_t h = prmt(x_flipped, 0x64646464u, sel);
  __half2 v = *reinterpret_cast<__half2*>(&h);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  v = __hsub2(v, bias);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace nvm
