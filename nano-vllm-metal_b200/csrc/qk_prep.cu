// qk_prep.cu -- fused per-layer attention preparation: q/k RMSNorm per head, rotary
// position embedding on q and k, and the paged KV scatter-write (with int8
// quantisation) of the rotated K and the raw V.
//
// Replaces the step sequence of Qwen3Attention.__call__ (src/nano_vllm_metal/models/
// qwen3.py:100-116) that runs before every attention call: q_norm / k_norm
// (layers/layernorm.py:4-14, mx.fast.rms_norm: x * rsqrt(mean(x^2) + eps) * weight in
// fp32, result in the input dtype), RoPE (layers/rotary_embedding.py:74-124, custom
// backend: fp32 cos/sin tables, halves rotated -- or interleaved pairs when
// traditional -- in fp32, result in the input dtype), then the pool write of
// cache.update_and_fetch_paged (cache/kv_cache.py:113-173 -> cache/paged.py:160-195,
// int8 through _quantize_page_slice, paged.py:152-158).
//
// A warp handles whole tokens; head rows [0, Hq) of a token are q heads, [Hq, Hq+Hkv)
// k heads, [Hq+Hkv, Hq+2*Hkv) v heads.  Lane l holds D/64 elements of each half of a
// row at the same slots, so the rotation partner of element i (i + D/2) is in the same
// lane.  Rounding points
// follow the reference: norm result rounded to the input dtype, rotation computed in
// fp32 from those rounded values with separately rounded products and sums, result
// rounded to the input dtype.  The cos/sin tables come from the caller (computed once,
// as the reference does), so kernel and oracle see the same table entries.
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "nvm_common.cuh"
#include "nvm_internal.h"

namespace nvm {
namespace {

constexpr int kWarps = 8;

int64_t env_int(const char* name, int64_t dflt) {
  const char* v = std::getenv(name);
  if (v == nullptr || v[0] == '\0') return dflt;
  return std::atoll(v);
}
constexpr int kBatch = 8;       // head rows whose loads are issued together
constexpr int kBlocksPerSm = 3;  // resident blocks per SM at <= 80 registers

struct QkPrepParams {
  const void* q;
  const void* k;
  const void* v;
  const void* wq;
  const void* wk;
  const float* cos_t;
  const float* sin_t;
  const int32_t* pos;
  void* q_out;
  void* kp;
  void* vp;
  void* ks;
  void* vs;
  const int64_t* slots;
  int* err;
  int64_t q_st, kv_st, table_rows, q_out_L, T, Hq, Hkv, P, ps;
  float eps;
  int dtype, kv_dtype, scale_dtype, traditional;
  int segs;  // work units per token (set at launch)
};

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// EH T values of one lane in one half of a row: 4 bytes (EH = 2, D = 128) or 2 (EH = 1)
template <typename T, int EH>
struct HalfVec;
template <typename T>
struct HalfVec<T, 2> {
  using V = uint32_t;
};
template <typename T>
struct HalfVec<T, 1> {
  using V = uint16_t;
};

template <typename T, int EH, typename V>
__device__ __forceinline__ void unpack(V raw, float* x) {
  const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int e = 0; e < EH; ++e) x[e] = to_f<T>(h[e]);
}

// round to nearest even into T; pairs go through one paired conversion
template <typename T, int EH, typename V>
__device__ __forceinline__ V pack(const float* x) {
  if constexpr (EH == 2) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(x[0], x[1]);
      return *reinterpret_cast<const uint32_t*>(&h);
    } else {
      const __half2 h = __floats2half2_rn(x[0], x[1]);
      return *reinterpret_cast<const uint32_t*>(&h);
    }
  } else {
    V raw;
    T* h = reinterpret_cast<T*>(&raw);
    h[0] = from_f<T>(x[0]);
    return raw;
  }
}

// Sum (or max) over the 32 lanes of eight per-row values at once.  Three halving steps
// (lane offsets 16, 8, 4) each hand half of the remaining rows to the partner lane, then
// two butterfly steps (2, 1) finish; lane l ends with row (l >> 2) & 7.  Every addition
// pairs the same two partial sums as the one-row butterfly v += shfl_xor(v, o) for
// o = 16, 8, 4, 2, 1, so each row's sum is bitwise the one-row result.
template <bool kMax>
__device__ __forceinline__ float reduce8(const float (&v)[8], int lane) {
  auto op = [](float a, float b) { return kMax ? fmaxf(a, b) : __fadd_rn(a, b); };
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float a[4], c[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b4 ? v[i] : v[i + 4], keep = b4 ? v[i + 4] : v[i];
    a[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b3 ? a[i] : a[i + 2], keep = b3 ? a[i + 2] : a[i];
    c[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
  float d = op(b2 ? c[1] : c[0], __shfl_xor_sync(0xffffffffu, b2 ? c[0] : c[1], 4));
  d = op(d, __shfl_xor_sync(0xffffffffu, d, 2));
  d = op(d, __shfl_xor_sync(0xffffffffu, d, 1));
  return d;
}

// int8 quantisation of one lane's 2*EH values of a row (both halves) whose scale s and
// its reciprocal r are known, written at dst + lo and dst + hi (same arithmetic as
// kv_write.cu: the quotient x / s rounded half to even and clipped to [-127, 127]).  The
// rare values near a half-integer are divided under one warp vote.
template <int EH>
__device__ __forceinline__ void quantize_row_lane(const float* x, float s, float r, int8_t* dst, int lo, int hi) {
  int q[2 * EH];
  bool amb[2 * EH];
  bool any = false;
#pragma unroll
  for (int e = 0; e < 2 * EH; ++e) {
    q[e] = quantize_i8_fast(x[e], r, amb[e]);
    any |= amb[e];
  }
  if (__any_sync(0xffffffffu, any)) {
#pragma unroll
    for (int e = 0; e < 2 * EH; ++e)
      if (amb[e]) q[e] = quantize_i8_div(x[e], s);
  }
  if constexpr (EH == 2) {
    *reinterpret_cast<uint16_t*>(dst + lo) = (uint16_t)((q[0] & 0xff) | ((q[1] & 0xff) << 8));
    *reinterpret_cast<uint16_t*>(dst + hi) = (uint16_t)((q[2] & 0xff) | ((q[3] & 0xff) << 8));
  } else {
    dst[lo] = (int8_t)q[0];
    dst[hi] = (int8_t)q[1];
  }
}

// Lane layout: lane l holds elements [l*EH, (l+1)*EH) of the first half of a row and the
// same slots of the second half (EH = D / 64), so the halves rotation partner (j, j + D/2)
// sits in the same lane, and so do the traditional pairs (2j, 2j+1) when EH = 2.  A lane's
// partial sum of squares runs over its first-half then second-half elements.
template <typename T, int D>
struct Lane {
  static constexpr int EH = D / 64;
  static constexpr int kHalf = D / 2;
  using V = typename HalfVec<T, EH>::V;
};

// The per-token rotation: cos / sin of each held element's angle.  Halves: element j and
// j + D/2 share angle j, so a lane needs EH angles; traditional: element j has angle j / 2.
template <int D, bool kTrad>
struct Rot {
  static constexpr int EH = D / 64;
  static constexpr int kAngles = kTrad ? 2 * EH : EH;
  float c[kAngles], s[kAngles];
};

// RMSNorm then RoPE of up to eight head rows (rows [h0, min(h0 + 8, count)) of one kind
// for one token), written by `emit(i, h, lo_bits, hi_bits)` (int8 pools: by quantising).
// Loads of the eight rows are issued first; the eight sums of squares are reduced
// together and 1 / sqrt(mean + eps) is evaluated once per row by the lanes that hold it.
template <typename T, int D, bool kTrad, typename Emit>
__device__ __forceinline__ void norm_rope_batch(const T* src_tok, int h0, int count, typename Lane<T, D>::V w_lo,
                                                typename Lane<T, D>::V w_hi, const Rot<D, kTrad>& rot, float eps,
                                                int lane, Emit&& emit) {
  using L = Lane<T, D>;
  using V = typename L::V;
  constexpr int EH = L::EH;
  const int lo = lane * EH, hi = L::kHalf + lane * EH;
  V rlo[kBatch], rhi[kBatch];
#pragma unroll
  for (int i = 0; i < kBatch; ++i) {
    rlo[i] = 0;
    rhi[i] = 0;
    if (h0 + i < count) {
      const T* src = src_tok + (h0 + i) * D;
      rlo[i] = __ldg(reinterpret_cast<const V*>(src + lo));
      rhi[i] = __ldg(reinterpret_cast<const V*>(src + hi));
    }
  }
  float red[kBatch];
#pragma unroll
  for (int i = 0; i < kBatch; ++i) {
    float x[2 * EH];
    unpack<T, EH>(rlo[i], x);
    unpack<T, EH>(rhi[i], x + EH);
    float ss = __fmul_rn(x[0], x[0]);
#pragma unroll
    for (int e = 1; e < 2 * EH; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
    red[i] = ss;
  }
  // mean = ss / D computed as ss * (1 / D): D is a power of two, so both are the same
  // correctly rounded value; 1 / sqrt as the correctly rounded reciprocal of the root
  const float inv_mine = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(reduce8<false>(red, lane), 1.0f / (float)D), eps)));
  float w[2 * EH];
  unpack<T, EH>(w_lo, w);
  unpack<T, EH>(w_hi, w + EH);
#pragma unroll
  for (int i = 0; i < kBatch; ++i) {
    const float inv = __shfl_sync(0xffffffffu, inv_mine, i * 4);
    if (h0 + i >= count) break;  // warp-uniform
    float x[2 * EH], y[2 * EH];
    unpack<T, EH>(rlo[i], x);
    unpack<T, EH>(rhi[i], x + EH);
    // normalised value rounded to T (pairs converted together)
#pragma unroll
    for (int e = 0; e < 2 * EH; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], inv), w[e]);
    unpack<T, EH>(pack<T, EH, V>(x), x);
    unpack<T, EH>(pack<T, EH, V>(x + EH), x + EH);
    if constexpr (kTrad) {
      if constexpr (EH == 2) {
        // pairs (x[0], x[1]) and (x[2], x[3]) sit in the lane
#pragma unroll
        for (int e = 0; e < 2 * EH; e += 2) {
          y[e] = __fsub_rn(__fmul_rn(x[e], rot.c[e]), __fmul_rn(x[e + 1], rot.s[e]));
          y[e + 1] = __fadd_rn(__fmul_rn(x[e], rot.s[e]), __fmul_rn(x[e + 1], rot.c[e]));
        }
      } else {
        // EH == 1: element 2j is held by an even lane, its partner 2j+1 by lane ^ 1
        const bool even = (lane & 1) == 0;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float other = __shfl_xor_sync(0xffffffffu, x[e], 1);
          const float x1 = even ? x[e] : other, x2 = even ? other : x[e];
          y[e] = even ? __fsub_rn(__fmul_rn(x1, rot.c[e]), __fmul_rn(x2, rot.s[e]))
                      : __fadd_rn(__fmul_rn(x1, rot.s[e]), __fmul_rn(x2, rot.c[e]));
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < EH; ++e) {
        const float x1 = x[e], x2 = x[EH + e];
        y[e] = __fsub_rn(__fmul_rn(x1, rot.c[e]), __fmul_rn(x2, rot.s[e]));
        y[EH + e] = __fadd_rn(__fmul_rn(x1, rot.s[e]), __fmul_rn(x2, rot.c[e]));
      }
    }
    emit(i, h0 + i, pack<T, EH, V>(y), pack<T, EH, V>(y + EH));
  }
}

// int8 write of up to eight rows already rounded to T (packed per lane in rlo / rhi):
// scale = absmax / 127 (1 for an all-zero row) reduced for the eight rows together.
template <typename T, int D>
__device__ __forceinline__ void quantize_batch(const typename Lane<T, D>::V (&rlo)[kBatch],
                                               const typename Lane<T, D>::V (&rhi)[kBatch], int h0, int count,
                                               int8_t* pool_row0, int64_t row_stride, void* scales, int64_t srow0,
                                               int64_t srow_stride, int scale_dtype, int lane) {
  using L = Lane<T, D>;
  constexpr int EH = L::EH;
  const int lo = lane * EH, hi = L::kHalf + lane * EH;
  float red[kBatch];
#pragma unroll
  for (int i = 0; i < kBatch; ++i) {
    float x[2 * EH];
    unpack<T, EH>(rlo[i], x);
    unpack<T, EH>(rhi[i], x + EH);
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < 2 * EH; ++e) m = fmaxf(m, fabsf(x[e]));
    red[i] = m;
  }
  const float amax_mine = reduce8<true>(red, lane);
  const float s_mine = amax_mine > 0.0f ? __fdiv_rn(amax_mine, 127.0f) : 1.0f;
  const float r_mine = __frcp_rn(s_mine);
#pragma unroll
  for (int i = 0; i < kBatch; ++i) {
    const float sc = __shfl_sync(0xffffffffu, s_mine, i * 4);
    const float rc = __shfl_sync(0xffffffffu, r_mine, i * 4);
    if (h0 + i >= count) break;  // warp-uniform
    float x[2 * EH];
    unpack<T, EH>(rlo[i], x);
    unpack<T, EH>(rhi[i], x + EH);
    quantize_row_lane<EH>(x, sc, rc, pool_row0 + (int64_t)(h0 + i) * row_stride, lo, hi);
    if (lane == 0) store_dyn(scales, srow0 + (int64_t)(h0 + i) * srow_stride, scale_dtype, sc);
  }
}

// Persistent grid over work units of one token's rows (all of them, or one segment of
// consecutive eight-row batches when tokens are few), grid-stride in token-major order.
// A unit reads the token's position and slot and its lanes' cos/sin entries once, then
// runs its batches of eight rows of one kind.  Rows whose result is not needed (q/k
// rows at a bad position, k/v rows of a skipped or bad slot) are not read.
template <typename T, int D, bool kTrad, bool kInt8>
__global__ void __launch_bounds__(kWarps * 32, kBlocksPerSm) qk_prep_kernel(const QkPrepParams p) {
  using L = Lane<T, D>;
  using V = typename L::V;
  constexpr int EH = L::EH;
  constexpr int kHalf = L::kHalf;
  static_assert(kBatch == 8, "reduce8 reduces eight rows");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Hq = (int)p.Hq, Hkv = (int)p.Hkv;
  const int64_t n_warps = (int64_t)gridDim.x * kWarps;
  const int lo = lane * EH, hi = kHalf + lane * EH;  // first element of each half
  const int64_t pool_head = p.ps * D;                 // elements between kv heads of a page
  // norm weights of the lane's elements, kept packed
  const V wq_lo = __ldg(reinterpret_cast<const V*>(static_cast<const T*>(p.wq) + lo));
  const V wq_hi = __ldg(reinterpret_cast<const V*>(static_cast<const T*>(p.wq) + hi));
  const V wk_lo = __ldg(reinterpret_cast<const V*>(static_cast<const T*>(p.wk) + lo));
  const V wk_hi = __ldg(reinterpret_cast<const V*>(static_cast<const T*>(p.wk) + hi));

  // work units: (token, segment), token-major.  A token's rows form nb batches of eight
  // rows of one kind -- [0, nbq) q rows, [nbq, nbq + nbk) k rows, [nbq + nbk, nb) v rows --
  // cut into p.segs segments of consecutive batches (one segment when there are enough
  // tokens to keep every warp busy; more when there are few, so the grid's tail stays short)
  const int nbq = (Hq + kBatch - 1) / kBatch, nbk = (Hkv + kBatch - 1) / kBatch, nb = nbq + 2 * nbk;
  const int S = p.segs, bs = (nb + S - 1) / S;
  const int64_t gw = (int64_t)blockIdx.x * kWarps + warp;
  int64_t t = gw / S;
  int sg = (int)(gw - t * S);
  const int64_t dt = n_warps / S;
  const int ds = (int)(n_warps - dt * S);
  for (; t < p.T; t += dt, sg += ds) {
    if (sg >= S) {
      sg -= S;
      ++t;
      if (t >= p.T) break;
    }
    const int b_begin = sg * bs, b_end = min(b_begin + bs, nb);
    if (b_begin >= b_end) continue;
    int pos = 0;
    bool rope_ok = false, kv_ok = false;
    if (b_begin < nbq + nbk) {
      pos = __ldg(p.pos + t);
      // every lane read the same value: the vote makes the branches warp-uniform
      rope_ok = __all_sync(0xffffffffu, pos >= 0 && (int64_t)pos < p.table_rows);
      if (lane == 0 && !rope_ok) record_error(p.err, kDevErrBadIndex);
    }
    int64_t prow0 = 0;  // pool row of kv head 0
    if (b_end > nbq) {
      const int64_t slot = __ldg(p.slots + t);
      int64_t pid = -1, off = 0;
      if (slot >= 0) {
        if (slot <= 0x7fffffffLL && p.ps <= 0x7fffffffLL) {
          const uint32_t pu = (uint32_t)slot / (uint32_t)p.ps;
          pid = pu;
          off = (uint32_t)slot - pu * (uint32_t)p.ps;
        } else {
          pid = slot / p.ps;
          off = slot - pid * p.ps;
        }
      }
      kv_ok = __all_sync(0xffffffffu, slot >= 0 && pid < p.P);
      if (lane == 0 && slot >= 0 && pid >= p.P) record_error(p.err, kDevErrBadIndex);
      prow0 = pid * p.Hkv * p.ps + off;
    }
    Rot<D, kTrad> rot;
    if (rope_ok) {
      const float* ct = p.cos_t + (int64_t)pos * kHalf;
      const float* st = p.sin_t + (int64_t)pos * kHalf;
#pragma unroll
      for (int e = 0; e < EH; ++e) {
        const int alo = kTrad ? (lo + e) >> 1 : lo + e;
        rot.c[e] = __ldg(ct + alo);
        rot.s[e] = __ldg(st + alo);
        if constexpr (kTrad) {
          rot.c[EH + e] = __ldg(ct + ((hi + e) >> 1));
          rot.s[EH + e] = __ldg(st + ((hi + e) >> 1));
        }
      }
    }

    // q rows -> q_out row ob + h * q_mul ([T, Hq, D], or [T / L, Hq, L, D] when q_out_L > 0)
    if (rope_ok && b_begin < nbq) {
      int64_t ob = t * p.Hq, q_mul = 1;
      if (p.q_out_L > 0) {
        const int64_t bb = t / p.q_out_L, l = t - bb * p.q_out_L;
        ob = bb * p.Hq * p.q_out_L + l;
        q_mul = p.q_out_L;
      }
      T* q_out = static_cast<T*>(p.q_out) + ob * D;
      const T* q_tok = static_cast<const T*>(p.q) + t * p.q_st;
      const int e_end = min(b_end, nbq);
      for (int bt = b_begin; bt < e_end; ++bt) {
        norm_rope_batch<T, D, kTrad>(q_tok, bt * kBatch, Hq, wq_lo, wq_hi, rot, p.eps, lane,
                                     [&](int, int h, V ylo, V yhi) {
                                       T* dst = q_out + (int64_t)h * q_mul * D;
                                       *reinterpret_cast<V*>(dst + lo) = ylo;
                                       *reinterpret_cast<V*>(dst + hi) = yhi;
                                     });
      }
    }
    // k rows -> the key pool (normalised and rotated)
    if (rope_ok && kv_ok) {
      const T* k_tok = static_cast<const T*>(p.k) + t * p.kv_st;
      const int e_end = min(b_end, nbq + nbk);
      for (int bt = max(b_begin, nbq); bt < e_end; ++bt) {
        const int h0 = (bt - nbq) * kBatch;
        if constexpr (kInt8) {
          V qlo[kBatch], qhi[kBatch];
#pragma unroll
          for (int i = 0; i < kBatch; ++i) qlo[i] = qhi[i] = 0;
          norm_rope_batch<T, D, kTrad>(k_tok, h0, Hkv, wk_lo, wk_hi, rot, p.eps, lane, [&](int i, int, V ylo, V yhi) {
#pragma unroll
            for (int j = 0; j < kBatch; ++j)
              if (j == i) {
                qlo[j] = ylo;
                qhi[j] = yhi;
              }
          });
          quantize_batch<T, D>(qlo, qhi, h0, Hkv, static_cast<int8_t*>(p.kp) + prow0 * D, pool_head, p.ks, prow0, p.ps,
                               p.scale_dtype, lane);
        } else {
          T* k_row0 = static_cast<T*>(p.kp) + prow0 * D;
          norm_rope_batch<T, D, kTrad>(k_tok, h0, Hkv, wk_lo, wk_hi, rot, p.eps, lane, [&](int, int h, V ylo, V yhi) {
            T* dst = k_row0 + (int64_t)h * pool_head;
            *reinterpret_cast<V*>(dst + lo) = ylo;
            *reinterpret_cast<V*>(dst + hi) = yhi;
          });
        }
      }
    }
    // v rows -> the value pool, unchanged (int8 pools: quantised)
    if (kv_ok) {
      const T* v_tok = static_cast<const T*>(p.v) + t * p.kv_st;
      for (int bt = max(b_begin, nbq + nbk); bt < b_end; ++bt) {
        const int h0 = (bt - nbq - nbk) * kBatch;
        V rlo[kBatch], rhi[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          rlo[i] = 0;
          rhi[i] = 0;
          if (h0 + i < Hkv) {
            const T* src = v_tok + (h0 + i) * D;
            rlo[i] = __ldg(reinterpret_cast<const V*>(src + lo));
            rhi[i] = __ldg(reinterpret_cast<const V*>(src + hi));
          }
        }
        if constexpr (kInt8) {
          quantize_batch<T, D>(rlo, rhi, h0, Hkv, static_cast<int8_t*>(p.vp) + prow0 * D, pool_head, p.vs, prow0,
                               p.ps, p.scale_dtype, lane);
        } else {
          T* v_row0 = static_cast<T*>(p.vp) + prow0 * D;
#pragma unroll
          for (int i = 0; i < kBatch; ++i) {
            if (h0 + i >= Hkv) break;
            T* dst = v_row0 + (int64_t)(h0 + i) * pool_head;
            *reinterpret_cast<V*>(dst + lo) = rlo[i];
            *reinterpret_cast<V*>(dst + hi) = rhi[i];
          }
        }
      }
    }
  }
}

template <typename T, int D, bool kTrad, bool kInt8>
void launch_one(const QkPrepParams& p, unsigned grid, cudaStream_t s) {
  qk_prep_kernel<T, D, kTrad, kInt8><<<grid, kWarps * 32, 0, s>>>(p);
}

template <typename T>
int launch_t(const QkPrepParams& p, int64_t D, cudaStream_t s) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      sms = n;
    if (sms <= 0) sms = 148;
  }
  // segments per token: about one unit per resident warp.  With int8 pools the segment
  // holding the k and v rows (quantised) outweighs the others, and whole tokens per warp
  // won once there are a quarter as many tokens as warps (8192 tokens: 2636 GB/s against
  // 2147 with two segments; 2048 tokens: 1924 against 1539).
  const int64_t nb = (p.Hq + kBatch - 1) / kBatch + 2 * ((p.Hkv + kBatch - 1) / kBatch);
  const int64_t warps_cap = (int64_t)sms * kBlocksPerSm * kWarps;
  QkPrepParams q = p;
  q.segs = (int)std::min<int64_t>(nb, std::max<int64_t>(1, (warps_cap + p.T - 1) / std::max<int64_t>(p.T, 1)));
  if (p.kv_dtype == NVM_I8 && 4 * p.T >= warps_cap) q.segs = 1;
  static const int64_t segs_env = env_int("NVM_QKPREP_SEGS", 0);
  if (segs_env > 0) q.segs = (int)std::min<int64_t>(nb, segs_env);
  const int64_t blocks_needed = (p.T * q.segs + kWarps - 1) / kWarps;
  const int64_t grid = std::min<int64_t>(blocks_needed, (int64_t)sms * kBlocksPerSm);
  const unsigned g = (unsigned)grid;
  const bool i8 = q.kv_dtype == NVM_I8;
  if (D == 128) {
    if (p.traditional)
      i8 ? launch_one<T, 128, true, true>(q, g, s) : launch_one<T, 128, true, false>(q, g, s);
    else
      i8 ? launch_one<T, 128, false, true>(q, g, s) : launch_one<T, 128, false, false>(q, g, s);
  } else {
    if (p.traditional)
      i8 ? launch_one<T, 64, true, true>(q, g, s) : launch_one<T, 64, true, false>(q, g, s);
    else
      i8 ? launch_one<T, 64, false, true>(q, g, s) : launch_one<T, 64, false, false>(q, g, s);
  }
  return check_cuda(cudaGetLastError(), "qk_norm_rope_write: kernel launch");
}

}  // namespace
}  // namespace nvm

using namespace nvm;

extern "C" int nvm_qk_norm_rope_write(const void* q, const void* k, const void* v, int dtype, int64_t q_stride_t,
                                      int64_t kv_stride_t, const void* q_norm_weight, const void* k_norm_weight,
                                      float eps, const float* cos_table, const float* sin_table, int64_t table_rows,
                                      int traditional, const int32_t* positions, void* q_out, int64_t q_out_L,
                                      void* k_pages, void* v_pages, int kv_dtype, void* k_scales, void* v_scales,
                                      int scale_dtype, const int64_t* slot_mapping, int64_t T, int64_t Hq,
                                      int64_t Hkv, int64_t D, int64_t P, int64_t page_size, void* stream) {
  const char* op = "qk_norm_rope_write";
  if (dtype != NVM_F16 && dtype != NVM_BF16)
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: q/k/v must be float16 or bfloat16", op);
  if (kv_dtype != dtype && kv_dtype != NVM_I8)
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: page dtype must equal the input dtype or be int8", op);
  if (kv_dtype == NVM_I8 && (k_scales == nullptr || v_scales == nullptr ||
                             (scale_dtype != NVM_F32 && scale_dtype != NVM_F16 && scale_dtype != NVM_BF16)))
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: int8 pages need floating-point key/value scales", op);
  if (D != 64 && D != 128) return fail(NVM_ERR_UNSUPPORTED, "%s: head dim must be 64 or 128 (got %lld)", op, (long long)D);
  if (T < 0 || Hq <= 0 || Hkv <= 0 || P < 0 || page_size <= 0 || table_rows <= 0)
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: sizes must be positive", op);
  if (Hq + 2 * Hkv > (1 << 20)) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: too many heads", op);
  if (q_stride_t < Hq * D || kv_stride_t < Hkv * D)
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: token strides must cover every head row", op);
  // lanes move D/32 elements (8 bytes for D = 128, 4 for 64) as one vector
  const int64_t vec_elems = D / 32;
  if (q_stride_t % vec_elems != 0 || kv_stride_t % vec_elems != 0 ||
      reinterpret_cast<uintptr_t>(q) % (vec_elems * 2) != 0 || reinterpret_cast<uintptr_t>(k) % (vec_elems * 2) != 0 ||
      reinterpret_cast<uintptr_t>(v) % (vec_elems * 2) != 0 ||
      reinterpret_cast<uintptr_t>(q_norm_weight) % (vec_elems * 2) != 0 ||
      reinterpret_cast<uintptr_t>(k_norm_weight) % (vec_elems * 2) != 0 ||
      reinterpret_cast<uintptr_t>(q_out) % (vec_elems * 2) != 0 ||
      reinterpret_cast<uintptr_t>(cos_table) % (vec_elems * 4) != 0 ||
      reinterpret_cast<uintptr_t>(sin_table) % (vec_elems * 4) != 0 ||
      reinterpret_cast<uintptr_t>(k_pages) % (vec_elems * 2) != 0 ||
      reinterpret_cast<uintptr_t>(v_pages) % (vec_elems * 2) != 0)
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: rows must start on %lld-byte boundaries (strides in whole vectors)", op,
                (long long)(vec_elems * 2));
  if (q_out_L < 0 || (q_out_L > 0 && T % q_out_L != 0))
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: q_out_L must divide the token count", op);
  if (T == 0) return NVM_OK;
  if (q == nullptr || k == nullptr || v == nullptr || q_norm_weight == nullptr || k_norm_weight == nullptr ||
      cos_table == nullptr || sin_table == nullptr || positions == nullptr || q_out == nullptr ||
      slot_mapping == nullptr || (P > 0 && (k_pages == nullptr || v_pages == nullptr)))
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: null pointer", op);
  QkPrepParams p{};
  p.q = q; p.k = k; p.v = v; p.wq = q_norm_weight; p.wk = k_norm_weight;
  p.cos_t = cos_table; p.sin_t = sin_table; p.pos = positions; p.q_out = q_out;
  p.kp = k_pages; p.vp = v_pages; p.ks = k_scales; p.vs = v_scales; p.slots = slot_mapping;
  p.err = device_error_word();
  p.q_st = q_stride_t; p.kv_st = kv_stride_t; p.table_rows = table_rows; p.q_out_L = q_out_L;
  p.T = T; p.Hq = Hq; p.Hkv = Hkv; p.P = P; p.ps = page_size; p.eps = eps;
  p.dtype = dtype; p.kv_dtype = kv_dtype; p.scale_dtype = scale_dtype; p.traditional = traditional ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == NVM_BF16 ? launch_t<__nv_bfloat16>(p, D, s) : launch_t<__half>(p, D, s);
}
