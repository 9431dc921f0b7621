// w4a16.cu -- 4-bit group-128 weight GEMV / small-M GEMM (W4A16) for decode.
//
// Replaces QuantizedMatmul (src/nano_vllm_metal/metal/src/quantized_matmul.cpp:7-270,
// kernels quantized_matmul.metal:5-123) as called by layers/linear.py:73-126:
//   out[m, k] = sum_n a[m, n] * (q[k, n] * scale[k, n / 128] + bias[k, n / 128])
// with a [M, N] and out [M, K] in bf16 / fp16, q packed eight nibbles per uint32
// (element n of a word is bits 4j..4j+3, j = n % 8), scales / biases [K, N / 128] in
// the activation dtype, fp32 accumulation, the result rounded to the dtype.
//
// B200 design: the contraction runs on the tensor cores.  Per 128-element group
//   sum_n a q s + b = s * (sum_n a[m, n] q[k, n]) + b * (sum_n a[m, n]),
// so a group's integer weights (exact in bf16 / fp16) meet the activations in
// mma.sync.m16n8k16 (16 output rows x 8 activation rows), and the scale and bias are
// applied once per group in fp32.  A warp streams a 16-row x 128-element tile (1 KB of
// packed weights, two full 32-byte sectors per row) per group, the nibbles turned into
// bf16 / fp16 pairs with one LOP3 + one subtract per pair (magic-exponent trick), the
// weights of two groups loaded before the first is multiplied.  A CTA's 8 warps split
// the groups of its 16 rows and reduce in shared memory; when a projection has fewer
// 16-row tiles than two per SM, the groups of a tile are further split over a cluster of
// up to 8 CTAs whose partial sums are added in rank 0's shared memory (read over DSMEM).  Weights are read once for
// up to 16 activation rows; the kernel is bound by HBM bytes (0.53 B per weight).
#include <cooperative_groups.h>
#include <algorithm>
#include <cstdint>
#include <cstdlib>

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
constexpr int kPF = 2;      // groups whose weights a warp loads before using any
constexpr int kRows = 16;   // output rows (weight rows) per CTA
constexpr int kGroup = 128;

struct W4Params {
  const void* a;
  const uint32_t* w;
  const void* scales;
  const void* biases;
  void* out;
  int64_t M, N, K;
  int64_t m0;  // first activation row of this launch
};

template <typename T>
struct W4Traits;
template <>
struct W4Traits<__nv_bfloat16> {
  static constexpr uint32_t kMagic = 0x43004300u;  // bf16 128.0 in both halves
  __device__ static uint32_t sub_magic(uint32_t h) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&h);
    v = __hsub2(v, __floats2bfloat162_rn(128.f, 128.f));
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ static void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    mma16816<__nv_bfloat16>(d, a, b0, b1);
  }
};
template <>
struct W4Traits<__half> {
  static constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024.0 in both halves
  __device__ static uint32_t sub_magic(uint32_t h) {
    __half2 v = *reinterpret_cast<__half2*>(&h);
    v = __hsub2(v, __floats2half2_rn(1024.f, 1024.f));
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ static void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    mma16816<__half>(d, a, b0, b1);
  }
};

// Nibbles j and j + 4 of a word as a (low, high) pair of exact T values.
template <typename T>
__device__ __forceinline__ uint32_t nib_pair(uint32_t x, int j) {
  uint32_t h;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(h) : "r"(x >> (4 * j)), "r"(0x000F000Fu), "r"(W4Traits<T>::kMagic));
  return W4Traits<T>::sub_magic(h);
}

// Elements j and j + 4 of eight consecutive T values held in a uint4, as a pair.
__device__ __forceinline__ uint32_t act_pair(const uint4& v, int j) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  const uint32_t lo = w[j >> 1], hi = w[(j >> 1) + 2];
  return __byte_perm(lo, hi, (j & 1) ? 0x7632u : 0x5410u);
}

// Grid: (ceil(K / 16), ceil(M / (8 NT))).  Lane (g, t) = (lane / 4, lane % 4) owns weight
// rows g and g + 8 of the CTA's tile and, in every group, elements [32 t, 32 t + 32)
// as four words of eight nibbles; the mma's k index is permuted consistently in the
// weights and the activations (pair (j, j + 4) of word w feeds k-step 2w + j / 2).
// kCluster: the groups are split over the gridDim.z CTAs of a thread-block cluster (for
// projections with few 16-row tiles); their partial sums meet in rank 0's shared memory.
template <typename T, int NT, bool kCluster>
__global__ void __launch_bounds__(kWarps * 32) w4a16_kernel(const W4Params p) {
  using Tr = W4Traits<T>;
  __shared__ float red[kWarps][32][4 * NT];
  __shared__ float part[32][4 * NT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t k0 = (int64_t)blockIdx.x * kRows;
  const int64_t mb = p.m0 + (int64_t)blockIdx.y * 8 * NT;  // first activation row of the CTA
  const int64_t G = p.N / kGroup, words = p.N / 8;
  const int64_t rA = k0 + g, rB = k0 + g + 8;
  const bool okA = rA < p.K, okB = rB < p.K;
  const uint4* wA = reinterpret_cast<const uint4*>(p.w + (okA ? rA : 0) * words) + t;
  const uint4* wB = reinterpret_cast<const uint4*>(p.w + (okB ? rB : 0) * words) + t;
  const T* sc = static_cast<const T*>(p.scales);
  const T* bi = static_cast<const T*>(p.biases);
  const T* act = static_cast<const T*>(p.a);

  float tot[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) tot[n][0] = tot[n][1] = tot[n][2] = tot[n][3] = 0.f;

  // warps of all CTAs of the split share the groups round-robin
  const int64_t nsplit = kCluster ? gridDim.z : 1;
  const int64_t wstride = (int64_t)kWarps * nsplit;
  const int64_t wid = (kCluster ? (int64_t)blockIdx.z * kWarps : 0) + warp;
  // kPF groups per warp in flight: their weight loads are issued before any of them is used
  for (int64_t base = wid; base < G; base += wstride * kPF) {
    uint4 cwA[kPF], cwB[kPF];
#pragma unroll
    for (int i = 0; i < kPF; ++i) {
      const int64_t grp = base + (int64_t)i * wstride;
      const bool ok = grp < G;
      cwA[i] = ok && okA ? __ldg(wA + grp * 4) : make_uint4(0, 0, 0, 0);
      cwB[i] = ok && okB ? __ldg(wB + grp * 4) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < kPF; ++i) {
      const int64_t grp = base + (int64_t)i * wstride;
      if (grp >= G) break;  // warp-uniform
      // activations of this group: row mb + 8n + g, elements [32 t, 32 t + 32)
      uint4 av[NT][4];
      float asum_own[NT];
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int64_t m = mb + 8 * n + g;
        const uint4* ap = reinterpret_cast<const uint4*>(act + (m < p.M ? m : 0) * p.N + grp * kGroup + 32 * t);
        float sm = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          av[n][q] = m < p.M ? __ldg(ap + q) : make_uint4(0, 0, 0, 0);
          const T* e = reinterpret_cast<const T*>(&av[n][q]);
#pragma unroll
          for (int j = 0; j < 8; ++j) sm += to_f32(e[j]);
        }
        asum_own[n] = sm;
      }
      // the group's products: two accumulator chains per n-tile
      float acc[NT][2][4];
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int c = 0; c < 2; ++c) acc[n][c][0] = acc[n][c][1] = acc[n][c][2] = acc[n][c][3] = 0.f;
      const uint32_t xa[4] = {cwA[i].x, cwA[i].y, cwA[i].z, cwA[i].w};
      const uint32_t xb[4] = {cwB[i].x, cwB[i].y, cwB[i].z, cwB[i].w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int jl = 2 * h, jh = 2 * h + 1;  // low / high pair of k-step 2w + h
          const uint32_t afr[4] = {nib_pair<T>(xa[w], jl), nib_pair<T>(xb[w], jl), nib_pair<T>(xa[w], jh),
                                   nib_pair<T>(xb[w], jh)};
#pragma unroll
          for (int n = 0; n < NT; ++n) Tr::mma(acc[n][h], afr, act_pair(av[n][w], jl), act_pair(av[n][w], jh));
        }
      }
      // per-group scale and bias: rows g / g + 8, activation rows 2t / 2t + 1
      const float sA = okA ? to_f32(sc[rA * G + grp]) : 0.f, bA = okA ? to_f32(bi[rA * G + grp]) : 0.f;
      const float sB = okB ? to_f32(sc[rB * G + grp]) : 0.f, bB = okB ? to_f32(bi[rB * G + grp]) : 0.f;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        float as = asum_own[n];
        as += __shfl_xor_sync(0xffffffffu, as, 1);
        as += __shfl_xor_sync(0xffffffffu, as, 2);  // every lane of quad g: sum for row 8n + g
        const float s0 = __shfl_sync(0xffffffffu, as, 8 * t), s1 = __shfl_sync(0xffffffffu, as, 8 * t + 4);
        const float d0 = acc[n][0][0] + acc[n][1][0], d1 = acc[n][0][1] + acc[n][1][1];
        const float d2 = acc[n][0][2] + acc[n][1][2], d3 = acc[n][0][3] + acc[n][1][3];
        tot[n][0] += sA * d0 + bA * s0;
        tot[n][1] += sA * d1 + bA * s1;
        tot[n][2] += sB * d2 + bB * s0;
        tot[n][3] += sB * d3 + bB * s1;
      }
    }
  }
  // reduce the warps' partial sums; fragment c0: (row g, act 2t), c1: (g, 2t+1),
  // c2: (g+8, 2t), c3: (g+8, 2t+1)
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) red[warp][lane][4 * n + e] = tot[n][e];
  __syncthreads();
  for (int idx = threadIdx.x; idx < 32 * 4 * NT; idx += kWarps * 32) {
    const int ln = idx / (4 * NT), ee = idx % (4 * NT);
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w][ln][ee];
    part[ln][ee] = s;
  }
  // every CTA of a cluster reaches both cluster barriers (no early exit above)
  namespace cg = cooperative_groups;
  if constexpr (kCluster) cg::this_cluster().sync();
  else __syncthreads();
  const bool writer = kCluster ? cg::this_cluster().block_rank() == 0 : true;
  T* out = static_cast<T*>(p.out);
  for (int idx = threadIdx.x; writer && idx < 32 * 4 * NT; idx += kWarps * 32) {
    const int ln = idx / (4 * NT), ee = idx % (4 * NT);
    float s = part[ln][ee];
    if constexpr (kCluster) {
      for (unsigned r = 1; r < cg::this_cluster().num_blocks(); ++r)
        s += cg::this_cluster().map_shared_rank(&part[0][0], r)[idx];
    }
    const int n = ee / 4, e = ee % 4;
    const int gg = ln >> 2, tt = ln & 3;
    const int64_t row = k0 + gg + ((e & 2) ? 8 : 0);
    const int64_t m = mb + 8 * n + 2 * tt + (e & 1);
    if (row < p.K && m < p.M) out[m * p.K + row] = from_f32<T>(s);
  }
  if constexpr (kCluster) cg::this_cluster().sync();  // peers keep their shared memory until read
}

int sm_count() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      sms = n;
    if (sms <= 0) sms = 148;
  }
  return sms;
}

template <typename T, int NT>
int launch_nt(const W4Params& base, unsigned gx, unsigned gy, cudaStream_t s) {
  // Fewer 16-row tiles than two per SM: split every tile's groups over a cluster of up to
  // 8 CTAs (each still with at least two groups per warp).
  const int64_t G = base.N / kGroup;
  int64_t split = (2LL * sm_count() + (int64_t)gx * gy - 1) / ((int64_t)gx * gy);
  split = std::min<int64_t>(split, 8);
  split = std::min<int64_t>(split, G / (2 * kWarps));
  if (env_int("NVM_W4_SPLIT", 0) > 0) split = std::min<int64_t>(env_int("NVM_W4_SPLIT", 0), 8);
  if (split <= 1) {
    w4a16_kernel<T, NT, false><<<dim3(gx, gy), kWarps * 32, 0, s>>>(base);
    return check_cuda(cudaGetLastError(), "quantized_matmul: kernel launch");
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(gx, gy, (unsigned)split);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)split;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, w4a16_kernel<T, NT, true>, base), "quantized_matmul: kernel launch");
}

template <typename T>
int launch_t(const W4Params& base, cudaStream_t s) {
  const unsigned gx = (unsigned)((base.K + kRows - 1) / kRows);
  if (base.M <= 8) return launch_nt<T, 1>(base, gx, 1, s);
  // 16 activation rows per CTA; the weight tile is re-read (from L2) per 16 rows
  const int64_t chunks = (base.M + 15) / 16;
  if (chunks > 65535) return fail(NVM_ERR_INVALID_ARGUMENT, "quantized_matmul: too many rows");
  return launch_nt<T, 2>(base, gx, (unsigned)chunks, s);
}

}  // namespace
}  // namespace nvm

using namespace nvm;

extern "C" int nvm_w4a16_matmul(const void* a, int dtype, const uint32_t* w, const void* scales, const void* biases,
                                void* out, int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t bits,
                                void* stream) {
  const char* op = "quantized_matmul";
  if (dtype != NVM_F16 && dtype != NVM_BF16)
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: scales must be float16 or bfloat16", op);
  if (bits != 4) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: bits must be 4", op);
  if (group_size != kGroup) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: group_size must be 128", op);
  if (M < 0 || K < 0 || N <= 0) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: invalid sizes", op);
  if (N % kGroup != 0) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: a columns must be divisible by group_size", op);
  if (K > 0x7fffffffLL || (K + kRows - 1) / kRows > 0x7fffffffLL)
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: too many output columns", op);
  if (M == 0 || K == 0) return NVM_OK;
  if (!a || !w || !scales || !biases || !out) return fail(NVM_ERR_INVALID_ARGUMENT, "%s: null tensor pointer", op);
  // 16-byte rows: weight rows are N / 2 bytes (a multiple of 64), activation rows 2 N bytes
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w)) & 15)
    return fail(NVM_ERR_INVALID_ARGUMENT, "%s: a and b must start on 16-byte boundaries", op);
  W4Params p{a, w, scales, biases, out, M, N, K, 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == NVM_BF16 ? launch_t<__nv_bfloat16>(p, s) : launch_t<__half>(p, s);
}
