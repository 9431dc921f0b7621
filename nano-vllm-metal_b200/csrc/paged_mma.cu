// paged_mma.cu -- tensor-core paged attention for decode, multi-token verify and
// chunked prefill (and dense attention viewed as one page per sequence).
//
// Replaces the reference's Metal kernels paged_attention_decode_split_kv
// (paged_attention.metal:276-408), paged_attention_kv (:6-128) and
// paged_attention_int8_decode_kv (:417-525), with the dispatch of
// paged_attention.cpp:413-642.  Same results, different decomposition:
//
//  * One CTA owns one (sequence b, kv head h, row block, key chunk).  The rows are
//    the g*L query rows that share kv head h (g = Hq/Hkv q heads x L tokens), packed
//    into 16-row m-tiles, so every K/V byte is read from HBM once per kv head instead
//    of once per q head as in the reference (grid = B*Hq there).
//  * Keys are processed in 16-token tiles.  A producer warp (on the n8 tile, each
//    consumer warp for the stages it consumes) streams each tile's K and V rows
//    ([16][D] contiguous inside one page) with plain tile-mode TMA tensor loads
//    (128-byte swizzle) into an NSTAGE-deep shared-memory ring guarded by mbarriers; page ids
//    come from the block table, holes are skipped.
//  * Consumer warps run the FA2-style online softmax on mma.sync m16n8k16 (fp32
//    accumulate): S = Q K^T from ldmatrix'd K, P kept in registers as the A operand
//    of O += P V with ldmatrix.trans'd V.  int8 pages are converted to f16 in
//    registers (exact), the per-token key scale multiplies S and the value scale
//    multiplies V, i.e. dequantisation happens in-kernel for every L.
//  * Split-K: long contexts are cut into chunks of `chunk_tiles` tiles handled by
//    separate CTAs; each writes (O, m, l) to the workspace and the last CTA of the
//    unit (atomic ticket) merges them with log-sum-exp weights and resets the ticket.
//  * Every mbarrier wait is bounded (nvm::mbar_wait); on expiry the kernel records an
//    error code, each issuing warp drains what it issued, and the CTA returns.
#include <cooperative_groups.h>
#include <type_traits>

#include <cstdio>
#include <cstdlib>
#include <atomic>
#include <mutex>

#include "nvm_common.cuh"
#include "nvm_internal.h"

namespace nvm {
namespace {

constexpr int kMaxChunkTiles = 256;
// Split-K tickets live in a fixed region at the start of the workspace that partial
// results never use, so one zero-filled workspace can serve calls of any shape.
constexpr size_t kCounterBytes = kTicketRegionBytes;
constexpr int64_t kMaxUnits = (int64_t)(kCounterBytes / sizeof(int));
constexpr int kDefaultDecodeVariant = 3;
constexpr int kDefaultN8Variant = 7;  // c4 int8 prefers 4 (2 warps, 8 stages) by 1%
constexpr int kDefaultM3Variant = 1;
// longest chunk (16-key tiles) the one-wave sizing of the n8 tile hands a CTA
constexpr int64_t kOneWaveTiles = 128;

struct MmaParams {
  const void* q;
  void* out;
  const int32_t* block_table;
  const int32_t* context_lens;
  float* part_o;      // [units][n_chunks][rows_real][D]
  float2* part_ml;    // [units][n_chunks][rows_real]
  int* counters;      // [units]
  int* err;
  int q_dtype, out_dtype;
  int64_t B, Hq, Hkv, L, P, ps, mp, dense_ctx;
  int64_t g, M;       // q heads per kv head, rows per (b, h)
  int64_t n_rb, rows_real, ct, n_chunks;
  float scale_log2;   // softmax scale * log2(e)
  int causal;
  int cluster;        // the n_chunks CTAs of a unit are one cluster: merge over DSMEM
};

template <typename KvT, int D, int NWM, int NWK, int NS_ = 0>
struct Cfg {
  static constexpr bool kI8 = std::is_same<KvT, int8_t>::value;
  using MmaT = typename std::conditional<kI8, __half, KvT>::type;
  static constexpr bool kSplitP = std::is_same<KvT, __nv_bfloat16>::value;
  // NWM == 0 selects the n8 tile: keys are the mma's M (16 per tile) and up to eight
  // query rows its N, so S^T = K Q^T and O^T = V^T P^T take half the mma.sync of the
  // 16-row tile when a kv head has at most eight query rows.
  static constexpr bool kN8 = NWM == 0;
  static constexpr int kCons = (kN8 ? 1 : NWM) * NWK;
  // The n8 tile has no producer warp: each consumer warp refills the ring
  // stages it consumes (stage s belongs to warp s % NWK), so a CTA is 64 threads and more
  // CTAs fit on an SM (the kernel is latency-bound there).
  static constexpr bool kSelfFeed = kN8;
  static constexpr int kThreads = (kCons + (kSelfFeed ? 0 : 1)) * 32;
  static constexpr int kRB = kN8 ? 8 : 16 * NWM;
  static constexpr int kTileBytes = 16 * D * (int)sizeof(KvT);
  // K scales at +0, V scales at +128 past the two tiles: TMA destinations are 128-byte aligned.
  static constexpr int kScaleBytes = kI8 ? 256 : 0;
  static constexpr int kStageBytes = ((2 * kTileBytes + kScaleBytes + 1023) / 1024) * 1024;
  static constexpr int kStages = NS_ > 0 ? NS_ : (kI8 ? 12 : 8);
  static constexpr int kBoxElems = 128 / (int)sizeof(KvT);  // 128-byte inner box (swizzle span)
  static constexpr int kBoxes = D / kBoxElems;
  static constexpr int kEpiBytes = NWK * kRB * D * 4 + 2 * NWK * kRB * 4;
  static constexpr int kRingBytes = kStages * kStageBytes;
  // cluster merge (n8 tile): this CTA's combined partial rows [kRB][D], their (m, l) and
  // the chunk weights [8][kRB] + sums [kRB], placed after the epilogue staging area
  static constexpr int kClusterOff = ((kEpiBytes + 15) / 16) * 16;
  static constexpr int kClusterBytes = kRB * D * 4 + kRB * 8 + 8 * kRB * 4 + kRB * 4;
  // only self-feeding CTAs (every warp is a consumer and reaches the cluster barriers)
  static constexpr bool kClusterFits = kN8 && kSelfFeed;
  static constexpr int kEpiAll = kClusterFits ? kClusterOff + kClusterBytes : kEpiBytes;
  static constexpr int kMainBytes = kRingBytes > kEpiAll ? kRingBytes : kEpiAll;
  static constexpr int kSmemBytes = 1024 + kMainBytes + kStages * 16 + kStages * 4 + kMaxChunkTiles * 4 + 16;
  static_assert(kStages % NWK == 0, "stage ring must be a multiple of the k-split");
  static_assert(D % 64 == 0, "head dim must be 64 or 128");
  static_assert(!kI8 || D == 128, "int8 path needs D == 128");
};

// 8x8 b16 matrix held in the mma accumulator layout (row lane/4, columns 2(lane%4), +1),
// transposed across the warp (PTX movmatrix)
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// bf16 pair of the rounding residuals (a - hi.x, b - hi.y) of a packed bf16 pair.
__device__ __forceinline__ uint32_t pack_residual(float a, float b, uint32_t hi) {
  const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&hi);
  return pack2<__nv_bfloat16>(a - __low2float(h), b - __high2float(h));
}

// Address of 16-byte chunk `q` of token row `tok` inside a TMA tile written with
// 128-byte swizzle: boxes of 128 bytes x 16 rows, 2048 bytes each, chunk index XOR row.
__device__ __forceinline__ uint32_t swz(uint32_t tile, int tok, int q) {
  return tile + (uint32_t)((q >> 3) * 2048 + tok * 128 + (((q & 7) ^ (tok & 7)) << 4));
}

template <typename KvT, typename ScaleT, int D, int NWM, int NWK, int NS_>
__global__ void __launch_bounds__(Cfg<KvT, D, NWM, NWK, NS_>::kThreads)
    paged_mma_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_ks, const __grid_constant__ CUtensorMap tm_vs,
                     const MmaParams p) {
  using C = Cfg<KvT, D, NWM, NWK, NS_>;
  using MmaT = typename C::MmaT;
  constexpr int NS = C::kStages;
  constexpr int NKS = D / 16;  // k-steps of Q K^T
  constexpr int NDT = D / 8;   // n8 tiles of the output

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kMainBytes);
  uint64_t* empty = full + NS;
  int* stage_valid = reinterpret_cast<int*>(empty + NS);
  int* tile_pid = stage_valid + NS;
  int* s_flag = tile_pid + kMaxChunkTiles;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 32-bit index arithmetic (the plan bounds units, rows and tiles below 2^31): a 64-bit
  // division costs about a hundred instructions, and these sit in front of the first
  // page copies.
  const int64_t unit = blockIdx.x;
  const uint32_t u32 = blockIdx.x, nrb = (uint32_t)p.n_rb, hkv = (uint32_t)p.Hkv;
  const uint32_t bh32 = u32 / nrb;
  const int64_t rb = u32 - bh32 * nrb;
  const uint32_t b32 = bh32 / hkv;
  const int64_t h = bh32 - b32 * hkv, b = b32;
  // paged: 16-token tiles per page (page_size is a multiple of 16)
  const uint32_t tpp = (uint32_t)(p.ps >> 4);
  const int64_t c = blockIdx.y;

  const int64_t ctx = p.context_lens ? (int64_t)p.context_lens[b] : p.dense_ctx;
  const int64_t cap = p.mp * p.ps;
  const int64_t ctx_limit = ctx < cap ? ctx : cap;
  const int64_t row0 = rb * C::kRB;
  const int64_t rows_here = (p.M - row0) < C::kRB ? (p.M - row0) : C::kRB;
  const int64_t t_begin = c * p.ct;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::kN8 ? 1 : NWM);
    }
    fence_mbar_init();
  }
  // Consumers load their Q fragments while the producer reads the block table: one
  // round of independent vector loads (pairs of elements), dtype dispatch outside.
  constexpr int kWM = C::kN8 ? 1 : NWM;
  const int wm = warp % kWM, wk = warp / kWM;
  const int r = lane >> 2, cq = lane & 3;
  const int64_t q_row0 = (b * p.Hq + h * p.g) * p.L;  // flat row of (b, h, m = 0)
  // this thread's two softmax rows (unit-relative): m16 tile rows r, r + 8; n8 tile
  // columns 2 cq, 2 cq + 1.  The n8 tile's Q operand is row r (loaded as "row A").
  const int64_t mA = C::kN8 ? row0 + r : row0 + wm * 16 + r, mB = C::kN8 ? p.M : mA + 8;
  const bool vA = mA < p.M, vB = mB < p.M;
  const int64_t sA = C::kN8 ? row0 + 2 * cq : mA, sB = C::kN8 ? sA + 1 : mB;
  uint32_t qa[NKS][4];
  if (warp < C::kCons) {
    const int64_t offA = (q_row0 + mA) * D, offB = (q_row0 + mB) * D;
    auto load_q = [&](auto tag) {
      using QT = decltype(tag);
      float2 va[NKS][2], vb[NKS][2];
#pragma unroll
      for (int ks = 0; ks < NKS; ++ks) {
        int d0, d1;  // first d of the low / high k pair of this thread in k-step ks
        if (C::kI8) {
          d0 = 32 * cq + 4 * ks;
          d1 = d0 + 2;
        } else {
          d0 = 16 * ks + 2 * cq;
          d1 = d0 + 8;
        }
        va[ks][0] = vA ? load_pair<QT>(p.q, offA + d0) : make_float2(0.f, 0.f);
        va[ks][1] = vA ? load_pair<QT>(p.q, offA + d1) : make_float2(0.f, 0.f);
        vb[ks][0] = vB ? load_pair<QT>(p.q, offB + d0) : make_float2(0.f, 0.f);
        vb[ks][1] = vB ? load_pair<QT>(p.q, offB + d1) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int ks = 0; ks < NKS; ++ks) {
        qa[ks][0] = pack2<MmaT>(va[ks][0].x, va[ks][0].y);
        qa[ks][1] = pack2<MmaT>(vb[ks][0].x, vb[ks][0].y);
        qa[ks][2] = pack2<MmaT>(va[ks][1].x, va[ks][1].y);
        qa[ks][3] = pack2<MmaT>(vb[ks][1].x, vb[ks][1].y);
      }
    };
    if (p.q_dtype == NVM_F32)
      load_q(float{});
    else if (p.q_dtype == NVM_F16)
      load_q(__half{});
    else
      load_q(__nv_bfloat16{});
  }
  // n8 tile, int8 pages: K enters the mma as int8 + 1152 (the byte-permute alone, exact in
  // f16), so every score carries 1152 * sum_d q[row][d] too; this lane's two rows'
  // corrections (rows 2cq, 2cq+1), from the f16 q values the mma multiplies.
  float kbias0 = 0.f, kbias1 = 0.f;
  if constexpr (C::kN8 && C::kI8) {
    float qs = 0.f;  // this lane's share of row r: d = 32 cq + 4 ks + {0..3}
#pragma unroll
    for (int ks = 0; ks < NKS; ++ks) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][0]));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][2]));
      qs += (a.x + a.y) + (b.x + b.y);
    }
    qs += __shfl_xor_sync(0xffffffffu, qs, 1);
    qs += __shfl_xor_sync(0xffffffffu, qs, 2);  // row r's sum on all four lanes of row r
    kbias0 = 1152.f * __shfl_sync(0xffffffffu, qs, 4 * (2 * cq));
    kbias1 = 1152.f * __shfl_sync(0xffffffffu, qs, 4 * (2 * cq + 1));
  }
  if (warp == (C::kSelfFeed ? 0 : C::kCons)) {
    // The chunk's block-table entries, read together with (not after) the context
    // length: the row holds mp entries, so entries past the context are in bounds and
    // simply never used.  All loads are issued before any is consumed.
    int64_t n_tab = (cap + 15) / 16 - t_begin;
    if (n_tab > p.ct) n_tab = p.ct;
    constexpr int kPer = kMaxChunkTiles / 32;
    int64_t pv[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = lane + 32 * j;
      pv[j] = -1;
      if (i < n_tab) {
        const uint32_t tile = (uint32_t)(t_begin + i);
        pv[j] = p.block_table ? (int64_t)__ldg(&p.block_table[b * p.mp + (tpp == 1 ? tile : tile / tpp)]) : b;
      }
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = lane + 32 * j;
      if (i < n_tab) tile_pid[i] = (pv[j] >= 0 && pv[j] < p.P) ? (int)pv[j] : -1;
    }
  }
  __syncthreads();

  int64_t need_keys = ctx_limit;
  if (p.causal) {
    const bool spans = rows_here >= p.L || (int64_t)((uint32_t)row0 % (uint32_t)p.L) + rows_here > p.L;
    const int64_t lmax = spans ? p.L - 1 : (int64_t)((uint32_t)(row0 + rows_here - 1) % (uint32_t)p.L);
    const int64_t lim = lmax + ctx - p.L + 1;
    if (lim < need_keys) need_keys = lim;
  }
  if (ctx <= 0 || need_keys < 0) need_keys = 0;
  const int64_t n_tiles = (need_keys + 15) / 16;
  const int64_t n_chunks = n_tiles > 0 ? (int64_t)((uint32_t)(n_tiles + p.ct - 1) / (uint32_t)p.ct) : 1;
  // A chunk past this unit's keys has nothing to do; inside a cluster it still takes
  // part in the cluster barriers of the merge (with no tiles), so it does not return.
  if (c >= n_chunks && !(C::kClusterFits && p.cluster)) return;
  int64_t n_left = n_tiles - t_begin;
  if (n_left > p.ct) n_left = p.ct;
  const int n_my = n_left > 0 ? (int)n_left : 0;

  // One ring stage's loads (tile i of the chunk into stage i % NS), by one thread.
  auto issue_tile = [&](int i) {
    const int s = i % NS;
    const int pid = tile_pid[i];
    stage_valid[s] = pid >= 0 ? 1 : 0;
    if (pid >= 0) {
      const uint32_t tile = (uint32_t)(t_begin + i);
      const int slot0 = p.block_table ? (tpp == 1 ? 0 : (int)((tile % tpp) * 16)) : (int)(((t_begin + i) * 16) % p.ps);
      uint8_t* st = smem + s * C::kStageBytes;
      mbar_arrive_expect_tx(&full[s], 2 * C::kTileBytes + (C::kI8 ? 64 : 0));
#pragma unroll
      for (int hb = 0; hb < C::kBoxes; ++hb) {
        tma_load_4d(st + hb * 2048, &tm_k, hb * C::kBoxElems, slot0, (int)h, pid, &full[s]);
        tma_load_4d(st + C::kTileBytes + hb * 2048, &tm_v, hb * C::kBoxElems, slot0, (int)h, pid, &full[s]);
      }
      if (C::kI8) {
        tma_load_3d(st + 2 * C::kTileBytes, &tm_ks, slot0, (int)h, pid, &full[s]);
        tma_load_3d(st + 2 * C::kTileBytes + 128, &tm_vs, slot0, (int)h, pid, &full[s]);
      }
    } else {
      mbar_arrive(&full[s]);
    }
  };

  // ------------------------------------------------------------------ producer
  if constexpr (!C::kSelfFeed) {
    if (warp == C::kCons) {
      if (lane == 0) {
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        if (C::kI8) {
          prefetch_tmap(&tm_ks);
          prefetch_tmap(&tm_vs);
        }
        int issued = 0;
        for (int i = 0; i < n_my; ++i) {
          const int s = i % NS;
          if (i >= NS && !mbar_wait(&empty[s], ((i / NS) & 1) ^ 1)) {
            record_error(p.err, kDevErrEmptyWait);
            break;
          }
          issue_tile(i);
          issued = i + 1;
        }
        // Drain: the last use of every stage must have landed before the CTA can exit.
        for (int s = 0; s < NS && s < issued; ++s) {
          const int last = s + ((issued - 1 - s) / NS) * NS;
          if (!mbar_wait(&full[s], (last / NS) & 1)) record_error(p.err, kDevErrDrainWait);
        }
      }
      return;
    }
  }
  int last_issued = -1;  // self-feed: the highest tile this warp has issued (lane 0)
  if constexpr (C::kSelfFeed) {
    // each consumer warp fills its own first stages
    if (lane == 0) {
      if (warp == 0) {
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        prefetch_tmap(&tm_ks);
        prefetch_tmap(&tm_vs);
      }
      for (int i = warp; i < n_my && i < NS; i += NWK) {
        issue_tile(i);
        last_issued = i;
      }
    }
    __syncwarp();
  }

  // ------------------------------------------------------------------ consumers

  // Inclusive last visible key of each row (rows past M never mask anything).
  const int64_t BIG = INT64_MAX / 4;
  int64_t limA = BIG, limB = BIG;
  if (p.causal) {
    if (sA < p.M) limA = (int64_t)((uint32_t)sA % (uint32_t)p.L) + ctx - p.L;
    if (sB < p.M) limB = (int64_t)((uint32_t)sB % (uint32_t)p.L) + ctx - p.L;
  }
  // Keys below `clean` are visible to every real row of this warp: no masking there.
  int64_t clean = ctx_limit;
  {
    int64_t mn = limA < limB ? limA : limB;
    mn = mn + 1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t x = __shfl_xor_sync(0xffffffffu, mn, o);
      mn = x < mn ? x : mn;
    }
    if (mn < clean) clean = mn;
  }

  float mrA = -INFINITY, mrB = -INFINITY, lA = 0.f, lB = 0.f;
  float o[NDT][4];
#pragma unroll
  for (int i = 0; i < NDT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  bool timed_out = false;
  for (int i = wk; i < n_my; i += NWK) {
    const int s = i % NS;
    if (!mbar_wait(&full[s], (i / NS) & 1)) {
      record_error(p.err, kDevErrFullWait);
      timed_out = true;
      break;
    }
    if (stage_valid[s]) {
      if constexpr (C::kN8) {
      const int64_t tok0 = (t_begin + i) * 16;
      const uint32_t kt = smem_u32(smem + s * C::kStageBytes);
      const uint32_t vt = kt + C::kTileBytes;
      // S^T = K Q^T (16 keys x 8 rows).  16-bit pages: the k-steps go round-robin into
      // four independent accumulator chains (the mma.sync result latency, not issue,
      // bounds a warp walking its tiles); int8 pages (issue-bound): two chains.
      constexpr int kQc = C::kI8 ? 2 : 4;
      float sacc[kQc][4];
#pragma unroll
      for (int q2 = 0; q2 < kQc; ++q2) sacc[q2][0] = sacc[q2][1] = sacc[q2][2] = sacc[q2][3] = 0.f;
      if constexpr (!C::kI8) {
        const int mi = lane >> 3;
        const int ktok = (mi >> 1) * 8 + (lane & 7);
#pragma unroll
        for (int ks = 0; ks < NKS; ++ks) {
          uint32_t k0, k1, k2, k3;
          ldsm_x4(swz(kt, ktok, 2 * ks + (mi & 1)), k0, k1, k2, k3);
          const uint32_t a[4] = {k0, k2, k1, k3};
          mma16816<MmaT>(sacc[ks % kQc], a, qa[ks][0], qa[ks][2]);
        }
      } else {
        // keys r and r + 8, bytes [32 cq, 32 cq + 32) of each (the k dimension is
        // permuted identically in Q: k pair (2cq, 2cq+1) <-> d 32cq + 4ks + {0,1},
        // k pair (2cq+8, 2cq+9) <-> d 32cq + 4ks + {2,3})
        uint32_t kw[2][8];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int tok = hf * 8 + r;
          lds128(swz(kt, tok, 2 * cq), kw[hf][0], kw[hf][1], kw[hf][2], kw[hf][3]);
          lds128(swz(kt, tok, 2 * cq + 1), kw[hf][4], kw[hf][5], kw[hf][6], kw[hf][7]);
        }
#pragma unroll
        for (int ks = 0; ks < NKS; ++ks) {
          const uint32_t x0 = kw[0][ks] ^ 0x80808080u, x1 = kw[1][ks] ^ 0x80808080u;
          // f16 value 1024 + (byte ^ 0x80) = int8 + 1152 (the bias is removed below)
          const uint32_t a[4] = {prmt(x0, 0x64646464u, 0x4140u), prmt(x1, 0x64646464u, 0x4140u),
                                 prmt(x0, 0x64646464u, 0x4342u), prmt(x1, 0x64646464u, 0x4342u)};
          mma16816<MmaT>(sacc[ks & 1], a, qa[ks][0], qa[ks][2]);
        }
      }
      // sv[0] = (key r, row 2cq), [1] = (key r, row 2cq+1), [2] = (key r+8, row 2cq), [3] = (key r+8, row 2cq+1)
      float sv[4];
      if constexpr (C::kI8) {
        // the +1152 bias of K removed per row, then each key's scale
        const ScaleT* ksp = reinterpret_cast<const ScaleT*>(smem + s * C::kStageBytes + 2 * C::kTileBytes);
        const float k0 = to_f32(ksp[r]), k1 = to_f32(ksp[r + 8]);
        sv[0] = ((sacc[0][0] + sacc[1][0]) - kbias0) * k0;
        sv[1] = ((sacc[0][1] + sacc[1][1]) - kbias1) * k0;
        sv[2] = ((sacc[0][2] + sacc[1][2]) - kbias0) * k1;
        sv[3] = ((sacc[0][3] + sacc[1][3]) - kbias1) * k1;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if constexpr (kQc == 4)
            sv[e] = (sacc[0][e] + sacc[1][e]) + (sacc[2][e] + sacc[3][e]);
          else
            sv[e] = sacc[0][e] + sacc[1][e];
        }
      }
      const bool need_mask = tok0 + 16 > clean;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = sv[e] * p.scale_log2;
        if (need_mask) {
          const int64_t tok = tok0 + r + 8 * (e >> 1);
          const int64_t lim = (e & 1) ? limB : limA;
          if (tok >= ctx_limit || tok > lim) v = -INFINITY;
        }
        sv[e] = v;
      }
      // row max over the 16 keys: two in the thread, the rest across r (lanes xor 4, 8, 16)
      float mxA = fmaxf(sv[0], sv[2]), mxB = fmaxf(sv[1], sv[3]);
#pragma unroll
      for (int o2 = 4; o2 < 32; o2 <<= 1) {
        mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, o2));
        mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, o2));
      }
      const float mnA = fmaxf(mrA, mxA), mnB = fmaxf(mrB, mxB);
      const float muA = mnA == -INFINITY ? 0.f : mnA, muB = mnB == -INFINITY ? 0.f : mnB;
      const float alA = ex2_ftz(mrA - muA), alB = ex2_ftz(mrB - muB);
      const bool moved = mrA != mnA || mrB != mnB;
      mrA = mnA;
      mrB = mnB;
      sv[0] = ex2_ftz(sv[0] - muA);
      sv[1] = ex2_ftz(sv[1] - muB);
      sv[2] = ex2_ftz(sv[2] - muA);
      sv[3] = ex2_ftz(sv[3] - muB);
      lA = lA * alA + (sv[0] + sv[2]);
      lB = lB * alB + (sv[1] + sv[3]);
      if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
        for (int j = 0; j < D / 16; ++j) {
          o[j][0] *= alA;
          o[j][1] *= alB;
          o[j][2] *= alA;
          o[j][3] *= alB;
        }
      }
      // P^T as the B operand (keys x rows): each 8 x 8 quadrant of P^T's accumulator
      // layout transposed in registers.  int8 pages: each key's value scale multiplies its
      // P entries here (keys r and r + 8 of this lane), so V enters the mma unscaled.
      if constexpr (C::kI8) {
        const ScaleT* vsp = reinterpret_cast<const ScaleT*>(smem + s * C::kStageBytes + 2 * C::kTileBytes + 128);
        const float v0 = to_f32(vsp[r]), v1 = to_f32(vsp[r + 8]);
        sv[0] *= v0;
        sv[1] *= v0;
        sv[2] *= v1;
        sv[3] *= v1;
      }
      uint32_t pb[2], pbl[2];
      pb[0] = movmatrix_t(pack2<MmaT>(sv[0], sv[1]));
      pb[1] = movmatrix_t(pack2<MmaT>(sv[2], sv[3]));
      if constexpr (C::kSplitP) {
        const uint32_t h0 = pack2<MmaT>(sv[0], sv[1]), h1 = pack2<MmaT>(sv[2], sv[3]);
        pbl[0] = movmatrix_t(pack_residual(sv[0], sv[1], h0));
        pbl[1] = movmatrix_t(pack_residual(sv[2], sv[3], h1));
      }
      // O^T += V^T P^T, one m16 tile of d per mma
      if constexpr (!C::kI8) {
        const int mi = lane >> 3;
        const int vtok = (mi & 1) * 8 + (lane & 7);
#pragma unroll
        for (int j = 0; j < D / 16; ++j) {
          uint32_t v0, v1, v2, v3;
          ldsm_x4_t(swz(vt, vtok, 2 * j + (mi >> 1)), v0, v1, v2, v3);
          const uint32_t a[4] = {v0, v2, v1, v3};
          mma16816<MmaT>(o[j], a, pb[0], pb[1]);
          if constexpr (C::kSplitP) mma16816<MmaT>(o[j], a, pbl[0], pbl[1]);
        }
      } else {
        // V rows 2cq, 2cq+1, 2cq+8, 2cq+9, bytes [16 r, 16 r + 16): tile j row r <-> d 16r + 2j,
        // row r + 8 <-> d 16r + 2j + 1
        uint32_t vw[4][4];
#pragma unroll
        for (int t4 = 0; t4 < 4; ++t4) {
          const int tok = 2 * cq + (t4 & 1) + (t4 >> 1) * 8;
          lds128(swz(vt, tok, r), vw[t4][0], vw[t4][1], vw[t4][2], vw[t4][3]);
        }
        // V enters unscaled (exact int8 -> f16); the value scales were folded into P^T
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const uint32_t y01 = prmt(vw[0][w], vw[1][w], 0x5140u) ^ 0x80808080u;
          const uint32_t y23 = prmt(vw[0][w], vw[1][w], 0x7362u) ^ 0x80808080u;
          const uint32_t z01 = prmt(vw[2][w], vw[3][w], 0x5140u) ^ 0x80808080u;
          const uint32_t z23 = prmt(vw[2][w], vw[3][w], 0x7362u) ^ 0x80808080u;
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const uint32_t y = jj ? y23 : y01, z = jj ? z23 : z01;
            const uint32_t a[4] = {i8pair_to_f16x2(y, 0x4140u), i8pair_to_f16x2(y, 0x4342u),
                                   i8pair_to_f16x2(z, 0x4140u), i8pair_to_f16x2(z, 0x4342u)};
            mma16816<MmaT>(o[2 * w + jj], a, pb[0], pb[1]);
          }
        }
      }
      } else {
      const int64_t tok0 = (t_begin + i) * 16;
      const uint32_t kt = smem_u32(smem + s * C::kStageBytes);
      const uint32_t vt = kt + C::kTileBytes;
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;

      if constexpr (!C::kI8) {
        // two accumulator sets (even / odd k-steps) halve the dependent mma chain
        float sd[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) sd[nt][0] = sd[nt][1] = sd[nt][2] = sd[nt][3] = 0.f;
        const int mi = lane >> 3;
        const int ktok = (mi >> 1) * 8 + (lane & 7);
#pragma unroll
        for (int ks = 0; ks < NKS; ++ks) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(swz(kt, ktok, 2 * ks + (mi & 1)), b0, b1, b2, b3);
          if (ks & 1) {
            mma16816<MmaT>(sd[0], qa[ks], b0, b1);
            mma16816<MmaT>(sd[1], qa[ks], b2, b3);
          } else {
            mma16816<MmaT>(sc[0], qa[ks], b0, b1);
            mma16816<MmaT>(sc[1], qa[ks], b2, b3);
          }
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[nt][e] += sd[nt][e];
      } else {
        uint32_t kw[2][8];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int tok = nt * 8 + r;
          lds128(swz(kt, tok, 2 * cq), kw[nt][0], kw[nt][1], kw[nt][2], kw[nt][3]);
          lds128(swz(kt, tok, 2 * cq + 1), kw[nt][4], kw[nt][5], kw[nt][6], kw[nt][7]);
        }
#pragma unroll
        for (int ks = 0; ks < NKS; ++ks) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const uint32_t x = kw[nt][ks] ^ 0x80808080u;
            mma16816<MmaT>(sc[nt], qa[ks], i8pair_to_f16x2(x, 0x4140u), i8pair_to_f16x2(x, 0x4342u));
          }
        }
        const ScaleT* ksp = reinterpret_cast<const ScaleT*>(smem + s * C::kStageBytes + 2 * C::kTileBytes);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const float k0 = to_f32(ksp[nt * 8 + 2 * cq]), k1 = to_f32(ksp[nt * 8 + 2 * cq + 1]);
          sc[nt][0] *= k0;
          sc[nt][1] *= k1;
          sc[nt][2] *= k0;
          sc[nt][3] *= k1;
        }
      }

      // scale, mask, online softmax (base 2)
      const bool need_mask = tok0 + 16 > clean;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = sc[nt][e] * p.scale_log2;
          if (need_mask) {
            const int64_t tok = tok0 + nt * 8 + 2 * cq + (e & 1);
            const int64_t lim = e < 2 ? limA : limB;
            if (tok >= ctx_limit || tok > lim) v = -INFINITY;
          }
          sc[nt][e] = v;
        }
      }
      float mxA = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
      float mxB = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
      mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
      mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
      mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
      mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
      const float mnA = fmaxf(mrA, mxA), mnB = fmaxf(mrB, mxB);
      const float muA = mnA == -INFINITY ? 0.f : mnA, muB = mnB == -INFINITY ? 0.f : mnB;
      // 2^x on the MUFU unit (ex2.approx.ftz: 2 ulp, -inf -> +0)
      const float alA = ex2_ftz(mrA - muA), alB = ex2_ftz(mrB - muB);
      const bool moved = mrA != mnA || mrB != mnB;  // a row max changed: O needs rescaling
      mrA = mnA;
      mrB = mnB;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        sc[nt][0] = ex2_ftz(sc[nt][0] - muA);
        sc[nt][1] = ex2_ftz(sc[nt][1] - muA);
        sc[nt][2] = ex2_ftz(sc[nt][2] - muB);
        sc[nt][3] = ex2_ftz(sc[nt][3] - muB);
      }
      lA = lA * alA + (sc[0][0] + sc[0][1] + sc[1][0] + sc[1][1]);
      lB = lB * alB + (sc[0][2] + sc[0][3] + sc[1][2] + sc[1][3]);
      // alpha is exactly 1 for rows whose max did not move (and for rows without a key
      // yet, whose O is 0): skipping the multiply then changes nothing
      if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
        for (int i2 = 0; i2 < NDT; ++i2) {
          o[i2][0] *= alA;
          o[i2][1] *= alA;
          o[i2][2] *= alB;
          o[i2][3] *= alB;
        }
      }
      uint32_t pa[4], pl[4];
      pa[0] = pack2<MmaT>(sc[0][0], sc[0][1]);
      pa[1] = pack2<MmaT>(sc[0][2], sc[0][3]);
      pa[2] = pack2<MmaT>(sc[1][0], sc[1][1]);
      pa[3] = pack2<MmaT>(sc[1][2], sc[1][3]);
      if constexpr (C::kSplitP) {
        // bf16 keeps 8 mantissa bits; the residual p - bf16(p) is a second bf16
        // operand so P reaches the tensor core with ~16 bits.
        pl[0] = pack_residual(sc[0][0], sc[0][1], pa[0]);
        pl[1] = pack_residual(sc[0][2], sc[0][3], pa[1]);
        pl[2] = pack_residual(sc[1][0], sc[1][1], pa[2]);
        pl[3] = pack_residual(sc[1][2], sc[1][3], pa[3]);
      }

      if constexpr (!C::kI8) {
        const int mi = lane >> 3;
        const int vtok = (mi & 1) * 8 + (lane & 7);
#pragma unroll
        for (int j = 0; j < D / 16; ++j) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(swz(vt, vtok, 2 * j + (mi >> 1)), b0, b1, b2, b3);
          mma16816<MmaT>(o[2 * j], pa, b0, b1);
          mma16816<MmaT>(o[2 * j + 1], pa, b2, b3);
          if constexpr (C::kSplitP) {
            mma16816<MmaT>(o[2 * j], pl, b0, b1);
            mma16816<MmaT>(o[2 * j + 1], pl, b2, b3);
          }
        }
      } else {
        uint32_t vw[4][4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int tok = 2 * cq + (t & 1) + (t >> 1) * 8;
          lds128(swz(vt, tok, r), vw[t][0], vw[t][1], vw[t][2], vw[t][3]);
        }
        const ScaleT* vsp = reinterpret_cast<const ScaleT*>(smem + s * C::kStageBytes + 2 * C::kTileBytes + 128);
        const __half2 vlo = __floats2half2_rn(to_f32(vsp[2 * cq]), to_f32(vsp[2 * cq + 1]));
        const __half2 vhi = __floats2half2_rn(to_f32(vsp[2 * cq + 8]), to_f32(vsp[2 * cq + 9]));
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const uint32_t y01 = prmt(vw[0][w], vw[1][w], 0x5140u) ^ 0x80808080u;
          const uint32_t y23 = prmt(vw[0][w], vw[1][w], 0x7362u) ^ 0x80808080u;
          const uint32_t z01 = prmt(vw[2][w], vw[3][w], 0x5140u) ^ 0x80808080u;
          const uint32_t z23 = prmt(vw[2][w], vw[3][w], 0x7362u) ^ 0x80808080u;
          const uint32_t ys[4] = {y01, y01, y23, y23};
          const uint32_t zs[4] = {z01, z01, z23, z23};
#pragma unroll
          for (int i2 = 0; i2 < 4; ++i2) {
            const uint32_t sel = (i2 & 1) ? 0x4342u : 0x4140u;
            uint32_t lo = i8pair_to_f16x2(ys[i2], sel), hi = i8pair_to_f16x2(zs[i2], sel);
            __half2 lo2 = __hmul2(*reinterpret_cast<__half2*>(&lo), vlo);
            __half2 hi2 = __hmul2(*reinterpret_cast<__half2*>(&hi), vhi);
            mma16816<MmaT>(o[4 * w + i2], pa, *reinterpret_cast<uint32_t*>(&lo2), *reinterpret_cast<uint32_t*>(&hi2));
          }
        }
      }
          }
    }
    __syncwarp();
    if constexpr (C::kSelfFeed) {
      // the stage's shared-memory reads are done: refill it with the warp's next tile
      if (lane == 0 && i + NS < n_my) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue_tile(i + NS);
        last_issued = i + NS;
      }
    } else {
      if (lane == 0) mbar_arrive(&empty[(i % NS)]);
    }
  }
  if constexpr (C::kSelfFeed) {
    // after a timed-out wait, loads this warp issued may still be landing in its stages
    if (timed_out && lane == 0) {
      for (int s = wk; s < NS && s <= last_issued; s += NWK) {
        const int last = s + ((last_issued - s) / NS) * NS;  // last tile issued into stage s
        if (!mbar_wait(&full[s], (last / NS) & 1)) record_error(p.err, kDevErrDrainWait);
      }
    }
  }
  // A consumer that timed out still joins the epilogue barriers below (so no other
  // warp waits forever); its rows carry garbage and the error word is set.
  (void)timed_out;

  if constexpr (C::kN8) {
    // row sums: partial over this thread's keys, reduced across r
#pragma unroll
    for (int o2 = 4; o2 < 32; o2 <<= 1) {
      lA += __shfl_xor_sync(0xffffffffu, lA, o2);
      lB += __shfl_xor_sync(0xffffffffu, lB, o2);
    }
  } else {
    lA += __shfl_xor_sync(0xffffffffu, lA, 1);
    lA += __shfl_xor_sync(0xffffffffu, lA, 2);
    lB += __shfl_xor_sync(0xffffffffu, lB, 1);
    lB += __shfl_xor_sync(0xffffffffu, lB, 2);
  }

  // ------------------------------------------------------------------ epilogue
  constexpr int NCT = C::kCons * 32;
  named_barrier(1, NCT);  // every consumer is done with the ring; reuse it
  float* eo = reinterpret_cast<float*>(smem);  // [NWK][RB][D]
  float* em = eo + NWK * C::kRB * D;            // [NWK][RB]
  float* el = em + NWK * C::kRB;                // [NWK][RB]
  if constexpr (C::kN8) {
    const int rlA = 2 * cq, rlB = rlA + 1;
#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = C::kI8 ? 16 * r + 2 * j + (e >> 1) : 16 * j + 8 * (e >> 1) + r;
        const int rl = (e & 1) ? rlB : rlA;
        eo[(wk * C::kRB + rl) * D + d] = o[j][e];
      }
    }
    if (r == 0) {
      em[wk * C::kRB + rlA] = mrA;
      el[wk * C::kRB + rlA] = lA;
      em[wk * C::kRB + rlB] = mrB;
      el[wk * C::kRB + rlB] = lB;
    }
  } else {
    const int rlA = wm * 16 + r, rlB = rlA + 8;
#pragma unroll
    for (int nd = 0; nd < NDT; ++nd) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = C::kI8 ? (32 * cq + 16 * (e & 1) + nd) : (nd * 8 + 2 * cq + (e & 1));
        const int rl = e < 2 ? rlA : rlB;
        eo[(wk * C::kRB + rl) * D + d] = o[nd][e];
      }
    }
    if (cq == 0) {
      em[wk * C::kRB + rlA] = mrA;
      el[wk * C::kRB + rlA] = lA;
      em[wk * C::kRB + rlB] = mrB;
      el[wk * C::kRB + rlB] = lB;
    }
  }
  named_barrier(1, NCT);
  const int tid = threadIdx.x;
  if constexpr (C::kClusterFits) {
    if (p.cluster) {
      // Split-K inside a thread-block cluster: the unit's chunks are CTAs 0 .. n_chunks-1
      // of one cluster (cluster rank == chunk index).  Each leaves its combined partial
      // rows (O, m, l) in its own shared memory; chunk 0 merges them over distributed
      // shared memory with the same operations, in the same chunk order, as the
      // workspace merge below.  Every CTA of the cluster, with or without keys, reaches
      // both cluster barriers; the second one keeps the partials alive until read.
      namespace cg = cooperative_groups;
      cg::cluster_group cluster = cg::this_cluster();
      float* cb_o = reinterpret_cast<float*>(smem + C::kClusterOff);  // [kRB][D]
      float2* cb_ml = reinterpret_cast<float2*>(cb_o + C::kRB * D);   // [kRB]
      float* cw = reinterpret_cast<float*>(cb_ml + C::kRB);           // [8][kRB] chunk weights
      float* cwl = cw + 8 * C::kRB;                                   // [kRB]
      for (int64_t idx = tid; idx < rows_here * D; idx += NCT) {
        const int rl = (int)(idx / D), d = (int)(idx % D);
        float ms = -INFINITY;
#pragma unroll
        for (int w = 0; w < NWK; ++w) ms = fmaxf(ms, em[w * C::kRB + rl]);
        float ls = 0.f, os = 0.f;
#pragma unroll
        for (int w = 0; w < NWK; ++w) {
          const float mw = em[w * C::kRB + rl];
          if (mw != -INFINITY) {
            const float f = exp2f(mw - ms);
            ls += el[w * C::kRB + rl] * f;
            os += eo[(w * C::kRB + rl) * D + d] * f;
          }
        }
        cb_o[rl * D + d] = os;
        if (d == 0) cb_ml[rl] = make_float2(ms, ls);
      }
      cluster.sync();
      if (c == 0) {
        const int nc = (int)n_chunks;  // chunks of this unit that hold keys (<= cluster size)
        for (int rl = tid; rl < rows_here; rl += NCT) {
          float ms = -INFINITY;
          for (int cc = 0; cc < nc; ++cc) ms = fmaxf(ms, cluster.map_shared_rank(cb_ml, cc)[rl].x);
          float ls = 0.f;
          for (int cc = 0; cc < nc; ++cc) {
            const float2 ml = cluster.map_shared_rank(cb_ml, cc)[rl];
            float f = -1.f;
            if (ml.x != -INFINITY) {
              f = exp2f(ml.x - ms);
              ls += ml.y * f;
            }
            cw[cc * C::kRB + rl] = f;
          }
          cwl[rl] = ls;
        }
        named_barrier(1, NCT);
        for (int64_t g4 = tid; g4 < rows_here * (D / 4); g4 += NCT) {
          const int rl = (int)(g4 / (D / 4)), d = (int)(g4 % (D / 4)) * 4;
          float o4[4] = {0.f, 0.f, 0.f, 0.f};
          for (int cc = 0; cc < nc; ++cc) {
            const float f = cw[cc * C::kRB + rl];
            if (f >= 0.f) {
              const float4 v = *reinterpret_cast<const float4*>(cluster.map_shared_rank(cb_o + rl * D + d, cc));
              o4[0] += v.x * f;
              o4[1] += v.y * f;
              o4[2] += v.z * f;
              o4[3] += v.w * f;
            }
          }
          const float ls = cwl[rl];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            store_dyn(p.out, (q_row0 + row0 + rl) * D + d + e, p.out_dtype, ls > 0.f ? o4[e] / ls : 0.f);
        }
      }
      cluster.sync();
      return;
    }
  }
  const bool single = n_chunks == 1;
  const int64_t wsrow = (unit * p.n_chunks + c) * p.rows_real;
  for (int64_t idx = tid; idx < rows_here * D; idx += NCT) {
    const int rl = (int)(idx / D), d = (int)(idx % D);
    float ms = -INFINITY;
#pragma unroll
    for (int w = 0; w < NWK; ++w) ms = fmaxf(ms, em[w * C::kRB + rl]);
    float ls = 0.f, os = 0.f;
#pragma unroll
    for (int w = 0; w < NWK; ++w) {
      const float mw = em[w * C::kRB + rl];
      if (mw != -INFINITY) {
        const float f = exp2f(mw - ms);
        ls += el[w * C::kRB + rl] * f;
        os += eo[(w * C::kRB + rl) * D + d] * f;
      }
    }
    if (single) {
      store_dyn(p.out, (q_row0 + row0 + rl) * D + d, p.out_dtype, ls > 0.f ? os / ls : 0.f);
    } else {
      p.part_o[(wsrow + rl) * D + d] = os;
      if (d == 0) p.part_ml[wsrow + rl] = make_float2(ms, ls);
    }
  }
  if (single) return;

  // Split-K: the last CTA of this unit merges every chunk's partial result.
  __threadfence();
  named_barrier(1, NCT);
  if (tid == 0) {
    const int prev = atomicAdd(&p.counters[unit], 1);
    *s_flag = prev == (int)n_chunks - 1;
  }
  named_barrier(1, NCT);
  if (!*s_flag) return;
  __threadfence();
  const int64_t base = unit * p.n_chunks * p.rows_real;
  if ((2 * n_chunks + 1) * rows_here * (int64_t)sizeof(float) <= C::kMainBytes) {
    // Stage every chunk's (m, l) in shared memory with one parallel round of loads, turn
    // them into the log-sum-exp weights f = 2^(m_c - max m) (-1 marks a chunk without
    // keys), then sum the partial O rows with all chunk loads independent of one another.
    // Same operations in the same chunk order as the one-thread-per-element loop below.
    float* wm = reinterpret_cast<float*>(smem);  // [n_chunks][rows_here]: m, then the weight f
    float* wlc = wm + n_chunks * rows_here;      // [n_chunks][rows_here]: l
    float* wl = wlc + n_chunks * rows_here;      // [rows_here]: sum of l * f
    for (int64_t i = tid; i < n_chunks * rows_here; i += NCT) {
      const uint32_t cc32 = (uint32_t)i / (uint32_t)rows_here;
      const int64_t cc = cc32, rl = (int64_t)((uint32_t)i - cc32 * (uint32_t)rows_here);
      const float2 ml = __ldcg(&p.part_ml[base + cc * p.rows_real + rl]);
      wm[i] = ml.x;
      wlc[i] = ml.y;
    }
    named_barrier(1, NCT);
    for (int64_t rl = tid; rl < rows_here; rl += NCT) {
      float ms = -INFINITY;
      for (int64_t cc = 0; cc < n_chunks; ++cc) ms = fmaxf(ms, wm[cc * rows_here + rl]);
      float ls = 0.f;
      for (int64_t cc = 0; cc < n_chunks; ++cc) {
        const float mc = wm[cc * rows_here + rl];
        float f = -1.f;
        if (mc != -INFINITY) {
          f = exp2f(mc - ms);
          ls += wlc[cc * rows_here + rl] * f;
        }
        wm[cc * rows_here + rl] = f;
      }
      wl[rl] = ls;
    }
    named_barrier(1, NCT);
    // four consecutive d per thread (16-byte loads), eight chunks' loads in flight at once
    const int64_t cstride = p.rows_real * D;
    for (int64_t g4 = tid; g4 < rows_here * (D / 4); g4 += NCT) {
      const int rl = (int)(g4 / (D / 4)), d = (int)(g4 % (D / 4)) * 4;
      const float* po = p.part_o + (base + rl) * D + d;
      float os[4] = {0.f, 0.f, 0.f, 0.f};
      for (int64_t cc = 0; cc < n_chunks; cc += 8) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          v[j] = cc + j < n_chunks ? __ldcg(reinterpret_cast<const float4*>(po + (cc + j) * cstride))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (cc + j >= n_chunks) break;
          const float f = wm[(cc + j) * rows_here + rl];
          if (f >= 0.f) {
            os[0] += v[j].x * f;
            os[1] += v[j].y * f;
            os[2] += v[j].z * f;
            os[3] += v[j].w * f;
          }
        }
      }
      const float ls = wl[rl];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        store_dyn(p.out, (q_row0 + row0 + rl) * D + d + e, p.out_dtype, ls > 0.f ? os[e] / ls : 0.f);
    }
    if (tid == 0) p.counters[unit] = 0;
    return;
  }
  for (int64_t idx = tid; idx < rows_here * D; idx += NCT) {
    const int rl = (int)(idx / D), d = (int)(idx % D);
    float ms = -INFINITY;
    for (int64_t cc = 0; cc < n_chunks; ++cc) ms = fmaxf(ms, __ldcg(&p.part_ml[base + cc * p.rows_real + rl].x));
    float ls = 0.f, os = 0.f;
    for (int64_t cc = 0; cc < n_chunks; ++cc) {
      const float2 ml = __ldcg(&p.part_ml[base + cc * p.rows_real + rl]);
      if (ml.x != -INFINITY) {
        const float f = exp2f(ml.x - ms);
        ls += ml.y * f;
        os += __ldcg(&p.part_o[(base + cc * p.rows_real + rl) * D + d]) * f;
      }
    }
    store_dyn(p.out, (q_row0 + row0 + rl) * D + d, p.out_dtype, ls > 0.f ? os / ls : 0.f);
  }
  if (tid == 0) p.counters[unit] = 0;
}

int64_t env_int(const char* name, int64_t dflt) {
  const char* v = std::getenv(name);
  if (v == nullptr || v[0] == '\0') return dflt;
  return std::atoll(v);
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Opts one kernel instance into its dynamic shared memory, once per device.
template <typename KvT, typename ScaleT, int D, int NWM, int NWK, int NS_>
int ensure_smem_attr() {
  using C = Cfg<KvT, D, NWM, NWK, NS_>;
  static std::mutex mu;
  static uint64_t done_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    int st = check_cuda(cudaFuncSetAttribute(paged_mma_kernel<KvT, ScaleT, D, NWM, NWK, NS_>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes),
                        "paged_attention: cudaFuncSetAttribute");
    if (st != NVM_OK) return st;
    done_mask |= 1ull << dev;
  }
  return NVM_OK;
}

// CTAs of one n8 kernel instance resident on an SM (registers and shared memory), asked
// of the runtime once; without a device (workspace sizing on a host) the shared-memory
// bound, at most 8 (the register bound of the instances built here: <= 128 a thread).
template <typename KvT, typename ScaleT, int D, int NWK, int NS_>
int n8_resident() {
  using C = Cfg<KvT, D, 0, NWK, NS_>;
  static std::atomic<int> cached{0};
  int n = cached.load(std::memory_order_relaxed);
  if (n > 0) return n;
  n = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || ensure_smem_attr<KvT, ScaleT, D, 0, NWK, NS_>() != NVM_OK ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, paged_mma_kernel<KvT, ScaleT, D, 0, NWK, NS_>, C::kThreads,
                                                    C::kSmemBytes) != cudaSuccess ||
      n <= 0) {
    cudaGetLastError();
    n = 233472 / (C::kSmemBytes + 1024);
    n = n < 1 ? 1 : (n > 8 ? 8 : n);
    return n;  // not cached: a later call with a device asks the runtime
  }
  cached.store(n, std::memory_order_relaxed);
  return n;
}

template <typename KvT, typename ScaleT, int D>
int n8_resident_variant(int variant) {
  switch (variant) {  // the (NWK, NS) of each variant, as launch_decode maps them
    case 0: return n8_resident<KvT, ScaleT, D, 4, 0>();
    case 1: return n8_resident<KvT, ScaleT, D, 4, 12>();
    case 2: return n8_resident<KvT, ScaleT, D, 2, 2>();
    case 4: return n8_resident<KvT, ScaleT, D, 2, 8>();
    case 5: return n8_resident<KvT, ScaleT, D, 4, 4>();
    case 6: return n8_resident<KvT, ScaleT, D, 1, 4>();
    case 7: return n8_resident<KvT, ScaleT, D, 2, 4>();
    case 8: return n8_resident<KvT, ScaleT, D, 1, 6>();
    default: return n8_resident<KvT, ScaleT, D, 2, 6>();
  }
}

int n8_resident_per_sm(const PagedArgs& a, int variant) {
  if (a.kv_dtype == NVM_I8) return n8_resident_variant<int8_t, __half, 128>(variant);
  if (a.kv_dtype == NVM_F16)
    return a.D == 64 ? n8_resident_variant<__half, __half, 64>(variant) : n8_resident_variant<__half, __half, 128>(variant);
  return a.D == 64 ? n8_resident_variant<__nv_bfloat16, __nv_bfloat16, 64>(variant)
                   : n8_resident_variant<__nv_bfloat16, __nv_bfloat16, 128>(variant);
}

int sm_count_cached() {
  static std::atomic<int> cached{0};
  int n = cached.load(std::memory_order_relaxed);
  if (n > 0) return n;
  int dev = 0;
  n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      n <= 0) {
    cudaGetLastError();
    return 148;
  }
  cached.store(n, std::memory_order_relaxed);
  return n;
}

template <typename KvT, typename ScaleT, int D, int NWM, int NWK, int NS_ = 0>
int launch_cfg(const PagedArgs& a, const MmaPlan& plan, void* ws, cudaStream_t s) {
  using C = Cfg<KvT, D, NWM, NWK, NS_>;
  auto kern = paged_mma_kernel<KvT, ScaleT, D, NWM, NWK, NS_>;
  {
    const int st = ensure_smem_attr<KvT, ScaleT, D, NWM, NWK, NS_>();
    if (st != NVM_OK) return st;
  }
  // Tensor maps: pools [P, Hkv, ps, D] -> dims (D, ps, Hkv, P); scales [P, Hkv, ps] -> (ps, Hkv, P).
  const CUtensorMapDataType dt = C::kI8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                        : (std::is_same<KvT, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                            : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  const uint64_t e = sizeof(KvT);
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)a.page_size, (uint64_t)a.Hkv, (uint64_t)a.P};
  const uint64_t strides[3] = {D * e, (uint64_t)a.page_size * D * e, (uint64_t)(a.Hkv * a.page_size) * D * e};
  const uint32_t box[4] = {(uint32_t)C::kBoxElems, 16u, 1u, 1u};
  CUtensorMap tk, tv, tks, tvs;
  int st = encode_tmap(&tk, dt, 4, a.k_pages, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVM_OK) return st;
  st = encode_tmap(&tv, dt, 4, a.v_pages, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVM_OK) return st;
  if (C::kI8) {
    const CUtensorMapDataType sdt =
        std::is_same<ScaleT, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint64_t sdims[3] = {(uint64_t)a.page_size, (uint64_t)a.Hkv, (uint64_t)a.P};
    const uint64_t sstr[2] = {(uint64_t)a.page_size * 2, (uint64_t)(a.Hkv * a.page_size) * 2};
    const uint32_t sbox[3] = {16u, 1u, 1u};
    st = encode_tmap(&tks, sdt, 3, a.k_scales, sdims, sstr, sbox, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != NVM_OK) return st;
    st = encode_tmap(&tvs, sdt, 3, a.v_scales, sdims, sstr, sbox, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != NVM_OK) return st;
  } else {
    tks = tk;
    tvs = tv;
  }
  MmaParams p{};
  p.q = a.q; p.out = a.out; p.block_table = a.block_table; p.context_lens = a.context_lens;
  if (plan.ws_bytes > 0) {
    char* w = static_cast<char*>(ws);
    p.counters = reinterpret_cast<int*>(w);
    w += kCounterBytes;
    p.part_ml = reinterpret_cast<float2*>(w);
    w += align256(plan.n_units * plan.n_chunks * plan.rows_real * sizeof(float2));
    p.part_o = reinterpret_cast<float*>(w);
  }
  p.err = device_error_word();
  p.q_dtype = a.q_dtype; p.out_dtype = a.out_dtype;
  p.B = a.B; p.Hq = a.Hq; p.Hkv = a.Hkv; p.L = a.L; p.P = a.P; p.ps = a.page_size; p.mp = a.max_pages;
  p.dense_ctx = a.dense_ctx;
  p.g = a.Hq / a.Hkv; p.M = p.g * a.L;
  p.n_rb = plan.n_row_blocks; p.rows_real = plan.rows_real; p.ct = plan.chunk_tiles; p.n_chunks = plan.n_chunks;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.causal = a.is_causal;
  p.cluster = 0;
  const dim3 grid((unsigned)plan.n_units, (unsigned)plan.n_chunks);
  if (plan.cluster && C::kClusterFits && plan.n_chunks > 1 && plan.n_chunks <= 8) {
    p.cluster = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(C::kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)plan.n_chunks;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, kern, tk, tv, tks, tvs, p),
                      "paged_attention: tensor-core kernel launch (cluster)");
  }
  if (plan.cluster) return fail(NVM_ERR_UNSUPPORTED, "paged_attention: cluster plan for a kernel without it");
  kern<<<grid, C::kThreads, C::kSmemBytes, s>>>(tk, tv, tks, tvs, p);
  return check_cuda(cudaGetLastError(), "paged_attention: tensor-core kernel launch");
}

// Kernel variants (consumer warps along keys NWK, stage depth NS) per shape class.
// Fewer warps and stages per CTA let more CTAs -- and more independent TMA
// producers -- share an SM, which keeps more page loads in flight: on B200 the
// 16-bit decode reached 98% of measured HBM bandwidth with 2 consumer warps and 6
// stages (4 CTAs per SM) against 64% with 4 warps and 8 stages (2 CTAs per SM).
// NVM_ATTN_DECODE_CFG selects another variant (for sweeps).
template <typename KvT, typename ScaleT, int D, int NWM>
int launch_decode(const PagedArgs& a, const MmaPlan& plan, void* ws, cudaStream_t s) {
  switch (plan.variant) {
    case 0: return launch_cfg<KvT, ScaleT, D, NWM, 4>(a, plan, ws, s);
    case 1: return launch_cfg<KvT, ScaleT, D, NWM, 4, 12>(a, plan, ws, s);
    case 2: return launch_cfg<KvT, ScaleT, D, NWM, 2, 2>(a, plan, ws, s);
    case 3: return launch_cfg<KvT, ScaleT, D, NWM, 2, 6>(a, plan, ws, s);
    case 4: return launch_cfg<KvT, ScaleT, D, NWM, 2, 8>(a, plan, ws, s);
    case 5: return launch_cfg<KvT, ScaleT, D, NWM, 4, 4>(a, plan, ws, s);
    case 6: return launch_cfg<KvT, ScaleT, D, NWM, 1, 4>(a, plan, ws, s);
    case 7: return launch_cfg<KvT, ScaleT, D, NWM, 2, 4>(a, plan, ws, s);
    case 8: return launch_cfg<KvT, ScaleT, D, NWM, 1, 6>(a, plan, ws, s);
    default: return launch_cfg<KvT, ScaleT, D, NWM, 2, 6>(a, plan, ws, s);
  }
}

// Three 16-row m-tiles (e.g. 8 q heads x 5 verify tokens = 40 rows).
template <typename KvT, typename ScaleT, int D>
int launch_m3(const PagedArgs& a, const MmaPlan& plan, void* ws, cudaStream_t s) {
  switch (plan.variant) {
    case 0: return launch_cfg<KvT, ScaleT, D, 3, 2>(a, plan, ws, s);
    case 1: return launch_cfg<KvT, ScaleT, D, 3, 1, 4>(a, plan, ws, s);
    case 2: return launch_cfg<KvT, ScaleT, D, 3, 1, 6>(a, plan, ws, s);
    case 3: return launch_cfg<KvT, ScaleT, D, 3, 2, 6>(a, plan, ws, s);
    default: return launch_cfg<KvT, ScaleT, D, 3, 1, 4>(a, plan, ws, s);
  }
}

template <typename KvT, typename ScaleT, int D>
int launch_d(const PagedArgs& a, const MmaPlan& plan, void* ws, cudaStream_t s) {
  switch (plan.nwm) {
    case 0: return launch_decode<KvT, ScaleT, D, 0>(a, plan, ws, s);
    case 1: return launch_decode<KvT, ScaleT, D, 1>(a, plan, ws, s);
    case 2: return launch_cfg<KvT, ScaleT, D, 2, 2>(a, plan, ws, s);
    case 3: return launch_m3<KvT, ScaleT, D>(a, plan, ws, s);
    default: return launch_cfg<KvT, ScaleT, D, 4, 1>(a, plan, ws, s);
  }
}

}  // namespace

MmaPlan plan_paged_mma(const PagedArgs& a) {
  MmaPlan plan{};
  plan.eligible = false;
  const bool kv16 = a.kv_dtype == NVM_F16 || a.kv_dtype == NVM_BF16;
  const bool kv8 = a.kv_dtype == NVM_I8 && a.D == 128 && (a.scale_dtype == NVM_F16 || a.scale_dtype == NVM_BF16);
  if (!(kv16 && (a.D == 64 || a.D == 128)) && !kv8) return plan;
  const bool dense = a.dense != 0;
  if (dense ? a.page_size < 16 : (a.page_size % 16) != 0) return plan;
  if (a.P <= 0 || a.P > INT32_MAX || a.Hkv > INT32_MAX || a.page_size > INT32_MAX) return plan;
  if (a.max_pages <= 0) return plan;
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (!al16(a.k_pages) || !al16(a.v_pages)) return plan;
  // q is read as element pairs
  if ((reinterpret_cast<uintptr_t>(a.q) & (a.q_dtype == NVM_F32 ? 7 : 3)) != 0) return plan;
  if (kv8 && (!al16(a.k_scales) || !al16(a.v_scales))) return plan;
  const int64_t M = (a.Hq / a.Hkv) * a.L;
  plan.nwm = M <= 16 ? 1 : (M <= 32 ? 2 : (M <= 48 ? 3 : 4));
  // at most eight query rows per kv head: the n8 tile (nwm = 0)
  if (M <= 8 && env_int("NVM_ATTN_N8", 1) != 0) plan.nwm = 0;
  plan.nwk = plan.nwm <= 1 ? 4 : (plan.nwm == 4 ? 1 : 2);
  // variant -> consumer warps along keys (must match launch_decode / launch_m3)
  plan.variant = -1;
  if (plan.nwm <= 1) {
    static const int kWarps1[9] = {4, 4, 2, 2, 2, 4, 1, 2, 1};
    // the n8 tile runs without a producer warp: small CTAs with a short ring
    // (2 warps x 4 stages) let the most of them share an SM (one CTA per unit with a
    // producer and 12 consumer warps measured 1.9x slower on config 1: a unit's pages
    // have to come through many SMs)
    int dflt = plan.nwm == 0 ? kDefaultN8Variant : kDefaultDecodeVariant;
    // n8 tile, 16-bit pages, short contexts, more units than the default variant's CTA
    // slots but no more than those of 2 warps x 2 stages (8 CTAs per SM against 6): the
    // smaller ring runs the launch as one wave (B = 128 at 1-1.1K keys, 32/8 heads: 92 us
    // against 112 us).  Launches that need several waves either way keep the deeper ring
    // (B = 160 at 600-1000 keys, 16/8 heads: 101 us against 107 us with 2 x 2; config 3:
    // 2 x 4 stages 7249-7292 GB/s against 7090-7137).
    if (plan.nwm == 0 && kv16 && !dense && env_int("NVM_ATTN_WAVE_RULE", 1) != 0) {
      const int64_t units = a.B * a.Hkv, sms = sm_count_cached();
      const int64_t tiles = (a.max_pages * a.page_size + 15) / 16;
      if (tiles <= kOneWaveTiles && units > sms * n8_resident_per_sm(a, dflt) && units <= sms * n8_resident_per_sm(a, 2))
        dflt = 2;
    }
    plan.variant = (int)env_int("NVM_ATTN_DECODE_CFG", dflt);
    if (plan.variant < 0 || plan.variant > 8) plan.variant = 3;
    plan.nwk = kWarps1[plan.variant];
  } else if (plan.nwm == 3) {
    static const int kWarps3[4] = {2, 1, 1, 2};
    plan.variant = (int)env_int("NVM_ATTN_M3_CFG", kDefaultM3Variant);
    if (plan.variant < 0 || plan.variant > 3) plan.variant = 1;
    plan.nwk = kWarps3[plan.variant];
  }
  plan.rows_per_block = plan.nwm == 0 ? 8 : 16 * plan.nwm;
  plan.n_row_blocks = (M + plan.rows_per_block - 1) / plan.rows_per_block;
  plan.rows_real = M < plan.rows_per_block ? M : plan.rows_per_block;
  plan.n_units = a.B * a.Hkv * plan.n_row_blocks;
  if (plan.n_units > INT32_MAX) return plan;
  const bool can_split = plan.n_units <= kMaxUnits;
  int64_t keys = a.max_pages * a.page_size;
  if (dense) keys = a.page_size;
  const int64_t tiles_max = (keys + 15) / 16;
  // the kernel's index arithmetic runs in 32 bits
  if (tiles_max >= INT32_MAX / 2 || M >= INT32_MAX) return plan;
  int64_t ct;
  if (dense || !can_split) {
    ct = tiles_max;  // dense callers pass no workspace: never split
  } else {
    // n8 tile: enough chunks for about six waves of its 8 CTAs per SM if every sequence
    // were as long as the longest: ragged contexts leave many chunks empty, and with
    // fewer waves the last one runs mostly idle (config 4, 64 sequences of 8K-32K keys:
    // 160-tile chunks 4777-4807 GB/s against 4533-4564 with 256; config 3 stays at the
    // 256 cap).  Multi-row tiles keep about 16 chunk CTAs per SM.
    const int64_t sms = sm_count_cached();
    const int64_t target = plan.nwm == 0 ? sms * 48 : sms * 16;
    ct = (plan.n_units * tiles_max + target - 1) / target;
    ct = ((ct + 15) / 16) * 16;
    if (ct < 16) ct = 16;
    if (ct > kMaxChunkTiles) ct = kMaxChunkTiles;
    // Short contexts (the n8 tile): many 16-tile chunks cost more in per-CTA set-up,
    // merges and partial waves than they gain in balance.  When the units fit in the
    // CTA slots the SMs hold at once, each is cut into the fewest equal chunks that give
    // about four CTAs per SM (enough page loads in flight to keep HBM busy), within one
    // wave, if those chunks are at most kOneWaveTiles long: B = 64 at 1-1.1K keys (32/8
    // heads) one 70-tile chunk a unit, 50.5 us against 65.5 us with five 14-tile chunks;
    // B = 32 at 2K keys three 44-tile chunks, 53 us against 66 us.  Otherwise chunks are
    // at least 48 tiles long (B = 128 at 1-1.1K keys: 2 x 35 tiles, 105 us against
    // 121 us; B = 256 at 512 keys: one 36-tile chunk, 104 us against 132 us).
    // NVM_ATTN_WAVE_RULE=0 keeps the six-wave sizing alone (sweeps).
    if (plan.nwm == 0 && env_int("NVM_ATTN_WAVE_RULE", 1) != 0) {
      const int64_t slots = sms * n8_resident_per_sm(a, plan.variant);
      bool one_wave = false;
      if (plan.n_units <= slots) {
        int64_t nc = (4 * sms + plan.n_units - 1) / plan.n_units;
        const int64_t nc_max = slots / plan.n_units;
        if (nc > nc_max) nc = nc_max;
        if (nc < 1) nc = 1;
        int64_t ct1 = (tiles_max + nc - 1) / nc;
        if (ct1 < 16) ct1 = 16;
        if (ct1 <= kOneWaveTiles) {
          ct = ct1;
          one_wave = true;
        }
      }
      if (!one_wave) {
        int64_t floor_ct = tiles_max < 48 ? tiles_max : 48;
        // Long contexts (>= 16K keys) with units enough for two waves of 128-tile chunks:
        // chunks of at least 128 tiles (one rank's kv-head shard of config 3 at 8 GPUs,
        // 256 units of 4K-32K keys: 380 us against 387 us with the six-wave 80 tiles;
        // config 4's 160 and config 3's 256 are above the floor anyway).
        if (tiles_max >= 1024 && plan.n_units * ((tiles_max + 127) / 128) >= 2 * slots) floor_ct = 128;
        if (ct < floor_ct) ct = floor_ct;
      }
    }
    // the longest context split evenly over that many chunks (B = 512 at 1024 tokens:
    // 2 x 32 tiles, 343 us, instead of 48 + 16, 391 us)
    if (ct < tiles_max) {
      const int64_t nc = (tiles_max + ct - 1) / ct;
      ct = (tiles_max + nc - 1) / nc;
    }
    const int64_t forced = env_int("NVM_ATTN_CHUNK_TILES", 0);
    if (forced > 0) ct = forced < kMaxChunkTiles ? forced : kMaxChunkTiles;
    if (ct > tiles_max) ct = tiles_max;
  }
  if (ct < 1) ct = 1;
  if (ct > kMaxChunkTiles && !dense) ct = kMaxChunkTiles;
  plan.chunk_tiles = ct;
  plan.n_chunks = (tiles_max + ct - 1) / ct;
  if (plan.n_chunks < 1) plan.n_chunks = 1;
  if (plan.n_chunks > 65535) return plan;
  // n8 tile with 2..8 chunks: the chunks of a unit merge inside a thread-block cluster
  // (distributed shared memory) instead of through the workspace, which takes the
  // global-memory round trips of the split-K merge off every unit's critical path.
  // Every CTA of a cluster stays resident until its unit is merged, so chunks without
  // keys (ragged contexts) idle in their slots, and a cluster launches only when all
  // its CTAs fit at once; the cluster merge is therefore used when the launch fits in
  // one wave (B = 128 at 1-1.1K keys, 2 chunks over two waves: 125 us in clusters
  // against 105 us through the workspace).
  // NVM_ATTN_CLUSTER: 0 never, 2 whenever 2..8 chunks (sweeps), otherwise the rule above.
  plan.cluster = 0;
  const int64_t cl_mode = env_int("NVM_ATTN_CLUSTER", 1);
  if (plan.nwm == 0 && plan.nwk <= 4 && !dense && can_split && plan.n_chunks >= 2 && plan.n_chunks <= 8 &&
      cl_mode != 0) {
    const bool one_wave = plan.n_units * plan.n_chunks <= sm_count_cached() * n8_resident_per_sm(a, plan.variant);
    if (cl_mode == 2 || one_wave) plan.cluster = 1;
  }
  if (dense && ct > kMaxChunkTiles) {
    // The per-CTA page table holds kMaxChunkTiles entries; a dense sequence longer
    // than that is still one page, so only its first entry is read -- but keep the
    // table bound honest by splitting into several single-page chunks is not allowed
    // without workspace.  Fall back to the generic kernel.
    return plan;
  }
  plan.ws_bytes = 0;
  if (plan.n_chunks > 1 && !plan.cluster) {
    plan.ws_bytes = kCounterBytes + align256(plan.n_units * plan.n_chunks * plan.rows_real * sizeof(float2)) +
                    (size_t)plan.n_units * plan.n_chunks * plan.rows_real * a.D * sizeof(float);
  }
  plan.eligible = true;
  return plan;
}

int launch_paged_mma(const PagedArgs& a, const MmaPlan& plan, void* ws, cudaStream_t s) {
  if (a.kv_dtype == NVM_F16) {
    return a.D == 64 ? launch_d<__half, __half, 64>(a, plan, ws, s) : launch_d<__half, __half, 128>(a, plan, ws, s);
  }
  if (a.kv_dtype == NVM_BF16) {
    return a.D == 64 ? launch_d<__nv_bfloat16, __nv_bfloat16, 64>(a, plan, ws, s)
                     : launch_d<__nv_bfloat16, __nv_bfloat16, 128>(a, plan, ws, s);
  }
  if (a.scale_dtype == NVM_F16) return launch_d<int8_t, __half, 128>(a, plan, ws, s);
  return launch_d<int8_t, __nv_bfloat16, 128>(a, plan, ws, s);
}

}  // namespace nvm
