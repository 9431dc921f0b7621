// flash_2q.cu -- tcgen05 / TMEM flash attention for long prefill: two 128-row query
// tiles of one head per CTA share every 128-key K/V tile.
//
// Serves prefill-shaped calls with at least 256 query rows per head (dense causal or
// full prefill, flash_attention.metal:6-153 / flash_attention.cpp:251-352 of the
// reference, and chunked prefill against 16-token pages, paged_attention.metal:6-128),
// 16-bit Q/K/V, head dim 128.  Same semantics as the reference: row l sees keys
// <= l + ctx - L when causal, holes are skipped, rows without a visible key are zero.
//
// One CTA per (q head, 256-row block), one CTA per SM (192 KB of shared memory, all 512
// tensor-memory columns), row blocks with the most causal work first:
//   warps 0-3  softmax of query tile 0 (thread i = query row i = TMEM lane i)
//   warps 4-7  softmax of query tile 1
//   warp 8     producer: TMA loads of both query tiles, then the K and V tiles (128 keys:
//              two 64-column boxes, or eight 16-token pages) into 2-stage rings
//   warp 9     MMA issuer: S_t = Q_t K_j^T (M 128, N 128, fp32 in TMEM columns
//              [128 t, 128 t + 128)), O_t += P_t V_j (A = P_t from TMEM, N 128, O_t in
//              columns [256 + 128 t, ...)), in the order S_0(0) S_1(0) | PV_0(j) S_0(j+1)
//              PV_1(j) S_1(j+1) | ..., so each softmax warpgroup works on its tile while
//              the tensor core runs the other tile's PV and S.
// The softmax writes P (16-bit pairs; bf16 as hi + lo when the tile's rows see few keys)
// over the first columns of S_t; the next S_t MMA is issued after the PV MMA that reads
// them (tcgen05.mma operations of one thread execute in issue order).  The O rescale of
// the lazy row max (threshold 2^8) happens in the softmax warps: when S_t(j) has landed,
// every earlier MMA of the thread, PV_t(j-1) included, has completed.
// Every mbarrier wait is bounded; on expiry the CTA records an error, lets its own copies
// and MMAs land (bounded), frees tensor memory and returns.
//
// Status: correct (tests/test_gpu_flash2q.py) but slower than flash_sm100.cu's one-tile
// kernel on every shape measured, so it is taken only with NVM_ATTN_2Q=1.  With ten warps
// the register cap is 168 per thread, which forces the softmax to read S in two 64-column
// passes; moving half the exponentials to the FMA pipe made it slower still, so the
// exponential unit is not what bounds it.
#include <cstdlib>
#include <mutex>

#include "nvm_common.cuh"
#include "nvm_internal.h"
#include "tcgen05.cuh"

namespace nvm {
namespace {

constexpr int kD = 128;                      // head dim
constexpr int kBM = 128;                     // rows per query tile
constexpr int kBN = 128;                     // keys per K/V tile
constexpr int kQTileBytes = kBM * kD * 2;    // 32 KB
constexpr int kTileBytes = kBN * kD * 2;     // 32 KB per K (or V) tile
constexpr int kStages = 2;                   // K ring and V ring depth
constexpr int kThreads = 320;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kTmemCols = 512;               // S0, S1, O0, O1
constexpr int kBarBytes = 256;
constexpr int kSmemBytes = 2 * kQTileBytes + 2 * kStages * kTileBytes + kBarBytes;  // 192.25 KB: one CTA per SM
constexpr int kPagesPerTile = kBN / 16;      // paged path: page_size == 16
constexpr float kRescaleThreshold = 8.0f;    // log2(256)
constexpr int64_t kSplitBelowKeys = 256;

int64_t env_i64(const char* name, int64_t dflt) {
  const char* v = std::getenv(name);
  if (v == nullptr || v[0] == '\0') return dflt;
  return std::atoll(v);
}

struct F2Params {
  void* out;
  const int32_t* block_table;
  const int32_t* context_lens;
  int* err;
  int out_dtype;
  int64_t B, Hq, Hkv, L, P, ps, mp, dense_ctx, g;
  int64_t n_outer, n_blocks;  // n_outer = B * Hq heads; n_blocks = ceil(L / 256)
  float scale_log2;
  int causal;
  int dense;
  int64_t split_below;
  int safe_order;  // 1: wait for PV_t(j) to complete before S_t(j+1) overwrites P_t (A/B check)
};

// 128-row tile t of the CTA's row block: rows, 128-key tiles it needs, hi/lo P split.
struct TileGeom {
  int64_t r0, rows, n_tiles;
  bool split;
};

__device__ __forceinline__ TileGeom tile_geom(const F2Params& p, int64_t rb, int t, int64_t ctx, int64_t ctx_limit,
                                              bool split_type) {
  TileGeom g;
  g.r0 = rb * (2 * kBM) + t * kBM;
  const int64_t left = p.L - g.r0;
  g.rows = left <= 0 ? 0 : (left < kBM ? left : kBM);
  int64_t need = ctx_limit;
  if (p.causal) {
    const int64_t lim = (g.r0 + g.rows - 1) + ctx - p.L + 1;
    if (lim < need) need = lim;
  }
  if (ctx <= 0 || g.rows <= 0 || need < 0) need = 0;
  g.n_tiles = (need + kBN - 1) / kBN;
  const int64_t min_keys = p.causal ? (g.r0 + ctx - p.L + 1) : ctx_limit;
  g.split = split_type && min_keys < p.split_below;
  return g;
}

// Page ids of one 128-key tile (paged path).
struct PageIds {
  int v[kPagesPerTile];
};

// 32 output values of a row (columns c0 .. c0 + 31) times inv, to global memory.
__device__ __forceinline__ void store_row32(uint8_t* orow, const float* ov, int c0, float inv, int out_dtype) {
  if (out_dtype == NVM_F32) {
    float4* d = reinterpret_cast<float4*>(orow + c0 * 4);
#pragma unroll
    for (int x = 0; x < 8; ++x)
      d[x] = make_float4(ov[4 * x] * inv, ov[4 * x + 1] * inv, ov[4 * x + 2] * inv, ov[4 * x + 3] * inv);
  } else {
    uint4* d = reinterpret_cast<uint4*>(orow + c0 * 2);
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      if (out_dtype == NVM_BF16) {
        d[x] = make_uint4(cvt_pack<__nv_bfloat16>(ov[8 * x] * inv, ov[8 * x + 1] * inv),
                          cvt_pack<__nv_bfloat16>(ov[8 * x + 2] * inv, ov[8 * x + 3] * inv),
                          cvt_pack<__nv_bfloat16>(ov[8 * x + 4] * inv, ov[8 * x + 5] * inv),
                          cvt_pack<__nv_bfloat16>(ov[8 * x + 6] * inv, ov[8 * x + 7] * inv));
      } else {
        d[x] = make_uint4(cvt_pack<__half>(ov[8 * x] * inv, ov[8 * x + 1] * inv),
                          cvt_pack<__half>(ov[8 * x + 2] * inv, ov[8 * x + 3] * inv),
                          cvt_pack<__half>(ov[8 * x + 4] * inv, ov[8 * x + 5] * inv),
                          cvt_pack<__half>(ov[8 * x + 6] * inv, ov[8 * x + 7] * inv));
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    flash2q_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const F2Params p) {
  constexpr bool kSplitType = std::is_same<T, __nv_bfloat16>::value;  // bf16 P may be split into hi + lo
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((smem_u32(smem) & 1023u) != 0) {  // 128B-swizzled tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) record_error(p.err, kDevErrSmemAlign);
    return;
  }
  uint8_t* sQ = smem;                              // [2] query tiles
  uint8_t* sK = smem + 2 * kQTileBytes;            // [kStages] K tiles
  uint8_t* sV = sK + kStages * kTileBytes;         // [kStages] V tiles
  uint64_t* q_full = reinterpret_cast<uint64_t*>(sV + kStages * kTileBytes);
  uint64_t* k_full = q_full + 1;                   // [kStages]
  uint64_t* k_empty = k_full + kStages;            // [kStages] both S MMAs of the tile are done with it
  uint64_t* v_full = k_empty + kStages;            // [kStages]
  uint64_t* v_empty = v_full + kStages;            // [kStages] both PV MMAs are done with it
  uint64_t* s_full = v_empty + kStages;            // [2] S_t(j) in TMEM (one completion per tile j)
  uint64_t* p_full = s_full + 2;                   // [2] P_t(j) written (count 128)
  uint64_t* o_done = p_full + 2;                   // [2] PV_t(j) complete (one completion per tile j)
  uint64_t* mma_done = o_done + 2;                 // every MMA of the CTA complete (teardown)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the CTA's work: row block rb of head n (heavy, late row blocks first across all heads)
  const int64_t rb = p.n_blocks - 1 - (int64_t)blockIdx.x / p.n_outer;
  const int64_t n = (int64_t)blockIdx.x % p.n_outer;
  const int64_t b = n / p.Hq;
  const int kvh = (int)((n % p.Hq) / p.g);
  const int64_t ctx = p.dense ? p.dense_ctx : (int64_t)p.context_lens[b];
  const int64_t cap = p.mp * p.ps;
  const int64_t ctx_limit = ctx < cap ? ctx : cap;
  const TileGeom g0 = tile_geom(p, rb, 0, ctx, ctx_limit, kSplitType);
  const TileGeom g1 = tile_geom(p, rb, 1, ctx, ctx_limit, kSplitType);
  const int nt0 = (int)g0.n_tiles, nt1 = (int)g1.n_tiles;
  const int n_tiles = nt0 > nt1 ? nt0 : nt1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 128);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int32_t* bt_row = p.dense ? nullptr : p.block_table + b * p.mp;

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------------- producer
    // One elected lane issues: both query tiles, then K_0, K_1, V_0, K_2, V_1, ...
    const bool leader = elect_one();
    bool ok = true;
    int gk = 0, gv = 0;
    if (n_tiles > 0) {
      if (leader) {
        mbar_arrive_expect_tx(q_full, 2 * kQTileBytes);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int row0 = (int)(rb * (2 * kBM) + t * kBM);
          tma_load_3d(sQ + t * kQTileBytes, &tm_q, 0, row0, (int)n, q_full);
          tma_load_3d(sQ + t * kQTileBytes + kBM * 128, &tm_q, 64, row0, (int)n, q_full);
        }
      }
      __syncwarp();
      // Paged: one page id per lane for 4 tiles (32 pages), loaded one block ahead; holes
      // and pages past the table load page P, outside the map (TMA fills zeros).
      auto load_ids = [&](int blk) -> int {
        const int pidx = blk * 32 + lane;
        const int id = pidx < (int)p.mp ? bt_row[pidx] : -1;
        return (id < 0 || id >= (int)p.P) ? (int)p.P : id;
      };
      int id_cur = 0, id_next = 0, id_blk = 0;
      if (!p.dense) {
        id_cur = load_ids(0);
        id_next = load_ids(1);
      }
      PageIds ids_k{}, ids_v{};
      auto issue = [&](const CUtensorMap* tm, uint8_t* dst, uint64_t* full, int t, const PageIds& pid) {
        if (leader) {
          mbar_arrive_expect_tx(full, kTileBytes);
          if (p.dense) {
            const int key0 = t * kBN;
            tma_load_4d(dst, tm, 0, key0, kvh, (int)b, full);
            tma_load_4d(dst + kBN * 128, tm, 64, key0, kvh, (int)b, full);
          } else {
#pragma unroll
            for (int gpg = 0; gpg < kPagesPerTile; ++gpg) {
              tma_load_4d(dst + gpg * 16 * 128, tm, 0, 0, kvh, pid.v[gpg], full);
              tma_load_4d(dst + kBN * 128 + gpg * 16 * 128, tm, 64, 0, kvh, pid.v[gpg], full);
            }
          }
        }
        __syncwarp();
      };
      for (int t = 0; ok && t <= n_tiles; ++t) {
        if (t < n_tiles) {  // K_t
          const int s = gk % kStages;
          if (gk >= kStages && !warp_wait(&k_empty[s], (uint32_t)(((gk / kStages) & 1) ^ 1))) {
            ok = false;
            break;
          }
          if (!p.dense) {
            if (t / 4 != id_blk) {
              id_cur = id_next;
              id_blk = t / 4;
              id_next = load_ids(id_blk + 1);
            }
#pragma unroll
            for (int gpg = 0; gpg < kPagesPerTile; ++gpg)
              ids_k.v[gpg] = __shfl_sync(0xffffffffu, id_cur, (t % 4) * kPagesPerTile + gpg);
          }
          issue(&tm_k, sK + s * kTileBytes, &k_full[s], t, ids_k);
          ++gk;
        }
        if (t >= 1) {  // V_{t-1}
          const int s = gv % kStages;
          if (gv >= kStages && !warp_wait(&v_empty[s], (uint32_t)(((gv / kStages) & 1) ^ 1))) {
            ok = false;
            break;
          }
          issue(&tm_v, sV + s * kTileBytes, &v_full[s], t - 1, ids_v);
          ++gv;
        }
        ids_v = ids_k;
        if (__any_sync(0xffffffffu, *(volatile int*)abort_flag != 0)) ok = false;
      }
    }
    if (leader) {
      if (!ok) {
        record_error(p.err, kDevErrEmptyWait);
        *(volatile int*)abort_flag = 1;
      }
      // drain: every issued load lands before the CTA may exit
      if (n_tiles > 0 && !mbar_wait(q_full, 0)) record_error(p.err, kDevErrDrainWait);
      auto drain = [&](uint64_t* full, int issued) {
        for (int s = 0; s < kStages && s < issued; ++s) {
          const int last = s + ((issued - 1 - s) / kStages) * kStages;
          if (!mbar_wait(&full[s], (uint32_t)((last / kStages) & 1))) record_error(p.err, kDevErrDrainWait);
        }
      };
      drain(k_full, gk);
      drain(v_full, gv);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    const bool leader = elect_one();
    const uint32_t id_qk = idesc<T>(false, kBN);
    const uint32_t id_pv = idesc<T>(true, kD);
    uint64_t dq[2][8];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const uint64_t q0 = smem_desc(smem_u32(sQ + t * kQTileBytes), 16, 1024);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) dq[t][ks] = q0 + (uint64_t)((((ks >> 2) * (kBM * 128)) + (ks & 3) * 32) >> 4);
    }
    const uint64_t dk = smem_desc(smem_u32(sK), 16, 1024);
    // V is MN-major: 64-column halves kBN*128 bytes apart (LBO), 8-token groups 1024 apart (SBO)
    const uint64_t dv = smem_desc(smem_u32(sV), kBN * 128, 1024);
    bool ok = true;
    auto issue_s = [&](int t, int j) {  // S_t = Q_t K_j^T
      const uint64_t dks = dk + (uint64_t)(((j % kStages) * kTileBytes) >> 4);
      uint64_t db[8];
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) db[ks] = dks + (uint64_t)((((ks >> 2) * (kBN * 128)) + (ks & 3) * 32) >> 4);
      const uint32_t td = tmem + (uint32_t)(t * kBN);
      if (leader) {
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) mma_f16(td, dq[t][ks], db[ks], id_qk, ks > 0 ? 1u : 0u);
        mma_commit(&s_full[t]);
      }
      __syncwarp();
    };
    auto issue_pv = [&](int t, int j) {  // O_t += P_t V_j
      const uint64_t dvs = dv + (uint64_t)(((j % kStages) * kTileBytes) >> 4);
      uint64_t db[8];
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) db[ks] = dvs + (uint64_t)((ks * 16 * 128) >> 4);
      const uint32_t tp = tmem + (uint32_t)(t * kBN);
      const uint32_t to = tmem + (uint32_t)(2 * kBN + t * kD);
      if (leader) {
#pragma unroll
        for (int ks = 0; ks < kBN / 16; ++ks) {
          mma_f16_ts(to, tp + (uint32_t)(ks * 8), db[ks], id_pv, (j > 0 || ks > 0) ? 1u : 0u);
          if (t == 0 ? g0.split : g1.split) mma_f16_ts(to, tp + (uint32_t)(kBN / 2 + ks * 8), db[ks], id_pv, 1u);
        }
        mma_commit(&o_done[t]);
      }
      __syncwarp();
    };
    if (n_tiles > 0) {
      ok = warp_wait(q_full, 0) && warp_wait(&k_full[0], 0);
      if (ok) {
        tc_fence_after();
        if (nt0 > 0) issue_s(0, 0);
        if (nt1 > 0) issue_s(1, 0);
        if (leader) mma_commit(&k_empty[0]);
        __syncwarp();
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        bool v_ready = false, k_ready = false;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int ntt = t == 0 ? nt0 : nt1;
          if (!ok || j >= ntt) continue;
          // P_t(j) written by the softmax warps; V_j landed
          if (!warp_wait(&p_full[t], (uint32_t)(j & 1))) {
            ok = false;
            break;
          }
          if (!v_ready) {
            if (!warp_wait(&v_full[j % kStages], (uint32_t)((j / kStages) & 1))) {
              ok = false;
              break;
            }
            v_ready = true;
          }
          tc_fence_after();
          issue_pv(t, j);
          if (j + 1 < ntt) {
            if (!k_ready) {
              if (!warp_wait(&k_full[(j + 1) % kStages], (uint32_t)(((j + 1) / kStages) & 1))) {
                ok = false;
                break;
              }
              k_ready = true;
            }
            if (p.safe_order && !warp_wait(&o_done[t], (uint32_t)(j & 1))) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(t, j + 1);
          }
        }
        if (!ok) break;
        if (leader) {
          mma_commit(&v_empty[j % kStages]);                         // both PVs of tile j issued
          if (j + 1 < n_tiles) mma_commit(&k_empty[(j + 1) % kStages]);  // both S of tile j+1 issued
        }
        __syncwarp();
      }
    }
    if (leader) {
      if (!ok) {
        record_error(p.err, kDevErrMmaWait);
        *(volatile int*)abort_flag = 1;
      }
      mma_commit(mma_done);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- softmax warps 0-7
    const int t = warp >> 2;                       // query tile of this warpgroup
    const int wq = warp & 3;
    const int row = wq * 32 + lane;                // TMEM lane == row in the tile
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + (uint32_t)(t * kBN);
    const uint32_t tO = tmem + lane_base + (uint32_t)(2 * kBN + t * kD);
    const TileGeom gt = t == 0 ? g0 : g1;
    const int nt = (int)gt.n_tiles;
    const bool split = gt.split;
    const bool row_ok = row < gt.rows;
    const int64_t lpos = gt.r0 + row;              // the row's position among the L query tokens
    const int esz = p.out_dtype == NVM_F32 ? 4 : 2;
    uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) + (n * p.L + lpos) * (int64_t)kD * esz;
    const float sl2 = p.scale_log2;                // > 0, so max(s) * sl2 == max(s * sl2)
    int64_t last_key = ctx_limit - 1;
    if (p.causal && lpos + ctx - p.L < last_key) last_key = lpos + ctx - p.L;
    if (!row_ok) last_key = -1;
    bool ok = true;
    // Paged holes: page ids two tiles ahead, lanes 0..7 hold page g = lane of a tile.
    auto load_pid = [&](int j) -> int {
      if (p.dense || lane >= kPagesPerTile || j >= nt) return 0;
      const int pidx = j * kPagesPerTile + lane;
      return pidx < (int)p.mp ? bt_row[pidx] : -1;
    };
    int pid0 = load_pid(0), pid1 = load_pid(1);
    float m = -INFINITY, lsum = 0.f;  // running max (log2 units, lazily updated) and sum
    for (int j = 0; j < nt; ++j) {
      if (!warp_wait(&s_full[t], (uint32_t)(j & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int pid_now = pid0;
      pid0 = pid1;
      pid1 = load_pid(j + 2);
      const int64_t key0 = (int64_t)j * kBN;
      // only tiles that cross some row's last visible key pay for the mask
      const int64_t vis64 = last_key - key0;
      const bool need_mask = __any_sync(0xffffffffu, vis64 < kBN - 1);
      const int vis = vis64 < -1 ? -1 : (vis64 > kBN ? kBN : (int)vis64);
      uint32_t holes = 0;
      if (!p.dense)  // the 16-token groups of missing pages are masked
        holes = __ballot_sync(0xffffffffu, lane < kPagesPerTile && (pid_now < 0 || pid_now >= (int)p.P)) & 0xFFu;
      // 64 scores of the row (columns c0 .. c0 + 63) from TMEM, masked
      auto load64 = [&](float (&sv)[64], int c0) {
        tmem_ld32(tS + c0, *reinterpret_cast<float(*)[32]>(&sv[0]));
        tmem_ld32(tS + c0 + 32, *reinterpret_cast<float(*)[32]>(&sv[32]));
        tmem_wait_ld();
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < 64; ++c) sv[c] = c0 + c <= vis ? sv[c] : -INFINITY;
        }
        if (holes != 0) {
#pragma unroll
          for (int gg = 0; gg < 4; ++gg) {
            if ((holes >> (c0 / 16 + gg)) & 1u) {
#pragma unroll
              for (int c = 0; c < 16; ++c) sv[gg * 16 + c] = -INFINITY;
            }
          }
        }
      };
      // pass 1: the row max, 64 scores at a time (8 independent chains)
      float mv[8];
#pragma unroll
      for (int x = 0; x < 8; ++x) mv[x] = -INFINITY;
#pragma unroll 1
      for (int c0 = 0; c0 < kBN; c0 += 64) {
        float sv[64];
        load64(sv, c0);
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
#pragma unroll
          for (int x = 0; x < 8; ++x) mv[x] = fmaxf(mv[x], sv[c + x]);
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mv[0], mv[1]), fmaxf(mv[2], mv[3])),
                             fmaxf(fmaxf(mv[4], mv[5]), fmaxf(mv[6], mv[7])));
      const float mx_s = mx * sl2;
      // lazy max: keep the old reference max unless the new one exceeds it by > 8
      float m_ref = m;
      bool rescale = false;
      if (mx_s > -INFINITY && (m == -INFINITY || mx_s > m + kRescaleThreshold)) {
        rescale = m != -INFINITY;
        m_ref = mx_s;
      }
      const float mu = m_ref == -INFINITY ? 0.f : m_ref;
      const float alpha = ex2_ftz(m - mu);  // 0 when m == -inf
      const float2 sl2v = make_float2(sl2, sl2), nmu = make_float2(-mu, -mu);
      float2 acc[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) acc[x] = make_float2(0.f, 0.f);
      // pass 2: p = 2^(s * sl2 - mu), the row sum, and P over the first columns of S_t:
      // packed pairs, hi in [0, kBN/2); for split tiles the rounding residual p - hi as
      // lo in [kBN/2, kBN).  The lo of the first half lands in columns the second half's
      // scores still occupy, so it is stored after they have been read.
      uint32_t lo_prev[32];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float sv[64];
        load64(sv, 64 * h);
        if (split && h == 1) tmem_st32u(tS + kBN / 2, lo_prev);
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const float2 x2 = __ffma2_rn(make_float2(sv[2 * q], sv[2 * q + 1]), sl2v, nmu);
          const float2 e = make_float2(ex2_ftz(x2.x), ex2_ftz(x2.y));
          sv[2 * q] = e.x;
          sv[2 * q + 1] = e.y;
          acc[q & 3] = __fadd2_rn(acc[q & 3], e);
        }
        uint32_t pk[32];
#pragma unroll
        for (int x = 0; x < 32; ++x) pk[x] = cvt_pack<T>(sv[2 * x], sv[2 * x + 1]);
        tmem_st32u(tS + h * 32, pk);
        if (split) {
#pragma unroll
          for (int x = 0; x < 32; ++x) {
            // bf16 -> f32 is exact: the bf16 bits become the high half of the f32
            const float h0 = __uint_as_float(pk[x] << 16), h1 = __uint_as_float(pk[x] & 0xFFFF0000u);
            lo_prev[x] = cvt_pack<T>(sv[2 * x] - h0, sv[2 * x + 1] - h1);
          }
          if (h == 1) tmem_st32u(tS + kBN / 2 + 32, lo_prev);
        }
      }
      const float2 a01 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
      const float rs = m_ref == -INFINITY ? 0.f : a01.x + a01.y;
      lsum = (m == -INFINITY ? 0.f : lsum * alpha) + rs;
      m = m_ref;
      if (__any_sync(0xffffffffu, rescale)) {
        // S_t(j) landed, so every earlier MMA of the issuing thread (PV_t(j-1) included)
        // has completed; PV_t(j) waits for this warpgroup's P_t(j) arrival below, so O_t
        // is rescaled between the two
        tc_fence_after();
        const float f = rescale ? alpha : 1.f;
#pragma unroll 1
        for (int c = 0; c < kD / 32; ++c) {
          float ov[32];
          tmem_ld32(tO + c * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) ov[x] *= f;
          tmem_st32(tO + c * 32, ov);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (ok && nt > 0 && !warp_wait(&o_done[t], (uint32_t)((nt - 1) & 1))) ok = false;
    if (ok) {
      tc_fence_after();
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
#pragma unroll 1
      for (int c = 0; c < kD; c += 32) {
        float ov[32];
        if (nt > 0) {
          tmem_ld32(tO + c, ov);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int x = 0; x < 32; ++x) ov[x] = 0.f;
        }
        if (row_ok) store_row32(orow, ov, c, nt > 0 ? inv : 0.f, p.out_dtype);
      }
    } else {
      record_error(p.err, kDevErrFullWait);
      *(volatile int*)abort_flag = 1;
    }
  }

  // ------------------------------------------------------------------ teardown
  if (warp == kMmaWarp && lane == 0) {
    if (!mbar_wait(mma_done, 0)) record_error(p.err, kDevErrMmaWait);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

template <typename T>
int launch_typed(dim3 grid, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                 const F2Params& p, cudaStream_t s) {
  static std::mutex mu;
  static uint64_t done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !(done & (1ull << dev))) {
      int r = check_cuda(cudaFuncSetAttribute(flash2q_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kSmemBytes),
                         "flash_attention: cudaFuncSetAttribute");
      if (r != NVM_OK) return r;
      done |= 1ull << dev;
    }
  }
  flash2q_kernel<T><<<grid, kThreads, kSmemBytes, s>>>(tq, tk, tv, p);
  return check_cuda(cudaGetLastError(), "flash_attention: two-tile kernel launch");
}

}  // namespace

bool flash2q_eligible(const PagedArgs& a) {
  // Opt-in (NVM_ATTN_2Q=1): measured slower than the one-tile kernel of flash_sm100.cu on
  // every prefill shape tried (config 2a causal 594 vs 707 TFLOP/s bf16, 696 vs 754 fp16).
  if (env_i64("NVM_ATTN_2Q", 0) == 0) return false;
  if (a.kv_dtype != NVM_F16 && a.kv_dtype != NVM_BF16) return false;
  if (a.q_dtype != a.kv_dtype || a.D != kD || !(a.scale > 0.f)) return false;
  if (a.L < 2 * kBM) return false;  // at least two query tiles per head
  if (a.dense) {
    if (a.page_size < kBN) return false;  // dense boxes are kBN rows
  } else if (a.page_size != 16) {
    return false;
  }
  if (a.out_dtype != NVM_F32 && a.out_dtype != NVM_F16 && a.out_dtype != NVM_BF16) return false;
  if (a.P <= 0 || a.P >= INT32_MAX || a.max_pages >= INT32_MAX || a.L >= INT32_MAX) return false;
  const int64_t n_blocks = (a.L + 2 * kBM - 1) / (2 * kBM);
  if (a.B * a.Hq > INT32_MAX || a.B * a.Hq * n_blocks > INT32_MAX) return false;
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  return al16(a.q) && al16(a.k_pages) && al16(a.v_pages) && al16(a.out);
}

int launch_flash2q(const PagedArgs& a, cudaStream_t s) {
  const CUtensorMapDataType dt =
      a.kv_dtype == NVM_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int64_t n_outer = a.B * a.Hq;
  // Q as [B*Hq, L, D] -> (D, L, B*Hq), 64 x 128 boxes (rows past L load as zeros)
  const uint64_t qd[3] = {(uint64_t)kD, (uint64_t)a.L, (uint64_t)n_outer};
  const uint64_t qs[2] = {kD * 2, (uint64_t)a.L * kD * 2};
  const uint32_t qb[3] = {64u, (uint32_t)kBM, 1u};
  CUtensorMap tq, tk, tv;
  int st = encode_tmap(&tq, dt, 3, a.q, qd, qs, qb, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVM_OK) return st;
  // pools [P, Hkv, ps, D] -> (D, ps, Hkv, P); dense K/V are one "page" of S rows per sequence
  const uint32_t box_rows = a.dense ? (uint32_t)kBN : 16u;
  const uint64_t kd[4] = {(uint64_t)kD, (uint64_t)a.page_size, (uint64_t)a.Hkv, (uint64_t)a.P};
  const uint64_t ks[3] = {kD * 2, (uint64_t)a.page_size * kD * 2, (uint64_t)(a.Hkv * a.page_size) * kD * 2};
  const uint32_t kb[4] = {64u, box_rows, 1u, 1u};
  st = encode_tmap(&tk, dt, 4, a.k_pages, kd, ks, kb, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVM_OK) return st;
  st = encode_tmap(&tv, dt, 4, a.v_pages, kd, ks, kb, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVM_OK) return st;

  F2Params p{};
  p.out = a.out;
  p.block_table = a.block_table;
  p.context_lens = a.context_lens;
  p.err = device_error_word();
  p.out_dtype = a.out_dtype;
  p.B = a.B; p.Hq = a.Hq; p.Hkv = a.Hkv; p.L = a.L; p.P = a.P; p.ps = a.page_size; p.mp = a.max_pages;
  p.dense_ctx = a.dense_ctx;
  p.g = a.Hq / a.Hkv;
  p.n_outer = n_outer;
  p.n_blocks = (a.L + 2 * kBM - 1) / (2 * kBM);
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.causal = a.is_causal;
  p.dense = a.dense;
  p.split_below = env_i64("NVM_SM100_SPLIT_BELOW", kSplitBelowKeys);
  p.safe_order = env_i64("NVM_2Q_SAFE_ORDER", 0) != 0 ? 1 : 0;
  const dim3 grid((unsigned)(n_outer * p.n_blocks));
  if (a.kv_dtype == NVM_F16) return launch_typed<__half>(grid, tq, tk, tv, p, s);
  return launch_typed<__nv_bfloat16>(grid, tq, tk, tv, p, s);
}

}  // namespace nvm
