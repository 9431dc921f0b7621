// flash_sm100.cu -- tcgen05 / TMEM flash attention for prefill-shaped calls:
// dense causal (or full) prefill and chunked prefill against paged context, 16-bit
// Q/K/V with head dim 128.
//
// Replaces, for L >= 64 query rows per head, the reference's FlashAttention Metal
// kernel (flash_attention.metal:6-153, dispatch flash_attention.cpp:251-352) and
// the multi-query paged kernel paged_attention_kv (paged_attention.metal:6-128);
// same semantics (causal key limit row + ctx - L, holes skipped, empty rows zero).
//
// One CTA computes a 128-row query tile of one q head (two CTAs per SM):
//   warps 0-3  softmax: thread i owns query row i = TMEM lane i.  Reads a 64-key S
//              row slice with tcgen05.ld, keeps the running max / sum in registers,
//              writes P (bf16/f16 pairs; bf16 as hi + lo for rows that see few keys)
//              back over S's TMEM columns with tcgen05.st, and rescales the O
//              accumulator in TMEM only when the row max grew by more than 2^8 (the
//              stale max keeps every p <= 256).  Masking costs one compare per score
//              and only in tiles that cross a row's last visible key.
//   warp 4     producer: TMA loads of the Q tile and of 64-token K and V tiles (pages
//              of 16 tokens for paged context, 64-row boxes for dense) into a 3-stage K
//              ring and a 2-stage V ring; holes load an out-of-range page (zero fill).
//   warp 5     MMA issuer: allocates 256 TMEM columns (S double buffer + O), issues
//              S = Q K^T (N=64) and O += P V (A = P from TMEM, N=128) as tcgen05.mma
//              kind::f16 with fp32 accumulate from one thread, and signals completion
//              with tcgen05.commit on mbarriers.
// Every mbarrier wait is bounded; on expiry the CTA records an error, lets its own
// copies and MMAs land (bounded), frees TMEM and returns.
#include <type_traits>

#include <cstdlib>
#include <mutex>

#include "nvm_common.cuh"
#include "nvm_internal.h"
#include "tcgen05.cuh"

namespace nvm {
namespace {

constexpr int kD = 128;          // head dim
constexpr int kBM = 128;         // query rows per CTA
constexpr int kBN = 64;          // keys per tile
constexpr int kKStages = 3;      // K ring: a K stage frees as soon as S_j = Q K_j^T is done
constexpr int kVStages = 2;      // V ring: a V stage frees when PV_j is done
constexpr int kTileBytes = kBN * kD * 2;  // 16 KB per K (or V) tile
constexpr int kQBytes = kBM * kD * 2;     // 32 KB
constexpr int kRingBytes = (kKStages + kVStages) * kTileBytes;  // 80 KB, also the epilogue's staging area
constexpr int kThreads = 192;
constexpr int kTmemCols = 256;   // S0 [0,64), S1 [64,128), O [128,256): two CTAs fit per SM
constexpr int kBarBytes = 512;   // mbarriers, TMEM address, flags, the 4-slot item ring
constexpr int kSmemBytes = kQBytes + kRingBytes + kBarBytes;  // 112.5 KB (+1 KB reserved each): two CTAs per SM
static_assert(kRingBytes >= kBM * kD * 4, "the epilogue stages a 128 x 128 fp32 tile in the K/V ring");
// bf16 P is split into hi + lo operands only for row tiles whose rows see fewer keys
// than this (few-key rows are where one bf16 P rounding shows in the output).
constexpr int64_t kSplitBelowKeys = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2(256)
// Split-K tickets: a fixed region at the start of the workspace (one int per unit); its
// last two ints are the work-item counter and the exit counter of the persistent grid.
constexpr size_t kSm100CounterBytes = kTicketRegionBytes;
constexpr int64_t kMaxTicketUnits = (int64_t)(kSm100CounterBytes / sizeof(int)) - 3;
constexpr int kPlanBins = 1024;  // tile-count bins of the plan's counting sort

int64_t env_int(const char* name, int64_t dflt) {
  const char* v = std::getenv(name);
  if (v == nullptr || v[0] == '\0') return dflt;
  return std::atoll(v);
}

struct Sm100Params {
  void* out;
  const int32_t* block_table;
  const int32_t* context_lens;
  int* err;
  int out_dtype;
  int64_t B, Hq, Hkv, L, P, ps, mp, dense_ctx;
  int64_t n_row_tiles;
  float scale_log2;
  int causal;
  int dense;
  int box_rows;   // rows of one K/V TMA box: 16 (pages) or kBN (dense)
  int64_t split_below;  // split bf16 P into hi + lo when the tile's first row sees fewer keys
  // Row units.  Prefill: a unit is the L rows of one q head (Q viewed as [B*Hq, L, D]).
  // Grouped (few query rows per head): a unit is the g*L rows of one kv head's query
  // group, which are contiguous in Q (viewed as [B*Hkv, g*L, D]); row r is q head
  // kvh*g + r/L at position l = r % L.
  int grouped;
  int64_t g, M_rows, n_outer, n_units;  // n_units = n_outer * n_row_tiles
  // Split-K over keys (grouped paged calls): chunk c of a unit covers 64-key tiles
  // [c*ct, (c+1)*ct); each chunk leaves (m, l) and unnormalised O rows in the workspace
  // and the unit's last chunk (atomic ticket) merges them.
  int64_t ct, n_chunks, rows_real;
  int64_t n_items;    // n_units * n_chunks work items
  int* work_counter;  // next item (in the workspace); null: item = blockIdx.x + k * gridDim.x
  const int* item_list;   // items with work, largest first (plan kernel); null: every item index
  const int* item_count;  // length of item_list
  int stage_out;      // one item per CTA: O leaves through shared memory and bulk tensor stores
  int pv_wait;        // 1: S_{j+2} waits for PV_j to complete (see the MMA issuer)
  int* exit_counter;  // CTAs done; the last one resets both counters
  int* counters;
  float2* part_ml;  // [n_units][n_chunks][rows_real]
  float* part_o;    // [n_units][n_chunks][rows_real][kD]
};

// Pairs q (keys 2q, 2q+1 of a 64-key tile) whose exponentials run on the FMA pipe.
// None by default: with two CTAs per SM the softmax warps are bound by instruction
// issue, not by the MUFU unit, and the polynomial costs more issue slots than ex2
// (measured: 25 % on the FMA pipe 730 TFLOP/s on config 2a, none 745, half 714).
constexpr uint32_t kEmuPairs = 0x0u;


// Geometry of one work item (a 128-row tile of a row unit x a chunk of 64-key tiles).
// Every warp role decodes the same item index to the same values.
struct Item {
  int64_t c, u, n, b, kvh, r0, rows, ctx, ctx_limit, l_first, t_begin, n_chunks_unit;
  int n_tiles;  // 64-key tiles of this item (0: no keys; still produces zero rows when valid)
  bool valid;   // false: a chunk past the unit's last key (nothing to do)
};

__device__ __forceinline__ Item decode_item(const Sm100Params& p, int64_t item) {
  Item it;
  // Chunk-major, last chunk first: a chunk c >= 1 exists only for long units and is then
  // full-size (except each unit's last), so handing out high chunks first and the mixed
  // chunk-0 items (short units included) last approximates longest-first scheduling.
  // The divisions run on 32-bit values (the plan bounds items, rows and tiles below
  // 2^31): 64-bit divisions here cost about a microsecond on the producer's path to
  // its first copy.
  const uint32_t item32 = (uint32_t)item, nu = (uint32_t)p.n_units, no = (uint32_t)p.n_outer;
  const uint32_t cq = item32 / nu, u32 = item32 - cq * nu;
  it.c = p.n_chunks - 1 - (int64_t)cq;
  it.u = u32;
  // Row-tile-major, heavy (late, causal) row tiles first across all heads: dispatch in
  // item order is then longest-first.
  const uint32_t rq = u32 / no, n32 = u32 - rq * no;
  const int64_t rt = p.n_row_tiles - 1 - (int64_t)rq;
  it.n = n32;  // flat (b, q head), or (b, kv head) when grouped
  const uint32_t hd = (uint32_t)(p.grouped ? p.Hkv : p.Hq);
  const uint32_t b32 = n32 / hd, h32 = n32 - b32 * hd;
  it.b = b32;
  it.kvh = p.grouped ? h32 : h32 / (uint32_t)p.g;
  it.ctx = p.dense ? p.dense_ctx : (int64_t)p.context_lens[it.b];
  const int64_t cap = p.mp * p.ps;
  it.ctx_limit = it.ctx < cap ? it.ctx : cap;
  it.r0 = rt * kBM;  // first row of the tile inside the unit
  it.rows = (p.M_rows - it.r0) < kBM ? (p.M_rows - it.r0) : kBM;
  // query positions l = r % L of the tile's rows: the smallest and the largest
  const int64_t r0_mod = (int64_t)((uint32_t)it.r0 % (uint32_t)p.L);
  const bool wraps = it.rows >= p.L || r0_mod + it.rows > p.L;
  it.l_first = wraps ? 0 : r0_mod;
  const int64_t l_last = wraps ? p.L - 1 : (int64_t)((uint32_t)(it.r0 + it.rows - 1) % (uint32_t)p.L);
  int64_t need = it.ctx_limit;
  if (p.causal) {
    const int64_t lim = l_last + it.ctx - p.L + 1;
    if (lim < need) need = lim;
  }
  if (it.ctx <= 0 || need < 0) need = 0;
  const int64_t n_tiles_unit = (need + kBN - 1) / kBN;
  it.n_chunks_unit = n_tiles_unit > 0 ? (int64_t)((uint32_t)(n_tiles_unit + p.ct - 1) / (uint32_t)p.ct) : 1;
  it.valid = it.c < it.n_chunks_unit;
  it.t_begin = it.c * p.ct;
  const int64_t left = n_tiles_unit - it.t_begin;
  it.n_tiles = it.valid && left > 0 ? (int)(left < p.ct ? left : p.ct) : 0;
  return it;
}

// Persistent: each CTA loops over work items (fetched from a counter in the workspace
// when there is one, else blockIdx.x + k * gridDim.x).  Rings and mbarrier phases run on
// per-CTA tile counters, so the next item's Q load, K/V loads and first S overlap the
// previous item's last tiles and epilogue.
template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    flash_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                       const Sm100Params p) {
  constexpr bool kSplit = std::is_same<T, __nv_bfloat16>::value;  // bf16 P = hi + lo
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((smem_u32(smem) & 1023u) != 0) {  // 128B-swizzled tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) record_error(p.err, kDevErrSmemAlign);
    return;
  }
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kQBytes;             // [kKStages] K tiles
  uint8_t* sV = sK + kKStages * kTileBytes;  // [kVStages] V tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sK + kRingBytes);
  uint64_t* q_full = bars;                   // Q of the CTA's i-th item with keys landed
  uint64_t* q_empty = q_full + 1;            // the last S of that item has read Q
  uint64_t* k_full = q_empty + 1;            // [kKStages] K tile landed
  uint64_t* k_empty = k_full + kKStages;     // [kKStages] S has read it
  uint64_t* v_full = k_empty + kKStages;     // [kVStages] V tile landed
  uint64_t* v_empty = v_full + kVStages;     // [kVStages] PV has read it
  uint64_t* s_full = v_empty + kVStages;     // [2] S_G in TMEM buffer G&1
  uint64_t* p_full = s_full + 2;             // [2] P_G written over S_G (count 128)
  uint64_t* o_done = p_full + 2;             // PV_G complete (only with pv_wait)
  uint64_t* item_done = o_done + 1;          // every PV of an item complete (one per item)
  uint64_t* o_free = item_done + 1;          // the softmax warps have read an item's O (count 128)
  uint64_t* mma_done = o_free + 1;           // every MMA of the CTA complete (teardown)
  uint64_t* item_full = mma_done + 1;        // [4] item index published in item_ring
  uint64_t* item_empty = item_full + 4;      // [4] read by the MMA warp and the 4 softmax warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_empty + 4);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* last_flag = abort_flag + 1;
  int64_t* item_ring = reinterpret_cast<int64_t*>(reinterpret_cast<uint8_t*>(bars) + 256);  // [4]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The producer warp's first lane sets up the barriers; with one item per CTA it then
  // requests that item's Q tile at once, before tensor memory is allocated and the CTA
  // synchronises (the first S waits on this copy).
  int q_early = 0;
  if (threadIdx.x == 4 * 32) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
    }
    mbar_init(o_done, 1);
    mbar_init(item_done, 1);
    mbar_init(o_free, 128);
    mbar_init(mma_done, 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 5);
    }
    *abort_flag = 0;
    fence_mbar_init();
    if (p.stage_out && (int64_t)blockIdx.x < p.n_items) {
      const Item it0 = decode_item(p, blockIdx.x);
      if (it0.valid && it0.n_tiles > 0) {
        mbar_arrive_expect_tx(q_full, kQBytes);
        tma_load_3d(sQ, &tm_q, 0, (int)it0.r0, (int)it0.n, q_full);
        tma_load_3d(sQ + kBM * 128, &tm_q, 64, (int)it0.r0, (int)it0.n, q_full);
        q_early = 1;
      }
    }
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 2 * kBN;
  constexpr int kPagesPerTile = kBN / 16;  // paged path: page_size == 16

  // consumers of the item ring: slot k & 3 of the k-th published item
  auto read_item = [&](int k, bool arrive) -> int64_t {
    if (!warp_wait(&item_full[k & 3], (k >> 2) & 1)) return -2;
    const int64_t v = *(volatile int64_t*)&item_ring[k & 3];
    __syncwarp();
    if (arrive && lane == 0) mbar_arrive(&item_empty[k & 3]);
    return v;
  };
  // the unit's fewest keys seen by a row: bf16 P is split into hi + lo below split_below
  auto split_of = [&](const Item& it) -> bool {
    const int64_t min_keys = p.causal ? (it.l_first + it.ctx - p.L + 1) : it.ctx_limit;
    return kSplit && min_keys < p.split_below;
  };

  if (warp == 4) {
    // ---------------------------------------------------------------- producer
    // The whole warp runs the loop and one elected lane issues the copies.  Per item:
    // publish the item index, load Q (once the previous item's last S has read sQ), then
    // K_0, K_1, V_0, K_2, V_1, ... into the rings.
    q_early = __shfl_sync(0xffffffffu, q_early, 0);  // the first item's Q is already on its way
    const bool leader = elect_one();
    const int leader_lane = __ffs(__ballot_sync(0xffffffffu, leader)) - 1;
    int gk = 0, gv = 0;  // K / V tiles issued by this CTA so far
    int kq = 0, iw = 0;      // items published, items with keys
    int64_t n_fetched = 0;   // item indices taken (static order: blockIdx.x + k * gridDim.x)
    bool ok = true;
    while (ok) {
      const int slot = kq & 3;
      if (kq >= 4 && !warp_wait(&item_empty[slot], ((kq >> 2) & 1) ^ 1)) {
        ok = false;
        break;
      }
      // Next item with work: chunks past a unit's last key are skipped here, without
      // taking a ring slot (the consumers would otherwise drain them only after their
      // current item, and the next real item's loads would start that late).
      int64_t item;
      Item it;
      for (;;) {
        if (p.item_list != nullptr) {
          int v = 0;
          if (leader) {
            const int k = atomicAdd(p.work_counter, 1);
            v = k < *p.item_count ? __ldcg(&p.item_list[k]) : INT32_MAX;
          }
          item = __shfl_sync(0xffffffffu, v, leader_lane);
        } else if (p.work_counter != nullptr) {
          int v = 0;
          if (leader) v = atomicAdd(p.work_counter, 1);
          item = __shfl_sync(0xffffffffu, v, leader_lane);
        } else {
          item = (int64_t)blockIdx.x + (int64_t)n_fetched * gridDim.x;
        }
        ++n_fetched;
        if (item >= p.n_items) {
          item = -1;
          break;
        }
        it = decode_item(p, item);
        if (it.valid) break;
      }
      if (leader) {
        *(volatile int64_t*)&item_ring[slot] = item;
        mbar_arrive(&item_full[slot]);
      }
      __syncwarp();
      ++kq;
      if (item < 0) break;
      if (it.n_tiles == 0) continue;  // no key: the softmax warps write zero rows
      const int kvh_i = (int)it.kvh, b_i = (int)it.b;
      const int32_t* bt_row = p.dense ? nullptr : p.block_table + it.b * p.mp;
      if (iw > 0 && !warp_wait(q_empty, (iw - 1) & 1)) {
        ok = false;
        break;
      }
      if (leader && !(iw == 0 && q_early)) {
        mbar_arrive_expect_tx(q_full, kQBytes);
        tma_load_3d(sQ, &tm_q, 0, (int)it.r0, (int)it.n, q_full);
        tma_load_3d(sQ + kBM * 128, &tm_q, 64, (int)it.r0, (int)it.n, q_full);
      }
      __syncwarp();
      ++iw;
      // Paged: the page ids of 8 tiles (32 pages) sit one per lane and are loaded one
      // block ahead; holes and pages past the table read as page P (TMA fills zeros).
      auto load_ids = [&](int blk) -> int {
        const int pidx = (int)(it.t_begin * kPagesPerTile) + blk * 32 + lane;
        const int id = pidx < (int)p.mp ? bt_row[pidx] : -1;
        return (id < 0 || id >= (int)p.P) ? (int)p.P : id;
      };
      int id_cur = 0, id_next = 0, id_blk = 0;
      if (!p.dense) {
        id_cur = load_ids(0);
        id_next = load_ids(1);
      }
      auto page_id = [&](int t, int g) -> int {
        const int v_cur = __shfl_sync(0xffffffffu, id_cur, (t % 8) * kPagesPerTile + g);
        const int v_next = __shfl_sync(0xffffffffu, id_next, (t % 8) * kPagesPerTile + g);
        return t / 8 == id_blk ? v_cur : v_next;
      };
      int ids_k[kPagesPerTile], ids_v[kPagesPerTile];
      auto issue = [&](const CUtensorMap* tm, uint8_t* dst, uint64_t* full, int t, const int* pid) {
        if (leader) {
          mbar_arrive_expect_tx(full, kTileBytes);
          if (p.dense) {
            const int key0 = (int)((it.t_begin + t) * kBN);
            tma_load_4d(dst, tm, 0, key0, kvh_i, b_i, full);
            tma_load_4d(dst + kBN * 128, tm, 64, key0, kvh_i, b_i, full);
          } else {
#pragma unroll
            for (int g = 0; g < kPagesPerTile; ++g) {
              tma_load_4d(dst + g * 16 * 128, tm, 0, 0, kvh_i, pid[g], full);
              tma_load_4d(dst + kBN * 128 + g * 16 * 128, tm, 64, 0, kvh_i, pid[g], full);
            }
          }
        }
        __syncwarp();
      };
      for (int t = 0; ok && t <= it.n_tiles; ++t) {
        if (t < it.n_tiles) {  // K_t
          const int s = gk % kKStages;
          if (gk >= kKStages && !warp_wait(&k_empty[s], (uint32_t)(((gk / kKStages) & 1) ^ 1))) {
            ok = false;
            break;
          }
          if (!p.dense) {
            if (t / 8 != id_blk) {
              id_cur = id_next;
              id_blk = t / 8;
              id_next = load_ids(id_blk + 1);
            }
#pragma unroll
            for (int g = 0; g < kPagesPerTile; ++g) ids_k[g] = page_id(t, g);
          }
          issue(&tm_k, sK + s * kTileBytes, &k_full[s], t, ids_k);
          ++gk;
        }
        if (t >= 1) {  // V_{t-1}
          const int s = gv % kVStages;
          if (gv >= kVStages && !warp_wait(&v_empty[s], (uint32_t)(((gv / kVStages) & 1) ^ 1))) {
            ok = false;
            break;
          }
          issue(&tm_v, sV + s * kTileBytes, &v_full[s], t - 1, ids_v);
          ++gv;
        }
#pragma unroll
        for (int g = 0; g < kPagesPerTile; ++g) ids_v[g] = ids_k[g];
        if (__any_sync(0xffffffffu, *(volatile int*)abort_flag != 0)) ok = false;
      }
    }
    if (leader) {
      if (!ok) {
        record_error(p.err, kDevErrEmptyWait);
        *(volatile int*)abort_flag = 1;
        // consumers waiting for an item index are released with the end marker
        for (int k = kq; k < kq + 4; ++k) {
          *(volatile int64_t*)&item_ring[k & 3] = -1;
          mbar_arrive(&item_full[k & 3]);
        }
      }
      // drain: every issued load lands before the CTA may exit
      if (iw > 0 && !mbar_wait(q_full, (iw - 1) & 1)) record_error(p.err, kDevErrDrainWait);
      auto drain = [&](uint64_t* full, int ns, int issued) {
        for (int s = 0; s < ns && s < issued; ++s) {
          const int last = s + ((issued - 1 - s) / ns) * ns;
          if (!mbar_wait(&full[s], (uint32_t)((last / ns) & 1))) record_error(p.err, kDevErrDrainWait);
        }
      };
      drain(k_full, kKStages, gk);
      drain(v_full, kVStages, gv);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp waits and loops; the MMAs and commits are issued through the
    // whole-warp forms, whose elect.sync picks the same lane every time (a commit tracks
    // the MMAs of the thread that issues it).
    const bool leader = elect_one();
    const uint32_t id_qk = idesc<T>(false, kBN);
    const uint32_t id_pv = idesc<T>(true, kD);
    // One thread can issue a tcgen05.mma only every ~47 cycles, and descriptor
    // arithmetic between two MMAs adds ~26 more: the Q descriptors are computed once,
    // a tile's K or V descriptors in one batch before its MMAs.
    uint64_t dq[8];
    {
      const uint64_t q0 = smem_desc(smem_u32(sQ), 16, 1024);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) dq[ks] = q0 + (uint64_t)((((ks >> 2) * (kBM * 128)) + (ks & 3) * 32) >> 4);
    }
    const uint64_t dk = smem_desc(smem_u32(sK), 16, 1024);
    const uint64_t dv = smem_desc(smem_u32(sV), kBN * 128, 1024);
    int gs = 0, gp = 0;  // S / PV tiles issued by this CTA so far
    int kq = 0, iw = 0;
    bool ok = true;
    // K of the next S landed (checked before the wait on the PV it overwrites, which it
    // does not depend on)
    auto wait_k = [&]() -> bool { return warp_wait(&k_full[gs % kKStages], (uint32_t)((gs / kKStages) & 1)); };
    // S_G = Q K^T into TMEM buffer G&1 from K stage G % kKStages (after wait_k)
    auto issue_s = [&](bool last_of_item) {
      const int s = gs % kKStages;
      tc_fence_after();
      const uint64_t dks = dk + (uint64_t)((s * kTileBytes) >> 4);
      uint64_t db[8];
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) db[ks] = dks + (uint64_t)((((ks >> 2) * (kBN * 128)) + (ks & 3) * 32) >> 4);
      const uint32_t td = tmem + (uint32_t)((gs & 1) * kBN);
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks) mma_f16_warp(td, dq[ks], db[ks], id_qk, ks > 0 ? 1u : 0u);
      mma_commit_warp(&s_full[gs & 1]);
      mma_commit_warp(&k_empty[s]);
      if (last_of_item) mma_commit_warp(q_empty);
      ++gs;
    };
    while (ok) {
      const int64_t item = read_item(kq, true);
      ++kq;
      if (item < 0) {
        ok = item == -1;
        break;
      }
      const Item it = decode_item(p, item);
      const int n = it.n_tiles;
      if (n == 0) continue;
      const bool split = split_of(it);
      // S buffers: every PV of the previous item done; Q of this item landed
      if (iw > 0 && !warp_wait(item_done, (iw - 1) & 1)) {
        ok = false;
        break;
      }
      if (!warp_wait(q_full, iw & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (!wait_k()) {
        ok = false;
        break;
      }
      issue_s(n == 1);
      if (n > 1) {
        if (!wait_k()) {
          ok = false;
          break;
        }
        issue_s(n == 2);
      }
      for (int j = 0; j < n; ++j) {
        // P_j written by the softmax warps, V_j landed; the first PV of an item overwrites
        // O, which the softmax warps must have read out for the previous item
        const int vs = gp % kVStages;
        if (!warp_wait(&p_full[gp & 1], (uint32_t)((gp >> 1) & 1)) ||
            !warp_wait(&v_full[vs], (uint32_t)((gp / kVStages) & 1)) ||
            (j == 0 && iw > 0 && !warp_wait(o_free, (iw - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // V is MN-major: 64-column halves kBN*128 bytes apart (LBO), 8-token groups 1024 apart (SBO)
        const uint64_t dvs = dv + (uint64_t)((vs * kTileBytes) >> 4);
        uint64_t db[4];
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) db[ks] = dvs + (uint64_t)((ks * 16 * 128) >> 4);
        const uint32_t tp = tmem + (uint32_t)((gp & 1) * kBN);
#pragma unroll
        for (int ks = 0; ks < kBN / 16; ++ks) {
          mma_f16_ts_warp(tO, tp + (uint32_t)(ks * 8), db[ks], id_pv, (j > 0 || ks > 0) ? 1u : 0u);
          if (split) mma_f16_ts_warp(tO, tp + (uint32_t)(kBN / 2 + ks * 8), db[ks], id_pv, 1u);
        }
        if (p.pv_wait) mma_commit_warp(o_done);
        mma_commit_warp(&v_empty[vs]);  // also tells the softmax warps that PV_j is complete
        if (j == n - 1) mma_commit_warp(item_done);
        const int gj = gp++;
        // S_{j+2} reuses S_j's TMEM columns, which hold P_j, the A operand of PV_j, so by
        // default it waits until PV_j has completed.  NVM_SM100_PV_WAIT=0 issues it right
        // behind PV_j instead, relying on one thread's MMAs executing in issue order: about
        // 1 % faster on prefill and bit-identical in every test, but no documented rule we
        // could confirm covers a later MMA overwriting an earlier one's A operand.
        if (j + 2 < n) {
          if (!wait_k() || (p.pv_wait && !warp_wait(o_done, (uint32_t)(gj & 1)))) {
            ok = false;
            break;
          }
          issue_s(j + 2 == n - 1);
        }
      }
      ++iw;
    }
    if (leader && !ok) {
      record_error(p.err, kDevErrMmaWait);
      *(volatile int*)abort_flag = 1;
    }
    __syncwarp();
    mma_commit_warp(mma_done);
  } else {
    // ---------------------------------------------------------------- softmax warps 0-3
    const int row = warp * 32 + lane;            // TMEM lane == query row in the tile
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float sl2 = p.scale_log2;              // > 0, so max(s) * sl2 == max(s * sl2)
    const int esz = p.out_dtype == NVM_F32 ? 4 : 2;
    const bool staged = p.stage_out != 0;  // O through shared memory and bulk tensor stores
    int gt = 0;  // tiles processed by this CTA so far
    int kq = 0, iw = 0;
    bool ok = true;
    // With one item per CTA (stage_out) the K/V ring is free once the item's MMAs are done:
    // O rows go to shared memory in the TMA store's 128B-swizzled box layout (boxes of 128
    // bytes of columns x 128 rows, 16 KB each; row r's 16-byte chunk c of a box at
    // r * 128 + ((c ^ (r & 7)) << 4)) and leave with bulk tensor stores.  Otherwise the
    // next item's tiles are already streaming into the ring and each row is stored directly.
    uint8_t* srow = sK + row * 128;
    auto stage32 = [&](const float* ov, int c0, float inv) {
      if (esz == 4) {
        uint8_t* box = srow + (c0 / 32) * (kBM * 128);
#pragma unroll
        for (int x = 0; x < 8; ++x)
          *reinterpret_cast<float4*>(box + ((x ^ (row & 7)) << 4)) =
              make_float4(ov[4 * x] * inv, ov[4 * x + 1] * inv, ov[4 * x + 2] * inv, ov[4 * x + 3] * inv);
      } else {
        uint8_t* box = srow + (c0 / 64) * (kBM * 128);
        const int ch0 = (c0 % 64) / 8;
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          uint4 v4;
          if (p.out_dtype == NVM_BF16) {
            v4 = make_uint4(cvt_pack<__nv_bfloat16>(ov[8 * x] * inv, ov[8 * x + 1] * inv),
                            cvt_pack<__nv_bfloat16>(ov[8 * x + 2] * inv, ov[8 * x + 3] * inv),
                            cvt_pack<__nv_bfloat16>(ov[8 * x + 4] * inv, ov[8 * x + 5] * inv),
                            cvt_pack<__nv_bfloat16>(ov[8 * x + 6] * inv, ov[8 * x + 7] * inv));
          } else {
            v4 = make_uint4(cvt_pack<__half>(ov[8 * x] * inv, ov[8 * x + 1] * inv),
                            cvt_pack<__half>(ov[8 * x + 2] * inv, ov[8 * x + 3] * inv),
                            cvt_pack<__half>(ov[8 * x + 4] * inv, ov[8 * x + 5] * inv),
                            cvt_pack<__half>(ov[8 * x + 6] * inv, ov[8 * x + 7] * inv));
          }
          *reinterpret_cast<uint4*>(box + (((ch0 + x) ^ (row & 7)) << 4)) = v4;
        }
      }
    };
    // the staged tile -> global memory (rows past the unit's end fall outside the tensor map)
    auto flush_staged = [&](const Item& it) {
      fence_async_smem();  // generic-proxy stores -> visible to the TMA engine
      named_barrier(1, 128);
      if (row == 0) {
        const int cols_per_box = esz == 4 ? 32 : 64;
        for (int bx = 0; bx < kD / cols_per_box; ++bx)
          tma_store_3d(&tm_o, sK + bx * (kBM * 128), bx * cols_per_box, (int)it.r0, (int)it.n);
        bulk_commit();
        bulk_wait_read_all();
      }
    };
    // 32 values of this row (columns c0 .. c0+31), times inv, straight to global memory
    auto store32 = [&](uint8_t* orow, const float* ov, int c0, float inv) {
      if (esz == 4) {
        float4* d = reinterpret_cast<float4*>(orow + c0 * 4);
#pragma unroll
        for (int x = 0; x < 8; ++x) d[x] = make_float4(ov[4 * x] * inv, ov[4 * x + 1] * inv, ov[4 * x + 2] * inv, ov[4 * x + 3] * inv);
      } else {
        uint4* d = reinterpret_cast<uint4*>(orow + c0 * 2);
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          if (p.out_dtype == NVM_BF16) {
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
    };
    while (ok) {
      const int64_t item = read_item(kq, true);
      ++kq;
      if (item < 0) {
        ok = item == -1;
        break;
      }
      const Item it = decode_item(p, item);
      if (!it.valid) continue;
      const int n = it.n_tiles;
      const bool row_ok = row < it.rows;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) + ((it.n * p.M_rows) + it.r0 + row) * (int64_t)kD * esz;
      if (n == 0) {  // no key: zero rows (a single chunk)
        float z[32];
#pragma unroll
        for (int x = 0; x < 32; ++x) z[x] = 0.f;
        if (row_ok)
          for (int c0 = 0; c0 < kD; c0 += 32) store32(orow, z, c0, 0.f);
        continue;
      }
      const bool split = split_of(it);
      const int64_t lpos = (it.r0 + row) % p.L;  // the row's position among the L query tokens
      // last key this row may see: inside the context and, when causal, key <= l + ctx - L
      int64_t last_key = it.ctx_limit - 1;
      if (p.causal && lpos + it.ctx - p.L < last_key) last_key = lpos + it.ctx - p.L;
      if (!row_ok) last_key = -1;
      // Paged: page ids two tiles ahead, lanes 0..3 hold page g = lane of a tile; the
      // hole test happens when the tile is processed, so the load latency is hidden.
      const int32_t* bt_row = p.dense ? nullptr : p.block_table + it.b * p.mp;
      auto load_pid = [&](int t) -> int {
        if (p.dense || lane >= kPagesPerTile || t >= n) return 0;
        const int pidx = (int)(it.t_begin + t) * kPagesPerTile + lane;
        return pidx < (int)p.mp ? bt_row[pidx] : -1;
      };
      int pid0 = load_pid(0), pid1 = load_pid(1);
      float m = -INFINITY, lsum = 0.f;  // running max (log2 units, lazily updated) and sum
      for (int j = 0; j < n; ++j) {
        const int g = gt + j;
        if (!warp_wait(&s_full[g & 1], (uint32_t)((g >> 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tS = tmem + lane_base + (uint32_t)((g & 1) * kBN);
        float sv[kBN];
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<float(*)[32]>(&sv[c * 32]));
        const int pid_now = pid0;
        pid0 = pid1;
        pid1 = load_pid(j + 2);
        tmem_wait_ld();
        const int64_t key0 = (it.t_begin + j) * kBN;
        // Only tiles that cross some row's last visible key (the causal diagonal, the
        // context end, rows past the unit) pay for the mask: one compare per score.
        const int64_t vis64 = last_key - key0;  // in-tile index of the row's last visible key
        if (__any_sync(0xffffffffu, vis64 < kBN - 1)) {
          const int vis = vis64 < -1 ? -1 : (int)vis64;
#pragma unroll
          for (int c = 0; c < kBN; ++c) sv[c] = c <= vis ? sv[c] : -INFINITY;
        }
        if (!p.dense) {  // holes: the 16-token groups of missing pages are masked
          const uint32_t holes =
              __ballot_sync(0xffffffffu, lane < kPagesPerTile && (pid_now < 0 || pid_now >= (int)p.P)) & 0xFu;
          if (holes != 0) {
#pragma unroll
            for (int gg = 0; gg < kPagesPerTile; ++gg) {
              if ((holes >> gg) & 1u) {
#pragma unroll
                for (int c = 0; c < 16; ++c) sv[gg * 16 + c] = -INFINITY;
              }
            }
          }
        }
        // row max as a tree of three-input maxima (8 independent chains of 8 scores, then
        // the 8 chain results): 36 instructions instead of 63
        float mv[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          float t = fmax3(sv[x], sv[8 + x], sv[16 + x]);
          t = fmax3(t, sv[24 + x], sv[32 + x]);
          t = fmax3(t, sv[40 + x], sv[48 + x]);
          mv[x] = fmaxf(t, sv[56 + x]);
        }
        const float mx = fmax3(fmax3(mv[0], mv[1], mv[2]), fmax3(mv[3], mv[4], mv[5]), fmaxf(mv[6], mv[7]));
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
        // p = 2^(s * sl2 - mu) on packed pairs, on the MUFU unit; outside split tiles the
        // pairs selected by kEmuPairs (none by default) run on the FMA pipe (exp2_fma2).
        const float2 sl2v = make_float2(sl2, sl2), nmu = make_float2(-mu, -mu);
        float2 acc[4];
#pragma unroll
        for (int x = 0; x < 4; ++x) acc[x] = make_float2(0.f, 0.f);
        if (split) {
#pragma unroll
          for (int q = 0; q < kBN / 2; ++q) {
            const float2 x2 = __ffma2_rn(make_float2(sv[2 * q], sv[2 * q + 1]), sl2v, nmu);
            const float2 e = make_float2(ex2_ftz(x2.x), ex2_ftz(x2.y));
            sv[2 * q] = e.x;
            sv[2 * q + 1] = e.y;
            acc[q & 3] = __fadd2_rn(acc[q & 3], e);
          }
        } else {
#pragma unroll
          for (int q = 0; q < kBN / 2; ++q) {
            const float2 x2 = __ffma2_rn(make_float2(sv[2 * q], sv[2 * q + 1]), sl2v, nmu);
            const float2 e = ((kEmuPairs >> q) & 1u) ? exp2_fma2<T>(x2) : make_float2(ex2_ftz(x2.x), ex2_ftz(x2.y));
            sv[2 * q] = e.x;
            sv[2 * q + 1] = e.y;
            acc[q & 3] = __fadd2_rn(acc[q & 3], e);
          }
        }
        const float2 a01 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
        // A row with no visible key yet keeps a zero sum (so it ends as zeros): exp2_fma2
        // turns its -inf scores into 2^-125, not 0.  Next to a visible key's p >= 2^-8,
        // 2^-125 is nothing.
        const float rs = m_ref == -INFINITY ? 0.f : a01.x + a01.y;
        lsum = (m == -INFINITY ? 0.f : lsum * alpha) + rs;
        m = m_ref;
        if (__any_sync(0xffffffffu, rescale)) {
          // O must hold PV_{j-1} before it is rescaled
          if (!warp_wait(&v_empty[(g - 1) % kVStages], (uint32_t)(((g - 1) / kVStages) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float f = rescale ? alpha : 1.f;
#pragma unroll 1
          for (int c = 0; c < kD / 32; ++c) {
            float ov[32];
            tmem_ld32(tO + lane_base + c * 32, ov);
            tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 32; ++x) ov[x] *= f;
            tmem_st32(tO + lane_base + c * 32, ov);
          }
        }
        // P over S_j's columns: packed pairs, hi in columns [0, kBN/2), lo (bf16 split) after
        {
          uint32_t hi[32];
#pragma unroll
          for (int x = 0; x < 32; ++x) hi[x] = cvt_pack<T>(sv[2 * x], sv[2 * x + 1]);
          tmem_st32u(tS, hi);
          if (split) {
            uint32_t lo[32];
#pragma unroll
            for (int x = 0; x < 32; ++x) {
              // bf16 -> f32 is exact: the bf16 bits become the high half of the f32
              const float h0 = __uint_as_float(hi[x] << 16), h1 = __uint_as_float(hi[x] & 0xFFFF0000u);
              lo[x] = cvt_pack<T>(sv[2 * x] - h0, sv[2 * x + 1] - h1);
            }
            tmem_st32u(tS + kBN / 2, lo);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[g & 1]);
      }
      if (!ok) break;
      gt += n;
      // Final O of the item: every PV done (item_done: one completion per item, so no
      // parity aliasing with the per-tile o_done phases).
      if (!warp_wait(item_done, iw & 1)) {
        ok = false;
        break;
      }
      ++iw;
      tc_fence_after();
      if (it.n_chunks_unit == 1) {
        const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
#pragma unroll 1
        for (int c1 = 0; c1 < kD; c1 += 64) {
          float ov2[64];
          tmem_ld32(tO + lane_base + c1, *reinterpret_cast<float(*)[32]>(&ov2[0]));
          tmem_ld32(tO + lane_base + c1 + 32, *reinterpret_cast<float(*)[32]>(&ov2[32]));
          tmem_wait_ld();
          if (c1 + 64 == kD) {  // O read out: the next item's first PV may overwrite it
            tc_fence_before();
            mbar_arrive(o_free);
          }
          if (staged) {
            stage32(ov2, c1, inv);
            stage32(ov2 + 32, c1 + 32, inv);
          } else if (row_ok) {
            store32(orow, ov2, c1, inv);
            store32(orow, ov2 + 32, c1 + 32, inv);
          }
        }
        if (staged) flush_staged(it);
      } else {
        // Split-K: leave this chunk's (m, l) and unnormalised O rows in the workspace ...
        const int64_t prow = (it.u * p.n_chunks + it.c) * p.rows_real + row;
        if (row_ok) p.part_ml[prow] = make_float2(m, lsum);  // m = -inf: no visible key in this chunk
#pragma unroll 1
        for (int c1 = 0; c1 < kD; c1 += 64) {
          float ov2[64];
          tmem_ld32(tO + lane_base + c1, *reinterpret_cast<float(*)[32]>(&ov2[0]));
          tmem_ld32(tO + lane_base + c1 + 32, *reinterpret_cast<float(*)[32]>(&ov2[32]));
          tmem_wait_ld();
          if (c1 + 64 == kD) {
            tc_fence_before();
            mbar_arrive(o_free);
          }
          if (row_ok) {
            float4* po = reinterpret_cast<float4*>(p.part_o + prow * kD + c1);
#pragma unroll
            for (int x = 0; x < 16; ++x) po[x] = make_float4(ov2[4 * x], ov2[4 * x + 1], ov2[4 * x + 2], ov2[4 * x + 3]);
          }
        }
        // ... and the unit's last chunk to finish merges them (log-sum-exp weights).
        __threadfence();
        named_barrier(1, 128);
        if (row == 0) *(volatile int*)last_flag = atomicAdd(&p.counters[it.u], 1) == (int)it.n_chunks_unit - 1;
        named_barrier(1, 128);
        const bool merge = *(volatile int*)last_flag != 0;
        named_barrier(1, 128);  // every thread has read the flag before it is reused
        if (merge) {
          __threadfence();
          const int64_t base = it.u * p.n_chunks * p.rows_real + row;  // + cc * rows_real
          const int nc = (int)it.n_chunks_unit;
          if (row_ok) {
            // the chunks' (m, l) with one round of loads, then log-sum-exp weights
            constexpr int kMaxC = 16;
            float wgt[kMaxC];
            float mxc = -INFINITY, lt = 0.f;
            if (nc <= kMaxC) {
              float2 mlc[kMaxC];
#pragma unroll
              for (int cc = 0; cc < kMaxC; ++cc)
                mlc[cc] = cc < nc ? __ldcg(&p.part_ml[base + cc * p.rows_real]) : make_float2(-INFINITY, 0.f);
#pragma unroll
              for (int cc = 0; cc < kMaxC; ++cc) mxc = fmaxf(mxc, mlc[cc].x);
#pragma unroll
              for (int cc = 0; cc < kMaxC; ++cc) {
                wgt[cc] = -1.f;  // chunk without a visible key: skipped
                if (mlc[cc].x != -INFINITY) {
                  wgt[cc] = exp2f(mlc[cc].x - mxc);
                  lt += mlc[cc].y * wgt[cc];
                }
              }
            } else {
              for (int64_t cc = 0; cc < nc; ++cc) mxc = fmaxf(mxc, __ldcg(&p.part_ml[base + cc * p.rows_real]).x);
              for (int64_t cc = 0; cc < nc; ++cc) {
                const float2 ml = __ldcg(&p.part_ml[base + cc * p.rows_real]);
                if (ml.x != -INFINITY) lt += ml.y * exp2f(ml.x - mxc);
              }
            }
            const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll 1
            for (int c0 = 0; c0 < kD; c0 += 32) {
              float acc2[32];
#pragma unroll
              for (int x = 0; x < 32; ++x) acc2[x] = 0.f;
              if (nc <= kMaxC) {
                // two chunks' rows in flight per round
#pragma unroll 1
                for (int cc = 0; cc < nc; cc += 2) {
                  float4 o4[2][8];
#pragma unroll
                  for (int j = 0; j < 2; ++j) {
                    const float4* po = reinterpret_cast<const float4*>(p.part_o + (base + (cc + j) * p.rows_real) * kD + c0);
#pragma unroll
                    for (int x = 0; x < 8; ++x) o4[j][x] = cc + j < nc ? __ldcg(po + x) : make_float4(0.f, 0.f, 0.f, 0.f);
                  }
#pragma unroll
                  for (int j = 0; j < 2; ++j) {
                    float w = -1.f;
#pragma unroll
                    for (int q = 0; q < kMaxC; ++q)
                      if (q == cc + j) w = wgt[q];
                    if (cc + j < nc && w >= 0.f) {
#pragma unroll
                      for (int x = 0; x < 8; ++x) {
                        acc2[4 * x] += w * o4[j][x].x;
                        acc2[4 * x + 1] += w * o4[j][x].y;
                        acc2[4 * x + 2] += w * o4[j][x].z;
                        acc2[4 * x + 3] += w * o4[j][x].w;
                      }
                    }
                  }
                }
              } else {
                for (int64_t cc = 0; cc < nc; ++cc) {
                  const float2 ml = __ldcg(&p.part_ml[base + cc * p.rows_real]);
                  if (ml.x == -INFINITY) continue;
                  const float w = exp2f(ml.x - mxc);
                  const float4* po = reinterpret_cast<const float4*>(p.part_o + (base + cc * p.rows_real) * kD + c0);
#pragma unroll
                  for (int x = 0; x < 8; ++x) {
                    const float4 o4 = __ldcg(po + x);
                    acc2[4 * x] += w * o4.x;
                    acc2[4 * x + 1] += w * o4.y;
                    acc2[4 * x + 2] += w * o4.z;
                    acc2[4 * x + 3] += w * o4.w;
                  }
                }
              }
              if (staged) stage32(acc2, c0, inv);
              else store32(orow, acc2, c0, inv);
            }
          }
          if (staged) flush_staged(it);
          if (row == 0) p.counters[it.u] = 0;  // tickets start at zero for the next call
        }
      }
    }
    if (!ok) {
      record_error(p.err, kDevErrFullWait);
      *(volatile int*)abort_flag = 1;
    }
  }

  // ------------------------------------------------------------------ teardown
  if (warp == 5 && lane == 0) {
    if (!mbar_wait(mma_done, 0)) record_error(p.err, kDevErrMmaWait);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  // the last CTA to leave resets the work counter for the next call
  if (threadIdx.x == 0 && p.work_counter != nullptr) {
    __threadfence();
    if (atomicAdd(p.exit_counter, 1) == (int)gridDim.x - 1) {
      *p.work_counter = 0;
      *p.exit_counter = 0;
    }
  }
}

// Work list for the persistent grid: every item with work, ordered by tile count, largest
// first (a counting sort; sizes >= kPlanBins - 1 share the first bin), so the dynamic
// fetch approximates longest-processing-time-first scheduling.  One CTA.
__global__ void __launch_bounds__(1024) sm100_plan_kernel(const Sm100Params p, int* list, int* count) {
  __shared__ int hist[kPlanBins];
  for (int i = threadIdx.x; i < kPlanBins; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int64_t item = threadIdx.x; item < p.n_items; item += blockDim.x) {
    const Item it = decode_item(p, item);
    if (!it.valid) continue;
    const int bin = kPlanBins - 1 - (it.n_tiles < kPlanBins - 1 ? it.n_tiles : kPlanBins - 1);
    atomicAdd(&hist[bin], 1);
  }
  __syncthreads();
  // Exclusive prefix sum of the bins, one bin per thread: a scan inside each warp, then
  // over the 32 warp totals (a serial loop over the 1024 bins by one thread took ~10 us).
  static_assert(kPlanBins == 1024, "one bin per thread of the 1024-thread plan CTA");
  __shared__ int wsum[32];
  {
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    const int v = hist[threadIdx.x];
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[wp] = x;
    __syncthreads();
    if (wp == 0) {
      int w = wsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      wsum[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int excl = x - v + (wp > 0 ? wsum[wp - 1] : 0);
    hist[threadIdx.x] = excl;
    if (threadIdx.x == kPlanBins - 1) *count = excl + v;
  }
  __syncthreads();
  for (int64_t item = threadIdx.x; item < p.n_items; item += blockDim.x) {
    const Item it = decode_item(p, item);
    if (!it.valid) continue;
    const int bin = kPlanBins - 1 - (it.n_tiles < kPlanBins - 1 ? it.n_tiles : kPlanBins - 1);
    list[atomicAdd(&hist[bin], 1)] = (int)item;
  }
}

// One opt-in to the dynamic shared memory size per kernel instantiation and device.
template <typename T>
int launch_typed(dim3 grid, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                 const CUtensorMap& to, const Sm100Params& p, cudaStream_t s) {
  static std::mutex mu;
  static uint64_t done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !(done & (1ull << dev))) {
      int r = check_cuda(cudaFuncSetAttribute(flash_sm100_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kSmemBytes),
                         "flash_attention: cudaFuncSetAttribute");
      if (r != NVM_OK) return r;
      done |= 1ull << dev;
    }
  }
  flash_sm100_kernel<T><<<grid, kThreads, kSmemBytes, s>>>(tq, tk, tv, to, p);
  return check_cuda(cudaGetLastError(), "flash_attention: sm100 kernel launch");
}

}  // namespace

// Workspace of a paged call: tickets + counters (1 MiB), the work list, then the split-K
// partials (m, l) and O.
struct WsOffsets {
  size_t list, ml, o, total;
};
WsOffsets sm100_ws_offsets(const Sm100Plan& plan) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  WsOffsets w{};
  const size_t items = (size_t)(plan.n_units * plan.n_chunks);
  w.list = kSm100CounterBytes;
  w.ml = w.list + al(items * sizeof(int));
  w.o = w.ml;
  w.total = w.ml;
  if (plan.n_chunks > 1) {
    w.o = w.ml + al(items * (size_t)plan.rows_real * sizeof(float2));
    w.total = w.o + items * (size_t)plan.rows_real * kD * sizeof(float);
  }
  return w;
}

Sm100Plan plan_sm100(const PagedArgs& a, bool sizing_only) {
  Sm100Plan plan{};
  plan.eligible = false;
  if (a.kv_dtype != NVM_F16 && a.kv_dtype != NVM_BF16) return plan;
  if (!sizing_only && a.q_dtype != a.kv_dtype) return plan;
  if (a.D != kD) return plan;
  if (!sizing_only && !(a.scale > 0.f)) return plan;  // the softmax takes row maxima before scaling
  if (a.dense) {
    if (a.page_size < kBN) return plan;  // dense boxes are kBN rows
  } else if (a.page_size != 16) {
    return plan;
  }
  if (a.P <= 0 || a.P >= INT32_MAX || a.B * a.Hq > INT32_MAX) return plan;
  if (!sizing_only) {
    auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    if (a.out_dtype != NVM_F32 && a.out_dtype != NVM_F16 && a.out_dtype != NVM_BF16) return plan;
    if (!(al16(a.q) && al16(a.k_pages) && al16(a.v_pages) && al16(a.out))) return plan;
  }
  const int64_t g = a.Hq / a.Hkv;
  // Prefill: >= 64 query rows per head.  Grouped: 2..63 query tokens with >= 16 rows per
  // kv head (g*L); fewer rows stay on the mma.sync decode kernel, which is HBM-bound there.
  const int64_t min_rows = env_int("NVM_SM100_GROUPED_MIN_ROWS", 16);
  if (a.L >= 64) {
    plan.grouped = 0;
    plan.M_rows = a.L;
    plan.n_outer = a.B * a.Hq;
  } else if ((a.L > 1 || min_rows <= g) && g * a.L >= min_rows && env_int("NVM_SM100_GROUPED", 1) != 0) {
    plan.grouped = 1;
    plan.M_rows = g * a.L;
    plan.n_outer = a.B * a.Hkv;
  } else {
    return plan;
  }
  if (plan.M_rows >= INT32_MAX) return plan;  // the item decode divides in 32 bits
  plan.n_row_tiles = (plan.M_rows + kBM - 1) / kBM;
  plan.n_units = plan.n_outer * plan.n_row_tiles;
  plan.rows_real = plan.M_rows < kBM ? plan.M_rows : kBM;
  const int64_t keys = a.dense ? a.page_size : a.max_pages * a.page_size;
  const int64_t tiles_max = (keys + kBN - 1) / kBN;
  if (tiles_max >= INT32_MAX / 2) return plan;
  plan.ct = tiles_max > 0 ? tiles_max : 1;
  plan.n_chunks = 1;
  // Split-K over keys for grouped paged calls (dense callers pass no workspace): aim at
  // a few CTAs per SM slot if every sequence were max_pages long; units whose context is
  // shorter leave their later chunks empty (those CTAs return at once).
  if (plan.grouped && !a.dense && plan.n_units <= kMaxTicketUnits) {
    int64_t ct = env_int("NVM_SM100_CHUNK_TILES", 0);
    if (ct <= 0) {
      const int64_t target = 148 * 2 * 4;
      ct = (plan.n_units * tiles_max + target - 1) / target;
      if (ct < 8) ct = 8;
    }
    if (ct < tiles_max) {
      plan.ct = ct;
      plan.n_chunks = (tiles_max + ct - 1) / ct;
    }
  }
  if (plan.n_units * plan.n_chunks > INT32_MAX) return plan;
  plan.ws_bytes = 0;
  // Paged calls take their work items from a counter in the workspace (dense callers
  // pass none and walk items by CTA index).
  if (!a.dense) plan.ws_bytes = sm100_ws_offsets(plan).total;
  plan.eligible = true;
  return plan;
}

int launch_sm100(const PagedArgs& a, const Sm100Plan& plan, void* ws, cudaStream_t s) {
  const CUtensorMapDataType dt = a.kv_dtype == NVM_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  // Q as [n_outer, M_rows, D] -> (D, M_rows, n_outer), 64 x 128 boxes (rows past a unit's end are
  // outside the map and load as zeros)
  const uint64_t qd[3] = {(uint64_t)kD, (uint64_t)plan.M_rows, (uint64_t)plan.n_outer};
  const uint64_t qs[2] = {kD * 2, (uint64_t)plan.M_rows * kD * 2};
  const uint32_t qb[3] = {64u, (uint32_t)kBM, 1u};
  CUtensorMap tq, tk, tv;
  int st = encode_tmap(&tq, dt, 3, a.q, qd, qs, qb, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVM_OK) return st;
  // pools [P, Hkv, ps, D] -> (D, ps, Hkv, P)
  const int box_rows = a.dense ? kBN : 16;  // dense: one box per 64-key half tile
  const uint64_t kd[4] = {(uint64_t)kD, (uint64_t)a.page_size, (uint64_t)a.Hkv, (uint64_t)a.P};
  const uint64_t ks[3] = {kD * 2, (uint64_t)a.page_size * kD * 2, (uint64_t)(a.Hkv * a.page_size) * kD * 2};
  const uint32_t kb[4] = {64u, (uint32_t)box_rows, 1u, 1u};
  st = encode_tmap(&tk, dt, 4, a.k_pages, kd, ks, kb, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVM_OK) return st;
  st = encode_tmap(&tv, dt, 4, a.v_pages, kd, ks, kb, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVM_OK) return st;
  // out, same [n_outer, M_rows, D] view, boxes of 128 bytes of columns x 128 rows
  CUtensorMap to;
  {
    const int esz = a.out_dtype == NVM_F32 ? 4 : 2;
    const CUtensorMapDataType odt = a.out_dtype == NVM_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                    : a.out_dtype == NVM_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                             : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint64_t od[3] = {(uint64_t)kD, (uint64_t)plan.M_rows, (uint64_t)plan.n_outer};
    const uint64_t os[2] = {(uint64_t)kD * esz, (uint64_t)plan.M_rows * kD * esz};
    const uint32_t ob[3] = {(uint32_t)(128 / esz), (uint32_t)kBM, 1u};
    st = encode_tmap(&to, odt, 3, a.out, od, os, ob, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != NVM_OK) return st;
  }

  Sm100Params p{};
  p.out = a.out; p.block_table = a.block_table; p.context_lens = a.context_lens; p.err = device_error_word();
  p.out_dtype = a.out_dtype;
  p.B = a.B; p.Hq = a.Hq; p.Hkv = a.Hkv; p.L = a.L; p.P = a.P; p.ps = a.page_size; p.mp = a.max_pages;
  p.dense_ctx = a.dense_ctx;
  p.n_row_tiles = plan.n_row_tiles;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.causal = a.is_causal; p.dense = a.dense; p.box_rows = box_rows;
  p.split_below = env_int("NVM_SM100_SPLIT_BELOW", kSplitBelowKeys);  // tuning: 0 = never, huge = always
  p.grouped = plan.grouped;
  p.g = a.Hq / a.Hkv;
  p.M_rows = plan.M_rows; p.n_outer = plan.n_outer; p.n_units = plan.n_units;
  p.ct = plan.ct; p.n_chunks = plan.n_chunks; p.rows_real = plan.rows_real;
  p.n_items = plan.n_units * plan.n_chunks;
  if (ws != nullptr && plan.ws_bytes > 0) {
    p.work_counter = reinterpret_cast<int*>(ws) + (kSm100CounterBytes / sizeof(int) - 2);
    p.exit_counter = p.work_counter + 1;
  }
  const WsOffsets wo = sm100_ws_offsets(plan);
  if (plan.n_chunks > 1) {
    uint8_t* w = static_cast<uint8_t*>(ws);
    p.counters = reinterpret_cast<int*>(w);
    p.part_ml = reinterpret_cast<float2*>(w + wo.ml);
    p.part_o = reinterpret_cast<float*>(w + wo.o);
  }

  // Grouped (decode-like) calls: persistent grid of two CTAs per SM taking items from the
  // work counter, so skewed contexts balance and item prologues overlap.  Prefill: one CTA
  // per item (the hardware scheduler balances the heavy-first causal tiles), which lets
  // the epilogue stage O in shared memory for bulk tensor stores.
  int64_t ctas = p.n_items;
  const int64_t persistent = env_int("NVM_SM100_PERSISTENT", plan.grouped ? 1 : 0);
  if (persistent != 0) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (ctas > 2 * (int64_t)sms) ctas = 2 * (int64_t)sms;
  }
  p.stage_out = ctas == p.n_items ? 1 : 0;
  p.pv_wait = env_int("NVM_SM100_PV_WAIT", 1) != 0 ? 1 : 0;
  if (p.stage_out) p.work_counter = p.exit_counter = nullptr;  // one item per CTA: item = blockIdx.x
  if (p.work_counter != nullptr && env_int("NVM_SM100_PLAN", 1) != 0) {
    int* list = reinterpret_cast<int*>(static_cast<uint8_t*>(ws) + wo.list);
    int* count = p.work_counter - 1;
    p.item_list = list;
    p.item_count = count;
    sm100_plan_kernel<<<1, 1024, 0, s>>>(p, list, count);
    const int st2 = check_cuda(cudaGetLastError(), "paged_attention: sm100 plan kernel launch");
    if (st2 != NVM_OK) return st2;
  }
  const dim3 grid((unsigned)ctas);
  if (a.kv_dtype == NVM_F16) return launch_typed<__half>(grid, tq, tk, tv, to, p, s);
  return launch_typed<__nv_bfloat16>(grid, tq, tk, tv, to, p, s);
}
}  // namespace nvm
