// Tree-masked paged attention on sm_100a (TMA + tcgen05 + TMEM).
//
// Work unit: request b, KV head h and a group of up to 264 query rows.  Query
// rows are (tree node, query head of h's GQA group) pairs, head fastest.  Rows
// 0-255 of the group form two 128-row tensor-core tiles; the remaining up to 8
// rows (for example the 65th node of a 65-node tree with 4 heads per KV head)
// run on mma.sync from the same staged K/V.
//
// Schedule.  With a workspace of pts_tree_attn_workspace_size bytes the grid
// is persistent (one CTA per SM) and the units' 64-token KV blocks, laid end to
// end, are cut into equal contiguous ranges, one per CTA: 16 requests x 8 KV
// heads = 128 units of 65 blocks keep all 148 SMs busy for 56 blocks each
// instead of 128 SMs for 65.  A CTA runs its range as segments (the part of a
// unit inside the range) through one pipeline: the ring, the barriers' phases
// and the TMA producer run on across segments, so the next segment's K/V is in
// flight while the current one finishes.  A unit cut by a range boundary is
// finished by the last CTA to reach its end: each CTA takes an arrival ticket
// on the unit's counter; all but the last write their unnormalised fp32 output
// rows with the row max and sum (a partial) and raise a flag; the last waits
// only for those flags (every writer has already arrived, so no wait depends
// on a CTA that has not started), merges the partials in CTA order (the same
// result whichever CTA is last) and writes the rows.  With a smaller workspace
// the grid is one CTA per unit.
//
// Per 64-token KV block (four 16-token pages), 16 warps:
//   warp 14           TMA producer: lane w loads page w of the block (K and V,
//                     two 64-column halves each, 128-byte swizzle) into a
//                     4-stage ring as soon as a stage is free;
//   warps 10-13       remainder rows (when there are any): warp 10 + w takes
//                     page w of every block, transposed on mma.sync m16n8k16:
//                     S^T = K Q^T (16 tokens x 8 rows per warp), P^T handed to
//                     the next MMA by movmatrix, O^T += V^T P^T, each warp with
//                     its own running max/sum, the four partials merged at the
//                     end;
//   warps 1 and 0     one MMA issuer per tile: S_t = Q_t K^T with Q_t resident in
//                     TMEM (A from TMEM, M=128, N=64, K=128), O_t += P_t V with
//                     P_t in shared memory (M=128, N=128, K=64).  The scores of
//                     block j+1 are issued as soon as the softmax warps have
//                     copied S_t(j) into registers, so the tensor pipe computes
//                     them while the exponentials of block j run;
//   warps 2-5, 6-9    one softmax warpgroup per tile: one thread per row reads
//                     its 64 scores with a single TMEM load, applies the scale
//                     and the tree mask, keeps a running max and sum (O_t is
//                     rescaled in TMEM only when the max grows by more than
//                     2^8), writes P_t as bf16 into one of two shared-memory
//                     buffers in the MMA's 128-byte-swizzled layout, and at the
//                     end normalises O_t;
//   warp 15           builds the schedule table, then idle.
// TMEM (512 columns): Q_t at 64t, S_t at 128 + 64t, O_t at 256 + 128t.  Q and
// the output pass through the tile's P buffers so that their global accesses
// are whole rows (512 contiguous bytes per warp instruction).
//
// The tree mask: KV slots below kv_len - N are the prefix (always visible);
// slot kv_len - N + j is visible to row i when bit j of i's mask is set.
// Without a mask the rows are causal: row i sees slots up to kv_len - N + i.
// Every barrier wait is bounded; on timeout the CTA records an error, drains
// its own tensor-core work and TMA copies, frees TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "sm100.cuh"

namespace pts {
namespace {

using namespace sm100;

constexpr int kStages = 4;
constexpr int kBlockN = 64;           // KV tokens per block
constexpr int kPage = 16;
constexpr int kD = 128;
constexpr int kTensorRows = 256;      // two 128-row tiles
constexpr int kSyncRows = 8;          // remainder rows on mma.sync (the N of its MMAs)
constexpr int kGroupRows = kTensorRows + kSyncRows;
constexpr int kThreads = 512;         // warps 0-1 MMA, 2-9 softmax, 10-13 remainder rows, 14 TMA, 15 idle
constexpr int kSyncWarps = 4;
constexpr int kRemWarp0 = 10;
constexpr int kProducerWarp = 14;
constexpr int kScheduleWarp = 15;
constexpr uint32_t kKvHalf = kBlockN * 128;                   // [64 tokens x 64 dims] bf16
constexpr uint32_t kStageBytes = 4 * kKvHalf;                 // K0 K1 V0 V1
constexpr uint32_t kPBytes = 128 * kBlockN * 2;               // one P buffer: [128 rows x 64 tokens] bf16
constexpr float kRescaleThreshold = 8.0f;
constexpr uint32_t kColQ = 0, kColS = 128, kColO = 256;
constexpr int kKvConsumers = 2 + kSyncWarps;  // arrivals that free a K/V stage: both issuers, the remainder warps

// Balanced schedule.  Table entries are requests (or (request, KV head) pairs
// with per-head page tables); a CTA's range is at least kMinBlocksPerCta blocks
// and long enough that a unit spans at most kMaxSpan CTAs, which bounds what
// the last CTA of a unit reads back.
constexpr int kMaxEntries = 1024;
constexpr int kMinBlocksPerCta = 4;
constexpr int kMaxSpan = 4;
// A partial (one slot): fp32 O of the 256 tile rows as [32 column quads][256
// rows] float4 (a warp's stores are 512 contiguous bytes), the rows' max and
// sum, and the remainder rows as [36][32 lanes] (per lane 32 O + 2 m + 2 l in
// the mma.sync fragment layout).  Two slots per CTA: its first segment (when
// it began before the range) and its last (when it ends after it).
constexpr uint32_t kSlotTileBytes = 32u * 256u * 16u;
constexpr uint32_t kSlotStatBytes = 2u * 256u * 4u;
constexpr uint32_t kSlotRemBytes = 36u * 32u * 4u;
constexpr uint32_t kSlotBytes = kSlotTileBytes + kSlotStatBytes + kSlotRemBytes;
static_assert(kSlotBytes % 256 == 0, "slots stay 256-byte aligned");

struct __align__(8) Bars {
  uint64_t q_ready[2];   // Q_t of the segment in TMEM          (4 softmax warps)
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];    // S_t(j) computed                  (tcgen05.commit)
  uint64_t s_free[2];    // S_t(j) copied out of TMEM          (4 softmax warps)
  uint64_t p_full[2];    // P_t(j) in shared memory, O_t ready (4 softmax warps)
  uint64_t p_empty[2][2];  // PV_t(j) done (O_t may be rescaled)      (tcgen05.commit)
  uint64_t o_full[2];    // every MMA of the tile's segment done   (tcgen05.commit)
  uint64_t drain[2];
  uint32_t tmem;
  int abort;
};

// The balanced schedule's table (warp 15 builds it): entry e covers blocks
// start[e] .. start[e+1] of the end-to-end order, units of nblk[e] blocks.
struct Sched {
  int total;             // blocks of all units
  int ctas;              // CTAs with a range (the rest exit)
  int max_nblk;
  int start[kMaxEntries + 1];
  int nblk[kMaxEntries];
};

constexpr uint32_t kOffKV = 0;
constexpr uint32_t kOffP = kOffKV + kStages * kStageBytes;        // 1024-aligned (swizzle atoms)
constexpr uint32_t kOffMerge = kOffP + 4 * kPBytes;                // remainder partials of warps 11-13
constexpr uint32_t kMergeFloats = 36;                             // per lane: 32 O + 2 m + 2 l
constexpr uint32_t kOffBars = kOffMerge + (kSyncWarps - 1) * 32 * kMergeFloats * 4;
constexpr uint32_t kOffSched = kOffBars + 512;
constexpr uint32_t kSmemBytes = kOffSched + (uint32_t)sizeof(Sched) + 1024;   // + alignment slack
static_assert(sizeof(Bars) <= 512, "barrier block");
static_assert(kOffP % 1024 == 0, "P tiles must sit on 1024-byte swizzle atoms");
static_assert(kSmemBytes <= 232448, "shared memory above the 227 KB per-CTA limit");

struct AttnParams {
  const uint16_t* q;
  const int32_t* qo_indptr;
  const int32_t* page_indptr;
  const int32_t* page_indices;
  const int32_t* last_page_len;
  const uint64_t* mask_bits;
  int mask_words;
  uint16_t* out;
  int Hq, Hkv, g;
  int head_pages;          // page tables per (request, KV head) instead of per request
  int max_pages;
  float scale_log2;
  int* err;
  long long wait_limit;    // SM clocks a progress wait may take before the CTA gives up
  int balanced;            // 1: balanced ranges over gridDim.x CTAs; 0: one unit per CTA (grid Hkv x B x groups)
  int n_entries;           // balanced: requests, or requests x KV heads with per-head page tables
  Sched* sched_out;        // balanced: CTA 0's copy of the schedule table, for the merge kernel
  float* part;             // balanced: the partial slots
};

// The part of one unit that one CTA computes.
struct Segment {
  int b, h, group;
  int q0, n_nodes, row0, tensor_rows, n_tiles, sync_rows;
  int p0, n_pages, kv_len, prefix;
  int ja, jb;              // blocks ja .. jb-1 of the unit
  int split;               // other CTAs compute the rest of the unit
  int slot;                // split: this CTA's partial slot
};

// Fills the unit's shape; false when it has no rows or no KV.
__device__ __forceinline__ bool fill_unit(const AttnParams& p, int b, int h, int group, Segment& s) {
  s.b = b;
  s.h = h;
  s.group = group;
  s.q0 = p.qo_indptr[b];
  s.n_nodes = p.qo_indptr[b + 1] - s.q0;
  const int rows = s.n_nodes * p.g;
  s.row0 = group * kGroupRows;
  if (s.row0 >= rows) return false;
  const int rows_here = min(kGroupRows, rows - s.row0);
  s.tensor_rows = min(kTensorRows, rows_here);
  s.n_tiles = (s.tensor_rows + 127) / 128;
  s.sync_rows = rows_here - s.tensor_rows;
  const int pt = p.head_pages ? b * p.Hkv + h : b;
  s.p0 = p.page_indptr[pt];
  s.n_pages = p.page_indptr[pt + 1] - s.p0;
  if (s.n_pages <= 0) return false;
  s.kv_len = (s.n_pages - 1) * kPage + p.last_page_len[pt];
  s.prefix = s.kv_len - s.n_nodes;
  return s.kv_len > 0;
}

// The CTA of the balanced schedule whose range holds block x.
__device__ __forceinline__ int cta_of(const Sched& S, int x) {
  return (int)(((long long)(x + 1) * S.ctas - 1) / S.total);
}
__device__ __forceinline__ int range_begin(const Sched& S, int c) { return (int)((long long)c * S.total / S.ctas); }

// The unit holding block `pos` of the end-to-end order: its first block, its
// length and its (request, KV head, row group).
__device__ __forceinline__ void locate_unit(const AttnParams& p, const Sched& S, int pos, int& first, int& nb,
                                            int& b, int& h, int& group) {
  int lo = 0, hi = p.n_entries;                     // start[lo] <= pos < start[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (S.start[mid] <= pos) lo = mid;
    else hi = mid;
  }
  const int e = lo;
  nb = S.nblk[e];
  const int u = (pos - S.start[e]) / nb;
  first = S.start[e] + u * nb;
  if (p.head_pages) {
    b = e / p.Hkv;
    h = e % p.Hkv;
    group = u;
  } else {
    const int groups = (S.start[e + 1] - S.start[e]) / nb / p.Hkv;
    b = e;
    h = u / groups;
    group = u % groups;
  }
}

// Segment k of this CTA (k = 0, 1, ... while it returns true).  `pos` carries
// the position in the end-to-end block order from one call to the next.
template <bool kBalanced>
__device__ bool next_segment(const AttnParams& p, const Sched& S, int k, int& pos, Segment& s) {
  if constexpr (!kBalanced) {
    if (k > 0) return false;
    if (!fill_unit(p, blockIdx.y, blockIdx.x, blockIdx.z, s)) return false;
    s.ja = 0;
    s.jb = (s.kv_len + kBlockN - 1) / kBlockN;
    s.split = 0;
    return true;
  }
  const int c = blockIdx.x;
  const int begin = range_begin(S, c), end = range_begin(S, c + 1);
  if (k == 0) pos = begin;
  if (pos >= end) return false;
  int first, nb, b, h, group;
  locate_unit(p, S, pos, first, nb, b, h, group);
  fill_unit(p, b, h, group, s);
  s.ja = pos - first;
  s.jb = min(first + nb, end) - first;
  s.split = first < begin || first + nb > end;
  s.slot = first < begin ? 2 * c : 2 * c + 1;
  pos = first + s.jb;
  return true;
}

// The partial slot of CTA c for a unit whose first CTA is c_first.
__device__ __forceinline__ int slot_of(int c, int c_first) { return c == c_first ? 2 * c + 1 : 2 * c; }

// Warp 15: per entry its blocks per unit and the running block count; then
// how many CTAs get a range.
__device__ void build_schedule(const AttnParams& p, Sched& S, int lane) {
  int run = 0, mx = 0;
  for (int e0 = 0; e0 < p.n_entries; e0 += 32) {
    const int e = e0 + lane;
    int cnt = 0, nb = 0;
    if (e < p.n_entries) {
      const int b = p.head_pages ? e / p.Hkv : e;
      const int n_nodes = p.qo_indptr[b + 1] - p.qo_indptr[b];
      const int groups = (n_nodes * p.g + kGroupRows - 1) / kGroupRows;
      const int n_pages = p.page_indptr[e + 1] - p.page_indptr[e];      // page table e in both layouts
      const int kv_len = n_pages > 0 ? (n_pages - 1) * kPage + p.last_page_len[e] : 0;
      nb = (n_nodes > 0 && kv_len > 0) ? (kv_len + kBlockN - 1) / kBlockN : 0;
      cnt = nb * groups * (p.head_pages ? 1 : p.Hkv);
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (e < p.n_entries) {
      S.start[e + 1] = run + incl;
      S.nblk[e] = nb;
    }
    run += __shfl_sync(0xffffffffu, incl, 31);
    mx = max(mx, nb);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) {
    S.start[0] = 0;
    S.total = run;
    S.max_nblk = mx;
    // ranges of at least kMinBlocksPerCta blocks, and long enough that a unit
    // spans at most kMaxSpan CTAs
    const int chunk = max(kMinBlocksPerCta, (mx + kMaxSpan - 2) / (kMaxSpan - 1));
    S.ctas = run > 0 ? max(1, min((int)gridDim.x, run / chunk)) : 0;
  }
}

__device__ __forceinline__ void record_abort(Bars& bars, const AttnParams& p, int code) {
  *(volatile int*)&bars.abort = 1;
  if (p.err) atomicExch(p.err, code);
}

__device__ __forceinline__ bool aborted(const Bars& bars) { return *(volatile const int*)&bars.abort != 0; }

// Named barrier `id` over `count` threads: wait for it / arrive without waiting.
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ uint64_t low_bits(int n) {          // n in [0, 64]
  return n >= 64 ? ~0ull : ((1ull << n) - 1ull);
}

// Visibility of the 64 KV slots kv0 .. kv0+63 to tree row `node` (bit c = slot
// kv0 + c): the prefix is visible, tree slot j is visible when bit j of the
// row's mask is set (j <= node without a mask), slots past kv_len are not.
__device__ __forceinline__ uint64_t block_visibility(const AttnParams& p, const uint64_t* mrow, int node, int kv0,
                                                     int kv_len, int prefix) {
  const int np = prefix - kv0;
  if (np >= kBlockN) return ~0ull;
  uint64_t v = np > 0 ? low_bits(np) : 0ull;
  const int c0 = max(np, 0);
  const int cend = min(kBlockN, kv_len - kv0);
  if (c0 < cend) {
    const int tn0 = kv0 + c0 - prefix;                           // tree slot of bit c0
    uint64_t bits;
    if (p.mask_bits == nullptr) {
      bits = low_bits(max(0, min(64, node - tn0 + 1)));
    } else {
      const int w = tn0 >> 6, sh = tn0 & 63;
      const uint64_t lo = w < p.mask_words ? __ldg(mrow + w) : 0ull;
      const uint64_t hi = (w + 1) < p.mask_words ? __ldg(mrow + w + 1) : 0ull;
      bits = sh ? ((lo >> sh) | (hi << (64 - sh))) : lo;
    }
    v |= (bits & low_bits(cend - c0)) << c0;
  }
  return v;
}

// block_visibility with the row's first two mask words held in registers
// (trees of up to 128 rows); wider masks read the rest from memory.
__device__ __forceinline__ uint64_t block_visibility_reg(const AttnParams& p, const uint64_t* mrow, uint64_t w0,
                                                         uint64_t w1, int node, int kv0, int kv_len, int prefix) {
  const int np = prefix - kv0;
  if (np >= kBlockN) return ~0ull;
  uint64_t v = np > 0 ? low_bits(np) : 0ull;
  const int c0 = max(np, 0);
  const int cend = min(kBlockN, kv_len - kv0);
  if (c0 < cend) {
    const int tn0 = kv0 + c0 - prefix;                           // tree slot of bit c0
    uint64_t bits;
    if (p.mask_bits == nullptr) {
      bits = low_bits(max(0, min(64, node - tn0 + 1)));
    } else {
      const int w = tn0 >> 6, sh = tn0 & 63;
      auto word = [&](int k) -> uint64_t {
        if (k >= p.mask_words) return 0ull;
        return k == 0 ? w0 : k == 1 ? w1 : __ldg(mrow + k);
      };
      const uint64_t lo = word(w), hi = word(w + 1);
      bits = sh ? ((lo >> sh) | (hi << (64 - sh))) : lo;
    }
    v |= (bits & low_bits(cend - c0)) << c0;
  }
  return v;
}

// Byte offset of (row, 16-byte chunk) in a 128-byte-swizzled [rows x 64] tile.
__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

template <bool kBalanced>
__global__ void __launch_bounds__(kThreads, 1)
    tree_attn_kernel(const AttnParams p, const __grid_constant__ CUtensorMap kv_map) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  Bars& bars = *reinterpret_cast<Bars*>(smem + kOffBars);
  Sched& S = *reinterpret_cast<Sched*>(smem + kOffSched);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // launched as a programmatic dependent: resident early, reads nothing before
  // the previous kernel (the tree preparation and K/V append) has completed
  pdl_wait();
  if constexpr (kBalanced) {
    if (warp == kScheduleWarp) {
      build_schedule(p, S, lane);
      __syncwarp();
      if (blockIdx.x == 0) {                            // the table for the merge kernel
        if (lane == 0) {
          p.sched_out->total = S.total;
          p.sched_out->ctas = S.ctas;
          p.sched_out->max_nblk = S.max_nblk;
        }
        for (int e = lane; e <= p.n_entries; e += 32) p.sched_out->start[e] = S.start[e];
        for (int e = lane; e < p.n_entries; e += 32) p.sched_out->nblk[e] = S.nblk[e];
      }
    }
    __syncthreads();
    if ((int)blockIdx.x >= S.ctas) return;            // no range (uniform over the CTA)
  } else {
    Segment s0;
    int pos0 = 0;
    if (!next_segment<kBalanced>(p, S, 0, pos0, s0)) return;     // no rows or no KV
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars.kv_full[s], 4);                   // one expect_tx arrival per producer lane (page)
      mbar_init(&bars.kv_empty[s], kKvConsumers);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars.q_ready[t], 4);
      mbar_init(&bars.s_full[t], 1);
      mbar_init(&bars.s_free[t], 4);
      mbar_init(&bars.p_full[t], 4);
      mbar_init(&bars.p_empty[t][0], 1);
      mbar_init(&bars.p_empty[t][1], 1);
      mbar_init(&bars.o_full[t], 1);
      mbar_init(&bars.drain[t], 1);
    }
    bars.abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&kv_map);
  }
  if (warp == 1) {
    tmem_alloc(&bars.tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem;

  if (warp == 0 || warp == 1) {
    // ------------------------------------------------------------ MMA issuers, one warp per tile
    // Counters that run on across segments: jg blocks through the ring, jt
    // blocks and st segments of this tile (the tile's barrier phases).
    const int t = warp == 1 ? 0 : 1;
    const uint32_t id_qk = idesc_bf16_f32(128, kBlockN, 0, 0);
    const uint32_t id_pv = idesc_bf16_f32(128, kD, 0, 1);
    const uint64_t kd0 = smem_desc(smem_u32(smem + kOffKV), 16, 1024, kSwizzle128B);
    const uint64_t vd0 = smem_desc(smem_u32(smem + kOffKV + 2 * kKvHalf), kKvHalf, 1024, kSwizzle128B);
    const uint64_t pd0 = smem_desc(smem_u32(smem + kOffP + 2 * t * kPBytes), 16, 1024, kSwizzle128B);
    const uint32_t s_col = tmem + kColS + 64 * t, q_col = tmem + kColQ + 64 * t, o_col = tmem + kColO + 128 * t;
    const bool leader = elect_one();
    auto issue_qk = [&](int stage) {
      if (leader) {
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const uint64_t bd = kd0 + (uint64_t)((stage * kStageBytes + (k / 4) * kKvHalf + (k % 4) * 32) >> 4);
          mma_bf16_ts(s_col, q_col + 8 * k, bd, id_qk, k > 0);
        }
        mma_commit(&bars.s_full[t]);
      }
      __syncwarp();
    };
    bool ok = true, issued = false;
    int jg = 0, jt = 0, st = 0, pos = 0;
    Segment sg;
    for (int k = 0; next_segment<kBalanced>(p, S, k, pos, sg); ++k) {
      const int nb = sg.jb - sg.ja;
      if (ok && __any_sync(0xffffffffu, aborted(bars))) ok = false;
      if (t >= sg.n_tiles) {
        // not in this segment: release each stage once it has been filled
        for (int j = 0; ok && j < nb; ++j) {
          const int g = jg + j;
          ok = __all_sync(0xffffffffu, mbar_wait(&bars.kv_full[g % kStages], (g / kStages) & 1, p.wait_limit) &&
                                           !aborted(bars));
          if (!ok) {
            if (lane == 0) record_abort(bars, p, 25);
          } else if (lane == 0) {
            mbar_arrive(&bars.kv_empty[g % kStages]);
          }
          __syncwarp();
        }
        jg += nb;
        continue;
      }
      if (ok) {
        ok = mbar_wait(&bars.q_ready[t], st & 1, p.wait_limit) &&
             mbar_wait(&bars.kv_full[jg % kStages], (jg / kStages) & 1, p.wait_limit);
        if (!ok && lane == 0) record_abort(bars, p, 21);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok) {
        tc_fence_after();
        issue_qk(jg % kStages);
      }
      for (int j = 0; ok && j < nb; ++j) {
        const int g = jg + j, tj = jt + j, ss = g % kStages;
        if (j + 1 < nb) {
          // scores of block j+1 once K(j+1) is staged and S_t(j) has been read
          const int s1 = (g + 1) % kStages;
          const bool w_ok = mbar_wait(&bars.kv_full[s1], ((g + 1) / kStages) & 1, p.wait_limit) &&
                            mbar_wait(&bars.s_free[t], tj & 1, p.wait_limit) && !aborted(bars);
          if (!__all_sync(0xffffffffu, w_ok)) {
            if (lane == 0) record_abort(bars, p, 23);
            ok = false;
            break;
          }
          tc_fence_after();
          issue_qk(s1);
        }
        const bool w_ok = mbar_wait(&bars.p_full[t], tj & 1, p.wait_limit) && !aborted(bars);
        if (!__all_sync(0xffffffffu, w_ok)) {
          if (lane == 0) record_abort(bars, p, 24);
          ok = false;
          break;
        }
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < kBlockN / 16; ++kk) {
            const uint64_t ad = pd0 + (uint64_t)(((tj & 1) * kPBytes + kk * 32) >> 4);
            const uint64_t bd = vd0 + (uint64_t)((ss * kStageBytes + kk * 2048) >> 4);
            mma_bf16_ss(o_col, ad, bd, id_pv, (j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&bars.p_empty[t][tj & 1]);
          mma_commit(&bars.kv_empty[ss]);
        }
        __syncwarp();
      }
      if (leader) mma_commit(&bars.o_full[t]);
      __syncwarp();
      issued = true;
      jg += nb;
      jt += nb;
      ++st;
    }
    if (issued) {
      if (leader) mma_commit(&bars.drain[t]);
      __syncwarp();
      mbar_wait(&bars.drain[t], 0);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ softmax warpgroups
    const int t = (warp - 2) >> 2;                      // tile of this warpgroup
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t prow = smem_u32(smem + kOffP + 2 * t * kPBytes) + r_local * 128;   // this row of P_t, buffer 0
    const uint32_t pswz = (uint32_t)(r_local & 7);
    bool cta_ok = true;
    bool owed = false;                                  // tile 1's last turn not yet taken by tile 0
    int jt = 0, st = 0, pos = 0;                        // this tile's blocks and segments so far
    Segment sg;
    for (int k = 0; next_segment<kBalanced>(p, S, k, pos, sg); ++k) {
    const int q0 = sg.q0, h = sg.h, row0 = sg.row0, tensor_rows = sg.tensor_rows, n_tiles = sg.n_tiles;
    const int kv_len = sg.kv_len, prefix = sg.prefix, nb = sg.jb - sg.ja;
    const int R = row0 + t * 128 + r_local;             // request-local query row
    const bool active_tile = t < n_tiles;
    const bool valid = active_tile && (t * 128 + r_local) < tensor_rows;
    const int node = R / p.g;
    const uint64_t* mrow = p.mask_bits ? p.mask_bits + (int64_t)(q0 + node) * p.mask_words : nullptr;
    const uint64_t mw0 = (valid && mrow) ? __ldg(mrow) : 0ull;
    const uint64_t mw1 = (valid && mrow && p.mask_words > 1) ? __ldg(mrow + 1) : 0ull;
    if (cta_ok && __any_sync(0xffffffffu, aborted(bars))) cta_ok = false;
    if (active_tile && cta_ok) {
      // The warp's 32 query rows: loaded two rows (512 contiguous bytes) per
      // instruction into this tile's P buffers (free until the segment's first
      // scores: the previous segment's MMAs have all completed), chunk c of a
      // row at position c ^ (row & 15); then each thread moves its own row into
      // TMEM columns 64t.. (two bf16 per column).
      const uint32_t qbuf = smem_u32(smem + kOffP + 2 * t * kPBytes);
      const int rows_valid = min(32, tensor_rows - (t * 128 + quarter * 32));
      const uint32_t chunk = (uint32_t)(lane & 15);
      uint4 qv[16];                                      // all sixteen loads in flight before any store
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int rw = 2 * i + (lane >> 4);
        const int Rw = row0 + t * 128 + quarter * 32 + rw;
        qv[i] = rw < rows_valid
                    ? __ldg((const uint4*)(p.q + ((int64_t)(q0 + Rw / p.g) * p.Hq + h * p.g + Rw % p.g) * kD) + chunk)
                    : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int rl = quarter * 32 + 2 * i + (lane >> 4);
        st_shared_v4(qbuf + (uint32_t)rl * 256u + ((chunk ^ (uint32_t)(rl & 15)) << 4), qv[i].x, qv[i].y, qv[i].z,
                     qv[i].w);
      }
      __syncwarp();
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t r[32];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const uint32_t chunk = (uint32_t)(half * 8 + v);
          const uint4 x = ld_shared_v4(qbuf + (uint32_t)r_local * 256u + ((chunk ^ (uint32_t)(r_local & 15)) << 4));
          r[4 * v + 0] = x.x;
          r[4 * v + 1] = x.y;
          r[4 * v + 2] = x.z;
          r[4 * v + 3] = x.w;
        }
        tmem_st32(tmem + lane_base + kColQ + 64 * t + 32 * half, r);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.q_ready[t]);
    }
    float m_used = -INFINITY, l_sum = 0.0f;
    bool ok = active_tile && cta_ok;
    // With two tiles, their warpgroups take turns at the exponentials (named
    // barriers 2 and 3 pass the turn), so one tile's exp2 phase has the MUFU
    // pipe to itself while the other loads S, takes the row max, stores P and
    // hands off.  Both warpgroups then run every block -- a named barrier
    // cannot time out, so an abort skips the work but never the turn.  With
    // several segments (balanced schedule) the turns alternate strictly over
    // the CTA's whole life: tile 1 passes the turn after its last block of a
    // segment too, and tile 0 takes that turn (owed) before its first block of
    // the next segment with two tiles, so neither warpgroup can arrive twice
    // at a barrier before the other has taken the first arrival.  A CTA of one
    // unit skips that last hand-over (measured 12 us faster).
    const bool turns = n_tiles == 2;
    const int turn_wait = t == 0 ? 2 : 3, turn_pass = t == 0 ? 3 : 2;
    for (int j = 0; j < nb && (ok || turns); ++j) {
      const int tj = jt + j;                            // this tile's block count: barrier phases, P buffer
      const bool wait_turn = turns && (t == 1 || j > 0 || (kBalanced && owed));
      const bool pass_turn = turns && (kBalanced || !(t == 1 && j == nb - 1));
      // warp-uniform decisions only: the warp's later steps are collectives
      if (ok && __any_sync(0xffffffffu, aborted(bars))) ok = false;
      if (ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars.s_full[t], tj & 1, p.wait_limit));
        if (!ok) record_abort(bars, p, 31);
      }
      if (!ok) {                                        // the turns only
        if (wait_turn) named_bar_sync(turn_wait, 256);
        if (pass_turn) named_bar_arrive(turn_pass, 256);
        continue;
      }
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld32_x2(tmem + lane_base + kColS + 64 * t, sr);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.s_free[t]);
      // visibility: whole block for prefix blocks, else per slot
      const int kv0 = (sg.ja + j) * kBlockN;
      if (!valid || kv0 + kBlockN > prefix) {
        const uint64_t vis = valid ? block_visibility_reg(p, mrow, mw0, mw1, node, kv0, kv_len, prefix) : 0ull;
#pragma unroll
        for (int c = 0; c < kBlockN; ++c)
          if (!((vis >> c) & 1ull)) sr[c] = __float_as_uint(-INFINITY);
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBlockN; c += 8) {
        mx0 = fmax3(mx0, __uint_as_float(sr[c + 0]), __uint_as_float(sr[c + 1]));
        mx1 = fmax3(mx1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
        mx2 = fmax3(mx2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
        mx3 = fmax3(mx3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
      }
      const float mblk = fmax3(mx0, mx1, fmaxf(mx2, mx3)) * p.scale_log2;
      // lazy rescale: per-row factor, O_t touched only when some row needs it
      const bool need = mblk > m_used + kRescaleThreshold;
      float alpha = 1.0f;
      if (need) {
        alpha = (m_used == -INFINITY) ? 0.0f : fast_exp2(m_used - mblk);
        l_sum *= alpha;
        m_used = mblk;
      }
      const float msub = m_used == -INFINITY ? 0.0f : m_used;
      if (wait_turn) named_bar_sync(turn_wait, 256);   // this tile's turn at the exponentials
      // column pairs: scale and shift, and the row sums, on the FMA pipe's
      // two-lane form
      const uint64_t sc2 = f2(p.scale_log2, p.scale_log2), nm2 = f2(-msub, -msub);
      uint64_t ls = f2(0.0f, 0.0f);
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < kBlockN; c += 2) {
        float a, b;
        f2_split(ffma2(f2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc2, nm2), a, b);
        const uint64_t e = f2(fast_exp2(a), fast_exp2(b));
        ls = fadd2(ls, e);
        float e0, e1;
        f2_split(e, e0, e1);
        pk[c / 2] = pack_bf16x2(e0, e1);
      }
      if (pass_turn) named_bar_arrive(turn_pass, 256);   // the other tile's turn
      float ls0, ls1;
      f2_split(ls, ls0, ls1);
      l_sum += ls0 + ls1;
      // P buffer tj % 2 is free: PV_t(tj-2) has completed, because the issuer
      // (one elected thread) issues S_t(tj) after PV_t(tj-2) and the s_full
      // commit waited on above tracks every earlier MMA of that thread
      const uint32_t pbuf = prow + (uint32_t)(tj & 1) * kPBytes;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch)
        st_shared_v4(pbuf + (((uint32_t)ch ^ pswz) << 4), pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
      fence_proxy_async_smem();
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O_t may be rescaled once its last update, PV_t(tj-1), has completed
        ok = __all_sync(0xffffffffu, mbar_wait(&bars.p_empty[t][(tj - 1) & 1], ((tj - 1) >> 1) & 1, p.wait_limit));
        if (!ok) {
          record_abort(bars, p, 35);
          continue;
        }
        tc_fence_after();
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t o[32];
          const uint32_t oa = tmem + lane_base + kColO + 128 * t + 32 * cb;
          tmem_ld32(oa, o);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st32(oa, o);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.p_full[t]);
    }
    if (kBalanced && turns) owed = true;
    // ------------------------------------------------------------ epilogue
    const bool tile_done = ok && __all_sync(0xffffffffu, mbar_wait(&bars.o_full[t], st & 1, p.wait_limit));
    if (ok && !tile_done) record_abort(bars, p, 32);
    if (tile_done) tc_fence_after();
    // Each row goes to this tile's P buffers (free: every MMA of the tile has
    // completed) as 16 chunks of 16 bytes, chunk c at position c ^ (row & 15)
    // so that a warp's stores hit distinct banks; the warp then writes its 32
    // rows out two rows (512 contiguous bytes) per instruction.
    const uint32_t obuf = smem_u32(smem + kOffP + 2 * t * kPBytes);
    const uint32_t swz = (uint32_t)(r_local & 15);
    const uint32_t o_tmem = tmem + lane_base + kColO + 128 * t;
    auto stage32 = [&](int cb, const uint32_t* o, float inv) {
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        const uint32_t chunk = (uint32_t)(cb * 4 + c / 8);
        st_shared_v4(obuf + (uint32_t)r_local * 256u + ((chunk ^ swz) << 4),
                     pack_bf16x2(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv),
                     pack_bf16x2(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv),
                     pack_bf16x2(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv),
                     pack_bf16x2(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv));
      }
    };
    auto store_rows = [&]() {
      __syncwarp();
      const int rows_valid = min(32, tensor_rows - (t * 128 + quarter * 32));   // valid rows are a prefix
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int rw = 2 * i + (lane >> 4);                // row of this warp's 32
        if (rw < rows_valid) {
          const int rl = quarter * 32 + rw;
          const uint32_t chunk = (uint32_t)(lane & 15);
          const uint4 v = ld_shared_v4(obuf + (uint32_t)rl * 256u + ((chunk ^ (uint32_t)(rl & 15)) << 4));
          const int Rw = row0 + t * 128 + rl;
          *(uint4*)(p.out + ((int64_t)(q0 + Rw / p.g) * p.Hq + h * p.g + Rw % p.g) * kD + chunk * 8) = v;
        }
      }
    };
    if (!kBalanced || !sg.split) {
      if (tile_done) {
        const float inv = (valid && l_sum > 0.0f) ? 1.0f / l_sum : 0.0f;
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t o[32];
          tmem_ld32(o_tmem + 32 * cb, o);
          tmem_ld_wait();
          stage32(cb, o, inv);
        }
        store_rows();
      }
    } else if (tile_done) {
      // a unit shared with other CTAs: unnormalised O, the row max it is
      // relative to and the row sum, for the merge kernel
      const int row = t * 128 + r_local;                 // the row's index in a partial slot
      float* slot = p.part + (size_t)sg.slot * (kSlotBytes / 4);
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t o[32];
        tmem_ld32(o_tmem + 32 * cb, o);
        tmem_ld_wait();
#pragma unroll
        for (int qd = 0; qd < 8; ++qd)
          *(float4*)(slot + ((size_t)(cb * 8 + qd) * 256 + row) * 4) =
              make_float4(__uint_as_float(o[4 * qd]), __uint_as_float(o[4 * qd + 1]), __uint_as_float(o[4 * qd + 2]),
                          __uint_as_float(o[4 * qd + 3]));
      }
      slot[kSlotTileBytes / 4 + row] = m_used;
      slot[kSlotTileBytes / 4 + 256 + row] = l_sum;
    }
    if (active_tile) {
      jt += nb;
      ++st;
    }
    }  // segments
    if (kBalanced && t == 0 && owed) named_bar_sync(2, 256);   // take tile 1's last turn
  } else if (warp == kProducerWarp) {
    // ------------------------------------------------------------ TMA producer
    // Lane w < 4 loads page w of every block (K and V, both 64-column halves)
    // into the 4-stage ring as soon as the stage is free.  The page indices
    // come in windows of eight blocks (lane l holds slot 32k + l of window k),
    // the next window loading while the current one is used.
    // The ring runs on across segments (stage and phase from the CTA's block
    // count g), so the next segment's first blocks load while the current one
    // finishes.  K/V is read once: its lines are marked first to leave L2.
    const int w = lane & 3;
    const uint64_t stream_once = l2_policy_evict_first();
    bool ok = true;
    int g = 0, pos = 0;
    Segment sg;
    for (int k = 0; ok && next_segment<kBalanced>(p, S, k, pos, sg); ++k) {
      const int h = sg.h, p0 = sg.p0, n_pages = sg.n_pages;
      auto window = [&](int wk) -> int {
        const int slot = 32 * wk + lane;
        const int phys = slot < n_pages ? __ldg(p.page_indices + p0 + slot) : p.max_pages;
        return (phys >= 0 && phys < p.max_pages) ? phys : p.max_pages;   // invalid: zero fill
      };
      int win_cur = window(sg.ja >> 3), win_next = window((sg.ja >> 3) + 1);
      for (int blk = sg.ja; blk < sg.jb; ++blk, ++g) {
        const int s = g % kStages;
        ok = __all_sync(0xffffffffu, mbar_wait_lazy(&bars.kv_empty[s], ((g / kStages) + 1) & 1, 200, p.wait_limit) &&
                                         !aborted(bars));
        if (!ok) break;
        const int page = __shfl_sync(0xffffffffu, win_cur, (blk & 7) * 4 + w);
        if (lane < 4) {
          mbar_arrive_expect_tx(&bars.kv_full[s], kStageBytes / 4);
          uint8_t* st = smem + kOffKV + s * kStageBytes + lane * (kPage * 128);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            tma_load_4d_hint(st + half * kKvHalf, &kv_map, &bars.kv_full[s], half * 64, h, 0, 2 * page, stream_once);
            tma_load_4d_hint(st + (2 + half) * kKvHalf, &kv_map, &bars.kv_full[s], half * 64, h, 0, 2 * page + 1,
                             stream_once);
          }
        }
        __syncwarp();
        if ((blk & 7) == 7) {
          win_cur = win_next;
          win_next = window((blk >> 3) + 2);
        }
      }
    }
    if (!ok && lane == 0) record_abort(bars, p, 41);
    // the copies this warp issued must land before the CTA can exit
    for (int blk = max(0, g - kStages); blk < g; ++blk) mbar_wait(&bars.kv_full[blk % kStages], (blk / kStages) & 1);
  } else if (warp >= kRemWarp0 && warp < kRemWarp0 + kSyncWarps) {
    // ------------------------------------------------------------ remainder rows
    // Warp kRemWarp0 + wr computes the remainder rows against page wr (16
    // tokens) of every block on mma.sync, transposed: S^T = K Q^T, P^T handed
    // to the next MMA by movmatrix, O^T += V^T P^T; the four partials are
    // merged at the end.
    const int wr = warp - kRemWarp0;
    const int gq = lane >> 2, tq = lane & 3;               // fragment group / thread in group
    const int mi = lane >> 3, rr = lane & 7;               // ldmatrix: matrix / row supplied by this lane
    const uint32_t kv_s = smem_u32(smem + kOffKV);
    bool ok = true;
    int g = 0, pos = 0;                                    // blocks through the ring so far
    Segment sg;
    for (int k = 0; next_segment<kBalanced>(p, S, k, pos, sg); ++k) {
    const int q0 = sg.q0, h = sg.h, row0 = sg.row0, sync_rows = sg.sync_rows;
    const int kv_len = sg.kv_len, prefix = sg.prefix, nb = sg.jb - sg.ja;
    if (ok && __any_sync(0xffffffffu, aborted(bars))) ok = false;
    if (sync_rows == 0) {
      // no remainder rows in this segment: release each stage once it has been filled
      for (int j = 0; ok && j < nb; ++j) {
        const int gg = g + j;
        ok = __all_sync(0xffffffffu, mbar_wait(&bars.kv_full[gg % kStages], (gg / kStages) & 1, p.wait_limit) &&
                                         !aborted(bars));
        if (!ok) {
          if (lane == 0) record_abort(bars, p, 43);
        } else if (lane == 0) {
          mbar_arrive(&bars.kv_empty[gg % kStages]);
        }
        __syncwarp();
      }
      g += nb;
      continue;
    }
    // Q^T as the B operand: column gq is remainder row gq
    uint32_t qb[8][2];
    {
      const int R = row0 + kTensorRows + gq;
      const bool v = gq < sync_rows;
      const uint16_t* qrow = p.q + ((int64_t)(q0 + R / p.g) * p.Hq + h * p.g + R % p.g) * kD;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qb[kk][0] = v ? *(const uint32_t*)(qrow + 16 * kk + 2 * tq) : 0u;
        qb[kk][1] = v ? *(const uint32_t*)(qrow + 16 * kk + 8 + 2 * tq) : 0u;
      }
    }
    // this lane's softmax rows: 2tq and 2tq+1
    int rnode[2];
    bool rvalid[2];
    const uint64_t* rmask[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = 2 * tq + i;
      rvalid[i] = r < sync_rows;
      rnode[i] = (row0 + kTensorRows + r) / p.g;
      rmask[i] = (p.mask_bits && rvalid[i]) ? p.mask_bits + (int64_t)(q0 + rnode[i]) * p.mask_words : nullptr;
    }
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
    for (int j = 0; ok && j < nb; ++j) {
      const int gg = g + j, s = gg % kStages;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars.kv_full[s], (gg / kStages) & 1, p.wait_limit) && !aborted(bars));
      if (!ok) break;
      const uint32_t kb = kv_s + s * kStageBytes, vb = kb + 2 * kKvHalf;
      // S^T (16 tokens x 8 rows), two accumulation chains
      float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int tok = 16 * wr + rr + 8 * (mi & 1), dim = 16 * kk + 8 * (mi >> 1);
        uint32_t a[4];
        ldmatrix_x4(kb + (dim / 64) * kKvHalf + sw128(tok, (dim % 64) / 8), a[0], a[1], a[2], a[3]);
        if (kk & 1) mma_m16n8k16(sb, a, qb[kk][0], qb[kk][1]);
        else mma_m16n8k16(sa, a, qb[kk][0], qb[kk][1]);
      }
      // element e: token gq + 8 (e >> 1), row 2tq + (e & 1)
      float x[4];
      const int kv0 = (sg.ja + j) * kBlockN;
      const bool full = kv0 + kBlockN <= prefix;
      uint64_t vis[2] = {~0ull, ~0ull};
      if (!full) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
          vis[i] = rvalid[i] ? block_visibility(p, rmask[i], rnode[i], kv0, kv_len, prefix) : 0ull;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = 16 * wr + gq + 8 * (e >> 1);
        x[e] = ((vis[e & 1] >> c) & 1ull) && rvalid[e & 1] ? (sa[e] + sb[e]) * p.scale_log2 : -INFINITY;
      }
      // Lazy rescale, as in the tiles: the subtracted max moves (and O and
      // the sums are rescaled) only when some score of the block exceeds it
      // by more than 2^8; otherwise no row max is taken at all.
      const bool grow = x[0] > m_run[0] + kRescaleThreshold || x[2] > m_run[0] + kRescaleThreshold ||
                        x[1] > m_run[1] + kRescaleThreshold || x[3] > m_run[1] + kRescaleThreshold;
      if (__any_sync(0xffffffffu, grow)) {
        float mx[2] = {fmaxf(x[0], x[2]), fmaxf(x[1], x[3])};
#pragma unroll
        for (int off = 4; off <= 16; off <<= 1) {
          mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], off));
          mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], off));
        }
        float alpha[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float nm = fmaxf(m_run[i], mx[i]);
          alpha[i] = (m_run[i] == -INFINITY) ? 0.0f : fast_exp2(m_run[i] - nm);
          m_run[i] = nm;
          l_run[i] *= alpha[i];
        }
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          o[mt][0] *= alpha[0];
          o[mt][1] *= alpha[1];
          o[mt][2] *= alpha[0];
          o[mt][3] *= alpha[1];
        }
      }
      const float msub[2] = {m_run[0] == -INFINITY ? 0.0f : m_run[0], m_run[1] == -INFINITY ? 0.0f : m_run[1]};
      float ex[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) ex[e] = fast_exp2(x[e] - msub[e & 1]);
      l_run[0] += ex[0] + ex[2];
      l_run[1] += ex[1] + ex[3];
      // P^T as the B operand: (token 2tq.., row gq) by transposing the 8x8 blocks
      const uint32_t pb0 = movmatrix_trans(pack_bf16x2(ex[0], ex[1]));
      const uint32_t pb1 = movmatrix_trans(pack_bf16x2(ex[2], ex[3]));
      // O^T (128 dims x 8 rows) += V^T P^T, A = V^T by transposing loads
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int tok = 16 * wr + 8 * (mi >> 1) + rr, dim = 16 * mt + 8 * (mi & 1);
        uint32_t a[4];
        ldmatrix_x4_trans(vb + (dim / 64) * kKvHalf + sw128(tok, (dim % 64) / 8), a[0], a[1], a[2], a[3]);
        mma_m16n8k16(o[mt], a, pb0, pb1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.kv_empty[s]);
    }
    g += nb;
    if (!ok && lane == 0) record_abort(bars, p, 42);
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], off);
      l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], off);
    }
    // merge the four warps' partial results (same fragment layout in every warp)
    float* slot = (float*)(smem + kOffMerge);
    if (wr > 0) {
      float* my = slot + ((wr - 1) * 32 + lane) * kMergeFloats;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) my[4 * mt + e] = o[mt][e];
      my[32] = m_run[0];
      my[33] = m_run[1];
      my[34] = l_run[0];
      my[35] = l_run[1];
    }
    named_bar_sync(1, kSyncWarps * 32);
    // warp 0 of the four: O (relative to M) and the sums L of this CTA's part
    float M[2] = {m_run[0], m_run[1]}, L[2] = {0.0f, 0.0f};
    if (wr == 0 && ok) {
      for (int w = 0; w < kSyncWarps - 1; ++w) {
        const float* other = slot + (w * 32 + lane) * kMergeFloats;
        M[0] = fmaxf(M[0], other[32]);
        M[1] = fmaxf(M[1], other[33]);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float f = (m_run[i] == -INFINITY) ? 0.0f : fast_exp2(m_run[i] - M[i]);
        L[i] = l_run[i] * f;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          o[mt][i] *= f;
          o[mt][2 + i] *= f;
        }
      }
      for (int w = 0; w < kSyncWarps - 1; ++w) {
        const float* other = slot + (w * 32 + lane) * kMergeFloats;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float f = (other[32 + i] == -INFINITY) ? 0.0f : fast_exp2(other[32 + i] - M[i]);
          L[i] += other[34 + i] * f;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            o[mt][i] += other[4 * mt + i] * f;
            o[mt][2 + i] += other[4 * mt + 2 + i] * f;
          }
        }
      }
    }
    // the 8 rows through shared memory (the merge area, read above by this
    // warp only), then two rows (512 contiguous bytes) per store instruction
    auto store_rem = [&]() {
      float inv[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) inv[i] = L[i] > 0.0f ? 1.0f / L[i] : 0.0f;
      __syncwarp();
      uint16_t* ostage = (uint16_t*)(smem + kOffMerge);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const uint32_t lo = pack_bf16x2(o[mt][i] * inv[i], o[mt][2 + i] * inv[i]);
          ostage[(2 * tq + i) * kD + 16 * mt + gq] = (uint16_t)(lo & 0xffffu);
          ostage[(2 * tq + i) * kD + 16 * mt + gq + 8] = (uint16_t)(lo >> 16);
        }
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < kSyncRows / 2; ++i) {
        const int r = 2 * i + (lane >> 4);
        if (r < sync_rows) {
          const int R = row0 + kTensorRows + r;
          const uint4 v = *(const uint4*)(ostage + r * kD + (lane & 15) * 8);
          *(uint4*)(p.out + ((int64_t)(q0 + R / p.g) * p.Hq + h * p.g + R % p.g) * kD + (lane & 15) * 8) = v;
        }
      }
    };
    if (!kBalanced || !sg.split) {
      if (wr == 0 && ok) store_rem();
    } else if (wr == 0 && ok) {
      // a unit shared with other CTAs: this CTA's part for the merge kernel
      float* rem = p.part + (size_t)sg.slot * (kSlotBytes / 4) + (kSlotTileBytes + kSlotStatBytes) / 4;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) rem[(4 * mt + e) * 32 + lane] = o[mt][e];
      rem[32 * 32 + lane] = M[0];
      rem[33 * 32 + lane] = M[1];
      rem[34 * 32 + lane] = L[0];
      rem[35 * 32 + lane] = L[1];
    }
    if (kBalanced) named_bar_sync(1, kSyncWarps * 32);     // the merge area is free for the next segment
    }  // segments
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Balanced schedule, after tree_attn_kernel: CTA (c, q) merges columns
// 32q .. 32q+31 of the unit that starts in CTA c's range and runs past its end
// (at most one per range), from the partials of its CTAs c .. c_last (at most
// kMaxSpan), summed in CTA order.  Thread r merges tile row r (fp32 O as
// [quad][row] float4, max and sum), with every load of the row issued before
// the first is used; warp 0 of CTA (c, 0) then merges the remainder rows in
// the mma.sync fragment layout they were written in.
__global__ void __launch_bounds__(256) tree_attn_merge_kernel(const AttnParams p) {
  pdl_wait();                                          // the partials and the table are complete
  const Sched& S = *p.sched_out;
  const int c = blockIdx.x, qg = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
  if (c + 1 >= S.ctas) return;
  const int begin = range_begin(S, c), end = range_begin(S, c + 1);
  int first, nb, b, h, group;
  locate_unit(p, S, end - 1, first, nb, b, h, group);
  if (first < begin || first + nb <= end) return;      // no unit starts here and runs on
  const int span = cta_of(S, first + nb - 1) - c + 1;  // 2 .. kMaxSpan
  Segment u;
  fill_unit(p, b, h, group, u);
  auto slot = [&](int ci) -> const float* { return p.part + (size_t)slot_of(c + ci, c) * (kSlotBytes / 4); };

  if (tid < u.tensor_rows) {
    const int r = tid;
    float m[kMaxSpan], l[kMaxSpan];
    float4 v[kMaxSpan][8];
#pragma unroll
    for (int ci = 0; ci < kMaxSpan; ++ci) {
      if (ci < span) {
        const float* sl = slot(ci);
        m[ci] = __ldcg(sl + kSlotTileBytes / 4 + r);
        l[ci] = __ldcg(sl + kSlotTileBytes / 4 + 256 + r);
#pragma unroll
        for (int qd = 0; qd < 8; ++qd) v[ci][qd] = __ldcg(reinterpret_cast<const float4*>(sl) + (qg * 8 + qd) * 256 + r);
      } else {
        m[ci] = -INFINITY;
        l[ci] = 0.0f;
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int ci = 0; ci < kMaxSpan; ++ci) M = fmaxf(M, m[ci]);
    float w[kMaxSpan], L = 0.0f;
#pragma unroll
    for (int ci = 0; ci < kMaxSpan; ++ci) {
      w[ci] = m[ci] == -INFINITY ? 0.0f : fast_exp2(m[ci] - M);
      L += w[ci] * l[ci];
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    float acc[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) acc[e] = 0.0f;
#pragma unroll
    for (int ci = 0; ci < kMaxSpan; ++ci) {
      if (ci >= span) break;
#pragma unroll
      for (int qd = 0; qd < 8; ++qd) {
        acc[4 * qd] += w[ci] * v[ci][qd].x;
        acc[4 * qd + 1] += w[ci] * v[ci][qd].y;
        acc[4 * qd + 2] += w[ci] * v[ci][qd].z;
        acc[4 * qd + 3] += w[ci] * v[ci][qd].w;
      }
    }
    const int R = u.row0 + r;
    uint16_t* orow = p.out + ((int64_t)(u.q0 + R / p.g) * p.Hq + h * p.g + R % p.g) * kD + qg * 32;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch)
      *(uint4*)(orow + ch * 8) = make_uint4(
          pack_bf16x2(acc[8 * ch] * inv, acc[8 * ch + 1] * inv), pack_bf16x2(acc[8 * ch + 2] * inv, acc[8 * ch + 3] * inv),
          pack_bf16x2(acc[8 * ch + 4] * inv, acc[8 * ch + 5] * inv),
          pack_bf16x2(acc[8 * ch + 6] * inv, acc[8 * ch + 7] * inv));
  }
  if (qg == 0 && tid < 32 && u.sync_rows > 0) {
    // element k = 4 mt + e of lane (gq, tq): query row 2 tq + (e & 1), dim 16 mt + gq + 8 (e >> 1)
    constexpr uint32_t kRemOff = (kSlotTileBytes + kSlotStatBytes) / 4;
    const int gq = lane >> 2, tq = lane & 3;
    float M[2] = {-INFINITY, -INFINITY};
    for (int ci = 0; ci < span; ++ci) {
      M[0] = fmaxf(M[0], __ldcg(slot(ci) + kRemOff + 32 * 32 + lane));
      M[1] = fmaxf(M[1], __ldcg(slot(ci) + kRemOff + 33 * 32 + lane));
    }
    float acc[32], L[2] = {0.0f, 0.0f};
#pragma unroll
    for (int k = 0; k < 32; ++k) acc[k] = 0.0f;
    for (int ci = 0; ci < span; ++ci) {
      const float* rem = slot(ci) + kRemOff;
      float x[36];
#pragma unroll
      for (int k = 0; k < 36; ++k) x[k] = __ldcg(rem + k * 32 + lane);
      float w[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        w[i] = x[32 + i] == -INFINITY ? 0.0f : fast_exp2(x[32 + i] - M[i]);
        L[i] += w[i] * x[34 + i];
      }
#pragma unroll
      for (int k = 0; k < 32; ++k) acc[k] += w[k & 1] * x[k];
    }
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const int i = k & 1, row = 2 * tq + i;
      if (row < u.sync_rows) {
        const int R = u.row0 + kTensorRows + row, dim = 16 * (k >> 2) + gq + 8 * ((k >> 1) & 1);
        const float inv = L[i] > 0.0f ? 1.0f / L[i] : 0.0f;
        p.out[((int64_t)(u.q0 + R / p.g) * p.Hq + h * p.g + R % p.g) * kD + dim] =
            (uint16_t)(pack_bf16x2(acc[k] * inv, 0.0f) & 0xffffu);
      }
    }
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)f;
  }
  return fn;
}

int encode_4d(CUtensorMap* map, const void* base, const cuuint64_t dims[4], const cuuint64_t strides_bytes[3],
              const cuuint32_t box[4]) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(PTS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult rc = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides_bytes, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return set_error(PTS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)rc);
  return PTS_OK;
}

}  // namespace
}  // namespace pts

namespace pts {
namespace {

// SMs of the current device (cached per device); 0 if it cannot be read.
int attn_sm_count() {
  static std::atomic<int> count[256];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return 0;
  int c = count[dev].load();
  if (!c) {
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    count[dev].store(c);
  }
  return c;
}

// Workspace of the balanced schedule over G CTAs: the error word and the CTA
// count of the last balanced launch (bytes 0-7), the counters (G words at byte
// 256), the flags (2G words after them), then 2G partial slots.
constexpr size_t kSchedOff = 256;
size_t slots_off() { return align_up(kSchedOff + sizeof(Sched), 256); }
size_t balanced_bytes(int G) { return slots_off() + 2 * (size_t)G * kSlotBytes; }

// 0: choose per launch, 1: one CTA per unit, 2: balanced ranges when possible.
std::atomic<int> g_attn_schedule{0};

// Whether balanced ranges should beat one CTA per unit, from the launch's
// bounds (units, and blocks of the longest unit).  A segment costs about
// kSegmentBlocks blocks' time beyond its blocks (measured on the benchmark
// shape: the pipeline drains before the output is read and refills behind the
// next queries), and a range holds its blocks plus up to two cut units, so
// the ranges pay when the units leave SMs idle by much more than that: few
// long units (one request of a long context), not 128 units of 65 blocks on
// 148 SMs.
bool balanced_pays(int G, long long units, long long nblk) {
  constexpr double kSegmentBlocks = 6.0;
  if (units <= 0 || nblk <= 0) return false;
  const long long waves = (units + G - 1) / G;
  const double per_unit = (double)waves * ((double)nblk + kSegmentBlocks);
  const long long chunk = std::max<long long>(kMinBlocksPerCta, (nblk + kMaxSpan - 2) / (kMaxSpan - 1));
  const long long ctas = std::max<long long>(1, std::min<long long>(G, units * nblk / chunk));
  const long long per_cta = (units * nblk + ctas - 1) / ctas;
  const double balanced = (double)per_cta + kSegmentBlocks * (double)(per_cta / nblk + 2);
  return balanced < 0.85 * per_unit;
}

}  // namespace
}  // namespace pts

extern "C" int pts_tree_attn_set_schedule(int mode) {
  if (mode < 0 || mode > 2) {
    pts::set_error(PTS_ERR_INVALID, "schedule %d (0 auto, 1 one CTA per unit, 2 balanced)", mode);
    return -1;
  }
  return pts::g_attn_schedule.exchange(mode);
}

using namespace pts;

extern "C" size_t pts_tree_attn_workspace_size(int, int, int, int, int) {
  const int G = attn_sm_count();
  return G > 0 ? balanced_bytes(G) : 256;
}

extern "C" int pts_tree_attn_check(void* workspace, int* status, pts_stream_t stream) {
  PTS_CHECK_ARG(workspace && status, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  PTS_CUDA_TRY(cudaMemcpyAsync(status, workspace, sizeof(int), cudaMemcpyDeviceToHost, st));
  PTS_CUDA_TRY(cudaStreamSynchronize(st));
  if (*status != 0) PTS_CUDA_TRY(cudaMemsetAsync(workspace, 0, sizeof(int), st));
  return PTS_OK;
}

static int tree_attn_launch(const void* q, const void* kv_layer, const int32_t* qo_indptr,
                            const int32_t* page_indptr, const int32_t* page_indices, const int32_t* last_page_len,
                            const uint64_t* mask_bits, int mask_words, void* out, int batch, int total_q,
                            int max_qo_len, int max_kv_len, int num_qo_heads, int num_kv_heads, int head_dim,
                            int page_len, int max_pages, float sm_scale, void* workspace, size_t workspace_bytes,
                            pts_stream_t stream, int head_pages) {
  PTS_CHECK_ARG(q && kv_layer && qo_indptr && page_indptr && page_indices && last_page_len && out, "null pointer");
  PTS_CHECK_ARG(batch > 0 && total_q > 0 && max_qo_len > 0 && max_kv_len > 0, "bad sizes");
  PTS_CHECK_ARG(num_qo_heads > 0 && num_kv_heads > 0 && num_qo_heads % num_kv_heads == 0, "bad head counts");
  if (head_dim != kD) return set_error(PTS_ERR_UNSUPPORTED, "head_dim %d (this build: 128)", head_dim);
  if (page_len != kPage) return set_error(PTS_ERR_UNSUPPORTED, "page_len %d (this build: 16)", page_len);
  const int g = num_qo_heads / num_kv_heads;
  if (g > 16) return set_error(PTS_ERR_UNSUPPORTED, "GQA group %d (this build: 1..16)", g);
  if (mask_bits) {
    if (max_qo_len > PTS_MAX_TREE_NODES)
      return set_error(PTS_ERR_CAPACITY, "tree of %d rows above %d", max_qo_len, PTS_MAX_TREE_NODES);
    PTS_CHECK_ARG(mask_words >= (max_qo_len + 63) / 64, "mask_words %d too small for %d rows", mask_words,
                  max_qo_len);
  }
  PTS_CHECK_ARG(((uintptr_t)q & 15) == 0 && ((uintptr_t)kv_layer & 15) == 0 && ((uintptr_t)out & 15) == 0,
                "q, kv_layer and out must be 16-byte aligned");
  if (!workspace || workspace_bytes < 256) return set_error(PTS_ERR_CAPACITY, "workspace of at least 256 bytes");
  if (batch > 65535 || num_kv_heads > 65535) return set_error(PTS_ERR_CAPACITY, "grid too large");

  CUtensorMap kv_map;
  {
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)num_kv_heads, (cuuint64_t)kPage,
                                (cuuint64_t)max_pages * 2};
    const cuuint64_t strides[3] = {(cuuint64_t)kD * 2, (cuuint64_t)num_kv_heads * kD * 2,
                                   (cuuint64_t)kPage * num_kv_heads * kD * 2};
    const cuuint32_t box[4] = {64, 1, (cuuint32_t)kPage, 1};
    int rc = encode_4d(&kv_map, kv_layer, dims, strides, box);
    if (rc) return rc;
  }
  AttnParams p{};
  p.q = (const uint16_t*)q;
  p.qo_indptr = qo_indptr;
  p.page_indptr = page_indptr;
  p.page_indices = page_indices;
  p.last_page_len = last_page_len;
  p.mask_bits = mask_bits;
  p.mask_words = mask_words;
  p.out = (uint16_t*)out;
  p.Hq = num_qo_heads;
  p.Hkv = num_kv_heads;
  p.g = g;
  p.head_pages = head_pages;
  p.max_pages = max_pages;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.err = (int*)workspace;
  p.wait_limit = wait_limit_cycles();
  if (int rc = ensure_smem_attr((const void*)tree_attn_kernel<false>, kSmemBytes)) return rc;
  if (int rc = ensure_smem_attr((const void*)tree_attn_kernel<true>, kSmemBytes)) return rc;
  const int groups = (max_qo_len * g + kGroupRows - 1) / kGroupRows;
  if (groups > 65535) return set_error(PTS_ERR_CAPACITY, "%d query rows per request is too many", max_qo_len);
  // Balanced ranges over one CTA per SM when the workspace holds their partials,
  // the schedule table fits and (by default) the estimate below favours them;
  // otherwise one CTA per unit.
  const int G = attn_sm_count();
  const int entries = head_pages ? batch * num_kv_heads : batch;
  dim3 grid(num_kv_heads, batch, groups);
  const bool can_balance =
      G > 0 && entries <= kMaxEntries && workspace_bytes >= balanced_bytes(G) && ((uintptr_t)workspace & 255) == 0;
  const int mode = g_attn_schedule.load();
  if (can_balance && (mode == 2 || (mode == 0 && balanced_pays(G, (long long)batch * num_kv_heads * groups,
                                                               (max_kv_len + kBlockN - 1) / kBlockN)))) {
    char* ws = (char*)workspace;
    p.balanced = 1;
    p.n_entries = entries;
    p.sched_out = (Sched*)(ws + kSchedOff);
    p.part = (float*)(ws + slots_off());
    grid = dim3(G);
  }
  if (!p.balanced) {
    PTS_CUDA_TRY(
        launch_pdl(tree_attn_kernel<false>, grid, dim3(kThreads), kSmemBytes, (cudaStream_t)stream, p, kv_map));
    return launch_status("tree_attn_kernel");
  }
  PTS_CUDA_TRY(launch_pdl(tree_attn_kernel<true>, grid, dim3(kThreads), kSmemBytes, (cudaStream_t)stream, p, kv_map));
  if (int rc = launch_status("tree_attn_kernel")) return rc;
  PTS_CUDA_TRY(launch_pdl(tree_attn_merge_kernel, dim3(G, kD / 32), dim3(256), 0, (cudaStream_t)stream, p));
  return launch_status("tree_attn_merge_kernel");
}

extern "C" int pts_tree_attn_run(const void* q, const void* kv_layer, const int32_t* qo_indptr,
                                 const int32_t* page_indptr, const int32_t* page_indices, const int32_t* last_page_len,
                                 const uint64_t* mask_bits, int mask_words, void* out, int batch, int total_q,
                                 int max_qo_len, int max_kv_len, int num_qo_heads, int num_kv_heads, int head_dim,
                                 int page_len, int max_pages, float sm_scale, void* workspace, size_t workspace_bytes,
                                 pts_stream_t stream) {
  return tree_attn_launch(q, kv_layer, qo_indptr, page_indptr, page_indices, last_page_len, mask_bits, mask_words,
                          out, batch, total_q, max_qo_len, max_kv_len, num_qo_heads, num_kv_heads, head_dim, page_len,
                          max_pages, sm_scale, workspace, workspace_bytes, stream, 0);
}

extern "C" int pts_tree_attn_run_head_pages(const void* q, const void* kv_layer, const int32_t* qo_indptr,
                                            const int32_t* head_page_indptr, const int32_t* head_page_indices,
                                            const int32_t* head_last_page_len, const uint64_t* mask_bits,
                                            int mask_words, void* out, int batch, int total_q, int max_qo_len,
                                            int max_kv_len, int num_qo_heads, int num_kv_heads, int head_dim,
                                            int page_len, int max_pages, float sm_scale, void* workspace,
                                            size_t workspace_bytes, pts_stream_t stream) {
  return tree_attn_launch(q, kv_layer, qo_indptr, head_page_indptr, head_page_indices, head_last_page_len, mask_bits,
                          mask_words, out, batch, total_q, max_qo_len, max_kv_len, num_qo_heads, num_kv_heads,
                          head_dim, page_len, max_pages, sm_scale, workspace, workspace_bytes, stream, 1);
}

namespace pts {
int tree_attn_simt_launch(const void* q, const void* kv_layer, const int32_t* qo_indptr, const int32_t* page_indptr,
                          const int32_t* page_indices, const int32_t* last_page_len, const uint64_t* mask_bits,
                          int mask_words, void* out, int batch, int max_qo_len, int num_qo_heads, int num_kv_heads,
                          int head_dim, int page_len, int max_pages, float sm_scale, int elem_bytes, int head_pages,
                          cudaStream_t stream);
}

extern "C" int pts_tree_attn_run_any(const void* q, const void* kv_layer, const int32_t* qo_indptr,
                                     const int32_t* page_indptr, const int32_t* page_indices,
                                     const int32_t* last_page_len, const uint64_t* mask_bits, int mask_words,
                                     void* out, int batch, int total_q, int max_qo_len, int max_kv_len,
                                     int num_qo_heads, int num_kv_heads, int head_dim, int page_len, int max_pages,
                                     float sm_scale, int elem_bytes, void* workspace, size_t workspace_bytes,
                                     pts_stream_t stream) {
  PTS_CHECK_ARG(q && kv_layer && qo_indptr && page_indptr && page_indices && last_page_len && out, "null pointer");
  PTS_CHECK_ARG(batch > 0 && total_q > 0 && max_qo_len > 0, "bad sizes");
  PTS_CHECK_ARG(num_qo_heads > 0 && num_kv_heads > 0 && num_qo_heads % num_kv_heads == 0, "bad head counts");
  PTS_CHECK_ARG(page_len > 0 && max_pages > 0, "bad page sizes");
  if (mask_bits) {
    if (max_qo_len > PTS_MAX_TREE_NODES)
      return set_error(PTS_ERR_CAPACITY, "tree of %d rows above %d", max_qo_len, PTS_MAX_TREE_NODES);
    PTS_CHECK_ARG(mask_words >= (max_qo_len + 63) / 64, "mask_words %d too small for %d rows", mask_words,
                  max_qo_len);
  }
  if (elem_bytes == 2 && head_dim == kD && page_len == kPage && num_qo_heads / num_kv_heads <= 16)
    return tree_attn_launch(q, kv_layer, qo_indptr, page_indptr, page_indices, last_page_len, mask_bits, mask_words,
                            out, batch, total_q, max_qo_len, max_kv_len, num_qo_heads, num_kv_heads, head_dim,
                            page_len, max_pages, sm_scale, workspace, workspace_bytes, stream, 0);
  return tree_attn_simt_launch(q, kv_layer, qo_indptr, page_indptr, page_indices, last_page_len, mask_bits,
                               mask_words, out, batch, max_qo_len, num_qo_heads, num_kv_heads, head_dim, page_len,
                               max_pages, sm_scale, elem_bytes, 0, (cudaStream_t)stream);
}
