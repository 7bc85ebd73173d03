// Tree-masked paged attention on sm_100a (TMA + tcgen05 + TMEM).
//
// Work unit (one CTA): request b, KV head h and a group of up to 264 query
// rows.  Query rows are (tree node, query head of h's GQA group) pairs, head
// fastest.  Rows 0-255 of the group form two 128-row tensor-core tiles; the
// remaining up to 8 rows (for example the 65th node of a 65-node tree with 4
// heads per KV head) run on mma.sync from the same staged K/V.
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
//   warp 15           idle.
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
constexpr uint32_t kKvHalf = kBlockN * 128;                   // [64 tokens x 64 dims] bf16
constexpr uint32_t kStageBytes = 4 * kKvHalf;                 // K0 K1 V0 V1
constexpr uint32_t kPBytes = 128 * kBlockN * 2;               // one P buffer: [128 rows x 64 tokens] bf16
constexpr float kRescaleThreshold = 8.0f;
constexpr uint32_t kColQ = 0, kColS = 128, kColO = 256;

struct __align__(8) Bars {
  uint64_t q_ready;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];    // S_t(j) computed                  (tcgen05.commit)
  uint64_t s_free[2];    // S_t(j) copied out of TMEM          (4 softmax warps)
  uint64_t p_full[2];    // P_t(j) in shared memory, O_t ready (4 softmax warps)
  uint64_t p_empty[2][2];  // PV_t(j) done (O_t may be rescaled)      (tcgen05.commit)
  uint64_t o_full[2];
  uint64_t drain[2];
  uint32_t tmem;
  int abort;
};

constexpr uint32_t kOffKV = 0;
constexpr uint32_t kOffP = kOffKV + kStages * kStageBytes;        // 1024-aligned (swizzle atoms)
constexpr uint32_t kOffMerge = kOffP + 4 * kPBytes;                // remainder partials of warps 11-13
constexpr uint32_t kMergeFloats = 36;                             // per lane: 32 O + 2 m + 2 l
constexpr uint32_t kOffBars = kOffMerge + (kSyncWarps - 1) * 32 * kMergeFloats * 4;
constexpr uint32_t kSmemBytes = kOffBars + 1024 + 1024;       // bars + alignment slack
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
};

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

__global__ void __launch_bounds__(kThreads, 1)
    tree_attn_kernel(const AttnParams p, const __grid_constant__ CUtensorMap kv_map) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  Bars& bars = *reinterpret_cast<Bars*>(smem + kOffBars);

  const int h = blockIdx.x, b = blockIdx.y, group = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // launched as a programmatic dependent: resident early, reads nothing before
  // the previous kernel (the tree preparation and K/V append) has completed
  pdl_wait();
  const int q0 = p.qo_indptr[b];
  const int n_nodes = p.qo_indptr[b + 1] - q0;
  const int rows = n_nodes * p.g;
  const int row0 = group * kGroupRows;
  if (row0 >= rows) return;
  const int rows_here = min(kGroupRows, rows - row0);
  const int tensor_rows = min(kTensorRows, rows_here);
  const int n_tiles = (tensor_rows + 127) / 128;
  const int sync_rows = rows_here - tensor_rows;
  const int pt = p.head_pages ? b * p.Hkv + h : b;     // this CTA's page table
  const int p0 = p.page_indptr[pt];
  const int n_pages = p.page_indptr[pt + 1] - p0;
  if (n_pages <= 0) return;
  const int kv_len = (n_pages - 1) * kPage + p.last_page_len[pt];
  const int prefix = kv_len - n_nodes;
  const int n_blocks = (kv_len + kBlockN - 1) / kBlockN;

  if (threadIdx.x == 0) {
    mbar_init(&bars.q_ready, 4 * n_tiles);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars.kv_full[s], 4);                   // one expect_tx arrival per producer lane (page)
      mbar_init(&bars.kv_empty[s], n_tiles + (sync_rows > 0 ? kSyncWarps : 0));
    }
    for (int t = 0; t < 2; ++t) {
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
    const int t = warp == 1 ? 0 : 1;
    if (t < n_tiles) {
      const uint32_t id_qk = idesc_bf16_f32(128, kBlockN, 0, 0);
      const uint32_t id_pv = idesc_bf16_f32(128, kD, 0, 1);
      const uint64_t kd0 = smem_desc(smem_u32(smem + kOffKV), 16, 1024, kSwizzle128B);
      const uint64_t vd0 = smem_desc(smem_u32(smem + kOffKV + 2 * kKvHalf), kKvHalf, 1024, kSwizzle128B);
      const uint64_t pd0 = smem_desc(smem_u32(smem + kOffP + 2 * t * kPBytes), 16, 1024, kSwizzle128B);
      const uint32_t s_col = tmem + kColS + 64 * t, q_col = tmem + kColQ + 64 * t, o_col = tmem + kColO + 128 * t;
      const bool leader = elect_one();
#define PTS_QK(S)                                                                                           \
  do {                                                                                                      \
    if (leader) {                                                                                           \
      _Pragma("unroll") for (int k = 0; k < kD / 16; ++k) {                                                 \
        const uint64_t bd = kd0 + (uint64_t)(((S) * kStageBytes + (k / 4) * kKvHalf + (k % 4) * 32) >> 4);  \
        mma_bf16_ts(s_col, q_col + 8 * k, bd, id_qk, k > 0);                                                \
      }                                                                                                     \
      mma_commit(&bars.s_full[t]);                                                                          \
    }                                                                                                       \
    __syncwarp();                                                                                           \
  } while (0)
      bool ok = mbar_wait(&bars.q_ready, 0, p.wait_limit) && mbar_wait(&bars.kv_full[0], 0, p.wait_limit);
      if (!ok && lane == 0) record_abort(bars, p, 21);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        PTS_QK(0);
      }
      for (int j0 = 0; ok && j0 < n_blocks; j0 += kStages) {
#pragma unroll
        for (int ss = 0; ss < kStages; ++ss) {
          const int j = j0 + ss;
          if (j >= n_blocks) break;
          const int s1 = (ss + 1) % kStages;
          if (j + 1 < n_blocks) {
            // scores of block j+1 once K(j+1) is staged and S_t(j) has been read
            const bool w_ok = mbar_wait(&bars.kv_full[s1], ((j + 1) / kStages) & 1, p.wait_limit) &&
                              mbar_wait(&bars.s_free[t], j & 1, p.wait_limit) && !aborted(bars);
            if (!__all_sync(0xffffffffu, w_ok)) {
              if (lane == 0) record_abort(bars, p, 23);
              ok = false;
              break;
            }
            tc_fence_after();
            PTS_QK(s1);
          }
          const bool w_ok = mbar_wait(&bars.p_full[t], j & 1, p.wait_limit) && !aborted(bars);
          if (!__all_sync(0xffffffffu, w_ok)) {
            if (lane == 0) record_abort(bars, p, 24);
            ok = false;
            break;
          }
          tc_fence_after();
          if (leader) {
#pragma unroll
            for (int k = 0; k < kBlockN / 16; ++k) {
              const uint64_t ad = pd0 + (uint64_t)(((ss & 1) * kPBytes + k * 32) >> 4);
              const uint64_t bd = vd0 + (uint64_t)((ss * kStageBytes + k * 2048) >> 4);
              mma_bf16_ss(o_col, ad, bd, id_pv, (j > 0 || k > 0) ? 1u : 0u);
            }
            mma_commit(&bars.p_empty[t][ss & 1]);
            mma_commit(&bars.kv_empty[ss]);
          }
          __syncwarp();
        }
      }
#undef PTS_QK
      if (leader) {
        mma_commit(&bars.o_full[t]);
        mma_commit(&bars.drain[t]);
      }
      __syncwarp();
      mbar_wait(&bars.drain[t], 0);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ softmax warpgroups
    const int t = (warp - 2) >> 2;                      // tile of this warpgroup
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int R = row0 + t * 128 + r_local;             // request-local query row
    const bool active_tile = t < n_tiles;
    const bool valid = active_tile && (t * 128 + r_local) < tensor_rows;
    const int node = R / p.g;
    const uint64_t* mrow = p.mask_bits ? p.mask_bits + (int64_t)(q0 + node) * p.mask_words : nullptr;
    const uint64_t mw0 = (valid && mrow) ? __ldg(mrow) : 0ull;
    const uint64_t mw1 = (valid && mrow && p.mask_words > 1) ? __ldg(mrow + 1) : 0ull;
    const uint32_t prow = smem_u32(smem + kOffP + 2 * t * kPBytes) + r_local * 128;   // this row of P_t, buffer 0
    const uint32_t pswz = (uint32_t)(r_local & 7);
    if (active_tile) {
      // The warp's 32 query rows: loaded two rows (512 contiguous bytes) per
      // instruction into this tile's P buffers (free until block 0's scores),
      // chunk c of a row at position c ^ (row & 15); then each thread moves its
      // own row into TMEM columns 64t.. (two bf16 per column).
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
      if (lane == 0) mbar_arrive(&bars.q_ready);
    }
    float m_used = -INFINITY, l_sum = 0.0f;
    bool ok = active_tile;
    // With two tiles, their warpgroups take turns at the exponentials (named
    // barriers 2 and 3 pass the turn), so one tile's exp2 phase has the MUFU
    // pipe to itself while the other loads S, takes the row max, stores P and
    // hands off.  Both warpgroups then run every block -- a named barrier
    // cannot time out, so an abort skips the work but never the turn.
    const bool turns = n_tiles == 2;
    const int turn_wait = t == 0 ? 2 : 3, turn_pass = t == 0 ? 3 : 2;
    for (int j = 0; j < n_blocks && (ok || turns); ++j) {
      const bool wait_turn = turns && (t == 1 || j > 0);
      const bool pass_turn = turns && !(t == 1 && j == n_blocks - 1);
      // warp-uniform decisions only: the warp's later steps are collectives
      if (ok && __any_sync(0xffffffffu, aborted(bars))) ok = false;
      if (ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars.s_full[t], j & 1, p.wait_limit));
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
      const int kv0 = j * kBlockN;
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
      // P buffer j % 2 is free: PV_t(j-2) has completed, because the issuer
      // (one elected thread) issues S_t(j) after PV_t(j-2) and the s_full
      // commit waited on above tracks every earlier MMA of that thread
      const uint32_t pbuf = prow + (uint32_t)(j & 1) * kPBytes;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch)
        st_shared_v4(pbuf + (((uint32_t)ch ^ pswz) << 4), pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
      fence_proxy_async_smem();
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O_t may be rescaled once its last update, PV_t(j-1), has completed
        ok = __all_sync(0xffffffffu, mbar_wait(&bars.p_empty[t][(j - 1) & 1], ((j - 1) >> 1) & 1, p.wait_limit));
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
    // ------------------------------------------------------------ epilogue
    if (ok && __all_sync(0xffffffffu, mbar_wait(&bars.o_full[t], 0, p.wait_limit))) {
      tc_fence_after();
      // Each row goes to this tile's P buffers (free: every MMA of the tile has
      // completed) as 16 chunks of 16 bytes, chunk c at position c ^ (row & 15)
      // so that a warp's stores hit distinct banks; the warp then writes its
      // 32 rows out two rows (512 contiguous bytes) per instruction.
      const float inv = (valid && l_sum > 0.0f) ? 1.0f / l_sum : 0.0f;
      const uint32_t obuf = smem_u32(smem + kOffP + 2 * t * kPBytes);
      const uint32_t swz = (uint32_t)(r_local & 15);
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + kColO + 128 * t + 32 * cb, o);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          const uint32_t chunk = (uint32_t)(cb * 4 + c / 8);
          st_shared_v4(obuf + (uint32_t)r_local * 256u + ((chunk ^ swz) << 4),
                       pack_bf16x2(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv),
                       pack_bf16x2(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv),
                       pack_bf16x2(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv),
                       pack_bf16x2(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv));
        }
      }
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
    } else if (ok) {
      record_abort(bars, p, 32);
    }
  } else if (warp == kProducerWarp) {
    // ------------------------------------------------------------ TMA producer
    // Lane w < 4 loads page w of every block (K and V, both 64-column halves)
    // into the 4-stage ring as soon as the stage is free.  The page indices
    // come in windows of eight blocks (lane l holds slot 32k + l of window k),
    // the next window loading while the current one is used.
    const int w = lane & 3;
    auto window = [&](int k) -> int {
      const int slot = 32 * k + lane;
      const int phys = slot < n_pages ? __ldg(p.page_indices + p0 + slot) : p.max_pages;
      return (phys >= 0 && phys < p.max_pages) ? phys : p.max_pages;   // invalid: zero fill
    };
    int win_cur = window(0), win_next = window(1);
    auto produce = [&](int blk) -> bool {
      const int s = blk % kStages;
      const bool w_ok =
          mbar_wait_lazy(&bars.kv_empty[s], ((blk / kStages) + 1) & 1, 200, p.wait_limit) && !aborted(bars);
      if (!__all_sync(0xffffffffu, w_ok)) return false;
      const int page = __shfl_sync(0xffffffffu, win_cur, (blk & 7) * 4 + w);
      if (lane < 4) {
        mbar_arrive_expect_tx(&bars.kv_full[s], kStageBytes / 4);
        uint8_t* st = smem + kOffKV + s * kStageBytes + lane * (kPage * 128);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          tma_load_4d(st + half * kKvHalf, &kv_map, &bars.kv_full[s], half * 64, h, 0, 2 * page);
          tma_load_4d(st + (2 + half) * kKvHalf, &kv_map, &bars.kv_full[s], half * 64, h, 0, 2 * page + 1);
        }
      }
      __syncwarp();
      if ((blk & 7) == 7) {
        win_cur = win_next;
        win_next = window((blk >> 3) + 2);
      }
      return true;
    };
    bool ok = true;
    int produced = 0;
    for (int blk = 0; ok && blk < n_blocks; ++blk) {
      ok = produce(blk);
      if (ok) produced = blk + 1;
    }
    if (!ok && lane == 0) record_abort(bars, p, 41);
    // the copies this warp issued must land before the CTA can exit
    for (int blk = max(0, produced - kStages); blk < produced; ++blk)
      mbar_wait(&bars.kv_full[blk % kStages], (blk / kStages) & 1);
  } else if (warp >= kRemWarp0 && warp < kRemWarp0 + kSyncWarps && sync_rows > 0) {
    // ------------------------------------------------------------ remainder rows
    // Warp kRemWarp0 + wr computes the remainder rows against page wr (16
    // tokens) of every block on mma.sync, transposed: S^T = K Q^T, P^T handed
    // to the next MMA by movmatrix, O^T += V^T P^T; the four partials are
    // merged at the end.
    const int wr = warp - kRemWarp0;
    const int gq = lane >> 2, tq = lane & 3;               // fragment group / thread in group
    const int mi = lane >> 3, rr = lane & 7;               // ldmatrix: matrix / row supplied by this lane
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
    const uint32_t kv_s = smem_u32(smem + kOffKV);
    bool ok = true;
    for (int j = 0; ok && j < n_blocks; ++j) {
      const int s = j % kStages;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars.kv_full[s], (j / kStages) & 1, p.wait_limit) && !aborted(bars));
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
      const int kv0 = j * kBlockN;
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
    if (!ok && lane == 0) record_abort(bars, p, 42);
    {
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
    asm volatile("bar.sync 1, %0;" ::"r"(kSyncWarps * 32) : "memory");
    if (wr == 0 && ok) {
      float M[2] = {m_run[0], m_run[1]};
      for (int w = 0; w < kSyncWarps - 1; ++w) {
        const float* other = slot + (w * 32 + lane) * kMergeFloats;
        M[0] = fmaxf(M[0], other[32]);
        M[1] = fmaxf(M[1], other[33]);
      }
      float L[2];
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
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float inv = L[i] > 0.0f ? 1.0f / L[i] : 0.0f;
        L[i] = inv;
      }
      // the 8 rows through shared memory (the merge area, read above by this
      // warp only), then two rows (512 contiguous bytes) per store instruction
      __syncwarp();
      uint16_t* ostage = (uint16_t*)(smem + kOffMerge);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const uint32_t lo = pack_bf16x2(o[mt][i] * L[i], o[mt][2 + i] * L[i]);
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
    }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
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

using namespace pts;

extern "C" size_t pts_tree_attn_workspace_size(int, int, int, int, int) { return 256; }

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
  if (int rc = ensure_smem_attr((const void*)tree_attn_kernel, kSmemBytes)) return rc;
  const int groups = (max_qo_len * g + kGroupRows - 1) / kGroupRows;
  if (groups > 65535) return set_error(PTS_ERR_CAPACITY, "%d query rows per request is too many", max_qo_len);
  dim3 grid(num_kv_heads, batch, groups);
  PTS_CUDA_TRY(launch_pdl(tree_attn_kernel, grid, dim3(kThreads), kSmemBytes, (cudaStream_t)stream, p, kv_map));
  return launch_status("tree_attn_kernel");
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
