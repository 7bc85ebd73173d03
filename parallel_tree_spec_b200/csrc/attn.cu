// Tree-masked paged attention on sm_100a (TMA + tcgen05 + TMEM).
//
// Work unit (one CTA): request b, KV head h and a group of up to 272 query
// rows.  Query rows are (tree node, query head of h's GQA group) pairs, head
// fastest.  Rows 0-255 of the group form two 128-row tensor-core tiles; the
// remaining up to 16 rows (for example the 65th node of a 65-node tree with 4
// heads per KV head) run on one warp with mma.sync from the same staged K/V.
//
// Per 64-token KV block (four 16-token pages):
//   warp 0 (TMA)      loads K and V of the four pages into a 6-stage ring
//                     (128-byte swizzle, two 64-column halves of D each);
//   warp 1 (MMA)      S_t = Q_t K^T with Q_t resident in TMEM (M=128, N=64,
//                     K=128), then O_t += P_t V with P_t in TMEM (M=128, N=128,
//                     K=64); every operand descriptor is a base descriptor plus
//                     a compile-time offset, issued from a converged warp;
//   warps 2-5, 6-9    one softmax warpgroup per tile: read S_t from TMEM, apply
//                     the scale and the tree mask, keep a running max and sum
//                     per row (O_t is rescaled in TMEM only when the max grows
//                     by more than 2^8), write P_t as bf16 into the first 32
//                     columns of S_t, and at the end normalise O_t;
//   warps 10-13       the remainder rows, FA2-style on mma.sync m16n8k16, each
//                     warp taking 16 of the block's 64 tokens with its own
//                     running max/sum; the four partial results are merged at
//                     the end (legacy mma.sync is slow on sm_100, so one warp
//                     alone could not keep pace with the tensor-core tiles).
// Reading A from TMEM keeps the tensor pipe at its rate: with both operands in
// shared memory a tcgen05 MMA is bound by ~128 bytes/clock of operand reads.
// TMEM (512 columns): Q_t at 64t, S_t/P_t at 128 + 64t, O_t at 256 + 128t.
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

constexpr int kStages = 5;
constexpr int kBlockN = 64;           // KV tokens per block
constexpr int kPage = 16;
constexpr int kD = 128;
constexpr int kTensorRows = 256;      // two 128-row tiles
constexpr int kSyncRows = 16;         // remainder rows on mma.sync
constexpr int kGroupRows = kTensorRows + kSyncRows;
constexpr int kThreads = 448;         // warp 0 TMA, 1 MMA, 2-9 softmax, 10-13 remainder rows
constexpr int kSyncWarps = 4;
constexpr int kMaxSmemPages = 2048;   // page-table entries staged in shared memory
constexpr uint32_t kKvHalf = kBlockN * 128;                   // [64 tokens x 64 dims] bf16
constexpr uint32_t kStageBytes = 4 * kKvHalf;                 // K0 K1 V0 V1
constexpr float kRescaleThreshold = 8.0f;
constexpr uint32_t kColQ = 0, kColS = 128, kColO = 256;

struct __align__(8) Bars {
  uint64_t q_ready;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem;
  int abort;
};

constexpr uint32_t kQxStride = 272;                           // padded row of the remainder queries
constexpr uint32_t kOffKV = 0;
constexpr uint32_t kOffQx = kOffKV + kStages * kStageBytes;
constexpr uint32_t kOffMerge = kOffQx + kSyncRows * kQxStride;   // remainder partials of warps 11-13
constexpr uint32_t kMergeFloats = 68;                            // per lane: 64 O + 2 m + 2 l
constexpr uint32_t kOffPages = kOffMerge + (kSyncWarps - 1) * 32 * kMergeFloats * 4;
constexpr uint32_t kOffBars = kOffPages + kMaxSmemPages * 4;
constexpr uint32_t kSmemBytes = kOffBars + 1024 + 1024;       // bars + alignment slack

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
  int max_pages;
  float scale_log2;
  int* err;
};

__device__ __forceinline__ void record_abort(Bars& bars, const AttnParams& p, int code) {
  *(volatile int*)&bars.abort = 1;
  if (p.err) atomicExch(p.err, code);
}

__device__ __forceinline__ bool aborted(const Bars& bars) { return *(volatile const int*)&bars.abort != 0; }

// Is KV slot `kv` visible to tree row `node` of a request with this prefix?
__device__ __forceinline__ bool visible(const AttnParams& p, const uint64_t* mrow, int node, int kv, int kv_len,
                                        int prefix) {
  if (kv >= kv_len) return false;
  if (kv < prefix) return true;
  const int tn = kv - prefix;
  if (p.mask_bits == nullptr) return tn <= node;
  return (tn / 64 < p.mask_words) && ((__ldg(mrow + tn / 64) >> (tn % 64)) & 1ull);
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
  int32_t* spages = (int32_t*)(smem + kOffPages);

  const int h = blockIdx.x, b = blockIdx.y, group = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q0 = p.qo_indptr[b];
  const int n_nodes = p.qo_indptr[b + 1] - q0;
  const int rows = n_nodes * p.g;
  const int row0 = group * kGroupRows;
  if (row0 >= rows) return;
  const int rows_here = min(kGroupRows, rows - row0);
  const int tensor_rows = min(kTensorRows, rows_here);
  const int n_tiles = (tensor_rows + 127) / 128;
  const int sync_rows = rows_here - tensor_rows;
  const int p0 = p.page_indptr[b];
  const int n_pages = p.page_indptr[b + 1] - p0;
  if (n_pages <= 0) return;
  const int kv_len = (n_pages - 1) * kPage + p.last_page_len[b];
  const int prefix = kv_len - n_nodes;
  const int n_blocks = (kv_len + kBlockN - 1) / kBlockN;

  if (threadIdx.x == 0) {
    mbar_init(&bars.q_ready, 4 * n_tiles);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars.kv_full[s], 1);
      mbar_init(&bars.kv_empty[s], sync_rows > 0 ? 1 + kSyncWarps : 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars.s_full[t], 1);
      mbar_init(&bars.p_full[t], 4);
    }
    mbar_init(&bars.o_full, 1);
    mbar_init(&bars.drain, 1);
    bars.abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&kv_map);
  }
  if (warp == 1) {
    tmem_alloc(&bars.tmem, 512);
    tmem_relinquish();
  }
  if (warp == 0) {
    for (int i = lane; i < min(n_pages, kMaxSmemPages); i += 32) spages[i] = p.page_indices[p0 + i];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < n_blocks; ++j) {
        const int s = j % kStages;
        if (!mbar_wait(&bars.kv_empty[s], ((j / kStages) + 1) & 1)) {
          record_abort(bars, p, 11);
          break;
        }
        if (aborted(bars)) break;
        mbar_arrive_expect_tx(&bars.kv_full[s], kStageBytes);
        uint8_t* st = smem + kOffKV + s * kStageBytes;
#pragma unroll
        for (int pg = 0; pg < kBlockN / kPage; ++pg) {
          const int slot = (kBlockN / kPage) * j + pg;
          const int phys = slot >= n_pages ? p.max_pages                                 // OOB -> zero fill
                           : (slot < kMaxSmemPages ? spages[slot] : p.page_indices[p0 + slot]);
          const int page = (phys >= 0 && phys < p.max_pages) ? phys : p.max_pages;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            tma_load_4d(st + half * kKvHalf + pg * (kPage * 128), &kv_map, &bars.kv_full[s], half * 64, h, 0,
                        2 * page);
            tma_load_4d(st + (2 + half) * kKvHalf + pg * (kPage * 128), &kv_map, &bars.kv_full[s], half * 64, h,
                        0, 2 * page + 1);
          }
        }
        issued = j + 1;
      }
      // wait for copies still in flight before the CTA can exit
      for (int j = max(0, issued - kStages); j < issued; ++j) mbar_wait(&bars.kv_full[j % kStages], (j / kStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t id_qk = idesc_bf16_f32(128, kBlockN, 0, 0);
    const uint32_t id_pv = idesc_bf16_f32(128, kD, 0, 1);
    const uint64_t kd0 = smem_desc(smem_u32(smem + kOffKV), 16, 1024, kSwizzle128B);
    const uint64_t vd0 = smem_desc(smem_u32(smem + kOffKV + 2 * kKvHalf), kKvHalf, 1024, kSwizzle128B);
    const bool leader = elect_one();
#define PTS_QK(T, S)                                                                                        \
  do {                                                                                                      \
    if (leader) {                                                                                           \
      _Pragma("unroll") for (int k = 0; k < kD / 16; ++k) {                                                 \
        const uint64_t bd = kd0 + (uint64_t)(((S) * kStageBytes + (k / 4) * kKvHalf + (k % 4) * 32) >> 4);  \
        mma_bf16_ts(tmem + kColS + 64 * (T), tmem + kColQ + 64 * (T) + 8 * k, bd, id_qk, k > 0);           \
      }                                                                                                     \
      mma_commit(&bars.s_full[T]);                                                                          \
    }                                                                                                       \
    __syncwarp();                                                                                           \
  } while (0)
    bool ok = mbar_wait(&bars.q_ready, 0) && mbar_wait(&bars.kv_full[0], 0);
    if (!ok && lane == 0) record_abort(bars, p, 21);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      PTS_QK(0, 0);
      if (n_tiles > 1) PTS_QK(1, 0);
    }
    for (int j0 = 0; ok && j0 < n_blocks; j0 += kStages) {
#pragma unroll
      for (int ss = 0; ss < kStages; ++ss) {
        const int j = j0 + ss;
        if (j >= n_blocks || !ok) break;
        const int s1 = (ss + 1) % kStages;
        const bool more = j + 1 < n_blocks;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (t >= n_tiles || !ok) break;
          bool w_ok = mbar_wait(&bars.p_full[t], j & 1) && !aborted(bars);
          if (!__all_sync(0xffffffffu, w_ok)) {
            if (lane == 0) record_abort(bars, p, 24);
            ok = false;
            break;
          }
          tc_fence_after();
          if (leader) {
#pragma unroll
            for (int k = 0; k < kBlockN / 16; ++k) {
              const uint64_t bd = vd0 + (uint64_t)((ss * kStageBytes + k * 2048) >> 4);
              mma_bf16_ts(tmem + kColO + 128 * t, tmem + kColS + 64 * t + 8 * k, bd, id_pv, (j > 0 || k > 0) ? 1u : 0u);
            }
            if (t == n_tiles - 1) mma_commit(&bars.kv_empty[ss]);
          }
          __syncwarp();
          if (more) {
            // S_t of the next block overwrites P_t only after this PV (in-order pipe)
            w_ok = (t != 0 || mbar_wait(&bars.kv_full[s1], ((j + 1) / kStages) & 1));
            if (!__all_sync(0xffffffffu, w_ok)) {
              if (lane == 0) record_abort(bars, p, 23);
              ok = false;
              break;
            }
            tc_fence_after();
            PTS_QK(t, s1);
          }
        }
      }
    }
#undef PTS_QK
    if (leader) {
      mma_commit(&bars.o_full);
      mma_commit(&bars.drain);
    }
    __syncwarp();
    mbar_wait(&bars.drain, 0);
  } else if (warp < 10) {
    // ------------------------------------------------------------ softmax warpgroups
    const int t = (warp - 2) >> 2;                      // tile of this warpgroup
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int R = row0 + t * 128 + r_local;             // request-local query row
    const bool active_tile = t < n_tiles;
    const bool valid = active_tile && (t * 128 + r_local) < tensor_rows;
    const int node = R / p.g, hh = R % p.g;
    const uint64_t* mrow = p.mask_bits ? p.mask_bits + (int64_t)(q0 + node) * p.mask_words : nullptr;
    if (active_tile) {
      // this row's query into TMEM columns 64t.. (two bf16 per column)
      const uint16_t* qrow = p.q + ((int64_t)(q0 + node) * p.Hq + h * p.g + hh) * kD;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t r[32];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          uint4 x = valid ? *(const uint4*)(qrow + half * 64 + 8 * v) : make_uint4(0, 0, 0, 0);
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
    for (int j = 0; ok && j < n_blocks; ++j) {
      if (!mbar_wait(&bars.s_full[t], j & 1)) {
        record_abort(bars, p, 31);
        ok = false;
        break;
      }
      tc_fence_after();
      const int kv0 = j * kBlockN;
      // visibility of the block's 64 slots: prefix, tree part (mask or causal), kv_len
      uint64_t vis = ~0ull;
      if (!valid) {
        vis = 0;
      } else if (kv0 + kBlockN > prefix) {
        vis = 0;
        for (int c = 0; c < kBlockN; ++c) {
          const int kv = kv0 + c;
          bool v;
          if (kv >= kv_len) v = false;
          else if (kv < prefix) v = true;
          else {
            const int tn = kv - prefix;
            v = p.mask_bits == nullptr ? (tn <= node)
                                       : (tn / 64 < p.mask_words) && ((__ldg(mrow + tn / 64) >> (tn % 64)) & 1ull);
          }
          vis |= (uint64_t)v << c;
        }
      }
      // pass 1: block max
      float mblk = -INFINITY;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sr[32];
        tmem_ld32(tmem + lane_base + kColS + 64 * t + 32 * half, sr);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if ((vis >> (32 * half + c)) & 1ull) mblk = fmaxf(mblk, __uint_as_float(sr[c]) * p.scale_log2);
      }
      // lazy rescale: warp-uniform decision, per-row factors
      const bool need = valid && (mblk > m_used + kRescaleThreshold);
      float alpha = 1.0f;
      if (need) {
        alpha = (m_used == -INFINITY) ? 0.0f : fast_exp2(m_used - mblk);
        l_sum *= alpha;
        m_used = mblk;
      }
      // pass 2: P = exp2(x - m_used) as bf16 pairs into the first 32 columns of S_t
      uint32_t pk[32];
      float ls = 0.0f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sr[32];
        tmem_ld32(tmem + lane_base + kColS + 64 * t + 32 * half, sr);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const int cc = 32 * half + c;
          const float e0 = ((vis >> cc) & 1ull) ? fast_exp2(__uint_as_float(sr[c]) * p.scale_log2 - m_used) : 0.0f;
          const float e1 = ((vis >> (cc + 1)) & 1ull) ? fast_exp2(__uint_as_float(sr[c + 1]) * p.scale_log2 - m_used) : 0.0f;
          ls += e0 + e1;
          pk[cc / 2] = pack_bf16x2(e0, e1);
        }
      }
      l_sum += ls;
      tmem_st32(tmem + lane_base + kColS + 64 * t, pk);
      tmem_st_wait();
      // O_t is stable here: its last update (PV of the previous block) completed
      // before this block's S_t was committed
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t o[32];
          const uint32_t oa = tmem + lane_base + kColO + 128 * t + 32 * cb;
          tmem_ld32(oa, o);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st32(oa, o);
          tmem_st_wait();
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.p_full[t]);
      if (aborted(bars)) ok = false;
    }
    // ------------------------------------------------------------ epilogue
    if (ok && mbar_wait(&bars.o_full, 0)) {
      tc_fence_after();
      const float inv = (valid && l_sum > 0.0f) ? 1.0f / l_sum : 0.0f;
      uint16_t* orow = p.out + ((int64_t)(q0 + node) * p.Hq + h * p.g + hh) * kD;
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + kColO + 128 * t + 32 * cb, o);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv);
            *(uint4*)(orow + cb * 32 + c) = v;
          }
        }
      }
    } else if (ok) {
      record_abort(bars, p, 32);
    }
  } else {
    // ------------------------------------------------------------ remainder rows (mma.sync)
    const int wr = warp - 10;                              // this warp's 16 tokens of every block
    const int gq = lane >> 2, tq = lane & 3;               // fragment row group / column pair
    const int rA = row0 + kTensorRows + gq, rB = rA + 8;  // this lane's two rows
    const bool vA = gq < sync_rows, vB = gq + 8 < sync_rows;
    const int nodeA = rA / p.g, nodeB = rB / p.g;
    const uint64_t* mA = (p.mask_bits && vA) ? p.mask_bits + (int64_t)(q0 + nodeA) * p.mask_words : nullptr;
    const uint64_t* mB = (p.mask_bits && vB) ? p.mask_bits + (int64_t)(q0 + nodeB) * p.mask_words : nullptr;
    // without remainder rows these warps take no part in the ring (they do not
    // gate kv_empty, so they must not wait on kv_full either)
    if (sync_rows > 0) {
      // remainder queries -> shared memory (padded rows), A fragments by ldmatrix
      uint8_t* qx = smem + kOffQx;
      for (int e = wr * 32 + lane; e < kSyncRows * 16; e += kSyncWarps * 32) {
        const int r = e / 16, v = e % 16;
        const int R = row0 + kTensorRows + r;
        uint4 x = make_uint4(0, 0, 0, 0);
        if (r < sync_rows)
          x = *(const uint4*)(p.q + ((int64_t)(q0 + R / p.g) * p.Hq + h * p.g + R % p.g) * kD + 8 * v);
        *(uint4*)(qx + r * kQxStride + 16 * v) = x;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kSyncWarps * 32) : "memory");
      const uint32_t qx_s = smem_u32(qx);
      const int mi = lane >> 3, rr = lane & 7;
      uint32_t qa[8][4];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        ldmatrix_x4(qx_s + (rr + 8 * (mi & 1)) * kQxStride + 2 * (16 * kk + 8 * (mi >> 1)), qa[kk][0], qa[kk][1],
                    qa[kk][2], qa[kk][3]);
      float o[16][4];
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
      float mA_run = -INFINITY, mB_run = -INFINITY, lA = 0.0f, lB = 0.0f;
      const uint32_t kv_s = smem_u32(smem + kOffKV);
      bool ok = true;
      for (int j = 0; ok && j < n_blocks; ++j) {
        const int s = j % kStages;
        if (!mbar_wait(&bars.kv_full[s], (j / kStages) & 1) || aborted(bars)) {
          if (lane == 0) record_abort(bars, p, 41);
          ok = false;
          break;
        }
        const uint32_t kb = kv_s + s * kStageBytes, vb = kb + 2 * kKvHalf;
        float sc[2][4];
#pragma unroll
        for (int n = 0; n < 2; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
#pragma unroll
        for (int kp = 0; kp < 4; ++kp) {                   // k-steps 2kp, 2kp+1 (32 dims)
          const int dim = 32 * kp + 8 * mi;
#pragma unroll
          for (int n = 0; n < 2; ++n) {
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(kb + (dim / 64) * kKvHalf + sw128(16 * wr + 8 * n + rr, (dim % 64) / 8), b0, b1, b2, b3);
            mma_m16n8k16(sc[n], qa[2 * kp], b0, b1);
            mma_m16n8k16(sc[n], qa[2 * kp + 1], b2, b3);
          }
        }
        const int kv0 = j * kBlockN + 16 * wr;
        float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int kv = kv0 + 8 * n + 2 * tq + e;
            const float xa = (vA && visible(p, mA, nodeA, kv, kv_len, prefix)) ? sc[n][e] * p.scale_log2 : -INFINITY;
            const float xb = (vB && visible(p, mB, nodeB, kv, kv_len, prefix)) ? sc[n][2 + e] * p.scale_log2 : -INFINITY;
            sc[n][e] = xa;
            sc[n][2 + e] = xb;
            mxA = fmaxf(mxA, xa);
            mxB = fmaxf(mxB, xb);
          }
        }
#pragma unroll
        for (int o2 = 1; o2 <= 2; o2 <<= 1) {
          mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, o2));
          mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, o2));
        }
        const float nA = fmaxf(mA_run, mxA), nB = fmaxf(mB_run, mxB);
        const float aA = (mA_run == -INFINITY) ? 0.0f : fast_exp2(mA_run - nA);
        const float aB = (mB_run == -INFINITY) ? 0.0f : fast_exp2(mB_run - nB);
        mA_run = nA;
        mB_run = nB;
        lA *= aA;
        lB *= aB;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          o[nt][0] *= aA;
          o[nt][1] *= aA;
          o[nt][2] *= aB;
          o[nt][3] *= aB;
        }
        uint32_t pa[4];
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          const float e0 = nA == -INFINITY ? 0.0f : fast_exp2(sc[n][0] - nA);
          const float e1 = nA == -INFINITY ? 0.0f : fast_exp2(sc[n][1] - nA);
          const float e2 = nB == -INFINITY ? 0.0f : fast_exp2(sc[n][2] - nB);
          const float e3 = nB == -INFINITY ? 0.0f : fast_exp2(sc[n][3] - nB);
          lA += e0 + e1;
          lB += e2 + e3;
          pa[2 * n + 0] = pack_bf16x2(e0, e1);
          pa[2 * n + 1] = pack_bf16x2(e2, e3);
        }
#pragma unroll
        for (int np = 0; np < 8; ++np) {                   // two 8-dim n-tiles per ldmatrix.x4.trans
          const int tok = 16 * wr + 8 * (mi & 1) + rr;
          const int dim = 16 * np + 8 * (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(vb + (dim / 64) * kKvHalf + sw128(tok, (dim % 64) / 8), b0, b1, b2, b3);
          mma_m16n8k16(o[2 * np], pa, b0, b1);
          mma_m16n8k16(o[2 * np + 1], pa, b2, b3);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.kv_empty[s]);
      }
#pragma unroll
      for (int o2 = 1; o2 <= 2; o2 <<= 1) {
        lA += __shfl_xor_sync(0xffffffffu, lA, o2);
        lB += __shfl_xor_sync(0xffffffffu, lB, o2);
      }
      // merge the four warps' partial results (same fragment layout in every warp)
      float* slot = (float*)(smem + kOffMerge);
      if (wr > 0) {
        float* my = slot + ((wr - 1) * 32 + lane) * kMergeFloats;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) my[4 * nt + e] = o[nt][e];
        my[64] = mA_run;
        my[65] = mB_run;
        my[66] = lA;
        my[67] = lB;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kSyncWarps * 32) : "memory");
      if (wr == 0 && ok) {
        float MA = mA_run, MB = mB_run;
        for (int w = 0; w < kSyncWarps - 1; ++w) {
          const float* other = slot + (w * 32 + lane) * kMergeFloats;
          MA = fmaxf(MA, other[64]);
          MB = fmaxf(MB, other[65]);
        }
        const float sA = (mA_run == -INFINITY) ? 0.0f : fast_exp2(mA_run - MA);
        const float sB = (mB_run == -INFINITY) ? 0.0f : fast_exp2(mB_run - MB);
        float LA = lA * sA, LB = lB * sB;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          o[nt][0] *= sA;
          o[nt][1] *= sA;
          o[nt][2] *= sB;
          o[nt][3] *= sB;
        }
        for (int w = 0; w < kSyncWarps - 1; ++w) {
          const float* other = slot + (w * 32 + lane) * kMergeFloats;
          const float fA = (other[64] == -INFINITY) ? 0.0f : fast_exp2(other[64] - MA);
          const float fB = (other[65] == -INFINITY) ? 0.0f : fast_exp2(other[65] - MB);
          LA += other[66] * fA;
          LB += other[67] * fB;
#pragma unroll
          for (int nt = 0; nt < 16; ++nt) {
            o[nt][0] += other[4 * nt + 0] * fA;
            o[nt][1] += other[4 * nt + 1] * fA;
            o[nt][2] += other[4 * nt + 2] * fB;
            o[nt][3] += other[4 * nt + 3] * fB;
          }
        }
        const float iA = LA > 0.0f ? 1.0f / LA : 0.0f, iB = LB > 0.0f ? 1.0f / LB : 0.0f;
        uint16_t* oA = p.out + ((int64_t)(q0 + nodeA) * p.Hq + h * p.g + rA % p.g) * kD;
        uint16_t* oB = p.out + ((int64_t)(q0 + nodeB) * p.Hq + h * p.g + rB % p.g) * kD;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          const int c = 8 * nt + 2 * tq;
          if (vA) *(uint32_t*)(oA + c) = pack_bf16x2(o[nt][0] * iA, o[nt][1] * iA);
          if (vB) *(uint32_t*)(oB + c) = pack_bf16x2(o[nt][2] * iB, o[nt][3] * iB);
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

extern "C" int pts_tree_attn_run(const void* q, const void* kv_layer, const int32_t* qo_indptr,
                                 const int32_t* page_indptr, const int32_t* page_indices, const int32_t* last_page_len,
                                 const uint64_t* mask_bits, int mask_words, void* out, int batch, int total_q,
                                 int max_qo_len, int max_kv_len, int num_qo_heads, int num_kv_heads, int head_dim,
                                 int page_len, int max_pages, float sm_scale, void* workspace, size_t workspace_bytes,
                                 pts_stream_t stream) {
  PTS_CHECK_ARG(q && kv_layer && qo_indptr && page_indptr && page_indices && last_page_len && out, "null pointer");
  PTS_CHECK_ARG(batch > 0 && total_q > 0 && max_qo_len > 0 && max_kv_len > 0, "bad sizes");
  PTS_CHECK_ARG(num_qo_heads > 0 && num_kv_heads > 0 && num_qo_heads % num_kv_heads == 0, "bad head counts");
  if (head_dim != kD) return set_error(PTS_ERR_UNSUPPORTED, "head_dim %d (this build: 128)", head_dim);
  if (page_len != kPage) return set_error(PTS_ERR_UNSUPPORTED, "page_len %d (this build: 16)", page_len);
  const int g = num_qo_heads / num_kv_heads;
  if (g > 16 || kGroupRows % g != 0) return set_error(PTS_ERR_UNSUPPORTED, "GQA group %d (this build: 1..16, power of 2)", g);
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
  p.max_pages = max_pages;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.err = (int*)workspace;
  static bool attr_set = false;
  if (!attr_set) {
    PTS_CUDA_TRY(cudaFuncSetAttribute(tree_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    attr_set = true;
  }
  const int groups = (max_qo_len * g + kGroupRows - 1) / kGroupRows;
  if (groups > 65535) return set_error(PTS_ERR_CAPACITY, "%d query rows per request is too many", max_qo_len);
  dim3 grid(num_kv_heads, batch, groups);
  tree_attn_kernel<<<grid, kThreads, kSmemBytes, (cudaStream_t)stream>>>(p, kv_map);
  return launch_status("tree_attn_kernel");
}
