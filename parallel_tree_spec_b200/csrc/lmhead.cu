// The target model's lm_head over the draft-tree rows with the acceptance
// statistics computed in the GEMM epilogue (TMA + tcgen05 + TMEM), so that the
// [rows x vocab] logits never go to memory.
//
// logits = hidden [M, K] x weight[V, K]^T (nn.Linear layout, both K-major bf16,
// fp32 accumulation), tiles of 128 rows x 256 vocabulary columns, K in steps of
// 64 through a four-stage TMA ring (48 KB a stage).  One persistent CTA per SM
// walks the tiles row-tile fastest, so the CTAs working at the same time share
// each weight tile through L2.  Six warps:
//   warp 0     TMA producer (hidden tile 128 x 64, weight tile 256 x 64, 128-byte
//              swizzle);
//   warp 1     MMA issuer (M=128 N=256 K=16 per instruction, A and B from shared
//              memory) into one of two TMEM accumulators (256 columns each), so
//              the epilogue of tile i overlaps the main loop of tile i+1;
//   warps 2-9  epilogue, two threads per row (warps 2-5 the first 128 columns of
//              the tile, warps 6-9 the other 128): every accumulator is rounded
//              to bf16 first (the value the model's bf16 logits would hold),
//              then scaled by 1/T and rounded again as the acceptance scales
//              logits.
// Statistics mode writes per (row, 128-column half tile): the partial (sum of
// exp(x - m_t) in fp64, m_t, first index of m_t) in the acceptance kernel's
// format; the node token logits (each node's token under its parent row, from
// the one tile holding the token); and, for tiles whose max could take part in
// a rounding tie of the row's argmax (|m_t| < 4), the tile's largest distinct
// values with their first indices.  Logits mode writes the bf16 logits (the
// unfused path and the fallback for unresolved ties).
//
// Then one warp per row merges its tiles in tile order (as the vocabulary-
// sharded merge does), settles the argmax of the bf16-rounded probabilities
// from the candidate lists when the row's largest value below the max rounds
// to the same probability, and the walks run from the merged statistics.
#include <cuda.h>
#include <float.h>
#include <limits.h>

#include "common.cuh"
#include "sm100.cuh"

namespace pts {
namespace {

using namespace sm100;

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr int kThreads = 320;                          // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpiWarps = 8;
constexpr int kSub = 128;                              // columns of a tile one epilogue thread reduces
constexpr uint32_t kABytes = kBM * kBK * 2;            // 16 KB
constexpr uint32_t kBBytes = kBN * kBK * 2;            // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024 + 1024;   // ring + barriers + alignment
constexpr int kCand = 4;                               // candidate values per (row, tile)
constexpr float kCandRange = 4.0f;                     // |m_t| below which a tile keeps candidates
constexpr float kLog2e = 1.4426950408889634f;
static_assert(kSmemBytes <= 232448, "shared memory above the 227 KB per-CTA limit");

struct __align__(16) LmPart {                          // the acceptance kernel's partial layout
  double s;
  float m;
  int idx;
};

struct Cand {
  float v;
  int idx;
};

struct RowStatOut {                                    // the acceptance kernel's row statistics layout
  float m;
  float s;
  int argmax;
  int flags;
};

struct __align__(8) LmBars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem;
  int abort;
};

struct LmParams {
  int M, V, K;
  int m_tiles, n_tiles, tiles, k_blocks;
  int n_sub;                   // 128-column partials per row (two per tile)
  int mode;                    // 0 statistics, 1 logits
  int use_temp;
  float inv_temp;
  uint16_t* logits;            // mode 1: [M, logits_stride] bf16
  int64_t logits_stride;
  LmPart* parts;               // mode 0: [M][n_sub]
  Cand* cands;                 // mode 0: [M][n_sub][kCand]
  const int32_t* child_ptr;    // [M+1]: row r's children, sorted by token
  const int32_t* child_tok;
  const int32_t* child_node;
  float* tok_logit;            // [M]: node's token logit under its parent row
  int* err;
};

// Round-to-nearest-even to bf16 for the finite accumulators (no NaN path).
__device__ __forceinline__ float rne_bf16(float x) {
  const uint32_t u = __float_as_uint(x);
  return __uint_as_float((u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u);
}

__device__ __forceinline__ float scaled_logit(const LmParams& p, float acc) {
  float x = rne_bf16(acc);
  if (p.use_temp) x = rne_bf16(__fmul_rn(x, p.inv_temp));
  return x;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kThreads, 1)
    lmhead_kernel(const LmParams p, const __grid_constant__ CUtensorMap a_map,
                  const __grid_constant__ CUtensorMap b_map) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  LmBars& bars = *reinterpret_cast<LmBars*>(smem + kStages * kStageBytes);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars.full[s], 1);
      mbar_init(&bars.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars.acc_full[b], 1);
      mbar_init(&bars.acc_empty[b], kEpiWarps);
    }
    mbar_init(&bars.drain, 1);
    bars.abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&a_map);
    tma_prefetch_desc(&b_map);
  }
  if (warp == 1) {
    tmem_alloc(&bars.tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    int g = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.tiles; tile += gridDim.x) {
      const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
      for (int kb = 0; kb < p.k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        ok = __all_sync(0xffffffffu, mbar_wait(&bars.empty[s], ((g / kStages) + 1) & 1) &&
                                         !(*(volatile int*)&bars.abort));
        if (!ok) break;
        if (lane == 0) {
          uint8_t* st = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&bars.full[s], kStageBytes);
          tma_load_2d(st, &a_map, &bars.full[s], kb * kBK, mt * kBM);
          tma_load_2d(st + kABytes, &b_map, &bars.full[s], kb * kBK, nt * kBN);
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      *(volatile int*)&bars.abort = 1;
      if (p.err) atomicExch(p.err, 51);
    }
    // the copies this warp issued must land before the CTA can exit
    for (int q = max(0, g - kStages); q < g; ++q) mbar_wait(&bars.full[q % kStages], (q / kStages) & 1);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_bf16_f32(kBM, kBN, 0, 0);
    const uint64_t d0 = smem_desc(smem_u32(smem), 16, 1024, kSwizzle128B);
    const bool leader = elect_one();
    int g = 0, i = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.tiles; tile += gridDim.x, ++i) {
      const int buf = i & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars.acc_empty[buf], ((i >> 1) + 1) & 1) &&
                                       !(*(volatile int*)&bars.abort));
      if (!ok) break;
      tc_fence_after();
      for (int kb = 0; kb < p.k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        ok = __all_sync(0xffffffffu, mbar_wait(&bars.full[s], (g / kStages) & 1));
        if (!ok) break;
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = d0 + (uint64_t)((s * kStageBytes + kk * 32) >> 4);
            const uint64_t bd = d0 + (uint64_t)((s * kStageBytes + kABytes + kk * 32) >> 4);
            mma_bf16_ss(tmem + 256 * buf, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&bars.empty[s]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (leader) mma_commit(&bars.acc_full[buf]);
      __syncwarp();
    }
    if (!ok && lane == 0) {
      *(volatile int*)&bars.abort = 1;
      if (p.err) atomicExch(p.err, 52);
    }
    // every MMA this warp issued has completed before the CTA moves on
    if (leader) mma_commit(&bars.drain);
    __syncwarp();
    mbar_wait(&bars.drain, 0);
  } else {
    // ------------------------------------------------------------ epilogue: two threads per row
    const int quarter = warp & 3;                        // TMEM lanes 32q .. 32q+31
    const int sub = (warp - 2) >> 2;                     // this thread's 128 columns of a tile
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    int i = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, ++i) {
      const int buf = i & 1;
      const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
      const bool w_ok = __all_sync(0xffffffffu, mbar_wait(&bars.acc_full[buf], (i >> 1) & 1) &&
                                                    !(*(volatile int*)&bars.abort));
      if (!w_ok) {
        if (lane == 0) {
          *(volatile int*)&bars.abort = 1;
          if (p.err) atomicExch(p.err, 53);
        }
        break;
      }
      tc_fence_after();
      const int row = mt * kBM + quarter * 32 + lane;
      const bool valid = row < p.M;
      const int n0 = nt * kBN + sub * kSub;              // first column of this thread's half tile
      const int ncols = max(0, min(kSub, p.V - n0));
      const uint32_t acc = tmem + lane_base + 256 * buf + sub * kSub;
      if (p.mode == 1) {
        // logits: bf16 of every accumulator
        uint16_t* out = p.logits + (int64_t)row * p.logits_stride + n0;
        for (int c = 0; c < kSub / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(acc + 32 * c, r);
          tmem_ld_wait();
          if (valid && 32 * c < ncols) {
            if (32 * c + 32 <= ncols && (((uintptr_t)(out + 32 * c)) & 15) == 0) {
#pragma unroll
              for (int v = 0; v < 32; v += 8) {
                uint4 w;
                w.x = pack_bf16x2(__uint_as_float(r[v + 0]), __uint_as_float(r[v + 1]));
                w.y = pack_bf16x2(__uint_as_float(r[v + 2]), __uint_as_float(r[v + 3]));
                w.z = pack_bf16x2(__uint_as_float(r[v + 4]), __uint_as_float(r[v + 5]));
                w.w = pack_bf16x2(__uint_as_float(r[v + 6]), __uint_as_float(r[v + 7]));
                *(uint4*)(out + 32 * c + v) = w;
              }
            } else {
#pragma unroll
              for (int v = 0; v < 32; ++v)
                if (32 * c + v < ncols) out[32 * c + v] = float_to_bf16_bits(__uint_as_float(r[v]));
            }
          }
        }
      } else {
        // pass 1: the half tile's max of the scaled bf16 logits and its first index
        float m_t = -INFINITY;
        int i_t = INT_MAX;
        for (int c = 0; c < kSub / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(acc + 32 * c, r);
          tmem_ld_wait();
          // four interleaved (max, first index) chains, merged in index order
          float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
          int ix[4] = {INT_MAX, INT_MAX, INT_MAX, INT_MAX};
#pragma unroll
          for (int v = 0; v < 32; ++v) {
            const float x = scaled_logit(p, __uint_as_float(r[v]));
            if (32 * c + v < ncols && x > mx[v & 3]) {
              mx[v & 3] = x;
              ix[v & 3] = n0 + 32 * c + v;
            }
          }
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (mx[k] > m_t || (mx[k] == m_t && ix[k] < i_t)) {
              m_t = mx[k];
              i_t = ix[k];
            }
        }
        // pass 2: the sum of exp(x - m_t), the children's token logits and the
        // candidate values of the rounding-tie rule
        const bool keep = valid && m_t > -kCandRange && m_t < kCandRange;
        Cand cl[kCand];
#pragma unroll
        for (int k = 0; k < kCand; ++k) cl[k] = Cand{-INFINITY, INT_MAX};
        int cp = valid ? p.child_ptr[row] : 0;
        const int ce = valid ? p.child_ptr[row + 1] : 0;
        while (cp < ce && p.child_tok[cp] < n0) ++cp;
        int next_tok = cp < ce ? p.child_tok[cp] : INT_MAX;
        const int last_col = n0 + ncols;                 // children at or past it belong to another half tile
        const float mlog = (m_t == -INFINITY) ? 0.0f : m_t * kLog2e;
        double s_t = 0.0;
        for (int c = 0; c < kSub / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(acc + 32 * c, r);
          tmem_ld_wait();
          float q0 = 0.0f, q1 = 0.0f, q2 = 0.0f, q3 = 0.0f;
          const bool tok_here = next_tok < n0 + 32 * c + 32 && next_tok < last_col;
          const bool cand_here = keep;
#pragma unroll
          for (int v = 0; v < 32; ++v) {
            const int col = 32 * c + v;
            const float x = scaled_logit(p, __uint_as_float(r[v]));
            const bool in = col < ncols;
            const float e = in ? ex2_approx(fmaf(x, kLog2e, -mlog)) : 0.0f;
            if ((v & 3) == 0) q0 += e;
            else if ((v & 3) == 1) q1 += e;
            else if ((v & 3) == 2) q2 += e;
            else q3 += e;
            if (tok_here && in && n0 + col == next_tok) {
              do {
                p.tok_logit[p.child_node[cp]] = x;
                ++cp;
                next_tok = cp < ce ? p.child_tok[cp] : INT_MAX;
              } while (n0 + col == next_tok);
            }
            if (cand_here && in && x > cl[kCand - 1].v) {
              // insert a new distinct value (a repeat keeps its first index)
              bool present = false;
#pragma unroll
              for (int k = 0; k < kCand; ++k) present |= (cl[k].v == x);
              if (!present) {
                Cand cur{x, n0 + col};
#pragma unroll
                for (int k = 0; k < kCand; ++k) {
                  if (cur.v > cl[k].v) {
                    const Cand t = cl[k];
                    cl[k] = cur;
                    cur = t;
                  }
                }
              }
            }
          }
          s_t += (double)((q0 + q1) + (q2 + q3));
        }
        if (valid) {
          const int slot = nt * 2 + sub;
          LmPart part;
          part.s = (m_t == -INFINITY) ? 0.0 : s_t;
          part.m = m_t;
          part.idx = i_t;
          p.parts[(int64_t)row * p.n_sub + slot] = part;
          if (keep) {
            Cand* dst = p.cands + ((int64_t)row * p.n_sub + slot) * kCand;
#pragma unroll
            for (int k = 0; k < kCand; ++k) dst[k] = cl[k];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// One CTA per request: each row's children sorted by token (for the epilogue's
// single pass over a tile's columns), and the node token logits reset to -inf.
__global__ void child_lists_kernel(const int32_t* row_indptr, const int32_t* parents, const int32_t* tokens,
                                   int32_t* child_ptr, int32_t* child_tok, int32_t* child_node, float* tok_logit) {
  __shared__ int cnt[PTS_MAX_TREE_NODES + 1];
  const int b = blockIdx.x;
  const int lo = row_indptr[b], n = row_indptr[b + 1] - lo;
  for (int i = threadIdx.x; i <= n; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    tok_logit[lo + i] = -INFINITY;
    const int pr = parents[lo + i];
    if (i > 0 && pr >= 0 && pr < i) atomicAdd(&cnt[pr], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = lo;                                        // children of this request's rows sit at [lo, lo + n)
    for (int r = 0; r < n; ++r) {
      const int c = cnt[r];
      cnt[r] = acc;
      acc += c;
    }
    cnt[n] = acc;
  }
  __syncthreads();
  for (int r = threadIdx.x; r <= n; r += blockDim.x) child_ptr[lo + r] = cnt[r];
  __syncthreads();
  // one thread per parent row: collect its children in node order, then sort by token
  for (int r = threadIdx.x; r < n; r += blockDim.x) {
    int k = cnt[r];
    for (int i = r + 1; i < n; ++i)
      if (parents[lo + i] == r) {
        child_tok[k] = tokens[lo + i];
        child_node[k] = lo + i;
        ++k;
      }
    for (int a = cnt[r] + 1; a < k; ++a) {               // insertion sort by token, stable
      const int t = child_tok[a], nd = child_node[a];
      int c = a - 1;
      while (c >= cnt[r] && child_tok[c] > t) {
        child_tok[c + 1] = child_tok[c];
        child_node[c + 1] = child_node[c];
        --c;
      }
      child_tok[c + 1] = t;
      child_node[c + 1] = nd;
    }
  }
}

__device__ __forceinline__ LmPart merge_part(const LmPart& a, const LmPart& b) {
  if (b.idx == INT_MAX) return a;
  if (a.idx == INT_MAX) return b;
  LmPart r;
  if (a.m == b.m) {
    r.s = a.s + b.s;
    r.m = a.m;
    r.idx = min(a.idx, b.idx);
  } else if (a.m > b.m) {
    r.s = a.s + b.s * (double)expf(b.m - a.m);
    r.m = a.m;
    r.idx = a.idx;
  } else {
    r.s = b.s + a.s * (double)expf(a.m - b.m);
    r.m = b.m;
    r.idx = b.idx;
  }
  return r;
}

__device__ __forceinline__ float prob_bf16(float x, float m, float s) {
  return round_to_bf16(__fdiv_rn(expf(x - m), s));
}

__device__ __forceinline__ float prev_bf16(float x) {
  uint32_t u = __float_as_uint(x) >> 16;
  if (x == 0.0f) return -__uint_as_float(1u << 16);
  u = (x > 0.0f) ? u - 1 : u + 1;
  return __uint_as_float(u << 16);
}

// One warp per row: the tiles' partials merged in tile order (each lane a run
// of consecutive tiles, then the lanes in order), the row statistics, and the
// argmax of the bf16-rounded probabilities settled from the candidate lists
// when the largest value below the max rounds to the same probability.  A row
// whose tie the lists cannot settle (a full list whose smallest value still
// ties) is marked in `unresolved`.
__global__ void lmhead_merge_kernel(const LmParams p, RowStatOut* out, int* unresolved) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= p.M) return;
  const LmPart* parts = p.parts + (int64_t)row * p.n_sub;
  const int per = (p.n_sub + 31) / 32;
  const int t0 = lane * per, t1 = min(p.n_sub, t0 + per);
  LmPart acc{0.0, -INFINITY, INT_MAX};
  for (int t = t0; t < t1; ++t) acc = merge_part(acc, parts[t]);
  // lanes in order: lane 0 takes lane 1's run, then lane 2's ...
  for (int o = 1; o < 32; ++o) {
    LmPart other;
    other.s = __shfl_sync(0xffffffffu, acc.s, o);
    other.m = __shfl_sync(0xffffffffu, acc.m, o);
    other.idx = __shfl_sync(0xffffffffu, acc.idx, o);
    if (lane == 0) acc = merge_part(acc, other);
  }
  RowStatOut rs;
  rs.m = __shfl_sync(0xffffffffu, acc.m, 0);
  rs.s = (float)__shfl_sync(0xffffffffu, acc.s, 0);
  rs.argmax = __shfl_sync(0xffffffffu, acc.idx, 0);
  rs.flags = 0;
  const float qmax = round_to_bf16(__fdiv_rn(1.0f, rs.s));
  const bool tie = (rs.m > -INFINITY) && (prob_bf16(prev_bf16(rs.m), rs.m, rs.s) == qmax);
  int bad = 0;
  if (tie) {
    int best = INT_MAX;
    for (int t = t0; t < t1; ++t) {
      // a tile whose max is <= -4 holds no value that can tie; one whose max
      // is >= 4 cannot belong to a tied row (ties need |m| < 2)
      if (!(parts[t].m > -kCandRange && parts[t].m < kCandRange)) continue;
      const Cand* cl = p.cands + ((int64_t)row * p.n_sub + t) * kCand;
      bool full = true;
      float last = INFINITY;
      for (int k = 0; k < kCand; ++k) {
        const Cand c = cl[k];
        if (c.idx == INT_MAX) {
          full = false;
          break;
        }
        last = c.v;
        if (prob_bf16(c.v, rs.m, rs.s) == qmax) best = min(best, c.idx);
      }
      if (full && prob_bf16(last, rs.m, rs.s) == qmax) bad = 1;
    }
    best = (int)__reduce_min_sync(0xffffffffu, (unsigned)best);
    bad = __any_sync(0xffffffffu, bad);
    rs.argmax = best;
  }
  if (lane == 0) {
    out[row] = rs;
    unresolved[row] = bad;
  }
}

// Requests with an unresolved row: counts[b][0] = -4 (the caller redoes them
// from materialised logits).
__global__ void mark_unresolved_kernel(const int32_t* row_indptr, const int* unresolved, int32_t* out_counts) {
  const int b = blockIdx.x;
  const int lo = row_indptr[b], hi = row_indptr[b + 1];
  int bad = 0;
  for (int r = lo + threadIdx.x; r < hi; r += blockDim.x) bad |= unresolved[r];
  bad = __syncthreads_or(bad);
  if (threadIdx.x == 0 && bad) out_counts[b * 4] = -4;
}

size_t lm_ws_layout(int M, int V, size_t* off_parts, size_t* off_cands, size_t* off_child, size_t* off_stats,
                    size_t* off_tok, size_t* off_unres) {
  const int n_sub = 2 * ((V + kBN - 1) / kBN);
  size_t o = 0;
  *off_parts = o;
  o = align_up(o + (size_t)M * n_sub * sizeof(LmPart), 256);
  *off_cands = o;
  o = align_up(o + (size_t)M * n_sub * kCand * sizeof(Cand), 256);
  *off_child = o;                                        // child_ptr [M+1], child_tok [M], child_node [M]
  o = align_up(o + (size_t)(3 * M + 1) * sizeof(int32_t), 256);
  *off_stats = o;
  o = align_up(o + (size_t)M * sizeof(RowStatOut), 256);
  *off_tok = o;
  o = align_up(o + (size_t)M * sizeof(float), 256);
  *off_unres = o;
  o = align_up(o + (size_t)M * sizeof(int) + 16, 256);   // per-row flags, then the error word
  return o;
}

int num_sms() {
  static int count[256] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return 148;
  if (!count[dev]) {
    int c = 0;
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
    count[dev] = c;
  }
  return count[dev];
}

int lmhead_launch(const void* hidden, const void* weight, int M, int V, int K, LmParams& p, cudaStream_t stream) {
  PTS_CHECK_ARG(hidden && weight, "null hidden or weight");
  PTS_CHECK_ARG(M > 0 && V > 0 && K > 0, "bad sizes");
  if (K % kBK) return set_error(PTS_ERR_UNSUPPORTED, "hidden size %d (this build: a multiple of %d)", K, kBK);
  PTS_CHECK_ARG(((uintptr_t)hidden & 15) == 0 && ((uintptr_t)weight & 15) == 0, "hidden/weight must be 16-byte aligned");
  CUtensorMap a_map, b_map;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
    if (int rc = encode_tiled_bf16_sw128(&a_map, 2, hidden, dims, strides, box)) return rc;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)V};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBN};
    if (int rc = encode_tiled_bf16_sw128(&b_map, 2, weight, dims, strides, box)) return rc;
  }
  p.M = M;
  p.V = V;
  p.K = K;
  p.m_tiles = (M + kBM - 1) / kBM;
  p.n_tiles = (V + kBN - 1) / kBN;
  p.n_sub = 2 * p.n_tiles;
  p.tiles = p.m_tiles * p.n_tiles;
  p.k_blocks = K / kBK;
  if (int rc = ensure_smem_attr((const void*)lmhead_kernel, kSmemBytes)) return rc;
  const int grid = min(p.tiles, num_sms());
  lmhead_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p, a_map, b_map);
  return launch_status("lmhead_kernel");
}

}  // namespace
}  // namespace pts

using namespace pts;

extern "C" int pts_lmhead_logits(const void* hidden, const void* weight, int num_rows, int vocab, int hidden_size,
                                 void* logits, int64_t logits_stride, pts_stream_t stream) {
  PTS_CHECK_ARG(logits, "null logits");
  PTS_CHECK_ARG(logits_stride >= vocab, "logits_stride %lld below vocab %d", (long long)logits_stride, vocab);
  LmParams p{};
  p.mode = 1;
  p.logits = (uint16_t*)logits;
  p.logits_stride = logits_stride;
  return lmhead_launch(hidden, weight, num_rows, vocab, hidden_size, p, (cudaStream_t)stream);
}

extern "C" size_t pts_lmhead_workspace_size(int num_rows, int vocab) {
  if (num_rows <= 0 || vocab <= 0) return 0;
  size_t a, b, c, d, e, f;
  return lm_ws_layout(num_rows, vocab, &a, &b, &c, &d, &e, &f);
}

extern "C" int pts_accept_walk_merged(void* row_stats, const float* token_logit, const int32_t* ties_all,
                                      int num_shards, const int32_t* row_indptr, const int32_t* parents,
                                      const int32_t* tokens, const float* draft_probs, int batch, int num_rows,
                                      int vocab, int max_nodes, int64_t eos_token_id, uint64_t philox_seed,
                                      uint64_t philox_offset, int32_t* out_tokens, int32_t* out_hidden,
                                      int32_t* out_counts, int out_stride, pts_stream_t stream);

extern "C" int pts_lmhead_accept(const void* hidden, const void* weight, int num_rows, int vocab, int hidden_size,
                                 const int32_t* row_indptr, const int32_t* parents, const int32_t* tokens,
                                 const float* draft_probs, int batch, int max_nodes, int64_t eos_token_id,
                                 int traversal, float temperature, uint64_t philox_seed, uint64_t philox_offset,
                                 int32_t* out_tokens, int32_t* out_hidden, int32_t* out_counts, int out_stride,
                                 void* workspace, size_t workspace_bytes, pts_stream_t stream) {
  PTS_CHECK_ARG(row_indptr && parents && tokens && out_tokens && out_hidden && out_counts, "null pointer");
  PTS_CHECK_ARG(!traversal || draft_probs, "null draft_probs");
  PTS_CHECK_ARG(batch > 0 && num_rows >= batch, "need batch > 0 and num_rows >= batch");
  PTS_CHECK_ARG(temperature > 0.0f, "temperature must be positive");
  if (max_nodes > PTS_MAX_TREE_NODES)
    return set_error(PTS_ERR_CAPACITY, "max_nodes %d above %d", max_nodes, PTS_MAX_TREE_NODES);
  size_t op, oc, och, ost, otk, oun;
  const size_t need = lm_ws_layout(num_rows, vocab, &op, &oc, &och, &ost, &otk, &oun);
  if (!workspace || workspace_bytes < need)
    return set_error(PTS_ERR_CAPACITY, "workspace of %zu bytes, need %zu", workspace_bytes, need);
  uint8_t* ws = (uint8_t*)workspace;
  cudaStream_t st = (cudaStream_t)stream;
  LmParams p{};
  p.mode = 0;
  const bool use_temp = traversal && temperature != 1.0f;
  p.use_temp = use_temp;
  p.inv_temp = 1.0f / temperature;
  p.parts = (LmPart*)(ws + op);
  p.cands = (Cand*)(ws + oc);
  int32_t* child = (int32_t*)(ws + och);
  p.child_ptr = child;
  p.child_tok = child + num_rows + 1;
  p.child_node = child + 2 * num_rows + 1;
  p.tok_logit = (float*)(ws + otk);
  int* unres = (int*)(ws + oun);
  p.err = unres + num_rows;
  child_lists_kernel<<<batch, 128, 0, st>>>(row_indptr, parents, tokens, child, (int32_t*)p.child_tok,
                                           (int32_t*)p.child_node, p.tok_logit);
  if (int rc = launch_status("child_lists_kernel")) return rc;
  if (int rc = lmhead_launch(hidden, weight, num_rows, vocab, hidden_size, p, st)) return rc;
  RowStatOut* stats = (RowStatOut*)(ws + ost);
  lmhead_merge_kernel<<<(num_rows * 32 + 255) / 256, 256, 0, st>>>(p, stats, unres);
  if (int rc = launch_status("lmhead_merge_kernel")) return rc;
  // the argmax of every row is final (flags 0), so the walk reads no tie indices
  if (int rc = pts_accept_walk_merged(stats, p.tok_logit, unres, 1, row_indptr, parents, tokens,
                                      traversal ? draft_probs : nullptr, batch, num_rows, vocab, max_nodes,
                                      eos_token_id, traversal ? philox_seed : 0, philox_offset, out_tokens,
                                      out_hidden, out_counts, out_stride, stream))
    return rc;
  mark_unresolved_kernel<<<batch, 128, 0, st>>>(row_indptr, unres, out_counts);
  return launch_status("mark_unresolved_kernel");
}
