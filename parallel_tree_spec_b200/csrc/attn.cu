// Tree-masked paged attention on sm_100a (TMA + tcgen05 + TMEM).
//
// Work unit (one CTA): request b, KV head h, and a group of up to three
// 128-row query tiles.  Query rows are (tree node, query head of h's GQA
// group) pairs, head fastest, so one tile holds 128/g consecutive nodes and
// is a single TMA box of the [T, Hq, D] query tensor.
//
// Per 32-token KV block (two 16-token pages):
//   warp 0 (TMA)      loads K and V of both pages into a 4-stage ring
//                     (128-byte swizzle, two 64-column halves of D each);
//   warp 1 (MMA)      issues S_t = Q_t K^T (M=128, N=32, K=128) into TMEM for
//                     each tile t, then O_t += P_t V (M=128, N=128, K=32);
//   warps 2-5, 6-9    (two softmax warpgroups: the first owns tiles 0 and 2,
//                     the second tile 1; warp w reads TMEM lanes 32*(w%4)..)
//                     read S_t, apply the scale and the tree mask, keep a
//                     running max and sum per row, write P_t (bf16) to shared
//                     memory, and rescale O_t in TMEM when the row max grows by
//                     more than 2^8 (lazy rescaling keeps exp2 arguments <= 8).
// The MMA warp issues S_t for block j+1 right after O_t's update for block j,
// so the tensor pipe works on the next block while the softmax warps finish
// the current one.  After the last block each warpgroup normalises its O_t by
// the row sum and stores bf16 rows.  TMEM: O_t at columns 128*t, S_t at
// 384 + 32*t.  The request's page table is staged in shared memory.
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
constexpr int kBlockN = 32;           // KV tokens per block
constexpr int kTilesPerCta = 3;
constexpr int kPage = 16;
constexpr int kD = 128;
constexpr int kThreads = 320;         // warp 0 TMA, warp 1 MMA, warps 2-9 softmax
constexpr int kMaxSmemPages = 2048;   // page-table entries staged in shared memory
constexpr uint32_t kTileBytes = 128 * kD * 2;                 // one Q tile (both halves)
constexpr uint32_t kHalfBytes = 128 * 128;                    // [128 rows x 64 cols] bf16
constexpr uint32_t kStageBytes = 4 * kBlockN * 128;           // K(2 halves) + V(2 halves)
constexpr uint32_t kPBytes = 128 * 128;                       // P tile in 128-byte rows
constexpr float kRescaleThreshold = 8.0f;

struct __align__(8) Bars {
  uint64_t q_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[kTilesPerCta];
  uint64_t s_free[kTilesPerCta];
  uint64_t p_full[kTilesPerCta];
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem;
  int abort;
};

constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffKV = kOffQ + kTilesPerCta * kTileBytes;
constexpr uint32_t kOffP = kOffKV + kStages * kStageBytes;
constexpr uint32_t kOffPages = kOffP + kTilesPerCta * kPBytes;
constexpr uint32_t kOffBars = kOffPages + kMaxSmemPages * 4;
constexpr uint32_t kSmemBytes = kOffBars + 1024 + 1024;       // bars + alignment slack

struct AttnParams {
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

__device__ __forceinline__ uint32_t sw128_chunk(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ void record_abort(Bars& bars, const AttnParams& p, int code) {
  *(volatile int*)&bars.abort = 1;
  if (p.err) atomicExch(p.err, code);
}

__device__ __forceinline__ bool aborted(const Bars& bars) { return *(volatile const int*)&bars.abort != 0; }

__global__ void __launch_bounds__(kThreads, 1)
    tree_attn_kernel(const AttnParams p, const __grid_constant__ CUtensorMap q_map,
                     const __grid_constant__ CUtensorMap kv_map) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  Bars& bars = *reinterpret_cast<Bars*>(smem + kOffBars);

  const int h = blockIdx.x, b = blockIdx.y, group = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q0 = p.qo_indptr[b];
  const int n_nodes = p.qo_indptr[b + 1] - q0;
  const int rows = n_nodes * p.g;
  const int tiles_total = (rows + 127) / 128;
  const int tile0 = group * kTilesPerCta;
  const int n_tiles = min(kTilesPerCta, tiles_total - tile0);
  if (n_tiles <= 0) return;
  const int p0 = p.page_indptr[b];
  const int n_pages = p.page_indptr[b + 1] - p0;
  if (n_pages <= 0) return;
  const int kv_len = (n_pages - 1) * kPage + p.last_page_len[b];
  const int prefix = kv_len - n_nodes;
  const int n_blocks = (kv_len + kBlockN - 1) / kBlockN;
  const int nodes_per_tile = 128 / p.g;

  if (threadIdx.x == 0) {
    mbar_init(&bars.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars.kv_full[s], 1);
      mbar_init(&bars.kv_empty[s], 1);
    }
    for (int t = 0; t < kTilesPerCta; ++t) {
      mbar_init(&bars.s_full[t], 1);
      mbar_init(&bars.s_free[t], 4);      // one arrival per softmax warp
      mbar_init(&bars.p_full[t], 4);
    }
    mbar_init(&bars.o_full, 1);
    mbar_init(&bars.drain, 1);
    bars.abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&q_map);
    tma_prefetch_desc(&kv_map);
  }
  if (warp == 1) {
    tmem_alloc(&bars.tmem, 512);
    tmem_relinquish();
  }
  int32_t* spages = (int32_t*)(smem + kOffPages);
  if (warp == 0) {
    for (int i = lane; i < min(n_pages, kMaxSmemPages); i += 32) spages[i] = p.page_indices[p0 + i];
  }
  if (warp >= 2) {
    // rows of P that no softmax thread writes must read as zero
    uint4* pz = (uint4*)(smem + kOffP);
    for (int i = threadIdx.x - 64; i < (int)(kTilesPerCta * kPBytes / 16); i += kThreads - 64)
      pz[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars.q_full, (uint32_t)n_tiles * kTileBytes);
      for (int t = 0; t < n_tiles; ++t) {
        const int node0 = q0 + (tile0 + t) * nodes_per_tile;
        for (int half = 0; half < 2; ++half)
          tma_load_4d(smem + kOffQ + t * kTileBytes + half * kHalfBytes, &q_map, &bars.q_full, half * 64, 0, h,
                      node0);
      }
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
        for (int pg = 0; pg < 2; ++pg) {
          const int slot = 2 * j + pg;
          const int phys = slot >= n_pages ? p.max_pages                                // OOB -> zero fill
                           : (slot < kMaxSmemPages ? spages[slot] : p.page_indices[p0 + slot]);
          const int page = (phys >= 0 && phys < p.max_pages) ? phys : p.max_pages;
          for (int half = 0; half < 2; ++half) {
            tma_load_4d(st + half * (kBlockN * 128) + pg * (kPage * 128), &kv_map, &bars.kv_full[s], half * 64, h,
                        0, 2 * page);
            tma_load_4d(st + 2 * (kBlockN * 128) + half * (kBlockN * 128) + pg * (kPage * 128), &kv_map,
                        &bars.kv_full[s], half * 64, h, 0, 2 * page + 1);
          }
        }
        issued = j + 1;
      }
      // wait for copies still in flight before the CTA can exit
      for (int j = max(0, issued - kStages); j < issued; ++j) mbar_wait(&bars.kv_full[j % kStages], (j / kStages) & 1);
      mbar_wait(&bars.q_full, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp walks the loop; one elected lane issues.  Every operand
    // descriptor is a base descriptor plus a compile-time offset (the block
    // loop is unrolled by the stage count), which keeps the issue rate at the
    // tensor pipe's rate.
    const uint32_t id_qk = idesc_bf16_f32(128, kBlockN, 0, 0);
    const uint32_t id_pv = idesc_bf16_f32(128, kD, 0, 1);
    const uint64_t qd0 = smem_desc(smem_u32(smem + kOffQ), 16, 1024, kSwizzle128B);
    const uint64_t kd0 = smem_desc(smem_u32(smem + kOffKV), 16, 1024, kSwizzle128B);
    const uint64_t vd0 = smem_desc(smem_u32(smem + kOffKV + 2 * kBlockN * 128), kBlockN * 128, 1024, kSwizzle128B);
    const uint64_t pd0 = smem_desc(smem_u32(smem + kOffP), 16, 1024, kSwizzle128B);
    const bool leader = elect_one();
#define PTS_QK(T, S)                                                                                          \
  do {                                                                                                        \
    if (leader) {                                                                                             \
      _Pragma("unroll") for (int k = 0; k < kD / 16; ++k) {                                                   \
        const uint64_t a = qd0 + (uint64_t)(((T) * kTileBytes + (k / 4) * kHalfBytes + (k % 4) * 32) >> 4);    \
        const uint64_t bd = kd0 + (uint64_t)(((S) * kStageBytes + (k / 4) * (kBlockN * 128) + (k % 4) * 32) >> 4); \
        mma_bf16_ss(tmem + 384 + 32 * (T), a, bd, id_qk, k > 0);                                              \
      }                                                                                                       \
      mma_commit(&bars.s_full[T]);                                                                            \
    }                                                                                                         \
    __syncwarp();                                                                                             \
  } while (0)
    bool ok = mbar_wait(&bars.q_full, 0) && mbar_wait(&bars.kv_full[0], 0);
    if (!ok && lane == 0) record_abort(bars, p, 21);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
#pragma unroll
      for (int t = 0; t < kTilesPerCta; ++t)
        if (t < n_tiles) PTS_QK(t, 0);
    }
    for (int j0 = 0; ok && j0 < n_blocks; j0 += kStages) {
#pragma unroll
      for (int ss = 0; ss < kStages; ++ss) {
        const int j = j0 + ss;
        if (j >= n_blocks || !ok) break;
        const int s1 = (ss + 1) % kStages;
        const bool more = j + 1 < n_blocks;
#pragma unroll
        for (int t = 0; t < kTilesPerCta; ++t) {
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
              const uint64_t a = pd0 + (uint64_t)((t * kPBytes + k * 32) >> 4);
              const uint64_t bd = vd0 + (uint64_t)((ss * kStageBytes + k * 2048) >> 4);
              mma_bf16_ss(tmem + 128 * t, a, bd, id_pv, (j > 0 || k > 0) ? 1u : 0u);
            }
            if (t == n_tiles - 1) mma_commit(&bars.kv_empty[ss]);
          }
          __syncwarp();
          if (more) {
            // S_t for the next block: its K stage must have landed and the
            // softmax must have read S_t of this block
            w_ok = (t != 0 || mbar_wait(&bars.kv_full[s1], ((j + 1) / kStages) & 1)) &&
                   mbar_wait(&bars.s_free[t], j & 1);
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
  } else {
    // ------------------------------------------------------------ softmax warpgroup
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;
    const int wg = (warp - 2) >> 2;                 // 0: tiles 0 and 2, 1: tile 1
    auto owns = [&](int t) { return wg == 0 ? (t != 1) : (t == 1); };
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float m_used[kTilesPerCta], l_sum[kTilesPerCta];
    bool valid[kTilesPerCta];
    int node[kTilesPerCta];
#pragma unroll
    for (int t = 0; t < kTilesPerCta; ++t) {
      const int R = (tile0 + t) * 128 + r_local;
      valid[t] = (t < n_tiles) && (R < rows);
      node[t] = R / p.g;
      m_used[t] = -INFINITY;
      l_sum[t] = 0.0f;
    }
    bool ok = true;
    for (int j = 0; ok && j < n_blocks; ++j) {
      const int kv0 = j * kBlockN;
      const bool plain = (kv0 + kBlockN <= prefix);
#pragma unroll
      for (int t = 0; t < kTilesPerCta; ++t) {
        if (t >= n_tiles) break;
        if (!owns(t)) continue;
        if (!mbar_wait(&bars.s_full[t], j & 1)) {
          record_abort(bars, p, 31);
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[32];
        tmem_ld32(tmem + lane_base + 384 + 32 * t, sr);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.s_free[t]);
        float x[32];
        float mblk = -INFINITY;
        if (valid[t]) {
          if (plain) {
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              x[c] = __uint_as_float(sr[c]) * p.scale_log2;
              mblk = fmaxf(mblk, x[c]);
            }
          } else {
            const uint64_t* mrow = p.mask_bits ? p.mask_bits + (int64_t)(q0 + node[t]) * p.mask_words : nullptr;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const int kv = kv0 + c;
              bool vis = kv < kv_len;
              if (vis && kv >= prefix) {
                const int tn = kv - prefix;
                vis = p.mask_bits == nullptr
                          ? (tn <= node[t])
                          : (tn / 64 < p.mask_words) && ((__ldg(mrow + tn / 64) >> (tn % 64)) & 1ull);
              }
              x[c] = vis ? __uint_as_float(sr[c]) * p.scale_log2 : -INFINITY;
              mblk = fmaxf(mblk, x[c]);
            }
          }
        }
        // lazy rescale: warp-uniform decision, per-row factors
        const bool need = valid[t] && (mblk > m_used[t] + kRescaleThreshold);
        float alpha = 1.0f;
        if (need) {
          const float mnew = mblk;
          alpha = (m_used[t] == -INFINITY) ? 0.0f : fast_exp2(m_used[t] - mnew);
          l_sum[t] *= alpha;
          m_used[t] = mnew;
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          for (int cb = 0; cb < 4; ++cb) {
            uint32_t o[32];
            const uint32_t oa = tmem + lane_base + 128 * t + 32 * cb;
            tmem_ld32(oa, o);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st32(oa, o);
          }
          tmem_st_wait();
        }
        if (valid[t]) {
          const float mu = m_used[t];
          float ls = 0.0f;
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float e0 = (mu == -INFINITY) ? 0.0f : fast_exp2(x[c] - mu);
            const float e1 = (mu == -INFINITY) ? 0.0f : fast_exp2(x[c + 1] - mu);
            ls += e0 + e1;
            pk[c / 2] = pack_bf16x2(e0, e1);
          }
          l_sum[t] += ls;
          uint8_t* prow = smem + kOffP + t * kPBytes;
#pragma unroll
          for (int ch = 0; ch < 4; ++ch)
            *(uint4*)(prow + sw128_chunk((uint32_t)r_local, (uint32_t)ch)) =
                make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.p_full[t]);
      }
      if (aborted(bars)) ok = false;
    }
    // ------------------------------------------------------------ epilogue
    if (ok && mbar_wait(&bars.o_full, 0)) {
      tc_fence_after();
      for (int t = 0; t < n_tiles; ++t) {
        if (!owns(t)) continue;
        const float inv = (valid[t] && l_sum[t] > 0.0f) ? 1.0f / l_sum[t] : 0.0f;
        const int R = (tile0 + t) * 128 + r_local;
        const int hh = R % p.g;
        uint16_t* orow = p.out + ((int64_t)(q0 + node[t]) * p.Hq + h * p.g + hh) * kD;
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + 128 * t + 32 * cb, o);
          tmem_ld_wait();
          if (valid[t]) {
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
      }
    } else if (ok) {
      record_abort(bars, p, 32);
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
  if (g > 128 || 128 % g != 0) return set_error(PTS_ERR_UNSUPPORTED, "GQA group %d must divide 128", g);
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

  CUtensorMap q_map, kv_map;
  {
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)g, (cuuint64_t)num_kv_heads, (cuuint64_t)total_q};
    const cuuint64_t strides[3] = {(cuuint64_t)kD * 2, (cuuint64_t)g * kD * 2, (cuuint64_t)num_qo_heads * kD * 2};
    const cuuint32_t box[4] = {64, (cuuint32_t)g, 1, (cuuint32_t)(128 / g)};
    int rc = encode_4d(&q_map, q, dims, strides, box);
    if (rc) return rc;
  }
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
  const int groups = ((max_qo_len * g + 127) / 128 + kTilesPerCta - 1) / kTilesPerCta;
  if (groups > 65535) return set_error(PTS_ERR_CAPACITY, "%d query rows per request is too many", max_qo_len);
  dim3 grid(num_kv_heads, batch, groups);
  tree_attn_kernel<<<grid, kThreads, kSmemBytes, (cudaStream_t)stream>>>(p, q_map, kv_map);
  return launch_status("tree_attn_kernel");
}
