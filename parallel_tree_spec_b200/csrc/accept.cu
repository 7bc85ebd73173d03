// Fused tree acceptance over bf16 logits (greedy and traversal verification).
//
// One launch does everything.  Each logits row is owned by a thread-block
// cluster of C = ceil(V / 16384) CTAs (256 threads x 64 elements each, the
// whole chunk held in registers after one 128-bit streaming load per vector;
// four CTAs per SM so loads of one CTA overlap the reductions of others):
//   1. every thread reduces its 64 values to (max m_t, sum_t exp(x - m_t),
//      first index of m_t) in one pass (packed bf16x2 max, ex2.approx);
//   2. warp, CTA and cluster merges combine the partials: m = max, s = sum of
//      s_t * exp(m_t - m) (CUDA expf factors, double above the warp level),
//      argmax = first index of m; every cluster rank pushes its partial into
//      rank 0 through distributed shared memory and a remote mbarrier arrive;
//   3. rank 0 takes the argmax of the bf16-rounded probabilities
//      bf16(exp(x - m) / s): the first index of m, unless a value just below m
//      can round to the same probability (only possible for small m), in
//      which case the row is rescanned with the exact rounding rule;
//   4. the last row of a request to finish (acquire/release counter) walks the
//      tree on the device: the greedy walk of verify_tree_exact
//      (verification.py:185-268) or the traversal loop of
//      verify_tree_traversal (verification.py:275-524).
// The probabilities that decide anything (per-node target probabilities,
// argmax ties) are computed like torch's softmax epilogue: expf(x - m) / s.
//
// Traversal walk.  The reference updates p_alpha of every descendant of the
// rejected node's siblings after each rejection (verification.py:461-477).
// Every such update recomputes pa[v] = min(pa[parent(v)] * Mb[v]/Ms[v], 1)
// from the parent's current value, and the only value ever set otherwise is
// pa[parent] = p_new at a rejection (:440), after which its whole subtree is
// recomputed.  So at every moment pa[v] equals min(pa[parent] * ratio(v), 1)
// with current values unless v was such a parent more recently than any of
// its ancestors: this walk keeps those "sticky" values with time stamps and
// evaluates every other p_alpha on demand along the descent path, which gives
// the reference's values with no descendant sweep.  After a rejection the
// path above the rejected node is unchanged, so the next descent restarts at
// its parent.  Fp32 tensor arithmetic and fp64 scalar arithmetic are replayed
// with explicitly rounded operations in the reference's order.
//
// Workspace (caller-owned): row stats and a per-request counter array that
// is cleared at the start of every call.
#include <cooperative_groups.h>
#include <float.h>
#include <limits.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace pts {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kVecPerThread = 8;                           // 8 x 16 B per thread
constexpr int kChunk = kThreads * kVecPerThread * 8;       // 16384 elements per CTA
constexpr int kMaxCluster = 16;                            // above 8 needs the non-portable opt-in
constexpr float kEps32 = 1e-8f;
constexpr double kEps = 1e-8;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxDraws = 2 * PTS_MAX_TREE_NODES + 2;

struct RowStat {
  float m;
  float s;
  int argmax;
  int flags;
};

struct AcceptParams {
  const uint16_t* logits;
  int64_t row_stride;
  const int32_t* row_indptr;
  const int32_t* parents;
  const int32_t* tokens;
  const float* draft_probs;
  int batch, num_rows, vocab, cluster, max_nodes, out_stride;
  int64_t eos;
  float inv_temp;
  int use_temp;
  int traversal;
  int vec_ok;
  uint64_t seed, offset;
  int32_t* out_tokens;
  int32_t* out_hidden;
  int32_t* out_counts;
  RowStat* row_ws;
  unsigned* req_ctr;
};

__device__ __forceinline__ float load_scaled(const AcceptParams& p, const uint16_t* row, int i) {
  float x = bf16_bits_to_float(row[i]);
  if (p.use_temp) x = round_to_bf16(__fmul_rn(x, p.inv_temp));
  return x;
}

// bf16-rounded softmax probability of value x in a row with max m, sum s,
// evaluated like torch's softmax epilogue: exp(x - m) / s.
__device__ __forceinline__ float prob_bf16(float x, float m, float s) {
  return round_to_bf16(__fdiv_rn(expf(x - m), s));
}

// Largest bf16 value strictly below the (finite, bf16-representable) x.
__device__ __forceinline__ float prev_bf16(float x) {
  uint32_t u = __float_as_uint(x) >> 16;
  if (x == 0.0f) return -__uint_as_float(1u << 16);
  u = (x > 0.0f) ? u - 1 : u + 1;
  return __uint_as_float(u << 16);
}

__device__ __forceinline__ uint4 ld_stream(const uint16_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t bf16x2_max(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t scale_pair(uint32_t v, float inv_t) {
  const float lo = round_to_bf16(__fmul_rn(__uint_as_float(v << 16), inv_t));
  const float hi = round_to_bf16(__fmul_rn(__uint_as_float(v & 0xffff0000u), inv_t));
  return (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
}

// (max, sum of exp(x - max), first index of max) partials.
struct Part {
  float m;
  double s;
  int idx;
};

__device__ __forceinline__ Part merge(const Part& a, const Part& b) {
  if (b.m == -INFINITY) return a;
  if (a.m == -INFINITY) return b;
  Part r;
  if (a.m == b.m) {
    r.m = a.m;
    r.s = a.s + b.s;
    r.idx = min(a.idx, b.idx);
  } else if (a.m > b.m) {
    r.m = a.m;
    r.s = a.s + b.s * (double)expf(b.m - a.m);
    r.idx = a.idx;
  } else {
    r.m = b.m;
    r.s = b.s + a.s * (double)expf(a.m - b.m);
    r.idx = b.idx;
  }
  return r;
}

__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t local = (uint32_t)__cvta_generic_to_shared(p), remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}

__device__ __forceinline__ void mbar_init_local(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(bar);
  uint64_t t0 = 0;
  for (int it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    if (it == 0) t0 = t;
    else if (t - t0 > 2000000000ull) return false;
  }
}

__device__ __forceinline__ int block_reduce_min(int v, int* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kWarps ? sm[lane] : INT_MAX;
#pragma unroll
    for (int o = kWarps / 2; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) sm[0] = v;
  }
  __syncthreads();
  return sm[0];
}

struct WalkSmem {
  int32_t token[PTS_MAX_TREE_NODES];
  int16_t sticky_t[PTS_MAX_TREE_NODES];    // time p_alpha was last set directly (-1: never)
  int16_t reset_t[PTS_MAX_TREE_NODES];     // time the node's subtree was last recomputed
  int16_t first_child[PTS_MAX_TREE_NODES];
  int16_t next_sib[PTS_MAX_TREE_NODES];
  int16_t first_valid[PTS_MAX_TREE_NODES];
  int16_t parent[PTS_MAX_TREE_NODES];
  int16_t path[PTS_MAX_TREE_NODES];
  int16_t path_rmax[PTS_MAX_TREE_NODES];
  int16_t sib[PTS_MAX_TREE_NODES];
  float path_pa[PTS_MAX_TREE_NODES];
  float mb[PTS_MAX_TREE_NODES];
  float ms[PTS_MAX_TREE_NODES];
  float stored_pa[PTS_MAX_TREE_NODES];
  float uni[kMaxDraws];
  uint8_t valid[PTS_MAX_TREE_NODES];
};

__device__ void write_counts(const AcceptParams& p, int b, int n_out, int total, int acc, int node) {
  int32_t* c = p.out_counts + (int64_t)b * 4;
  c[0] = n_out;
  c[1] = total;
  c[2] = acc;
  c[3] = node;
}

// Greedy walk (verify_tree_exact, verification.py:185-268), one thread.
__device__ void walk_greedy(const AcceptParams& p, int b, int lo, const WalkSmem& w) {
  int32_t* ot = p.out_tokens + (int64_t)b * p.out_stride;
  int32_t* oh = p.out_hidden + (int64_t)b * p.out_stride;
  int cur = 0, total = 0, acc = 0, n_out = 0;
  int bonus = -1, last_tok = -1;
  while (w.first_child[cur] >= 0) {                                   // :232
    total++;
    const int tok = __ldcg(&p.row_ws[lo + cur].argmax);               // :73
    int match = -1;
    for (int c = w.first_child[cur]; c >= 0; c = w.next_sib[c])
      if (w.token[c] == tok) {
        match = c;
        break;
      }
    if (match >= 0) {                                                 // :237
      bonus = -1;
      acc++;
      if (n_out < p.out_stride) {
        ot[n_out] = tok;
        oh[n_out] = cur;
      }
      n_out++;
      last_tok = tok;
      if (p.eos >= 0 && (int64_t)tok == p.eos) break;                 // :242
      cur = match;                                                    // :245
      if (w.first_child[cur] < 0) break;                              // :249
    } else {
      bonus = tok;
      break;
    }
  }
  if (n_out == 0 || p.eos < 0 || (int64_t)last_tok != p.eos) {        // :257
    if (bonus < 0) bonus = __ldcg(&p.row_ws[lo + cur].argmax);        // :260-262
    if (n_out < p.out_stride) {
      ot[n_out] = bonus;
      oh[n_out] = cur;
    }
    n_out++;
  }
  write_counts(p, b, n_out > p.out_stride ? -2 : n_out, total, acc, cur);
}

__device__ __forceinline__ float ratio_of(float mb, float ms) {
  return ms > kEps32 ? __fdiv_rn(mb, ms) : 0.0f;
}

// Traversal verification (verify_tree_traversal, verification.py:377-524) by
// one warp; see the file comment for the lazily evaluated p_alpha.
__device__ void walk_traversal(const AcceptParams& p, int b, int lo, int n, WalkSmem& w) {
  const int lane = threadIdx.x & 31;
  __shared__ int s_state, s_parent, s_nsib;
  __shared__ double s_old_ms_rej, s_p_old;
  int16_t* s_sib = w.sib;
  int accepted = 0;
  int depth = 0;           // path[0..depth] is the current descent path (lane 0)
  int draw = 0;
  int T = 1;               // time stamp of the next direct p_alpha assignment
  if (lane == 0) {
    w.path[0] = 0;
    w.path_pa[0] = w.stored_pa[0];
    w.path_rmax[0] = -1;
  }
  const int max_iter = 2 * n + 2;
  for (int it = 0; it < max_iter; ++it) {                             // :377
    if (lane == 0) {
      // descend to the first valid leaf (:379-389), p_alpha evaluated lazily
      int u = w.path[depth];
      for (int c = w.first_valid[u]; c >= 0; c = w.first_valid[u]) {
        const int rmax = max(w.path_rmax[depth], w.reset_t[u]);
        const float pa = w.sticky_t[c] > rmax ? w.stored_pa[c]
                                               : fminf(__fmul_rn(w.path_pa[depth], ratio_of(w.mb[c], w.ms[c])), 1.0f);
        ++depth;
        w.path[depth] = (int16_t)c;
        w.path_pa[depth] = pa;
        w.path_rmax[depth] = (int16_t)rmax;
        u = c;
      }
      const int cand = u;
      int state = 0;
      if (!w.valid[cand]) {                                           // :391
        state = 1;
      } else {
        const float p_val = w.path_pa[depth];                         // :395
        const float eta = w.uni[draw++];                              // :396
        if (eta < p_val) {
          accepted = cand;
          state = 1;
        } else {
          w.valid[cand] = 0;                                          // :403
          const int parent = w.parent[cand];
          s_old_ms_rej = (double)w.ms[cand];
          w.ms[cand] = 0.0f;
          if (parent < 0) {                                           // :408
            accepted = 0;
            state = 1;
          } else {
            if (w.first_valid[parent] == cand) {
              int c = w.next_sib[cand];
              while (c >= 0 && !w.valid[c]) c = w.next_sib[c];
              w.first_valid[parent] = (int16_t)c;
            }
            --depth;                                                  // back to the parent
            if (w.first_valid[parent] >= 0) {                         // :417 any active sibling
              int ns = 0;
              for (int c = w.first_child[parent]; c >= 0; c = w.next_sib[c]) s_sib[ns++] = (int16_t)c;
              s_nsib = ns;
              s_parent = parent;
              s_p_old = (double)w.path_pa[depth];                     // :422
              state = 2;
            }
          }
        }
      }
      s_state = state;
    }
    __syncwarp();
    const int state = s_state;
    if (state == 1) break;
    if (state != 2) continue;
    // ---- rejection update (:421-458); per-child terms in parallel, sums in order
    const int parent = s_parent, ns = s_nsib;
    const double p_old = s_p_old;
    const float p_old32 = (float)p_old;
    const double old_ms_rej = s_old_ms_rej;
    float s_tree = 0.0f, sum_mb = 0.0f;
    for (int base = 0; base < ns; base += 32) {
      const int i = base + lane;
      float t = 0.0f, mbv = 0.0f;
      if (i < ns) {
        const int c = s_sib[i];
        mbv = w.mb[c];
        t = fmaxf(__fsub_rn(__fmul_rn(p_old32, mbv), w.ms[c]), 0.0f);
      }
      const int cnt = min(32, ns - base);
      for (int k = 0; k < cnt; ++k) {                                 // :432-433 left to right
        s_tree = __fadd_rn(s_tree, __shfl_sync(0xffffffffu, t, k));
        sum_mb = __fadd_rn(sum_mb, __shfl_sync(0xffffffffu, mbv, k));
      }
    }
    double ms_denom = __dsub_rn(1.0, old_ms_rej);                     // :424
    if (ms_denom < kEps) ms_denom = kEps;
    double S = __dadd_rn((double)s_tree, __dmul_rn(p_old, __dsub_rn(1.0, (double)sum_mb)));
    if (S < kEps) S = kEps;                                           // :435
    const double p_new = __ddiv_rn(S, __dsub_rn(__dadd_rn(S, 1.0), p_old));   // :439
    const float ms_denom32 = __double2float_rn(ms_denom);
    const float S32 = __double2float_rn(S);
    for (int i = lane; i < ns; i += 32) {                             // :443-448
      const int c = s_sib[i];
      if (!w.valid[c]) continue;
      const float msv = w.ms[c], mbv = w.mb[c];
      w.ms[c] = __fdiv_rn(msv, ms_denom32);
      w.mb[c] = __fdiv_rn(fmaxf(__fsub_rn(__fmul_rn(p_old32, mbv), msv), 0.0f), S32);
    }
    if (lane == 0) {
      const int cand = w.path[depth + 1];
      const double old_mb_rej = (double)w.mb[cand];                   // :451-452
      w.mb[cand] = __double2float_rn(
          __ddiv_rn(fmax(__dsub_rn(__dmul_rn(p_old, old_mb_rej), old_ms_rej), 0.0), S));
      const float p_new32 = __double2float_rn(p_new);                 // :440 (sticky)
      w.stored_pa[parent] = p_new32;
      w.sticky_t[parent] = (int16_t)T;
      w.reset_t[parent] = (int16_t)T;
      w.path_pa[depth] = p_new32;
      ++T;
    }
    __syncwarp();
  }
  if (lane != 0) return;
  // :480-524 output
  int d = 0;
  for (int c = accepted; c >= 0; c = w.parent[c]) w.path[d++] = (int16_t)c;   // reversed path
  int32_t* ot = p.out_tokens + (int64_t)b * p.out_stride;
  int32_t* oh = p.out_hidden + (int64_t)b * p.out_stride;
  int n_out = 0;
  int last_tok = -1;
  for (int i = d - 2; i >= 0; --i) {
    const int node = w.path[i];
    const int tok = w.token[node];
    if (n_out < p.out_stride) {
      ot[n_out] = tok;
      oh[n_out] = node;
    }
    n_out++;
    last_tok = tok;
    if (p.eos >= 0 && (int64_t)tok == p.eos) break;
  }
  if (!(n_out > 0 && p.eos >= 0 && (int64_t)last_tok == p.eos)) {
    const int bonus = __ldcg(&p.row_ws[lo + accepted].argmax);        // :511
    if (n_out < p.out_stride) {
      ot[n_out] = bonus;
      oh[n_out] = accepted;
    }
    n_out++;
  }
  write_counts(p, b, n_out > p.out_stride ? -2 : n_out, n_out, n_out > 0 ? n_out - 1 : 0, accepted);
}

__global__ void __launch_bounds__(kThreads, 4) accept_kernel(const AcceptParams p) {
  __shared__ Part s_warp[kWarps];
  __shared__ Part s_rank[kMaxCluster];
  __shared__ __align__(8) uint64_t s_bar;
  __shared__ int s_red_i[kWarps];
  __shared__ int s_flag;
  __shared__ float s_m, s_s, s_qmax;
  __shared__ int s_arg, s_tie, s_ok;
  __shared__ int s_b, s_lo, s_n;
  extern __shared__ __align__(16) uint8_t dyn_smem[];
  WalkSmem& w = *reinterpret_cast<WalkSmem*>(dyn_smem);

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int row = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint16_t* rp = p.logits + (int64_t)row * p.row_stride;
  const int base = rank * kChunk;

  if (rank == 0 && tid == 0) {
    mbar_init_local(&s_bar, (uint32_t)p.cluster);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }

  // ---- 1. load the chunk and reduce each thread's values ---------------------
  uint32_t raw[kVecPerThread * 4];
#pragma unroll
  for (int k = 0; k < kVecPerThread; ++k) {
    const int e0 = base + (k * kThreads + tid) * 8;
    if (p.vec_ok && e0 + 8 <= p.vocab) {
      const uint4 v = ld_stream(rp + e0);
      raw[4 * k + 0] = v.x;
      raw[4 * k + 1] = v.y;
      raw[4 * k + 2] = v.z;
      raw[4 * k + 3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int e = e0 + 2 * j;
        const uint32_t lo16 = e < p.vocab ? rp[e] : 0xff80u;          // -inf padding
        const uint32_t hi16 = e + 1 < p.vocab ? rp[e + 1] : 0xff80u;
        raw[4 * k + j] = lo16 | (hi16 << 16);
      }
    }
  }
  // rank 0's barrier must be initialised before any rank arrives on it
  cluster.sync();
  if (p.use_temp) {
#pragma unroll
    for (int i = 0; i < kVecPerThread * 4; ++i) raw[i] = scale_pair(raw[i], p.inv_temp);
  }
  uint32_t m2 = raw[0];
#pragma unroll
  for (int i = 1; i < kVecPerThread * 4; ++i) m2 = bf16x2_max(m2, raw[i]);
  const float mt = fmaxf(__uint_as_float(m2 << 16), __uint_as_float(m2 & 0xffff0000u));
  const float mlog = mt * kLog2e;
  float st = 0.0f;
  int first = INT_MAX;
#pragma unroll
  for (int k = kVecPerThread - 1; k >= 0; --k) {
    const int e0 = base + (k * kThreads + tid) * 8;
#pragma unroll
    for (int j = 3; j >= 0; --j) {
      const uint32_t v = raw[4 * k + j];
      const float x0 = __uint_as_float(v << 16), x1 = __uint_as_float(v & 0xffff0000u);
      st += ex2_approx(fmaf(x0, kLog2e, -mlog));
      st += ex2_approx(fmaf(x1, kLog2e, -mlog));
      if (x1 == mt && e0 + 2 * j + 1 < p.vocab) first = e0 + 2 * j + 1;
      if (x0 == mt && e0 + 2 * j < p.vocab) first = e0 + 2 * j;
    }
  }
  Part part{mt, (double)st, first};
  if (mt == -INFINITY) part = Part{-INFINITY, 0.0, INT_MAX};
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Part other;
    other.m = __shfl_xor_sync(0xffffffffu, part.m, o);
    other.s = __shfl_xor_sync(0xffffffffu, part.s, o);
    other.idx = __shfl_xor_sync(0xffffffffu, part.idx, o);
    part = (lane & o) ? merge(other, part) : merge(part, other);
  }
  if (lane == 0) s_warp[warp] = part;
  __syncthreads();
  if (tid == 0) {
    Part c = s_warp[0];
    for (int i = 1; i < kWarps; ++i) c = merge(c, s_warp[i]);
    // push this CTA's partial into rank 0's slot and arrive on its barrier
    Part* dst = cluster.map_shared_rank(&s_rank[rank], 0);
    *dst = c;
    mbar_arrive_remote(mapa_shared(&s_bar, 0));
  }
  if (rank != 0) return;

  // ---- 2. row statistics (rank 0) ---------------------------------------------
  if (tid == 0) {
    s_ok = mbar_wait_cluster(&s_bar, 0);
    if (s_ok) {
      Part r = s_rank[0];
      for (int i = 1; i < p.cluster; ++i) r = merge(r, s_rank[i]);
      const float sf = (float)r.s;
      const float qmax = round_to_bf16(__fdiv_rn(1.0f, sf));
      s_m = r.m;
      s_s = sf;
      s_qmax = qmax;
      s_arg = r.idx;
      // a smaller value can only tie with the max after rounding if the
      // largest bf16 value below m already does
      s_tie = (r.m > -INFINITY) && (prob_bf16(prev_bf16(r.m), r.m, sf) == qmax);
    }
  }
  __syncthreads();
  if (!s_ok) return;
  if (s_tie) {
    int best = INT_MAX;
    for (int e = tid; e < p.vocab; e += kThreads) {
      if (prob_bf16(load_scaled(p, rp, e), s_m, s_s) == s_qmax) {
        best = e;
        break;
      }
    }
    best = block_reduce_min(best, s_red_i);
    if (tid == 0) s_arg = best;
  }
  if (tid == 0) {
    int lo = 0, hi = p.batch - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.row_indptr[mid] <= row) lo = mid;
      else hi = mid - 1;
    }
    RowStat rs;
    rs.m = s_m;
    rs.s = s_s;
    rs.argmax = s_arg;
    rs.flags = s_tie;
    p.row_ws[row] = rs;
    s_b = lo;
    s_lo = p.row_indptr[lo];
    s_n = p.row_indptr[lo + 1] - s_lo;
    unsigned prev;    // release: this row's stats; acquire: every earlier row's
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&p.req_ctr[lo]) : "memory");
    s_flag = (prev == (unsigned)(s_n - 1));
  }
  __syncthreads();
  if (!s_flag) return;

  // ---- 3. tree walk (last row CTA of the request) ----------------------------
  const int b = s_b, lo = s_lo, n = s_n;
  if (n > p.max_nodes || n > PTS_MAX_TREE_NODES) {
    if (tid == 0) write_counts(p, b, -1, 0, 0, 0);
    return;
  }
  int bad = 0;
  for (int i = tid; i < n; i += kThreads) {
    const int par = p.parents[lo + i];
    const int tok = p.tokens[lo + i];
    if ((i == 0 && par != -1) || (i > 0 && (par < 0 || par >= i))) bad = 1;
    w.parent[i] = (int16_t)par;
    w.token[i] = tok;
    w.valid[i] = 1;
    w.sticky_t[i] = i == 0 ? 0 : -1;
    w.reset_t[i] = -1;
    w.stored_pa[i] = 1.0f;
    if (p.traversal) {
      if (i == 0) {
        w.mb[0] = 1.0f;
        w.ms[0] = 1.0f;
      } else if (par >= 0 && par < i) {
        const RowStat* rs = p.row_ws + lo + par;
        const float pm = __ldcg(&rs->m), ps = __ldcg(&rs->s);
        const float x = (tok >= 0 && tok < p.vocab)
                            ? load_scaled(p, p.logits + (int64_t)(lo + par) * p.row_stride, tok)
                            : -INFINITY;
        w.mb[i] = prob_bf16(x, pm, ps);                                // :349
        w.ms[i] = p.draft_probs[lo + i];                               // :353
      }
    }
  }
  if (p.traversal)
    for (int k = tid; k < 2 * n + 2; k += kThreads) w.uni[k] = philox_uniform(p.seed, p.offset, (uint32_t)b, (uint32_t)k);
  bad = block_reduce_min(bad ? 0 : 1, s_red_i) == 0;
  if (bad) {
    if (tid == 0) write_counts(p, b, -1, 0, 0, 0);
    return;
  }
  if (tid == 0) {
    for (int i = 0; i < n; ++i) w.first_child[i] = -1;
    for (int i = n - 1; i >= 1; --i) {                                 // ascending child lists
      const int par = w.parent[i];
      w.next_sib[i] = w.first_child[par];
      w.first_child[par] = (int16_t)i;
    }
    w.next_sib[0] = -1;
    for (int i = 0; i < n; ++i) w.first_valid[i] = w.first_child[i];
    if (!p.traversal) walk_greedy(p, b, lo, w);
  }
  __syncthreads();
  if (p.traversal && warp == 0) walk_traversal(p, b, lo, n, w);
}

size_t ws_layout(int num_rows, size_t* off_rows, size_t* off_qctr) {
  size_t o = 0;
  *off_rows = o;
  o = align_up(o + (size_t)num_rows * sizeof(RowStat), 256);
  *off_qctr = o;
  o = align_up(o + (size_t)num_rows * sizeof(unsigned), 256);
  return o;
}

int accept_launch(AcceptParams p, int traversal, float temperature, void* workspace, size_t ws_bytes,
                  cudaStream_t stream) {
  PTS_CHECK_ARG(p.logits && p.row_indptr && p.parents && p.tokens, "null input pointer");
  PTS_CHECK_ARG(p.out_tokens && p.out_hidden && p.out_counts, "null output pointer");
  PTS_CHECK_ARG(p.batch > 0 && p.num_rows >= p.batch, "need batch > 0 and num_rows >= batch");
  PTS_CHECK_ARG(p.vocab > 0 && p.row_stride >= p.vocab, "need vocab > 0 and row_stride >= vocab");
  PTS_CHECK_ARG(p.max_nodes > 0, "max_nodes must be positive");
  if (p.max_nodes > PTS_MAX_TREE_NODES)
    return set_error(PTS_ERR_CAPACITY, "max_nodes %d above PTS_MAX_TREE_NODES %d", p.max_nodes,
                     PTS_MAX_TREE_NODES);
  if (p.vocab > kMaxCluster * kChunk)
    return set_error(PTS_ERR_UNSUPPORTED, "vocab %d above %d", p.vocab, kMaxCluster * kChunk);
  PTS_CHECK_ARG(p.out_stride >= 1, "out_stride must be positive");
  PTS_CHECK_ARG(temperature > 0.0f, "temperature must be positive");
  if (p.num_rows > 65535) return set_error(PTS_ERR_CAPACITY, "num_rows %d above 65535", p.num_rows);
  size_t orw, oqc;
  const size_t need = ws_layout(p.num_rows, &orw, &oqc);
  if (!workspace || ws_bytes < need)
    return set_error(PTS_ERR_CAPACITY, "workspace of %zu bytes, need %zu", ws_bytes, need);
  PTS_CHECK_ARG(((uintptr_t)workspace & 255) == 0, "workspace must be 256-byte aligned");
  char* ws = (char*)workspace;
  p.cluster = (p.vocab + kChunk - 1) / kChunk;
  p.row_ws = (RowStat*)(ws + orw);
  p.req_ctr = (unsigned*)(ws + oqc);
  p.traversal = traversal;
  p.use_temp = (temperature != 1.0f);
  p.inv_temp = 1.0f / temperature;
  p.vec_ok = (((uintptr_t)p.logits & 15) == 0) && (p.row_stride % 8 == 0);
  PTS_CUDA_TRY(cudaMemsetAsync(ws + oqc, 0, need - oqc, stream));
  static bool smem_attr = false;
  if (!smem_attr) {
    PTS_CUDA_TRY(cudaFuncSetAttribute(accept_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(WalkSmem)));
    smem_attr = true;
  }
  if (p.cluster > 8) {
    static bool nonportable = false;
    if (!nonportable) {
      PTS_CUDA_TRY(cudaFuncSetAttribute(accept_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
      nonportable = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.cluster, p.num_rows, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = sizeof(WalkSmem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PTS_CUDA_TRY(cudaLaunchKernelEx(&cfg, accept_kernel, p));
  return launch_status("accept_kernel");
}

}  // namespace
}  // namespace pts

using namespace pts;

extern "C" size_t pts_accept_workspace_size(int num_rows, int vocab) {
  size_t a, b;
  if (num_rows <= 0 || vocab <= 0) return 0;
  return ws_layout(num_rows, &a, &b);
}

extern "C" int pts_accept_greedy(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                                 const int32_t* parents, const int32_t* tokens, int batch, int num_rows,
                                 int vocab, int max_nodes, int64_t eos_token_id, int32_t* out_tokens,
                                 int32_t* out_hidden, int32_t* out_counts, int out_stride,
                                 void* workspace, size_t workspace_bytes, pts_stream_t stream) {
  AcceptParams p{};
  p.logits = logits;
  p.row_stride = row_stride;
  p.row_indptr = row_indptr;
  p.parents = parents;
  p.tokens = tokens;
  p.draft_probs = nullptr;
  p.batch = batch;
  p.num_rows = num_rows;
  p.vocab = vocab;
  p.max_nodes = max_nodes;
  p.out_stride = out_stride;
  p.eos = eos_token_id;
  p.out_tokens = out_tokens;
  p.out_hidden = out_hidden;
  p.out_counts = out_counts;
  return accept_launch(p, 0, 1.0f, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int pts_accept_traversal(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                                    const int32_t* parents, const int32_t* tokens, const float* draft_probs,
                                    int batch, int num_rows, int vocab, int max_nodes, int64_t eos_token_id,
                                    float temperature, float top_p, int do_sample, uint64_t philox_seed,
                                    uint64_t philox_offset, int32_t* out_tokens, int32_t* out_hidden,
                                    int32_t* out_counts, int out_stride, void* workspace,
                                    size_t workspace_bytes, pts_stream_t stream) {
  if (!draft_probs) return set_error(PTS_ERR_INVALID, "null draft_probs");
  if (!(top_p > 0.0f && top_p <= 1.0f)) return set_error(PTS_ERR_INVALID, "top_p must be in (0, 1]");
  if (top_p < 1.0f) return set_error(PTS_ERR_UNSUPPORTED, "top_p < 1 is not implemented");
  if (do_sample) return set_error(PTS_ERR_UNSUPPORTED, "do_sample is not implemented");
  AcceptParams p{};
  p.logits = logits;
  p.row_stride = row_stride;
  p.row_indptr = row_indptr;
  p.parents = parents;
  p.tokens = tokens;
  p.draft_probs = draft_probs;
  p.batch = batch;
  p.num_rows = num_rows;
  p.vocab = vocab;
  p.max_nodes = max_nodes;
  p.out_stride = out_stride;
  p.eos = eos_token_id;
  p.seed = philox_seed;
  p.offset = philox_offset;
  p.out_tokens = out_tokens;
  p.out_hidden = out_hidden;
  p.out_counts = out_counts;
  return accept_launch(p, 1, temperature, workspace, workspace_bytes, (cudaStream_t)stream);
}
