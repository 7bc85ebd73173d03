// Fused tree acceptance over bf16 logits (greedy and traversal verification).
//
// One launch does everything:
//   1. every CTA streams one 8192-element tile of one logits row (128-bit
//      loads, read once) and reduces it to (max, first argmax, largest value
//      below the max, fp32-partial sum of exp(x - tile max));
//   2. the last tile CTA of a row (atomic counter) merges the row's tiles:
//      row max m, sum s = sum_t s_t * exp(m_t - m) in double, and the argmax of
//      the bf16-rounded probabilities bf16(exp(x - m) / s), resolving the rare
//      case where a smaller logit rounds to the same probability as the max by
//      rescanning that row;
//   3. the last row CTA of a request walks the request's tree on the device:
//      the greedy walk of verify_tree_exact (verification.py:185-268) or the
//      traversal verification loop of verify_tree_traversal
//      (verification.py:275-524), replaying its fp32-tensor / fp64-scalar
//      arithmetic with explicitly rounded operations (no contraction).
//
// Workspace (caller-owned): tile stats, row stats and two counter arrays that
// are cleared at the start of every call.
#include <float.h>
#include <limits.h>

#include "common.cuh"

namespace pts {
namespace {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;                           // 4 x 16 B per thread
constexpr int kTile = kThreads * kVecPerThread * 8;        // 8192 elements per CTA
constexpr float kEps32 = 1e-8f;
constexpr double kEps = 1e-8;

struct TileStat {
  float m;
  int idx;
  float x2;
  int pad;
  double s;
  double pad2;
};

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
  int batch, num_rows, vocab, tiles, max_nodes, out_stride;
  int64_t eos;
  float inv_temp;
  int use_temp;
  int traversal;
  int vec_ok;
  uint64_t seed, offset;
  int32_t* out_tokens;
  int32_t* out_hidden;
  int32_t* out_counts;
  TileStat* tile_ws;
  RowStat* row_ws;
  unsigned* row_ctr;
  unsigned* req_ctr;
};

struct MaxIdx {
  float m;
  int idx;
  float x2;
};

// Merge two (max, first index of max, largest value below max) summaries;
// idx == INT_MAX marks an empty summary.
__device__ __forceinline__ MaxIdx merge(MaxIdx a, MaxIdx b) {
  if (a.idx == INT_MAX) return b;
  if (b.idx == INT_MAX) return a;
  if (a.m == b.m) return MaxIdx{a.m, min(a.idx, b.idx), fmaxf(a.x2, b.x2)};
  if (a.m > b.m) return MaxIdx{a.m, a.idx, fmaxf(a.x2, b.m)};
  return MaxIdx{b.m, b.idx, fmaxf(b.x2, a.m)};
}

__device__ __forceinline__ float load_scaled(const AcceptParams& p, const uint16_t* row, int i) {
  float x = bf16_bits_to_float(row[i]);
  if (p.use_temp) x = round_to_bf16(__fmul_rn(x, p.inv_temp));
  return x;
}

__device__ __forceinline__ float scale(const AcceptParams& p, float x) {
  return p.use_temp ? round_to_bf16(__fmul_rn(x, p.inv_temp)) : x;
}

// bf16-rounded softmax probability of value x in a row with max m, sum s.
__device__ __forceinline__ float prob_bf16(float x, float m, float s) {
  return round_to_bf16(__fdiv_rn(expf(x - m), s));
}

__device__ __forceinline__ uint4 ld_stream(const uint16_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <typename T>
__device__ __forceinline__ T block_reduce_maxidx(T v, T* sm) {
  // warp level
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    T w;
    w.m = __shfl_xor_sync(0xffffffffu, v.m, o);
    w.idx = __shfl_xor_sync(0xffffffffu, v.idx, o);
    w.x2 = __shfl_xor_sync(0xffffffffu, v.x2, o);
    v = merge(v, w);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kThreads / 32 ? sm[lane] : T{-INFINITY, INT_MAX, -INFINITY};
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      T w;
      w.m = __shfl_xor_sync(0xffffffffu, v.m, o);
      w.idx = __shfl_xor_sync(0xffffffffu, v.idx, o);
      w.x2 = __shfl_xor_sync(0xffffffffu, v.x2, o);
      v = merge(v, w);
    }
    if (lane == 0) sm[0] = v;
  }
  __syncthreads();
  T r = sm[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ double block_reduce_sum(double v, double* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kThreads / 32 ? sm[lane] : 0.0;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sm[0] = v;
  }
  __syncthreads();
  double r = sm[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ int block_reduce_min(int v, int* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kThreads / 32 ? sm[lane] : INT_MAX;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) sm[0] = v;
  }
  __syncthreads();
  int r = sm[0];
  __syncthreads();
  return r;
}

struct WalkSmem {
  int16_t first_child[PTS_MAX_TREE_NODES];
  int16_t next_sib[PTS_MAX_TREE_NODES];
  int16_t parent[PTS_MAX_TREE_NODES];
  int16_t queue[PTS_MAX_TREE_NODES];
  float mb[PTS_MAX_TREE_NODES];
  float ms[PTS_MAX_TREE_NODES];
  float pa[PTS_MAX_TREE_NODES];
  uint8_t valid[PTS_MAX_TREE_NODES];
};

__device__ void write_counts(const AcceptParams& p, int b, int n_out, int total, int acc, int node) {
  int32_t* c = p.out_counts + (int64_t)b * 4;
  c[0] = n_out;
  c[1] = total;
  c[2] = acc;
  c[3] = node;
}

// Greedy walk (verify_tree_exact, verification.py:185-268), thread 0 only.
__device__ void walk_greedy(const AcceptParams& p, int b, int lo, int n, const WalkSmem& w) {
  int32_t* ot = p.out_tokens + (int64_t)b * p.out_stride;
  int32_t* oh = p.out_hidden + (int64_t)b * p.out_stride;
  int cur = 0, total = 0, acc = 0, n_out = 0;
  int bonus = -1, last_tok = -1;
  while (w.first_child[cur] >= 0) {                                   // :232
    total++;
    const int tok = __ldcg(&p.row_ws[lo + cur].argmax);               // :73
    int match = -1;
    for (int c = w.first_child[cur]; c >= 0; c = w.next_sib[c])
      if (p.tokens[lo + c] == tok) {
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
  if (n_out == 0 || p.eos < 0 || (int64_t)last_tok != p.eos) {      // :257
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

// Traversal verification (verify_tree_traversal, verification.py:377-524),
// thread 0 only; w.mb / w.ms / w.pa initialised by the caller.
__device__ void walk_traversal(const AcceptParams& p, int b, int lo, int n, WalkSmem& w) {
  int accepted = 0;
  uint32_t draw = 0;
  const int max_iter = 2 * n + 2;
  for (int it = 0; it < max_iter; ++it) {                             // :377
    int curr = 0;
    for (;;) {
      int fc = -1;
      for (int c = w.first_child[curr]; c >= 0; c = w.next_sib[c])
        if (w.valid[c]) {
          fc = c;
          break;
        }
      if (fc < 0) break;
      curr = fc;
    }
    const int cand = curr;
    if (!w.valid[cand]) break;                                        // :391
    const float p_val = w.pa[cand];                                   // :395
    const float eta = philox_uniform(p.seed, p.offset, (uint32_t)b, draw++);   // :396
    if (eta < p_val) {
      accepted = cand;
      break;
    }
    w.valid[cand] = 0;                                                // :403
    const double old_ms_rej = (double)w.ms[cand];
    w.ms[cand] = 0.0f;
    const int parent = w.parent[cand];
    if (parent < 0) {                                                 // :408
      accepted = 0;
      break;
    }
    bool any_active = false;
    for (int c = w.first_child[parent]; c >= 0; c = w.next_sib[c]) any_active |= (w.valid[c] != 0);
    if (!any_active) continue;                                        // :417
    const float p_old32 = w.pa[parent];                               // :422
    const double p_old = (double)p_old32;
    double ms_denom = __dsub_rn(1.0, old_ms_rej);                     // :424
    if (ms_denom < kEps) ms_denom = kEps;
    float s_tree = 0.0f, sum_mb = 0.0f;                               // :429-433
    for (int c = w.first_child[parent]; c >= 0; c = w.next_sib[c]) {
      const float t = fmaxf(__fsub_rn(__fmul_rn(p_old32, w.mb[c]), w.ms[c]), 0.0f);
      s_tree = __fadd_rn(s_tree, t);
      sum_mb = __fadd_rn(sum_mb, w.mb[c]);
    }
    double S = __dadd_rn((double)s_tree, __dmul_rn(p_old, __dsub_rn(1.0, (double)sum_mb)));
    if (S < kEps) S = kEps;                                           // :435
    const double p_new = __ddiv_rn(S, __dsub_rn(__dadd_rn(S, 1.0), p_old));   // :439
    const float p_new32 = __double2float_rn(p_new);
    w.pa[parent] = p_new32;
    const float ms_denom32 = __double2float_rn(ms_denom);
    const float S32 = __double2float_rn(S);
    for (int c = w.first_child[parent]; c >= 0; c = w.next_sib[c]) { // :443-448
      if (!w.valid[c]) continue;
      const float nms = __fdiv_rn(w.ms[c], ms_denom32);
      const float nmb = __fdiv_rn(fmaxf(__fsub_rn(__fmul_rn(p_old32, w.mb[c]), w.ms[c]), 0.0f), S32);
      w.ms[c] = nms;
      w.mb[c] = nmb;
    }
    const double old_mb_rej = (double)w.mb[cand];                     // :451-452
    w.mb[cand] = __double2float_rn(
        __ddiv_rn(fmax(__dsub_rn(__dmul_rn(p_old, old_mb_rej), old_ms_rej), 0.0), S));
    int head = 0, tail = 0;
    for (int c = w.first_child[parent]; c >= 0; c = w.next_sib[c]) { // :455-458
      if (!w.valid[c]) continue;
      w.pa[c] = fminf(__fmul_rn(p_new32, ratio_of(w.mb[c], w.ms[c])), 1.0f);
      w.queue[tail++] = (int16_t)c;
    }
    while (head < tail) {                                             // :461-477
      const int u = w.queue[head++];
      const float p_u = w.pa[u];
      for (int c = w.first_child[u]; c >= 0; c = w.next_sib[c]) {
        if (!w.valid[c]) continue;
        w.pa[c] = fminf(__fmul_rn(p_u, ratio_of(w.mb[c], w.ms[c])), 1.0f);
        if (tail < n) w.queue[tail++] = (int16_t)c;
      }
    }
  }
  // :480-524 output
  int depth = 0;
  for (int c = accepted; c >= 0; c = w.parent[c]) w.queue[depth++] = (int16_t)c;   // reversed path
  int32_t* ot = p.out_tokens + (int64_t)b * p.out_stride;
  int32_t* oh = p.out_hidden + (int64_t)b * p.out_stride;
  int n_out = 0;
  int last_tok = -1;
  for (int i = depth - 2; i >= 0; --i) {
    const int node = w.queue[i];
    const int tok = p.tokens[lo + node];
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

__global__ void __launch_bounds__(kThreads) accept_kernel(const AcceptParams p) {
  __shared__ MaxIdx s_mi[kThreads / 32];
  __shared__ double s_d[kThreads / 32];
  __shared__ int s_i[kThreads / 32];
  __shared__ int s_flag;
  __shared__ WalkSmem w;

  const int tile = blockIdx.x, row = blockIdx.y, tid = threadIdx.x;
  const uint16_t* rp = p.logits + (int64_t)row * p.row_stride;
  const int base = tile * kTile;

  // ---- 1. tile statistics -------------------------------------------------
  uint32_t raw[kVecPerThread * 4];
#pragma unroll
  for (int k = 0; k < kVecPerThread; ++k) {
    const int e0 = base + (k * kThreads + tid) * 8;
    if (p.vec_ok && e0 + 8 <= p.vocab) {
      uint4 v = ld_stream(rp + e0);
      raw[4 * k + 0] = v.x;
      raw[4 * k + 1] = v.y;
      raw[4 * k + 2] = v.z;
      raw[4 * k + 3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int e = e0 + 2 * j;
        uint32_t lo16 = e < p.vocab ? rp[e] : 0xff80u;           // -inf padding
        uint32_t hi16 = e + 1 < p.vocab ? rp[e + 1] : 0xff80u;
        raw[4 * k + j] = lo16 | (hi16 << 16);
      }
    }
  }
  MaxIdx mi{-INFINITY, INT_MAX, -INFINITY};
#pragma unroll
  for (int k = 0; k < kVecPerThread; ++k) {
    const int e0 = base + (k * kThreads + tid) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + j;
      if (e >= p.vocab) continue;
      const uint32_t h = (raw[4 * k + (j >> 1)] >> ((j & 1) * 16)) & 0xffffu;
      const float x = scale(p, bf16_bits_to_float(h));
      if (x > mi.m || mi.idx == INT_MAX) {
        if (mi.idx != INT_MAX) mi.x2 = fmaxf(mi.x2, mi.m);
        mi.m = x;
        mi.idx = e;
      } else if (x < mi.m && x > mi.x2) {
        mi.x2 = x;
      }
    }
  }
  const MaxIdx tmi = block_reduce_maxidx(mi, s_mi);
  float part = 0.0f;
#pragma unroll
  for (int k = 0; k < kVecPerThread; ++k) {
    const int e0 = base + (k * kThreads + tid) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + j;
      if (e >= p.vocab) continue;
      const uint32_t h = (raw[4 * k + (j >> 1)] >> ((j & 1) * 16)) & 0xffffu;
      part = __fadd_rn(part, expf(scale(p, bf16_bits_to_float(h)) - tmi.m));
    }
  }
  const double tsum = block_reduce_sum((double)part, s_d);
  if (tid == 0) {
    TileStat ts;
    ts.m = tmi.m;
    ts.idx = tmi.idx;
    ts.x2 = tmi.x2;
    ts.pad = 0;
    ts.s = tsum;
    ts.pad2 = 0.0;
    p.tile_ws[(int64_t)row * p.tiles + tile] = ts;
    __threadfence();
    const unsigned prev = atomicAdd(&p.row_ctr[row], 1u);
    s_flag = (prev == (unsigned)(p.tiles - 1));
  }
  __syncthreads();
  if (!s_flag) return;

  // ---- 2. row statistics (last tile CTA of the row) ------------------------
  __threadfence();
  __shared__ float s_m, s_s, s_qmax;
  __shared__ int s_arg, s_tie;
  if (tid == 0) {
    const TileStat* ts = p.tile_ws + (int64_t)row * p.tiles;
    MaxIdx r{-INFINITY, INT_MAX, -INFINITY};
    for (int t = 0; t < p.tiles; ++t) {
      MaxIdx o{__ldcg(&ts[t].m), __ldcg(&ts[t].idx), __ldcg(&ts[t].x2)};
      r = merge(r, o);
    }
    double s = 0.0;
    for (int t = 0; t < p.tiles; ++t) {
      const float mt = __ldcg(&ts[t].m);
      const double st = __ldcg(&ts[t].s);
      if (st > 0.0) s += st * (double)expf(mt - r.m);
    }
    const float sf = (float)s;
    const float qmax = round_to_bf16(__fdiv_rn(1.0f, sf));
    s_m = r.m;
    s_s = sf;
    s_qmax = qmax;
    s_arg = r.idx;
    s_tie = (r.x2 > -INFINITY) && (prob_bf16(r.x2, r.m, sf) == qmax);
    p.row_ctr[row] = 0u;
  }
  __syncthreads();
  if (s_tie) {
    // A value below the max rounds to the max probability: first index among
    // all values whose rounded probability equals the maximum.
    int best = INT_MAX;
    for (int e = tid; e < p.vocab; e += kThreads) {
      const float x = load_scaled(p, rp, e);
      if (prob_bf16(x, s_m, s_s) == s_qmax) {
        best = e;
        break;
      }
    }
    best = block_reduce_min(best, s_i);
    if (tid == 0) s_arg = best;
  }
  __syncthreads();
  // request of this row
  __shared__ int s_b, s_lo, s_n, s_last;
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
    __threadfence();
    const unsigned prev = atomicAdd(&p.req_ctr[lo], 1u);
    s_last = (prev == (unsigned)(s_n - 1));
  }
  __syncthreads();
  if (!s_last) return;

  // ---- 3. tree walk (last row CTA of the request) --------------------------
  __threadfence();
  const int b = s_b, lo = s_lo, n = s_n;
  if (n > p.max_nodes || n > PTS_MAX_TREE_NODES) {
    if (tid == 0) write_counts(p, b, -1, 0, 0, 0);
    return;
  }
  int bad = 0;
  for (int i = tid; i < n; i += kThreads) {
    const int par = p.parents[lo + i];
    if ((i == 0 && par != -1) || (i > 0 && (par < 0 || par >= i))) bad = 1;
    w.parent[i] = (int16_t)par;
    w.valid[i] = 1;
    if (p.traversal) {
      if (i == 0) {
        w.mb[0] = 1.0f;
        w.ms[0] = 1.0f;
      } else if (par >= 0 && par < i) {
        const RowStat* rs = p.row_ws + lo + par;
        const float pm = __ldcg(&rs->m), ps = __ldcg(&rs->s);
        const int tok = p.tokens[lo + i];
        const float x = (tok >= 0 && tok < p.vocab) ? load_scaled(p, p.logits + (int64_t)(lo + par) * p.row_stride, tok)
                                                    : -INFINITY;
        w.mb[i] = prob_bf16(x, pm, ps);                                // :349
        w.ms[i] = p.draft_probs[lo + i];                               // :353
      }
    }
  }
  bad = block_reduce_min(bad ? 0 : 1, s_i) == 0;
  if (bad) {
    if (tid == 0) {
      write_counts(p, b, -1, 0, 0, 0);
      p.req_ctr[b] = 0u;
    }
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
    if (p.traversal) {
      w.pa[0] = 1.0f;                                                  // :355-371
      for (int i = 1; i < n; ++i)
        w.pa[i] = fminf(__fmul_rn(w.pa[w.parent[i]], ratio_of(w.mb[i], w.ms[i])), 1.0f);
      walk_traversal(p, b, lo, n, w);
    } else {
      walk_greedy(p, b, lo, n, w);
    }
    p.req_ctr[b] = 0u;
  }
}

size_t ws_layout(int num_rows, int vocab, size_t* off_tiles, size_t* off_rows, size_t* off_rctr,
                 size_t* off_qctr) {
  const int tiles = (vocab + kTile - 1) / kTile;
  size_t o = 0;
  *off_tiles = o;
  o = align_up(o + (size_t)num_rows * tiles * sizeof(TileStat), 256);
  *off_rows = o;
  o = align_up(o + (size_t)num_rows * sizeof(RowStat), 256);
  *off_rctr = o;
  o = align_up(o + (size_t)num_rows * sizeof(unsigned), 256);
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
  PTS_CHECK_ARG(p.out_stride >= 1, "out_stride must be positive");
  PTS_CHECK_ARG((int64_t)p.num_rows * p.row_stride < ((int64_t)1 << 40), "logits too large");
  PTS_CHECK_ARG(temperature > 0.0f, "temperature must be positive");
  size_t ot, orw, orc, oqc;
  const size_t need = ws_layout(p.num_rows, p.vocab, &ot, &orw, &orc, &oqc);
  if (!workspace || ws_bytes < need)
    return set_error(PTS_ERR_CAPACITY, "workspace of %zu bytes, need %zu", ws_bytes, need);
  PTS_CHECK_ARG(((uintptr_t)workspace & 255) == 0, "workspace must be 256-byte aligned");
  char* ws = (char*)workspace;
  p.tiles = (p.vocab + kTile - 1) / kTile;
  p.tile_ws = (TileStat*)(ws + ot);
  p.row_ws = (RowStat*)(ws + orw);
  p.row_ctr = (unsigned*)(ws + orc);
  p.req_ctr = (unsigned*)(ws + oqc);
  p.traversal = traversal;
  p.use_temp = (temperature != 1.0f);
  p.inv_temp = 1.0f / temperature;
  p.vec_ok = (((uintptr_t)p.logits & 15) == 0) && (p.row_stride % 8 == 0);
  PTS_CUDA_TRY(cudaMemsetAsync(ws + orc, 0, need - orc, stream));
  dim3 grid(p.tiles, p.num_rows);
  if (p.num_rows > 65535) return set_error(PTS_ERR_CAPACITY, "num_rows %d above 65535", p.num_rows);
  accept_kernel<<<grid, kThreads, 0, stream>>>(p);
  return launch_status("accept_kernel");
}

}  // namespace
}  // namespace pts

using namespace pts;

extern "C" size_t pts_accept_workspace_size(int num_rows, int vocab) {
  size_t a, b, c, d;
  if (num_rows <= 0 || vocab <= 0) return 0;
  return ws_layout(num_rows, vocab, &a, &b, &c, &d);
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
