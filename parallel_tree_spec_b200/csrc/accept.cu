// Fused tree acceptance over bf16 logits (greedy and traversal verification).
//
// One launch does everything.  Each logits row is split into C = ceil(V/16384)
// chunks, one CTA each (256 threads x 64 elements, the chunk held in
// registers after one 128-bit streaming load per vector; four CTAs per SM so
// the loads of one CTA overlap the reductions of others):
//   1. every thread reduces its 64 values to (max m_t, sum_t exp(x - m_t),
//      first index of m_t) in one pass (packed bf16x2 max, ex2.approx);
//   2. warp and CTA merges combine the partials: m = max, s = sum of
//      s_t * exp(m_t - m) (CUDA expf factors, double accumulation),
//      argmax = first index of m; the CTA's partial goes to the workspace and
//      the last chunk of the row to finish (acquire/release counter) merges
//      the row's partials in chunk order;
//   3. that CTA takes the argmax of the bf16-rounded probabilities
//      bf16(exp(x - m) / s): the first index of m, unless a value just below m
//      can round to the same probability (only possible for small m), in
//      which case the row is rescanned with the exact rounding rule;
//   4. the last row of a request to finish walks the tree on the device: the
//      greedy walk of verify_tree_exact (verification.py:185-268) or the
//      traversal loop of verify_tree_traversal (verification.py:275-524).
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
// Workspace (caller-owned): chunk partials, row stats, and per-row and
// per-request counters that are cleared at the start of every call.
#include <cuda.h>
#include <float.h>
#include <limits.h>

#include <mutex>

#include "common.cuh"

namespace pts {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kVecPerThread = 8;                           // 8 x 16 B per thread
constexpr int kChunk = kThreads * kVecPerThread * 8;       // 16384 elements per CTA
constexpr int kMaxChunks = 64;                             // vocabularies up to 1,048,576
constexpr float kEps32 = 1e-8f;
constexpr double kEps = 1e-8;
constexpr float kLog2e = 1.4426950408889634f;

// Pools with at most this many (layer, K/V, head) rows per token are
// compacted by the walks themselves; larger ones by the compaction kernel.
constexpr int kFusedCompactMaxRows = 32;

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
  int batch, num_rows, vocab, max_nodes, out_stride;
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
  struct Part* part_ws;
  unsigned* row_ctr;
  unsigned* req_ctr;
  unsigned* walk_ctr;      // [1]: requests claimed by the persistent kernel's walkers
  unsigned* row_done;      // per row: 1 once its statistics are in row_ws (release/acquire)
  // vocabulary-sharded (tensor-parallel) acceptance
  struct Part* parts_out;  // shard partials mode: per row the merged (sum, max, first index), no walks
  float* tok_logit_out;    // shard partials mode: per node its token's (scaled) logit if this shard holds it
  int vocab_offset;        // first vocabulary column of this shard
  const float* tok_logit;  // merged mode: per node its token's scaled logit (instead of reading logits)
  int stats_ready;         // merged mode: row_ws is complete, no waiting
  // top-p (nucleus) target distribution
  int no_walk;             // row statistics only (the walks run in a later launch)
  const float* topp_thresh;  // per row: smallest (scaled) logit value inside the nucleus
  const float* topp_mass;    // per row: sum of exp(x - m) over the nucleus
  const float* logits_f32;   // fp32 logits (instead of bf16): probabilities stay fp32
  // KV compaction of the accepted paths by the walks (pts_accept_*_compact)
  int compact;
  pts_kv_compact_args cp;
  // stream order export (top-p): position -> row, and the rows' flags of the
  // next pass cleared
  int32_t* order_out;
  unsigned* order_done;
  // greedy path chain (greedy_chain_kernel): the walk posts each row it needs
  // to its request's slot in req_ctr ((sequence << 16) | node); no other row
  // is reduced.  step_form: set by the compacting entry points (a
  // verification step, whose row statistics only feed its walks), which lets
  // accept_launch choose the chain for greedy batches
  int chain;
  int step_form;
  // top-p without a sampled bonus: the nucleus of a leaf row is never read
  // (a node's target probability comes from its parent's row, the bonus is
  // the row's argmax), so the statistics pass marks leaf rows' nucleus flags
  // done and the nucleus pass skips them
  int topp_skip_leaves;
};

constexpr long long kRowWaitLimit = 4000000000ll;   // clock cycles, about 2 s

// Publishes row `row`'s statistics (already stored by this thread in row_ws).
__device__ __forceinline__ void publish_row(const AcceptParams& p, int row) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p.row_done + row), "r"(1u) : "memory");
}

__device__ __forceinline__ bool row_published(const AcceptParams& p, int row) {
  if (p.stats_ready) return true;
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.row_done + row) : "memory");
  return v != 0;
}

// Bounded wait, by a whole warp, until every lane's row (row < 0: none) is
// published; false (in every lane) on timeout.  The loop condition is
// warp-uniform, so the warp leaves it converged.
__device__ __forceinline__ bool wait_rows_warp(const AcceptParams& p, int row) {
  bool ready = row < 0 || row_published(p, row);
  if (__all_sync(0xffffffffu, ready)) return true;
  const long long t0 = clock64();
  for (;;) {
    __nanosleep(128);
    if (!ready) ready = row_published(p, row);
    if (__all_sync(0xffffffffu, ready)) return true;
    if (__any_sync(0xffffffffu, clock64() - t0 > kRowWaitLimit)) return false;
  }
}

// Bounded wait until row `row`'s statistics are published; false on timeout.
__device__ __forceinline__ bool wait_row(const AcceptParams& p, int row) {
  if (p.stats_ready) return true;
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.row_done + row) : "memory");
  if (v) return true;
  const long long t0 = clock64();
  for (;;) {
    __nanosleep(128);
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.row_done + row) : "memory");
    if (v) return true;
    if (clock64() - t0 > kRowWaitLimit) return false;
  }
}

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

// Index of a partial whose max was not located (its warp skipped values below
// a larger one found elsewhere): it never wins a tie of the final max.
constexpr int kNotCandidate = INT_MAX - 1;

// (max, sum of exp(x - max), first index of max) partials.
struct __align__(16) Part {
  double s;
  float m;
  int idx;
};

__device__ __forceinline__ Part merge(const Part& a, const Part& b) {
  if (b.idx == INT_MAX) return a;
  if (a.idx == INT_MAX) return b;
  Part r;
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

// Walk state in dynamic shared memory, sized for the call's largest tree
// (capacity `cap` nodes), so streaming CTAs of small trees stay light.
//
// Children are numbered in CSR order: the children of every node occupy
// consecutive "slots" in ascending node order (the order Tree.add_nodes
// appends them, tree.py:108-119); the root takes slot n-1.  A node's Mb, Ms
// and valid flag live at its slot, so a sibling group is one contiguous run
// of slots, read in one round of loads.  The node record holds what a descent
// step reads (first 16 bytes) and the node's slot, its sibling run and its
// child run (second 16 bytes).
struct __align__(16) NodeRec {
  int16_t first_valid;     // first child still valid (-1: none)
  int16_t sticky_t;        // time p_alpha was last set directly (-1: never)
  int16_t reset_t;         // time the node's subtree was last recomputed (-1: never)
  int16_t parent;
  float stored_pa;         // p_alpha set directly at time sticky_t
  float ratio;             // Mb / Ms (0 when Ms <= eps), kept current with Mb and Ms
  int16_t slot;            // this node's slot
  int16_t sib_start;       // slots of its parent's children (the root: its own slot)
  int16_t sib_cnt;
  int16_t child_start;     // slots of its children
  int16_t child_cnt;
  int16_t pad[3];
};
static_assert(sizeof(NodeRec) == 32, "node record is two 16-byte words");

struct WalkSmem {
  NodeRec* rec;            // by node
  int32_t* token;          // by node
  float2* val;             // by slot: (Mb, Ms); during set-up: child counts and slot bases
  int16_t* sid;            // by slot: node
  uint8_t* valid;          // by slot
  int16_t* path;           // the descent path (nodes); during set-up: nothing
  int16_t* path_rmax;
  float* path_pa;          // during set-up: the nodes' Ms
  float* uni;              // 2 * cap + 2 uniforms
  float* xtok;             // by node (lazy walks): its token's scaled logit under its parent's row
  uint8_t* expanded;       // by node (lazy walks): its children's Mb are in place
};

__host__ __device__ inline size_t walk_smem_bytes(int cap) {
  cap = (cap + 15) & ~15;
  return (size_t)cap * (32 + 4 + 8 + 2 + 1 + 2 + 2 + 4 + 4 + 1) + (size_t)(2 * cap + 2) * 4 + 192;
}

__device__ inline WalkSmem walk_smem(uint8_t* base, int cap) {
  cap = (cap + 15) & ~15;
  WalkSmem w;
  uint8_t* q = base;
  auto take = [&](size_t bytes) {
    uint8_t* r = q;
    q += (bytes + 15) & ~(size_t)15;
    return r;
  };
  w.rec = (NodeRec*)take((size_t)cap * 32);
  w.val = (float2*)take((size_t)cap * 8);
  w.token = (int32_t*)take((size_t)cap * 4);
  w.path_pa = (float*)take((size_t)cap * 4);
  w.uni = (float*)take((size_t)(2 * cap + 2) * 4);
  w.sid = (int16_t*)take((size_t)cap * 2);
  w.path = (int16_t*)take((size_t)cap * 2);
  w.path_rmax = (int16_t*)take((size_t)cap * 2);
  w.valid = (uint8_t*)take((size_t)cap);
  w.xtok = (float*)take((size_t)cap * 4);
  w.expanded = (uint8_t*)take((size_t)cap);
  return w;
}

__device__ void write_counts(const AcceptParams& p, int b, int n_out, int total, int acc, int node) {
  int32_t* c = p.out_counts + (int64_t)b * 4;
  c[0] = n_out;
  c[1] = total;
  c[2] = acc;
  c[3] = node;
}

// KV compaction of request b's accepted path by one warp, right after its
// walk stored the hidden indices and counts (pts_kv_compact's semantics:
// slot offsets[b] + hidden[i] -> offsets[b] + i for every layer, K and V, and
// head, i < count).  With a shared-memory `stage` that holds the whole path,
// every source piece is copied in with cp.async before any destination is
// written (two HBM round trips for the path).  Otherwise entries go in order
// of i, each one's rows spread over the lanes: a path's hidden indices rise
// (hidden[i] >= i; the bonus entry repeats the last node), so a slot is
// written only after every entry that reads it -- the staged result again.
__device__ void compact_request_warp(const AcceptParams& p, int b, uint8_t* stage = nullptr,
                                     size_t stage_bytes = 0) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  const pts_kv_compact_args& a = p.cp;
  const int na = min(max(p.out_counts[(int64_t)b * 4], 0), p.out_stride);
  const int32_t* acc = p.out_hidden + (int64_t)b * p.out_stride;
  const int off = a.offsets[b];
  const int p0 = a.page_indptr[b], np = a.page_indptr[b + 1] - p0;
  const int head_bytes = a.head_dim * a.elem_bytes, vec = head_bytes / 16;
  const int64_t row_bytes = (int64_t)a.num_kv_heads * head_bytes;
  const int64_t layer_bytes = (int64_t)a.max_pages * 2 * a.page_len * row_bytes;
  const int per_kv = a.num_kv_heads * vec;                // 16-byte pieces of one slot's K (or V) row
  const int items = a.num_layers * 2 * per_kv;
  // the path's slots lie in pages off / page_len onward: lane l holds the l-th
  // of them and the l-th hidden index, so an entry needs no dependent lookups
  // (paths longer than 32 entries or windows wider than 32 pages look up)
  const int pg0 = off >= 0 ? off / a.page_len : 0;
  int my_page = -1;
  if (pg0 + lane < np) {
    const int pg = a.page_indices[p0 + pg0 + lane];
    my_page = (pg >= 0 && pg < a.max_pages) ? pg : -1;
  }
  const int my_src = lane < na ? acc[lane] : 0;
  auto page_of = [&](int slot) -> int {
    const int pi = slot / a.page_len;
    int page = __shfl_sync(0xffffffffu, my_page, (pi - pg0) & 31);
    if (slot < 0 || pi >= np) return -1;
    if (pi < pg0 || pi - pg0 >= 32) {
      page = a.page_indices[p0 + pi];
      page = (page >= 0 && page < a.max_pages) ? page : -1;
    }
    return page;
  };
  if (stage && (size_t)na * items * 16 <= stage_bytes) {
    for (int i = 0; i < na; ++i) {                    // every source piece in flight at once
      const int src = i < 32 ? __shfl_sync(0xffffffffu, my_src, i) : acc[i];
      const int sp = src != i ? page_of(off + src) : -1;
      if (sp >= 0) {
        const int ss = (off + src) % a.page_len;
        for (int e = lane; e < items; e += 32) {
          const int layer = e / (2 * per_kv), kv = (e / per_kv) & 1, q = e % per_kv;
          const char* from = (const char*)a.kv_pool + layer * layer_bytes + (int64_t)q * 16 +
                             ((int64_t)(sp * 2 + kv) * a.page_len + ss) * row_bytes;
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                       ::"r"((uint32_t)__cvta_generic_to_shared(stage + ((size_t)i * items + e) * 16)), "l"(from)
                       : "memory");
        }
      }
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    for (int i = 0; i < na; ++i) {
      const int src = i < 32 ? __shfl_sync(0xffffffffu, my_src, i) : acc[i];
      const int sp = src != i ? page_of(off + src) : -1, dp = src != i ? page_of(off + i) : -1;
      if (sp >= 0 && dp >= 0) {
        const int ds = (off + i) % a.page_len;
        for (int e = lane; e < items; e += 32) {
          const int layer = e / (2 * per_kv), kv = (e / per_kv) & 1, q = e % per_kv;
          char* to = (char*)a.kv_pool + layer * layer_bytes + (int64_t)q * 16 +
                     ((int64_t)(dp * 2 + kv) * a.page_len + ds) * row_bytes;
          *(uint4*)to = *(const uint4*)(stage + ((size_t)i * items + e) * 16);
        }
      }
    }
    __syncwarp();
  } else {
  for (int i = 0; i < na; ++i) {
    const int src = i < 32 ? __shfl_sync(0xffffffffu, my_src, i) : acc[i];
    if (src != i) {
      const int sp = page_of(off + src), dp = page_of(off + i);
      if (sp >= 0 && dp >= 0) {
        const int ss = (off + src) % a.page_len, ds = (off + i) % a.page_len;
        for (int e = lane; e < items; e += 32) {
          const int layer = e / (2 * per_kv), kv = (e / per_kv) & 1, q = e % per_kv;
          char* base = (char*)a.kv_pool + layer * layer_bytes + (int64_t)q * 16;
          const uint4 x = *(const uint4*)(base + ((int64_t)(sp * 2 + kv) * a.page_len + ss) * row_bytes);
          *(uint4*)(base + ((int64_t)(dp * 2 + kv) * a.page_len + ds) * row_bytes) = x;
        }
      }
    }
    __syncwarp();
  }
  }
  if (lane == 0) {
    const int len = off + na;
    if (a.new_kv_len) a.new_kv_len[b] = len;
    if (a.new_last_page_len) a.new_last_page_len[b] = len == 0 ? 0 : (len - 1) % a.page_len + 1;
  }
  __syncwarp();
}

// Correctly rounded a / b for a >= 0 and b > 0 normal, without sending a zero
// dividend into the division: zero operands leave the division's fast path,
// and one lane on the slow path holds up the whole warp.
__device__ __forceinline__ float div_nn(float a, float b) {
  const float q = __fdiv_rn(a == 0.0f ? 1.0f : a, b);
  return a == 0.0f ? 0.0f : q;
}
__device__ __forceinline__ double ddiv_nn(double a, double b) {
  const double q = __ddiv_rn(a == 0.0 ? 1.0 : a, b);
  return a == 0.0 ? 0.0 : q;
}

__device__ __forceinline__ float ratio_of(float mb, float ms) {
  return ms > kEps32 ? div_nn(mb, ms) : 0.0f;
}

// First child of `node` whose token is `tok` (-1: none), by one warp.
__device__ __forceinline__ int match_child(const WalkSmem& w, const NodeRec& r, int tok) {
  const int lane = threadIdx.x & 31;
  for (int base = 0; base < r.child_cnt; base += 32) {
    const int k = base + lane;
    const int c = k < r.child_cnt ? w.sid[r.child_start + k] : -1;
    const unsigned m = __ballot_sync(0xffffffffu, c >= 0 && w.token[c] == tok);
    if (m) return __shfl_sync(0xffffffffu, c, __ffs(m) - 1);
  }
  return -1;
}

// Path chain: request b's next row is node `node` of its tree (sequence
// number seq, counting from 1); 0xffff as the sequence ends the request.
// Posts only raise the slot (atomic max), so a late post of a step that was
// already posted changes nothing.
constexpr unsigned kChainDone = 0xffffu;
__device__ __forceinline__ void chain_post_lane(const AcceptParams& p, int b, unsigned seq, int node) {
  asm volatile("red.release.gpu.global.max.u32 [%0], %1;" ::"l"(p.req_ctr + b), "r"((seq << 16) | (unsigned)node)
               : "memory");
}
__device__ __forceinline__ void chain_post(const AcceptParams& p, int b, unsigned seq, int node) {
  if ((threadIdx.x & 31) == 0) chain_post_lane(p, b, seq, node);
  __syncwarp();
}

// Greedy walk (verify_tree_exact, verification.py:185-268), by one warp.
__device__ void walk_greedy_warp(const AcceptParams& p, int b, int lo, const WalkSmem& w) {
  const int lane = threadIdx.x & 31;
  int32_t* ot = p.out_tokens + (int64_t)b * p.out_stride;
  int32_t* oh = p.out_hidden + (int64_t)b * p.out_stride;
  int cur = 0, total = 0, acc = 0, n_out = 0;
  int bonus = -1, last_tok = -1;
  unsigned seq = 1;                                                   // path chain: requests posted so far
  NodeRec r = w.rec[0];
  while (r.child_cnt > 0) {                                           // :232
    total++;
    if (p.chain) chain_post(p, b, seq++, cur);
    if (!wait_rows_warp(p, lo + cur)) {
      if (lane == 0) write_counts(p, b, -3, 0, 0, 0);
      return;
    }
    const int tok = __ldcg(&p.row_ws[lo + cur].argmax);               // :73
    const int match = match_child(w, r, tok);
    if (match >= 0) {                                                 // :237
      bonus = -1;
      acc++;
      if (lane == 0 && n_out < p.out_stride) {
        ot[n_out] = tok;
        oh[n_out] = cur;
      }
      n_out++;
      last_tok = tok;
      if (p.eos >= 0 && (int64_t)tok == p.eos) break;                 // :242
      cur = match;                                                    // :245
      r = w.rec[cur];
      if (r.child_cnt == 0) break;                                    // :249
    } else {
      bonus = tok;
      break;
    }
  }
  if (n_out == 0 || p.eos < 0 || (int64_t)last_tok != p.eos) {        // :257
    if (bonus < 0) {
      if (p.chain) chain_post(p, b, seq++, cur);
      if (!wait_rows_warp(p, lo + cur)) {
        if (lane == 0) write_counts(p, b, -3, 0, 0, 0);
        return;
      }
      bonus = __ldcg(&p.row_ws[lo + cur].argmax);                     // :260-262
    }
    if (lane == 0 && n_out < p.out_stride) {
      ot[n_out] = bonus;
      oh[n_out] = cur;
    }
    n_out++;
  }
  if (lane == 0) write_counts(p, b, n_out > p.out_stride ? -2 : n_out, total, acc, cur);
}

// Output of a traversal walk (verification.py:480-524), by one thread.
__device__ void traversal_output(const AcceptParams& p, int b, int lo, int accepted, const WalkSmem& w) {
  int d = 0;
  for (int c = accepted; c >= 0; c = w.rec[c].parent) w.path[d++] = (int16_t)c;   // reversed path
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
    if (!wait_row(p, lo + accepted)) {                                // a leaf row may still stream
      write_counts(p, b, -3, 0, 0, 0);
      return;
    }
    const int bonus = __ldcg(&p.row_ws[lo + accepted].argmax);        // :511
    if (n_out < p.out_stride) {
      ot[n_out] = bonus;
      oh[n_out] = accepted;
    }
    n_out++;
  }
  write_counts(p, b, n_out > p.out_stride ? -2 : n_out, n_out, n_out > 0 ? n_out - 1 : 0, accepted);
}

// ---- lazy walks (persistent kernel) ------------------------------------------
// The walker warp starts a traversal walk as soon as the request's tree is
// loaded; an expander warp of the same CTA fills in each internal node's
// children's Mb when the node's row is published, and the walker waits (in
// shared memory) only when it descends through a node not yet expanded.  The
// stream order hands every request its internal rows in walk order, so the
// walk overlaps the streaming instead of following it.

// Target probability of a node's token (scaled logit x) under its parent's
// row (m, s): the softmax entry (verification.py:349), renormalised over the
// nucleus under top-p, fp32 for fp32 logits.
__device__ __forceinline__ float node_mb(const AcceptParams& p, float x, int prow, float m, float s) {
  if (p.logits_f32) return __fdiv_rn(expf(x - m), s);
  if (p.topp_mass) return x >= p.topp_thresh[prow] ? prob_bf16(x, m, p.topp_mass[prow]) : 0.0f;
  return prob_bf16(x, m, s);
}

// One thread: node v's children's Mb and Mb/Ms from v's published row.
__device__ void expand_node(const AcceptParams& p, int lo, const WalkSmem& w, int v) {
  const float m = __ldcg(&p.row_ws[lo + v].m), s = __ldcg(&p.row_ws[lo + v].s);
  const NodeRec rv = w.rec[v];
  for (int k = 0; k < rv.child_cnt; ++k) {
    const int sl = rv.child_start + k;
    const int c = w.sid[sl];
    const float mb = node_mb(p, w.xtok[c], lo + v, m, s);
    w.val[sl].x = mb;
    w.rec[c].ratio = ratio_of(mb, w.val[sl].y);
  }
}

// Walker (whole warp, one node): bounded wait until node u is expanded; the
// fence after the flag orders the expander's stores before the walker's loads.
__device__ __forceinline__ bool wait_expanded(const WalkSmem& w, int u) {
  const volatile uint8_t* f = w.expanded + u;
  if (*f) {
    __threadfence_block();
    return true;
  }
  const long long t0 = clock64();
  for (;;) {
    __nanosleep(32);
    if (__all_sync(0xffffffffu, *f != 0)) {
      __threadfence_block();
      return true;
    }
    if (__any_sync(0xffffffffu, clock64() - t0 > kRowWaitLimit)) return false;
  }
}

// Expander (whole warp): expands request b's internal nodes as their rows are
// published.  Lane l owns nodes l, l + 32, ...; each pass polls the owned
// pending nodes' publication flags with independent relaxed loads (the fence
// after a set flag makes the row's statistics visible), expands the
// published ones and sets their flags.  Returns when no node is pending, the
// walk has ended (*walk_done) or the wait limit passed.
__device__ void expand_request(const AcceptParams& p, int lo, int n, const WalkSmem& w, const volatile int* walk_done) {
  const int lane = threadIdx.x & 31;
  uint32_t pending = 0;                                    // bit j: node lane + 32 j
  for (int j = 0; lane + 32 * j < n; ++j)
    if (w.rec[lane + 32 * j].child_cnt > 0) pending |= 1u << j;
  const long long t0 = clock64();
  for (;;) {
    uint32_t ready = 0;
    if (p.stats_ready) {
      ready = pending;
    } else {
      for (int j0 = 0; j0 < 32 && (pending >> j0); j0 += 4) {
        unsigned f[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          f[q] = 0;
          if ((pending >> (j0 + q)) & 1u)
            asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];"
                         : "=r"(f[q]) : "l"(p.row_done + lo + lane + 32 * (j0 + q)) : "memory");
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (f[q]) ready |= 1u << (j0 + q);
      }
      if (ready) __threadfence();
    }
    for (uint32_t r = ready; r; r &= r - 1) {
      const int v = lane + 32 * (__ffs(r) - 1);
      expand_node(p, lo, w, v);
      __threadfence_block();
      *(volatile uint8_t*)(w.expanded + v) = 1;
    }
    pending &= ~ready;
    if (!__any_sync(0xffffffffu, pending != 0u)) return;
    if (__any_sync(0xffffffffu, *walk_done != 0 || clock64() - t0 > kRowWaitLimit)) return;
    __nanosleep(64);
  }
}

// Traversal verification (verify_tree_traversal, verification.py:377-524) by
// one warp.  The loop is sequential (each iteration depends on the last), so
// the warp keeps its dependent chain short: every lane computes the same
// control values (lane 0 alone stores the shared ones: stores of one
// sub-word location by all 32 lanes measured up to 8x slower), a descent
// step is one record load and a multiply
// (Mb/Ms is kept current per node), the rejected node's sibling group is one
// run of slots spread over the lanes, its fp32 sums are taken left to right
// from shuffles issued eight at a time, the siblings' fp32 divisions run in
// parallel lanes, and p_new and the rejected node's Mb share one fp64
// division (lanes 0 and 1).  Fp32 tensor and fp64 scalar operations are
// replayed with explicitly rounded operations in the reference's order.  See
// the file comment for the lazily evaluated p_alpha.
template <bool kLazy = false>
__device__ void walk_traversal_warp(const AcceptParams& p, int b, int lo, int n, const WalkSmem& w) {
  const int lane = threadIdx.x & 31;
  constexpr unsigned kFull = 0xffffffffu;
  int accepted = 0;
  int depth = 0;           // w.path[0..depth]: the current descent path
  int draw = 0;
  int T = 1;               // time stamp of the next direct p_alpha assignment
  int u = 0;               // the node the next descent starts from (w.path[depth])
  if (lane == 0) {
    w.path[0] = 0;
    w.path_pa[0] = w.rec[0].stored_pa;
    w.path_rmax[0] = -1;
  }
  const int max_iter = 2 * n + 2;
  for (int it = 0; it < max_iter; ++it) {                             // :377
    __syncwarp();
    const float eta = w.uni[draw++];                                  // :396, drawn once per iteration
    // descend to the first valid leaf (:379-389), p_alpha evaluated lazily
    NodeRec ru = w.rec[u];
    float pa_u = w.path_pa[depth];
    int rmax_u = w.path_rmax[depth];
    bool late = false;
    while (ru.first_valid >= 0) {
      if (kLazy && !wait_expanded(w, u)) {             // u's children's Mb come from u's row
        late = true;
        break;
      }
      const int c = ru.first_valid;
      const NodeRec rc = w.rec[c];
      const int rmax = max(rmax_u, (int)ru.reset_t);
      const float pa = rc.sticky_t > rmax ? rc.stored_pa : fminf(__fmul_rn(pa_u, rc.ratio), 1.0f);
      ++depth;
      if (lane == 0) {
        w.path[depth] = (int16_t)c;
        w.path_pa[depth] = pa;
        w.path_rmax[depth] = (int16_t)rmax;
      }
      u = c;
      ru = rc;
      pa_u = pa;
      rmax_u = rmax;
    }
    if (late) {
      if (lane == 0) write_counts(p, b, -3, 0, 0, 0);
      return;
    }
    const int cand = u;
    if (eta < pa_u) {                                                 // :395-400
      accepted = cand;
      break;
    }
    const int parent = ru.parent;
    if (parent < 0) {                                                 // :408
      accepted = 0;
      break;
    }
    --depth;                                                          // back to the parent
    u = parent;
    const int s0 = ru.sib_start, nc = ru.sib_cnt, cslot = ru.slot;
    __syncwarp();                                                     // lane 0's path entries
    const float p_old32 = w.path_pa[depth];                           // :422
    const float2 cv = w.val[cslot];
    const float old_mb32 = cv.x, old_ms32 = cv.y;
    double q;
    // the parent's children left to right (:429-433): the rejected node counts
    // with Ms = 0 (:404) and is no longer valid; it was the parent's first
    // valid child, so the lowest valid slot after it is the new first one
    if (nc <= 32) {
      const int sl = s0 + lane;
      const bool has = lane < nc;
      const float2 v = has ? w.val[sl] : make_float2(0.0f, 0.0f);
      const int ck = has ? w.sid[sl] : 0;
      const bool vk = has && sl != cslot && w.valid[sl];
      const unsigned vm = __ballot_sync(kFull, vk);
      const int next = vm ? __shfl_sync(kFull, ck, __ffs(vm) - 1) : -1;
      if (lane == 0) {
        w.valid[cslot] = 0;                                           // :403
        w.val[cslot].y = 0.0f;                                        // :404
        w.rec[parent].first_valid = (int16_t)next;
      }
      if (vm == 0u) continue;                                         // :417 no active sibling
      const float mbk = v.x, msk = sl == cslot ? 0.0f : v.y;
      const float tk = has ? fmaxf(__fsub_rn(__fmul_rn(p_old32, mbk), msk), 0.0f) : 0.0f;
      // left-to-right fp32 sums; terms past the group add +0.0, which leaves
      // these non-negative sums unchanged
      float s_tree = 0.0f, sum_mb = 0.0f;
      for (int j0 = 0; j0 < nc; j0 += 8) {
        float a[8], m[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          a[q] = __shfl_sync(kFull, tk, (j0 + q) & 31);
          m[q] = __shfl_sync(kFull, mbk, (j0 + q) & 31);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const bool in = j0 + q < nc;
          s_tree = __fadd_rn(s_tree, in ? a[q] : 0.0f);
          sum_mb = __fadd_rn(sum_mb, in ? m[q] : 0.0f);
        }
      }
      double S = __dadd_rn((double)s_tree, __dmul_rn((double)p_old32, __dsub_rn(1.0, (double)sum_mb)));
      if (S < kEps) S = kEps;                                         // :435
      double ms_denom = __dsub_rn(1.0, (double)old_ms32);             // :424
      if (ms_denom < kEps) ms_denom = kEps;
      const float ms_denom32 = __double2float_rn(ms_denom);
      const float S32 = __double2float_rn(S);
      // lane 1: the rejected node's Mb (:451); every other lane: p_new (:439)
      const double p_old = (double)p_old32;
      const double num = lane == 1 ? fmax(__dsub_rn(__dmul_rn(p_old, (double)old_mb32), (double)old_ms32), 0.0) : S;
      const double den = lane == 1 ? S : __dsub_rn(__dadd_rn(S, 1.0), p_old);
      q = ddiv_nn(num, den);
      // every lane divides (no divergent branch); valid siblings store (:443-448)
      const float ms_new = div_nn(msk, ms_denom32);
      const float mb_new = div_nn(tk, S32);
      const float ratio = div_nn(mb_new, ms_new > kEps32 ? ms_new : 1.0f);
      if (vk) {
        w.val[sl] = make_float2(mb_new, ms_new);
        w.rec[ck].ratio = ms_new > kEps32 ? ratio : 0.0f;
      }
    } else {
      float s_tree = 0.0f, sum_mb = 0.0f;
      int next = -1;
      for (int base = 0; base < nc; base += 32) {
        const int k = base + lane;
        const bool has = k < nc;
        const int sl = s0 + k;
        const float2 v = has ? w.val[sl] : make_float2(0.0f, 0.0f);
        const int ck = has ? w.sid[sl] : 0;
        const bool vk = has && sl != cslot && w.valid[sl];
        const float mbk = v.x, msk = sl == cslot ? 0.0f : v.y;
        const float tk = has ? fmaxf(__fsub_rn(__fmul_rn(p_old32, mbk), msk), 0.0f) : 0.0f;
        const int cnt = min(32, nc - base);
        for (int j = 0; j < cnt; ++j) {
          s_tree = __fadd_rn(s_tree, __shfl_sync(kFull, tk, j));
          sum_mb = __fadd_rn(sum_mb, __shfl_sync(kFull, mbk, j));
        }
        const unsigned vm = __ballot_sync(kFull, vk);
        if (next < 0 && vm) next = __shfl_sync(kFull, ck, __ffs(vm) - 1);
      }
      if (lane == 0) {
        w.valid[cslot] = 0;                                           // :403
        w.val[cslot].y = 0.0f;                                        // :404
        w.rec[parent].first_valid = (int16_t)next;
      }
      if (next < 0) continue;                                         // :417 no active sibling
      double S = __dadd_rn((double)s_tree, __dmul_rn((double)p_old32, __dsub_rn(1.0, (double)sum_mb)));
      if (S < kEps) S = kEps;                                         // :435
      double ms_denom = __dsub_rn(1.0, (double)old_ms32);             // :424
      if (ms_denom < kEps) ms_denom = kEps;
      const float ms_denom32 = __double2float_rn(ms_denom);
      const float S32 = __double2float_rn(S);
      const double p_old = (double)p_old32;
      const double num = lane == 1 ? fmax(__dsub_rn(__dmul_rn(p_old, (double)old_mb32), (double)old_ms32), 0.0) : S;
      const double den = lane == 1 ? S : __dsub_rn(__dadd_rn(S, 1.0), p_old);
      q = ddiv_nn(num, den);
      __syncwarp();
      for (int base = 0; base < nc; base += 32) {
        const int sl = s0 + base + lane;
        if (base + lane >= nc || sl == cslot || !w.valid[sl]) continue;
        const float2 v = w.val[sl];
        const float t = fmaxf(__fsub_rn(__fmul_rn(p_old32, v.x), v.y), 0.0f);
        const float ms_new = div_nn(v.y, ms_denom32);
        const float mb_new = div_nn(t, S32);
        w.val[sl] = make_float2(mb_new, ms_new);
        w.rec[w.sid[sl]].ratio = ratio_of(mb_new, ms_new);
      }
    }
    const float p_new32 = __double2float_rn(__shfl_sync(kFull, q, 0));       // :440, direct assignment
    const float mb_rej32 = __double2float_rn(__shfl_sync(kFull, q, 1));      // :452
    if (lane == 0) {
      w.val[cslot].x = mb_rej32;
      w.rec[parent].stored_pa = p_new32;
      w.rec[parent].sticky_t = (int16_t)T;
      w.rec[parent].reset_t = (int16_t)T;
      w.path_pa[depth] = p_new32;
    }
    ++T;
  }
  __syncwarp();
  if (lane == 0) traversal_output(p, b, lo, accepted, w);
  __syncwarp();
}

// Thread groups that run the set-up of a tree walk: the whole CTA (streaming
// kernel for unaligned rows) or one warp (walker warp of the persistent
// kernel).  The walk itself always runs on the group's first warp.
struct CtaGroup {
  __device__ int rank() const { return threadIdx.x; }
  __device__ int size() const { return kThreads; }
  __device__ void sync() const { __syncthreads(); }
  __device__ bool any(bool v, int* sm) const { return block_reduce_min(v ? 0 : 1, sm) == 0; }
};
struct WarpGroup {
  __device__ int rank() const { return threadIdx.x & 31; }
  __device__ int size() const { return 32; }
  __device__ void sync() const { __syncwarp(); }
  __device__ bool any(bool v, int*) const {
    __syncwarp();
    return __any_sync(0xffffffffu, v);
  }
};

// Load request b's tree (rows lo .. lo+n-1) and the traversal uniforms, build
// the child runs (a stable counting sort of the nodes by parent), then
// (traversal) wait for the parents' rows and compute the target probability
// of every node's token under its parent's row, and walk.  Work that needs no
// row statistics comes first, so it overlaps the streaming.
//
// kLazy (the persistent kernel's traversal walker): the set-up only, with each
// node's token logit read and every expansion flag cleared; returns whether
// the walk is to run (the caller runs it against its expander warp).
template <bool kLazy = false, class G>
__device__ bool walk_request(const AcceptParams& p, int b, int lo, int n, const WalkSmem& w, G g, int* red_sm,
                             uint8_t* stage = nullptr, size_t stage_bytes = 0) {
  if (n <= 0 || n > p.max_nodes || n > PTS_MAX_TREE_NODES) {
    if (g.rank() == 0) write_counts(p, b, -1, 0, 0, 0);
    if (!kLazy && p.compact && g.rank() < 32) compact_request_warp(p, b);   // (the lengths)
    return false;
  }
  int* cnt = reinterpret_cast<int*>(w.val);               // child counts, then slot bases
  int* basep = cnt + ((n + 1) & ~1);
  for (int i = g.rank(); i < n; i += g.size()) cnt[i] = 0;
  g.sync();
  int bad = 0;
  for (int i = g.rank(); i < n; i += g.size()) {
    const int par = p.parents[lo + i];
    const int tok = p.tokens[lo + i];
    const float ms = (p.traversal && i > 0) ? p.draft_probs[lo + i] : 1.0f;   // :353
    if ((i == 0 && par != -1) || (i > 0 && (par < 0 || par >= i))) bad = 1;
    NodeRec r;
    r.first_valid = -1;
    r.sticky_t = i == 0 ? 0 : -1;
    r.reset_t = -1;
    r.parent = (int16_t)par;
    r.stored_pa = 1.0f;
    r.ratio = 0.0f;
    r.slot = r.sib_start = r.sib_cnt = r.child_start = r.child_cnt = 0;
    r.pad[0] = r.pad[1] = r.pad[2] = 0;
    w.rec[i] = r;
    w.token[i] = tok;
    w.path_pa[i] = ms;
    if (i > 0 && par >= 0 && par < i) atomicAdd(&cnt[par], 1);
  }
  if (p.traversal)
    for (int k = g.rank(); k < 2 * n + 2; k += g.size())
      w.uni[k] = philox_uniform(p.seed, p.offset, (uint32_t)b, (uint32_t)k);
  bad = g.any(bad != 0, red_sm);
  g.sync();
  if (bad) {
    if (g.rank() == 0) write_counts(p, b, -1, 0, 0, 0);
    if (!kLazy && p.compact && g.rank() < 32) compact_request_warp(p, b);
    return false;
  }
  if (g.rank() < 32) {
    // child runs: exclusive scan of the counts, then a stable scatter of the
    // nodes in ascending order (ranks within a chunk of 32 from match_any)
    const int lane = g.rank();
    int carry = 0;
    for (int base = 0; base < n; base += 32) {
      const int i = base + lane;
      const int c = i < n ? cnt[i] : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (i < n) {
        basep[i] = carry + incl - c;
        w.rec[i].child_start = (int16_t)(carry + incl - c);
        w.rec[i].child_cnt = (int16_t)c;
      }
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    __syncwarp();
    for (int base = 0; base < n; base += 32) {
      const int i = base + lane;
      const int par = (i >= 1 && i < n) ? (int)w.rec[i].parent : -2 - lane;    // unique key when unused
      const unsigned same = __match_any_sync(0xffffffffu, par);
      const int rank = __popc(same & ((1u << lane) - 1u));
      int slot = n - 1;                                    // the root's slot
      if (i >= 1 && i < n) slot = basep[par] + rank;
      __syncwarp();
      if (i >= 1 && i < n && (same >> lane) == 1u) basep[par] += __popc(same);   // the group's last lane
      if (i < n) {
        w.sid[slot] = (int16_t)i;
        w.rec[i].slot = (int16_t)slot;
      }
      __syncwarp();
    }
  }
  g.sync();
  for (int i = g.rank(); i < n; i += g.size()) {
    const NodeRec r = w.rec[i];
    w.rec[i].first_valid = r.child_cnt > 0 ? w.sid[r.child_start] : (int16_t)-1;
    w.rec[i].sib_start = i == 0 ? r.slot : w.rec[r.parent].child_start;
    w.rec[i].sib_cnt = i == 0 ? (int16_t)1 : w.rec[r.parent].child_cnt;
  }
  g.sync();                                                // every count and base read: the values may go in
  for (int i = g.rank(); i < n; i += g.size()) {
    const int sl = w.rec[i].slot;
    w.val[sl] = make_float2(1.0f, w.path_pa[i]);           // root: Mb = Ms = 1 (:344-345)
    w.valid[sl] = 1;
  }
  g.sync();
  if (kLazy && p.traversal) {
    for (int i = g.rank(); i < n; i += g.size()) {
      float x = -INFINITY;
      const int tk = w.token[i];
      if (i > 0 && tk >= 0 && tk < p.vocab) {
        const int pr = lo + w.rec[i].parent;
        if (p.logits_f32) {
          x = p.logits_f32[(int64_t)pr * p.row_stride + tk];
          if (p.use_temp) x = __fmul_rn(x, p.inv_temp);
        } else {
          x = p.tok_logit ? p.tok_logit[lo + i] : load_scaled(p, p.logits + (int64_t)pr * p.row_stride, tk);
        }
      }
      w.xtok[i] = x;
      w.expanded[i] = 0;
    }
    g.sync();
    return true;
  }
  if (p.traversal) {
    // Mb[i] = p[parent(i), token(i)] (:349) once the parent's row is published
    // (the warps wait with warp-uniform loops and stay converged)
    int late = 0;
    for (int i0 = 1 + (g.rank() & ~31); i0 < n; i0 += g.size()) {
      const int i = i0 + (g.rank() & 31);
      const NodeRec r = w.rec[i < n ? i : 0];
      const int pr = lo + r.parent;
      if (!wait_rows_warp(p, i < n ? pr : -1)) {
        late = 1;
        break;
      }
      if (i >= n) continue;
      const float pm = __ldcg(&p.row_ws[pr].m), ps = __ldcg(&p.row_ws[pr].s);
      const int tk = w.token[i];
      if (p.logits_f32) {                                      // fp32 rows: fp32 probabilities
        float xf = -INFINITY;
        if (tk >= 0 && tk < p.vocab) {
          xf = p.logits_f32[(int64_t)pr * p.row_stride + tk];
          if (p.use_temp) xf = __fmul_rn(xf, p.inv_temp);
        }
        const float mbf = __fdiv_rn(expf(xf - pm), ps);
        w.val[r.slot].x = mbf;
        w.rec[i].ratio = ratio_of(mbf, w.val[r.slot].y);
        continue;
      }
      const float x = (tk < 0 || tk >= p.vocab) ? -INFINITY
                      : p.tok_logit ? p.tok_logit[lo + i]
                                    : load_scaled(p, p.logits + (int64_t)pr * p.row_stride, tk);
      // nucleus rows: tokens below the threshold get 0, the rest renormalise
      const float mb = p.topp_mass ? (x >= p.topp_thresh[pr] ? prob_bf16(x, pm, p.topp_mass[pr]) : 0.0f)
                                   : prob_bf16(x, pm, ps);
      w.val[r.slot].x = mb;
      w.rec[i].ratio = ratio_of(mb, w.val[r.slot].y);
    }
    late = g.any(late != 0, red_sm);
    g.sync();
    if (late) {
      if (g.rank() == 0) write_counts(p, b, -3, 0, 0, 0);
      if (p.compact && g.rank() < 32) compact_request_warp(p, b);
      return false;
    }
    if (g.rank() < 32) walk_traversal_warp(p, b, lo, n, w);
  } else if (g.rank() < 32) {
    walk_greedy_warp(p, b, lo, w);
  }
  if (p.compact && g.rank() < 32) compact_request_warp(p, b, stage, stage_bytes);
  g.sync();
  return false;
}

// Request of `row`: the warp finds the last request whose first row is <= row
// with one parallel sweep over row_indptr (no dependent load chain).
__device__ __forceinline__ int find_request(const int32_t* row_indptr, int batch, int row) {
  const int lane = threadIdx.x & 31;
  int best = 0;
  for (int base = 0; base < batch; base += 32) {
    const int b = base + lane;
    const bool le = b < batch && row_indptr[b] <= row;
    const unsigned m = __ballot_sync(0xffffffffu, le);
    if (m) best = base + 31 - __clz(m);
    if (m != 0xffffffffu) break;
  }
  return best;
}

__global__ void __launch_bounds__(kThreads, 4) accept_kernel(const AcceptParams p) {
  __shared__ Part s_warp[kWarps];
  __shared__ int s_red_i[kWarps];
  __shared__ int s_flag;
  __shared__ float s_m, s_s, s_qmax;
  __shared__ int s_arg, s_tie;
  __shared__ int s_b, s_lo, s_n;
  extern __shared__ __align__(16) uint8_t dyn_smem[];

  const int chunk = blockIdx.x, row = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nchunks = gridDim.x;
  const uint16_t* rp = p.logits + (int64_t)row * p.row_stride;
  const int base = chunk * kChunk;

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
  if (p.use_temp) {
#pragma unroll
    for (int i = 0; i < kVecPerThread * 4; ++i) raw[i] = scale_pair(raw[i], p.inv_temp);
  }
  uint32_t m2 = raw[0];
#pragma unroll
  for (int i = 1; i < kVecPerThread * 4; ++i) m2 = bf16x2_max(m2, raw[i]);
  const float mt = fmaxf(__uint_as_float(m2 << 16), __uint_as_float(m2 & 0xffff0000u));
  const float mlog = mt == -INFINITY ? 0.0f : mt * kLog2e;   // all -inf: every term is 0
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
  Part part{(double)st, mt, first};
  if (first == INT_MAX) part = Part{0.0, -INFINITY, INT_MAX};
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Part other;
    other.s = __shfl_xor_sync(0xffffffffu, part.s, o);
    other.m = __shfl_xor_sync(0xffffffffu, part.m, o);
    other.idx = __shfl_xor_sync(0xffffffffu, part.idx, o);
    part = (lane & o) ? merge(other, part) : merge(part, other);
  }
  if (lane == 0) s_warp[warp] = part;
  __syncthreads();
  if (tid == 0) {
    Part c = s_warp[0];
    for (int i = 1; i < kWarps; ++i) c = merge(c, s_warp[i]);
    p.part_ws[(int64_t)row * nchunks + chunk] = c;
    unsigned prev;    // release: this chunk's partial; acquire: the row's others
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&p.row_ctr[row]) : "memory");
    s_flag = (prev == (unsigned)(nchunks - 1));
  }
  __syncthreads();
  if (!s_flag) return;

  // ---- 2. row statistics (last chunk of the row) ------------------------------
  if (tid == 0) {
    const Part* pp = p.part_ws + (int64_t)row * nchunks;
    Part r{__ldcg(&pp[0].s), __ldcg(&pp[0].m), __ldcg(&pp[0].idx)};
    for (int i = 1; i < nchunks; ++i) r = merge(r, Part{__ldcg(&pp[i].s), __ldcg(&pp[i].m), __ldcg(&pp[i].idx)});
    const float sf = (float)r.s;
    const float qmax = round_to_bf16(__fdiv_rn(1.0f, sf));
    s_m = r.m;
    s_s = sf;
    s_qmax = qmax;
    s_arg = r.idx;
    // a smaller value can only tie with the max after rounding if the
    // largest bf16 value below m already does
    s_tie = (r.m > -INFINITY) && (prob_bf16(prev_bf16(r.m), r.m, sf) == qmax);
    s_warp[0] = r;
  }
  __syncthreads();
  if (p.parts_out) {
    // shard partials mode: the row's partial and node `row`'s token logit
    if (warp == 0) {
      const int b = find_request(p.row_indptr, p.batch, row);
      if (lane == 0) {
        Part r = s_warp[0];
        if (r.idx < kNotCandidate) r.idx += p.vocab_offset;
        p.parts_out[row] = r;
        const int lo = p.row_indptr[b], pj = p.parents[row], tk = p.tokens[row] - p.vocab_offset;
        float xv = -INFINITY;
        if (row > lo && pj >= 0 && pj < row - lo && tk >= 0 && tk < p.vocab)
          xv = load_scaled(p, p.logits + (int64_t)(lo + pj) * p.row_stride, tk);
        p.tok_logit_out[row] = xv;
      }
    }
    return;
  }
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
  if (warp == 0) {
    const int b = find_request(p.row_indptr, p.batch, row);
    if (lane == 0) {
      RowStat rs;
      rs.m = s_m;
      rs.s = s_s;
      rs.argmax = s_arg;
      rs.flags = s_tie;
      p.row_ws[row] = rs;
      publish_row(p, row);
      s_b = b;
      s_lo = p.row_indptr[b];
      s_n = p.row_indptr[b + 1] - s_lo;
      unsigned prev;    // release: this row's stats; acquire: every earlier row's
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&p.req_ctr[b]) : "memory");
      s_flag = (prev == (unsigned)(s_n - 1));
    }
  }
  __syncthreads();
  if (!s_flag || p.no_walk) return;

  // ---- 3. tree walk (last row CTA of the request) ----------------------------
  walk_request(p, s_b, s_lo, s_n, walk_smem(dyn_smem, p.max_nodes), CtaGroup{}, s_red_i);
}

// ---------------------------------------------------------------------------
// Persistent streaming kernel (rows 16-byte aligned, vocabulary a multiple of 8).
//
// One CTA per SM.  The rows are dealt out whole, round-robin (CTA c takes rows
// c, c + G, ...), so a row's chunks are reduced inside one CTA; only the last
// num_rows % G rows are split by chunk over all CTAs and merged through the
// workspace (partials + acquire/release counter), which keeps every CTA's item
// count within one of the others.  Each CTA streams its items -- 32 KB chunks
// of a row -- through a ring of shared-memory slots:
//   warp 0        producer: one cp.async.bulk (1-D, no multicast) per item,
//                 kSSlots items ahead of the consumers;
//   warps 1-16    consumers: 32 values per thread (four 16-byte shared loads,
//                 the slot released right after), thread max by packed bf16x2
//                 max, sum of exp(x - max) with packed f32x2 FMA/add and MUFU
//                 exp2, folded into a running (max, sum) per thread; the warp's
//                 max and its first index are updated only when a chunk raises
//                 it (searched by the threads that hold it), and the warp's
//                 partial of the row is reduced and handed over once per row;
//   warp 17       merger: combines the 16 warp partials of a row (or of a chunk
//                 of a split row), derives the row statistics with the tie
//                 rescan, and counts the request's finished rows;
//   warp 18       walker: claims the next request (a grid-wide counter) and
//                 runs its tree walk (the walks of different requests run on
//                 different SMs while the other warps stream); a traversal
//                 walk starts as soon as the tree is loaded and waits only for
//                 nodes whose rows have not streamed yet;
//   warp 19       expander (traversal): fills in the walked request's
//                 children's target probabilities row by row as the rows are
//                 published (named barriers 1 and 2 pair it with the walker).
constexpr int kSChunk = 16384;                 // elements per item (32 KB)
constexpr int kSSlots = 5;
constexpr int kSConsumerWarps = 16;
constexpr int kSConsumers = kSConsumerWarps * 32;
constexpr int kSThreads = kSConsumers + 128;   // + producer, merger, walker and expander warps
constexpr int kSVec = kSChunk / 8 / kSConsumers;   // 16-byte vectors per consumer thread (4)
constexpr long long kSpinLimit = 4000000000ll;     // clock cycles, about 2 s
constexpr size_t kMaxDynSmem = 232448;             // 227 KB per CTA

struct __align__(16) StreamCtl {
  uint64_t full[kSSlots];
  uint64_t empty[kSSlots];
  uint64_t seg_full[2];       // 16 consumer warps wrote their partials of a segment
  uint64_t seg_empty[2];      // the merger has read them
  unsigned long long seg_max; // (segment + 1) << 32 | key of the largest value any warp located in it
  Part seg[2][kSConsumerWarps];
  int walk_b;                 // the walker's request for the expander (-1: no more, -2: skip)
  int walk_done;              // the walker has finished the request's walk
};

constexpr size_t kSRingBytes = (size_t)kSSlots * kSChunk * 2;
constexpr size_t kSCtlOff = kSRingBytes;
constexpr size_t kSWalkOff = (kSCtlOff + sizeof(StreamCtl) + 127) & ~(size_t)127;

// The work of CTA c.  Rows are taken in "stream order": the internal rows
// (every request's root and every row with children) of all requests first,
// then the leaf rows in row order.  Internal rows go in row order, or (dfs)
// ordered by their rank in the depth-first preorder of their tree, the
// requests interleaved at each rank: the order in which traversal walks
// descend through them, so every walk receives its rows while it runs.
// Position q of the stream order is a whole row of CTA q % G while
// q < split_first_row; the remaining num_rows % G positions are split by
// chunk over all CTAs when they are few or every CTA streams few rows.  A
// traversal walk needs the statistics of internal rows only (its target
// probabilities come from the parents' rows) and one leaf row at most (the
// bonus token), so the walks start while the leaf rows still stream.
struct StreamPlan {
  int G, nchunks, whole_rows_per_cta, split_first_row, split_items;   // whole_rows_per_cta: the most of any CTA
  int num_rows, mask_words;
  int dfs, key_bits;          // depth-first order of the internal rows; bits per level of its keys
  int walkers;                // CTAs G .. G + walkers - 1 only walk (0: every CTA streams and walks)
  __device__ int whole_rows(int c) const { return c < split_first_row ? (split_first_row - c + G - 1) / G : 0; }
  __device__ int items(int c) const {
    const int extra = split_items > c ? (split_items - c + G - 1) / G : 0;
    return whole_rows(c) * nchunks + extra;
  }
  // row, chunk and whether item k ends a segment (a whole row, or one split
  // chunk); `mine` lists the CTA's whole rows, `split` the split rows
  __device__ void item(int c, int k, const uint16_t* mine, const uint16_t* split, int& row, int& chunk,
                       bool& seg_end, bool& whole) const {
    const int n1 = whole_rows(c) * nchunks;
    if (k < n1) {
      row = mine[k / nchunks];
      chunk = k % nchunks;
      seg_end = chunk == nchunks - 1;
      whole = true;
    } else {
      const int j = c + (k - n1) * G;
      row = split[j / nchunks];
      chunk = j % nchunks;
      seg_end = true;
      whole = nchunks == 1;
    }
  }
};

// Requests whose row_indptr the prologue copies into shared memory (larger
// batches search it in global memory).
constexpr int kSmemIndptr = 4096;

// Largest launch whose internal rows go in depth-first order (the prologue's
// rank search is O(rows * (tree + batch)) per CTA).
constexpr int kDfsMaxRows = 4096, kDfsMaxBatch = 256, kDfsMaxNodes = 256;

// Shared-memory bytes of the stream-order tables (internal-row bit mask, the
// CTA's whole rows, the split rows, scan scratch, a copy of row_indptr; dfs:
// the rows' preorder keys and the requests' internal-row counts), placed after
// the walk state.
__host__ __device__ inline size_t order_smem_bytes(const StreamPlan& pl, int batch) {
  const size_t base = (size_t)pl.mask_words * 4 + (((size_t)pl.whole_rows_per_cta * 2 + 15) & ~(size_t)15) +
                      (((size_t)(pl.num_rows - pl.split_first_row) * 2 + 15) & ~(size_t)15) + 32 * 4 +
                      (batch < kSmemIndptr ? (size_t)(batch + 1) * 4 : 0);
  return pl.dfs ? ((base + 7) & ~(size_t)7) + (size_t)pl.num_rows * 14 + (size_t)batch * 4 +
                       (size_t)(kDfsMaxNodes + 1) * 8 + 32
                 : base;
}

// First row of the request that holds `row` (binary search over row_indptr).
// Barrier `id` over `count` threads (whole warps) of the CTA.
__device__ __forceinline__ void named_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ int request_index(const int32_t* indptr, int batch, int row) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (indptr[mid] <= row) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ int request_first_row(const int32_t* indptr, int batch, int row) {
  return indptr[request_index(indptr, batch, row)];
}

// Order-preserving integer key of a float (for the single-instruction warp
// max reduction): non-negative values keep their bits, negative ones flip the
// magnitude bits.  key_float inverts it.
__device__ __forceinline__ int float_key(float x) {
  const int b = __float_as_int(x);
  return b >= 0 ? b : (b ^ 0x7fffffff);
}
__device__ __forceinline__ float key_float(int k) { return __int_as_float(k >= 0 ? k : (k ^ 0x7fffffff)); }

__device__ __forceinline__ uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   su32(dst)),
               "l"(src), "r"(bytes), "r"(su32(bar))
               : "memory");
}
__device__ __forceinline__ void s_mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void s_mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(su32(bar)) : "memory");
}
__device__ __forceinline__ void s_mbar_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(su32(bar)),
               "r"(bytes)
               : "memory");
}
// Bounded wait (kSpinLimit clocks); false on timeout.  sleep_ns > 0 for
// waiters that can react late.
__device__ __forceinline__ bool s_mbar_wait(uint64_t* bar, uint32_t parity, uint32_t sleep_ns) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > kSpinLimit) return false;
    if (sleep_ns) __nanosleep(sleep_ns);
  }
}
// Row statistics from the row's merged partial `r` (valid in lane 0), by one
// warp (the warp rescans the row when a value below the max can round to the
// same probability), stored and published in the workspace.
__device__ int finish_row_warp(const AcceptParams& p, int row, Part r) {
  const int lane = threadIdx.x & 31;
  float m = 0.0f, sf = 0.0f, qmax = 0.0f;
  int arg = 0, tie = 0;
  if (lane == 0) {
    m = r.m;
    sf = (float)r.s;
    qmax = round_to_bf16(__fdiv_rn(1.0f, sf));
    arg = r.idx;
    tie = (r.m > -INFINITY) && (prob_bf16(prev_bf16(r.m), r.m, sf) == qmax);
  }
  m = __shfl_sync(0xffffffffu, m, 0);
  sf = __shfl_sync(0xffffffffu, sf, 0);
  qmax = __shfl_sync(0xffffffffu, qmax, 0);
  arg = __shfl_sync(0xffffffffu, arg, 0);
  tie = __shfl_sync(0xffffffffu, tie, 0);
  if (tie) {
    const uint16_t* rp = p.logits + (int64_t)row * p.row_stride;
    int best = INT_MAX;
    for (int e = lane; e < p.vocab; e += 32)
      if (prob_bf16(load_scaled(p, rp, e), m, sf) == qmax) {
        best = e;
        break;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
    arg = best;
  }
  if (lane == 0) {
    RowStat rs;
    rs.m = m;
    rs.s = sf;
    rs.argmax = arg;
    rs.flags = tie;
    p.row_ws[row] = rs;
    publish_row(p, row);
  }
  __syncwarp();
  return arg;                                          // the same in every lane
}

__device__ __forceinline__ Part shfl_part(const Part& x, int src_lane_xor) {
  Part o;
  o.s = __shfl_xor_sync(0xffffffffu, x.s, src_lane_xor);
  o.m = __shfl_xor_sync(0xffffffffu, x.m, src_lane_xor);
  o.idx = __shfl_xor_sync(0xffffffffu, x.idx, src_lane_xor);
  return o;
}

// Zeroes the workspace's counters and flags ahead of an acceptance launch
// (launched as a programmatic dependent: it waits for the previous kernel,
// which may be an acceptance on the same workspace, before writing).
__global__ void zero_ws_kernel(uint32_t* ws, size_t words) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += (size_t)gridDim.x * blockDim.x)
    ws[i] = 0u;
}

__global__ void __launch_bounds__(kSThreads, 1) accept_stream_kernel(const AcceptParams p, const StreamPlan plan) {
  extern __shared__ __align__(128) uint8_t sm[];
  pdl_trigger();
  pdl_wait();                           // launched as a programmatic dependent: nothing is read before this
  uint8_t* ring = sm;
  StreamCtl& ctl = *reinterpret_cast<StreamCtl*>(sm + kSCtlOff);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  const bool streams = c < plan.G;      // CTAs past G (dedicated walkers) stream nothing
  const int n_items = streams ? plan.items(c) : 0;
  const Part kNone{0.0, -INFINITY, INT_MAX};

  // stream-order tables after the walk state
  uint8_t* otab = sm + ((kSWalkOff + walk_smem_bytes(p.max_nodes) + 15) & ~(size_t)15);
  uint32_t* imask = reinterpret_cast<uint32_t*>(otab);
  uint16_t* mine = reinterpret_cast<uint16_t*>(otab + (size_t)plan.mask_words * 4);
  uint16_t* split = mine + ((plan.whole_rows_per_cta + 7) & ~7);
  int* scan = reinterpret_cast<int*>(split + ((plan.num_rows - plan.split_first_row + 7) & ~7));
  int* sindptr = scan + 32;
  const int32_t* indptr = p.batch < kSmemIndptr ? sindptr : p.row_indptr;
  if (p.batch < kSmemIndptr)
    for (int i = tid; i <= p.batch; i += kSThreads) sindptr[i] = p.row_indptr[i];
  // dfs tables (plan.dfs implies batch < kSmemIndptr)
  unsigned long long* okeys = reinterpret_cast<unsigned long long*>(
      (reinterpret_cast<uintptr_t>(sindptr + (p.batch < kSmemIndptr ? p.batch + 1 : 0)) + 7) & ~(uintptr_t)7);
  int* nint = reinterpret_cast<int*>(okeys + plan.num_rows);
  int16_t* spar = reinterpret_cast<int16_t*>(nint + p.batch);   // request-local parents (-1: none)
  int16_t* orank = spar + plan.num_rows;                         // internal rows: preorder rank
  int* rank_base = reinterpret_cast<int*>((reinterpret_cast<uintptr_t>(orank + plan.num_rows) + 3) & ~(uintptr_t)3);
  // rank_base[k]: the internal rows of rank below k over all requests (sum of min(nint, k))
  uint32_t* gtmask = reinterpret_cast<uint32_t*>(rank_base + kDfsMaxNodes + 1);
  // gtmask[k] (batches of at most 32): bit b set when request b has more than k internal rows
  int16_t* rreq = reinterpret_cast<int16_t*>(gtmask + kDfsMaxNodes + 1);   // dfs: the request of each row

  if (tid == 0) {
    for (int i = 0; i < kSSlots; ++i) {
      s_mbar_init(&ctl.full[i], 1);
      s_mbar_init(&ctl.empty[i], kSConsumerWarps);
    }
    for (int i = 0; i < 2; ++i) {
      s_mbar_init(&ctl.seg_full[i], kSConsumerWarps);
      s_mbar_init(&ctl.seg_empty[i], 1);
    }
    ctl.seg_max = 0ull;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // ---- stream order (every streaming CTA computes it for its own rows) -------
  if (streams) {
    // this thread's first two parents load while the row_indptr copy lands
    int pre[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) pre[u] = tid + u * kSThreads < plan.num_rows ? p.parents[tid + u * kSThreads] : -1;
    for (int i = tid; i < plan.mask_words; i += kSThreads) imask[i] = 0u;
    __syncthreads();
    for (int j = tid, u = 0; j < plan.num_rows; j += kSThreads, ++u) {
      const int b = request_index(indptr, p.batch, j);
      const int lo = indptr[b];
      const int pj = u < 2 ? pre[u] : p.parents[j];
      const bool has = j > lo && pj >= 0 && pj < j - lo;
      const int r = (j == lo) ? j : (has ? lo + pj : -1);
      if (r >= 0) atomicOr(&imask[r >> 5], 1u << (r & 31));
      if (plan.dfs) {
        spar[j] = (int16_t)(has ? pj : -1);
        rreq[j] = (int16_t)b;
      }
    }
    __syncthreads();
    if (plan.dfs) {
      // One warp per request.  Preorder key of every internal row: its
      // ancestors' node indices below the root (and its own), key_bits each,
      // the shallowest in the top bits and zeros below the node's depth, so a
      // node sorts before its subtree and siblings by index; the low 8 bits
      // hold the node's own index instead (unique keys; a request has at most
      // kDfsMaxNodes = 256 nodes here).  A chain longer than the key keeps its
      // top levels, one longer than the climb limit sorts last.  The keys of
      // the request's internal rows are packed at okeys[lo ..], then each
      // one's rank is the number of smaller keys: a permutation whatever the
      // tree.
      const int levels = 64 / plan.key_bits;
      for (int b = warp; b < p.batch; b += kSThreads / 32) {
        const int lo = indptr[b], n = indptr[b + 1] - lo;
        int m = 0;
        for (int i0 = 0; i0 < n; i0 += 32) {
          const int i = i0 + lane, j = lo + i;
          const bool in = i < n && ((imask[j >> 5] >> (j & 31)) & 1u);
          unsigned long long key = 0ull;
          if (in) {
            int v = i;
            for (int d = 0; v > 0 && d <= levels + 8; ++d) {   // parents precede children: v decreases
              key = (key >> plan.key_bits) | ((unsigned long long)v << (64 - plan.key_bits));
              v = max((int)spar[lo + v], 0);
            }
            key = ((v > 0 ? ~0ull : key) & ~0xffull) | (unsigned long long)i;
          }
          const unsigned bal = __ballot_sync(0xffffffffu, in);
          const int slot = m + __popc(bal & ((1u << lane) - 1u));
          if (in) {
            okeys[lo + slot] = key;
            if (n > kDfsMaxNodes) orank[j] = (int16_t)slot;     // (invalid sizes) row order
          }
          m += __popc(bal);
        }
        if (lane == 0) nint[b] = m;
        __syncwarp();
        for (int s0 = 0; n <= kDfsMaxNodes && s0 < m; s0 += 32) {
          const int sidx = s0 + lane;
          const unsigned long long kr = sidx < m ? okeys[lo + sidx] : ~0ull;
          int k = 0, t = 0;
          for (; t + 8 <= m; t += 8) {
            unsigned long long kk[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) kk[q] = okeys[lo + t + q];
#pragma unroll
            for (int q = 0; q < 8; ++q) k += kk[q] < kr ? 1 : 0;
          }
          for (; t < m; ++t) k += okeys[lo + t] < kr ? 1 : 0;
          if (sidx < m) orank[lo + (int)(kr & 0xffull)] = (int16_t)k;
        }
      }
      __syncthreads();
      for (int k = tid; k <= kDfsMaxNodes; k += kSThreads) {
        int sum = 0;
        uint32_t gt = 0u;
        for (int b2 = 0; b2 < p.batch; ++b2) {
          const int nb = nint[b2];
          sum += min(nb, k);
          if (b2 < 32 && nb > k) gt |= 1u << b2;
        }
        rank_base[k] = sum;
        gtmask[k] = gt;
      }
      __syncthreads();
    }
    const int per = (plan.num_rows + kSThreads - 1) / kSThreads;
    const int r0 = min(tid * per, plan.num_rows), r1 = min(r0 + per, plan.num_rows);
    int cnt = 0;
    for (int r = r0; r < r1; ++r) cnt += (imask[r >> 5] >> (r & 31)) & 1;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) scan[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int v = lane < kSThreads / 32 ? scan[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      if (lane < kSThreads / 32) scan[lane] = v;
    }
    __syncthreads();
    const int n_int = scan[kSThreads / 32 - 1];
    int ib = (warp ? scan[warp - 1] : 0) + incl - cnt;       // internal rows before r0
    for (int r = r0; r < r1; ++r) {
      const int in = (imask[r >> 5] >> (r & 31)) & 1;
      int q = in ? ib : n_int + (r - ib);
      if (in && plan.dfs) {
        // the internal rows go rank by rank, requests in order within a rank
        const int b = rreq[r];
        const int k = orank[r];
        if (k <= kDfsMaxNodes) {
          q = rank_base[k];
        } else {
          q = 0;
          for (int b2 = 0; b2 < p.batch; ++b2) q += min(nint[b2], k);
        }
        if (p.batch <= 32 && k <= kDfsMaxNodes) {
          q += __popc(gtmask[k] & ((1u << b) - 1u));
        } else {
          for (int b2 = 0; b2 < b; ++b2) q += nint[b2] > k ? 1 : 0;
        }
      }
      ib += in;
      if (q < plan.split_first_row) {
        if (q % plan.G == c) mine[q / plan.G] = (uint16_t)r;
      } else {
        split[q - plan.split_first_row] = (uint16_t)r;
      }
    }
  }
  __syncthreads();
  if (p.order_out && streams) {
    // the order for the next pass (every position once over the CTAs), and
    // its per-row flags cleared (leaf rows' set, when the next pass skips them)
    auto flag0 = [&](int r) -> unsigned {
      return (p.topp_skip_leaves && !((imask[r >> 5] >> (r & 31)) & 1u)) ? 1u : 0u;
    };
    for (int k = tid; k < plan.whole_rows(c); k += kSThreads) {
      const int r = mine[k];
      p.order_out[c + k * plan.G] = r;
      p.order_done[r] = flag0(r);
    }
    if (c == 0)
      for (int i = tid; i < plan.num_rows - plan.split_first_row; i += kSThreads) {
        const int r = split[i];
        p.order_out[plan.split_first_row + i] = r;
        p.order_done[r] = flag0(r);
      }
  }

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    int issued = 0;
    for (int k = 0; k < n_items; ++k) {
      const int slot = k % kSSlots;
      const bool ok = s_mbar_wait(&ctl.empty[slot], ((k / kSSlots) + 1) & 1, 32);
      if (!__all_sync(0xffffffffu, ok)) break;                       // consumers gave up
      if (lane == 0) {
        int row, chunk;
        bool seg_end, whole;
        plan.item(c, k, mine, split, row, chunk, seg_end, whole);
        const int n_el = min(kSChunk, p.vocab - chunk * kSChunk);
        s_mbar_expect(&ctl.full[slot], (uint32_t)n_el * 2);
        bulk_g2s(ring + (size_t)slot * kSChunk * 2, p.logits + (int64_t)row * p.row_stride + (int64_t)chunk * kSChunk,
                 (uint32_t)n_el * 2, &ctl.full[slot]);
      }
      __syncwarp();
      issued = k + 1;
    }
    // copies in flight must land before the CTA exits
    for (int k = max(0, issued - kSSlots); k < issued; ++k) s_mbar_wait(&ctl.full[k % kSSlots], (k / kSSlots) & 1, 32);
  } else if (warp <= kSConsumerWarps) {
    // ---------------------------------------------------------------- consumers
    const int ct = tid - 32, cw = warp - 1;
    // running partial of the current segment: per thread (max, sum relative to
    // it), per warp (max, first index of it; the same in every lane)
    float m_t = -INFINITY;
    double s_t = 0.0;
    float w_m = -INFINITY;
    int w_idx = INT_MAX;
    int seg = 0;
    for (int k = 0; k < n_items; ++k) {
      const int slot = k % kSSlots;
      int row, chunk;
      bool seg_end, whole;
      plan.item(c, k, mine, split, row, chunk, seg_end, whole);
      const int base = chunk * kSChunk;
      const int n_el = min(kSChunk, p.vocab - base);
      if (!s_mbar_wait(&ctl.full[slot], (k / kSSlots) & 1, 0)) break;
      const uint8_t* src = ring + (size_t)slot * kSChunk * 2;
      uint32_t v[kSVec * 4];
#pragma unroll
      for (int q = 0; q < kSVec; ++q) {
        const int vi = q * kSConsumers + ct;
        uint4 x = make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);   // -inf padding
        if (vi * 8 < n_el) x = *reinterpret_cast<const uint4*>(src + (size_t)vi * 16);
        v[4 * q + 0] = x.x;
        v[4 * q + 1] = x.y;
        v[4 * q + 2] = x.z;
        v[4 * q + 3] = x.w;
      }
      __syncwarp();
      if (lane == 0) s_mbar_arrive(&ctl.empty[slot]);
      if (p.use_temp) {
#pragma unroll
        for (int i = 0; i < kSVec * 4; ++i) v[i] = scale_pair(v[i], p.inv_temp);
      }
      uint32_t m2 = v[0];
#pragma unroll
      for (int i = 1; i < kSVec * 4; ++i) m2 = bf16x2_max(m2, v[i]);
      const float mt = fmaxf(__uint_as_float(m2 << 16), __uint_as_float(m2 & 0xffff0000u));
      if (mt > -INFINITY) {
        const float mlog = mt * kLog2e;
        const uint64_t sc2 = f2(kLog2e, kLog2e), nm2 = f2(-mlog, -mlog);
        uint64_t acc_a = f2(0.0f, 0.0f), acc_b = f2(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < kSVec * 4; ++i) {
          float a, b;
          f2_split(ffma2(f2(__uint_as_float(v[i] << 16), __uint_as_float(v[i] & 0xffff0000u)), sc2, nm2), a, b);
          const uint64_t e = f2(ex2_approx(a), ex2_approx(b));
          if (i & 1) acc_b = fadd2(acc_b, e);
          else acc_a = fadd2(acc_a, e);
        }
        float s0, s1, s2, s3;
        f2_split(acc_a, s0, s1);
        f2_split(acc_b, s2, s3);
        const double st = (double)((s0 + s1) + (s2 + s3));
        // fold into this thread's running partial of the segment
        if (mt > m_t) {
          s_t = s_t * (double)ex2_approx((m_t - mt) * kLog2e) + st;
          m_t = mt;
        } else {
          s_t += st * (double)ex2_approx((mt - m_t) * kLog2e);
        }
      }
      // the first index of the warp's max changes only when some lane raises it
      // (an equal max keeps the earlier, smaller index); a value below the
      // largest one another warp has located in this segment cannot be the
      // segment's max, so the warp skips it (the warp that holds the max
      // always locates it: the shared value never exceeds it)
      const unsigned long long cm = *reinterpret_cast<volatile unsigned long long*>(&ctl.seg_max);
      const float cmax = (unsigned)(cm >> 32) == (unsigned)(seg + 1) ? key_float((int)((unsigned)cm ^ 0x80000000u))
                                                                      : -INFINITY;
      if (__any_sync(0xffffffffu, mt > w_m && mt >= cmax)) {
        const float wm = key_float(__reduce_max_sync(0xffffffffu, float_key(mt)));
        // claim the value first: a warp whose max is already below one
        // another warp has claimed skips the scan (its max is not the
        // segment's), so of the warps that raise their max on the same chunk
        // only those at the running maximum scan
        unsigned long long prev = 0ull;
        if (lane == 0)
          prev = atomicMax(&ctl.seg_max,
                           ((unsigned long long)(unsigned)(seg + 1) << 32) | ((unsigned)float_key(wm) ^ 0x80000000u));
        prev = __shfl_sync(0xffffffffu, prev, 0);
        const float claimed =
            (unsigned)(prev >> 32) == (unsigned)(seg + 1) ? key_float((int)((unsigned)prev ^ 0x80000000u)) : -INFINITY;
        w_m = wm;
        if (wm >= claimed) {
          // branchless scan from the last value to the first: the smallest
          // index holding wm wins (padding is -inf and never equals the finite wm)
          int fi = INT_MAX;
#pragma unroll
          for (int q = kSVec - 1; q >= 0; --q) {
#pragma unroll
            for (int j = 3; j >= 0; --j) {
              const int e = base + (q * kSConsumers + ct) * 8 + 2 * j;
              const uint32_t u = v[4 * q + j];
              fi = (__uint_as_float(u & 0xffff0000u) == wm) ? e + 1 : fi;
              fi = (__uint_as_float(u << 16) == wm) ? e : fi;
            }
          }
          w_idx = (int)__reduce_min_sync(0xffffffffu, (unsigned)fi);
        } else {
          w_idx = kNotCandidate;
        }
      }
      if (seg_end) {
        // the warp's partial of the segment: sums relative to the warp max; the
        // index is a candidate only if the warp located that max
        const float wmax = key_float(__reduce_max_sync(0xffffffffu, float_key(m_t)));
        double ws = (m_t == -INFINITY) ? 0.0 : s_t * (double)ex2_approx((m_t - wmax) * kLog2e);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
        const int buf = seg & 1;
        if (!s_mbar_wait(&ctl.seg_empty[buf], ((seg >> 1) + 1) & 1, 0)) break;
        if (lane == 0) {
          ctl.seg[buf][cw] = (wmax == -INFINITY) ? kNone : Part{ws, wmax, w_m == wmax ? w_idx : kNotCandidate};
          s_mbar_arrive(&ctl.seg_full[buf]);
        }
        __syncwarp();
        m_t = -INFINITY;
        s_t = 0.0;
        w_m = -INFINITY;
        w_idx = INT_MAX;
        ++seg;
      }
    }
  } else if (warp == kSConsumerWarps + 1) {
    // ---------------------------------------------------------------- merger
    int seg = 0;
    for (int k = 0; k < n_items; ++k) {
      int row, chunk;
      bool seg_end, whole;
      plan.item(c, k, mine, split, row, chunk, seg_end, whole);
      if (!seg_end) continue;
      const int buf = seg & 1;
      if (!s_mbar_wait(&ctl.seg_full[buf], (seg >> 1) & 1, 0)) break;
      // the 16 warp partials, merged pairwise in warp order
      Part x = lane < kSConsumerWarps ? ctl.seg[buf][lane] : kNone;
      __syncwarp();
      if (lane == 0) s_mbar_arrive(&ctl.seg_empty[buf]);
#pragma unroll
      for (int o = 1; o < kSConsumerWarps; o <<= 1) {
        const Part y = shfl_part(x, o);
        x = (lane & o) ? merge(y, x) : merge(x, y);
      }
      ++seg;
      bool row_done = whole;
      if (!whole) {
        // one chunk of a split row: publish it; the last chunk to arrive merges the row
        unsigned prev = 0;
        if (lane == 0) {
          p.part_ws[(int64_t)row * plan.nchunks + chunk] = x;
          asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&p.row_ctr[row]) : "memory");
        }
        row_done = __shfl_sync(0xffffffffu, prev, 0) == (unsigned)(plan.nchunks - 1);
        if (row_done && lane == 0) {
          const Part* pp = p.part_ws + (int64_t)row * plan.nchunks;
          x = Part{__ldcg(&pp[0].s), __ldcg(&pp[0].m), __ldcg(&pp[0].idx)};
          for (int i = 1; i < plan.nchunks; ++i)
            x = merge(x, Part{__ldcg(&pp[i].s), __ldcg(&pp[i].m), __ldcg(&pp[i].idx)});
        }
      }
      if (!row_done) continue;
      if (p.parts_out) {
        if (lane == 0) {
          if (x.idx < kNotCandidate) x.idx += p.vocab_offset;
          p.parts_out[row] = x;
        }
        __syncwarp();
        continue;
      }
      finish_row_warp(p, row, x);
    }
  } else if (warp == kSConsumerWarps + 2) {
    // ---------------------------------------------------------------- walker
    // Claims the next request and walks it, waiting for each row it reads
    // (parents' rows, the bonus row) to be published: the walks of different
    // requests run on different SMs while the leaf rows still stream.
    if (p.no_walk || (plan.walkers && streams)) return;
    if (p.parts_out) {
      // shard partials mode: each node's token logit, if this shard holds the token
      for (int r = c * 32 + lane; r < p.num_rows; r += plan.G * 32) {
        const int lo = request_first_row(indptr, p.batch, r);
        const int pj = p.parents[r], tk = p.tokens[r] - p.vocab_offset;
        float xv = -INFINITY;
        if (r > lo && pj >= 0 && pj < r - lo && tk >= 0 && tk < p.vocab)
          xv = load_scaled(p, p.logits + (int64_t)(lo + pj) * p.row_stride, tk);
        p.tok_logit_out[r] = xv;
      }
      return;
    }
    const WalkSmem w = walk_smem(sm + kSWalkOff, p.max_nodes);
    for (;;) {
      unsigned t = 0;
      if (lane == 0) t = atomicAdd(&p.walk_ctr[1], 1u);
      t = __shfl_sync(0xffffffffu, t, 0);
      const int b = t < (unsigned)p.batch ? (int)t : -1;
      if (!p.traversal) {
        if (b < 0) break;
        const int lo = p.row_indptr[b];
        walk_request(p, b, lo, p.row_indptr[b + 1] - lo, w, WarpGroup{}, nullptr, streams ? nullptr : ring,
                     streams ? 0 : kSRingBytes);
        continue;
      }
      // traversal: set-up, hand the request to the expander, walk lazily
      int lo = 0, n = 0;
      bool go = false;
      if (b >= 0) {
        lo = p.row_indptr[b];
        n = p.row_indptr[b + 1] - lo;
        go = walk_request<true>(p, b, lo, n, w, WarpGroup{}, nullptr);
      }
      if (lane == 0) {
        ctl.walk_b = b < 0 ? -1 : go ? b : -2;
        ctl.walk_done = 0;
      }
      named_barrier(1, 64);
      if (b < 0) break;
      if (go) walk_traversal_warp<true>(p, b, lo, n, w);
      // a walker CTA streams nothing: its copy ring stages the compaction
      if (p.compact) compact_request_warp(p, b, streams ? nullptr : ring, streams ? 0 : kSRingBytes);
      if (lane == 0) *(volatile int*)&ctl.walk_done = 1;
      named_barrier(2, 64);
    }
  } else {
    // -------------------------------------------------------------- expander
    if (p.no_walk || p.parts_out || !p.traversal || (plan.walkers && streams)) return;
    const WalkSmem w = walk_smem(sm + kSWalkOff, p.max_nodes);
    for (;;) {
      named_barrier(1, 64);
      const int b = *(volatile int*)&ctl.walk_b;
      if (b == -1) break;
      if (b >= 0) {
        const int lo = p.row_indptr[b];
        expand_request(p, lo, p.row_indptr[b + 1] - lo, w, &ctl.walk_done);
      }
      named_barrier(2, 64);
    }
  }
}

// ---- greedy path chain ------------------------------------------------------
// A greedy walk reads the statistics of the rows on its accepted path only
// (the root's, then each accepted node's: at most the tree's depth + 1 rows,
// verification.py:232-262), so the compacting greedy step reduces exactly
// those rows, each as soon as its walk asks for it, instead of every row.
// Request b belongs to group b % groups of gs CTAs; member 0's walker warp
// runs the unchanged greedy walk (walk_request / walk_greedy_warp with
// p.chain set: it posts each row it waits for), and the group's 16 reducer
// warps per CTA split that row's 32 KB chunks over the members: chunk k of
// the row on member k % gs.  A chunk is reduced with the streaming kernel's
// consumer arithmetic (the same lanes and values per thread, the same warp
// reduction and warp-order merge) and published as a partial of a split
// row; the chunk that arrives last merges the row's partials in chunk order
// and derives the row statistics (finish_row_warp), so a row's statistics
// are the ones the streaming kernel gives a split row.  Every wait is
// bounded: a group that gives up leaves its walk to report -3.
constexpr int kChainWarps = kSConsumerWarps + 1;   // 16 reducer warps + the walker
constexpr int kChainThreads = kChainWarps * 32;

// Chunk `k` of row `row` by the 16 reducer warps of the CTA (threads
// 0..511): the chunk's partial into part_ws; the last chunk of the row to
// arrive merges the row and publishes its statistics.
__device__ void chain_reduce_chunk(const AcceptParams& p, int b, int lo, int n, int cur, unsigned seq, int k,
                                   int nchunks, Part* wparts, const int* tpar, const int* ttok) {
  const int row = lo + cur;
  const int ct = threadIdx.x, lane = ct & 31, warp = ct >> 5;
  const int base = k * kSChunk;
  const int n_el = min(kSChunk, p.vocab - base);
  const uint16_t* src = p.logits + (int64_t)row * p.row_stride + base;
  uint32_t v[kSVec * 4];
#pragma unroll
  for (int q = 0; q < kSVec; ++q) {
    const int vi = q * kSConsumers + ct;
    uint4 x = make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);   // -inf padding
    if (vi * 8 < n_el) x = ld_stream(src + (size_t)vi * 8);
    v[4 * q + 0] = x.x;
    v[4 * q + 1] = x.y;
    v[4 * q + 2] = x.z;
    v[4 * q + 3] = x.w;
  }
  if (p.use_temp) {
#pragma unroll
    for (int i = 0; i < kSVec * 4; ++i) v[i] = scale_pair(v[i], p.inv_temp);
  }
  uint32_t m2 = v[0];
#pragma unroll
  for (int i = 1; i < kSVec * 4; ++i) m2 = bf16x2_max(m2, v[i]);
  const float mt = fmaxf(__uint_as_float(m2 << 16), __uint_as_float(m2 & 0xffff0000u));
  // this thread's partial of the chunk, as the streaming consumer folds its
  // first chunk of a segment into an empty partial
  float m_t = -INFINITY;
  double s_t = 0.0;
  if (mt > -INFINITY) {
    const float mlog = mt * kLog2e;
    const uint64_t sc2 = f2(kLog2e, kLog2e), nm2 = f2(-mlog, -mlog);
    uint64_t acc_a = f2(0.0f, 0.0f), acc_b = f2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < kSVec * 4; ++i) {
      float a, b;
      f2_split(ffma2(f2(__uint_as_float(v[i] << 16), __uint_as_float(v[i] & 0xffff0000u)), sc2, nm2), a, b);
      const uint64_t e = f2(ex2_approx(a), ex2_approx(b));
      if (i & 1) acc_b = fadd2(acc_b, e);
      else acc_a = fadd2(acc_a, e);
    }
    float s0, s1, s2, s3;
    f2_split(acc_a, s0, s1);
    f2_split(acc_b, s2, s3);
    const double st = (double)((s0 + s1) + (s2 + s3));
    s_t = s_t * (double)ex2_approx((m_t - mt) * kLog2e) + st;
    m_t = mt;
  }
  // the warp's partial: its max, the first index holding it, the sum relative to it
  const float wmax = key_float(__reduce_max_sync(0xffffffffu, float_key(m_t)));
  int fi = INT_MAX;
#pragma unroll
  for (int q = kSVec - 1; q >= 0; --q) {
#pragma unroll
    for (int j = 3; j >= 0; --j) {
      const int e = base + (q * kSConsumers + ct) * 8 + 2 * j;
      const uint32_t u = v[4 * q + j];
      fi = (__uint_as_float(u & 0xffff0000u) == wmax) ? e + 1 : fi;
      fi = (__uint_as_float(u << 16) == wmax) ? e : fi;
    }
  }
  const int w_idx = (int)__reduce_min_sync(0xffffffffu, (unsigned)fi);
  double ws = (m_t == -INFINITY) ? 0.0 : s_t * (double)ex2_approx((m_t - wmax) * kLog2e);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
  if (lane == 0) wparts[warp] = (wmax == -INFINITY) ? Part{0.0, -INFINITY, INT_MAX} : Part{ws, wmax, w_idx};
  named_barrier(2, kSConsumers);
  if (warp == 0) {
    // the 16 warp partials, merged pairwise in warp order; the chunk's partial
    // published; the row's last chunk merges the row
    Part x = lane < kSConsumerWarps ? wparts[lane] : Part{0.0, -INFINITY, INT_MAX};
#pragma unroll
    for (int o = 1; o < kSConsumerWarps; o <<= 1) {
      const Part y = shfl_part(x, o);
      x = (lane & o) ? merge(y, x) : merge(x, y);
    }
    unsigned prev = 0;
    if (lane == 0) {
      p.part_ws[(int64_t)row * nchunks + k] = x;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&p.row_ctr[row]) : "memory");
    }
    if (__shfl_sync(0xffffffffu, prev, 0) == (unsigned)(nchunks - 1)) {
      if (lane == 0) {
        const Part* pp = p.part_ws + (int64_t)row * nchunks;
        x = Part{__ldcg(&pp[0].s), __ldcg(&pp[0].m), __ldcg(&pp[0].idx)};
        for (int i = 1; i < nchunks; ++i) x = merge(x, Part{__ldcg(&pp[i].s), __ldcg(&pp[i].m), __ldcg(&pp[i].idx)});
      }
      const int tok = finish_row_warp(p, row, x);
      // the walk's next row, posted here instead of after the walker has
      // read this one: the first child of `cur` (index order, as the walk's
      // child runs) whose token is the row's argmax, unless that token ends
      // the path (EOS); no child matches: the walk needs no further row
      int match = INT_MAX;
      if (!(p.eos >= 0 && (int64_t)tok == p.eos)) {
        for (int i0 = cur + 1; i0 < n && match == INT_MAX; i0 += 32) {
          const int i = i0 + lane;
          const bool hit = i < n && tpar[i] == cur && ttok[i] == tok;
          const unsigned bal = __ballot_sync(0xffffffffu, hit);
          if (bal) match = i0 + __ffs(bal) - 1;
        }
      }
      if (lane == 0 && match != INT_MAX) chain_post_lane(p, b, seq + 1, match);
      __syncwarp();
    }
  }
  named_barrier(2, kSConsumers);                       // wparts free again
}

__global__ void __launch_bounds__(kChainThreads, 1) greedy_chain_kernel(const AcceptParams p, int gs, int groups) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ Part wparts[kSConsumerWarps];
  __shared__ int s_cmd[2];
  pdl_trigger();
  pdl_wait();                           // launched as a programmatic dependent: nothing is read before this
  const int c = blockIdx.x, warp = threadIdx.x >> 5;
  if (c >= groups * gs) return;
  const int gi = c / gs, m = c % gs;
  const int nchunks = (p.vocab + kSChunk - 1) / kSChunk;
  // the reducers' copy of the current request's parents and tokens (after the walker's state)
  int* tpar = reinterpret_cast<int*>(sm + ((walk_smem_bytes(p.max_nodes) + 15) & ~(size_t)15));
  int* ttok = tpar + p.max_nodes;
  if (warp == kSConsumerWarps) {
    // ------------------------------------------------------------ walker (member 0)
    if (m != 0) return;
    const WalkSmem w = walk_smem(sm, p.max_nodes);
    for (int b = gi; b < p.batch; b += groups) {
      const int lo = p.row_indptr[b], n = p.row_indptr[b + 1] - lo;
      if (n > 0) chain_post(p, b, 1, 0);               // the root's row: reduced while the tree loads
      walk_request<false>(p, b, lo, n, w, WarpGroup{}, nullptr);
      chain_post(p, b, kChainDone, 0);
    }
    return;
  }
  // -------------------------------------------------------------- reducers
  int phase = 0;
  for (int b = gi; b < p.batch; b += groups) {
    const int lo = p.row_indptr[b], n = p.row_indptr[b + 1] - lo;
    // (every reducer of the previous request is past its last barrier: its
    // merges are done; the first barrier below publishes these copies)
    for (int i = threadIdx.x; i < min(n, p.max_nodes); i += kSConsumers) {
      tpar[i] = __ldg(p.parents + lo + i);
      ttok[i] = __ldg(p.tokens + lo + i);
    }
    unsigned seq = 1;
    for (;;) {
      if (threadIdx.x == 0) {
        // the next request of this walk: sequence seq or later, or the end
        int cmd = -1;
        const long long t0 = clock64();
        for (;;) {
          unsigned v;
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.req_ctr + b) : "memory");
          const unsigned sq = v >> 16;
          if (sq == kChainDone) break;
          if (sq >= seq) {
            seq = sq;
            cmd = (int)(v & 0xffffu);
            break;
          }
          if (clock64() - t0 > kRowWaitLimit) break;   // the walk reports the rows it does not get
          __nanosleep(32);
        }
        s_cmd[phase] = cmd;
      }
      named_barrier(1, kSConsumers);
      const int cmd = s_cmd[phase];
      phase ^= 1;
      if (cmd < 0 || cmd >= n || n > p.max_nodes) break;
      for (int k = m; k < nchunks; k += gs) chain_reduce_chunk(p, b, lo, n, cmd, seq, k, nchunks, wparts, tpar, ttok);
      ++seq;
    }
  }
}

int stream_sm_count() {
  static int count[256] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return 0;
  if (!count[dev]) {
    int c = 0;
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    count[dev] = c;
  }
  return count[dev];
}

size_t ws_layout(int num_rows, int vocab, size_t* off_parts, size_t* off_rows, size_t* off_rctr,
                 size_t* off_qctr, size_t* off_walk = nullptr) {
  const int nchunks = (vocab + kChunk - 1) / kChunk;
  size_t o = 0;
  *off_parts = o;
  o = align_up(o + (size_t)num_rows * nchunks * sizeof(Part), 256);
  *off_rows = o;
  o = align_up(o + (size_t)num_rows * sizeof(RowStat), 256);
  *off_rctr = o;
  o = align_up(o + (size_t)num_rows * sizeof(unsigned), 256);
  *off_qctr = o;
  o = align_up(o + (size_t)num_rows * sizeof(unsigned), 256);
  if (off_walk) *off_walk = o;
  o = align_up(o + 2 * sizeof(unsigned) + (size_t)num_rows * sizeof(unsigned), 256);   // walk_ctr, row_done
  return o;
}

int accept_launch(AcceptParams p, int traversal, float temperature, void* workspace, size_t ws_bytes,
                  cudaStream_t stream, bool* streamed = nullptr) {
  PTS_CHECK_ARG(p.logits && p.row_indptr && p.parents && p.tokens, "null input pointer");
  PTS_CHECK_ARG(p.parts_out ? (p.tok_logit_out != nullptr) : (p.out_tokens && p.out_hidden && p.out_counts),
                "null output pointer");
  PTS_CHECK_ARG(p.batch > 0 && p.num_rows >= p.batch, "need batch > 0 and num_rows >= batch");
  PTS_CHECK_ARG(p.vocab > 0 && p.row_stride >= p.vocab, "need vocab > 0 and row_stride >= vocab");
  PTS_CHECK_ARG(p.max_nodes > 0, "max_nodes must be positive");
  if (p.max_nodes > PTS_MAX_TREE_NODES)
    return set_error(PTS_ERR_CAPACITY, "max_nodes %d above PTS_MAX_TREE_NODES %d", p.max_nodes,
                     PTS_MAX_TREE_NODES);
  if (p.vocab > kMaxChunks * kChunk)
    return set_error(PTS_ERR_UNSUPPORTED, "vocab %d above %d", p.vocab, kMaxChunks * kChunk);
  PTS_CHECK_ARG(p.parts_out || p.out_stride >= 1, "out_stride must be positive");
  PTS_CHECK_ARG(temperature > 0.0f, "temperature must be positive");
  if (p.num_rows > 65535) return set_error(PTS_ERR_CAPACITY, "num_rows %d above 65535", p.num_rows);
  size_t opt, orw, orc, oqc, owk;
  const size_t need = ws_layout(p.num_rows, p.vocab, &opt, &orw, &orc, &oqc, &owk);
  if (!workspace || ws_bytes < need)
    return set_error(PTS_ERR_CAPACITY, "workspace of %zu bytes, need %zu", ws_bytes, need);
  PTS_CHECK_ARG(((uintptr_t)workspace & 255) == 0, "workspace must be 256-byte aligned");
  char* ws = (char*)workspace;
  const int nchunks = (p.vocab + kChunk - 1) / kChunk;
  p.part_ws = (Part*)(ws + opt);
  p.row_ws = (RowStat*)(ws + orw);
  p.row_ctr = (unsigned*)(ws + orc);
  p.req_ctr = (unsigned*)(ws + oqc);
  p.walk_ctr = (unsigned*)(ws + owk);
  p.row_done = (unsigned*)(ws + owk + 2 * sizeof(unsigned));
  p.traversal = traversal;
  p.use_temp = (temperature != 1.0f);
  p.inv_temp = 1.0f / temperature;
  p.vec_ok = (((uintptr_t)p.logits & 15) == 0) && (p.row_stride % 8 == 0);
  {
    const size_t words = (need - orc) / 4;
    const size_t want = (words + 255) / 256;
    const int blocks = (int)(want < 148 ? want : 148);
    PTS_CUDA_TRY(launch_pdl(zero_ws_kernel, dim3(blocks > 0 ? blocks : 1), dim3(256), 0, stream,
                            (uint32_t*)(ws + orc), words));
  }
  const int sms = stream_sm_count();
  int dev = 0;
  PTS_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 256) return set_error(PTS_ERR_UNSUPPORTED, "device ordinal %d", dev);
  if (p.vec_ok && p.vocab % 8 == 0 && sms > 0 && p.step_form && !p.traversal && !p.parts_out && !p.no_walk &&
      !p.order_out && p.max_nodes <= 0xffff) {
    // greedy step: the rows on the accepted paths only, each reduced when its
    // walk asks for it (greedy_chain_kernel); gs CTAs per request, at most one
    // per chunk of a row
    const int gs = max(1, min(nchunks, sms / p.batch));
    const int groups = min(p.batch, max(1, sms / gs));
    const size_t smem = ((walk_smem_bytes(p.max_nodes) + 15) & ~(size_t)15) + (size_t)p.max_nodes * 8;
    if (smem <= kMaxDynSmem - 8 * 1024) {
      p.chain = 1;
      if (int rc = ensure_smem_attr((const void*)greedy_chain_kernel, smem)) return rc;
      PTS_CUDA_TRY(launch_pdl(greedy_chain_kernel, dim3(groups * gs), dim3(kChainThreads), smem, stream, p, gs,
                              groups));
      if (streamed) *streamed = true;
      return launch_status("greedy_chain_kernel");
    }
  }
  if (p.vec_ok && p.vocab % 8 == 0 && sms > 0) {
    StreamPlan plan;
    // small traversal batches: one CTA per walk that streams nothing, so the
    // walk's dependent chain does not share issue slots with the consumers
    plan.walkers = (p.traversal && !p.parts_out && !p.no_walk && p.batch <= sms / 8) ? p.batch : 0;
    plan.G = min(sms - plan.walkers, p.num_rows * nchunks);
    plan.nchunks = nchunks;
    // the rows past the last full round of G are split by chunk over all CTAs
    // when that adds at most two chunks per CTA or every CTA streams few rows
    // (a split chunk costs its merger a global atomic and, for the last
    // chunk, the row's merge); otherwise they go whole, one more row for some
    const int rounds = p.num_rows / plan.G;
    const int rem = p.num_rows - rounds * plan.G;
    plan.split_first_row = (rounds < 4 || rem * nchunks <= 2 * plan.G) ? rounds * plan.G : p.num_rows;
    plan.whole_rows_per_cta = (plan.split_first_row + plan.G - 1) / plan.G;
    plan.split_items = (p.num_rows - plan.split_first_row) * nchunks;
    plan.num_rows = p.num_rows;
    plan.mask_words = (p.num_rows + 31) / 32;
    plan.dfs = p.traversal && p.num_rows <= kDfsMaxRows && p.batch <= kDfsMaxBatch && p.max_nodes <= kDfsMaxNodes;
    plan.key_bits = p.max_nodes > 1 ? 32 - __builtin_clz((unsigned)(p.max_nodes - 1)) : 1;
    const size_t ssmem =
        ((kSWalkOff + walk_smem_bytes(p.max_nodes) + 15) & ~(size_t)15) + order_smem_bytes(plan, p.batch);
    if (ssmem <= kMaxDynSmem) {
      if (int rc = ensure_smem_attr((const void*)accept_stream_kernel, ssmem)) return rc;
      PTS_CUDA_TRY(launch_pdl(accept_stream_kernel, dim3(plan.G + plan.walkers), dim3(kSThreads), ssmem, stream, p,
                              plan));
      if (streamed) *streamed = true;
      return launch_status("accept_stream_kernel");
    }
  }
  const size_t smem = walk_smem_bytes(p.max_nodes);
  if (int rc = ensure_smem_attr((const void*)accept_kernel, smem, true)) return rc;
  accept_kernel<<<dim3(nchunks, p.num_rows), kThreads, smem, stream>>>(p);
  return launch_status("accept_kernel");
}

// ---------------------------------------------------------------------------
// Top-p (nucleus) target distribution and sampled bonus tokens.  Neither has a
// counterpart in the reference's acceptance (it renormalises nothing and takes
// the bonus by argmax unless do_sample, verification.py:508-511), so the rules
// are stated here and restated exactly by the oracle:
//   nucleus of a row   all tokens whose (scaled) logit is >= t*, where t* is
//                      the largest logit value whose cumulative mass from the
//                      top, sum over values v >= t* of count(v) * expf(v - m)
//                      (fp64, values in descending order), reaches
//                      top_p * s (s = the row's fp32 sum of exp(x - m));
//                      that cumulative mass, rounded to fp32, is the
//                      nucleus mass s_N; p'(x) = bf16(expf(x - m) / s_N);
//   sampled bonus      inverse CDF over the accepted row's bf16-rounded
//                      probabilities (p' under top-p): 1024 consecutive
//                      segments summed in fp64, their sums accumulated in
//                      order, target = u * total with u the Philox draw
//                      2 * PTS_MAX_TREE_NODES of the request's stream; the
//                      first index whose running sum exceeds the target.

constexpr int kToppThreads = 512;
constexpr int kToppFirstWindow = 256;    // distinct values counted by the first pass (two binades)
constexpr int kToppMaxWindow = 4096;     // later passes widen the window up to this

// Order-preserving 16-bit key of a bf16 value (-0 folded onto +0).
__device__ __forceinline__ uint32_t bf16_key(uint32_t bits) {
  if (bits == 0x8000u) bits = 0u;
  return (bits & 0x8000u) ? (~bits & 0xffffu) : (bits | 0x8000u);
}
__device__ __forceinline__ float key_bf16(uint32_t key) {
  const uint32_t bits = (key & 0x8000u) ? (key & 0x7fffu) : (~key & 0xffffu);
  return __uint_as_float(bits << 16);
}

__device__ __forceinline__ uint32_t scaled_bits(const AcceptParams& p, const uint16_t* row, int e) {
  return __float_as_uint(load_scaled(p, row, e)) >> 16;
}

// Counts a window of positive values over a row of nv 16-byte groups: every
// bf16 bit pattern b in [hi - span, hi] adds one to cnt[hi - b].  Such a
// window is one contiguous range of bit patterns that no negative value (and
// no -inf padding) reaches, so i = hi - b (unsigned) is in the window exactly
// when i <= span.  Every value takes one shared-memory increment, with no
// branch: a value outside the window goes to slot span + 1 + lane past the
// window (cnt holds 32 slots more than the widest window; they are never
// read), one bank per lane, so those increments do not conflict with each
// other.  (Increments predicated off instead measured slower.)  Two sets of
// four groups per thread alternate: the next set's loads are in flight while
// the current set is counted.
template <int kGroups>
__device__ __forceinline__ void load_groups(uint4 (&x)[kGroups], const uint16_t* rp, int v0, int nv) {
#pragma unroll
  for (int u = 0; u < kGroups; ++u) {
    // groups past the row read as -inf (never counted); the load is
    // predicated off for them rather than branched around
    const int vi = v0 + u * kToppThreads;
    const uint16_t* src = rp + (int64_t)min(vi, nv - 1) * 8;
    asm volatile(
        "{\n\t.reg .pred q;\n\t"
        "setp.lt.s32 q, %4, %5;\n\t"
        "mov.b32 %0, 0xff80ff80;\n\tmov.b32 %1, 0xff80ff80;\n\t"
        "mov.b32 %2, 0xff80ff80;\n\tmov.b32 %3, 0xff80ff80;\n\t"
        "@q ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%6];\n\t}"
        : "=r"(x[u].x), "=r"(x[u].y), "=r"(x[u].z), "=r"(x[u].w)
        : "r"(vi), "r"(nv), "l"(src));
  }
}

template <bool kTemp>
__device__ __forceinline__ void count_pos_window(const uint16_t* rp, int nv, uint32_t hi, uint32_t span, float inv_t,
                                                 uint32_t* cnt) {
  constexpr int kGroups = 4;
  const uint32_t dummy = span + 1u + (threadIdx.x & 31u);
  auto count = [&](const uint4 (&x)[kGroups]) {
#pragma unroll
    for (int u = 0; u < kGroups; ++u) {
      uint32_t w[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (kTemp) w[k] = scale_pair(w[k], inv_t);
        atomicAdd(&cnt[min(hi - (w[k] & 0xffffu), dummy)], 1u);
        atomicAdd(&cnt[min(hi - (w[k] >> 16), dummy)], 1u);
      }
    }
  };
  uint4 a[kGroups], b[kGroups];
  constexpr int kStep = kGroups * kToppThreads;
  int v0 = threadIdx.x;
  if (v0 >= nv) return;
  load_groups(a, rp, v0, nv);
  for (;;) {
    v0 += kStep;
    const bool more_b = v0 < nv;
    if (more_b) load_groups(b, rp, v0, nv);
    count(a);
    if (!more_b) break;
    v0 += kStep;
    const bool more_a = v0 < nv;
    if (more_a) load_groups(a, rp, v0, nv);
    count(b);
    if (!more_a) break;
  }
}

// One CTA per row.  Each pass counts the occurrences of every distinct value
// in a window of keys below the previous one (the first window holds the row
// max and the 255 values below it; later windows are wider), then takes the
// cumulative mass from the top, sum of count(v) * expf(v - m) in descending
// value order in fp64, until it reaches top_p * s.
//
// The cumulative sums are taken as a parallel prefix over the window.  That
// equals the ordered fp64 sum whenever no partial sum rounds: every term is a
// multiple of the ulp u of the smallest term involved (an integer times an fp32
// value of at least that size), so every partial sum is exact while it stays
// below 2^53 u.  The pass checks that bound (with a margin far above its own
// rounding) and otherwise walks the window in order on one thread, as the rule
// states.
__device__ void topp_row(const AcceptParams& p, float top_p, float* thresh, float* mass, int row) {
  __shared__ uint32_t cnt[kToppMaxWindow + 32];               // index i: key hi_key - i (descending values)
  __shared__ double wtot[kToppThreads / 32];
  __shared__ int s_cross, s_last, s_done;
  __shared__ float s_t;
  __shared__ double s_cum, s_pre;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const RowStat rs = p.row_ws[row];
  const uint16_t* rp = p.logits + (int64_t)row * p.row_stride;
  const double target = (double)top_p * (double)rs.s;
  const bool vec = (((uintptr_t)p.logits & 15) == 0) && (p.row_stride % 8 == 0);
  auto term = [&](int hi_key, int i, uint32_t c) -> double {
    return (double)c * (double)expf(key_bf16((uint32_t)(hi_key - i)) - rs.m);
  };
  if (tid == 0) {
    s_cum = 0.0;
    s_t = -INFINITY;
    s_done = 0;
  }
  int width = kToppFirstWindow;
  for (int hi_key = (int)bf16_key(__float_as_uint(rs.m) >> 16); hi_key >= 0;
       hi_key -= width, width = min(2 * width, kToppMaxWindow)) {
    const int lo_key = max(0, hi_key - width + 1);
    const int n = hi_key - lo_key + 1;
    // a value is counted when its key is in [lo_key, hi_key]; the float test
    // is a cheap superset of that (it merges -0 and +0), the key test decides
    const float vlo = key_bf16((uint32_t)lo_key), vhi = key_bf16((uint32_t)hi_key);
    for (int i = tid; i < n; i += kToppThreads) cnt[i] = 0u;
    if (tid == 0) {
      s_cross = INT_MAX;
      s_last = -1;
    }
    __syncthreads();
    // A window of positive values (the usual case) is a contiguous range of
    // bf16 bit patterns [lo_bits, hi_bits] that no negative value reaches, and
    // its key is bits | 0x8000: one unsigned compare decides, no key math.
    const bool pos_window = vlo > 0.0f;
    const uint32_t lo_bits = __float_as_uint(vlo) >> 16, span = (__float_as_uint(vhi) >> 16) - lo_bits;
    const uint32_t hi_bits = lo_bits + span;
    auto count1 = [&](uint32_t bits) {
      if (pos_window) {
        if (bits - lo_bits <= span) atomicAdd(&cnt[hi_bits - bits], 1u);
        return;
      }
      const float a = __uint_as_float(bits << 16);
      if (a >= vlo && a <= vhi) {
        const int k = (int)bf16_key(bits);
        if (k >= lo_key && k <= hi_key) atomicAdd(&cnt[hi_key - k], 1u);
      }
    };
    int e_tail = 0;
    if (vec && pos_window) {
      const int nv = p.vocab / 8;
      if (p.use_temp) {
        count_pos_window<true>(rp, nv, hi_bits, span, p.inv_temp, cnt);
      } else {
        count_pos_window<false>(rp, nv, hi_bits, span, p.inv_temp, cnt);
      }
      e_tail = nv * 8;
    } else if (vec) {
      const int nv = p.vocab / 8;
      for (int v0 = tid; v0 < nv; v0 += 4 * kToppThreads) {
        uint4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int vi = v0 + u * kToppThreads;
          x[u] = vi < nv ? ld_stream(rp + (int64_t)vi * 8)
                         : make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);   // -inf: never counted
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t w[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (p.use_temp) w[k] = scale_pair(w[k], p.inv_temp);
            count1(w[k] & 0xffffu);
            count1(w[k] >> 16);
          }
        }
      }
      e_tail = nv * 8;
    }
    for (int e = e_tail + tid; e < p.vocab; e += kToppThreads) count1(scaled_bits(p, rp, e));
    __syncthreads();
    // per-thread sums over entries [i0, i0 + E), then a block-wide exclusive prefix
    const int E = (n + kToppThreads - 1) / kToppThreads;
    const int i0 = min(tid * E, n), i1 = min(i0 + E, n);
    double loc = 0.0;
    for (int i = i0; i < i1; ++i)
      if (cnt[i]) loc += term(hi_key, i, cnt[i]);
    double inc = loc;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const double o = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += o;
    }
    if (lane == 31) wtot[warp] = inc;
    __syncthreads();
    double pre = s_cum + inc - loc;
    for (int w = 0; w < warp; ++w) pre += wtot[w];
    int my_cross = INT_MAX, my_last = -1;
    double my_pre = 0.0;
    for (int i = i0; i < i1; ++i) {
      const uint32_t c = cnt[i];
      if (!c) continue;
      pre += term(hi_key, i, c);
      my_last = i;
      if (pre >= target) {
        my_cross = i;
        my_pre = pre;
        break;
      }
    }
    if (my_cross != INT_MAX) atomicMin(&s_cross, my_cross);
    if (my_last >= 0) atomicMax(&s_last, my_last);
    __syncthreads();
    if (my_cross != INT_MAX && my_cross == s_cross) s_pre = my_pre;
    __syncthreads();
    if (tid == 0) {
      const bool crossed = s_cross != INT_MAX;
      double reach = s_cum;                              // the largest partial sum involved
      if (crossed) {
        reach = s_pre;
      } else {
        for (int w = 0; w < kToppThreads / 32; ++w) reach += wtot[w];
      }
      const int small_i = crossed ? s_cross : s_last;    // the smallest term involved
      bool exact = true;
      if (small_i >= 0) {
        int ex = 0;
        const float small = expf(key_bf16((uint32_t)(hi_key - small_i)) - rs.m);
        frexpf(small, &ex);                              // small = f 2^ex, f in [0.5, 1)
        exact = small >= 1.17549435e-38f && reach < ldexp(1.0, 30 + (ex - 1)) * (1.0 - 1e-9);
      }
      if (exact) {
        s_cum = reach;
        if (crossed) {
          s_t = key_bf16((uint32_t)(hi_key - s_cross));
          s_done = 1;
        }
      } else {
        // the rule's own order
        double cum = s_cum;
        for (int i = 0; i < n; ++i) {
          const uint32_t c = cnt[i];
          if (!c) continue;
          cum += term(hi_key, i, c);
          if (cum >= target) {
            s_t = key_bf16((uint32_t)(hi_key - i));
            s_done = 1;
            break;
          }
        }
        s_cum = cum;
      }
    }
    __syncthreads();
    if (s_done) break;
  }
  if (tid == 0) {
    thresh[row] = s_t;                       // -inf: the whole row, when rounding keeps the mass below the target
    mass[row] = (float)s_cum;
  }
}

// The nucleus pass with the walks running alongside it.  CTAs 0 .. walkers-1
// walk request b = blockIdx.x lazily (warp 0 walks, warp 1 expands the nodes
// whose rows are done), as the streaming kernel's walker CTAs do; the other
// CTAs take the rows in the order `order` lists (the row-statistics pass's
// stream order: internal rows by depth-first rank first), compute each row's
// nucleus and raise its flag in `done`, which p.row_done points at.  A walk
// waits only for the rows it descends through, so it ends shortly after its
// last such row instead of after the whole pass.
// Two CTAs per SM (64 registers a thread): the nucleus rows need the warps more
// than the walker CTAs need registers.
__global__ void __launch_bounds__(kToppThreads, 2) topp_walk_kernel(const AcceptParams p, float top_p, float* thresh,
                                                                 float* mass, const int32_t* order, unsigned* done,
                                                                 int walkers) {
  extern __shared__ __align__(128) uint8_t wsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if ((int)blockIdx.x < walkers) {
    if (warp > 1) return;
    const WalkSmem w = walk_smem(wsm, p.max_nodes);
    volatile int* ctl = reinterpret_cast<volatile int*>(wsm + ((walk_smem_bytes(p.max_nodes) + 15) & ~(size_t)15));
    const int b = blockIdx.x;
    if (warp == 0) {
      const int lo = p.row_indptr[b], n = p.row_indptr[b + 1] - lo;
      const bool go = walk_request<true>(p, b, lo, n, w, WarpGroup{}, nullptr);
      if (lane == 0) {
        ctl[0] = go ? b : -2;
        ctl[1] = 0;
      }
      named_barrier(1, 64);
      if (go) walk_traversal_warp<true>(p, b, lo, n, w);
      if (p.compact) compact_request_warp(p, b);
      if (lane == 0) ctl[1] = 1;
    } else {
      named_barrier(1, 64);
      const int bb = ctl[0];
      if (bb >= 0) {
        const int lo = p.row_indptr[bb];
        expand_request(p, lo, p.row_indptr[bb + 1] - lo, w, ctl + 1);
      }
    }
    return;
  }
  const int k = blockIdx.x - walkers;
  const int row = order ? order[k] : k;
  if (order && __ldcg(done + row)) return;     // a leaf row whose nucleus nothing reads (topp_skip_leaves)
  topp_row(p, top_p, thresh, mass, row);
  if (threadIdx.x == 0) {
    __threadfence();
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(done + row), "r"(1u) : "memory");
  }
}

// One CTA per request: replace the bonus token (the last output, present when
// the output is one longer than the accepted node's depth) by a draw from the
// accepted row's distribution.
__global__ void __launch_bounds__(1024) sample_bonus_kernel(const AcceptParams p) {
  __shared__ double seg[1024];
  __shared__ double s_target;
  __shared__ int s_row, s_skip, s_pick;
  const int b = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) {
    const int32_t* c = p.out_counts + (int64_t)b * 4;
    const int n_out = c[0], node = c[3];
    const int lo = p.row_indptr[b];
    int depth = 0;
    for (int u = node; u > 0; u = p.parents[lo + u]) ++depth;
    s_skip = !(n_out > 0 && n_out == depth + 1 && n_out <= p.out_stride);
    s_row = lo + node;
    s_pick = -1;
  }
  __syncthreads();
  if (s_skip) return;
  const int row = s_row;
  const RowStat rs = p.row_ws[row];
  const float t = p.topp_thresh ? p.topp_thresh[row] : -INFINITY;
  const float sn = p.topp_mass ? p.topp_mass[row] : rs.s;
  const uint16_t* rp = p.logits + (int64_t)row * p.row_stride;
  const int per = (p.vocab + 1023) / 1024;
  const int e0 = min(tid * per, p.vocab), e1 = min(e0 + per, p.vocab);
  double local = 0.0;
  for (int e = e0; e < e1; ++e) {
    const float x = load_scaled(p, rp, e);
    if (x >= t) local += (double)prob_bf16(x, rs.m, sn);
  }
  seg[tid] = local;
  __syncthreads();
  if (tid == 0) {
    double total = 0.0;
    for (int i = 0; i < 1024; ++i) {
      const double v = seg[i];
      seg[i] = total;                       // exclusive prefix
      total += v;
    }
    s_target = (double)philox_uniform(p.seed, p.offset, (uint32_t)b, 2u * PTS_MAX_TREE_NODES) * total;
  }
  __syncthreads();
  const double target = s_target;
  if (seg[tid] <= target && target < seg[tid] + local) {
    double cum = seg[tid];
    for (int e = e0; e < e1; ++e) {
      const float x = load_scaled(p, rp, e);
      if (x < t) continue;
      cum += (double)prob_bf16(x, rs.m, sn);
      if (cum > target) {
        atomicMax(&s_pick, e);
        break;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    int pick = s_pick;
    if (pick < 0) {                         // target at the very end: the last token with mass
      for (int e = p.vocab - 1; e >= 0; --e) {
        const float x = load_scaled(p, rp, e);
        if (x >= t && prob_bf16(x, rs.m, sn) > 0.0f) {
          pick = e;
          break;
        }
      }
    }
    if (pick >= 0) p.out_tokens[(int64_t)b * p.out_stride + p.out_counts[(int64_t)b * 4] - 1] = pick;
  }
}

// ---------------------------------------------------------------------------
// fp32 logits (small fp32 models, for example the reference's 2-layer
// configuration): the probabilities stay fp32, as torch's softmax of fp32
// logits does (verification.py:46-55).  One CTA per row computes the max, the
// sum of expf(x - m) (fp64 per thread, combined in thread order) and the
// argmax of the fp32 probabilities: the first index whose probability
// expf(x - m) / s equals the max's 1 / s (values just below the max can round
// to it).  The walks then run from these statistics.
constexpr int kF32Threads = 512;

__global__ void walk_merged_kernel(const AcceptParams p, const int* ties, int shards);

__device__ __forceinline__ float load_f32(const AcceptParams& p, const float* row, int e) {
  const float x = row[e];
  return p.use_temp ? __fmul_rn(x, p.inv_temp) : x;
}

__global__ void __launch_bounds__(kF32Threads) f32_row_stats_kernel(const AcceptParams p) {
  __shared__ float s_max[kF32Threads / 32];
  __shared__ double s_sum[kF32Threads];
  __shared__ int s_first[kF32Threads / 32];
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* rp = p.logits_f32 + (int64_t)row * p.row_stride;
  float m = -INFINITY;
  for (int e = tid; e < p.vocab; e += kF32Threads) m = fmaxf(m, load_f32(p, rp, e));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) s_max[warp] = m;
  __syncthreads();
  m = s_max[0];
  for (int i = 1; i < kF32Threads / 32; ++i) m = fmaxf(m, s_max[i]);
  double acc = 0.0;
  for (int e = tid; e < p.vocab; e += kF32Threads) acc += (double)expf(load_f32(p, rp, e) - m);
  s_sum[tid] = acc;
  __syncthreads();
  __shared__ float s_s;
  if (tid == 0) {
    double t = 0.0;
    for (int i = 0; i < kF32Threads; ++i) t += s_sum[i];
    s_s = (float)t;
  }
  __syncthreads();
  const float sf = s_s;
  const float pmax = __fdiv_rn(1.0f, sf);
  int first = INT_MAX;
  for (int e = tid; e < p.vocab; e += kF32Threads)
    if (__fdiv_rn(expf(load_f32(p, rp, e) - m), sf) == pmax) {
      first = e;
      break;
    }
  first = (int)__reduce_min_sync(0xffffffffu, (unsigned)first);
  if (lane == 0) s_first[warp] = first;
  __syncthreads();
  if (tid == 0) {
    int f = INT_MAX;
    for (int i = 0; i < kF32Threads / 32; ++i) f = min(f, s_first[i]);
    RowStat rs;
    rs.m = m;
    rs.s = sf;
    rs.argmax = f;
    rs.flags = 0;
    p.row_ws[row] = rs;
  }
}

int accept_f32_launch(AcceptParams p, float temperature, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  PTS_CHECK_ARG(p.logits_f32 && p.row_indptr && p.parents && p.tokens, "null input pointer");
  PTS_CHECK_ARG(p.out_tokens && p.out_hidden && p.out_counts && p.out_stride >= 1, "bad outputs");
  PTS_CHECK_ARG(p.batch > 0 && p.num_rows >= p.batch && p.vocab > 0 && p.row_stride >= p.vocab, "bad sizes");
  PTS_CHECK_ARG(p.max_nodes > 0 && temperature > 0.0f, "bad max_nodes or temperature");
  if (p.max_nodes > PTS_MAX_TREE_NODES)
    return set_error(PTS_ERR_CAPACITY, "max_nodes %d above PTS_MAX_TREE_NODES %d", p.max_nodes, PTS_MAX_TREE_NODES);
  size_t opt, orw, orc, oqc, owk;
  const size_t need = ws_layout(p.num_rows, p.vocab, &opt, &orw, &orc, &oqc, &owk);
  if (!workspace || ws_bytes < need) return set_error(PTS_ERR_CAPACITY, "workspace of %zu bytes, need %zu", ws_bytes, need);
  p.row_ws = (RowStat*)((char*)workspace + orw);
  p.use_temp = (temperature != 1.0f);
  p.inv_temp = 1.0f / temperature;
  p.stats_ready = 1;
  f32_row_stats_kernel<<<p.num_rows, kF32Threads, 0, stream>>>(p);
  int rc = launch_status("f32_row_stats_kernel");
  if (rc) return rc;
  const size_t smem = walk_smem_bytes(p.max_nodes);
  if (smem > kMaxDynSmem) return set_error(PTS_ERR_CAPACITY, "walk state of %zu bytes", smem);
  if (int rc = ensure_smem_attr((const void*)walk_merged_kernel, smem)) return rc;
  walk_merged_kernel<<<p.batch, 32, smem, stream>>>(p, nullptr, 0);
  return launch_status("walk_merged_kernel");
}

// ---------------------------------------------------------------------------
// Vocabulary-sharded (tensor-parallel) acceptance.  Each rank holds the logits
// of a vocabulary shard; pts_accept_shard_partials reduces them to per-row
// partials (the persistent streaming kernel in partials mode), the ranks
// all-gather the partials, and every rank then merges them in shard order
// (merge_shards_kernel), resolves rounding ties of the argmax with one more
// all-gather of per-shard first indices (shard_ties_kernel), and walks the
// trees from the merged statistics (walk_merged_kernel), so every rank gets
// the same accepted paths.

__global__ void merge_shards_kernel(const Part* parts, const float* tok_in, int shards, int rows, RowStat* out,
                                    float* tok_out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  Part acc = parts[r];
  float t = tok_in[r];
  for (int k = 1; k < shards; ++k) {
    acc = merge(acc, parts[(int64_t)k * rows + r]);
    t = fmaxf(t, tok_in[(int64_t)k * rows + r]);
  }
  RowStat rs;
  rs.m = acc.m;
  rs.s = (float)acc.s;
  rs.argmax = acc.idx;
  const float qmax = round_to_bf16(__fdiv_rn(1.0f, rs.s));
  // as in finish_row_warp: a value below the max can only take the argmax of
  // the rounded probabilities if the largest bf16 value below the max does
  rs.flags = (acc.m > -INFINITY) && (prob_bf16(prev_bf16(acc.m), acc.m, rs.s) == qmax);
  out[r] = rs;
  tok_out[r] = t;
}

// One warp per row: for rows flagged with a rounding tie, the first index of
// this shard whose rounded probability equals the row's largest one.
__global__ void shard_ties_kernel(const AcceptParams p, const RowStat* rows, int* out_first) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= p.num_rows) return;
  const RowStat rs = rows[warp];
  int best = INT_MAX;
  if (rs.flags & 1) {
    const float qmax = round_to_bf16(__fdiv_rn(1.0f, rs.s));
    const uint16_t* rp = p.logits + (int64_t)warp * p.row_stride;
    for (int e = lane; e < p.vocab; e += 32)
      if (prob_bf16(load_scaled(p, rp, e), rs.m, rs.s) == qmax) {
        best = e + p.vocab_offset;
        break;
      }
    best = (int)__reduce_min_sync(0xffffffffu, (unsigned)best);
  }
  if (lane == 0) out_first[warp] = best;
}

// One warp per request: settle the argmax of tied rows (smallest index over
// all shards), then walk from the merged statistics.
__global__ void walk_merged_kernel(const AcceptParams p, const int* ties, int shards) {
  extern __shared__ __align__(128) uint8_t wsm[];
  const int b = blockIdx.x, lane = threadIdx.x & 31;
  const int lo = p.row_indptr[b], n = p.row_indptr[b + 1] - lo;
  for (int r = lo + lane; shards > 0 && r < lo + n; r += 32) {
    if (p.row_ws[r].flags & 1) {
      int best = INT_MAX;
      for (int k = 0; k < shards; ++k) best = min(best, ties[(int64_t)k * p.num_rows + r]);
      p.row_ws[r].argmax = best;
    }
  }
  __syncwarp();
  walk_request(p, b, lo, n, walk_smem(wsm, p.max_nodes), WarpGroup{}, nullptr);
}

// Traversal with a top-p target and/or a sampled bonus: row statistics first
// (no walks), then the nuclei, then the walks from the finished statistics,
// then the bonus draws.  The nucleus thresholds and masses follow the main
// workspace.
// Top-p region after the main workspace: per row the nucleus threshold and
// mass, the stream order of the statistics pass and the nucleus-done flags.
size_t topp_ws_bytes(int num_rows) { return align_up((size_t)num_rows * 16, 256); }

int accept_traversal_extended(AcceptParams p, float temperature, float top_p, int do_sample, void* workspace,
                              size_t ws_bytes, cudaStream_t stream) {
  size_t opt, orw, orc, oqc, owk;
  const size_t need = ws_layout(p.num_rows, p.vocab, &opt, &orw, &orc, &oqc, &owk);
  const bool topp = top_p < 1.0f;
  if (!workspace || ws_bytes < need + (topp ? topp_ws_bytes(p.num_rows) : 0))
    return set_error(PTS_ERR_CAPACITY, "workspace of %zu bytes, need %zu (top-p adds %zu)", ws_bytes, need,
                     topp_ws_bytes(p.num_rows));
  char* ws = (char*)workspace;
  float* th = (float*)(ws + need);
  float* ms = th + p.num_rows;
  int32_t* order = (int32_t*)(ms + p.num_rows);
  unsigned* done = (unsigned*)(order + p.num_rows);
  AcceptParams stats = p;
  stats.no_walk = 1;
  if (topp) {
    // the streaming pass lists its row order and clears the nucleus flags
    stats.order_out = order;
    stats.order_done = done;
    stats.topp_skip_leaves = do_sample ? 0 : 1;
  }
  bool streamed = false;
  int rc = accept_launch(stats, 1, temperature, workspace, ws_bytes, stream, &streamed);
  if (rc) return rc;
  // the launch above filled in the workspace pointers and the scaling
  AcceptParams q = p;
  q.part_ws = (Part*)(ws + opt);
  q.row_ws = (RowStat*)(ws + orw);
  q.row_ctr = (unsigned*)(ws + orc);
  q.req_ctr = (unsigned*)(ws + oqc);
  q.walk_ctr = (unsigned*)(ws + owk);
  q.row_done = (unsigned*)(ws + owk + 2 * sizeof(unsigned));
  q.traversal = 1;
  q.use_temp = (temperature != 1.0f);
  q.inv_temp = 1.0f / temperature;
  q.stats_ready = 1;
  if (topp) {
    // the nuclei, with the walks following the rows they need as they finish
    if (!streamed) PTS_CUDA_TRY(cudaMemsetAsync(done, 0, (size_t)p.num_rows * sizeof(unsigned), stream));
    q.topp_thresh = th;
    q.topp_mass = ms;
    q.row_done = done;
    q.stats_ready = 0;
    const size_t smem = ((walk_smem_bytes(p.max_nodes) + 15) & ~(size_t)15) + 16;
    if (smem > kMaxDynSmem - 20 * 1024) return set_error(PTS_ERR_CAPACITY, "walk state of %zu bytes", smem);
    if (int rc = ensure_smem_attr((const void*)topp_walk_kernel, smem)) return rc;
    topp_walk_kernel<<<p.batch + p.num_rows, kToppThreads, smem, stream>>>(q, top_p, th, ms,
                                                                           streamed ? order : nullptr, done, p.batch);
    rc = launch_status("topp_walk_kernel");
    if (rc || !do_sample) return rc;
    q.stats_ready = 1;
    sample_bonus_kernel<<<p.batch, 1024, 0, stream>>>(q);
    return launch_status("sample_bonus_kernel");
  }
  const size_t smem = walk_smem_bytes(p.max_nodes);
  if (smem > kMaxDynSmem) return set_error(PTS_ERR_CAPACITY, "walk state of %zu bytes", smem);
  if (int rc = ensure_smem_attr((const void*)walk_merged_kernel, smem)) return rc;
  walk_merged_kernel<<<p.batch, 32, smem, stream>>>(q, nullptr, 0);
  rc = launch_status("walk_merged_kernel");
  if (rc || !do_sample) return rc;
  sample_bonus_kernel<<<p.batch, 1024, 0, stream>>>(q);
  return launch_status("sample_bonus_kernel");
}

}  // namespace
}  // namespace pts

using namespace pts;

extern "C" size_t pts_accept_workspace_size(int num_rows, int vocab) {
  size_t a, b, c, d;
  if (num_rows <= 0 || vocab <= 0) return 0;
  return ws_layout(num_rows, vocab, &a, &b, &c, &d) + topp_ws_bytes(num_rows);
}

namespace pts {
namespace {

// One thread per row: the row's argmax as the last acceptance call on this
// workspace determined it, and the row's node probability Mb = p[parent, token]
// from the same row statistics and the same device arithmetic the walks use.
__global__ void export_row_stats_kernel(AcceptParams p, const RowStat* rows, int32_t* out_argmax, float* out_mb) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= p.num_rows) return;
  out_argmax[r] = rows[r].argmax;
  // the request holding row r: binary search over row_indptr
  int lo = 0, hi = p.batch;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (p.row_indptr[mid] <= r) lo = mid;
    else hi = mid;
  }
  const int base = p.row_indptr[lo];
  const int par = p.parents[r];
  const int tk = p.tokens[r];
  float mb = 1.0f;
  if (par >= 0) {
    const int pr = base + par;
    const float x = (tk < 0 || tk >= p.vocab) ? -INFINITY : load_scaled(p, p.logits + (int64_t)pr * p.row_stride, tk);
    mb = node_mb(p, x, pr, rows[pr].m, rows[pr].s);
  }
  out_mb[r] = mb;
}

}  // namespace
}  // namespace pts

extern "C" int pts_accept_export_row_stats(const void* workspace, size_t workspace_bytes, const uint16_t* logits,
                                           int64_t row_stride, const int32_t* row_indptr, const int32_t* parents,
                                           const int32_t* tokens, int batch, int num_rows, int vocab,
                                           float temperature, int32_t* out_argmax, float* out_mb,
                                           pts_stream_t stream) {
  PTS_CHECK_ARG(workspace && logits && row_indptr && parents && tokens && out_argmax && out_mb, "null pointer");
  PTS_CHECK_ARG(batch > 0 && num_rows >= batch && vocab > 0 && row_stride >= vocab, "bad sizes");
  PTS_CHECK_ARG(temperature > 0.0f, "temperature must be positive");
  size_t opt, orw, orc, oqc;
  const size_t need = ws_layout(num_rows, vocab, &opt, &orw, &orc, &oqc);
  if (workspace_bytes < need) return set_error(PTS_ERR_CAPACITY, "workspace of %zu bytes, need %zu", workspace_bytes,
                                               need);
  AcceptParams p{};
  p.logits = logits;
  p.row_stride = row_stride;
  p.row_indptr = row_indptr;
  p.parents = parents;
  p.tokens = tokens;
  p.batch = batch;
  p.num_rows = num_rows;
  p.vocab = vocab;
  p.use_temp = (temperature != 1.0f);
  p.inv_temp = 1.0f / temperature;
  const RowStat* rows = (const RowStat*)((const uint8_t*)workspace + orw);
  export_row_stats_kernel<<<(num_rows + 255) / 256, 256, 0, (cudaStream_t)stream>>>(p, rows, out_argmax, out_mb);
  return launch_status("export_row_stats_kernel");
}

// The compaction arguments into p (nullptr: none), checked like pts_kv_compact's.
static int set_compact(AcceptParams& p, const pts_kv_compact_args* c) {
  if (!c) return PTS_OK;
  PTS_CHECK_ARG(c->kv_pool && c->page_indptr && c->page_indices && c->offsets, "null compaction pointer");
  PTS_CHECK_ARG(c->elem_bytes == 2 || c->elem_bytes == 4, "elem_bytes must be 2 or 4");
  PTS_CHECK_ARG(c->num_layers > 0 && c->max_pages > 0 && c->page_len > 0 && c->num_kv_heads > 0 && c->head_dim > 0,
                "bad compaction shape");
  PTS_CHECK_ARG((c->head_dim * c->elem_bytes) % 16 == 0, "head_dim * elem_bytes must be a multiple of 16");
  PTS_CHECK_ARG(((uintptr_t)c->kv_pool & 15) == 0, "pool must be 16-byte aligned");
  // The walks copy their request's rows one warp at a time, which pays for
  // pools of a few (layer, K/V, head) rows per token.  Larger pools (many
  // layers) are compacted by the grid-wide compaction kernel right after the
  // acceptance launch, in the same call.
  p.compact = 2 * c->num_layers * c->num_kv_heads <= kFusedCompactMaxRows ? 1 : 0;
  p.cp = *c;
  return PTS_OK;
}

// After a successful acceptance launch: the compaction that set_compact left
// to the grid-wide kernel, if any.
static int finish_compact(int rc, const AcceptParams& p, const pts_kv_compact_args* c, cudaStream_t stream) {
  if (rc != PTS_OK || !c || p.compact) return rc;
  return pts_kv_compact(c->kv_pool, c->num_layers, c->max_pages, c->page_len, c->num_kv_heads, c->head_dim,
                        c->elem_bytes, c->page_indptr, c->page_indices, p.out_hidden, p.out_stride, p.out_counts, 4,
                        c->offsets, p.batch, min(p.out_stride, p.max_nodes), c->new_kv_len, c->new_last_page_len,
                        (pts_stream_t)stream);
}

extern "C" int pts_accept_greedy(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                                 const int32_t* parents, const int32_t* tokens, int batch, int num_rows,
                                 int vocab, int max_nodes, int64_t eos_token_id, int32_t* out_tokens,
                                 int32_t* out_hidden, int32_t* out_counts, int out_stride,
                                 void* workspace, size_t workspace_bytes, pts_stream_t stream) {
  return pts_accept_greedy_compact(logits, row_stride, row_indptr, parents, tokens, batch, num_rows, vocab,
                                   max_nodes, eos_token_id, out_tokens, out_hidden, out_counts, out_stride, workspace,
                                   workspace_bytes, nullptr, stream);
}

extern "C" int pts_accept_greedy_compact(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                                         const int32_t* parents, const int32_t* tokens, int batch, int num_rows,
                                         int vocab, int max_nodes, int64_t eos_token_id, int32_t* out_tokens,
                                         int32_t* out_hidden, int32_t* out_counts, int out_stride,
                                         void* workspace, size_t workspace_bytes,
                                         const pts_kv_compact_args* compact, pts_stream_t stream) {
  AcceptParams p{};
  if (int rc = set_compact(p, compact)) return rc;
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
  // with a compaction the call is a verification step: the greedy walks'
  // rows are reduced on demand (pts_accept_export_row_stats then covers the
  // rows the walks read)
  p.step_form = compact != nullptr;
  return finish_compact(accept_launch(p, 0, 1.0f, workspace, workspace_bytes, (cudaStream_t)stream), p, compact,
                        (cudaStream_t)stream);
}

extern "C" int pts_accept_traversal(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                                    const int32_t* parents, const int32_t* tokens, const float* draft_probs,
                                    int batch, int num_rows, int vocab, int max_nodes, int64_t eos_token_id,
                                    float temperature, float top_p, int do_sample, uint64_t philox_seed,
                                    uint64_t philox_offset, int32_t* out_tokens, int32_t* out_hidden,
                                    int32_t* out_counts, int out_stride, void* workspace,
                                    size_t workspace_bytes, pts_stream_t stream) {
  return pts_accept_traversal_compact(logits, row_stride, row_indptr, parents, tokens, draft_probs, batch, num_rows,
                                      vocab, max_nodes, eos_token_id, temperature, top_p, do_sample, philox_seed,
                                      philox_offset, out_tokens, out_hidden, out_counts, out_stride, workspace,
                                      workspace_bytes, nullptr, stream);
}

extern "C" int pts_accept_traversal_compact(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                                            const int32_t* parents, const int32_t* tokens, const float* draft_probs,
                                            int batch, int num_rows, int vocab, int max_nodes, int64_t eos_token_id,
                                            float temperature, float top_p, int do_sample, uint64_t philox_seed,
                                            uint64_t philox_offset, int32_t* out_tokens, int32_t* out_hidden,
                                            int32_t* out_counts, int out_stride, void* workspace,
                                            size_t workspace_bytes, const pts_kv_compact_args* compact,
                                            pts_stream_t stream) {
  if (!draft_probs) return set_error(PTS_ERR_INVALID, "null draft_probs");
  if (!(top_p > 0.0f && top_p <= 1.0f)) return set_error(PTS_ERR_INVALID, "top_p must be in (0, 1]");
  AcceptParams p{};
  if (int rc = set_compact(p, compact)) return rc;
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
  const int rc = (top_p >= 1.0f && !do_sample)
                     ? accept_launch(p, 1, temperature, workspace, workspace_bytes, (cudaStream_t)stream)
                     : accept_traversal_extended(p, temperature, top_p, do_sample, workspace, workspace_bytes,
                                                 (cudaStream_t)stream);
  return finish_compact(rc, p, compact, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Vocabulary-sharded acceptance (tensor parallelism): C ABI.

extern "C" int pts_accept_shard_partials(const uint16_t* logits_shard, int64_t row_stride, const int32_t* row_indptr,
                                         const int32_t* parents, const int32_t* tokens, int batch, int num_rows,
                                         int shard_vocab, int vocab_offset, float temperature, void* out_partials,
                                         float* out_token_logit, void* workspace, size_t workspace_bytes,
                                         pts_stream_t stream) {
  PTS_CHECK_ARG(out_partials && out_token_logit, "null output pointer");
  PTS_CHECK_ARG(vocab_offset >= 0, "vocab_offset must be non-negative");
  AcceptParams p{};
  p.logits = logits_shard;
  p.row_stride = row_stride;
  p.row_indptr = row_indptr;
  p.parents = parents;
  p.tokens = tokens;
  p.batch = batch;
  p.num_rows = num_rows;
  p.vocab = shard_vocab;
  p.max_nodes = 1;
  p.eos = -1;
  p.parts_out = (Part*)out_partials;
  p.tok_logit_out = out_token_logit;
  p.vocab_offset = vocab_offset;
  return accept_launch(p, 0, temperature, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int pts_accept_merge_shards(const void* partials_all, const float* token_logit_all, int num_shards,
                                       int num_rows, void* out_row_stats, float* out_token_logit,
                                       pts_stream_t stream) {
  PTS_CHECK_ARG(partials_all && token_logit_all && out_row_stats && out_token_logit, "null pointer");
  PTS_CHECK_ARG(num_shards >= 1 && num_rows >= 1, "need num_shards >= 1 and num_rows >= 1");
  merge_shards_kernel<<<(num_rows + 127) / 128, 128, 0, (cudaStream_t)stream>>>(
      (const Part*)partials_all, token_logit_all, num_shards, num_rows, (RowStat*)out_row_stats, out_token_logit);
  return launch_status("merge_shards_kernel");
}

extern "C" int pts_accept_shard_ties(const uint16_t* logits_shard, int64_t row_stride, int num_rows, int shard_vocab,
                                     int vocab_offset, float temperature, const void* row_stats, int32_t* out_first,
                                     pts_stream_t stream) {
  PTS_CHECK_ARG(logits_shard && row_stats && out_first, "null pointer");
  PTS_CHECK_ARG(num_rows >= 1 && shard_vocab >= 1 && row_stride >= shard_vocab, "bad sizes");
  PTS_CHECK_ARG(temperature > 0.0f, "temperature must be positive");
  AcceptParams p{};
  p.logits = logits_shard;
  p.row_stride = row_stride;
  p.num_rows = num_rows;
  p.vocab = shard_vocab;
  p.vocab_offset = vocab_offset;
  p.use_temp = (temperature != 1.0f);
  p.inv_temp = 1.0f / temperature;
  shard_ties_kernel<<<(num_rows + 7) / 8, 256, 0, (cudaStream_t)stream>>>(p, (const RowStat*)row_stats, out_first);
  return launch_status("shard_ties_kernel");
}

extern "C" int pts_accept_walk_merged(void* row_stats, const float* token_logit, const int32_t* ties_all,
                                      int num_shards, const int32_t* row_indptr, const int32_t* parents,
                                      const int32_t* tokens, const float* draft_probs, int batch, int num_rows,
                                      int vocab, int max_nodes, int64_t eos_token_id, uint64_t philox_seed,
                                      uint64_t philox_offset, int32_t* out_tokens, int32_t* out_hidden,
                                      int32_t* out_counts, int out_stride, pts_stream_t stream) {
  PTS_CHECK_ARG(row_stats && token_logit && ties_all && row_indptr && parents && tokens, "null input pointer");
  PTS_CHECK_ARG(out_tokens && out_hidden && out_counts && out_stride >= 1, "bad outputs");
  PTS_CHECK_ARG(batch > 0 && num_rows >= batch && num_shards >= 1 && vocab > 0 && max_nodes > 0, "bad sizes");
  if (max_nodes > PTS_MAX_TREE_NODES)
    return set_error(PTS_ERR_CAPACITY, "max_nodes %d above PTS_MAX_TREE_NODES %d", max_nodes, PTS_MAX_TREE_NODES);
  AcceptParams p{};
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
  p.traversal = draft_probs != nullptr;
  p.seed = philox_seed;
  p.offset = philox_offset;
  p.out_tokens = out_tokens;
  p.out_hidden = out_hidden;
  p.out_counts = out_counts;
  p.row_ws = (RowStat*)row_stats;
  p.tok_logit = token_logit;
  p.stats_ready = 1;
  const size_t smem = walk_smem_bytes(max_nodes);
  if (smem > 232448) return set_error(PTS_ERR_CAPACITY, "walk state of %zu bytes", smem);
  if (int rc = ensure_smem_attr((const void*)walk_merged_kernel, smem)) return rc;
  walk_merged_kernel<<<batch, 32, smem, (cudaStream_t)stream>>>(p, ties_all, num_shards);
  return launch_status("walk_merged_kernel");
}

// ---------------------------------------------------------------------------
// fp32 logits: C ABI.

extern "C" int pts_accept_greedy_f32(const float* logits, int64_t row_stride, const int32_t* row_indptr,
                                     const int32_t* parents, const int32_t* tokens, int batch, int num_rows,
                                     int vocab, int max_nodes, int64_t eos_token_id, int32_t* out_tokens,
                                     int32_t* out_hidden, int32_t* out_counts, int out_stride, void* workspace,
                                     size_t workspace_bytes, pts_stream_t stream) {
  AcceptParams p{};
  p.logits_f32 = logits;
  p.row_stride = row_stride;
  p.row_indptr = row_indptr;
  p.parents = parents;
  p.tokens = tokens;
  p.batch = batch;
  p.num_rows = num_rows;
  p.vocab = vocab;
  p.max_nodes = max_nodes;
  p.out_stride = out_stride;
  p.eos = eos_token_id;
  p.out_tokens = out_tokens;
  p.out_hidden = out_hidden;
  p.out_counts = out_counts;
  return accept_f32_launch(p, 1.0f, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int pts_accept_traversal_f32(const float* logits, int64_t row_stride, const int32_t* row_indptr,
                                        const int32_t* parents, const int32_t* tokens, const float* draft_probs,
                                        int batch, int num_rows, int vocab, int max_nodes, int64_t eos_token_id,
                                        float temperature, uint64_t philox_seed, uint64_t philox_offset,
                                        int32_t* out_tokens, int32_t* out_hidden, int32_t* out_counts,
                                        int out_stride, void* workspace, size_t workspace_bytes,
                                        pts_stream_t stream) {
  if (!draft_probs) return set_error(PTS_ERR_INVALID, "null draft_probs");
  AcceptParams p{};
  p.logits_f32 = logits;
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
  p.traversal = 1;
  p.seed = philox_seed;
  p.offset = philox_offset;
  p.out_tokens = out_tokens;
  p.out_hidden = out_hidden;
  p.out_counts = out_counts;
  return accept_f32_launch(p, temperature, workspace, workspace_bytes, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Traversal acceptance that allocates nothing.
//
// Some callers cannot hand this library a workspace: a host program that only
// receives device pointers from another runtime and has no device allocator
// of its own, or a serving process whose device memory is planned once at
// start-up and may not call cudaMalloc afterwards (cudaMalloc can synchronise
// the device and fragments the planned pool).  For them the scratch that
// pts_accept_traversal takes from the caller lives instead in the fixed
// device array below.  The array exists in every GPU that loads the library
// and stays there until the process exits.
namespace pts {
namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)2 << 20;   // 2 MiB
static __device__ __align__(256) uint8_t g_accept_scratch[kNoAllocScratchBytes];

// The array's name in host code is only a host-side handle; the kernel needs
// the device address, looked up with the device current.  That address
// belongs to the CUDA context the module was loaded into, so the cache is
// keyed on the current context's unique id (cuCtxGetId): a caller that makes
// another context current, or a device reset that recreates the primary
// context, gets a fresh lookup instead of a stale address.
int noalloc_scratch(void** out) {
  struct Entry {
    unsigned long long ctx_id;
    void* addr;
  };
  static std::mutex mu;
  static Entry cache[256] = {};
  int dev = 0;
  PTS_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 256) return set_error(PTS_ERR_UNSUPPORTED, "device ordinal %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  unsigned long long id = 0;
  const bool have_ctx = current_context_id(&id) == PTS_OK;
  if (have_ctx && cache[dev].addr && cache[dev].ctx_id == id) {
    *out = cache[dev].addr;
    return PTS_OK;
  }
  // first call in this context (the lookup also makes the device's primary
  // context current when no context is yet)
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_accept_scratch);
  if (e != cudaSuccess || !p)
    return set_error(PTS_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
  int rc = current_context_id(&id);
  if (rc != PTS_OK) return rc;
  cache[dev].ctx_id = id;
  cache[dev].addr = p;
  *out = p;
  return PTS_OK;
}

}  // namespace
}  // namespace pts

// Same arguments and results as pts_accept_traversal, without the workspace.
// The first call in a CUDA context (per device, and again after the current
// context changes) looks up the scratch array's device address; make that
// first call before capturing the stream into a CUDA graph.  All calls share
// the one array (its counters are cleared at the start of every call), so two
// calls whose kernels overlap on the same GPU (for example on two streams at
// once) race and must be serialised by the caller.  Sizes whose scratch
// exceeds 2 MiB (about 300 bytes per tree row at a 262144-entry vocabulary,
// so about 6900 rows there) are rejected with PTS_ERR_CAPACITY.
extern "C" int pts_accept_traversal_noalloc(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                                            const int32_t* parents, const int32_t* tokens, const float* draft_probs,
                                            int batch, int num_rows, int vocab, int max_nodes, int64_t eos_token_id,
                                            float temperature, float top_p, int do_sample, uint64_t philox_seed,
                                            uint64_t philox_offset, int32_t* out_tokens, int32_t* out_hidden,
                                            int32_t* out_counts, int out_stride, pts_stream_t stream) {
  if (num_rows <= 0 || vocab <= 0) return set_error(PTS_ERR_INVALID, "need num_rows > 0 and vocab > 0");
  // the pointer checks of pts_accept_traversal, here before the scratch lookup touches the device
  PTS_CHECK_ARG(logits && row_indptr && parents && tokens, "null input pointer");
  PTS_CHECK_ARG(draft_probs, "null draft_probs");
  PTS_CHECK_ARG(out_tokens && out_hidden && out_counts, "null output pointer");
  size_t a, b, c, d;
  const size_t need = ws_layout(num_rows, vocab, &a, &b, &c, &d) + topp_ws_bytes(num_rows);
  if (need > kNoAllocScratchBytes)
    return set_error(PTS_ERR_CAPACITY,
                     "pts_accept_traversal_noalloc: %d rows at vocab %d need %zu bytes of scratch, above the fixed %zu",
                     num_rows, vocab, need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != PTS_OK) return rc;
  return pts_accept_traversal(logits, row_stride, row_indptr, parents, tokens, draft_probs, batch, num_rows, vocab,
                              max_nodes, eos_token_id, temperature, top_p, do_sample, philox_seed, philox_offset,
                              out_tokens, out_hidden, out_counts, out_stride, scratch, kNoAllocScratchBytes, stream);
}
