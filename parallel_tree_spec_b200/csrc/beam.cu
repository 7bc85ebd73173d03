// Draft beam search: the per-step candidate selection and the copy-on-write
// page copies of the reference's beam_search (beam_search.py:432-604).
//
// Selection.  The reference scores every (beam, token) pair as
//   cum[beam] + log(bf16(p + 1e-10)),  p = softmax(logits[beam] / T) in bf16
// and keeps the K best of the flattened [beams x vocab] scores (topk), each
// with its p (the new node's probability); the first step keeps the K best
// p of the prompt row.  Each row is cut into slices, one CTA per (slice,
// row), about two CTAs per SM over all rows: one launch takes the slices'
// maxima, one the slices' fp64 sums of expf(x - m) with the row max, one
// scores every slice against the row's (max, sum) -- the sum is the slices'
// sums in slice order, rounded to fp32 -- and keeps the slice's best k (score
// descending, index ascending) in per-thread sorted lists merged across the
// CTA, and one CTA merges all slices' lists.  p = bf16(expf(x - m) / s), the log
// and the sum are bf16-rounded, the add is an fp32 add -- torch's bf16
// arithmetic.
//
// Page copies.  Copy-on-write of a shared partial page copies its first
// `tokens` slots of every layer, keys and values, to a fresh page
// (beam_search.py:92-96); one launch copies every pair of a step.
#include <float.h>
#include <limits.h>

#include "common.cuh"

namespace pts {
namespace {

constexpr int kSelThreads = 256;
constexpr int kMaxSel = 16;            // beams (and picks) per step this build supports

struct Cand {
  float score;
  int idx;                             // flat index row * vocab + token
  float prob;
};

// a ranks before b: higher score, then smaller flat index
__device__ __forceinline__ bool before(float sa, int ia, float sb, int ib) {
  return sa > sb || (sa == sb && ia < ib);
}

__device__ __forceinline__ float load_logit(const void* row, int e, int elem_bytes, float inv_t, bool scale) {
  float x = elem_bytes == 2 ? bf16_bits_to_float(((const uint16_t*)row)[e]) : ((const float*)row)[e];
  if (scale) x = elem_bytes == 2 ? round_to_bf16(__fmul_rn(x, inv_t)) : __fmul_rn(x, inv_t);
  return x;
}

// Block-wide max / fp64 sum of one value per thread (result in every thread).
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = fmaxf(r, red[w]);
  return r;
}

// Each row is split into `chunks` slices, one CTA per (slice, row).
struct Slice {
  int e0, e1;
};
__device__ __forceinline__ Slice slice_of(int vocab, int chunks, int c) {
  const int per = (vocab + chunks - 1) / chunks;
  return Slice{min(c * per, vocab), min(c * per + per, vocab)};
}

// Pass 1: each slice's max.
__global__ void __launch_bounds__(kSelThreads) beam_max_kernel(const void* logits, int64_t row_stride,
                                                               int elem_bytes, int vocab, int chunks, float inv_t,
                                                               int scale, float* part_m) {
  __shared__ float red[kSelThreads / 32];
  const int c = blockIdx.x, row = blockIdx.y;
  const char* rp = (const char*)logits + (int64_t)row * row_stride * elem_bytes;
  const Slice sl = slice_of(vocab, chunks, c);
  float m = -INFINITY;
  for (int e = sl.e0 + threadIdx.x; e < sl.e1; e += kSelThreads)
    m = fmaxf(m, load_logit(rp, e, elem_bytes, inv_t, scale));
  m = block_max(m, red);
  if (threadIdx.x == 0) part_m[row * chunks + c] = m;
}

// Pass 2: each slice's fp64 sum of expf(x - m) with the row max m.
__global__ void __launch_bounds__(kSelThreads) beam_sum_kernel(const void* logits, int64_t row_stride,
                                                               int elem_bytes, int vocab, int chunks, float inv_t,
                                                               int scale, const float* part_m, double* part_s) {
  __shared__ double red[kSelThreads / 32];
  const int c = blockIdx.x, row = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const char* rp = (const char*)logits + (int64_t)row * row_stride * elem_bytes;
  float m = -INFINITY;
  for (int q = 0; q < chunks; ++q) m = fmaxf(m, part_m[row * chunks + q]);
  const Slice sl = slice_of(vocab, chunks, c);
  double sum = 0.0;
  for (int e = sl.e0 + threadIdx.x; e < sl.e1; e += kSelThreads)
    sum += (double)expf(load_logit(rp, e, elem_bytes, inv_t, scale) - m);
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kSelThreads / 32; ++w) t += red[w];
    part_s[row * chunks + c] = t;
  }
}

// Pass 3: each slice's best k candidates, in order, into lists[(row * chunks + c) * k ..].
__global__ void __launch_bounds__(kSelThreads) beam_slice_kernel(const void* logits, int64_t row_stride,
                                                                 int elem_bytes, int vocab, int chunks, float inv_t,
                                                                 int scale, const float* part_m, const double* part_s,
                                                                 const float* cum, int k, Cand* lists) {
  __shared__ float red_m[kSelThreads / 32];
  __shared__ int red_i[2 * (kSelThreads / 32)];
  __shared__ Cand heads[kSelThreads];
  __shared__ int s_winner;
  const int c = blockIdx.x, row = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const char* rp = (const char*)logits + (int64_t)row * row_stride * elem_bytes;
  float m = -INFINITY;
  double ss = 0.0;
  for (int q = 0; q < chunks; ++q) {                   // the row's max and sum, slices in order
    m = fmaxf(m, part_m[row * chunks + q]);
    ss += part_s[row * chunks + q];
  }
  const float s = (float)ss;
  const float cr = cum ? cum[row] : 0.0f;
  const Slice sl = slice_of(vocab, chunks, c);
  // this thread's best k, sorted (visited in ascending index, so a later
  // equal score never displaces an earlier one)
  float ls[kMaxSel];
  int li[kMaxSel];
  float lp[kMaxSel];
#pragma unroll
  for (int q = 0; q < kMaxSel; ++q) {
    ls[q] = -INFINITY;
    li[q] = INT_MAX;
    lp[q] = 0.0f;
  }
  float worst = -INFINITY;                             // ls[k - 1], kept in a register
  for (int e = sl.e0 + tid; e < sl.e1; e += kSelThreads) {
    const float x = load_logit(rp, e, elem_bytes, inv_t, scale);
    float p = __fdiv_rn(expf(x - m), s);
    if (elem_bytes == 2) p = round_to_bf16(p);
    float score;
    if (cum) {
      float a = __fadd_rn(p, 1e-10f);
      if (elem_bytes == 2) a = round_to_bf16(a);
      float l = logf(a);
      if (elem_bytes == 2) l = round_to_bf16(l);
      score = __fadd_rn(cr, l);
    } else {
      score = p;
    }
    if (!(score > worst)) continue;                    // strictly better than this thread's k-th
    float cs = score, cp = p;
    int ci = row * vocab + e;
#pragma unroll
    for (int q = 0; q < kMaxSel; ++q) {
      if (q < k && before(cs, ci, ls[q], li[q])) {
        const float ts = ls[q], tp = lp[q];
        const int ti = li[q];
        ls[q] = cs;
        li[q] = ci;
        lp[q] = cp;
        cs = ts;
        ci = ti;
        cp = tp;
      }
    }
#pragma unroll
    for (int q = 0; q < kMaxSel; ++q)
      if (q == k - 1) worst = ls[q];
  }
  // merge the threads' lists: k rounds of a block-wide best head
  int head = 0;
  for (int r = 0; r < k; ++r) {
    float hs = -INFINITY, hp = 0.0f;
    int hi = INT_MAX;
#pragma unroll
    for (int q = 0; q < kMaxSel; ++q)
      if (q == head) {
        hs = ls[q];
        hi = li[q];
        hp = lp[q];
      }
    heads[tid] = Cand{hs, hi, hp};
    float bs = hs;
    int bi = hi, bt = tid;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int ot = __shfl_xor_sync(0xffffffffu, bt, o);
      if (before(os, oi, bs, bi)) {
        bs = os;
        bi = oi;
        bt = ot;
      }
    }
    if (lane == 0) {
      red_m[warp] = bs;
      red_i[2 * warp] = bi;
      red_i[2 * warp + 1] = bt;
    }
    __syncthreads();
    if (tid == 0) {
      float ws = red_m[0];
      int wi = red_i[0], wt = red_i[1];
      for (int w = 1; w < kSelThreads / 32; ++w)
        if (before(red_m[w], red_i[2 * w], ws, wi)) {
          ws = red_m[w];
          wi = red_i[2 * w];
          wt = red_i[2 * w + 1];
        }
      s_winner = wt;
      lists[((int64_t)row * chunks + c) * k + r] = heads[wt];
    }
    __syncthreads();
    if (tid == s_winner) ++head;
    __syncthreads();
  }
}

// One CTA: merges n_lists sorted lists of k (thread i follows list i) into
// the k best overall.
__global__ void __launch_bounds__(1024) beam_merge_kernel(const Cand* lists, int n_lists, int k, float* out_score,
                                                          int64_t* out_index, float* out_prob) {
  __shared__ float red_m[32];
  __shared__ int red_i[64];
  __shared__ int s_winner;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int head = 0;
  for (int r = 0; r < k; ++r) {
    float bs = -INFINITY;
    int bi = INT_MAX, bt = tid;
    if (tid < n_lists && head < k) {
      const Cand c = lists[(int64_t)tid * k + head];
      bs = c.score;
      bi = c.idx;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int ot = __shfl_xor_sync(0xffffffffu, bt, o);
      if (before(os, oi, bs, bi)) {
        bs = os;
        bi = oi;
        bt = ot;
      }
    }
    if (lane == 0) {
      red_m[warp] = bs;
      red_i[2 * warp] = bi;
      red_i[2 * warp + 1] = bt;
    }
    __syncthreads();
    if (tid == 0) {
      float ws = red_m[0];
      int wi = red_i[0], wt = red_i[1];
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (before(red_m[w], red_i[2 * w], ws, wi)) {
          ws = red_m[w];
          wi = red_i[2 * w];
          wt = red_i[2 * w + 1];
        }
      s_winner = wt;
    }
    __syncthreads();
    if (tid == s_winner && tid < n_lists && head < k) {
      const Cand c = lists[(int64_t)tid * k + head];
      out_score[r] = c.score;
      out_index[r] = c.idx;
      out_prob[r] = c.prob;
      ++head;
    }
    __syncthreads();
  }
}

// Copies the first `tokens` slots of (layer, src page, K and V) to the same
// place of the dst page, one CTA per (pair, layer, K/V), 16-byte vectors.
__global__ void kv_copy_pages_kernel(char* pool, int64_t layer_bytes, int64_t page_bytes, int64_t half_bytes,
                                     const int32_t* src, const int32_t* dst, int max_pages, int64_t bytes) {
  const int pair = blockIdx.x, l = blockIdx.y, kv = blockIdx.z;
  const int sp = src[pair], dp = dst[pair];
  if (sp < 0 || sp >= max_pages || dp < 0 || dp >= max_pages) return;   // pages outside the pool: no copy
  const int64_t base = (int64_t)l * layer_bytes + (int64_t)kv * half_bytes;
  const uint4* s = (const uint4*)(pool + base + (int64_t)sp * page_bytes);
  uint4* d = (uint4*)(pool + base + (int64_t)dp * page_bytes);
  for (int64_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = s[i];
}

}  // namespace
}  // namespace pts

using namespace pts;

namespace pts {
namespace {
// slices per row: about two CTAs per SM of a B200 over all rows, at most 1024 lists to merge
int beam_chunks(int rows) { return max(1, min(1024 / rows, (296 + rows - 1) / rows)); }

struct BeamWs {
  float* part_m;
  double* part_s;
  Cand* lists;
  size_t bytes;
};
BeamWs beam_ws(void* base, int rows, int k) {
  const int n = rows * beam_chunks(rows);
  char* b = (char*)base;
  BeamWs w;
  const size_t om = 0, os = align_up(om + (size_t)n * sizeof(float), 256),
               ol = align_up(os + (size_t)n * sizeof(double), 256);
  w.part_m = (float*)(b + om);
  w.part_s = (double*)(b + os);
  w.lists = (Cand*)(b + ol);
  w.bytes = align_up(ol + (size_t)n * k * sizeof(Cand), 256);
  return w;
}
}  // namespace
}  // namespace pts

extern "C" size_t pts_beam_select_workspace_size(int rows, int k) {
  if (rows <= 0 || k <= 0) return 0;
  return beam_ws(nullptr, rows, k).bytes;
}

extern "C" int pts_beam_select(const void* logits, int64_t row_stride, int elem_bytes, int rows, int vocab,
                               float temperature, const float* cum_log_probs, int k, float* out_score,
                               int64_t* out_index, float* out_prob, void* workspace, size_t workspace_bytes,
                               pts_stream_t stream) {
  PTS_CHECK_ARG(logits && out_score && out_index && out_prob && workspace, "null pointer");
  PTS_CHECK_ARG(rows > 0 && vocab > 0 && k > 0 && row_stride >= vocab, "bad sizes");
  PTS_CHECK_ARG(elem_bytes == 2 || elem_bytes == 4, "elem_bytes must be 2 (bf16) or 4 (fp32)");
  PTS_CHECK_ARG(temperature > 0.0f, "temperature must be positive");
  PTS_CHECK_ARG(k <= rows * vocab, "k above the number of candidates");
  if (k > kMaxSel || rows > 32) return set_error(PTS_ERR_UNSUPPORTED, "beam width %d / %d rows (this build: 16 / 32)", k, rows);
  if ((int64_t)rows * vocab > INT_MAX) return set_error(PTS_ERR_CAPACITY, "rows x vocab above 2^31");
  const BeamWs w = beam_ws(workspace, rows, k);
  if (workspace_bytes < w.bytes)
    return set_error(PTS_ERR_CAPACITY, "workspace of %zu bytes, need %zu", workspace_bytes, w.bytes);
  cudaStream_t st = (cudaStream_t)stream;
  const float inv_t = 1.0f / temperature;
  const int scale = temperature != 1.0f;
  const int chunks = beam_chunks(rows);
  const dim3 grid(chunks, rows);
  beam_max_kernel<<<grid, kSelThreads, 0, st>>>(logits, row_stride, elem_bytes, vocab, chunks, inv_t, scale, w.part_m);
  if (int rc = launch_status("beam_max_kernel")) return rc;
  beam_sum_kernel<<<grid, kSelThreads, 0, st>>>(logits, row_stride, elem_bytes, vocab, chunks, inv_t, scale, w.part_m,
                                                 w.part_s);
  if (int rc = launch_status("beam_sum_kernel")) return rc;
  beam_slice_kernel<<<grid, kSelThreads, 0, st>>>(logits, row_stride, elem_bytes, vocab, chunks, inv_t, scale,
                                                   w.part_m, w.part_s, cum_log_probs, k, w.lists);
  if (int rc = launch_status("beam_slice_kernel")) return rc;
  beam_merge_kernel<<<1, 1024, 0, st>>>(w.lists, rows * chunks, k, out_score, out_index, out_prob);
  return launch_status("beam_merge_kernel");
}

extern "C" int pts_kv_copy_pages(void* kv_pool, int num_layers, int max_pages, int page_len, int row_bytes,
                                 const int32_t* src_pages, const int32_t* dst_pages, int num_pairs, int tokens,
                                 pts_stream_t stream) {
  PTS_CHECK_ARG(kv_pool && src_pages && dst_pages, "null pointer");
  PTS_CHECK_ARG(num_layers > 0 && max_pages > 0 && page_len > 0 && row_bytes > 0 && num_pairs >= 0, "bad sizes");
  PTS_CHECK_ARG(tokens >= 0 && tokens <= page_len, "tokens %d outside [0, page_len %d]", tokens, page_len);
  PTS_CHECK_ARG(row_bytes % 16 == 0 && ((uintptr_t)kv_pool & 15) == 0, "rows must be whole 16-byte vectors");
  if (num_pairs == 0 || tokens == 0) return PTS_OK;
  if (num_layers > 65535) return set_error(PTS_ERR_CAPACITY, "too many layers");
  const int64_t half = (int64_t)page_len * row_bytes, page = 2 * half, layer = (int64_t)max_pages * page;
  dim3 grid(num_pairs, num_layers, 2);
  kv_copy_pages_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>((char*)kv_pool, layer, page, half, src_pages,
                                                               dst_pages, max_pages, (int64_t)tokens * row_bytes);
  return launch_status("kv_copy_pages_kernel");
}
