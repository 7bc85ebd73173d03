// Draft beam search: the per-step candidate selection and the copy-on-write
// page copies of the reference's beam_search (beam_search.py:432-604).
//
// Selection.  The reference scores every (beam, token) pair as
//   cum[beam] + log(bf16(p + 1e-10)),  p = softmax(logits[beam] / T) in bf16
// and keeps the K best of the flattened [beams x vocab] scores (topk), each
// with its p (the new node's probability); the first step keeps the K best
// p of the prompt row.  Here one CTA per beam row takes the row max and the
// fp64 sum of expf(x - m) (rounded to fp32, as the softmax's fp32 sum), then
// scores the row and keeps its best k (score descending, index ascending)
// in per-thread sorted lists merged across the CTA; a second launch merges
// the rows' lists in flat-index order.  p = bf16(expf(x - m) / s), the log
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

// One CTA per beam row: the row's best k candidates, in order, into rows_out[row * k ..].
__global__ void __launch_bounds__(kSelThreads) beam_row_kernel(const void* logits, int64_t row_stride, int elem_bytes,
                                                               int vocab, float inv_t, int scale,
                                                               const float* cum, int k, Cand* rows_out) {
  __shared__ float red_m[kSelThreads / 32];
  __shared__ double red_s[kSelThreads / 32];
  __shared__ float s_m, s_s;
  __shared__ Cand heads[kSelThreads];
  __shared__ int s_winner;
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const char* rp = (const char*)logits + (int64_t)row * row_stride * elem_bytes;
  // row max
  float m = -INFINITY;
  for (int e = tid; e < vocab; e += kSelThreads) m = fmaxf(m, load_logit(rp, e, elem_bytes, inv_t, scale));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red_m[warp] = m;
  __syncthreads();
  if (tid == 0) {
    float mm = red_m[0];
    for (int w = 1; w < kSelThreads / 32; ++w) mm = fmaxf(mm, red_m[w]);
    s_m = mm;
  }
  __syncthreads();
  m = s_m;
  // fp64 sum of the fp32 exponentials, rounded to fp32
  double sum = 0.0;
  for (int e = tid; e < vocab; e += kSelThreads) sum += (double)expf(load_logit(rp, e, elem_bytes, inv_t, scale) - m);
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red_s[warp] = sum;
  __syncthreads();
  if (tid == 0) {
    double ss = 0.0;
    for (int w = 0; w < kSelThreads / 32; ++w) ss += red_s[w];
    s_s = (float)ss;
  }
  __syncthreads();
  const float s = s_s;
  const float c = cum ? cum[row] : 0.0f;
  // this thread's best k, sorted (visited in ascending index, so a later
  // element ties never displace an earlier one)
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
  for (int e = tid; e < vocab; e += kSelThreads) {
    const float x = load_logit(rp, e, elem_bytes, inv_t, scale);
    float p = __fdiv_rn(expf(x - m), s);
    if (elem_bytes == 2) p = round_to_bf16(p);
    float score;
    if (cum) {
      float a = __fadd_rn(p, 1e-10f);
      if (elem_bytes == 2) a = round_to_bf16(a);
      float l = logf(a);
      if (elem_bytes == 2) l = round_to_bf16(l);
      score = __fadd_rn(c, l);
    } else {
      score = p;
    }
    const int idx = row * vocab + e;
    if (!(score > worst)) continue;                     // strictly better than this thread's k-th
    // insert, keeping the list sorted
    float cs = score, cp = p;
    int ci = idx;
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
    // warp best
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
      ((int*)red_s)[2 * warp] = bi;
      ((int*)red_s)[2 * warp + 1] = bt;
    }
    __syncthreads();
    if (tid == 0) {
      float ws = red_m[0];
      int wi = ((int*)red_s)[0], wt = ((int*)red_s)[1];
      for (int w = 1; w < kSelThreads / 32; ++w) {
        const float os = red_m[w];
        const int oi = ((int*)red_s)[2 * w];
        if (before(os, oi, ws, wi)) {
          ws = os;
          wi = oi;
          wt = ((int*)red_s)[2 * w + 1];
        }
      }
      s_winner = wt;
      rows_out[(int64_t)row * k + r] = heads[wt];
    }
    __syncthreads();
    if (tid == s_winner) ++head;
    __syncthreads();
  }
}

// One CTA: merges the rows' sorted lists into the k best overall.
__global__ void __launch_bounds__(32) beam_merge_kernel(const Cand* rows_in, int rows, int k, float* out_score,
                                                        int64_t* out_index, float* out_prob) {
  const int lane = threadIdx.x;
  int head = 0;                                        // lane r < rows follows row r's list
  for (int r = 0; r < k; ++r) {
    float bs = -INFINITY;
    int bi = INT_MAX, bl = lane;
    if (lane < rows && head < k) {
      const Cand c = rows_in[(int64_t)lane * k + head];
      bs = c.score;
      bi = c.idx;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
      if (before(os, oi, bs, bi)) {
        bs = os;
        bi = oi;
        bl = ol;
      }
    }
    if (lane == bl && lane < rows && head < k) {
      const Cand c = rows_in[(int64_t)lane * k + head];
      out_score[r] = c.score;
      out_index[r] = c.idx;
      out_prob[r] = c.prob;
      ++head;
    }
    __syncwarp();
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

extern "C" size_t pts_beam_select_workspace_size(int rows, int k) {
  if (rows <= 0 || k <= 0) return 0;
  return align_up((size_t)rows * k * sizeof(Cand), 256);
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
  if (workspace_bytes < pts_beam_select_workspace_size(rows, k))
    return set_error(PTS_ERR_CAPACITY, "workspace of %zu bytes, need %zu", workspace_bytes,
                     pts_beam_select_workspace_size(rows, k));
  cudaStream_t st = (cudaStream_t)stream;
  const float inv_t = 1.0f / temperature;
  beam_row_kernel<<<rows, kSelThreads, 0, st>>>(logits, row_stride, elem_bytes, vocab, inv_t, temperature != 1.0f,
                                                 cum_log_probs, k, (Cand*)workspace);
  if (int rc = launch_status("beam_row_kernel")) return rc;
  beam_merge_kernel<<<1, 32, 0, st>>>((const Cand*)workspace, rows, k, out_score, out_index, out_prob);
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
