// Sparse page sets per KV head: attention of a long-prefix request restricted
// to a subset of its pages, chosen per KV head.
//
// page_key_sums_kernel   per page and KV head, the fp32 sum of the page's 16
//                        keys (a page summary, computed once when a page is
//                        full and kept beside the cache);
// select_pages_kernel    per (request, KV head): the first n_first and last
//                        n_last full prefix pages, the n_top middle pages of
//                        highest score q . key_sum (q = the root query
//                        averaged over the head's GQA group; ties go to the
//                        earlier page), and every page from the first one
//                        holding a tree token to the end, in position order.
//
// The selection follows the page-importance idea of the reference's sparse
// attention (sparse_attention/pillar.py:83-216: q . k scores aggregated per
// page, top-k pages plus a recent window), which the reference applies to the
// draft's decode with one page set for all heads; here the set is per KV head
// and feeds the verification attention (pts_tree_attn_run_head_pages).  Every
// fp32 operation is explicitly rounded and ordered so that a host restatement
// reproduces the selection exactly.
#include "common.cuh"

namespace pts {
namespace {

constexpr int kSelThreads = 1024;
constexpr int kMaxCandidates = 8192;

__global__ void page_key_sums_kernel(const uint16_t* layer, const int32_t* page_ids, int Hkv, int D, int page_len,
                                     float* out) {
  const int i = blockIdx.x, t4 = threadIdx.x;       // t4: four consecutive (head, dim) entries
  const int per = Hkv * D / 4;
  if (t4 >= per) return;
  const int64_t tok = (int64_t)Hkv * D;             // elements per token
  const uint16_t* k = layer + (int64_t)page_ids[i] * 2 * page_len * tok + (int64_t)t4 * 4;   // K half of the page
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  for (int t = 0; t < page_len; ++t) {
    const uint2 v = *reinterpret_cast<const uint2*>(k + t * tok);
    a0 = __fadd_rn(a0, bf16_bits_to_float(v.x & 0xffffu));
    a1 = __fadd_rn(a1, bf16_bits_to_float(v.x >> 16));
    a2 = __fadd_rn(a2, bf16_bits_to_float(v.y & 0xffffu));
    a3 = __fadd_rn(a3, bf16_bits_to_float(v.y >> 16));
  }
  *reinterpret_cast<float4*>(out + (int64_t)i * Hkv * D + (int64_t)t4 * 4) = make_float4(a0, a1, a2, a3);
}

struct SelParams {
  const float* key_sums;         // [page table entries, Hkv, 128], aligned with page_indices
  const int32_t* page_indptr;    // [B + 1]
  const int32_t* page_indices;
  const int32_t* last_page_len;  // [B]
  const uint16_t* q;             // [T, Hq, 128] bf16
  const int32_t* qo_indptr;      // [B + 1]
  int batch, Hq, Hkv, page_len, n_first, n_top, n_last;
  int max_sort;                  // sort capacity (a power of two, <= kMaxCandidates)
  int32_t* out_indptr;           // [B * Hkv + 1]
  int32_t* out_indices;
  int32_t* out_last;             // [B * Hkv]
};

// Full prefix pages (F) and selected pages per head of request b.
__device__ __forceinline__ void request_counts(const SelParams& p, int b, int& F, int& n_pages, int& count) {
  n_pages = p.page_indptr[b + 1] - p.page_indptr[b];
  const int kv_len = n_pages > 0 ? (n_pages - 1) * p.page_len + p.last_page_len[b] : 0;
  const int prefix = max(0, kv_len - (p.qo_indptr[b + 1] - p.qo_indptr[b]));
  F = min(prefix / p.page_len, n_pages);
  const int keep = F <= p.n_first + p.n_top + p.n_last ? F : p.n_first + p.n_top + p.n_last;
  count = keep + (n_pages - F);
}

__device__ __forceinline__ uint32_t score_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kSelThreads) select_pages_kernel(const SelParams p) {
  __shared__ float qbar[128];
  __shared__ uint32_t chosen[kMaxCandidates / 32];
  extern __shared__ unsigned long long keys[];        // p.max_sort entries
  __shared__ int base_out;
  const int b = blockIdx.x / p.Hkv, h = blockIdx.x % p.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = p.Hq / p.Hkv;
  int F, n_pages, count;
  request_counts(p, b, F, n_pages, count);
  if (tid == 0) {
    int off = 0;
    for (int bb = 0; bb < b; ++bb) {
      int f2, np2, c2;
      request_counts(p, bb, f2, np2, c2);
      off += p.Hkv * c2;
    }
    base_out = off + h * count;
    p.out_indptr[blockIdx.x] = base_out;
    p.out_last[blockIdx.x] = p.last_page_len[b];
    if (blockIdx.x == gridDim.x - 1) p.out_indptr[gridDim.x] = base_out + count;
  }
  // the root query of the head's group, averaged: sum over the group in head
  // order, then one division
  if (tid < 128) {
    const uint16_t* qr = p.q + ((int64_t)p.qo_indptr[b] * p.Hq + (int64_t)h * g) * 128 + tid;
    float s = 0.0f;
    for (int j = 0; j < g; ++j) s = __fadd_rn(s, bf16_bits_to_float(qr[j * 128]));
    qbar[tid] = __fdiv_rn(s, (float)g);
  }
  for (int i = tid; i < kMaxCandidates / 32; i += kSelThreads) chosen[i] = 0u;
  __syncthreads();
  const int pi0 = p.page_indptr[b];
  const int mid0 = p.n_first, mid1 = F - p.n_last;
  const bool sparse = F > p.n_first + p.n_top + p.n_last;
  const int cand = sparse ? min(mid1 - mid0, p.max_sort) : 0;   // the host sizes max_sort for every request
  int M = 1;
  while (M < cand) M <<= 1;
  // scores of the middle pages: one warp per page, lane l covers dims 4l..4l+3
  // (sequential within the lane), then a butterfly sum over the lanes
  for (int i = warp; i < M; i += kSelThreads / 32) {
    unsigned long long key = 0ull;                     // padding sorts last
    if (i < cand) {
      const float4 ks = *reinterpret_cast<const float4*>(
          p.key_sums + ((int64_t)(pi0 + mid0 + i) * p.Hkv + h) * 128 + lane * 4);
      float s = __fmul_rn(qbar[lane * 4 + 0], ks.x);
      s = __fadd_rn(s, __fmul_rn(qbar[lane * 4 + 1], ks.y));
      s = __fadd_rn(s, __fmul_rn(qbar[lane * 4 + 2], ks.z));
      s = __fadd_rn(s, __fmul_rn(qbar[lane * 4 + 3], ks.w));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
      key = ((unsigned long long)score_key(s) << 32) | (0xffffffffu - (uint32_t)i);
    }
    if (lane == 0) keys[i] = key;
  }
  __syncthreads();
  // bitonic sort, descending: higher score first, earlier page first on ties
  for (int k = 2; k <= M; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < M; i += kSelThreads) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long a = keys[i], c = keys[l];
          const bool desc = (i & k) == 0;
          if (desc ? a < c : a > c) {
            keys[i] = c;
            keys[l] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int t = tid; t < min(p.n_top, cand); t += kSelThreads) {
    const int i = (int)(0xffffffffu - (uint32_t)(keys[t] & 0xffffffffull));
    atomicOr(&chosen[i >> 5], 1u << (i & 31));
  }
  __syncthreads();
  if (warp == 0) {
    int32_t* out = p.out_indices + base_out;
    int o = 0;
    if (!sparse) {
      for (int i = lane; i < n_pages; i += 32) out[i] = p.page_indices[pi0 + i];
    } else {
      for (int i = lane; i < p.n_first; i += 32) out[i] = p.page_indices[pi0 + i];
      o = p.n_first;
      for (int w0 = 0; w0 < (cand + 31) / 32; w0 += 32) {
        const int wi = w0 + lane;
        const uint32_t m = wi < (cand + 31) / 32 ? chosen[wi] : 0u;
        const int c = __popc(m);
        int incl = c;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, d);
          if (lane >= d) incl += y;
        }
        int pos = o + incl - c;
        for (uint32_t r = m; r; r &= r - 1) out[pos++] = p.page_indices[pi0 + mid0 + wi * 32 + __ffs(r) - 1];
        o += __shfl_sync(0xffffffffu, incl, 31);
      }
      for (int i = lane; i < n_pages - mid1; i += 32) out[o + i] = p.page_indices[pi0 + mid1 + i];
    }
  }
}

}  // namespace
}  // namespace pts

using namespace pts;

extern "C" int pts_page_key_sums(const void* kv_layer, const int32_t* page_ids, int num_pages, int num_kv_heads,
                                 int head_dim, int page_len, float* out, pts_stream_t stream) {
  PTS_CHECK_ARG(kv_layer && page_ids && out, "null pointer");
  PTS_CHECK_ARG(num_pages >= 0 && num_kv_heads > 0 && head_dim > 0 && page_len > 0, "bad sizes");
  PTS_CHECK_ARG(head_dim % 4 == 0 && num_kv_heads * head_dim / 4 <= 1024, "need head_dim % 4 == 0 and Hkv*D <= 4096");
  PTS_CHECK_ARG(((uintptr_t)kv_layer & 7) == 0 && ((uintptr_t)out & 15) == 0, "kv_layer 8-byte, out 16-byte aligned");
  if (num_pages == 0) return PTS_OK;
  page_key_sums_kernel<<<num_pages, num_kv_heads * head_dim / 4, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)kv_layer, page_ids, num_kv_heads, head_dim, page_len, out);
  return launch_status("page_key_sums_kernel");
}

extern "C" int pts_select_pages(const float* key_sums, const int32_t* page_indptr, const int32_t* page_indices,
                                const int32_t* last_page_len, const void* q, const int32_t* qo_indptr, int batch,
                                int num_qo_heads, int num_kv_heads, int head_dim, int page_len, int n_first,
                                int n_top, int n_last, int max_prefix_pages, int32_t* out_head_indptr,
                                int32_t* out_head_indices, int32_t* out_head_last_page_len, pts_stream_t stream) {
  PTS_CHECK_ARG(key_sums && page_indptr && page_indices && last_page_len && q && qo_indptr, "null input pointer");
  PTS_CHECK_ARG(out_head_indptr && out_head_indices && out_head_last_page_len, "null output pointer");
  PTS_CHECK_ARG(batch > 0 && num_kv_heads > 0 && num_qo_heads % num_kv_heads == 0, "bad head counts");
  PTS_CHECK_ARG(n_first >= 0 && n_top >= 0 && n_last >= 0 && page_len > 0, "bad selection sizes");
  if (head_dim != 128) return set_error(PTS_ERR_UNSUPPORTED, "head_dim %d (this build: 128)", head_dim);
  if (max_prefix_pages > kMaxCandidates)
    return set_error(PTS_ERR_CAPACITY, "%d prefix pages above %d", max_prefix_pages, kMaxCandidates);
  PTS_CHECK_ARG(((uintptr_t)key_sums & 15) == 0, "key_sums must be 16-byte aligned");
  if ((long long)batch * num_kv_heads > 2147483647ll) return set_error(PTS_ERR_CAPACITY, "grid too large");
  SelParams p{};
  p.key_sums = key_sums;
  p.page_indptr = page_indptr;
  p.page_indices = page_indices;
  p.last_page_len = last_page_len;
  p.q = (const uint16_t*)q;
  p.qo_indptr = qo_indptr;
  p.batch = batch;
  p.Hq = num_qo_heads;
  p.Hkv = num_kv_heads;
  p.page_len = page_len;
  p.n_first = n_first;
  p.n_top = n_top;
  p.n_last = n_last;
  p.out_indptr = out_head_indptr;
  p.out_indices = out_head_indices;
  p.out_last = out_head_last_page_len;
  int M = 1;
  while (M < max_prefix_pages) M <<= 1;
  p.max_sort = M;
  const size_t smem = (size_t)M * sizeof(unsigned long long);
  if (smem > 48 * 1024)
    if (int rc = ensure_smem_attr((const void*)select_pages_kernel, smem)) return rc;
  select_pages_kernel<<<batch * num_kv_heads, kSelThreads, smem, (cudaStream_t)stream>>>(p);
  return launch_status("select_pages_kernel");
}
