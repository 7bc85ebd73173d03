// Tree-masked paged attention for the shapes the tensor-core kernel does not
// take: fp32 caches and queries, head_dim other than 128 (a multiple of 32 up
// to 256), other page lengths.  The reference's small fp32 configurations
// (for example a 2-layer model with head_dim 64) run through it.  It is a
// plain SIMT kernel, one warp per (query row, query head): per KV token the
// lanes split the head dimension, a butterfly sums the dot product, and an
// online softmax in fp32 accumulates the output; it is a correctness path
// for small shapes, not a bandwidth path.
//
// Mask semantics are those of tree_attn_kernel: KV slots below kv_len - N
// are the prefix (always visible); slot kv_len - N + j is visible to tree row
// i when bit j of row i's mask is set (j <= i without a mask).
#include "common.cuh"

namespace pts {
namespace {

constexpr int kSimtWarps = 8;            // query rows per CTA

struct SimtParams {
  const void* q;
  const void* kv;
  const int32_t* qo_indptr;
  const int32_t* page_indptr;
  const int32_t* page_indices;
  const int32_t* last_page_len;
  const uint64_t* mask_bits;
  int mask_words;
  void* out;
  int Hq, Hkv, D, page_len, max_pages, head_pages;
  float scale;
};

template <class T>
__device__ __forceinline__ float ld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, int64_t i) {
  return p[i];
}
template <>
__device__ __forceinline__ float ld<uint16_t>(const uint16_t* p, int64_t i) {
  return bf16_bits_to_float(p[i]);
}
template <class T>
__device__ __forceinline__ void st(T* p, int64_t i, float v);
template <>
__device__ __forceinline__ void st<float>(float* p, int64_t i, float v) {
  p[i] = v;
}
template <>
__device__ __forceinline__ void st<uint16_t>(uint16_t* p, int64_t i, float v) {
  p[i] = float_to_bf16_bits(v);
}

template <class T>
__global__ void __launch_bounds__(kSimtWarps * 32) tree_attn_simt_kernel(const SimtParams p) {
  const int hq = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = p.qo_indptr[b], n_nodes = p.qo_indptr[b + 1] - q0;
  const int node = blockIdx.z * kSimtWarps + warp;
  if (node >= n_nodes) return;
  const int g = p.Hq / p.Hkv, h = hq / g;
  const int pt = p.head_pages ? b * p.Hkv + h : b;
  const int p0 = p.page_indptr[pt], n_pages = p.page_indptr[pt + 1] - p0;
  const int kv_len = n_pages > 0 ? (n_pages - 1) * p.page_len + p.last_page_len[pt] : 0;
  const int prefix = kv_len - n_nodes;
  const int per = p.D / 32;                              // dims per lane (<= 8)
  const T* q = (const T*)p.q + ((int64_t)(q0 + node) * p.Hq + hq) * p.D;
  const T* kv = (const T*)p.kv;
  float qv[8], o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    qv[i] = i < per ? ld(q, lane + 32 * i) : 0.0f;
    o[i] = 0.0f;
  }
  const uint64_t* mrow = p.mask_bits ? p.mask_bits + (int64_t)(q0 + node) * p.mask_words : nullptr;
  float m = -INFINITY, l = 0.0f;
  const int64_t tok = (int64_t)p.Hkv * p.D;              // elements per token row
  for (int j = 0; j < kv_len; ++j) {
    bool vis = j < prefix;
    if (!vis) {
      const int t = j - prefix;
      vis = mrow ? ((t >> 6) < p.mask_words && ((mrow[t >> 6] >> (t & 63)) & 1ull)) : (t <= node);
    }
    if (!vis) continue;
    const int pi = j / p.page_len, slot = j % p.page_len;
    const int page = p.page_indices[p0 + pi];
    if (page < 0 || page >= p.max_pages) continue;
    const int64_t kb = ((int64_t)(page * 2) * p.page_len + slot) * tok + (int64_t)h * p.D;
    const int64_t vb = kb + (int64_t)p.page_len * tok;
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < per) s = fmaf(qv[i], ld(kv, kb + lane + 32 * i), s);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    s *= p.scale;
    const float mn = fmaxf(m, s);
    const float alpha = (m == -INFINITY) ? 0.0f : expf(m - mn);
    const float e = expf(s - mn);
    l = l * alpha + e;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < per) o[i] = o[i] * alpha + e * ld(kv, vb + lane + 32 * i);
    m = mn;
  }
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
  T* out = (T*)p.out + ((int64_t)(q0 + node) * p.Hq + hq) * p.D;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < per) st(out, lane + 32 * i, o[i] * inv);
}

}  // namespace

// Launch of the SIMT kernel (called from the attention entry points).
int tree_attn_simt_launch(const void* q, const void* kv_layer, const int32_t* qo_indptr, const int32_t* page_indptr,
                          const int32_t* page_indices, const int32_t* last_page_len, const uint64_t* mask_bits,
                          int mask_words, void* out, int batch, int max_qo_len, int num_qo_heads, int num_kv_heads,
                          int head_dim, int page_len, int max_pages, float sm_scale, int elem_bytes, int head_pages,
                          cudaStream_t stream) {
  if (head_dim % 32 || head_dim > 256)
    return set_error(PTS_ERR_UNSUPPORTED, "head_dim %d (a multiple of 32 up to 256)", head_dim);
  if (elem_bytes != 2 && elem_bytes != 4) return set_error(PTS_ERR_UNSUPPORTED, "element size %d", elem_bytes);
  if (batch > 65535) return set_error(PTS_ERR_CAPACITY, "grid too large");
  SimtParams p{};
  p.q = q;
  p.kv = kv_layer;
  p.qo_indptr = qo_indptr;
  p.page_indptr = page_indptr;
  p.page_indices = page_indices;
  p.last_page_len = last_page_len;
  p.mask_bits = mask_bits;
  p.mask_words = mask_words;
  p.out = out;
  p.Hq = num_qo_heads;
  p.Hkv = num_kv_heads;
  p.D = head_dim;
  p.page_len = page_len;
  p.max_pages = max_pages;
  p.head_pages = head_pages;
  p.scale = sm_scale;
  const int zb = (max_qo_len + kSimtWarps - 1) / kSimtWarps;
  if (zb > 65535) return set_error(PTS_ERR_CAPACITY, "%d query rows per request is too many", max_qo_len);
  dim3 grid(num_qo_heads, batch, zb);
  if (elem_bytes == 4) {
    tree_attn_simt_kernel<float><<<grid, kSimtWarps * 32, 0, stream>>>(p);
  } else {
    tree_attn_simt_kernel<uint16_t><<<grid, kSimtWarps * 32, 0, stream>>>(p);
  }
  return launch_status("tree_attn_simt_kernel");
}

}  // namespace pts
