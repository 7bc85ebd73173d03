// Paged-KV kernels: batch positions, append, compaction; tree mask packing.
//
// All of these are byte movers bounded by HBM bandwidth: 16-byte vector
// accesses, one CTA per (token) or (request, layer, K|V, head) slice, page
// slots resolved through the request's page table.
#include <cuda_bf16.h>

#include "common.cuh"

namespace pts {
namespace {

// ------------------------------------------------------------ batch positions
__global__ void batch_positions_kernel(const int32_t* __restrict__ append_indptr,
                                       const int32_t* __restrict__ seq_lens, int batch, int num_tokens,
                                       int32_t* __restrict__ batch_indices, int32_t* __restrict__ positions) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= num_tokens) return;
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (append_indptr[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  const int n = append_indptr[lo + 1] - append_indptr[lo];
  batch_indices[t] = lo;
  positions[t] = seq_lens[lo] - n + (t - append_indptr[lo]);
}

// ----------------------------------------------------------------- KV append
// grid.x = tokens; each thread moves 16-byte vectors of one token's K and V.
__global__ void kv_append_kernel(const char* __restrict__ k, const char* __restrict__ v, int64_t k_stride_b,
                                 int64_t v_stride_b, char* __restrict__ layer,
                                 const int32_t* __restrict__ batch_indices, const int32_t* __restrict__ positions,
                                 const int32_t* __restrict__ page_indptr, const int32_t* __restrict__ page_indices,
                                 int row_bytes, int page_len, int max_pages) {
  const int t = blockIdx.x;
  const int b = batch_indices[t];
  const int pos = positions[t];
  const int lo = page_indptr[b], hi = page_indptr[b + 1];
  const int pi = pos / page_len;
  if (pos < 0 || lo + pi >= hi) return;
  const int page = page_indices[lo + pi];
  if (page < 0 || page >= max_pages) return;
  const int slot = pos % page_len;
  char* kd = layer + ((int64_t)(page * 2 + 0) * page_len + slot) * row_bytes;
  char* vd = layer + ((int64_t)(page * 2 + 1) * page_len + slot) * row_bytes;
  const char* ks = k + (int64_t)t * k_stride_b;
  const char* vs = v + (int64_t)t * v_stride_b;
  for (int o = threadIdx.x * 16; o < row_bytes; o += blockDim.x * 16) {
    *(uint4*)(kd + o) = *(const uint4*)(ks + o);
    *(uint4*)(vd + o) = *(const uint4*)(vs + o);
  }
}

// ------------------------------------------------------------- KV compaction
// One CTA per (request, layer * 2 + kv, head).  All source rows of the slice
// are staged in shared memory before any destination row is written, which
// gives index_select-then-index_copy semantics for overlapping slots
// (cache_manager.py:133-134).
__global__ void kv_compact_kernel(char* __restrict__ pool, int64_t layer_bytes, int max_pages, int page_len,
                                  int heads, int head_bytes, const int32_t* __restrict__ page_indptr,
                                  const int32_t* __restrict__ page_indices, const int32_t* __restrict__ accepted,
                                  int acc_stride, const int32_t* __restrict__ acc_counts, int counts_stride,
                                  int max_accepted, const int32_t* __restrict__ offsets) {
  extern __shared__ uint4 stage[];
  const int b = blockIdx.z;
  const int lkv = blockIdx.y;           // layer * 2 + kv
  const int h = blockIdx.x;
  const int layer = lkv >> 1, kv = lkv & 1;
  const int32_t* acc = accepted + (int64_t)b * acc_stride;
  const int na = min(max(acc_counts[(int64_t)b * counts_stride], 0), max_accepted);
  const int p0 = page_indptr[b], np = page_indptr[b + 1] - p0;
  const int off = offsets[b];
  const int vec = head_bytes / 16;
  const int64_t row_bytes = (int64_t)heads * head_bytes;
  char* lbase = pool + layer * layer_bytes;
  auto slot_ptr = [&](int s) -> char* {
    const int pi = s / page_len;
    if (s < 0 || pi >= np) return nullptr;
    const int page = page_indices[p0 + pi];
    if (page < 0 || page >= max_pages) return nullptr;
    return lbase + ((int64_t)(page * 2 + kv) * page_len + s % page_len) * row_bytes + (int64_t)h * head_bytes;
  };
  for (int e = threadIdx.x; e < na * vec; e += blockDim.x) {
    const int i = e / vec, j = e % vec;
    const int src = acc[i];
    const char* sp = (src == i) ? nullptr : slot_ptr(off + src);
    if (sp) stage[e] = ((const uint4*)sp)[j];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < na * vec; e += blockDim.x) {
    const int i = e / vec, j = e % vec;
    const int src = acc[i];
    if (src == i) continue;
    char* sp = slot_ptr(off + src);
    char* dp = slot_ptr(off + i);
    if (sp && dp) ((uint4*)dp)[j] = stage[e];
  }
}

__global__ void kv_compact_lengths_kernel(const int32_t* __restrict__ acc_counts, int counts_stride, int max_accepted,
                                          const int32_t* __restrict__ offsets, int batch, int page_len,
                                          int32_t* new_kv_len, int32_t* new_last) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int len = offsets[b] + min(max(acc_counts[(int64_t)b * counts_stride], 0), max_accepted);
  if (new_kv_len) new_kv_len[b] = len;
  if (new_last) new_last[b] = len == 0 ? 0 : (len - 1) % page_len + 1;
}

// ------------------------------------------------------------- tree masks
// One thread per row: OR of the bits of the node and all its ancestors.
__global__ void mask_from_parents_kernel(const int32_t* __restrict__ parents, const int32_t* __restrict__ qo_indptr,
                                         int batch, int total_q, int words, uint64_t* __restrict__ bits) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= total_q) return;
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (qo_indptr[mid] <= r) lo = mid;
    else hi = mid - 1;
  }
  const int base = qo_indptr[lo];
  uint64_t* out = bits + (int64_t)r * words;
  for (int w = 0; w < words; ++w) out[w] = 0ull;
  int node = r - base;
  for (int guard = 0; node >= 0 && guard <= PTS_MAX_TREE_NODES; ++guard) {
    if (node / 64 < words) out[node / 64] |= 1ull << (node % 64);
    const int p = parents[base + node];
    node = (p >= 0 && p < node) ? p : -1;
  }
}

// One CTA per request: the tree's parents staged in shared memory, then per
// row the ancestor bitmask (each word from one walk up the chain) and, when
// asked, the append batch index and position of the row's token.
__global__ void tree_prepare_kernel(const int32_t* __restrict__ parents, const int32_t* __restrict__ qo_indptr,
                                    const int32_t* __restrict__ seq_lens, int words, uint64_t* __restrict__ bits,
                                    int32_t* __restrict__ batch_indices, int32_t* __restrict__ positions) {
  __shared__ int16_t sp[PTS_MAX_TREE_NODES];
  const int b = blockIdx.x;
  const int base = qo_indptr[b], n = qo_indptr[b + 1] - base;
  const bool staged = n <= PTS_MAX_TREE_NODES;
  if (staged)
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int p = parents[base + i];
      sp[i] = (int16_t)((p >= 0 && p < i) ? p : -1);
    }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    uint64_t* out = bits + (int64_t)(base + i) * words;
    for (int w = 0; w < words; ++w) {
      uint64_t acc = 0ull;
      int node = i;
      for (int guard = 0; node >= 0 && guard <= PTS_MAX_TREE_NODES; ++guard) {
        if ((node >> 6) == w) acc |= 1ull << (node & 63);
        int p;
        if (staged) {
          p = sp[node];
        } else {
          p = parents[base + node];
          p = (p >= 0 && p < node) ? p : -1;
        }
        node = p;
      }
      out[w] = acc;
    }
    if (positions) {
      batch_indices[base + i] = b;
      positions[base + i] = seq_lens[b] - n + i;
    }
  }
}

// Tree preparation and KV append in one launch: CTAs 0 .. batch-1 are
// tree_prepare_kernel (masks, batch indices, positions); CTA batch + t appends
// token t, whose request and position it derives itself (the same
// seq_lens[b] - n_b + i as the positions), so the two halves do not wait on
// each other.
constexpr int kPrepSmemIndptr = 1024;    // requests whose qo_indptr the append CTAs stage in shared memory

// Rotary position embedding applied by the append (pts_tree_prepare_append_rope).
struct RopeArgs {
  const char* q;             // [T, Hq, D] at q_stride bytes per token
  int64_t q_stride;
  char* q_out;               // [T, Hq, D] contiguous
  int hq;
  const char* cos;           // [T, D] at cs_stride bytes per token (the model's position embeddings)
  const char* sin;
  int64_t cs_stride;
  int head_dim;
};

__device__ __forceinline__ float bf16_at(const uint4& v, int e) {
  const uint32_t w = (&v.x)[e >> 1];
  return __uint_as_float((e & 1) ? (w & 0xffff0000u) : (w << 16));
}
__device__ __forceinline__ float round_bf16f(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One 16-byte piece (elements i0 .. i0 + 16/elem - 1) of a rotated head row,
// x * cos + rotate_half(x) * sin with rotate_half(x) = cat(-x[D/2:], x[:D/2])
// (apply_rotary_pos_emb of the reference's model, attention.py:83).  Each
// product and the sum are rounded to the element type, as torch's eager
// elementwise operations round them.
template <int kElem>
__device__ __forceinline__ uint4 rope_piece(const char* x_row, const char* c_row, const char* s_row, int D, int i0) {
  const int half = D / 2;
  const int j0 = i0 < half ? i0 + half : i0 - half;
  const float sign = i0 < half ? -1.0f : 1.0f;
  const uint4 xv = *(const uint4*)(x_row + i0 * kElem), pv = *(const uint4*)(x_row + j0 * kElem);
  const uint4 cv = *(const uint4*)(c_row + i0 * kElem), sv = *(const uint4*)(s_row + i0 * kElem);
  uint4 o;
  if (kElem == 2) {
    uint32_t* ow = &o.x;
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      float r[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float p1 = round_bf16f(__fmul_rn(bf16_at(xv, e + h), bf16_at(cv, e + h)));
        const float p2 = round_bf16f(__fmul_rn(sign * bf16_at(pv, e + h), bf16_at(sv, e + h)));
        r[h] = __fadd_rn(p1, p2);
      }
      const __nv_bfloat162 b = __floats2bfloat162_rn(r[0], r[1]);
      ow[e >> 1] = *reinterpret_cast<const uint32_t*>(&b);
    }
  } else {
    const float* x = (const float*)&xv; const float* pp = (const float*)&pv;
    const float* c = (const float*)&cv; const float* sn = (const float*)&sv;
    float* of = (float*)&o;
#pragma unroll
    for (int e = 0; e < 4; ++e) of[e] = __fadd_rn(__fmul_rn(x[e], c[e]), __fmul_rn(sign * pp[e], sn[e]));
  }
  return o;
}

template <bool kRope, int kElem>
__global__ void tree_prepare_append_kernel(const int32_t* __restrict__ parents, const int32_t* __restrict__ qo_indptr,
                                           const int32_t* __restrict__ seq_lens, int batch, int words,
                                           uint64_t* __restrict__ bits, int32_t* __restrict__ batch_indices,
                                           int32_t* __restrict__ positions, const char* __restrict__ k,
                                           const char* __restrict__ v, int64_t k_stride_b, int64_t v_stride_b,
                                           char* __restrict__ layer, const int32_t* __restrict__ page_indptr,
                                           const int32_t* __restrict__ page_indices, int row_bytes, int page_len,
                                           int max_pages, RopeArgs rope) {
  __shared__ int16_t sp[PTS_MAX_TREE_NODES];
  __shared__ int32_t sq[kPrepSmemIndptr + 1];
  pdl_trigger();                                       // the attention launch may get its SMs ready
  pdl_wait();                                          // the previous step's writes (compaction) are done
  if ((int)blockIdx.x < batch) {
    const int b = blockIdx.x;
    const int base = qo_indptr[b], n = qo_indptr[b + 1] - base;
    const bool staged = n <= PTS_MAX_TREE_NODES;
    if (staged)
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int p = parents[base + i];
        sp[i] = (int16_t)((p >= 0 && p < i) ? p : -1);
      }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      uint64_t* out = bits + (int64_t)(base + i) * words;
      for (int w = 0; w < words; ++w) {
        uint64_t acc = 0ull;
        int node = i;
        for (int guard = 0; node >= 0 && guard <= PTS_MAX_TREE_NODES; ++guard) {
          if ((node >> 6) == w) acc |= 1ull << (node & 63);
          int p;
          if (staged) {
            p = sp[node];
          } else {
            p = parents[base + node];
            p = (p >= 0 && p < node) ? p : -1;
          }
          node = p;
        }
        out[w] = acc;
      }
      batch_indices[base + i] = b;
      positions[base + i] = seq_lens[b] - n + i;
    }
    return;
  }
  const int t = blockIdx.x - batch;
  const bool in_smem = batch <= kPrepSmemIndptr;
  if (in_smem)
    for (int i = threadIdx.x; i <= batch; i += blockDim.x) sq[i] = qo_indptr[i];
  __syncthreads();
  const int32_t* qi = in_smem ? sq : qo_indptr;
  int lo = 0, hi = batch - 1;                          // the last request whose first row is <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (qi[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  const int b = lo;
  if (t < qi[b] || t >= qi[b + 1]) return;
  const int pos = seq_lens[b] - (qi[b + 1] - qi[b]) + (t - qi[b]);
  const int p0 = page_indptr[b], p1 = page_indptr[b + 1];
  const int pi = pos / page_len;
  if (pos < 0 || p0 + pi >= p1) return;
  const int page = page_indices[p0 + pi];
  if (page < 0 || page >= max_pages) return;
  const int slot = pos % page_len;
  char* kd = layer + ((int64_t)(page * 2 + 0) * page_len + slot) * row_bytes;
  char* vd = layer + ((int64_t)(page * 2 + 1) * page_len + slot) * row_bytes;
  const char* ks = k + (int64_t)t * k_stride_b;
  const char* vs = v + (int64_t)t * v_stride_b;
  if (!kRope) {
    for (int o = threadIdx.x * 16; o < row_bytes; o += blockDim.x * 16) {
      *(uint4*)(kd + o) = *(const uint4*)(ks + o);
      *(uint4*)(vd + o) = *(const uint4*)(vs + o);
    }
    return;
  }
  // K rotated into the cache, V copied, Q rotated into q_out
  const int D = rope.head_dim, per_head = D * kElem / 16;
  const char* cr = rope.cos + (int64_t)t * rope.cs_stride;
  const char* sr = rope.sin + (int64_t)t * rope.cs_stride;
  const int hkv = row_bytes / (D * kElem);
  for (int pc = threadIdx.x; pc < hkv * per_head; pc += blockDim.x) {
    const int h = pc / per_head, i0 = (pc % per_head) * (16 / kElem);
    const int64_t o = (int64_t)h * D * kElem + i0 * kElem;
    *(uint4*)(kd + o) = rope_piece<kElem>(ks + (int64_t)h * D * kElem, cr, sr, D, i0);
    *(uint4*)(vd + o) = *(const uint4*)(vs + o);
  }
  const char* qs = rope.q + (int64_t)t * rope.q_stride;
  char* qd = rope.q_out + (int64_t)t * rope.hq * D * kElem;
  for (int pc = threadIdx.x; pc < rope.hq * per_head; pc += blockDim.x) {
    const int h = pc / per_head, i0 = (pc % per_head) * (16 / kElem);
    *(uint4*)(qd + (int64_t)h * D * kElem + i0 * kElem) = rope_piece<kElem>(qs + (int64_t)h * D * kElem, cr, sr, D, i0);
  }
}

// pts_kv_append with the rotary embedding: token t's k rotated into its
// slot, v copied, q rotated into q_out.
template <int kElem>
__global__ void kv_append_rope_kernel(const char* __restrict__ k, const char* __restrict__ v, int64_t k_stride_b,
                                      int64_t v_stride_b, char* __restrict__ layer,
                                      const int32_t* __restrict__ batch_indices,
                                      const int32_t* __restrict__ positions, const int32_t* __restrict__ page_indptr,
                                      const int32_t* __restrict__ page_indices, int row_bytes, int page_len,
                                      int max_pages, RopeArgs rope) {
  const int t = blockIdx.x;
  const int D = rope.head_dim, per_head = D * kElem / 16;
  const char* cr = rope.cos + (int64_t)t * rope.cs_stride;
  const char* sr = rope.sin + (int64_t)t * rope.cs_stride;
  const char* qs = rope.q + (int64_t)t * rope.q_stride;
  char* qd = rope.q_out + (int64_t)t * rope.hq * D * kElem;
  for (int pc = threadIdx.x; pc < rope.hq * per_head; pc += blockDim.x) {
    const int h = pc / per_head, i0 = (pc % per_head) * (16 / kElem);
    *(uint4*)(qd + (int64_t)h * D * kElem + i0 * kElem) = rope_piece<kElem>(qs + (int64_t)h * D * kElem, cr, sr, D, i0);
  }
  const int b = batch_indices[t];
  const int pos = positions[t];
  const int lo = page_indptr[b], hi = page_indptr[b + 1];
  const int pi = pos / page_len;
  if (pos < 0 || lo + pi >= hi) return;
  const int page = page_indices[lo + pi];
  if (page < 0 || page >= max_pages) return;
  const int slot = pos % page_len;
  char* kd = layer + ((int64_t)(page * 2 + 0) * page_len + slot) * row_bytes;
  char* vd = layer + ((int64_t)(page * 2 + 1) * page_len + slot) * row_bytes;
  const char* ks = k + (int64_t)t * k_stride_b;
  const char* vs = v + (int64_t)t * v_stride_b;
  const int hkv = row_bytes / (D * kElem);
  for (int pc = threadIdx.x; pc < hkv * per_head; pc += blockDim.x) {
    const int h = pc / per_head, i0 = (pc % per_head) * (16 / kElem);
    const int64_t o = (int64_t)h * D * kElem + i0 * kElem;
    *(uint4*)(kd + o) = rope_piece<kElem>(ks + (int64_t)h * D * kElem, cr, sr, D, i0);
    *(uint4*)(vd + o) = *(const uint4*)(vs + o);
  }
}

// One warp per row of the flattened boolean custom mask.
__global__ void mask_from_bool_kernel(const uint8_t* __restrict__ mask, const int32_t* __restrict__ qo_indptr,
                                      const int32_t* __restrict__ mask_indptr, const int32_t* __restrict__ kv_lens,
                                      int batch, int total_q, int words, uint64_t* __restrict__ bits,
                                      int32_t* bad_rows) {
  const int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= total_q) return;
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (qo_indptr[mid] <= r) lo = mid;
    else hi = mid - 1;
  }
  const int n = qo_indptr[lo + 1] - qo_indptr[lo];
  const int kvl = kv_lens[lo];
  const int prefix = kvl - n;
  const uint8_t* row = mask + mask_indptr[lo] + (int64_t)(r - qo_indptr[lo]) * kvl;
  int bad = 0;
  for (int j = lane; j < prefix; j += 32) bad |= (row[j] == 0);
  bad = __any_sync(0xffffffffu, bad);
  uint64_t* out = bits + (int64_t)r * words;
  for (int w = 0; w < words; ++w) {
    uint32_t lo32 = 0, hi32 = 0;
    for (int half = 0; half < 2; ++half) {
      const int j = w * 64 + half * 32 + lane;
      const bool on = j < n && row[prefix + j] != 0;
      const uint32_t m = __ballot_sync(0xffffffffu, on);
      if (half == 0) lo32 = m;
      else hi32 = m;
    }
    if (lane == 0) out[w] = (uint64_t)lo32 | ((uint64_t)hi32 << 32);
  }
  if (lane == 0 && bad && bad_rows) atomicAdd(bad_rows, 1);
}

}  // namespace
}  // namespace pts

using namespace pts;

extern "C" int pts_batch_positions(const int32_t* append_indptr, const int32_t* seq_lens, int batch,
                                   int num_tokens, int32_t* batch_indices, int32_t* positions,
                                   pts_stream_t stream) {
  PTS_CHECK_ARG(append_indptr && seq_lens && batch_indices && positions, "null pointer");
  PTS_CHECK_ARG(batch > 0 && num_tokens >= 0, "bad batch/num_tokens");
  if (num_tokens == 0) return PTS_OK;
  batch_positions_kernel<<<(num_tokens + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
      append_indptr, seq_lens, batch, num_tokens, batch_indices, positions);
  return launch_status("batch_positions_kernel");
}

extern "C" int pts_kv_append(const void* k, const void* v, int64_t k_token_stride, int64_t v_token_stride,
                             void* kv_layer, const int32_t* batch_indices, const int32_t* positions,
                             const int32_t* page_indptr, const int32_t* page_indices, int num_tokens,
                             int num_kv_heads, int head_dim, int page_len, int max_pages, int elem_bytes,
                             pts_stream_t stream) {
  PTS_CHECK_ARG(k && v && kv_layer && batch_indices && positions && page_indptr && page_indices, "null pointer");
  PTS_CHECK_ARG(elem_bytes == 2 || elem_bytes == 4, "elem_bytes must be 2 or 4");
  PTS_CHECK_ARG(num_kv_heads > 0 && head_dim > 0 && page_len > 0 && max_pages > 0, "bad shape");
  const int row_bytes = num_kv_heads * head_dim * elem_bytes;
  PTS_CHECK_ARG(row_bytes % 16 == 0, "Hkv * D * elem_bytes must be a multiple of 16");
  PTS_CHECK_ARG((k_token_stride * elem_bytes) % 16 == 0 && (v_token_stride * elem_bytes) % 16 == 0,
                "token strides must be multiples of 16 bytes");
  PTS_CHECK_ARG((((uintptr_t)k | (uintptr_t)v | (uintptr_t)kv_layer) & 15) == 0, "pointers must be 16-byte aligned");
  if (num_tokens <= 0) return PTS_OK;
  int threads = row_bytes / 16;
  threads = threads > 256 ? 256 : (threads < 32 ? 32 : threads);
  kv_append_kernel<<<num_tokens, threads, 0, (cudaStream_t)stream>>>(
      (const char*)k, (const char*)v, k_token_stride * elem_bytes, v_token_stride * elem_bytes, (char*)kv_layer,
      batch_indices, positions, page_indptr, page_indices, row_bytes, page_len, max_pages);
  return launch_status("kv_append_kernel");
}

extern "C" int pts_kv_compact(void* kv_pool, int num_layers, int max_pages, int page_len, int num_kv_heads,
                              int head_dim, int elem_bytes, const int32_t* page_indptr,
                              const int32_t* page_indices, const int32_t* accepted, int accepted_stride,
                              const int32_t* accepted_counts, int counts_stride, const int32_t* offsets, int batch,
                              int max_accepted, int32_t* new_kv_len, int32_t* new_last_page_len,
                              pts_stream_t stream) {
  PTS_CHECK_ARG(kv_pool && page_indptr && page_indices && accepted && accepted_counts && offsets, "null pointer");
  PTS_CHECK_ARG(accepted_stride >= max_accepted && counts_stride >= 1, "bad accepted/counts strides");
  PTS_CHECK_ARG(elem_bytes == 2 || elem_bytes == 4, "elem_bytes must be 2 or 4");
  PTS_CHECK_ARG(num_layers > 0 && max_pages > 0 && page_len > 0 && num_kv_heads > 0 && head_dim > 0, "bad shape");
  PTS_CHECK_ARG(batch > 0 && max_accepted >= 0, "bad batch/max_accepted");
  const int head_bytes = head_dim * elem_bytes;
  PTS_CHECK_ARG(head_bytes % 16 == 0, "head_dim * elem_bytes must be a multiple of 16");
  PTS_CHECK_ARG(((uintptr_t)kv_pool & 15) == 0, "pool must be 16-byte aligned");
  const size_t smem = (size_t)max_accepted * head_bytes;
  if (smem > 200 * 1024) return set_error(PTS_ERR_CAPACITY, "max_accepted %d too large", max_accepted);
  cudaStream_t st = (cudaStream_t)stream;
  if (max_accepted > 0) {
    if (smem > 48 * 1024)
      if (int rc = ensure_smem_attr((const void*)kv_compact_kernel, smem)) return rc;
    if (2 * num_layers > 65535 || batch > 65535) return set_error(PTS_ERR_CAPACITY, "grid too large");
    const int64_t layer_bytes = (int64_t)max_pages * 2 * page_len * num_kv_heads * head_bytes;
    dim3 grid(num_kv_heads, 2 * num_layers, batch);
    kv_compact_kernel<<<grid, 128, smem, st>>>((char*)kv_pool, layer_bytes, max_pages, page_len, num_kv_heads,
                                               head_bytes, page_indptr, page_indices, accepted, accepted_stride,
                                               accepted_counts, counts_stride, max_accepted, offsets);
    int rc = launch_status("kv_compact_kernel");
    if (rc) return rc;
  }
  if (new_kv_len || new_last_page_len) {
    kv_compact_lengths_kernel<<<(batch + 127) / 128, 128, 0, st>>>(accepted_counts, counts_stride, max_accepted,
                                                                   offsets, batch, page_len, new_kv_len,
                                                                   new_last_page_len);
    return launch_status("kv_compact_lengths_kernel");
  }
  return PTS_OK;
}

extern "C" int pts_tree_mask_from_parents(const int32_t* parents, const int32_t* qo_indptr, int batch, int total_q,
                                          int mask_words, uint64_t* mask_bits, pts_stream_t stream) {
  PTS_CHECK_ARG(parents && qo_indptr && mask_bits, "null pointer");
  PTS_CHECK_ARG(batch > 0 && total_q >= 0 && mask_words > 0, "bad sizes");
  if (total_q == 0) return PTS_OK;
  mask_from_parents_kernel<<<(total_q + 127) / 128, 128, 0, (cudaStream_t)stream>>>(parents, qo_indptr, batch,
                                                                                   total_q, mask_words, mask_bits);
  return launch_status("mask_from_parents_kernel");
}

extern "C" int pts_tree_mask_from_bool(const uint8_t* mask, const int32_t* qo_indptr, const int32_t* mask_indptr,
                                       const int32_t* kv_lens, int batch, int total_q, int mask_words,
                                       uint64_t* mask_bits, int32_t* bad_rows, pts_stream_t stream) {
  PTS_CHECK_ARG(mask && qo_indptr && mask_indptr && kv_lens && mask_bits, "null pointer");
  PTS_CHECK_ARG(batch > 0 && total_q >= 0 && mask_words > 0, "bad sizes");
  if (total_q == 0) return PTS_OK;
  mask_from_bool_kernel<<<(total_q + 3) / 4, 128, 0, (cudaStream_t)stream>>>(
      mask, qo_indptr, mask_indptr, kv_lens, batch, total_q, mask_words, mask_bits, bad_rows);
  return launch_status("mask_from_bool_kernel");
}

extern "C" int pts_tree_prepare(const int32_t* parents, const int32_t* qo_indptr, const int32_t* seq_lens, int batch,
                                int mask_words, uint64_t* mask_bits, int32_t* batch_indices, int32_t* positions,
                                pts_stream_t stream) {
  PTS_CHECK_ARG(parents && qo_indptr && mask_bits, "null pointer");
  PTS_CHECK_ARG(batch > 0 && mask_words > 0, "bad sizes");
  PTS_CHECK_ARG((batch_indices == nullptr) == (positions == nullptr) && (!positions || seq_lens),
                "batch_indices, positions and seq_lens go together");
  tree_prepare_kernel<<<batch, 128, 0, (cudaStream_t)stream>>>(parents, qo_indptr, seq_lens, mask_words, mask_bits,
                                                              batch_indices, positions);
  return launch_status("tree_prepare_kernel");
}

extern "C" int pts_tree_prepare_append(const int32_t* parents, const int32_t* qo_indptr, const int32_t* seq_lens,
                                       int batch, int mask_words, uint64_t* mask_bits, int32_t* batch_indices,
                                       int32_t* positions, const void* k, const void* v, int64_t k_token_stride,
                                       int64_t v_token_stride, void* kv_layer, const int32_t* page_indptr,
                                       const int32_t* page_indices, int num_tokens, int num_kv_heads, int head_dim,
                                       int page_len, int max_pages, int elem_bytes, pts_stream_t stream) {
  PTS_CHECK_ARG(parents && qo_indptr && seq_lens && mask_bits && batch_indices && positions, "null pointer");
  PTS_CHECK_ARG(k && v && kv_layer && page_indptr && page_indices, "null pointer");
  PTS_CHECK_ARG(batch > 0 && mask_words > 0 && num_tokens >= 0, "bad sizes");
  PTS_CHECK_ARG(elem_bytes == 2 || elem_bytes == 4, "elem_bytes must be 2 or 4");
  PTS_CHECK_ARG(num_kv_heads > 0 && head_dim > 0 && page_len > 0 && max_pages > 0, "bad shape");
  const int row_bytes = num_kv_heads * head_dim * elem_bytes;
  PTS_CHECK_ARG(row_bytes % 16 == 0, "Hkv * D * elem_bytes must be a multiple of 16");
  PTS_CHECK_ARG((k_token_stride * elem_bytes) % 16 == 0 && (v_token_stride * elem_bytes) % 16 == 0,
                "token strides must be multiples of 16 bytes");
  PTS_CHECK_ARG((((uintptr_t)k | (uintptr_t)v | (uintptr_t)kv_layer) & 15) == 0, "pointers must be 16-byte aligned");
  PTS_CHECK_ARG((int64_t)batch + num_tokens <= 0x7fffffff, "too many blocks");
  PTS_CUDA_TRY(launch_pdl(tree_prepare_append_kernel<false, 2>, dim3(batch + num_tokens), dim3(128), 0,
                          (cudaStream_t)stream, parents, qo_indptr, seq_lens, batch, mask_words, mask_bits,
                          batch_indices, positions, (const char*)k, (const char*)v, (int64_t)k_token_stride * elem_bytes,
                          (int64_t)v_token_stride * elem_bytes, (char*)kv_layer, page_indptr, page_indices, row_bytes,
                          page_len, max_pages, RopeArgs{}));
  return launch_status("tree_prepare_append_kernel");
}

extern "C" int pts_tree_prepare_append_rope(const int32_t* parents, const int32_t* qo_indptr, const int32_t* seq_lens,
                                            int batch, int mask_words, uint64_t* mask_bits, int32_t* batch_indices,
                                            int32_t* positions, const void* q, int64_t q_token_stride, void* q_out,
                                            int num_qo_heads, const void* k, const void* v, int64_t k_token_stride,
                                            int64_t v_token_stride, const void* cos, const void* sin,
                                            int64_t cos_sin_token_stride, void* kv_layer, const int32_t* page_indptr,
                                            const int32_t* page_indices, int num_tokens, int num_kv_heads,
                                            int head_dim, int page_len, int max_pages, int elem_bytes,
                                            pts_stream_t stream) {
  PTS_CHECK_ARG(parents && qo_indptr && seq_lens && mask_bits && batch_indices && positions, "null pointer");
  PTS_CHECK_ARG(q && q_out && k && v && cos && sin && kv_layer && page_indptr && page_indices, "null pointer");
  PTS_CHECK_ARG(batch > 0 && mask_words > 0 && num_tokens >= 0, "bad sizes");
  PTS_CHECK_ARG(elem_bytes == 2 || elem_bytes == 4, "elem_bytes must be 2 or 4");
  PTS_CHECK_ARG(num_kv_heads > 0 && num_qo_heads > 0 && page_len > 0 && max_pages > 0, "bad shape");
  PTS_CHECK_ARG(head_dim > 0 && (head_dim * elem_bytes) % 32 == 0,
                "head_dim * elem_bytes must be a multiple of 32 (each half of a head in 16-byte pieces)");
  const int row_bytes = num_kv_heads * head_dim * elem_bytes;
  PTS_CHECK_ARG((q_token_stride * elem_bytes) % 16 == 0 && (k_token_stride * elem_bytes) % 16 == 0 &&
                    (v_token_stride * elem_bytes) % 16 == 0 && (cos_sin_token_stride * elem_bytes) % 16 == 0,
                "token strides must be multiples of 16 bytes");
  PTS_CHECK_ARG((((uintptr_t)q | (uintptr_t)q_out | (uintptr_t)k | (uintptr_t)v | (uintptr_t)cos | (uintptr_t)sin |
                  (uintptr_t)kv_layer) & 15) == 0,
                "pointers must be 16-byte aligned");
  PTS_CHECK_ARG((int64_t)batch + num_tokens <= 0x7fffffff, "too many blocks");
  RopeArgs r;
  r.q = (const char*)q;
  r.q_stride = q_token_stride * elem_bytes;
  r.q_out = (char*)q_out;
  r.hq = num_qo_heads;
  r.cos = (const char*)cos;
  r.sin = (const char*)sin;
  r.cs_stride = cos_sin_token_stride * elem_bytes;
  r.head_dim = head_dim;
  auto kernel = elem_bytes == 2 ? tree_prepare_append_kernel<true, 2> : tree_prepare_append_kernel<true, 4>;
  PTS_CUDA_TRY(launch_pdl(kernel, dim3(batch + num_tokens), dim3(128), 0, (cudaStream_t)stream, parents, qo_indptr,
                          seq_lens, batch, mask_words, mask_bits, batch_indices, positions, (const char*)k,
                          (const char*)v, (int64_t)k_token_stride * elem_bytes, (int64_t)v_token_stride * elem_bytes,
                          (char*)kv_layer, page_indptr, page_indices, row_bytes, page_len, max_pages, r));
  return launch_status("tree_prepare_append_kernel");
}

extern "C" int pts_kv_append_rope(const void* q, int64_t q_token_stride, void* q_out, int num_qo_heads, const void* k,
                                  const void* v, int64_t k_token_stride, int64_t v_token_stride, const void* cos,
                                  const void* sin, int64_t cos_sin_token_stride, void* kv_layer,
                                  const int32_t* batch_indices, const int32_t* positions, const int32_t* page_indptr,
                                  const int32_t* page_indices, int num_tokens, int num_kv_heads, int head_dim,
                                  int page_len, int max_pages, int elem_bytes, pts_stream_t stream) {
  PTS_CHECK_ARG(q && q_out && k && v && cos && sin && kv_layer && batch_indices && positions && page_indptr &&
                    page_indices,
                "null pointer");
  PTS_CHECK_ARG(elem_bytes == 2 || elem_bytes == 4, "elem_bytes must be 2 or 4");
  PTS_CHECK_ARG(num_kv_heads > 0 && num_qo_heads > 0 && page_len > 0 && max_pages > 0, "bad shape");
  PTS_CHECK_ARG(head_dim > 0 && (head_dim * elem_bytes) % 32 == 0,
                "head_dim * elem_bytes must be a multiple of 32 (each half of a head in 16-byte pieces)");
  PTS_CHECK_ARG((q_token_stride * elem_bytes) % 16 == 0 && (k_token_stride * elem_bytes) % 16 == 0 &&
                    (v_token_stride * elem_bytes) % 16 == 0 && (cos_sin_token_stride * elem_bytes) % 16 == 0,
                "token strides must be multiples of 16 bytes");
  PTS_CHECK_ARG((((uintptr_t)q | (uintptr_t)q_out | (uintptr_t)k | (uintptr_t)v | (uintptr_t)cos | (uintptr_t)sin |
                  (uintptr_t)kv_layer) & 15) == 0,
                "pointers must be 16-byte aligned");
  if (num_tokens <= 0) return PTS_OK;
  const int row_bytes = num_kv_heads * head_dim * elem_bytes;
  RopeArgs r;
  r.q = (const char*)q;
  r.q_stride = q_token_stride * elem_bytes;
  r.q_out = (char*)q_out;
  r.hq = num_qo_heads;
  r.cos = (const char*)cos;
  r.sin = (const char*)sin;
  r.cs_stride = cos_sin_token_stride * elem_bytes;
  r.head_dim = head_dim;
  auto kernel = elem_bytes == 2 ? kv_append_rope_kernel<2> : kv_append_rope_kernel<4>;
  kernel<<<num_tokens, 128, 0, (cudaStream_t)stream>>>(
      (const char*)k, (const char*)v, k_token_stride * elem_bytes, v_token_stride * elem_bytes, (char*)kv_layer,
      batch_indices, positions, page_indptr, page_indices, row_bytes, page_len, max_pages, r);
  return launch_status("kv_append_rope_kernel");
}
