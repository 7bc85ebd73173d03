/*
 * pts_b200.h -- C ABI of the B200 tree-verification library (libpts_b200.so).
 *
 * Plain pointers and sizes only.  Every device pointer must point to memory
 * of the current CUDA device; every function enqueues its work on `stream`
 * and returns without synchronising.  The library never allocates: buffers
 * and workspaces belong to the caller.  Return value: PTS_OK (0) or one of
 * the PTS_ERR_* codes below; pts_last_error() gives a message for the
 * calling thread's last failure.
 *
 * Layouts (the reference's, parallel_tree_spec/src/parallel_tree_spec):
 *   paged KV layer   [max_pages, 2, page_len, Hkv, D]   (NHD, K = 0, V = 1)
 *                    flashinfer/cache_manager.py:55-72
 *   KV pool          [L, max_pages, 2, page_len, Hkv, D]
 *   queries / keys   [tokens, heads, D] contiguous      flashinfer/attention_wrapper.py:176-182
 *   logits           [rows, V] bf16, row stride given   verification.py:139
 *   trees            back-to-back per request, row_indptr[B+1]; parents are
 *                    local indices (root = row 0 of its request, parent -1),
 *                    BFS order (parent < child)         tree.py:145-159
 */
#ifndef PTS_B200_H
#define PTS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* pts_stream_t; /* cudaStream_t */

#define PTS_OK 0
#define PTS_ERR_INVALID 1     /* bad argument (maps to ValueError)                      */
#define PTS_ERR_CAPACITY 2    /* workspace too small or size above a stated maximum     */
#define PTS_ERR_CUDA 3        /* a CUDA runtime call or launch failed                    */
#define PTS_ERR_UNSUPPORTED 4 /* shape or option this build does not implement           */
#define PTS_ERR_INDEX 5       /* index out of range (maps to IndexError)                */

/* Largest tree (rows per request) the acceptance and attention kernels take. */
#define PTS_MAX_TREE_NODES 1024

const char* pts_last_error(void);
int pts_version(void);

/* Failure handling (no counterpart in the reference).  Every wait of this
 * library's kernels on other warps, other CTAs or in-flight copies is bounded:
 * after the limit (SM clock cycles, default 4e9, about 2 s at the top clock)
 * the kernel records an error, drains its own tensor-core work and copies,
 * frees its TMEM and returns, so the CUDA context stays usable.
 * pts_set_wait_limit sets the limit for launches made after it, process-wide
 * (cycles <= 0 restores the default), and returns the previous limit; a small
 * limit makes waits run out on purpose, to test the error paths. */
long long pts_set_wait_limit(long long cycles);

/* ------------------------------------------------------------------ acceptance
 * Fused acceptance: one pass over the bf16 logits computes, per row, the max,
 * the fp32 sum of exp(x - max), and the argmax of the bf16-rounded softmax
 * (first index on ties), then walks each request's tree on the device.
 *
 * Outputs per request b (out_stride = max entries per request >= its depth+1):
 *   out_tokens[b*out_stride + i], out_hidden[b*out_stride + i]   i < n_out
 *   out_counts[b*4 + {0,1,2,3}] = {n_out, total_len, accept_len, accepted_node}
 * eos_token_id < 0 means "no EOS".
 */
size_t pts_accept_workspace_size(int num_rows, int vocab);

/* Replaces verify_tree_exact + _verify_step_greedy + _sample_probs
 * (verification.py:185-268, 58-77, 46-55). */
int pts_accept_greedy(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                      const int32_t* parents, const int32_t* tokens, int batch, int num_rows,
                      int vocab, int max_nodes, int64_t eos_token_id, int32_t* out_tokens,
                      int32_t* out_hidden, int32_t* out_counts, int out_stride, void* workspace,
                      size_t workspace_bytes, pts_stream_t stream);

/* Replaces verify_tree_traversal (verification.py:275-524) with the
 * per-iteration torch.rand(1) draw (verification.py:396) taken from the
 * Philox4x32-10 stream u(b, k) = (philox(key = seed, ctr = (k>>2, b,
 * offset_lo, offset_hi))[k&3] >> 8) * 2^-24.  draft_probs[r] is node r's
 * cumulative_probability (tree.py:30).  top_p < 1 restricts the target
 * distribution to its nucleus (no counterpart in the reference): the tokens
 * whose scaled logit is >= t*, t* the largest logit value whose cumulative
 * mass from the top (fp64 sum of count(v) * expf(v - m) over the distinct
 * values v >= t*) reaches top_p * s; inside it p'(x) = bf16(expf(x - m) /
 * s_N), s_N that mass in fp32.  do_sample != 0 draws the bonus token from
 * the accepted row's distribution (p' under top-p) instead of taking its
 * argmax (verification.py:508-511), by inverse CDF with the Philox draw
 * 2*PTS_MAX_TREE_NODES: the row's rounded probabilities summed in fp64 over
 * 1024 consecutive segments, the segment sums accumulated in order, the
 * first index whose running sum exceeds u * total.  Both run the walks in a
 * second launch after the row statistics (and the nuclei). */
int pts_accept_traversal(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                         const int32_t* parents, const int32_t* tokens, const float* draft_probs,
                         int batch, int num_rows, int vocab, int max_nodes, int64_t eos_token_id,
                         float temperature, float top_p, int do_sample, uint64_t philox_seed,
                         uint64_t philox_offset, int32_t* out_tokens, int32_t* out_hidden,
                         int32_t* out_counts, int out_stride, void* workspace,
                         size_t workspace_bytes, pts_stream_t stream);

/* The KV compaction of the accepted paths (pts_kv_compact with accepted =
 * out_hidden, accepted_stride = max_accepted = out_stride, counts =
 * out_counts column 0), done by the acceptance launch itself: each walk
 * compacts its request as soon as its path is known.  kv_pool is
 * [num_layers, max_pages, 2, page_len, Hkv, D]; offsets[b] is the cache slot of
 * request b's tree row 0; new_kv_len / new_last_page_len (nullable) receive
 * offsets[b] + count and its last-page fill.  The pool's tree rows must be
 * written before the acceptance launch (stream order) and read by nothing else
 * during it.  Replaces reorder_cache_with_offset after verification
 * (flashinfer/cache_manager.py:103-140, 196-213). */
typedef struct pts_kv_compact_args {
  void* kv_pool;
  int num_layers, max_pages, page_len, num_kv_heads, head_dim, elem_bytes;
  const int32_t* page_indptr;
  const int32_t* page_indices;
  const int32_t* offsets;
  int32_t* new_kv_len;
  int32_t* new_last_page_len;
} pts_kv_compact_args;

/* pts_accept_greedy / pts_accept_traversal followed, in the same launch, by
 * the KV compaction described by *compact (NULL: none).  With a compaction
 * (a verification step) and bf16 rows that start 16-byte aligned with a
 * vocabulary that is a multiple of 8, the greedy form reduces only the rows
 * its walks read (each request's root and accepted nodes, verification.py:
 * 232-262), each when its walk reaches it: the same outputs, and
 * pts_accept_export_row_stats afterwards covers those rows only. */
int pts_accept_greedy_compact(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                              const int32_t* parents, const int32_t* tokens, int batch, int num_rows,
                              int vocab, int max_nodes, int64_t eos_token_id, int32_t* out_tokens,
                              int32_t* out_hidden, int32_t* out_counts, int out_stride,
                              void* workspace, size_t workspace_bytes,
                              const pts_kv_compact_args* compact, pts_stream_t stream);
int pts_accept_traversal_compact(const uint16_t* logits, int64_t row_stride, const int32_t* row_indptr,
                                 const int32_t* parents, const int32_t* tokens, const float* draft_probs,
                                 int batch, int num_rows, int vocab, int max_nodes, int64_t eos_token_id,
                                 float temperature, float top_p, int do_sample, uint64_t philox_seed,
                                 uint64_t philox_offset, int32_t* out_tokens, int32_t* out_hidden,
                                 int32_t* out_counts, int out_stride, void* workspace,
                                 size_t workspace_bytes, const pts_kv_compact_args* compact,
                                 pts_stream_t stream);

/* The per-row statistics the last bf16 acceptance call (pts_accept_greedy*,
 * pts_accept_traversal* without top-p) on `workspace` used: out_argmax[r] =
 * the argmax of row r's rounded softmax, out_mb[r] = the rounded probability
 * of row r's token under its parent's row (1 for roots), with the same
 * arithmetic the walks use.  The same logits, trees and temperature as that
 * call.  These are _sample_probs(...).argmax() (verification.py:46-77) and
 * probs[parent, token] (verification.py:310-349) as this library computes
 * them, exported for diagnostics and parity measurements.  After a greedy
 * call with a compaction, only the rows that call's walks read have
 * statistics (see pts_accept_greedy_compact). */
int pts_accept_export_row_stats(const void* workspace, size_t workspace_bytes, const uint16_t* logits,
                                int64_t row_stride, const int32_t* row_indptr, const int32_t* parents,
                                const int32_t* tokens, int batch, int num_rows, int vocab,
                                float temperature, int32_t* out_argmax, float* out_mb,
                                pts_stream_t stream);

/* verify_tree_exact / verify_tree_traversal over fp32 logits (small fp32
 * models, for example the reference's 2-layer configuration): the
 * probabilities stay fp32 as torch's softmax of fp32 logits does
 * (verification.py:46-55, 310-311), p = expf(x - m) / s; the greedy argmax is
 * the first index of the largest fp32 probability.  Same outputs as the bf16
 * entry points; the walks run in a second launch after the row statistics.
 * Workspace: pts_accept_workspace_size. */
int pts_accept_greedy_f32(const float* logits, int64_t row_stride, const int32_t* row_indptr,
                          const int32_t* parents, const int32_t* tokens, int batch, int num_rows,
                          int vocab, int max_nodes, int64_t eos_token_id, int32_t* out_tokens,
                          int32_t* out_hidden, int32_t* out_counts, int out_stride, void* workspace,
                          size_t workspace_bytes, pts_stream_t stream);
int pts_accept_traversal_f32(const float* logits, int64_t row_stride, const int32_t* row_indptr,
                             const int32_t* parents, const int32_t* tokens, const float* draft_probs,
                             int batch, int num_rows, int vocab, int max_nodes, int64_t eos_token_id,
                             float temperature, uint64_t philox_seed, uint64_t philox_offset,
                             int32_t* out_tokens, int32_t* out_hidden, int32_t* out_counts,
                             int out_stride, void* workspace, size_t workspace_bytes,
                             pts_stream_t stream);

/* ------------------------------------------------------ vocabulary-sharded acceptance
 * Tensor-parallel acceptance: each rank holds the logits of one vocabulary
 * shard (columns [vocab_offset, vocab_offset + shard_vocab) of the rows the
 * reference softmaxes whole, verification.py:55,212-213,310-311).  The
 * reference has no tensor parallelism; this is the exchange step of the
 * 8-way vocabulary split:
 *   1. pts_accept_shard_partials on every rank: per row a 16-byte partial
 *      {f64 sum of exp(x - m), f32 max m, i32 first (global) index of m}
 *      and per node the scaled logit of its token under its parent's row if
 *      this shard holds the token (else -inf);
 *   2. all-gather both arrays (shard order);
 *   3. pts_accept_merge_shards on every rank: 16-byte row statistics
 *      {f32 m, f32 s, i32 argmax, i32 flags}, flags bit 0 = a rounding tie
 *      decides the argmax of the rounded probabilities, plus merged token
 *      logits;
 *   4. pts_accept_shard_ties on every rank: per tied row the first index of
 *      this shard with the largest rounded probability (INT_MAX otherwise);
 *   5. all-gather those indices;
 *   6. pts_accept_walk_merged on every rank: the walks of verify_tree_exact
 *      (draft_probs == NULL) or verify_tree_traversal (Philox stream as in
 *      pts_accept_traversal) from the merged statistics; it rewrites the
 *      argmax of tied rows in row_stats.
 * Every rank obtains the same accepted paths. */
int pts_accept_shard_partials(const uint16_t* logits_shard, int64_t row_stride,
                              const int32_t* row_indptr, const int32_t* parents,
                              const int32_t* tokens, int batch, int num_rows, int shard_vocab,
                              int vocab_offset, float temperature, void* out_partials,
                              float* out_token_logit, void* workspace, size_t workspace_bytes,
                              pts_stream_t stream);
int pts_accept_merge_shards(const void* partials_all, const float* token_logit_all, int num_shards,
                            int num_rows, void* out_row_stats, float* out_token_logit,
                            pts_stream_t stream);
int pts_accept_shard_ties(const uint16_t* logits_shard, int64_t row_stride, int num_rows,
                          int shard_vocab, int vocab_offset, float temperature,
                          const void* row_stats, int32_t* out_first, pts_stream_t stream);
int pts_accept_walk_merged(void* row_stats, const float* token_logit, const int32_t* ties_all,
                           int num_shards, const int32_t* row_indptr, const int32_t* parents,
                           const int32_t* tokens, const float* draft_probs, int batch, int num_rows,
                           int vocab, int max_nodes, int64_t eos_token_id, uint64_t philox_seed,
                           uint64_t philox_offset, int32_t* out_tokens, int32_t* out_hidden,
                           int32_t* out_counts, int out_stride, pts_stream_t stream);

/* pts_accept_traversal without a workspace argument.  No counterpart in the
 * reference: it is for callers that cannot allocate device memory (a host
 * program holding only device pointers handed over by another runtime, or a
 * server whose device memory is planned up front and may not call cudaMalloc
 * later).  Scratch comes from a fixed 2 MiB device array inside the library
 * (present on every GPU that loads it, until exit); sizes needing more are
 * rejected with PTS_ERR_CAPACITY.  The first call on a device (and the first
 * after another CUDA context is made current there) looks up that array's
 * device address -- make it before any stream capture.  Calls share the
 * array: calls whose kernels overlap on the GPU race. */
int pts_accept_traversal_noalloc(const uint16_t* logits, int64_t row_stride,
                                 const int32_t* row_indptr, const int32_t* parents,
                                 const int32_t* tokens, const float* draft_probs, int batch,
                                 int num_rows, int vocab, int max_nodes, int64_t eos_token_id,
                                 float temperature, float top_p, int do_sample,
                                 uint64_t philox_seed, uint64_t philox_offset, int32_t* out_tokens,
                                 int32_t* out_hidden, int32_t* out_counts, int out_stride,
                                 pts_stream_t stream);

/* ------------------------------------------------------------------ lm_head
 * The target's lm_head over the tree rows, logits = hidden x weight^T
 * (flashinfer/modeling_llama.py:104, `self.lm_head(hidden_states[...])`):
 * hidden [num_rows, hidden_size] and weight [vocab, hidden_size] bf16, rows
 * contiguous, hidden_size a multiple of 64; fp32 accumulation on the tensor
 * cores, every logit rounded to bf16 as the model's bf16 output is.
 *
 * pts_lmhead_logits writes the bf16 logits [num_rows, logits_stride].
 *
 * pts_lmhead_accept runs the same GEMM without writing the logits: its
 * epilogue reduces every 256-column tile of a row to the acceptance
 * statistics (max, sum of exp(x - max), first index of the max; each node's
 * token logit under its parent row; for rows whose max could tie under
 * bf16 rounding, the tile's largest distinct values with their first
 * indices), the tiles are merged per row, and the walks of pts_accept_greedy
 * (traversal = 0) or pts_accept_traversal (traversal = 1, top-p 1, no bonus
 * sampling; Philox stream as there) run from the merged statistics.  Same
 * outputs as pts_lmhead_logits followed by the bf16 acceptance on those
 * logits.  A request containing a row whose rounding tie the candidate lists
 * cannot settle (more tied distinct values in one tile than it keeps, for
 * example a near-constant row) gets out_counts[b*4] = -4: redo it from
 * pts_lmhead_logits and the acceptance.  Workspace:
 * pts_lmhead_workspace_size. */
int pts_lmhead_logits(const void* hidden, const void* weight, int num_rows, int vocab, int hidden_size,
                      void* logits, int64_t logits_stride, pts_stream_t stream);
size_t pts_lmhead_workspace_size(int num_rows, int vocab);
int pts_lmhead_accept(const void* hidden, const void* weight, int num_rows, int vocab, int hidden_size,
                      const int32_t* row_indptr, const int32_t* parents, const int32_t* tokens,
                      const float* draft_probs, int batch, int max_nodes, int64_t eos_token_id,
                      int traversal, float temperature, uint64_t philox_seed, uint64_t philox_offset,
                      int32_t* out_tokens, int32_t* out_hidden, int32_t* out_counts, int out_stride,
                      void* workspace, size_t workspace_bytes, pts_stream_t stream);

/* ------------------------------------------------------------- sparse page sets
 * Long-prefix requests restricted to a page subset per KV head.  The
 * reference selects important pages (q . k scores aggregated per page, top-k
 * plus a recent window) only for the draft's decode and with one set for all
 * heads (sparse_attention/pillar.py:83-216); these entry points select a set
 * per (request, KV head) for the verification attention.
 *
 * pts_page_key_sums: out[i, h, :] = fp32 sum of the page_len keys of page
 * page_ids[i], head h (a page summary kept beside the cache, [n, Hkv, D]).
 *
 * pts_select_pages: key_sums aligned with page_indices ([entries, Hkv, 128]);
 * per (request b, KV head h), in position order: the first n_first and last
 * n_last full prefix pages, the n_top middle pages of highest score
 * qbar . key_sum (qbar = the root query row qo_indptr[b] averaged over h's
 * GQA group; ties to the earlier page), then every page from the first one
 * holding a tree token.  Outputs per-head tables for
 * pts_tree_attn_run_head_pages: out_head_indptr [B*Hkv+1],
 * out_head_indices (capacity Hkv * entries of page_indices),
 * out_head_last_page_len [B*Hkv].  max_prefix_pages bounds the pages of any
 * request (at most 8192). */
int pts_page_key_sums(const void* kv_layer, const int32_t* page_ids, int num_pages, int num_kv_heads,
                      int head_dim, int page_len, float* out, pts_stream_t stream);
int pts_select_pages(const float* key_sums, const int32_t* page_indptr, const int32_t* page_indices,
                     const int32_t* last_page_len, const void* q, const int32_t* qo_indptr, int batch,
                     int num_qo_heads, int num_kv_heads, int head_dim, int page_len, int n_first,
                     int n_top, int n_last, int max_prefix_pages, int32_t* out_head_indptr,
                     int32_t* out_head_indices, int32_t* out_head_last_page_len,
                     pts_stream_t stream);

/* ------------------------------------------------------------------ paged KV
 * Per appended token t: batch_indices[t] = b and positions[t] = seq_lens[b] -
 * (append_indptr[b+1] - append_indptr[b]) + (t - append_indptr[b]).
 * Replaces flashinfer.get_batch_indices_positions as called by
 * getKvCacheBatchPosition(mode="tree") (flashinfer/cache_manager.py:263-271),
 * one append segment per request. */
int pts_batch_positions(const int32_t* append_indptr, const int32_t* seq_lens, int batch,
                        int num_tokens, int32_t* batch_indices, int32_t* positions,
                        pts_stream_t stream);

/* Scatter new K/V rows ([T, Hkv, D], token stride in elements) into one
 * layer's pages.  Replaces flashinfer.append_paged_kv_cache
 * (flashinfer/attention_wrapper.py:201-212).  elem_bytes = 2 (bf16/fp16) or 4. */
int pts_kv_append(const void* k, const void* v, int64_t k_token_stride, int64_t v_token_stride,
                  void* kv_layer, const int32_t* batch_indices, const int32_t* positions,
                  const int32_t* page_indptr, const int32_t* page_indices, int num_tokens,
                  int num_kv_heads, int head_dim, int page_len, int max_pages, int elem_bytes,
                  pts_stream_t stream);

/* KV compaction: request b's accepted list is accepted[b*accepted_stride + i],
 * i < accepted_counts[b*counts_stride]; slot offsets[b] + accepted[..i] is
 * copied to slot offsets[b] + i in every layer, K and V, all reads before any
 * write, slots mapped through the request's page table.  The acceptance
 * kernels' out_hidden / out_counts (counts_stride 4) plug in directly.
 * Replaces KvCachePool.reorder_cache_with_offset and
 * RequestKvCache.reorder_cache_with_offset (flashinfer/cache_manager.py:103-140,
 * 196-213): the request-level call's offset is offsets[b] + 1; with
 * page_indices = 0..max_pages-1 it is the pool-level flat-slot form.
 * new_kv_len / new_last_page_len (nullable) receive offsets[b] + count and
 * its last-page fill (cache_manager.py:203-207). */
int pts_kv_compact(void* kv_pool, int num_layers, int max_pages, int page_len, int num_kv_heads,
                   int head_dim, int elem_bytes, const int32_t* page_indptr,
                   const int32_t* page_indices, const int32_t* accepted, int accepted_stride,
                   const int32_t* accepted_counts, int counts_stride, const int32_t* offsets,
                   int batch, int max_accepted, int32_t* new_kv_len, int32_t* new_last_page_len,
                   pts_stream_t stream);

/* ------------------------------------------------------------------ attention
 * Ancestor bitmask of every tree row: bit j of row i's mask_words-word mask is
 * set when node j of the same request is i itself or one of its ancestors.
 * Replaces Tree.create_attention_mask (tree.py:167-194) for the tree block. */
int pts_tree_mask_from_parents(const int32_t* parents, const int32_t* qo_indptr, int batch,
                               int total_q, int mask_words, uint64_t* mask_bits,
                               pts_stream_t stream);

/* Once per tree step, in one launch: the ancestor bitmasks of every row
 * (pts_tree_mask_from_parents) and, when batch_indices / positions are
 * given, the append batch index and position of every tree token
 * (pts_batch_positions with one segment per request, seq_lens including the
 * tree).  Replaces Tree.create_attention_mask + the mask packing of
 * prepareAttention (tree.py:167-194, attention_wrapper.py:141) and
 * flashinfer.get_batch_indices_positions (cache_manager.py:263-271). */
int pts_tree_prepare(const int32_t* parents, const int32_t* qo_indptr, const int32_t* seq_lens, int batch,
                     int mask_words, uint64_t* mask_bits, int32_t* batch_indices, int32_t* positions,
                     pts_stream_t stream);

/* pts_tree_prepare (with batch indices and positions) and pts_kv_append of
 * the tree tokens' K/V, [num_tokens = qo_indptr[batch]] rows at the
 * token strides given, in one launch.  The append derives each token's page
 * slot itself (the same position seq_lens[b] - N_b + i), so it does not wait
 * for the masks.  Replaces Tree.create_attention_mask + the mask packing,
 * get_batch_indices_positions and append_paged_kv_cache of one layer
 * (tree.py:167-194, flashinfer/cache_manager.py:263-271,
 * flashinfer/attention_wrapper.py:201-212). */
int pts_tree_prepare_append(const int32_t* parents, const int32_t* qo_indptr, const int32_t* seq_lens, int batch,
                            int mask_words, uint64_t* mask_bits, int32_t* batch_indices, int32_t* positions,
                            const void* k, const void* v, int64_t k_token_stride, int64_t v_token_stride,
                            void* kv_layer, const int32_t* page_indptr, const int32_t* page_indices,
                            int num_tokens, int num_kv_heads, int head_dim, int page_len, int max_pages,
                            int elem_bytes, pts_stream_t stream);

/* pts_kv_append with the rotary position embedding applied on the way (the
 * per-layer form of pts_tree_prepare_append_rope, for callers that have the
 * batch indices and positions): k rotated into the cache, v copied, q
 * rotated into q_out [num_tokens, Hq, D] (contiguous); the same rounding
 * as pts_tree_prepare_append_rope.  Replaces apply_rotary_pos_emb +
 * append_paged_kv_cache (flashinfer/attention.py:83-88,
 * flashinfer/attention_wrapper.py:201-212). */
int pts_kv_append_rope(const void* q, int64_t q_token_stride, void* q_out, int num_qo_heads, const void* k,
                       const void* v, int64_t k_token_stride, int64_t v_token_stride, const void* cos,
                       const void* sin, int64_t cos_sin_token_stride, void* kv_layer,
                       const int32_t* batch_indices, const int32_t* positions, const int32_t* page_indptr,
                       const int32_t* page_indices, int num_tokens, int num_kv_heads, int head_dim,
                       int page_len, int max_pages, int elem_bytes, pts_stream_t stream);

/* pts_tree_prepare_append with the rotary position embedding applied on the
 * way: the tree tokens' k [num_tokens, Hkv, D] are rotated into the cache, v
 * copied, and q [num_tokens, Hq, D] rotated into q_out (contiguous), as
 * x * cos + rotate_half(x) * sin with each product and the sum rounded to the
 * element type (bf16 or fp32), as the reference's model applies
 * apply_rotary_pos_emb before the append (flashinfer/attention.py:83-88).
 * cos / sin [num_tokens, D] are the model's position embeddings of the tree
 * tokens (token stride cos_sin_token_stride elements); head_dim * elem_bytes
 * must be a multiple of 32. */
int pts_tree_prepare_append_rope(const int32_t* parents, const int32_t* qo_indptr, const int32_t* seq_lens,
                                 int batch, int mask_words, uint64_t* mask_bits, int32_t* batch_indices,
                                 int32_t* positions, const void* q, int64_t q_token_stride, void* q_out,
                                 int num_qo_heads, const void* k, const void* v, int64_t k_token_stride,
                                 int64_t v_token_stride, const void* cos, const void* sin,
                                 int64_t cos_sin_token_stride, void* kv_layer, const int32_t* page_indptr,
                                 const int32_t* page_indices, int num_tokens, int num_kv_heads, int head_dim,
                                 int page_len, int max_pages, int elem_bytes, pts_stream_t stream);

/* Pack a boolean custom mask [sum_b N_b * kv_len_b] (FlashInfer's flattened
 * custom_mask, flashinfer/attention_wrapper.py:141) into tree bitmasks.
 * Columns before kv_len_b - N_b must all be true; *bad_rows (device int,
 * nullable) counts rows where they are not. */
int pts_tree_mask_from_bool(const uint8_t* mask, const int32_t* qo_indptr, const int32_t* mask_indptr,
                            const int32_t* kv_lens, int batch, int total_q, int mask_words,
                            uint64_t* mask_bits, int32_t* bad_rows, pts_stream_t stream);

/* Tree-masked paged attention, bf16 in / bf16 out, fp32 accumulation on the
 * tcgen05 tensor cores.  Query row i of request b sees the request's KV slots
 * [0, kv_len_b - N_b) (the prefix) and the tree slots kv_len_b - N_b + j whose
 * bit j is set in its mask; mask_bits == NULL makes the rows causal (row i
 * sees slots up to kv_len_b - N_b + i: prefill and decode).  kv_len_b = (page_indptr[b+1]-page_indptr[b]-1) *
 * page_len + last_page_len[b].  Replaces BatchPrefillWithPagedKVCacheWrapper
 * plan/run with custom_mask, causal=False (flashinfer/attention_wrapper.py:
 * 131-144, 250-252).  head_dim 128, page_len 16, Hq/Hkv = 4 in this build.
 *
 * Workspace: zeroed before its first use, 256-byte aligned, used by one
 * stream at a time.  With at least pts_tree_attn_workspace_size bytes (about
 * 40 MB on a 148-SM part: two partial-result slots per SM) the kernel may run
 * the balanced schedule -- one CTA per SM over equal ranges of 64-token KV
 * blocks, units cut by a range merged by their last CTA -- and leaves the
 * workspace zeroed again after every complete launch; with 256 bytes it runs
 * one CTA per (request, KV head, group of 264 query rows). */
size_t pts_tree_attn_workspace_size(int batch, int total_q, int num_qo_heads, int head_dim,
                                    int max_kv_len);
/* The error word pts_tree_attn_run* leave in `workspace` when a CTA gave up
 * waiting (0: none; nonzero: which wait).  Synchronises the stream, copies the
 * word to *status and clears it in the workspace, together with the counters
 * and flags of split units that an abandoned balanced launch left behind. */
int pts_tree_attn_check(void* workspace, int* status, pts_stream_t stream);
/* Process-wide choice of the attention schedule: 0 (the default) chooses per
 * launch from its sizes (balanced ranges only where units would leave many
 * SMs idle, e.g. a few long requests), 1 always one CTA per unit, 2 balanced
 * ranges whenever the workspace allows.  Returns the previous choice, or -1
 * for a value outside 0-2.  No counterpart in the reference (FlashInfer plans
 * its own split-KV schedule inside BatchPrefillWithPagedKVCacheWrapper.plan). */
int pts_tree_attn_set_schedule(int mode);

int pts_tree_attn_run(const void* q, const void* kv_layer, const int32_t* qo_indptr,
                      const int32_t* page_indptr, const int32_t* page_indices,
                      const int32_t* last_page_len, const uint64_t* mask_bits, int mask_words,
                      void* out, int batch, int total_q, int max_qo_len, int max_kv_len,
                      int num_qo_heads, int num_kv_heads, int head_dim, int page_len,
                      int max_pages, float sm_scale, void* workspace, size_t workspace_bytes,
                      pts_stream_t stream);

/* pts_tree_attn_run for any supported element type and shape: elem_bytes 2
 * (bf16) or 4 (fp32), head_dim a multiple of 32 up to 256, any page_len.
 * bf16 / head_dim 128 / page_len 16 / GQA group <= 16 takes the tensor-core
 * kernel, everything else a SIMT kernel (a correctness path for small fp32
 * models such as the reference's 2-layer, head_dim-64 configuration).  Same
 * reference interface as pts_tree_attn_run. */
int pts_tree_attn_run_any(const void* q, const void* kv_layer, const int32_t* qo_indptr,
                          const int32_t* page_indptr, const int32_t* page_indices,
                          const int32_t* last_page_len, const uint64_t* mask_bits, int mask_words,
                          void* out, int batch, int total_q, int max_qo_len, int max_kv_len,
                          int num_qo_heads, int num_kv_heads, int head_dim, int page_len, int max_pages,
                          float sm_scale, int elem_bytes, void* workspace, size_t workspace_bytes,
                          pts_stream_t stream);

/* pts_tree_attn_run with page tables per (request, KV head): head_page_indptr
 * [B*Hkv+1] and head_last_page_len [B*Hkv] indexed b * Hkv + h, every list
 * ending with the request's tree (its last N slots), for example the sparse
 * sets of pts_select_pages.  Replaces the same FlashInfer paged prefill
 * (attention_wrapper.py:131-144, 250-252) when each KV head attends its own
 * page subset. */
int pts_tree_attn_run_head_pages(const void* q, const void* kv_layer, const int32_t* qo_indptr,
                                 const int32_t* head_page_indptr, const int32_t* head_page_indices,
                                 const int32_t* head_last_page_len, const uint64_t* mask_bits,
                                 int mask_words, void* out, int batch, int total_q, int max_qo_len,
                                 int max_kv_len, int num_qo_heads, int num_kv_heads, int head_dim,
                                 int page_len, int max_pages, float sm_scale, void* workspace,
                                 size_t workspace_bytes, pts_stream_t stream);

/* --------------------------------------------------------- draft beam search
 * The draft's beam search builds the tree the path verifies
 * (beam_search.py:315-616).  Two of its device steps:
 *
 * pts_beam_select replaces the per-step scoring and selection
 *   probs = torch.softmax(logits[:, -1, :] / T, dim=-1)
 *   flat  = (cum[:, None] + torch.log(probs + 1e-10)).reshape(-1)
 *   scores, ids = flat.topk(K);  step_prob = probs[ids // V, ids % V]
 * (beam_search.py:549-561), and, with cum_log_probs NULL, the first step's
 * torch.softmax(logits / T).topk(K) (:432-433): logits [rows, row_stride]
 * (elem_bytes 2: bf16, rounded as torch's bf16 arithmetic rounds; 4: fp32),
 * the k best scores (k <= 16, rows <= 32) in descending order into out_score,
 * their flat indices row * vocab + token into out_index and their p into
 * out_prob.  Ties go to the smaller flat index (torch leaves their order
 * unspecified).  workspace: pts_beam_select_workspace_size(rows, k) bytes. */
size_t pts_beam_select_workspace_size(int rows, int k);
int pts_beam_select(const void* logits, int64_t row_stride, int elem_bytes, int rows, int vocab,
                    float temperature, const float* cum_log_probs, int k, float* out_score,
                    int64_t* out_index, float* out_prob, void* workspace, size_t workspace_bytes,
                    pts_stream_t stream);

/* Copy-on-write page copies of one decode step, _copy_block's
 *   cache_data[:, new_page, :, :off] = cache_data[:, src_page, :, :off]
 * (beam_search.py:92-96) for num_pairs (src_pages[i] -> dst_pages[i]) pairs
 * in one launch: the first `tokens` slots of every layer, keys and values, of
 * a pool laid out [num_layers, max_pages, 2, page_len, row_bytes]
 * (row_bytes = num_kv_heads * head_dim * element size, a multiple of 16).
 * Pairs naming a page outside [0, max_pages) are skipped. */
int pts_kv_copy_pages(void* kv_pool, int num_layers, int max_pages, int page_len, int row_bytes,
                      const int32_t* src_pages, const int32_t* dst_pages, int num_pairs, int tokens,
                      pts_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PTS_B200_H */
