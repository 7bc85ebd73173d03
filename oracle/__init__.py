"""CPU oracle for the tree-verification step (test infrastructure only).

This package restates, in NumPy and plain Python, the reference's algorithms
for the tree-verification path of parallel_tree_spec:

* ``accept``    -- softmax over bf16 logits, greedy tree walk
  (``verification.py:185-268``) and traversal verification
  (``verification.py:275-524``), fed by the ``philox`` uniform stream.
* ``kv``        -- paged-KV append, batch positions and KV compaction
  (``flashinfer/cache_manager.py:103-140,196-213,216-280``).
* ``attention`` -- tree-masked paged attention with FlashInfer's custom-mask
  semantics (``flashinfer/attention_wrapper.py:131-144``,
  ``tree.py:167-194``).
* ``philox``    -- Philox4x32-10 (Salmon et al., SC'11) and the uniform
  stream that replaces ``torch.rand(1)`` inside the traversal loop.
* ``pages``     -- page key sums, per-KV-head sparse page selection and tree
  attention over per-head page tables (long-prefix requests; parity
  unpinned: the reference selects pages for the draft only, one set for all
  heads, ``sparse_attention/pillar.py:83-216``).

It is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it.
Parity of ``accept`` and ``kv`` is pinned against golden vectors produced by
running the reference's own functions (``tests/golden/gen_golden.py``).
The attention restatement is pinned only by the reference's mask builder;
the attention arithmetic itself is FlashInfer's (third party), so its parity
is "unpinned" beyond the 2e-2 max-abs / 1e-3 mean-abs tolerance.
"""
