"""Draft beam search with copy-on-write pages (``beam_search.py:1-616`` of the
reference): same names, signatures and results.

The page bookkeeping (reference counts, copy-on-write, the trie of beams) is
host logic, as in the reference, and hands out the same pages in the same
order (``KvCachePool.allocate`` gives the lowest free pages).  The device
work differs:

* the per-step scoring and selection -- softmax, ``log(p + 1e-10)``, the
  beams' cumulative scores and the flattened top-K -- is one fused
  selection (``kernels.beam_select``, two launches) instead of a chain of
  torch kernels, and its results come back in one device-to-host copy;
* the copy-on-write copies of a step go out in one launch
  (``kernels.kv_copy_pages``) after the step's allocations;
* batch positions carry the per-beam lengths on the host, so planning the
  decode attention syncs nothing.

Ties among equal scores go to the smaller flat index (torch's top-k leaves
their order unspecified).
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch

from . import kernels as K
from .attention_wrapper import BeFlashinferWrapper
from .cache_manager import KvCacheBatchPosition, KvCachePool, RequestKvCache, getKvCacheBatchPosition
from .tree import Tree, TreeNode


def _extract_last_token_q(model: torch.nn.Module, input_ids: torch.Tensor, kv_len: int,
                          device: torch.device) -> torch.Tensor:
    """The last prompt token's query averaged over the layers, [heads, dim]
    (``beam_search.py:28-79``), for the sparse strategy's q-k scoring."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    hidden = model.model.embed_tokens(input_ids[:, -1:])
    position_ids = torch.tensor([[kv_len - 1]], dtype=torch.long, device=device)
    cos, sin = model.model.rotary_emb(hidden, position_ids)
    acc, n = None, 0
    for layer in model.model.layers:
        attn = layer.self_attn
        q = attn.q_proj(hidden)
        q = q.view(1, 1, q.shape[-1] // attn.head_dim, attn.head_dim).transpose(1, 2)
        q, _ = apply_rotary_pos_emb(q, q, cos, sin)
        q = q.squeeze(2).squeeze(0).float()
        acc = q if acc is None else acc + q
        n += 1
    return acc / n


@dataclass
class BeamSearchConfig:
    """``beam_search.py:82-88``."""
    topk_len: int = 6          # beam width K
    max_depth: int = 10        # number of decode steps
    temperature: float = 1.0   # softmax temperature
    use_cuda_graph: bool = False  # capture decode steps in a CUDA graph


def _copy_block(kvCachePool: KvCachePool, src_page: int, off: int) -> int:
    """COW (``beam_search.py:92-96``): a fresh page holding src_page's first
    `off` slots of every layer."""
    new_page = kvCachePool.allocate(1)[0]
    dev = kvCachePool.cache_data.device
    K.kv_copy_pages(kvCachePool.cache_data, torch.tensor([src_page], dtype=torch.int32, device=dev),
                    torch.tensor([new_page], dtype=torch.int32, device=dev), off)
    return new_page


def _with_host_lens(bp: KvCacheBatchPosition, K_: int, current_pos: int) -> KvCacheBatchPosition:
    bp.host_qo_lens = [1] * K_
    bp.host_kv_lens = [current_pos + 1] * K_
    return bp


def _build_beam_batch_position(beam_pages_list: List[List[int]], current_pos: int, page_size: int,
                               device: torch.device) -> KvCacheBatchPosition:
    """``beam_search.py:99-122``: K beams each writing one token at current_pos."""
    K_ = len(beam_pages_list)
    indices, indptr = [], [0]
    for pages in beam_pages_list:
        indices.extend(pages)
        indptr.append(len(indices))
    last = current_pos % page_size + 1
    bp = KvCacheBatchPosition(
        seq_indptr=torch.arange(K_ + 1, dtype=torch.int32, device=device),
        kv_page_indptr=torch.tensor(indptr, dtype=torch.int32, device=device),
        kv_page_indices=torch.tensor(indices, dtype=torch.int32, device=device),
        kv_last_page_len=torch.tensor([last] * K_, dtype=torch.int32, device=device),
        batch_indices=torch.arange(K_, dtype=torch.int32, device=device),
        positions=torch.tensor([current_pos] * K_, dtype=torch.int32, device=device),
    )
    return _with_host_lens(bp, K_, current_pos)


class StaticBatchPosition:
    """Pre-allocated batch-position buffers (``beam_search.py:125-176``):
    pinned host staging copied asynchronously into fixed device buffers."""

    def __init__(self, K: int, max_pages_per_beam: int, device: torch.device):
        max_idx = K * max_pages_per_beam
        pin = torch.cuda.is_available()
        self._cpu_indices = torch.zeros(max_idx, dtype=torch.int32, pin_memory=pin)
        self._cpu_indptr = torch.zeros(K + 1, dtype=torch.int32, pin_memory=pin)
        self._gpu_indices = torch.zeros(max_idx, dtype=torch.int32, device=device)
        self._gpu_indptr = torch.zeros(K + 1, dtype=torch.int32, device=device)
        self._seq_indptr = torch.arange(K + 1, dtype=torch.int32, device=device)
        self._batch_indices = torch.arange(K, dtype=torch.int32, device=device)
        self._last_page_len = torch.zeros(K, dtype=torch.int32, device=device)
        self._positions = torch.zeros(K, dtype=torch.int32, device=device)
        self._copied = None

    def fill(self, beam_pages_list: List[List[int]], current_pos: int, page_size: int) -> KvCacheBatchPosition:
        """Populate the buffers from the beams' page lists."""
        if self._copied is not None:            # the staging is reused: the last copy must have left it
            self._copied.synchronize()
        K_ = len(beam_pages_list)
        off = 0
        for i, pages in enumerate(beam_pages_list):
            self._cpu_indptr[i] = off
            n = len(pages)
            self._cpu_indices[off:off + n] = torch.as_tensor(pages, dtype=torch.int32)
            off += n
        self._cpu_indptr[K_] = off
        self._gpu_indptr[:K_ + 1].copy_(self._cpu_indptr[:K_ + 1], non_blocking=True)
        self._gpu_indices[:off].copy_(self._cpu_indices[:off], non_blocking=True)
        if self._gpu_indices.is_cuda:
            self._copied = torch.cuda.Event()
            self._copied.record()
        self._last_page_len.fill_(current_pos % page_size + 1)
        self._positions.fill_(current_pos)
        bp = KvCacheBatchPosition(
            seq_indptr=self._seq_indptr,
            kv_page_indptr=self._gpu_indptr[:K_ + 1],
            kv_page_indices=self._gpu_indices[:off],
            kv_last_page_len=self._last_page_len,
            batch_indices=self._batch_indices,
            positions=self._positions,
        )
        return _with_host_lens(bp, K_, current_pos)


class CudaGraphRunner:
    """Captures and replays the decode forward (``beam_search.py:183-307``)."""

    def __init__(self, K: int, max_num_pages: int, device: torch.device):
        self.K = K
        self.device = device
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.static_output = None
        self.input_ids_buf = torch.zeros((K, 1), dtype=torch.long, device=device)
        self.position_ids_buf = torch.zeros((K, 1), dtype=torch.long, device=device)
        self.batch_position = KvCacheBatchPosition(
            seq_indptr=torch.arange(K + 1, dtype=torch.int32, device=device),
            kv_page_indptr=torch.zeros(K + 1, dtype=torch.int32, device=device),
            kv_page_indices=torch.zeros(K * max_num_pages, dtype=torch.int32, device=device),
            kv_last_page_len=torch.zeros(K, dtype=torch.int32, device=device),
            batch_indices=torch.arange(K, dtype=torch.int32, device=device),
            positions=torch.zeros(K, dtype=torch.int32, device=device),
        )
        _with_host_lens(self.batch_position, K, 0)

    def _forward(self, model, flashinfer_wrapper, kvCachePool):
        return model(self.input_ids_buf, position_ids=self.position_ids_buf, past_key_values=None, use_cache=False,
                     kvCachePool=kvCachePool, batch_position=self.batch_position, mode="decode",
                     flashinferWrapper=flashinfer_wrapper)

    def capture(self, model: torch.nn.Module, flashinfer_wrapper: BeFlashinferWrapper, kvCachePool: KvCachePool,
                page_size: int, dtype: torch.dtype):
        """Warm up on K scratch pages, then capture one decode forward."""
        K_ = self.K
        temp_pages = kvCachePool.allocate(K_)
        self.input_ids_buf.fill_(0)
        self.position_ids_buf.fill_(0)
        self.batch_position.kv_page_indptr.copy_(torch.arange(K_ + 1, dtype=torch.int32, device=self.device))
        self.batch_position.kv_page_indices[:K_].copy_(torch.tensor(temp_pages, dtype=torch.int32, device=self.device))
        self.batch_position.kv_last_page_len.fill_(1)
        self.batch_position.positions.fill_(0)
        _with_host_lens(self.batch_position, K_, 0)
        for _ in range(2):
            flashinfer_wrapper.prepareAttention("decode", self.batch_position, page_size, "NONE", dtype)
            self._forward(model, flashinfer_wrapper, kvCachePool)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        flashinfer_wrapper.prepareAttention("decode", self.batch_position, page_size, "NONE", dtype)
        with torch.cuda.graph(self.graph):
            self.static_output = self._forward(model, flashinfer_wrapper, kvCachePool)
        kvCachePool.deallocate(temp_pages)

    def replay(self, beam_input_ids: torch.Tensor, beam_position_ids: torch.Tensor,
               batch_position: KvCacheBatchPosition, flashinfer_wrapper: BeFlashinferWrapper, page_size: int,
               dtype: torch.dtype, sparse_batch_position: Optional[KvCacheBatchPosition] = None):
        """Copy the step's inputs into the captured buffers and replay."""
        self.input_ids_buf.copy_(beam_input_ids)
        self.position_ids_buf.copy_(beam_position_ids)
        self.batch_position.kv_page_indptr.copy_(batch_position.kv_page_indptr)
        n_idx = batch_position.kv_page_indices.shape[0]
        self.batch_position.kv_page_indices[:n_idx].copy_(batch_position.kv_page_indices)
        self.batch_position.kv_last_page_len.copy_(batch_position.kv_last_page_len)
        self.batch_position.positions.copy_(batch_position.positions)
        self.batch_position.host_qo_lens = batch_position.host_qo_lens
        self.batch_position.host_kv_lens = batch_position.host_kv_lens
        plan_pos = sparse_batch_position if sparse_batch_position is not None else self.batch_position
        flashinfer_wrapper.prepareAttention("decode", plan_pos, page_size, "NONE", dtype)
        self.graph.replay()
        return self.static_output


@torch.no_grad()
def beam_search(model: torch.nn.Module, request_kv_cache: RequestKvCache, input_ids: torch.Tensor,
                config: BeamSearchConfig, flashinfer_wrapper: BeFlashinferWrapper,
                prefilled_logits: Optional[torch.Tensor] = None,
                cuda_graph_runner: Optional[CudaGraphRunner] = None,
                sparse_strategy=None) -> Tuple[Tree, List[float], Optional[CudaGraphRunner]]:
    """K-beam search on the draft model (``beam_search.py:315-616``): returns
    the draft tree, the per-step times in seconds and the graph runner."""
    device = input_ids.device
    dtype = model.lm_head.weight.dtype
    K_ = config.topk_len
    max_depth = config.max_depth
    T = config.temperature
    kvCachePool = request_kv_cache.kvCachePool
    PAGE_SIZE = kvCachePool.page_len
    kv_len = request_kv_cache.get_seq_length()
    if isinstance(kv_len, torch.Tensor):
        kv_len = kv_len.item()
    input_len = input_ids.shape[1]

    # --- prefill (or the target's, shared) ---------------------------- :363-393
    t_prefill_start = time.perf_counter()
    if prefilled_logits is not None:
        logits = prefilled_logits
    else:
        request_kv_cache.increment(input_len)
        bp = getKvCacheBatchPosition(request_kv_caches=[request_kv_cache], mode="tree", device=device,
                                     treeTokens=input_len)
        flashinfer_wrapper.prepareAttention("prefill", bp, PAGE_SIZE, "NONE", kvCachePool.cache_data[0].dtype)
        position_ids = torch.arange(kv_len, kv_len + input_len, dtype=torch.long, device=device).unsqueeze(0)
        logits = model(input_ids, position_ids=position_ids, past_key_values=None, use_cache=False,
                       kvCachePool=kvCachePool, batch_position=bp, mode="prefill",
                       flashinferWrapper=flashinfer_wrapper).logits
        kv_len += input_len

    use_sparse = sparse_strategy is not None and sparse_strategy.config.enabled
    cuda_runner = None
    if config.use_cuda_graph:                                          # :395-408
        if cuda_graph_runner is not None and cuda_graph_runner.graph is not None:
            cuda_runner = cuda_graph_runner
        else:
            flashinfer_wrapper.init_cuda_graph_decode(K_, kvCachePool.max_pages, device)
            cuda_runner = cuda_graph_runner if cuda_graph_runner is not None else \
                CudaGraphRunner(K_, kvCachePool.max_pages, device)
    step_times = [time.perf_counter() - t_prefill_start]

    tree = Tree(input_ids[0, -1], dtype)
    prompt_pages = list(request_kv_cache.kv_page_indices)
    if use_sparse:                                                     # :415-430
        sparse_strategy.reset()
        q_vectors = None
        if sparse_strategy.config.importance_method == "qk_score":
            q_vectors = _extract_last_token_q(model, input_ids, kv_len, device)
        sparse_strategy.update_importance(kv_cache=kvCachePool.cache_data, page_indices=prompt_pages, seq_len=kv_len,
                                          page_len=PAGE_SIZE, num_kv_heads=kvCachePool.num_heads,
                                          head_dim=kvCachePool.head_dims, q=q_vectors)

    # --- the K first tokens: the prompt row's best probabilities ------ :432-461
    row = logits[0, -1:, :]
    _, ids0, p0 = K.beam_select(row, K_, T)
    topk_probs = p0.to(row.dtype)
    host = torch.stack([ids0.double(), topk_probs.double()]).cpu()
    cum = torch.log(topk_probs).float()                                # torch.log of the bf16 picks
    node_pages = {}
    page_ref_counts = {}
    beam_node: List[int] = []
    for i in range(K_):
        new_idx = tree.current_size
        tn = TreeNode(parent=0, token_id=int(host[0, i]), cumulative_probability=float(host[1, i]), depth=1)
        tree.nodes[0].children.append(new_idx)
        tree.nodes.append(tn)
        tree.current_size += 1
        node_pages[new_idx] = list(prompt_pages)
        for p in prompt_pages:
            page_ref_counts[p] = page_ref_counts.get(p, 0) + 1
        beam_node.append(new_idx)
    tree.available_leaves = list(beam_node)

    max_pages_per_beam = len(prompt_pages) + max_depth
    static_bp = StaticBatchPosition(K_, max_pages_per_beam, device)
    static_bp_sparse = StaticBatchPosition(K_, max_pages_per_beam, device) if use_sparse else None

    # --- decode loop ------------------------------------------------- :463-604
    current_pos = kv_len
    for _step in range(max_depth - 1):
        t_step_start = time.perf_counter()
        off = current_pos % PAGE_SIZE
        pli = current_pos // PAGE_SIZE
        unique_nodes = list(set(beam_node))                           # the reference's order
        if off == 0:
            new_pages = kvCachePool.allocate(len(unique_nodes))
            for node_idx, new_page in zip(unique_nodes, new_pages):
                node_pages[node_idx].append(new_page)
                page_ref_counts[new_page] = 1
        else:
            src, dst = [], []
            for node_idx in unique_nodes:
                write_page = node_pages[node_idx][pli]
                if page_ref_counts[write_page] > 1:
                    new_page = kvCachePool.allocate(1)[0]             # _copy_block, its copy batched below
                    src.append(write_page)
                    dst.append(new_page)
                    page_ref_counts[write_page] -= 1
                    if page_ref_counts[write_page] == 0:
                        kvCachePool.deallocate([write_page])
                        del page_ref_counts[write_page]
                    node_pages[node_idx][pli] = new_page
                    page_ref_counts[new_page] = 1
            if src:
                K.kv_copy_pages(kvCachePool.cache_data, torch.tensor(src, dtype=torch.int32).to(device, non_blocking=True),
                                torch.tensor(dst, dtype=torch.int32).to(device, non_blocking=True), off)

        beam_pages_list = [node_pages[beam_node[k]] for k in range(K_)]
        full_batch_position = static_bp.fill(beam_pages_list, current_pos, PAGE_SIZE)
        append_batch_position = None
        if use_sparse:
            sparse_pages_list = [sparse_strategy.filter_pages(pages, seq_len=current_pos, page_len=PAGE_SIZE)
                                 for pages in beam_pages_list]
            batch_position = static_bp_sparse.fill(sparse_pages_list, current_pos, PAGE_SIZE)
            append_batch_position = full_batch_position
        else:
            batch_position = full_batch_position

        beam_input_ids = torch.tensor([[tree.nodes[beam_node[k]].token_id] for k in range(K_)], dtype=torch.long,
                                      device=device)
        beam_position_ids = torch.full((K_, 1), current_pos, dtype=torch.long, device=device)
        if cuda_runner is not None and cuda_runner.graph is not None:
            outputs = cuda_runner.replay(beam_input_ids, beam_position_ids, full_batch_position, flashinfer_wrapper,
                                         PAGE_SIZE, dtype, sparse_batch_position=batch_position if use_sparse else None)
        else:
            flashinfer_wrapper.prepareAttention("decode", batch_position, PAGE_SIZE, "NONE",
                                                kvCachePool.cache_data[0].dtype)
            fwd_kwargs = dict(position_ids=beam_position_ids, past_key_values=None, use_cache=False,
                              kvCachePool=kvCachePool, batch_position=batch_position, mode="decode",
                              flashinferWrapper=flashinfer_wrapper)
            if append_batch_position is not None:
                fwd_kwargs["append_batch_position"] = append_batch_position
            outputs = model(beam_input_ids, **fwd_kwargs)
            if cuda_runner is not None and cuda_runner.graph is None:
                cuda_runner.capture(model, flashinfer_wrapper, kvCachePool, PAGE_SIZE, dtype)

        # score and select: one fused selection, one copy to the host  :546-561
        scores, flat, step_p = K.beam_select(outputs.logits[:, -1, :], K_, T, cum)
        host = torch.stack([flat.double(), step_p.double()]).cpu()
        vocab_size = outputs.logits.shape[-1]
        flat_ids = [int(v) for v in host[0].tolist()]
        parent_list = [f // vocab_size for f in flat_ids]
        new_tok_list = [f % vocab_size for f in flat_ids]
        step_probs = host[1].tolist()

        seen_pairs = {}
        new_beam_node: List[int] = []
        for i in range(K_):                                           # :563-591
            parent_node = beam_node[parent_list[i]]
            tok = new_tok_list[i]
            key = (parent_node, tok)
            if key in seen_pairs:
                new_node = seen_pairs[key]
            else:
                existing = tree.find_child_index(parent_node, tok)
                if existing != -1 and existing in node_pages:
                    new_node = existing
                else:
                    new_node = tree.current_size
                    tn = TreeNode(parent=parent_node, token_id=tok, cumulative_probability=step_probs[i],
                                  depth=tree.nodes[parent_node].depth + 1)
                    tree.nodes[parent_node].children.append(new_node)
                    tree.nodes.append(tn)
                    tree.current_size += 1
                    node_pages[new_node] = list(node_pages[parent_node])
                    for p in node_pages[new_node]:
                        page_ref_counts[p] += 1
                seen_pairs[key] = new_node
            new_beam_node.append(new_node)

        for old_node in set(beam_node):                               # :593-603
            pages_to_free = []
            for p in node_pages[old_node]:
                page_ref_counts[p] -= 1
                if page_ref_counts[p] == 0:
                    pages_to_free.append(p)
                    del page_ref_counts[p]
            for p in pages_to_free:
                kvCachePool.deallocate([p])
            del node_pages[old_node]

        tree.available_leaves = list(set(new_beam_node))
        beam_node = new_beam_node
        cum = scores
        current_pos += 1
        step_times.append(time.perf_counter() - t_step_start)

    prompt_pages_set = set(prompt_pages)                               # :606-614
    pages_to_free = set()
    for pages in node_pages.values():
        for p in pages:
            if p not in prompt_pages_set:
                pages_to_free.add(p)
    for p in pages_to_free:
        kvCachePool.deallocate([p])
    return tree, step_times, cuda_runner
