"""ctypes binding of libpts_b200.so (the C ABI declared in include/pts_b200.h).

There is no fallback: if the library cannot be loaded, every operation of
this package raises.  Set ``PTS_B200_LIB`` to load a library from another
path.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("PTS_B200_LIB", os.path.join(_PKG, "libpts_b200.so"))

PTS_OK = 0
PTS_ERR_INVALID = 1
PTS_ERR_CAPACITY = 2
PTS_ERR_CUDA = 3
PTS_ERR_UNSUPPORTED = 4
PTS_ERR_INDEX = 5
PTS_MAX_TREE_NODES = 1024

_lock = threading.Lock()
_lib = None

i32, i64, u64, f32, sz, vp = C.c_int32, C.c_int64, C.c_uint64, C.c_float, C.c_size_t, C.c_void_p

class KvCompactArgs(C.Structure):
    """pts_kv_compact_args: the KV compaction an acceptance launch performs."""
    _fields_ = [("kv_pool", C.c_void_p), ("num_layers", C.c_int), ("max_pages", C.c_int), ("page_len", C.c_int),
                ("num_kv_heads", C.c_int), ("head_dim", C.c_int), ("elem_bytes", C.c_int),
                ("page_indptr", C.c_void_p), ("page_indices", C.c_void_p), ("offsets", C.c_void_p),
                ("new_kv_len", C.c_void_p), ("new_last_page_len", C.c_void_p)]


SIGNATURES = {
    "pts_last_error": (C.c_char_p, []),
    "pts_version": (C.c_int, []),
    "pts_set_wait_limit": (C.c_longlong, [C.c_longlong]),
    "pts_tree_attn_check": (C.c_int, [vp, vp, vp]),
    "pts_tree_attn_set_schedule": (C.c_int, [C.c_int]),
    "pts_accept_workspace_size": (sz, [C.c_int, C.c_int]),
    "pts_accept_greedy": (C.c_int, [vp, i64, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, i64, vp, vp, vp,
                                    C.c_int, vp, sz, vp]),
    "pts_accept_traversal": (C.c_int, [vp, i64, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, i64, f32, f32,
                                       C.c_int, u64, u64, vp, vp, vp, C.c_int, vp, sz, vp]),
    "pts_accept_greedy_compact": (C.c_int, [vp, i64, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, i64, vp, vp,
                                            vp, C.c_int, vp, sz, vp, vp]),
    "pts_accept_traversal_compact": (C.c_int, [vp, i64, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, i64, f32,
                                               f32, C.c_int, u64, u64, vp, vp, vp, C.c_int, vp, sz, vp, vp]),
    "pts_accept_traversal_noalloc": (C.c_int, [vp, i64, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, i64,
                                               f32, f32, C.c_int, u64, u64, vp, vp, vp, C.c_int, vp]),
    "pts_accept_export_row_stats": (C.c_int, [vp, sz, vp, i64, vp, vp, vp, C.c_int, C.c_int, C.c_int, f32, vp, vp,
                                              vp]),
    "pts_lmhead_logits": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, vp, i64, vp]),
    "pts_lmhead_workspace_size": (sz, [C.c_int, C.c_int]),
    "pts_beam_select_workspace_size": (sz, [C.c_int, C.c_int]),
    "pts_beam_select": (C.c_int, [vp, i64, C.c_int, C.c_int, C.c_int, f32, vp, C.c_int, vp, vp, vp, vp, sz, vp]),
    "pts_kv_copy_pages": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp, C.c_int, C.c_int, vp]),
    "pts_lmhead_accept": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, vp, vp, C.c_int, C.c_int, i64,
                                    C.c_int, f32, u64, u64, vp, vp, vp, C.c_int, vp, sz, vp]),
    "pts_accept_shard_partials": (C.c_int, [vp, i64, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, f32, vp, vp,
                                            vp, sz, vp]),
    "pts_accept_merge_shards": (C.c_int, [vp, vp, C.c_int, C.c_int, vp, vp, vp]),
    "pts_accept_shard_ties": (C.c_int, [vp, i64, C.c_int, C.c_int, C.c_int, f32, vp, vp, vp]),
    "pts_accept_walk_merged": (C.c_int, [vp, vp, vp, C.c_int, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                         i64, u64, u64, vp, vp, vp, C.c_int, vp]),
    "pts_accept_greedy_f32": (C.c_int, [vp, i64, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, i64, vp, vp, vp,
                                        C.c_int, vp, sz, vp]),
    "pts_accept_traversal_f32": (C.c_int, [vp, i64, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, i64, f32,
                                           u64, u64, vp, vp, vp, C.c_int, vp, sz, vp]),
    "pts_batch_positions": (C.c_int, [vp, vp, C.c_int, C.c_int, vp, vp, vp]),
    "pts_kv_append": (C.c_int, [vp, vp, i64, i64, vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                C.c_int, vp]),
    "pts_kv_compact": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp, vp, C.c_int,
                                 vp, C.c_int, vp, C.c_int, C.c_int, vp, vp, vp]),
    "pts_tree_mask_from_parents": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, vp, vp]),
    "pts_tree_prepare": (C.c_int, [vp, vp, vp, C.c_int, C.c_int, vp, vp, vp, vp]),
    "pts_kv_append_rope": (C.c_int, [vp, i64, vp, C.c_int, vp, vp, i64, i64, vp, vp, i64, vp, vp, vp, vp, vp,
                                     C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp]),
    "pts_tree_prepare_append_rope": (C.c_int, [vp, vp, vp, C.c_int, C.c_int, vp, vp, vp, vp, i64, vp, C.c_int, vp, vp,
                                               i64, i64, vp, vp, i64, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                               C.c_int, C.c_int, vp]),
    "pts_tree_prepare_append": (C.c_int, [vp, vp, vp, C.c_int, C.c_int, vp, vp, vp, vp, vp, i64, i64, vp, vp, vp,
                                          C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp]),
    "pts_tree_mask_from_bool": (C.c_int, [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, vp]),
    "pts_tree_attn_run_any": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, f32, C.c_int, vp, sz, vp]),
    "pts_tree_attn_run_head_pages": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, C.c_int, vp, C.c_int, C.c_int, C.c_int,
                                               C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, f32, vp, sz,
                                               vp]),
    "pts_page_key_sums": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp]),
    "pts_select_pages": (C.c_int, [vp, vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.c_int, C.c_int, C.c_int, vp, vp, vp, vp]),
    "pts_tree_attn_workspace_size": (sz, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "pts_tree_attn_run": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, f32, vp, sz, vp]),
}


class PtsError(RuntimeError):
    def __init__(self, code: int, fn: str, msg: str):
        super().__init__(f"{fn} failed (code {code}): {msg}")
        self.code = code


def lib():
    """Load the library (once) and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"libpts_b200.so not found at {LIB_PATH}; build it with "
                                  f"`python -m parallel_tree_spec_b200.build`")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(code: int, fn: str) -> None:
    if code == PTS_OK:
        return
    msg = lib().pts_last_error().decode(errors="replace")
    if code == PTS_ERR_INVALID:
        raise ValueError(f"{fn}: {msg}")
    if code == PTS_ERR_INDEX:
        raise IndexError(f"{fn}: {msg}")
    raise PtsError(code, fn, msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
