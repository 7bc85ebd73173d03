"""The C-ABI library loads and exports every function include/pts_b200.h declares
(no GPU needed: nothing is called except the error-string and version getters)."""
import ctypes as C
import os
import re

from parallel_tree_spec_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "pts_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pts_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_version_and_error_string():
    lib = _lib.lib()
    assert lib.pts_version() >= 1
    assert isinstance(lib.pts_last_error(), bytes)


def test_host_side_argument_checks_need_no_gpu():
    lib = _lib.lib()
    # null pointers are rejected before anything touches a device
    rc = lib.pts_accept_greedy(None, 0, None, None, None, 1, 1, 10, 1, -1, None, None, None, 1, None, 0, None)
    assert rc == _lib.PTS_ERR_INVALID
    rc = lib.pts_kv_append(None, None, 0, 0, None, None, None, None, None, 1, 8, 128, 16, 10, 2, None)
    assert rc == _lib.PTS_ERR_INVALID
    assert lib.pts_accept_workspace_size(1040, 128256) > 0


# entries that set a process-wide choice and return the previous one
_SETTERS = {"pts_tree_attn_set_schedule"}


def test_every_entry_rejects_null_pointers_on_the_host():
    """Every status-returning entry, given null pointers and sizes of 1,
    returns PTS_ERR_INVALID from its host-side checks, before any CUDA call
    (which here, without a GPU, would give PTS_ERR_CUDA instead)."""
    lib = _lib.lib()
    checked = 0
    for name, (res, args) in sorted(_lib.SIGNATURES.items()):
        if res is not C.c_int or not args or name in _SETTERS:
            continue
        vals = [None if a is C.c_void_p else 1.0 if a in (C.c_float, C.c_double) else 1 for a in args]
        rc = getattr(lib, name)(*vals)
        assert rc == _lib.PTS_ERR_INVALID, (name, rc, lib.pts_last_error())
        checked += 1
    assert checked >= 20


def test_wait_limit_setting_round_trips():
    """pts_set_wait_limit returns the previous limit; <= 0 restores the default
    (host-side only, no launch)."""
    lib = _lib.lib()
    default = lib.pts_set_wait_limit(0)
    assert default > 10 ** 8
    assert lib.pts_set_wait_limit(5000) == default
    assert lib.pts_set_wait_limit(-1) == 5000
    assert lib.pts_set_wait_limit(0) == default


def test_attention_schedule_setting_round_trips():
    """pts_tree_attn_set_schedule returns the previous choice and rejects values
    outside 0-2 with -1 (host-side only, no launch)."""
    lib = _lib.lib()
    prev = lib.pts_tree_attn_set_schedule(1)
    assert prev in (0, 1, 2)
    assert lib.pts_tree_attn_set_schedule(2) == 1
    assert lib.pts_tree_attn_set_schedule(7) == -1
    assert lib.pts_tree_attn_set_schedule(prev) == 2
