#!/usr/bin/env python
"""Tree-verification step benchmark (B200).

One step = the verification of one batch of draft trees against the target's
paged KV cache, for one attention layer, on one GPU:

  1. tree masks, append positions and the append of the tree tokens' K/V
     into the pages, in one launch                      (pts_tree_prepare_append)
  2. tree-masked paged attention                        (pts_tree_attn_run)
  3. acceptance over the [B*N, V] bf16 logits + walk, with the compaction of
     each accepted path's KV in the same launch         (pts_accept_traversal_compact;
                                                          greedy: pts_accept_greedy + pts_kv_compact)

Workload (default): 16 requests, 4096-token prefix, 65-row trees (root + 8
levels of 8), 32 query / 8 KV heads, head_dim 128, 16-token pages, logits
[16*65, 128256] bf16 N(0, 3) with planted child tokens, traversal
verification at temperature 1.0.  Seeded synthetic inputs; per step the KV
(273 MB) and logits (267 MB) are each larger than L2.

`--impl reference` times the CPU restatement of the same path (the reference
is Python; its tree-verification path runs as the NumPy oracle on the host
cores) on a bounded sample of the workload.

For N > 1 the driver launches this under torchrun: every rank verifies its own
batch (weak scaling, no collective on the data path); timing is the max over
ranks of the device-timed region.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "tree-verify steps/s and verified tree tokens/s per GPU at bs=16, 4k prefix"
UNIT = "steps/s"


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--mode", choices=["traversal", "greedy"], default="traversal")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--prefix", type=int, default=4096)
    ap.add_argument("--width", type=int, default=8)
    ap.add_argument("--depth", type=int, default=8)
    ap.add_argument("--vocab", type=int, default=128256)
    ap.add_argument("--hq", type=int, default=32)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--top-p", type=float, default=1.0, help="nucleus target distribution for traversal (extension)")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--cpu-time-budget", type=float, default=90.0,
                    help="seconds after which the reference arm stops timing further steps")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", choices=["lmhead", "config3", "sparse", "flashinfer", "beam"], default=None,
                    help="run one sub-record alone and print it (for profiling one kernel on a small footprint)")
    ap.add_argument("--no-sub", action="store_true",
                    help="skip the sub-records (other acceptance modes, the config-3 path, tensor-parallel and "
                         "strong-scaling steps)")
    ap.add_argument("--sparse", action="store_true",
                    help="long-context sparse step (batch 8, 32768-token prefixes, 129-row trees, attention over "
                         "per-KV-head sets of 4 first + 64 top-scored + 8 last prefix pages, greedy)")
    ap.add_argument("--tp", action="store_true",
                    help="tensor-parallel step (70B-shaped target: 64 query / 8 KV heads split over the ranks, "
                         "vocabulary split over the ranks, batch 64, prefixes U[512, 8192]); run under torchrun")
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args(argv)


def workload_name(a):
    mode = f"traversal T={a.temperature}" if a.mode == "traversal" else "greedy"
    if a.mode == "traversal" and a.top_p < 1.0:
        mode += f" top-p {a.top_p}"
    n = 1 + a.width * a.depth
    return (f"tree-verify step: B={a.batch} requests, prefix={a.prefix}, tree rows={n} (width {a.width}, depth "
            f"{a.depth}), Hq={a.hq}, Hkv={a.hkv}, D=128, page=16, vocab={a.vocab}, {mode}")


def algorithmic_bytes(a):
    n = 1 + a.width * a.depth
    kv_len = a.prefix + n
    kv_read = a.batch * a.hkv * kv_len * 128 * 2 * 2
    q_o = 2 * a.batch * n * a.hq * 128 * 2
    append = a.batch * n * a.hkv * 128 * 2 * 2
    logits = a.batch * n * a.vocab * 2
    compact = 2 * a.batch * (a.depth + 1) * a.hkv * 128 * 2 * 2
    return dict(attention=kv_read + q_o, kv_read=kv_read, q_o=q_o, append=append, accept=logits,
                compact=compact, step=kv_read + q_o + append + logits + compact)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Sustained dense bf16 TFLOP/s (the attention kernel runs inside a long step)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured (sustained)"
        return float(d["bf16_tflops"]), "measured (burst)"
    return 1400.0, "fallback (sustained)"


def traffic_table():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML in a thread."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int, period: float = 0.005):
        self.index, self.period = index, period
        self.samples = []
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            self.max_mhz = None

    def _run(self):
        while not self._stop.is_set():
            try:
                sm = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), sm, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self._ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def stop(self):
        self._stop.set()
        if self._ok:
            self._t.join(timeout=1)

    def summary(self, t0=None, t1=None):
        s = [x for x in self.samples if (t0 is None or x[0] >= t0) and (t1 is None or x[0] <= t1)]
        window = "timed region"
        if not s:
            s, window = self.samples, "around timed region"
        if not s:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mask = 0
        for x in s:
            mask |= int(x[2])
        reasons = [n for b, n in self.REASONS.items() if mask & b]
        return {"sm_mhz": statistics.median([x[1] for x in s]), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(s), "window": window}


# ---------------------------------------------------------------- workload
def over_ranks(values, op, device):
    """``values`` (floats) reduced element-wise over all ranks with op "max"
    or "min", in one all-reduce; the values themselves without a process
    group."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN}[op])
    return [float(v) for v in t.tolist()]


def attn_workspace(device):
    """The attention workspace at its full size, so every record may take the
    balanced schedule when it pays (a smaller one forces one CTA per unit)."""
    from parallel_tree_spec_b200 import _lib, kernels as K
    return K.workspace(device, "attn", max(256, _lib.lib().pts_tree_attn_workspace_size(0, 0, 0, 0, 0)))


def build_workload(a, device, seed):
    import torch
    from parallel_tree_spec_b200 import kernels as K
    from parallel_tree_spec_b200 import workload as wl

    rng = np.random.default_rng(seed + 2)
    trees = [wl.make_tree(rng, a.width, a.depth, a.vocab) for _ in range(a.batch)]
    n = trees[0].size
    indptr, par, tok, dp = wl.stack_trees(trees)
    B, P, Hq, Hkv, D, pl = a.batch, a.prefix, a.hq, a.hkv, 128, 16
    kv_len = P + n
    pages_per = (kv_len + pl - 1) // pl
    max_pages = B * pages_per + 16
    g = torch.Generator(device=device)
    g.manual_seed(seed + 1)
    layer = torch.empty(max_pages, 2, pl, Hkv, D, dtype=torch.bfloat16, device=device)
    layer.normal_(0.0, 1.0 / math.sqrt(D), generator=g)
    perm = torch.randperm(max_pages, generator=g, device=device)[: B * pages_per].to(torch.int32)
    g.manual_seed(seed)
    q = torch.randn(B * n, Hq, D, generator=g, device=device).to(torch.bfloat16)
    k_new = (torch.randn(B * n, Hkv, D, generator=g, device=device) / math.sqrt(D)).to(torch.bfloat16)
    v_new = (torch.randn(B * n, Hkv, D, generator=g, device=device) / math.sqrt(D)).to(torch.bfloat16)
    g.manual_seed(seed + 3)
    logits = (torch.randn(B * n, a.vocab, generator=g, device=device) * 3.0).to(torch.bfloat16)
    # plant: each row's children get logits near the row max (long accepted paths)
    par_t = torch.from_numpy(par.astype(np.int64))
    rows = torch.arange(B * n)
    child = rows[par_t >= 0]
    parent_row = (torch.from_numpy(indptr[:-1].astype(np.int64)).repeat_interleave(n))[par_t >= 0] + par_t[par_t >= 0]
    ctok = torch.from_numpy(tok.astype(np.int64))[child]
    rmax = logits.float().amax(dim=1)
    boost = torch.rand(child.numel(), generator=torch.Generator().manual_seed(seed + 4)) * 3.0 - 0.5
    logits[parent_row.to(device), ctok.to(device)] = (rmax[parent_row.to(device)] + boost.to(device)).to(torch.bfloat16)

    dev_i32 = lambda x: torch.as_tensor(np.ascontiguousarray(x), dtype=torch.int32, device=device)
    # the per-step tree inputs in one buffer (parents | tokens | draft probabilities), so a step's
    # host-to-device transfer is one copy
    T = B * n
    tree_in = torch.empty(3 * T, dtype=torch.int32, device=device)
    tree_in[:T] = dev_i32(par)
    tree_in[T:2 * T] = dev_i32(tok)
    tree_in[2 * T:] = torch.as_tensor(dp, dtype=torch.float32, device=device).view(torch.int32)
    W = dict(
        trees=trees, n=n, kv_len=kv_len, layer=layer, pool=layer.view(1, *layer.shape), q=q, k_new=k_new,
        v_new=v_new, logits=logits, tree_in=tree_in,
        qo_indptr=dev_i32(indptr), parents=tree_in[:T], tokens=tree_in[T:2 * T],
        draft_probs=tree_in[2 * T:].view(torch.float32),
        page_indptr=dev_i32(np.arange(B + 1) * pages_per), page_indices=perm.contiguous(),
        last_page_len=dev_i32(np.full(B, (kv_len - 1) % pl + 1)), seq_lens=dev_i32(np.full(B, kv_len)),
        offsets=dev_i32(np.full(B, P)), mask_words=K.mask_words_for(n),
        host=dict(parents=par, tokens=tok, draft_probs=dp, indptr=indptr),
    )
    W["out"] = torch.empty_like(q)
    # the per-step results in one buffer (tokens | hidden indices | counts): one device-to-host copy
    res = torch.empty(2 * B * n + 4 * B, dtype=torch.int32, device=device)
    W["res"] = res
    W["ot"] = res[:B * n].view(B, n)
    W["oh"] = res[B * n:2 * B * n].view(B, n)
    W["oc"] = res[2 * B * n:].view(B, 4)
    W["bits"] = torch.empty(B * n, W["mask_words"], dtype=torch.int64, device=device)
    W["bi"] = torch.empty(B * n, dtype=torch.int32, device=device)
    W["pos"] = torch.empty(B * n, dtype=torch.int32, device=device)
    return W


class Step:
    """The verification step as raw C-ABI launches on the current stream.  The
    argument tuples are built once (every buffer stays in place), so a step
    costs the host only the three or four foreign calls."""

    def __init__(self, a, W, device, philox_seed=5):
        import torch
        from parallel_tree_spec_b200 import _lib, kernels as K
        self.a, self.W, self.K, self.L = a, W, K, _lib.lib()
        self.dev = device
        s = self.stream = torch.cuda.current_stream(device).cuda_stream
        B, n = a.batch, W["n"]
        L = self.L
        self.acc_ws = K.workspace(device, "accept", L.pts_accept_workspace_size(B * n, a.vocab))
        self.attn_ws = K.workspace(device, "attn", max(256, L.pts_tree_attn_workspace_size(
            B, B * n, a.hq, 128, W["kv_len"])))
        self.philox_seed = philox_seed
        self.step_index = 0
        # this library's launches per step: tree preparation with the append, attention (one
        # launch at the benchmark shapes, where one CTA per unit is the schedule chosen), the
        # acceptance's workspace zeroing and the acceptance itself (top-p: statistics, then the
        # nucleus pass with the walks)
        self.launches_per_step = 4 + (1 if (a.mode == "traversal" and a.top_p < 1.0) else 0)
        pool, lay, P, x = W["pool"], W["layer"], W["page_indptr"], W["logits"]
        self.compact = _lib.KvCompactArgs(pool.data_ptr(), 1, lay.shape[0], 16, a.hkv, 128, 2, P.data_ptr(),
                                          W["page_indices"].data_ptr(), W["offsets"].data_ptr(), None, None)
        self.prep = (L.pts_tree_prepare_append,
                     (W["parents"].data_ptr(), W["qo_indptr"].data_ptr(), W["seq_lens"].data_ptr(), B,
                      W["mask_words"], W["bits"].data_ptr(), W["bi"].data_ptr(), W["pos"].data_ptr(),
                      W["k_new"].data_ptr(), W["v_new"].data_ptr(), a.hkv * 128, a.hkv * 128, lay.data_ptr(),
                      P.data_ptr(), W["page_indices"].data_ptr(), B * n, a.hkv, 128, 16, lay.shape[0], 2, s))
        self.attn = (L.pts_tree_attn_run,
                     (W["q"].data_ptr(), lay.data_ptr(), W["qo_indptr"].data_ptr(), P.data_ptr(),
                      W["page_indices"].data_ptr(), W["last_page_len"].data_ptr(), W["bits"].data_ptr(),
                      W["mask_words"], W["out"].data_ptr(), B, B * n, n, W["kv_len"], a.hq, a.hkv, 128, 16,
                      lay.shape[0], 1.0 / math.sqrt(128), self.attn_ws.data_ptr(), self.attn_ws.numel(), s))
        if a.mode == "traversal":
            # acceptance; each walk then compacts its request's accepted KV in the same launch
            self.acc_head = (x.data_ptr(), x.stride(0), W["qo_indptr"].data_ptr(), W["parents"].data_ptr(),
                             W["tokens"].data_ptr(), W["draft_probs"].data_ptr(), B, B * n, a.vocab, n, -1,
                             a.temperature, a.top_p, 0, self.philox_seed)
            self.acc_tail = (W["ot"].data_ptr(), W["oh"].data_ptr(), W["oc"].data_ptr(), n, self.acc_ws.data_ptr(),
                             self.acc_ws.numel(), ctypes.byref(self.compact), s)
        else:
            # greedy step: the walks reduce the rows on their accepted paths only (the path
            # chain) and compact their requests' KV in the same launch
            self.acc = (L.pts_accept_greedy_compact,
                        (x.data_ptr(), x.stride(0), W["qo_indptr"].data_ptr(), W["parents"].data_ptr(),
                         W["tokens"].data_ptr(), B, B * n, a.vocab, n, -1, W["ot"].data_ptr(), W["oh"].data_ptr(),
                         W["oc"].data_ptr(), n, self.acc_ws.data_ptr(), self.acc_ws.numel(),
                         ctypes.byref(self.compact), s))

    def run(self, ev=None):
        from parallel_tree_spec_b200._lib import check
        check(self.prep[0](*self.prep[1]), "prepare+append")
        if ev is not None:
            ev[0].record()
        check(self.attn[0](*self.attn[1]), "attention")
        if ev is not None:
            ev[1].record()
        if self.a.mode == "traversal":
            check(self.L.pts_accept_traversal_compact(*self.acc_head, self.step_index, *self.acc_tail),
                  "accept+compact")
        else:
            check(self.acc[0](*self.acc[1]), "accept+compact")
        if ev is not None:
            ev[2].record()
        self.step_index += 1


# ---------------------------------------------------------------- CPU (oracle port)
def _cpu_request_inputs(a, seed, r):
    """Request r's inputs of the CPU sample (seeded per request, so every
    worker builds the same inputs for the same request)."""
    from oracle import attention as oatt
    from parallel_tree_spec_b200 import workload as wl
    rng = np.random.default_rng([seed + 100, r])
    n = 1 + a.width * a.depth
    kv_len = a.prefix + n
    npg = (kv_len + 15) // 16
    t = wl.make_tree(rng, a.width, a.depth, a.vocab)
    x = wl.make_logits(rng, t, a.vocab, plant=1.0, soft=True)
    layer = (rng.standard_normal((npg, 2, 16, a.hkv, 128), dtype=np.float32) / np.sqrt(128)).astype(np.float32)
    q = rng.standard_normal((n, a.hq, 128), dtype=np.float32)
    return dict(r=r, t=t, x=x, layer=layer, q=q, mask=oatt.tree_mask(t.parents, a.prefix), npg=npg, kv_len=kv_len)


def _cpu_request_path(a, inp):
    """The path on the host for one request: attention over its prefix KV for
    every query head, acceptance over its [N, V] logits and the walk, the
    compaction of the accepted path (the NumPy restatement)."""
    from oracle import accept as oacc
    from oracle import attention as oatt
    from oracle import kv as okv
    from oracle.philox import UniformStream
    t, n = inp["t"], inp["t"].size
    oatt.tree_attention(inp["q"], inp["layer"], [list(range(inp["npg"]))], [inp["kv_len"]], [0, n], [inp["mask"]],
                        1 / math.sqrt(128))
    am, p = oacc.row_stats(inp["x"], a.temperature if a.mode == "traversal" else 1.0)
    if a.mode == "traversal":
        mb = oacc.mb_from_probs(t.parents, t.tokens, p)
        s, h, tl, al, _ = oacc.traversal_walk(t.parents, t.tokens, t.draft_probs, mb, am,
                                              UniformStream(5, 0, inp["r"]))
    else:
        s, h, tl, al = oacc.greedy_walk(t.parents, t.tokens, am)
        h = list(h)
    layer = inp["layer"].copy()
    okv.request_reorder(layer[None], list(range(inp["npg"])), inp["kv_len"], h, a.prefix + 1)


def _cpu_worker(conn, a_dict, seed, reqs):
    """One host process: builds its requests' inputs once, then runs the path
    over all of them on every "go" (single-threaded NumPy)."""
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(1)
    except Exception:
        pass
    a = argparse.Namespace(**a_dict)
    inputs = [_cpu_request_inputs(a, seed, r) for r in reqs]
    conn.send("ready")
    while conn.recv() == "go":
        for inp in inputs:
            _cpu_request_path(a, inp)
        conn.send("done")


class CpuPath:
    """The path over ``requests`` requests on the host cores: one process per
    core (started with spawn), each owning a fixed share of the requests, so a
    step's wall time is the batch over all cores."""

    def __init__(self, a, requests, seed):
        import multiprocessing as mp
        ncpu = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
        self.workers = max(1, min(ncpu, requests))
        self.requests, self.cpus = requests, ncpu
        ctx = mp.get_context("spawn")
        self.conns, self.procs = [], []
        for w in range(self.workers):
            here, there = ctx.Pipe()
            reqs = list(range(w, requests, self.workers))
            pr = ctx.Process(target=_cpu_worker, args=(there, vars(a), seed, reqs), daemon=True)
            pr.start()
            self.conns.append(here)
            self.procs.append(pr)
        for c in self.conns:
            assert c.recv() == "ready"

    def step(self) -> float:
        t0 = time.perf_counter()
        for c in self.conns:
            c.send("go")
        for c in self.conns:
            assert c.recv() == "done"
        return time.perf_counter() - t0

    def close(self):
        for c in self.conns:
            try:
                c.send("stop")
            except Exception:
                pass
        for pr in self.procs:
            pr.join(timeout=10)


def cpu_threads():
    """Host cores available to this process."""
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    n = 1 + a.width * a.depth
    requests = a.batch * max(world, a.gpus)                        # the same global batch as the GPU arm
    cpu = CpuPath(a, requests, a.seed)
    try:
        for _ in range(max(1, min(a.warmup, 3))):
            cpu.step()
        times = []
        t_start = time.perf_counter()
        for _ in range(max(1, a.steps)):
            times.append(cpu.step())
            if time.perf_counter() - t_start > a.cpu_time_budget:
                break
    finally:
        cpu.close()
    step_s = statistics.mean(times)
    value = 1.0 / step_s
    rec = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": a.gpus, "steps": len(times),
        "warmup": a.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": workload_name(a), "global_batch": requests, "prefix": a.prefix, "tree_rows": n,
                   "vocab": a.vocab, "mode": a.mode},
        "tokens_per_s": value * requests * n,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu.workers, "host_cpus": cpu.cpus, "kind": "port",
                         "sample": f"every step is the whole {requests}-request batch (attention for all heads, "
                                   f"acceptance over [{n}, {a.vocab}] per request, compaction) on {cpu.workers} "
                                   f"single-threaded host processes; {len(times)} timed steps"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(rec), flush=True)
    return 0


# ---------------------------------------------------------------- GPU arm
def time_steps(run, steps, n_events=3):
    """Time ``steps`` calls of ``run(ev)`` on the current stream: total CUDA-event
    milliseconds and the per-step event lists (ev[0..n_events-1] recorded by run)."""
    import torch
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_events)] for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for i in range(steps):
        run(evs[i])
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end), evs


def mode_record(a, W, device, mode, top_p, steps, peak):
    """One more acceptance mode of the same workload (greedy, or traversal with
    a top-p target) timed on its own: steps/s, kernel times and the HBM
    fraction of the slower hot kernel."""
    import copy
    b = copy.copy(a)
    b.mode, b.top_p = mode, top_p
    st = Step(b, W, device)
    for _ in range(3):
        st.run()
    # the steps back to back (an event between two kernels keeps the second from
    # starting early as a programmatic dependent), then the per-kernel times
    # from a second run with events between the kernels
    el, _ = time_steps(lambda ev: st.run(), steps, n_events=0)
    _, evs = time_steps(st.run, steps)
    attn = statistics.mean(e[0].elapsed_time(e[1]) for e in evs) * 1e3
    acc = statistics.mean(e[1].elapsed_time(e[2]) for e in evs) * 1e3
    ab = algorithmic_bytes(b)
    if mode == "greedy":
        # the greedy walks read the rows of their accepted paths only: the root and each accepted node
        ab["accept"] = float((W["oc"][:, 2].double() + 1).sum().item()) * a.vocab * 2
    dom, dom_bytes, dom_us = (("tree_attn_kernel", ab["attention"], attn) if attn >= acc
                              else ("acceptance", ab["accept"], acc))
    return {"workload": workload_name(b), "value": steps / (el / 1e3), "unit": UNIT, "steps": steps,
            "ms_per_step": el / steps,
            "kernels_us": {"tree_attn": attn, "accept_with_compaction": acc},
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": dom_bytes / (dom_us * 1e-6) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": dom_bytes / (dom_us * 1e-6) / 1e9 / peak,
                         "accept_frac": ab["accept"] / (acc * 1e-6) / 1e9 / peak},
            "accept_len_mean": float(W["oc"][:, 2].float().mean().item())}


def run_b200(a):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise RuntimeError("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    from parallel_tree_spec_b200 import _lib
    _lib.lib()
    W = build_workload(a, device, a.seed + 1000 * rank)
    step = Step(a, W, device)
    for _ in range(max(3, a.warmup)):
        step.run()
    torch.cuda.synchronize()

    sampler = ClockSampler(local).start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_host0 = time.perf_counter()
    # the steps back to back, no events between their kernels (an event between two
    # kernels would keep the second from starting early as a programmatic dependent)
    elapsed_ms, _ = time_steps(lambda ev: step.run(), a.steps, n_events=0)
    t_host1 = time.perf_counter()
    # per-kernel times from a second run with events between the kernels
    _, evs = time_steps(step.run, min(a.steps, 50))
    if world > 1:
        dist.barrier()
    sampler.stop()
    attn_ms = [e[0].elapsed_time(e[1]) for e in evs]
    acc_ms = [e[1].elapsed_time(e[2]) for e in evs]
    elapsed_ms, = over_ranks([elapsed_ms], "max", device)          # the slowest rank's time
    ms_per_step = elapsed_ms / a.steps
    value = world * a.steps / (elapsed_ms / 1e3)
    accept_len = float(W["oc"][:, 2].float().mean().item())

    # e2e: tree inputs from pinned host memory, results back to the host every step
    e2e = run_e2e(a, W, step, device)
    e2e["value"] = over_ranks([e2e["value"]], "min", device)[0] * world   # the slowest rank's rate, N times

    ab = algorithmic_bytes(a)
    if a.mode == "greedy":
        # the greedy walks read the rows of their accepted paths only: the root and each accepted node
        ab["accept"] = float((W["oc"][:, 2].double() + 1).sum().item()) * a.vocab * 2
        ab["step"] = ab["kv_read"] + ab["q_o"] + ab["append"] + ab["accept"] + ab["compact"]
    peak, peak_kind = measured_peaks()
    tpeak, tpeak_kind = measured_tensor_peak()
    k_attn = statistics.mean(attn_ms) * 1e-3
    k_acc = statistics.mean(acc_ms) * 1e-3
    dom = "tree_attn_kernel" if k_attn >= k_acc else "accept_stream_kernel"
    dom_bytes = ab["attention"] if dom == "tree_attn_kernel" else ab["accept"]
    dom_s = max(k_attn, k_acc)
    achieved = dom_bytes / dom_s / 1e9
    traffic = traffic_table().get(dom)
    n = W["n"]
    sub_steps = max(10, min(a.steps, 50))
    sub = {}
    if not a.no_sub:
        # the other acceptance modes of the same workload (greedy; traversal with top-p 0.9)
        sub["greedy"] = mode_record(a, W, device, "greedy", 1.0, sub_steps, peak)
        sub["traversal_top_p_0.9"] = mode_record(a, W, device, "traversal", 0.9, sub_steps, peak)
        if world == 1:
            sub["config3_path"] = config3_record(a, device, sub_steps, peak)
            sub["lmhead"] = lmhead_record(a, device, 10, tpeak)
            sub["beam_select"] = beam_record(a, device, 50)
            sub["config4_sparse"] = sparse_record(a, device, sub_steps, peak)
            sub["flashinfer_attention"] = flashinfer_record(a, W, device, 20, k_attn * 1e6)
        else:
            sub["tp"] = tp_record(a, world, rank, device, sub_steps)
            sub["strong"] = strong_record(a, world, rank, device, sub_steps)
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cp = CpuPath(a, a.batch, a.seed)
        try:
            cp.step()
            ts = [cp.step() for _ in range(2)]
        finally:
            cp.close()
        cpu = {"value": 1.0 / statistics.mean(ts), "unit": UNIT, "cores": cp.workers, "host_cpus": cp.cpus,
               "kind": "port",
               "sample": f"the whole {a.batch}-request step (attention for all heads, acceptance over [{n}, "
                         f"{a.vocab}] per request, compaction) on {cp.workers} single-threaded host processes, "
                         f"mean of 2 timed steps"}
    flops = 4.0 * a.batch * a.hq * n * W["kv_len"] * 128
    rec = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": workload_name(a), "global_batch": a.batch * world, "prefix": a.prefix,
                   "tree_rows": n, "vocab": a.vocab, "mode": a.mode, "parallelism": f"batch-sharded x{world}",
                   "l2": "inputs larger than L2 every step (KV 273 MB, logits 267 MB)"},
        "tokens_per_s": value * a.batch * n,
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": traffic, "algorithmic_bytes_per_launch": dom_bytes,
                     "attention_tensor": {"flops_per_launch": flops, "achieved_tflops": flops / k_attn / 1e12,
                                          "peak_tflops": tpeak, "peak_kind": tpeak_kind,
                                          "frac": flops / k_attn / 1e12 / tpeak},
                     "attention_hbm_frac": ab["attention"] / k_attn / 1e9 / peak,
                     "accept_hbm_frac": ab["accept"] / k_acc / 1e9 / peak},
        "step_roofline": {"algorithmic_bytes": ab["step"], "achieved_gbs": ab["step"] / (ms_per_step * 1e-3) / 1e9,
                          "frac": ab["step"] / (ms_per_step * 1e-3) / 1e9 / peak},
        "kernels_us": {"tree_attn": k_attn * 1e6, "accept_with_compaction": k_acc * 1e6},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": step.launches_per_step * a.steps,
        "clocks": sampler.summary(t_host0, t_host1),
        "accept_len_mean": accept_len,
        "sub": sub,
    }
    if rank == 0:
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_e2e(a, W, step, device):
    """Same step through host buffers: the tree inputs (parents, tokens, draft
    probabilities) are copied from pinned host memory and the accepted
    tokens / hidden indices / counts are read back every step."""
    import torch
    h = W["host"]
    hin = torch.cat([torch.from_numpy(h["parents"].astype(np.int32)), torch.from_numpy(h["tokens"].astype(np.int32)),
                     torch.from_numpy(h["draft_probs"].astype(np.float32)).view(torch.int32)]).pin_memory()
    hres = torch.empty_like(W["res"], device="cpu").pin_memory()
    h2d = hin.numel() * 4
    d2h = hres.numel() * 4

    stream = torch.cuda.current_stream(device)
    tree_in, res = W["tree_in"], W["res"]

    def one():
        tree_in.copy_(hin, non_blocking=True)
        step.run()
        hres.copy_(res, non_blocking=True)
        stream.synchronize()

    for _ in range(3):
        one()
    t0 = time.perf_counter()
    for _ in range(a.e2e_steps):
        one()
    dt = time.perf_counter() - t0
    return {"value": a.e2e_steps / dt, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}


# ---------------------------------------------------------------- tensor-parallel step
def tp_record(a, world, rank, dev, steps):
    """Tensor-parallel verification step of a 70B-shaped target: every rank
    holds 8/N of the 8 KV heads (64/N query heads) and 1/N of the vocabulary;
    attention is local, acceptance exchanges per-row partials and tie indices
    over NCCL, and every rank walks the same trees.  Batch 64, prefixes drawn
    uniformly from [512, 8192], 65-row trees, random N(0, 3) logits (no
    planting: nearly every node is rejected, the longest walks).  Every rank
    calls this with the same arguments (it runs collectives)."""
    import torch
    from parallel_tree_spec_b200 import _lib, kernels as K
    from parallel_tree_spec_b200 import workload as wl
    from parallel_tree_spec_b200._lib import check

    if 8 % world:
        raise ValueError("--tp needs 1, 2, 4 or 8 ranks")
    L = _lib.lib()
    B, V, D, pl = 64, a.vocab, 128, 16
    hq, hkv = 64 // world, 8 // world
    rng = np.random.default_rng(a.seed + 7)                       # the same on every rank
    trees = [wl.make_tree(rng, 8, 8, V) for _ in range(B)]
    n = trees[0].size
    prefix = rng.integers(512, 8193, size=B)
    indptr, par, tok, dp = wl.stack_trees(trees)
    kv_lens = prefix + n
    npg = (kv_lens + pl - 1) // pl
    page_indptr = np.concatenate([[0], np.cumsum(npg)]).astype(np.int32)
    max_pages = int(page_indptr[-1]) + 16
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed + 100 + rank)
    layer = torch.empty(max_pages, 2, pl, hkv, D, dtype=torch.bfloat16, device=dev).normal_(0, 1 / math.sqrt(D),
                                                                                          generator=g)
    perm = torch.randperm(max_pages, generator=g, device=dev)[: page_indptr[-1]].to(torch.int32)
    T = B * n
    q = torch.randn(T, hq, D, generator=g, device=dev).to(torch.bfloat16)
    kn = (torch.randn(T, hkv, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
    vn = (torch.randn(T, hkv, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
    step_v = V // world
    v0, v1 = rank * step_v, (V if rank == world - 1 else (rank + 1) * step_v)
    xs = (torch.randn(T, v1 - v0, generator=g, device=dev) * 3.0).to(torch.bfloat16)
    d = lambda x: torch.as_tensor(np.ascontiguousarray(x), dtype=torch.int32, device=dev)
    qo, parents, tokens = d(indptr), d(par), d(tok)
    draft = torch.as_tensor(dp, device=dev)
    pind, lastp, seqlens, offs = d(page_indptr), d((kv_lens - 1) % pl + 1), d(kv_lens), d(prefix)
    mw = K.mask_words_for(n)
    bits = torch.empty(T, mw, dtype=torch.int64, device=dev)
    bi = torch.empty(T, dtype=torch.int32, device=dev)
    pos = torch.empty(T, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    attn_ws = attn_workspace(dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    pool = layer.view(1, *layer.shape)

    gather = K.gather_shards

    res = {}

    def one(ev=None):
        check(L.pts_tree_prepare_append(parents.data_ptr(), qo.data_ptr(), seqlens.data_ptr(), B, mw,
                                        bits.data_ptr(), bi.data_ptr(), pos.data_ptr(), kn.data_ptr(), vn.data_ptr(),
                                        hkv * D, hkv * D, layer.data_ptr(), pind.data_ptr(), perm.data_ptr(), T, hkv,
                                        D, pl, max_pages, 2, s), "prepare+append")
        if ev is not None:
            ev[0].record()
        check(L.pts_tree_attn_run(q.data_ptr(), layer.data_ptr(), qo.data_ptr(), pind.data_ptr(), perm.data_ptr(),
                                  lastp.data_ptr(), bits.data_ptr(), mw, out.data_ptr(), B, T, n, int(kv_lens.max()),
                                  hq, hkv, D, pl, max_pages, 1 / math.sqrt(D), attn_ws.data_ptr(), attn_ws.numel(),
                                  s), "attention")
        if ev is not None:
            ev[1].record()
        parts, tk = K.accept_shard_partials(xs, v0, qo, parents, tokens)
        stats, tkm = K.accept_merge_shards(gather(parts), gather(tk))
        ties = gather(K.accept_shard_ties(xs, v0, stats))
        ot, oh, oc = K.accept_walk_merged(stats, tkm, ties, V, qo, parents, tokens, draft, seed=5, offset=0,
                                          max_nodes=n)
        if ev is not None:
            ev[2].record()
        K.kv_compact(pool, pind, perm, oh, oc, offs)
        res["oc"] = oc

    for _ in range(3):
        one()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    el, _ = time_steps(lambda ev: one(), steps, n_events=0)   # back to back; kernel times below
    _, evs = time_steps(one, steps)
    attn = statistics.mean(e[0].elapsed_time(e[1]) for e in evs) * 1e3
    acc = statistics.mean(e[1].elapsed_time(e[2]) for e in evs) * 1e3
    el, attn, acc = over_ranks([el, attn, acc], "max", dev)
    if world > 1:
        counts = gather(res["oc"])
        same = bool(all(torch.equal(counts[0], counts[k]) for k in range(world)))
    else:
        same = True
    return {
        "metric": "tree-verify steps/s, tensor-parallel (vocabulary and KV heads split over the ranks)",
        "value": steps / (el / 1e3), "unit": UNIT, "n_gpus": world, "steps": steps,
        "ms_per_step": el / steps, "scaling": "strong",
        "workload": "tensor-parallel tree-verify step: B=64 requests, prefixes U[512, 8192], tree rows 65, Hq=64, "
                    "Hkv=8, D=128, page 16, vocab 128256, traversal T=1.0, one layer",
        "parallelism": f"tp{world} (KV heads and vocabulary)",
        "tokens_per_s": steps / (el / 1e3) * B * n,
        "kernels_us": {"tree_attn": attn, "accept_with_exchange": acc},
        "ranks_agree": same,
    }


def config3_record(a, dev, steps, peak):
    """The path of a Llama-3-8B-shaped verify step: B=32 requests, prefixes
    U[1024, 2048], 49-row trees (width 8, depth 6), 32 query / 8 KV heads,
    32 attention layers (per layer: the tree K/V append and the tree
    attention; layer 0's append shares a launch with the tree masks and
    positions), then traversal acceptance at T=0.8 over [1568, 128256] bf16
    logits with the accepted paths' KV compacted in all 32 layers.  The model's
    projections, MLPs, norms and lm_head (library GEMMs, outside the path) do
    not run: every layer's q and new k/v are seeded synthetic tensors."""
    import torch
    from parallel_tree_spec_b200 import _lib, kernels as K
    from parallel_tree_spec_b200 import workload as wl
    from parallel_tree_spec_b200._lib import check

    L, B, Hq, Hkv, D, pl, V, temp = 32, 32, 32, 8, 128, 16, a.vocab, 0.8
    lib = _lib.lib()
    rng = np.random.default_rng(a.seed + 31)
    trees = [wl.make_tree(rng, 8, 6, V) for _ in range(B)]
    n = trees[0].size
    prefix = rng.integers(1024, 2049, size=B)
    indptr, par, tok, dp = wl.stack_trees(trees)
    kv_lens = prefix + n
    npg = (kv_lens + pl - 1) // pl
    page_indptr = np.concatenate([[0], np.cumsum(npg)]).astype(np.int32)
    max_pages = int(page_indptr[-1]) + 16
    T = B * n
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed + 33)
    pool = torch.empty(L, max_pages, 2, pl, Hkv, D, dtype=torch.bfloat16, device=dev).normal_(0, 1 / math.sqrt(D),
                                                                                            generator=g)
    perm = torch.randperm(max_pages, generator=g, device=dev)[: page_indptr[-1]].to(torch.int32)
    q = torch.randn(L, T, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    kn = (torch.randn(L, T, Hkv, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
    vn = (torch.randn(L, T, Hkv, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
    x = (torch.randn(T, V, generator=g, device=dev) * 3.0).to(torch.bfloat16)
    # children's tokens near their parent row's max, so walks go deep
    prow = np.concatenate([indptr[b] + np.maximum(par[indptr[b]:indptr[b + 1]], 0) for b in range(B)])
    child = np.nonzero(par >= 0)[0]
    pr_t = torch.from_numpy(prow[child].astype(np.int64)).to(dev)
    tk_t = torch.from_numpy(tok[child].astype(np.int64)).to(dev)
    boost = torch.rand(child.size, generator=g, device=dev) * 3.0 - 0.5
    x[pr_t, tk_t] = (x[pr_t].float().amax(dim=1) + boost).to(torch.bfloat16)
    d = lambda v: torch.as_tensor(np.ascontiguousarray(v), dtype=torch.int32, device=dev)
    qo, parents, tokens = d(indptr), d(par), d(tok)
    draft = torch.as_tensor(dp, device=dev)
    pind, lastp, seqlens, offs = d(page_indptr), d((kv_lens - 1) % pl + 1), d(kv_lens), d(prefix)
    mw = K.mask_words_for(n)
    bits = torch.empty(T, mw, dtype=torch.int64, device=dev)
    bi = torch.empty(T, dtype=torch.int32, device=dev)
    pos = torch.empty(T, dtype=torch.int32, device=dev)
    out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=dev)
    attn_ws = attn_workspace(dev)
    acc_ws = K.workspace(dev, "accept", lib.pts_accept_workspace_size(T, V))
    ot = torch.empty(B, n, dtype=torch.int32, device=dev)
    oh = torch.empty(B, n, dtype=torch.int32, device=dev)
    oc = torch.empty(B, 4, dtype=torch.int32, device=dev)
    cargs = _lib.KvCompactArgs(pool.data_ptr(), L, max_pages, pl, Hkv, D, 2, pind.data_ptr(), perm.data_ptr(),
                               offs.data_ptr(), None, None)
    s = torch.cuda.current_stream(dev).cuda_stream
    layer_bytes = pool[0].numel() * 2
    state = {"off": 0}

    def one(ev=None):
        if ev is not None:
            ev[0].record()
        for l in range(L):
            lay = pool.data_ptr() + l * layer_bytes
            if l == 0:
                check(lib.pts_tree_prepare_append(parents.data_ptr(), qo.data_ptr(), seqlens.data_ptr(), B, mw,
                                                  bits.data_ptr(), bi.data_ptr(), pos.data_ptr(), kn[0].data_ptr(),
                                                  vn[0].data_ptr(), Hkv * D, Hkv * D, lay, pind.data_ptr(),
                                                  perm.data_ptr(), T, Hkv, D, pl, max_pages, 2, s), "prepare+append")
            else:
                check(lib.pts_kv_append(kn[l].data_ptr(), vn[l].data_ptr(), Hkv * D, Hkv * D, lay, bi.data_ptr(),
                                        pos.data_ptr(), pind.data_ptr(), perm.data_ptr(), T, Hkv, D, pl, max_pages, 2,
                                        s), "append")
            check(lib.pts_tree_attn_run(q[l].data_ptr(), lay, qo.data_ptr(), pind.data_ptr(), perm.data_ptr(),
                                        lastp.data_ptr(), bits.data_ptr(), mw, out.data_ptr(), B, T, n,
                                        int(kv_lens.max()), Hq, Hkv, D, pl, max_pages, 1 / math.sqrt(D),
                                        attn_ws.data_ptr(), attn_ws.numel(), s), "attention")
        if ev is not None:
            ev[1].record()
        check(lib.pts_accept_traversal_compact(x.data_ptr(), x.stride(0), qo.data_ptr(), parents.data_ptr(),
                                               tokens.data_ptr(), draft.data_ptr(), B, T, V, n, -1, temp, 1.0, 0, 5,
                                               state["off"], ot.data_ptr(), oh.data_ptr(), oc.data_ptr(), n,
                                               acc_ws.data_ptr(), acc_ws.numel(), ctypes.byref(cargs), s),
              "accept+compact")
        state["off"] += 1
        if ev is not None:
            ev[2].record()

    for _ in range(3):
        one()
    el, _ = time_steps(lambda ev: one(), steps, n_events=0)   # back to back; kernel times below
    _, evs = time_steps(one, steps)
    layers_us = statistics.mean(e[0].elapsed_time(e[1]) for e in evs) * 1e3
    acc_us = statistics.mean(e[1].elapsed_time(e[2]) for e in evs) * 1e3
    kv_read = int(np.sum(kv_lens)) * Hkv * D * 2 * 2 * L
    qo_bytes = 2 * T * Hq * D * 2 * L
    append = T * Hkv * D * 2 * 2 * L
    logit_bytes = T * V * 2
    return {"workload": f"config-3 verify-step path: B={B} requests, prefixes U[1024, 2048], tree rows {n} (width 8, "
                        f"depth 6), Hq={Hq}, Hkv={Hkv}, D=128, page 16, {L} attention layers, vocab {V}, traversal "
                        f"T={temp}, compaction in all {L} layers; model GEMMs excluded",
            "value": steps / (el / 1e3), "unit": UNIT, "steps": steps, "ms_per_step": el / steps,
            "tokens_per_s": steps / (el / 1e3) * T,
            "kernels_us": {"append_and_attention_32_layers": layers_us, "accept_with_compaction": acc_us},
            "roofline": {"bound": "hbm", "peak": peak, "unit": "GB/s",
                         "layers_frac": (kv_read + qo_bytes + append) / (layers_us * 1e-6) / 1e9 / peak,
                         "accept_frac": logit_bytes / (acc_us * 1e-6) / 1e9 / peak,
                         "step_frac": (kv_read + qo_bytes + append + logit_bytes) / (el / steps * 1e-3) / 1e9 / peak},
            "accept_len_mean": float(oc[:, 2].float().mean().item())}


def beam_record(a, dev, steps):
    """One decode step's candidate selection of the draft beam search
    (beam_search.py:549-561) for 8 beams over the 128256-entry vocabulary
    (bf16 logits, T = 1): the reference's torch chain (softmax, + 1e-10,
    log, + the beams' cumulative scores, flattened topk, the picks'
    probabilities) against pts_beam_select; the same picks either way."""
    import torch
    from parallel_tree_spec_b200 import kernels as K

    Kb, V = 8, a.vocab
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed + 51)
    x = (torch.randn(Kb, V, generator=g, device=dev) * 3.0).to(torch.bfloat16)
    cum = -torch.rand(Kb, generator=g, device=dev) * 4.0

    def chain():
        probs = torch.softmax(x / 1.0, dim=-1)
        flat = (cum[:, None] + torch.log(probs + 1e-10)).reshape(-1)
        sc, ids = flat.topk(Kb)
        return sc, ids, probs.reshape(-1)[ids]

    def fused():
        return K.beam_select(x, Kb, 1.0, cum)

    out = {"workload": f"beam-search selection: {Kb} beams x vocabulary {V}, bf16 logits, T=1.0", "unit": "us"}
    for name, fn in (("torch_chain", chain), ("beam_select", fused)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        out[name + "_us"] = e0.elapsed_time(e1) * 1e3 / steps
    ref, got = chain(), fused()
    out["same_picks"] = bool(torch.equal(ref[1], got[1]) and torch.equal(ref[0], got[0]))
    return out


def lmhead_record(a, dev, steps, tpeak):
    """The lm_head of the benchmark step's 16 x 65 tree rows (hidden 4096,
    vocabulary 128256, bf16, random weights) followed by traversal acceptance
    at T=1.0, three ways: torch.matmul (cuBLAS) writing the logits + the
    acceptance kernel; this library's tcgen05 GEMM writing the logits + the
    acceptance kernel; the same GEMM with the acceptance statistics in its
    epilogue (no logits in memory) + the walks (pts_lmhead_accept)."""
    import torch
    from parallel_tree_spec_b200 import kernels as K
    from parallel_tree_spec_b200 import workload as wl

    B, H, V = a.batch, 4096, a.vocab
    rng = np.random.default_rng(a.seed + 41)
    trees = [wl.make_tree(rng, a.width, a.depth, V) for _ in range(B)]
    n = trees[0].size
    indptr, par, tok, dp = wl.stack_trees(trees)
    d = lambda v: torch.as_tensor(np.ascontiguousarray(v), device=dev)
    ind, par, tok, dp = d(indptr), d(par), d(tok), d(dp)
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed + 43)
    hidden = torch.randn(B * n, H, generator=g, device=dev).to(torch.bfloat16)
    weight = (torch.randn(V, H, generator=g, device=dev) * (3.0 / H ** 0.5)).to(torch.bfloat16)
    flops = 2.0 * B * n * V * H

    def cublas(ev=None):
        x = torch.matmul(hidden, weight.t())
        if ev is not None:
            ev[0].record()
        K.accept_traversal(x, ind, par, tok, dp, seed=5, offset=0, max_nodes=n)

    def unfused(ev=None):
        x = K.lmhead_logits(hidden, weight)
        if ev is not None:
            ev[0].record()
        K.accept_traversal(x, ind, par, tok, dp, seed=5, offset=0, max_nodes=n)

    def fused(ev=None):
        K.lmhead_accept(hidden, weight, ind, par, tok, dp, method="traversal", seed=5, offset=0, max_nodes=n,
                        fallback=False)
        if ev is not None:
            ev[0].record()

    out = {"workload": f"lm_head of {B} x {n} tree rows (hidden {H}, vocabulary {V}, bf16) + traversal "
                       f"acceptance T=1.0", "flops": flops, "unit": "us"}
    for name, fn in (("cublas_gemm_then_accept", cublas), ("gemm_then_accept", unfused),
                     ("fused_gemm_statistics", fused)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        starts = []
        for _ in range(steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            em = torch.cuda.Event(enable_timing=True)
            e0.record()
            fn([em])
            e1.record()
            starts.append((e0, em, e1))
        torch.cuda.synchronize()
        total = statistics.mean(e0.elapsed_time(e1) for e0, em, e1 in starts) * 1e3
        gemm = statistics.mean(e0.elapsed_time(em) for e0, em, e1 in starts) * 1e3
        rec = {"total_us": total}
        if name != "fused_gemm_statistics":
            rec["gemm_us"] = gemm
            rec["accept_us"] = total - gemm
        rec["tensor_frac_of_total"] = flops / (total * 1e-6) / 1e12 / tpeak
        out[name] = rec
    out["tensor_peak_tflops"] = tpeak
    return out


def flashinfer_record(a, W, dev, steps, ours_us):
    """The reference's own attention kernel on the benchmark workload: FlashInfer's
    BatchPrefillWithPagedKVCacheWrapper with the tree masks as a custom boolean
    mask (flashinfer/attention_wrapper.py:131-144,250-252), the same queries and
    paged cache; its time beside this library's kernel, and the largest output
    difference.  None where FlashInfer cannot be imported or built."""
    import torch
    from parallel_tree_spec_b200._lib import check
    st = Step(a, W, dev)                                      # the tree rows' K/V back in place, fresh output
    check(st.prep[0](*st.prep[1]), "prepare+append")
    check(st.attn[0](*st.attn[1]), "attention")
    try:
        import flashinfer
        from oracle import attention as oatt
        mask = torch.cat([torch.from_numpy(oatt.tree_mask(t.parents, a.prefix).reshape(-1)) for t in W["trees"]])
        ws = torch.empty(256 << 20, dtype=torch.int8, device=dev)
        w = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, kv_layout="NHD")
        w.plan(W["qo_indptr"], W["page_indptr"], W["page_indices"], W["last_page_len"], a.hq, a.hkv, 128, 16,
               custom_mask=mask.to(dev), q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16,
               sm_scale=1.0 / math.sqrt(128))
        o = w.run(W["q"], W["layer"])
    except Exception as e:
        return {"unavailable": str(e)[:200]}
    ref_out = W["out"].float()
    diff = float((o.float() - ref_out).abs().max())
    for _ in range(3):
        w.run(W["q"], W["layer"])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        w.run(W["q"], W["layer"])
    e1.record()
    torch.cuda.synchronize()
    fi_us = e0.elapsed_time(e1) / steps * 1e3
    return {"kernel": f"flashinfer {flashinfer.__version__} BatchPrefillWithPagedKVCacheWrapper, custom_mask",
            "flashinfer_us": fi_us, "tree_attn_us": ours_us, "speedup": fi_us / ours_us,
            "max_abs_diff_vs_tree_attn": diff}


def strong_record(a, world, rank, dev, steps):
    """Strong scaling of the batch-sharded step: the 16 requests of the
    benchmark workload split over the ranks (16/N each).  At N >= 4 a rank's KV
    and logits fit in L2, so a 256 MB buffer is written between steps, outside
    the timed events.  Every rank calls this (it reduces over ranks)."""
    import copy
    import torch
    b = copy.copy(a)
    b.batch = max(1, a.batch // world)
    W = build_workload(b, dev, a.seed + 5000 + 1000 * rank)
    st = Step(b, W, dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(3):
        st.run()
    per = []
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        st.run()
        e1.record()
        per.append((e0, e1))
    torch.cuda.synchronize()
    ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in per)
    ms, = over_ranks([ms], "max", dev)
    return {"workload": workload_name(b).replace(f"B={b.batch} requests", f"B={a.batch} requests in total "
                                                                        f"({b.batch} per rank)"),
            "value": 1e3 / ms, "unit": UNIT, "n_gpus": world, "steps": steps, "ms_per_step": ms,
            "scaling": "strong", "l2": "256 MB written between timed steps (outside the timed events)",
            "tokens_per_s": 1e3 / ms * a.batch * W["n"]}


def run_tp(a):
    """``--tp``: the tensor-parallel step alone, one JSON line."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    sampler = ClockSampler(local).start()
    t0 = time.perf_counter()
    r = tp_record(a, world, rank, dev, a.steps)
    t1 = time.perf_counter()
    sampler.stop()
    rec = {"metric": r["metric"], "value": r["value"], "unit": UNIT, "n_gpus": world, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
           "config": {"workload": r["workload"], "parallelism": r["parallelism"]},
           "tokens_per_s": r["tokens_per_s"], "kernels_us": r["kernels_us"], "ranks_agree": r["ranks_agree"],
           "clocks": sampler.summary(t0, t1)}
    if rank == 0:
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if r["ranks_agree"] else 1


# ---------------------------------------------------------------- long-context sparse step
def sparse_record(a, dev, steps, peak):
    """Long-context verification step: 8 requests with 32768-token prefixes
    and 129-row trees (width 16, depth 8), Hq=32 / Hkv=8.  The per-KV-head
    page sets (first 4 + 64 highest root-query . key-sum scores + last 8
    prefix pages, plus the tree's pages) are selected once after the prefill
    from page key sums (timed separately); each step packs masks, appends the
    tree K/V, runs attention over the per-head page tables, greedy acceptance
    over [1032, 128256] bf16 logits and compaction."""
    import torch
    from parallel_tree_spec_b200 import _lib, kernels as K
    from parallel_tree_spec_b200 import workload as wl
    from parallel_tree_spec_b200._lib import check

    L = _lib.lib()
    B, P, Hq, Hkv, D, pl, V = 8, 32768, 32, 8, 128, 16, a.vocab
    rng = np.random.default_rng(a.seed + 11)
    trees = [wl.make_tree(rng, 16, 8, V) for _ in range(B)]
    n = trees[0].size
    indptr, par, tok, dp = wl.stack_trees(trees)
    kv_len = P + n
    npg = (kv_len + pl - 1) // pl
    max_pages = B * npg + 16
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed + 21)
    layer = torch.empty(max_pages, 2, pl, Hkv, D, dtype=torch.bfloat16, device=dev).normal_(0, 1 / math.sqrt(D),
                                                                                          generator=g)
    perm = torch.randperm(max_pages, generator=g, device=dev)[: B * npg].to(torch.int32)
    T = B * n
    q = torch.randn(T, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    kn = (torch.randn(T, Hkv, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
    vn = (torch.randn(T, Hkv, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
    x = (torch.randn(T, V, generator=g, device=dev) * 3.0).to(torch.bfloat16)
    d = lambda v: torch.as_tensor(np.ascontiguousarray(v), dtype=torch.int32, device=dev)
    qo, parents, tokens = d(indptr), d(par), d(tok)
    pind = d(np.arange(B + 1) * npg)
    lastp, seqlens, offs = d(np.full(B, (kv_len - 1) % pl + 1)), d(np.full(B, kv_len)), d(np.full(B, P))
    # page sets, once after the prefill
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(2):
        e0.record()
        ks = K.page_key_sums(layer, perm)
        hi, hx, hl = K.select_pages(ks, pind, perm, lastp, q, qo, Hkv, n_first=4, n_top=64, n_last=8,
                                    max_prefix_pages=npg)
        e1.record()
        torch.cuda.synchronize()
    select_us = e0.elapsed_time(e1) * 1e3
    sel_pages = int(hi[1].item() - hi[0].item())
    mw = K.mask_words_for(n)
    bits = torch.empty(T, mw, dtype=torch.int64, device=dev)
    bi = torch.empty(T, dtype=torch.int32, device=dev)
    pos = torch.empty(T, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    attn_ws = attn_workspace(dev)
    acc_ws = K.workspace(dev, "accept", L.pts_accept_workspace_size(T, V))
    ot = torch.empty(B, n, dtype=torch.int32, device=dev)
    oh = torch.empty(B, n, dtype=torch.int32, device=dev)
    oc = torch.empty(B, 4, dtype=torch.int32, device=dev)
    pool = layer.view(1, *layer.shape)
    cargs = _lib.KvCompactArgs(pool.data_ptr(), 1, max_pages, pl, Hkv, D, 2, pind.data_ptr(), perm.data_ptr(),
                               offs.data_ptr(), None, None)
    s = torch.cuda.current_stream(dev).cuda_stream

    def one(ev=None):
        check(L.pts_tree_prepare_append(parents.data_ptr(), qo.data_ptr(), seqlens.data_ptr(), B, mw,
                                        bits.data_ptr(), bi.data_ptr(), pos.data_ptr(), kn.data_ptr(), vn.data_ptr(),
                                        Hkv * D, Hkv * D, layer.data_ptr(), pind.data_ptr(), perm.data_ptr(), T, Hkv,
                                        D, pl, max_pages, 2, s), "prepare+append")
        if ev is not None:
            ev[0].record()
        check(L.pts_tree_attn_run_head_pages(q.data_ptr(), layer.data_ptr(), qo.data_ptr(), hi.data_ptr(),
                                             hx.data_ptr(), hl.data_ptr(), bits.data_ptr(), mw, out.data_ptr(), B, T,
                                             n, sel_pages * pl, Hq, Hkv, D, pl, max_pages, 1 / math.sqrt(D),
                                             attn_ws.data_ptr(), attn_ws.numel(), s), "attention")
        if ev is not None:
            ev[1].record()
        check(L.pts_accept_greedy_compact(x.data_ptr(), x.stride(0), qo.data_ptr(), parents.data_ptr(),
                                          tokens.data_ptr(), B, T, V, n, -1, ot.data_ptr(), oh.data_ptr(),
                                          oc.data_ptr(), n, acc_ws.data_ptr(), acc_ws.numel(), ctypes.byref(cargs),
                                          s), "accept+compact")
        if ev is not None:
            ev[2].record()

    for _ in range(3):
        one()
    el, _ = time_steps(lambda ev: one(), steps, n_events=0)   # back to back; kernel times below
    _, evs = time_steps(one, steps)
    attn = statistics.mean(e[0].elapsed_time(e[1]) for e in evs) * 1e3
    acc = statistics.mean(e[1].elapsed_time(e[2]) for e in evs) * 1e3
    groups = (n * (Hq // Hkv) + 263) // 264
    kv_bytes = B * Hkv * groups * sel_pages * pl * D * 2 * 2
    return {
        "workload": f"long-context sparse tree-verify step: B={B} requests, prefix {P}, tree rows {n} (width 16, "
                    f"depth 8), Hq={Hq}, Hkv={Hkv}, D=128, page 16, {sel_pages} pages per KV head (4 first + 64 top + "
                    f"8 last + tree pages), vocab {V}, greedy with compaction, one layer",
        "value": steps / (el / 1e3), "unit": UNIT, "steps": steps, "ms_per_step": el / steps,
        "tokens_per_s": steps / (el / 1e3) * B * n,
        "kernels_us": {"tree_attn_head_pages": attn, "accept_with_compaction": acc, "select_once": select_us},
        "roofline": {"bound": "hbm", "peak": peak, "unit": "GB/s",
                     "attention_kv_gbs": kv_bytes / (attn * 1e-6) / 1e9,
                     "attention_frac": kv_bytes / (attn * 1e-6) / 1e9 / peak,
                     "accept_frac": T * V * 2 / (acc * 1e-6) / 1e9 / peak},
    }


def run_sparse(a):
    """``--sparse``: the long-context step alone, one JSON line."""
    import torch
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    peak, _ = measured_peaks()
    sampler = ClockSampler(local).start()
    t0 = time.perf_counter()
    r = sparse_record(a, dev, a.steps, peak)
    t1 = time.perf_counter()
    sampler.stop()
    rec = {"metric": "tree-verify steps/s, long-context sparse (per-KV-head page sets)", "value": r["value"],
           "unit": UNIT, "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": r["ms_per_step"],
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (seeded)", "config": {"workload": r["workload"]}, "tokens_per_s": r["tokens_per_s"],
           "kernels_us": r["kernels_us"], "roofline": r["roofline"], "clocks": sampler.summary(t0, t1)}
    print(json.dumps(rec), flush=True)
    return 0


def run_only(a):
    """``--only NAME``: one sub-record of the N=1 run, alone."""
    import torch
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    peak, _ = measured_peaks()
    tpeak, _ = measured_tensor_peak()
    steps = max(3, min(a.steps, 50))
    if a.only == "lmhead":
        rec = lmhead_record(a, dev, steps, tpeak)
    elif a.only == "config3":
        rec = config3_record(a, dev, steps, peak)
    elif a.only == "sparse":
        rec = sparse_record(a, dev, steps, peak)
    elif a.only == "beam":
        rec = beam_record(a, dev, steps)
    else:
        W = build_workload(a, dev, a.seed)
        st = Step(a, W, dev)
        for _ in range(3):
            st.run()
        el, evs = time_steps(st.run, steps)
        rec = flashinfer_record(a, W, dev, steps, statistics.mean(e[0].elapsed_time(e[1]) for e in evs) * 1e3)
    print(json.dumps({"only": a.only, **rec}), flush=True)
    return 0


def main(argv=None):
    a = parse_args(argv)
    if a.impl == "reference":
        return run_reference(a)
    if a.only:
        return run_only(a)
    if a.sparse:
        return run_sparse(a)
    if a.tp:
        return run_tp(a)
    return run_b200(a)


if __name__ == "__main__":
    sys.exit(main())
