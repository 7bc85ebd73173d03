"""CPU checks of bench.py's contract: the roofline numerators and the JSON line
of the reference arm (the oracle port timed on the host), on a reduced
workload so that it runs in seconds."""
import json
import os
import subprocess
import sys

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_algorithmic_bytes_of_the_benchmark_step():
    a = bench.parse_args([])
    n = 1 + a.width * a.depth
    assert (a.batch, a.prefix, n, a.hq, a.hkv, a.vocab) == (16, 4096, 65, 32, 8, 128256)
    ab = bench.algorithmic_bytes(a)
    # KV read: 16 requests x 8 KV heads x 4161 positions x 128 x (K and V) x 2 bytes
    assert ab["kv_read"] == 16 * 8 * 4161 * 128 * 2 * 2 == 272_695_296
    # logits: 16 x 65 rows x 128256 x 2 bytes, read once
    assert ab["accept"] == 16 * 65 * 128256 * 2 == 266_772_480
    # q read and output written, bf16
    assert ab["q_o"] == 2 * 16 * 65 * 32 * 128 * 2
    assert ab["attention"] == ab["kv_read"] + ab["q_o"]
    assert ab["step"] == ab["attention"] + ab["append"] + ab["accept"] + ab["compact"]


def test_over_ranks_without_a_process_group():
    assert bench.over_ranks([3, 1.5], "max", "cpu") == [3.0, 1.5]


def test_reference_arm_prints_one_contract_line():
    cmd = [sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "1", "--batch", "2",
           "--prefix", "48", "--width", "2", "--depth", "2", "--vocab", "1024", "--hq", "4", "--hkv", "2"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in rec, key
    assert rec["value"] > 0 and rec["higher_is_better"] is True and rec["unit"] == rec["e2e"]["unit"]
    assert rec["e2e"]["value"] == rec["value"]
    assert rec["e2e"]["h2d_bytes_per_step"] == 0 and rec["e2e"]["d2h_bytes_per_step"] == 0
    assert rec["cpu_baseline"]["kind"] == "port" and rec["cpu_baseline"]["cores"] >= 1
    assert "B=2 requests, prefix=48" in rec["config"]["workload"]
