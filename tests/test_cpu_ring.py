"""Ring attention on CPU gloo ranks against full softmax attention over the
concatenated sequence (no GPU)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("np,case", [(2, "config1"), (4, "causal")])
def test_cpu_ring(np, case):
    cmd = [sys.executable, "-m", "ring_attention_benchmark_b200.launch", "-np", str(np),
           "--timeout", "120", sys.executable, os.path.join(ROOT, "tests", "_cpu_ring_worker.py"),
           case]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=180)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count(" ok ") == np


@pytest.mark.parametrize("case,expect", [
    ("fault_nan", "received from rank 1 at ring step 1 is not finite"),
    ("fault_exit", "rank 1 leaves before the ring"),
])
def test_cpu_ring_fault_injection(case, expect):
    """Host-side fault injection on 3 gloo ranks: a NaN shard is named by the
    receiver; a rank that leaves makes the job fail within the timeouts instead
    of hanging."""
    cmd = [sys.executable, "-m", "ring_attention_benchmark_b200.launch", "-np", "3",
           "--timeout", "60", sys.executable, os.path.join(ROOT, "tests", "_cpu_ring_worker.py"),
           case]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=120)
    out = r.stdout + r.stderr
    assert r.returncode != 0, out
    assert expect in out, out[-3000:]
