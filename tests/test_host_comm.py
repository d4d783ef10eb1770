"""Host control plane on CPU, world sizes 2-4, through the local launcher:
barrier, max-reduction, ring exchange larger than the mailbox fragments, and
failure detection without any GPU (a rank that leaves, an aborting rank, a
dropped message)."""
import os
import subprocess
import sys
import uuid

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "_host_worker.py")


def _launch(np, case, timeout=60):
    name = f"/rab_test_{uuid.uuid4().hex[:10]}"
    cmd = [sys.executable, "-m", "ring_attention_benchmark_b200.launch", "-np", str(np),
           "--timeout", str(timeout), sys.executable, WORKER, name, case]
    return subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=timeout + 30)


@pytest.mark.parametrize("np", [2, 3, 4])
def test_barrier_reduce_ring(np):
    r = _launch(np, "ok")
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count(" ok") == np


def test_dead_rank_is_named():
    r = _launch(3, "dead_rank")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "missing ranks: 2" in r.stdout or "aborted" in r.stdout


def test_abort_propagates():
    r = _launch(3, "abort")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "injected failure" in r.stdout or "missing" in r.stdout


def test_dropped_message_times_out():
    r = _launch(2, "dropped_message")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "timed out" in r.stdout


def test_launcher_watchdog_stops_other_ranks():
    code = ("import os,sys,time\n"
            "r=int(os.environ['RANK'])\n"
            "sys.exit(3) if r==1 else time.sleep(60)\n")
    cmd = [sys.executable, "-m", "ring_attention_benchmark_b200.launch", "-np", "3",
           sys.executable, "-c", code]
    import time

    t0 = time.time()
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=60)
    assert r.returncode == 3
    assert time.time() - t0 < 30
    assert "rank 1 exited with 3" in r.stderr
