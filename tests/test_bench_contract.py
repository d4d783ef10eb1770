"""The `bench.py` output contract: the reference arm's line, argument checks,
the preset table (CPU), and the full JSON line of a short 1-GPU run (GPU)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BENCH = os.path.join(ROOT, "bench.py")

TOP_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
            "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
            "clocks", "e2e", "gpu_launches"}
CONFIG_KEYS = {"model", "global_batch", "seq_len", "parallelism", "l2"}
E2E_KEYS = {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"}
CLOCK_KEYS = {"sm_mhz", "sm_max_mhz", "reasons"}


def check_line(d, n_gpus, steps, warmup):
    """Every key the benchmark driver reads, with the types and relations it expects."""
    missing = TOP_KEYS - d.keys()
    assert not missing, missing
    assert d["n_gpus"] == n_gpus and d["steps"] == steps and d["warmup"] == warmup
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    assert d["scaling"] in ("weak", "strong") and isinstance(d["unit"], str)
    assert CONFIG_KEYS <= d["config"].keys(), CONFIG_KEYS - d["config"].keys()
    assert CLOCK_KEYS <= d["clocks"].keys() and isinstance(d["clocks"]["reasons"], list)
    assert E2E_KEYS <= d["e2e"].keys() and d["e2e"]["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] > 0 and d["e2e"]["d2h_bytes_per_step"] > 0
    assert isinstance(d["gpu_launches"], int) and d["gpu_launches"] >= steps
    # the output check against the float64 recomputation ran and passed
    chk = d["config"]["check"]
    assert chk["passed"] is True and chk["max_abs_err"] <= chk["tol"], chk


def _run(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, BENCH] + list(args), cwd=ROOT, env=e,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_unavailable_line():
    r = _run("--impl", "reference", "--steps", "5", "--warmup", "3", env={"RANK": "0"})
    assert r.returncode == 0, r.stderr
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unavailable"]
    # only rank 0 prints
    r1 = _run("--impl", "reference", env={"RANK": "1"})
    assert r1.returncode == 0 and not r1.stdout.strip()


def test_too_few_warmup_steps_rejected():
    r = _run("--warmup", "2")
    assert r.returncode == 2 and "warm-up" in r.stderr


def test_presets_are_well_formed():
    sys.path.insert(0, ROOT)
    try:
        import bench
    finally:
        sys.path.pop(0)
    assert "ref-fp32" in bench.PRESETS  # the default (headline) preset
    for name, (seq, heads, heads_kv, d, dt, causal, mult, seed) in bench.PRESETS.items():
        assert seq % 256 == 0 and heads % heads_kv == 0 and d in (64, 128), name
        assert dt in ("fp32", "bf16") and isinstance(causal, bool) and mult > 0, name


@pytest.mark.gpu
def test_short_run_json_line():
    r = _run("--steps", "3", "--warmup", "3")
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    check_line(json.loads(lines[0]), n_gpus=1, steps=3, warmup=3)
