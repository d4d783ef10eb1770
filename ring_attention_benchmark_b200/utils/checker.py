"""Correctness checker for ``ring_output_rank<r>.bin`` dumps.

Compare mode reproduces the reference checker
(``check_attention_correctness.sh`` lines 114-178): load both dumps of every
rank as raw little-endian fp32, accumulate max / mean absolute error and max
relative error ``|a-b| / max(|a|, |b|, 1e-12)``, and PASS when
``max_abs <= ABS_TOL or max_rel <= REL_TOL`` (same output line, same exit code).

Oracle mode checks one run's dumps against the float64 oracle of the ring
(independent of any GPU schedule), for the data the programs generate:

    python -m ring_attention_benchmark_b200.utils.checker compare LABEL REF_DIR TEST_DIR NP [ABS_TOL REL_TOL]
    python -m ring_attention_benchmark_b200.utils.checker oracle LABEL TEST_DIR NP KV_SIZE_BYTES [ABS_TOL REL_TOL] [--data normal|ref_compat]
"""
from __future__ import annotations

import argparse
import os
import sys
from dataclasses import dataclass
from typing import List, Sequence

import numpy as np


@dataclass
class CompareResult:
    passed: bool
    elements: int
    max_abs: float
    mean_abs: float
    max_rel: float
    worst_rank: int
    abs_tol: float
    rel_tol: float

    def line(self, label: str) -> str:
        status = "PASS" if self.passed else "FAIL"
        return (f"{label}: {status} elements={self.elements} max_abs_err={self.max_abs:.6e} "
                f"mean_abs_err={self.mean_abs:.6e} max_rel_err={self.max_rel:.6e} "
                f"worst_rank={self.worst_rank} abs_tol={self.abs_tol:.1e} "
                f"rel_tol={self.rel_tol:.1e}")


def load_f32(path: str) -> np.ndarray:
    size = os.path.getsize(path)
    if size % 4 != 0:
        raise RuntimeError(f"{path}: size is not a multiple of float32")
    return np.fromfile(path, dtype="<f4")


def compare_arrays(refs: Sequence[np.ndarray], tests: Sequence[np.ndarray], abs_tol: float,
                   rel_tol: float) -> CompareResult:
    total, sum_abs, max_abs, max_rel, worst = 0, 0.0, 0.0, 0.0, -1
    for rank, (a, b) in enumerate(zip(refs, tests)):
        if a.size != b.size:
            raise RuntimeError(f"rank {rank}: length mismatch {a.size} vs {b.size}")
        a64 = a.astype(np.float64)
        b64 = b.astype(np.float64)
        diff = np.abs(a64 - b64)
        denom = np.maximum(np.maximum(np.abs(a64), np.abs(b64)), 1e-12)
        total += a.size
        sum_abs += float(diff.sum())
        if diff.size:
            m = float(diff.max())
            if m > max_abs:
                max_abs, worst = m, rank
            max_rel = max(max_rel, float((diff / denom).max()))
    mean_abs = sum_abs / total if total else 0.0
    passed = max_abs <= abs_tol or max_rel <= rel_tol
    return CompareResult(passed, total, max_abs, mean_abs, max_rel, worst, abs_tol, rel_tol)


def compare_dirs(ref_dir: str, test_dir: str, np_: int, abs_tol: float = 1e-3,
                 rel_tol: float = 1e-5) -> CompareResult:
    refs = [load_f32(os.path.join(ref_dir, f"ring_output_rank{r}.bin")) for r in range(np_)]
    tests = [load_f32(os.path.join(test_dir, f"ring_output_rank{r}.bin")) for r in range(np_)]
    return compare_arrays(refs, tests, abs_tol, rel_tol)


def oracle_outputs(np_: int, kv_size_bytes: int, data: str = "normal") -> List[np.ndarray]:
    """Float64 ring-attention outputs of every rank for the programs' inputs."""
    from ..models import inputs, oracle

    seq = inputs.size_to_seq(kv_size_bytes)
    if data == "ref_compat":
        xs = [inputs.ref_compat_inputs(r, seq) for r in range(np_)]
    else:
        xs = [inputs.normal_inputs(r, seq, 1, 64) for r in range(np_)]
    outs = oracle.ring_attention([x.q for x in xs], [x.k for x in xs], [x.v for x in xs],
                                 xs[0].scale)
    return [o.reshape(-1).numpy() for o in outs]


def check_oracle(test_dir: str, np_: int, kv_size_bytes: int, data: str = "normal",
                 abs_tol: float = 1e-3, rel_tol: float = 1e-5) -> CompareResult:
    refs = oracle_outputs(np_, kv_size_bytes, data)
    tests = [load_f32(os.path.join(test_dir, f"ring_output_rank{r}.bin")) for r in range(np_)]
    return compare_arrays(refs, tests, abs_tol, rel_tol)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="mode", required=True)
    c = sub.add_parser("compare")
    c.add_argument("label")
    c.add_argument("ref_dir")
    c.add_argument("test_dir")
    c.add_argument("np", type=int)
    c.add_argument("abs_tol", type=float, nargs="?", default=1e-3)
    c.add_argument("rel_tol", type=float, nargs="?", default=1e-5)
    o = sub.add_parser("oracle")
    o.add_argument("label")
    o.add_argument("test_dir")
    o.add_argument("np", type=int)
    o.add_argument("kv_size_bytes", type=int)
    o.add_argument("abs_tol", type=float, nargs="?", default=1e-3)
    o.add_argument("rel_tol", type=float, nargs="?", default=1e-5)
    o.add_argument("--data", choices=("normal", "ref_compat"), default="normal")
    a = ap.parse_args(argv)
    if a.mode == "compare":
        res = compare_dirs(a.ref_dir, a.test_dir, a.np, a.abs_tol, a.rel_tol)
    else:
        res = check_oracle(a.test_dir, a.np, a.kv_size_bytes, a.data, a.abs_tol, a.rel_tol)
    print(res.line(a.label), flush=True)
    return 0 if res.passed else 1


if __name__ == "__main__":
    sys.exit(main())
