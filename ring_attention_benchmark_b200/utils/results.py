"""Output lines of the benchmark programs.

The reference's grammars are kept byte-compatible, label quirks included, so
existing log parsers keep working:

* comm (``src/loop/ring_loop_*.cu``, RESULT printf at e.g. ``ring_loop_staged.cu``
  lines 240-244): ``staged_Isendrecv`` prints ``backend=isendrecv`` and both
  CUDA-aware loops print ``backend=cuda_aware``; GB/s = (np-1)*bytes / avg ms.
* attention (``src/attention/*_gpu_bench.cu``): a header
  ``<label> bench: warmup=W iters=I`` and one ``avg_total=… ms …`` line whose
  fields depend on the backend.

Fields the reference does not print are appended after its own fields
(``step_ms=``, ``TFLOPs=``, ``roofline_frac=``, ...) and every result can also be
appended as one JSON record to the file named by ``RAB_RESULTS_JSONL``.
"""
from __future__ import annotations

import json
import os
import time
from typing import List, Dict, Optional

COMM_LABEL = {
    "staged": "staged",
    "staged_Isendrecv": "isendrecv",
    "cuda_aware": "cuda_aware",
    "cuda_aware_Isendrecv": "cuda_aware",
    "nccl": "nccl",
    "b200_fused": "b200_fused",
}

ATTN_HEADER = {
    "staged": "staged bench",
    "staged_Isendrecv": "staged Isendrecv bench",
    "staged_Isendrecv_overlap": "staged Isendrecv OVERLAP bench",
    "cuda_aware": "cuda_aware bench",
    "cuda_aware_Isendrecv": "CUDA-aware Isendrecv bench",
    "cuda_aware_Isendrecv_overlap": "CUDA-aware Isendrecv OVERLAP bench",
    "nccl": "nccl bench",
    "b200_fused": "b200_fused bench",
}

ATTN_FIELDS = {
    "staged": ["D2H", "MPI", "H2D"],
    "staged_Isendrecv": ["D2H", "MPI", "H2D"],
    "staged_Isendrecv_overlap": ["D2H", "MPI", "H2D"],
    "cuda_aware": ["MPI"],
    "cuda_aware_Isendrecv": ["CUDA-aware"],
    "cuda_aware_Isendrecv_overlap": ["CUDA-aware"],
    "nccl": ["NCCL"],
    "b200_fused": ["prep"],
}

# Isendrecv programs dump only when ATTENTION_DUMP_OUTPUT is set; the others
# always dump (reference behaviour, e.g. ring_attention_staged_gpu_bench.cu:469-474).
DUMP_ALWAYS = {"staged", "cuda_aware", "nccl"}


def gbps(payload_bytes: float, ms: float) -> Optional[float]:
    if ms <= 0 or payload_bytes <= 0:
        return None
    return payload_bytes / (ms / 1e3) / 1e9


def _g(v: Optional[float]) -> str:
    return "n/a" if v is None else f"{v:.3f}"


def comm_result_line(backend: str, nbytes: int, ranks: int, warmup: int, iters: int,
                     avg: Dict[str, float]) -> str:
    payload = (ranks - 1) * nbytes
    total = avg["total"]
    label = COMM_LABEL[backend]
    head = f"RESULT backend={label} bytes={nbytes} ranks={ranks} warmup={warmup} iters={iters} "
    if backend in ("staged", "staged_Isendrecv"):
        return head + (f"avg_d2h_ms={avg['d2h']:.3f} avg_mpi_ms={avg['mpi']:.3f} "
                       f"avg_h2d_ms={avg['h2d']:.3f} avg_total_ms={total:.3f} "
                       f"total_GBps={_g(gbps(payload, total))} mpi_GBps={_g(gbps(payload, avg['mpi']))}")
    if backend in ("cuda_aware", "cuda_aware_Isendrecv"):
        return head + (f"avg_mpi_ms={avg['mpi']:.3f} avg_total_ms={total:.3f} "
                       f"total_GBps={_g(gbps(payload, total))} mpi_GBps={_g(gbps(payload, avg['mpi']))}")
    if backend == "nccl":
        return head + (f"avg_nccl_ms={avg['mpi']:.3f} avg_total_ms={total:.3f} "
                       f"total_GBps={_g(gbps(payload, total))} nccl_GBps={_g(gbps(payload, avg['mpi']))}")
    # b200_fused: p2p = host-timed launch+sync, kernel = device-timed ring kernel
    return head + (f"avg_p2p_ms={avg['mpi']:.3f} avg_total_ms={total:.3f} "
                   f"total_GBps={_g(gbps(payload, total))} p2p_GBps={_g(gbps(payload, avg['mpi']))} "
                   f"avg_kernel_ms={avg['kernel']:.3f} kernel_GBps={_g(gbps(payload, avg['kernel']))}")


def attn_header(backend: str, warmup: int, iters: int) -> str:
    return f"{ATTN_HEADER[backend]}: warmup={warmup} iters={iters}"


def attn_result_line(backend: str, avg: Dict[str, float], extra: Optional[Dict] = None) -> str:
    parts = [f"avg_total={avg['total']:.3f} ms"]
    for f in ATTN_FIELDS[backend]:
        parts.append(f"avg_{f}={avg.get(f, 0.0):.3f}")
    parts += [f"avg_attn={avg.get('attn', 0.0):.3f}", f"avg_merge={avg.get('merge', 0.0):.3f}",
              f"avg_final={avg.get('final', 0.0):.3f}"]
    line = " ".join(parts)
    if extra:
        line += " " + " ".join(f"{k}={v}" for k, v in extra.items())
    return line


def append_jsonl(record: Dict) -> None:
    path = os.environ.get("RAB_RESULTS_JSONL")
    if not path:
        return
    rec = dict(record)
    rec.setdefault("time", time.time())
    with open(path, "a") as f:
        f.write(json.dumps(rec, sort_keys=True) + "\n")


def has_record(path: str, **match) -> bool:
    """True when the JSONL file holds a record whose fields equal `match`
    (a resumed sweep skips such configurations).  Unreadable lines are ignored."""
    if not path or not os.path.exists(path):
        return False
    with open(path) as f:
        for line in f:
            try:
                rec = json.loads(line)
            except ValueError:
                continue
            if all(rec.get(k) == v for k, v in match.items()):
                return True
    return False


def load_records(path: str) -> List[Dict]:
    out = []
    with open(path) as f:
        for line in f:
            try:
                out.append(json.loads(line))
            except ValueError:
                continue
    return out


def sweep_table(records: List[Dict], kind: str) -> str:
    """Markdown table of a sweep's records: one row per (ranks, backend), one
    column per size.  comm: total GB/s ((np-1) * bytes / avg_total), and for
    the b200_fused kernel its device-timed GB/s in brackets; attention:
    avg_total ms and TFLOP/s.  The last record of a configuration wins."""
    cells: Dict = {}
    sizes, rows = set(), []
    for r in records:
        if r.get("kind") != kind:
            continue
        key = (r["ranks"], r["backend"])
        if key not in rows:
            rows.append(key)
        sizes.add(r["bytes"])
        total = r["avg_ms"].get("total", 0.0)
        if kind == "comm":
            g = gbps((r["ranks"] - 1) * r["bytes"], total)
            cell = "n/a" if g is None else f"{g:.1f}"
            kg = gbps((r["ranks"] - 1) * r["bytes"], r["avg_ms"].get("kernel", 0.0))
            if kg is not None and r["avg_ms"].get("kernel", 0.0) > 0:
                cell += f" ({kg:.1f})"
            cells[key + (r["bytes"],)] = cell
        else:
            cells[key + (r["bytes"],)] = f"{total:.3f} ms / {r.get('tflops', 0.0):.2f}"
    cols = sorted(sizes)
    unit = "bytes" if kind == "comm" else "bytes (tokens/rank = bytes/256)"
    head = "| np | backend | " + " | ".join(str(c) for c in cols) + " |"
    lines = [f"({kind}; columns: shard size in {unit}; cells: "
             + ("total GB/s (kernel GB/s)" if kind == "comm" else "avg_total ms / TFLOP/s")
             + ")", "",
             head, "|" + "---|" * (len(cols) + 2)]
    for key in sorted(rows, key=lambda k: (k[0], rows.index(k))):
        lines.append(f"| {key[0]} | {key[1]} | " +
                     " | ".join(cells.get(key + (c,), "") for c in cols) + " |")
    return "\n".join(lines)


def main(argv=None) -> int:
    """``python -m ring_attention_benchmark_b200.utils.results has --kind comm
    --backend B --bytes N --ranks R --warmup W --iters I [--prec P --data D]``:
    exit 0 when $RAB_RESULTS_JSONL already records that configuration, 1 when
    not (used by the wrappers' RESUME=1)."""
    import argparse

    ap = argparse.ArgumentParser(prog="results")
    sub = ap.add_subparsers(dest="cmd", required=True)
    h = sub.add_parser("has")
    h.add_argument("--kind", required=True, choices=("comm", "attention"))
    h.add_argument("--backend", required=True)
    for k in ("bytes", "ranks", "warmup", "iters"):
        h.add_argument("--" + k, type=int, required=True)
    h.add_argument("--prec")
    h.add_argument("--data")
    t = sub.add_parser("table")
    t.add_argument("path")
    t.add_argument("--kind", required=True, choices=("comm", "attention"))
    a = ap.parse_args(argv)
    if a.cmd == "table":
        print(sweep_table(load_records(a.path), a.kind))
        return 0
    match = {"kind": a.kind, "backend": a.backend, "bytes": a.bytes, "ranks": a.ranks,
             "warmup": a.warmup, "iters": a.iters}
    if a.prec:
        match["prec"] = a.prec
    if a.data:
        match["data"] = a.data
    return 0 if has_record(os.environ.get("RAB_RESULTS_JSONL", ""), **match) else 1


if __name__ == "__main__":
    raise SystemExit(main())
