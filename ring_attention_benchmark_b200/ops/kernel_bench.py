"""Microbenchmark of the standalone hot ops on one GPU.

    python -m ring_attention_benchmark_b200.ops.kernel_bench [--iters N] [--rows R]

Times every memory-bound kernel of the unfused ring schedules on inputs larger
than the 126 MB L2 (an L2 flush runs between timed launches anyway) and prints
one line per kernel: device time, algorithmic bytes, achieved GB/s and the
fraction of the measured HBM copy bandwidth.  The exact-order CUDA-core
attention kernel is reported in GFLOP/s.  ``--iters 1`` runs every kernel once
(used for ncu captures).
"""
from __future__ import annotations

import argparse
import json

import torch

from .._ext import load
from ..utils.roofline import load_peaks


def _time(fn, iters, flush):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.fill_(0)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    ts.sort()
    return ts[len(ts) // 2]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--rows", type=int, default=1 << 20, help="query rows (seq*heads)")
    ap.add_argument("--dim", type=int, default=64)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    C = load()
    dev = torch.device("cuda", 0)
    peaks = load_peaks()
    rows, d = a.rows, a.dim
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    results = []

    def report(name, ms, nbytes=None, flops=None):
        r = {"kernel": name, "ms": round(ms, 4)}
        if nbytes:
            gbs = nbytes / (ms * 1e-3) / 1e9
            r.update(bytes=nbytes, GBps=round(gbs, 1),
                     hbm_frac=round(gbs / peaks.hbm_gbs, 3), peak_source=peaks.source)
        if flops:
            r.update(GFLOPs=round(flops / (ms * 1e-3) / 1e9, 1))
        results.append(r)
        if not a.json:
            print(" ".join(f"{k}={v}" for k, v in r.items()), flush=True)

    acc_r = torch.randn(rows, d, device=dev)
    acc_n = torch.randn(rows, d, device=dev)
    m_r = torch.randn(rows, device=dev)
    l_r = torch.rand(rows, device=dev) + 1
    m_n = torch.randn(rows, device=dev)
    l_n = torch.rand(rows, device=dev) + 1
    ms = _time(lambda: C.merge_lse(m_r, l_r, acc_r, m_n, l_n, acc_n), a.iters, flush)
    report("merge_lse", ms, nbytes=(3 * rows * d + 6 * rows) * 4)

    out32 = torch.empty(rows, d, device=dev)
    out16 = torch.empty(rows, d, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(rows, device=dev)
    ms = _time(lambda: C.normalize(acc_r, m_r, l_r, out32, lse), a.iters, flush)
    report("normalize_fp32_out", ms, nbytes=(2 * rows * d + 3 * rows) * 4)
    ms = _time(lambda: C.normalize(acc_r, m_r, l_r, out16, None), a.iters, flush)
    report("normalize_bf16_out", ms, nbytes=rows * d * 6 + 2 * rows * 4)

    n = rows * d
    x = acc_r.view(-1)
    ms = _time(lambda: C.cast(x, out16.view(-1)), a.iters, flush)
    report("cast_f32_bf16", ms, nbytes=n * 6)
    ms = _time(lambda: C.cast(out16.view(-1), out32.view(-1)), a.iters, flush)
    report("cast_bf16_f32", ms, nbytes=n * 6)
    big, small = torch.empty_like(x), torch.empty_like(x)
    ms = _time(lambda: C.split_tf32(x, big, small), a.iters, flush)
    report("split_tf32", ms, nbytes=n * 12)

    # ring-format preparation of one fp32 block: K -> 2 planes, V -> 2 transposed planes
    skv = rows // 4
    k = torch.randn(skv, 4, d, device=dev)
    v = torch.randn(skv, 4, d, device=dev)
    slot = torch.empty(C.ring_block_bytes(1, skv, 4, d), dtype=torch.uint8, device=dev)
    ms = _time(lambda: C.ring_format(1, k, v, slot), a.iters, flush)
    report("ring_format_fp32", ms, nbytes=k.numel() * 4 * 2 * 3)

    # exact-order fp32 CUDA-core attention (reference arithmetic), 4096 x 4096, d=64
    q = torch.randn(4096, 1, 64, device=dev)
    kk = torch.randn(4096, 1, 64, device=dev)
    acc = torch.empty(4096, 1, 64, device=dev)
    mm = torch.empty(4096, 1, device=dev)
    ll = torch.empty(4096, 1, device=dev)
    ms = _time(lambda: C.simt_partial_attention(q, kk, kk, acc, mm, ll, 0.125, -1, False),
               max(1, a.iters // 2), flush)
    # the exact-max pass recomputes QK^T: 6*sq*sk*d FLOPs issued, 4*sq*sk*d useful
    report("simt_partial_attention_4096", ms, flops=4.0 * 4096 * 4096 * 64)

    if a.json:
        print(json.dumps(results))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
