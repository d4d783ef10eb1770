"""The benchmark programs behind ``bin/``.

``bin/ring_loop_<backend> <kv_size_bytes> [warmup] [iters]`` (comm-only ring)
and ``bin/ring_attention_<backend>_gpu_bench <kv_size_bytes> [warmup] [iters]``
(full ring attention) keep the reference programs' command line, defaults,
validation, per-rank info lines, rank-0 summary lines and
``ring_output_rank<r>.bin`` dumps (``src/loop/ring_loop_staged.cu`` lines 68-86,
``src/attention/ring_attention_staged_gpu_bench.cu`` lines 225-260 and 461-474).

Differences, all deliberate:
* one rank is allowed (the ring then has no steps; GB/s prints ``n/a``);
* the attention data defaults to i.i.d. N(0,1) Q/K/V (seed = rank, scale
  1/sqrt(64)); ``RAB_DATA=ref_compat`` selects the reference's own data
  (K = V = rank*1000 + i, one Q row pattern, no scale) - ill-conditioned for
  tensor cores, so the unfused schedules then default to the exact-order
  CUDA-core kernel (``RAB_KERNEL``);
* ``RAB_PREC=bf16`` runs bf16 inputs (fp32 is the default, like the reference);
* the ring runs over the native runtime (shared-memory control plane, CUDA IPC,
  NCCL) instead of MPI, and any launcher that sets rank variables works
  (torchrun, the bundled local launcher, mpirun, srun).
"""
from __future__ import annotations

import math
import os
import sys
from typing import List

import torch

from ._ext import load
from .models import inputs as inp
from .models.oracle import attention_flops
from .parallel.dist import RingRuntime, detect_ranks
from .utils import results, roofline

COMM_BACKENDS = ("staged", "staged_Isendrecv", "cuda_aware", "cuda_aware_Isendrecv", "nccl",
                 "b200_fused")
ATTN_BACKENDS = ("staged", "staged_Isendrecv", "staged_Isendrecv_overlap", "cuda_aware",
                 "cuda_aware_Isendrecv", "cuda_aware_Isendrecv_overlap", "nccl", "b200_fused")
ATTN_DEFAULT_ITERS = {"staged": 50, "cuda_aware": 50, "nccl": 50}


def _print(*a):
    print(*a, flush=True)


def _device_line(rt: RingRuntime) -> str:
    p = torch.cuda.get_device_properties(rt.device)
    return (f"[Rank {rt.rank} local_rank {rt.info.local_rank}] GPU {rt.device}: {p.name} "
            f"({p.total_memory / 1e6:.0f} MB total)")


def comm_main(backend: str, argv: List[str]) -> int:
    if backend not in COMM_BACKENDS:
        _print(f"unknown backend {backend}")
        return 1
    info = detect_ranks()
    if len(argv) < 1:
        if info.rank == 0:
            _print(f"Usage: <launcher> -np N ./ring_loop_{backend} <kv_size_bytes> [warmup] [iters]")
        return 1
    try:
        kv_size = int(argv[0])
        warmup = int(argv[1]) if len(argv) > 1 else 10
        iters = int(argv[2]) if len(argv) > 2 else 100
    except ValueError:
        kv_size, warmup, iters = 0, -1, 0
    if kv_size <= 0 or kv_size % 4 or warmup < 0 or iters <= 0:
        if info.rank == 0:
            _print("Invalid arguments: kv_size must be a positive multiple of 4, warmup >= 0, "
                   "iters > 0.")
        return 1
    C = load()
    rt = RingRuntime(C.comm_arena_bytes(kv_size), need_nccl=(backend == "nccl"), info=info)
    try:
        _run_comm(rt, backend, kv_size, warmup, iters)
    finally:
        rt.close()
    return 0


def _run_comm(rt: RingRuntime, backend: str, kv_size: int, warmup: int, iters: int) -> None:
    """One comm-only run on an existing runtime: info lines, RESULT line, JSONL record."""
    C = load()
    _print(_device_line(rt))
    _print(f"[Rank {rt.rank}] KV shard: {kv_size} bytes ({kv_size / 1024.0:.1f} KB), "
           f"neighbors: left={(rt.rank - 1) % rt.world} right={(rt.rank + 1) % rt.world}")
    slices = int(os.environ.get("RAB_P2P_SLICES", "0"))
    mode = {"vector": 0, "bulk": 1, "vector32": 2, "pull": 3}[os.environ.get("RAB_P2P_MODE",
                                                                              "vector")]
    avg = C.run_comm_bench(rt.ctx, backend, kv_size, warmup, iters, slices, True, mode)
    if rt.rank == 0:
        _print(results.comm_result_line(backend, kv_size, rt.world, warmup, iters, avg))
        results.append_jsonl({"kind": "comm", "backend": backend, "bytes": kv_size,
                              "ranks": rt.world, "warmup": warmup, "iters": iters,
                              "avg_ms": avg})


def _attention_inputs(rank: int, seq: int, prec: str, data: str):
    if data == "ref_compat":
        x = inp.ref_compat_inputs(rank, seq)
    else:
        x = inp.normal_inputs(rank, seq, 1, 64)
    dtype = torch.float32 if prec == "fp32" else torch.bfloat16
    return x.q.to(dtype).contiguous(), x.k.to(dtype).contiguous(), x.v.to(dtype).contiguous(), x


def attention_main(backend: str, argv: List[str]) -> int:
    if backend not in ATTN_BACKENDS:
        _print(f"unknown backend {backend}")
        return 1
    info = detect_ranks()
    try:
        kv_size = int(argv[0]) if argv else 262144
        warmup = int(argv[1]) if len(argv) > 1 else 10
        iters = int(argv[2]) if len(argv) > 2 else ATTN_DEFAULT_ITERS.get(backend, 100)
    except ValueError:
        kv_size, warmup, iters = 0, -1, 0
    if kv_size <= 0 or kv_size % (64 * 4) or warmup < 0 or iters <= 0:
        if info.rank == 0:
            _print(f"Usage: ./ring_attention_{backend}_gpu_bench <kv_size_bytes> [warmup>=0] "
                   "[iters>0]\nkv_size_bytes must be a positive multiple of 256 bytes.")
        return 1
    data = os.environ.get("RAB_DATA", "normal")
    prec = os.environ.get("RAB_PREC", "fp32")
    seq = kv_size // (64 * 4)  # tokens per rank, as in the reference (bytes of one fp32 shard)
    C = load()
    arena = C.AttnBench.arena_bytes(prec, seq, 1, 64, data == "ref_compat", info.world)
    rt = RingRuntime(arena, need_nccl=(backend == "nccl"), info=info)
    try:
        _run_attention(rt, backend, kv_size, warmup, iters)
    finally:
        rt.close()
    return 0


def _run_attention(rt: RingRuntime, backend: str, kv_size: int, warmup: int, iters: int) -> None:
    """One attention run on an existing runtime: info lines, the two summary
    lines, the JSONL record and (where the reference dumps) the output file."""
    data = os.environ.get("RAB_DATA", "normal")
    prec = os.environ.get("RAB_PREC", "fp32")
    kernel = os.environ.get("RAB_KERNEL", "simt" if data == "ref_compat" else "tcgen05")
    chain = os.environ.get("RAB_RING_MODE", "direct") == "chain"
    seq = kv_size // (64 * 4)  # tokens per rank, as in the reference (bytes of one fp32 shard)
    C = load()
    kv_shared = data == "ref_compat"
    _print(_device_line(rt))
    _print(f"[Rank {rt.rank}] seq_q={seq}, seq_k={seq}, dim=64, KV shard={kv_size / 1024.0:.1f} KB")
    q, k, v, x = _attention_inputs(rt.rank, seq, prec, data)
    bench = C.AttnBench(rt.ctx, backend, prec, seq, 1, 1, 64, x.scale, kv_shared, False,
                        False, kernel, chain, warmup, iters,
                        float(os.environ.get("RAB_TIMEOUT_S", "10")))
    bench.set_inputs(q, k, v)
    res = bench.run()
    if rt.rank == 0:
        flops = attention_flops(seq, seq * rt.world, 1, 64)
        tflops = flops / (res["total"] * 1e-3) / 1e12
        extra = {"TFLOPs": f"{tflops:.3f}", "data": data, "prec": prec,
                 "kernel": "fused" if backend == "b200_fused" else kernel}
        if backend == "b200_fused" and res.get("attn", 0) > 0:
            kv_bytes = seq * 64 * (2 if prec == "bf16" else 4) * (1 if kv_shared else 2)
            roof = roofline.attention_roofline_ms(flops, kv_bytes * (rt.world - 1), prec)
            extra["kernel_TFLOPs"] = f"{flops / (res['attn'] * 1e-3) / 1e12:.3f}"
            extra["roofline_frac"] = f"{roof / res['attn']:.3f}"
        _print(results.attn_header(backend, warmup, iters))
        _print(results.attn_result_line(backend, res, extra))
        results.append_jsonl({"kind": "attention", "backend": backend, "bytes": kv_size,
                              "ranks": rt.world, "warmup": warmup, "iters": iters,
                              "seq": seq, "data": data, "prec": prec, "kernel": kernel,
                              "avg_ms": {k2: v2 for k2, v2 in res.items() if k2 != "step_ms"},
                              "tflops": tflops})
    if backend in results.DUMP_ALWAYS or os.environ.get("ATTENTION_DUMP_OUTPUT") is not None:
        out_dtype = torch.float32 if prec == "fp32" else torch.bfloat16
        out = torch.empty(seq, 1, 64, dtype=out_dtype)
        bench.output(out)
        fname = f"ring_output_rank{rt.rank}.bin"
        out.float().contiguous().numpy().tofile(fname)
        _print(f"[Rank {rt.rank}] output dumped to {fname}")
    del bench


def sweep_main(argv: List[str]) -> int:
    """Every (backend, size) of a sweep in ONE launch: the runtime (shared
    memory, IPC peer mappings, NCCL communicator) is set up once and each run
    prints the same lines and records as its program would.

        sweep comm|attention <warmup> <iters> <size_bytes>[,...] <backend>[,...]
    """
    if len(argv) != 5 or argv[0] not in ("comm", "attention"):
        _print("usage: sweep comm|attention <warmup> <iters> <sizes,...> <backends,...>")
        return 1
    kind = argv[0]
    warmup, iters = int(argv[1]), int(argv[2])
    sizes = [int(x) for x in argv[3].split(",") if x]
    backends = [b for b in argv[4].split(",") if b]
    known = COMM_BACKENDS if kind == "comm" else ATTN_BACKENDS
    bad = [b for b in backends if b not in known]
    unit = 4 if kind == "comm" else 64 * 4
    if bad or not sizes or any(sz <= 0 or sz % unit for sz in sizes) or warmup < 0 or iters <= 0:
        _print(f"sweep: bad arguments (unknown backends {bad}, sizes must be positive multiples "
               f"of {unit} bytes, warmup >= 0, iters > 0)")
        return 1
    info = detect_ranks()
    C = load()
    if kind == "comm":
        arena = max(C.comm_arena_bytes(sz) for sz in sizes)
    else:
        data, prec = os.environ.get("RAB_DATA", "normal"), os.environ.get("RAB_PREC", "fp32")
        arena = max(C.AttnBench.arena_bytes(prec, sz // 256, 1, 64, data == "ref_compat",
                                            info.world) for sz in sizes)
    rt = RingRuntime(arena, need_nccl="nccl" in backends, info=info)
    try:
        for b in backends:
            if rt.rank == 0:
                _print(f"===== backend={b} =====")
            for sz in sizes:
                if rt.rank == 0:
                    _print(f"--- kv_size={sz} bytes ---")
                if kind == "comm":
                    _run_comm(rt, b, sz, warmup, iters)
                else:
                    _run_attention(rt, b, sz, warmup, iters)
                rt.barrier()
    finally:
        rt.close()
    return 0


def program_main(prog: str, argv: List[str]) -> int:
    """Dispatch on the program name used by the reference (bin/<name>)."""
    # a program (not a library import) asks for the native backtrace on a fatal signal
    os.environ.setdefault("RAB_CRASH_HANDLER", "1")
    name = os.path.basename(prog)
    if name == "sweep":
        return sweep_main(argv)
    if name.startswith("ring_loop_"):
        return comm_main(name[len("ring_loop_"):], argv)
    if name.startswith("ring_attention_") and name.endswith("_gpu_bench"):
        return attention_main(name[len("ring_attention_"):-len("_gpu_bench")], argv)
    print(f"unknown program {name}", file=sys.stderr)
    return 1


if __name__ == "__main__":  # python -m ring_attention_benchmark_b200.cli <program> args...
    sys.exit(program_main(sys.argv[1], sys.argv[2:]))
