"""One rank of the multi-GPU tests (started by tests/test_multigpu.py through the
local launcher).  Every check compares against the float64 oracle computed from
the same seeded inputs of all ranks, so each rank can verify its own output.

    python tests/_ring_worker.py <case> [args]
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from ring_attention_benchmark_b200 import RingAttention, _ext  # noqa: E402
from ring_attention_benchmark_b200.models import inputs, oracle  # noqa: E402
from ring_attention_benchmark_b200.parallel.dist import RingRuntime, detect_ranks  # noqa: E402


def all_inputs(world, spr, h, hk, d, dtype, causal):
    """Every rank's shard of one global sequence (zigzag for causal)."""
    g = torch.Generator().manual_seed(1234)
    total = world * spr
    q = torch.randn(total, h, d, generator=g) * 0.5
    k = torch.randn(total, hk, d, generator=g) * 0.5
    v = torch.randn(total, hk, d, generator=g) * 0.5
    if causal:
        qs = [oracle.zigzag_shard(q, r, world) for r in range(world)]
        ks = [oracle.zigzag_shard(k, r, world) for r in range(world)]
        vs = [oracle.zigzag_shard(v, r, world) for r in range(world)]
        pos = [oracle.zigzag_positions(r, world, spr) for r in range(world)]
    else:
        qs = list(q.chunk(world))
        ks = list(k.chunk(world))
        vs = list(v.chunk(world))
        pos = None
    cast = lambda xs: [x.to(dtype).contiguous() for x in xs]  # noqa: E731
    return cast(qs), cast(ks), cast(vs), pos


def case_fused(dtype_name, causal, hq, hk, d, spr, mode):
    dtype = torch.float32 if dtype_name == "fp32" else torch.bfloat16
    info = detect_ranks()
    world, rank = info.world, info.rank
    qs, ks, vs, pos = all_inputs(world, spr, hq, hk, d, dtype, causal)
    scale = d ** -0.5
    attn = RingAttention(spr, hq, d, heads_kv=hk, dtype=dtype, causal=causal,
                         ring_mode=mode)
    dev = torch.device("cuda", attn.runtime.device)
    q, k, v = qs[rank].to(dev), ks[rank].to(dev), vs[rank].to(dev)
    for _ in range(3):  # repeated calls exercise the epoch / flag protocol
        out, lse = attn(q, k, v, return_lse=True, check=True)
    torch.cuda.synchronize(dev)
    ref = oracle.ring_attention([x.double() for x in qs], [x.double() for x in ks],
                                [x.double() for x in vs], scale, pos)[rank]
    err = (out.double().cpu() - ref).abs().max().item()
    tol = 2e-5 if dtype == torch.float32 else 2e-2
    attn.close()
    if not err < tol:
        raise SystemExit(f"rank {rank}: fused {dtype_name} causal={causal} mode={mode} "
                         f"err {err} > {tol}")
    print(f"rank {rank}: fused ok err={err:.2e}", flush=True)


def case_graph(dtype_name, causal, hq, hk, d, spr):
    """Device-side epochs: one call captured into a CUDA graph on every rank,
    then replayed in step with fresh inputs written into the captured tensors;
    each replay checked against the float64 oracle (and, in between, an eager
    call on the same engine keeps the call counter in step)."""
    dtype = torch.float32 if dtype_name == "fp32" else torch.bfloat16
    info = detect_ranks()
    world, rank = info.world, info.rank
    scale = d ** -0.5
    attn = RingAttention(spr, hq, d, heads_kv=hk, dtype=dtype, causal=causal, graph_safe=True)
    dev = torch.device("cuda", attn.runtime.device)
    qs, ks, vs, pos = all_inputs(world, spr, hq, hk, d, dtype, causal)
    q, k, v = qs[rank].to(dev), ks[rank].to(dev), vs[rank].to(dev)
    graph, out = attn.capture(q, k, v)
    tol = 2e-5 if dtype == torch.float32 else 2e-2
    for rep in range(3):
        g = torch.Generator().manual_seed(100 + rep)
        total = world * spr
        glob = [torch.randn(total, hq, d, generator=g) * 0.5,
                torch.randn(total, hk, d, generator=g) * 0.5,
                torch.randn(total, hk, d, generator=g) * 0.5]
        if causal:
            sh = [[oracle.zigzag_shard(t, r, world).to(dtype) for t in glob] for r in range(world)]
        else:
            sh = [[t.chunk(world)[r].to(dtype).contiguous() for t in glob] for r in range(world)]
        for dst, src in zip((q, k, v), sh[rank]):
            dst.copy_(src)
        graph.replay()
        if rep == 1:  # an eager call between replays advances the same counter
            attn(q, k, v, check=True)
        torch.cuda.synchronize(dev)
        attn.check()
        ref = oracle.ring_attention([s[0].double() for s in sh], [s[1].double() for s in sh],
                                    [s[2].double() for s in sh], scale, pos)[rank]
        err = (out.double().cpu() - ref).abs().max().item()
        if not err < tol:
            raise SystemExit(f"rank {rank}: graph replay {rep} err {err} > {tol}")
    del graph
    attn.close()
    print(f"rank {rank}: graph ok", flush=True)


def case_comm(nbytes):
    C = _ext.load()
    info = detect_ranks()
    rt = RingRuntime(C.comm_arena_bytes(nbytes), need_nccl=True, info=info)
    for b in ("staged", "staged_Isendrecv", "cuda_aware", "cuda_aware_Isendrecv", "nccl",
              "b200_fused"):
        avg = C.run_comm_bench(rt.ctx, b, nbytes, 1, 3, 0, True)  # precheck verifies delivery
        if rt.rank == 0:
            print(f"comm {b}: {avg}", flush=True)
    # every data path of the b200_fused kernel: 16-byte and 32-byte pushes, TMA
    # bulk pushes, 16-byte pulls (the run ends with a full-content check)
    for mode in (0, 1, 2, 3):
        avg = C.run_comm_bench(rt.ctx, "b200_fused", nbytes, 1, 3, 0, True, mode)
        if rt.rank == 0:
            print(f"comm b200_fused mode {mode}: {avg}", flush=True)
    rt.close()


def case_attn_backends(spr):
    """All eight attention schedules on N(0,1) fp32 data against the oracle."""
    C = _ext.load()
    info = detect_ranks()
    world, rank = info.world, info.rank
    xs = [inputs.normal_inputs(r, spr, 1, 64) for r in range(world)]
    ref = oracle.ring_attention([x.q for x in xs], [x.k for x in xs], [x.v for x in xs],
                                xs[0].scale)[rank]
    arena = C.AttnBench.arena_bytes("fp32", spr, 1, 64, False, world)
    rt = RingRuntime(arena, need_nccl=True, info=info)
    for b in ("staged", "staged_Isendrecv", "staged_Isendrecv_overlap", "cuda_aware",
              "cuda_aware_Isendrecv", "cuda_aware_Isendrecv_overlap", "nccl", "b200_fused"):
        for kernel in (("tcgen05", "simt") if b == "nccl" else ("tcgen05",)):
            bench = C.AttnBench(rt.ctx, b, "fp32", spr, 1, 1, 64, xs[rank].scale, False, False,
                                False, kernel, False, 1, 2, 10.0)
            bench.set_inputs(xs[rank].q, xs[rank].k, xs[rank].v)
            res = bench.run()
            out = torch.empty(spr, 1, 64)
            bench.output(out)
            err = (out.double() - ref).abs().max().item()
            if not err < 5e-5:
                raise SystemExit(f"rank {rank}: {b}/{kernel} err {err}")
            if rank == 0:
                print(f"attn {b}/{kernel}: total {res['total']:.3f} ms err {err:.2e}", flush=True)
            del bench
    rt.close()


if __name__ == "__main__":
    c = sys.argv[1]
    if c == "fused":
        case_fused(sys.argv[2], sys.argv[3] == "1", int(sys.argv[4]), int(sys.argv[5]),
                   int(sys.argv[6]), int(sys.argv[7]), sys.argv[8])
    elif c == "graph":
        case_graph(sys.argv[2], sys.argv[3] == "1", int(sys.argv[4]), int(sys.argv[5]),
                   int(sys.argv[6]), int(sys.argv[7]))
    elif c == "comm":
        case_comm(int(sys.argv[2]))
    elif c == "attn":
        case_attn_backends(int(sys.argv[2]))
    else:
        raise SystemExit(f"unknown case {c}")
