#!/usr/bin/env python3
"""Headline benchmark: fused ring attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the reference's full ring attention at its largest ATTENTION_SIZES
entry, with N(0,1) data): every rank holds a 1,048,576-element K/V block laid
out as [16384 tokens, 1 head, d=64] plus Q of the same shape, fp32, i.i.d.
N(0,1) with seed = rank, softmax scale 1/sqrt(64), non-causal.  One step is one
full ring-attention forward over all N blocks (N*16384 keys) on every rank,
through the `b200_fused` engine: one persistent tcgen05 kernel per rank pulls
the other ranks' blocks over NVLink while it computes.  Per-rank work grows
with N (weak scaling in tokens per rank).

Timing: W untimed warm-up steps; then K steps, each preceded by a host
barrier and an L2 flush (a 256 MiB buffer write enqueued on the launching
stream just ahead of the start event, so it is outside the timed interval and
the host has enqueued the step by the time the GPU reaches it), timed with
CUDA events on the launching stream; the step time is the max over ranks,
and the K-step loop is bracketed by a barrier plus torch.cuda.synchronize().
value = total attention FLOPs of all ranks / max-rank step time.  The e2e
number runs the same steps through the public `RingAttention` call with the
inputs copied host->device from pinned memory and the output read back every
step.  nvidia-smi samples the clocks during the timed loop.

--preset selects the workload: ref-fp32 (the headline above), mha-bf16-causal
(32 heads, d=128, 16384 tokens per rank, bf16, causal with zigzag sharding) or
gqa-bf16-long (32 query / 8 key-value heads, d=128, 65536 tokens per rank,
bf16 N(0,1)*0.5 from seed 1234, causal zigzag); causal FLOPs count the visible
(query, key) pairs only.

With --gpus N > 1 the script expects torchrun (RANK/WORLD_SIZE/LOCAL_RANK); run
directly it re-launches itself on N local ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ring_attention_fwd_tflops"
HOLD_CYCLES = 1_000_000  # device-side hold before each timed step: ~0.5 ms at 1965 MHz
# name: (tokens per rank, q heads, kv heads, head dim, dtype, causal, input scale, seed)
PRESETS = {
    # the reference's full ring attention at its largest ATTENTION_SIZES entry
    # (config.example.env:31) read as fp32 elements: 1048576 elements = 16384
    # tokens x d=64 per rank, 4194304 bytes on the reference's command line
    "ref-fp32": (16384, 1, 1, 64, "fp32", False, 1.0, None),
    # multi-head bf16, causal with zigzag sharding
    "mha-bf16-causal": (16384, 32, 32, 128, "bf16", True, 1.0, None),
    # the same shape without a mask
    "mha-bf16": (16384, 32, 32, 128, "bf16", False, 1.0, None),
    # long-context GQA layer shape: 32 q / 8 kv heads, causal zigzag, N(0,1)*0.5 seed 1234
    "gqa-bf16-long": (65536, 32, 8, 128, "bf16", True, 0.5, 1234),
}
L2_FLUSH_BYTES = 256 << 20
def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--preset", choices=tuple(PRESETS), default="ref-fp32")
    ap.add_argument("--seq", type=int, default=0, help="tokens per rank (0: preset)")
    ap.add_argument("--ring-mode", choices=("direct", "chain"), default="direct")
    ap.add_argument("--no-e2e", action="store_true")
    return ap.parse_args()


# The reference's attention programs compared with this framework's fused
# ring: its NCCL program and its best overlapped MPI program (CUDA-aware
# Isend/Irecv, the data moved GPU to GPU).
REFERENCE_BACKENDS = ("nccl", "cuda_aware_Isendrecv_overlap")


def reference_arm(args) -> int:
    """The unmodified reference programs (built by baseline/reference_arm.py with
    their own Makefile) on the same workload: 16384 fp32 tokens x d=64 per rank
    (kv_size = 4194304 bytes on their command line), one process per GPU.
    Its metric is turned into this one: 4*S*(N*S)*64 FLOPs per rank over its
    avg_total (host wall clock per iteration, max over ranks)."""
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    import reference_arm as ra

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))

    def unavailable(why):
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return 0

    seq, heads, heads_kv, head_dim, dt, causal, _, _ = PRESETS[args.preset]
    seq = args.seq or seq
    if (heads, heads_kv, head_dim, dt, causal) != (1, 1, 64, "fp32", False):
        return unavailable("the reference computes single-head fp32 d=64 non-causal attention "
                           f"only; preset {args.preset} has no counterpart")
    missing = [b for b in REFERENCE_BACKENDS
               if not os.path.exists(ra.program(f"ring_attention_{b}_gpu_bench"))]
    if missing and rank == 0 and os.path.isdir(ra.REF_SRC_DIR):
        try:  # same image on every machine: rebuild from the copied sources
            ra.install()
        except Exception as exc:  # reported below through `missing`
            print(f"bench.py: reference build failed: {exc}", file=sys.stderr)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=3600))
        dist.barrier()
    missing = [b for b in REFERENCE_BACKENDS
               if not os.path.exists(ra.program(f"ring_attention_{b}_gpu_bench"))]
    if missing:
        return unavailable(f"reference programs not built ({', '.join(missing)}); run "
                           "`python baseline/reference_arm.py install`")
    from ring_attention_benchmark_b200.utils.clocks import ClockSampler

    kv_bytes = seq * head_dim * 4
    sampler = ClockSampler(gpus=list(range(world)))
    if rank == 0:
        sampler.start()
    per_backend, first_fail = {}, None
    for b in REFERENCE_BACKENDS:
        work = os.path.join(ROOT, "baseline", "_ref", "run", f"{b}_np{world}_rank{rank}")
        rc, out, err = ra.run_attention(b, kv_bytes, args.warmup, args.steps, work)
        ms = ra.parse_avg_total_ms(out) if rank == 0 else None
        if rank == 0:
            if rc != 0 or ms is None:
                tail = (out.strip().splitlines() or err.strip().splitlines() or ["no output"])
                first_fail = first_fail or f"{b}: exit {rc}: {tail[-1].strip()}"
            else:
                lines = out.strip().splitlines()
                per_backend[b] = {"avg_total_ms": ms, "summary": [
                    l.strip() for l in lines if " bench:" in l or l.startswith("avg_total=")]}
    clocks = sampler.stop() if rank == 0 else None
    if rank != 0:
        return 0
    if not per_backend:
        return unavailable(f"the reference's own programs did not produce a result: {first_fail}")
    flops_total = 4.0 * seq * (world * seq) * head_dim * world
    for b, r in per_backend.items():
        r["tflops"] = round(flops_total / (r["avg_total_ms"] * 1e-3) / 1e12, 4)
    best = min(per_backend, key=lambda b: per_backend[b]["avg_total_ms"])
    ms = per_backend[best]["avg_total_ms"]
    value = round(flops_total / (ms * 1e-3) / 1e12, 4)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (the reference's own inputs: K = V = rank*1000 + i, its Q formula)",
        "config": {
            "model": "ring attention fwd, 1 head, d=64, non-causal, fp32 (the reference's "
                     "row-per-CTA CUDA-core kernel and merge kernel)",
            "global_batch": 1, "seq_len": world * seq, "seq_per_rank": seq,
            "kv_size_bytes_arg": kv_bytes, "parallelism": f"cp{world} (reference ring)",
            "backend": best, "per_backend": per_backend,
            "build": f"reference Makefile `make all`, NVCCFLAGS='{ra.NVCCFLAGS}', MPI_HOME="
                     "baseline/minimpi build (MPI subset: shared memory, CUDA IPC), NCCL from "
                     "torch",
            "timing": "the reference's avg_total: host wall clock per iteration, max over "
                      "ranks (its MPI_Reduce MAX), averaged over its timed iterations; it "
                      "includes its device-to-host copy of acc/l and host normalisation",
            "flops_per_step_total": flops_total,
        },
        "clocks": clocks,
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": seq * head_dim * 4 + seq * 4,
                "note": "the reference's own avg_total already ends with its D2H of acc and l "
                        "and the host normalisation; its inputs are created on the host once"},
        "gpu_launches": 2 * world * args.steps,
    }
    print(json.dumps(line), flush=True)
    return 0


def relaunch(args) -> int:
    from ring_attention_benchmark_b200.launch import launch

    return launch(args.gpus, [sys.executable] + sys.argv, timeout=1800)


def main() -> int:
    args = parse()
    os.environ.setdefault("RAB_CRASH_HANDLER", "1")  # native backtrace on a fatal signal
    if args.impl == "reference":
        return reference_arm(args)
    if args.gpus > 1 and "WORLD_SIZE" not in os.environ:
        return relaunch(args)
    if args.warmup < 3:
        print("bench.py: at least 3 warm-up steps are required", file=sys.stderr)
        return 2

    import torch

    from ring_attention_benchmark_b200 import RingAttention
    from ring_attention_benchmark_b200.models import inputs
    from ring_attention_benchmark_b200.models.oracle import attention_flops
    from ring_attention_benchmark_b200.utils.clocks import ClockSampler

    seq, heads, heads_kv, head_dim, dt, causal, mult, seed = PRESETS[args.preset]
    seq = args.seq or seq
    attn = RingAttention(seq, heads, head_dim, heads_kv=heads_kv,
                         dtype=torch.float32 if dt == "fp32" else torch.bfloat16,
                         causal=causal, zigzag=causal, ring_mode=args.ring_mode)
    rt = attn.runtime
    world, rank = rt.world, rt.rank
    if world != args.gpus:
        print(f"bench.py: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
        return 2
    dev = torch.device("cuda", rt.device)
    dtype = attn.dtype
    # before any pinned host buffer exists: keep host<->device copies on the GPU's socket
    from ring_attention_benchmark_b200.utils.affinity import bind_to_gpu
    host_affinity = bind_to_gpu(rt.device)
    def gen(r):  # rank r's inputs, drawn on this GPU (any rank can redraw any other's)
        return inputs.normal_inputs_device(r, seq, heads, head_dim, heads_kv=heads_kv,
                                           seed=r if seed is None else seed + r, mult=mult,
                                           dtype=dtype, device=dev)

    x = gen(rank)
    q = x.q.contiguous()
    k = x.k.contiguous()
    v = x.v.contiguous()
    out = torch.empty_like(q)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    total_tokens = seq * world
    if causal:  # visible (query, key) pairs of a causal mask over the global sequence
        flops_total = 4.0 * head_dim * heads * total_tokens * (total_tokens + 1) / 2
    else:
        flops_total = attention_flops(seq, total_tokens, heads, head_dim) * world

    # ---- warm-up ----
    for _ in range(args.warmup):
        attn(q, k, v, out=out)
    attn.check()

    # ---- device-timed steps ----
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(gpus=list(range(world)) if world > 1 else [rt.device])
    torch.cuda.synchronize(dev)
    rt.barrier()
    if rank == 0:
        sampler.start()
    t_wall0 = time.perf_counter()
    for i in range(args.steps):
        torch.cuda.synchronize(dev)
        rt.barrier()
        # A fixed ~0.5 ms device-side delay (torch's cycle-count spin kernel)
        # and the L2 flush (a 256 MiB write) are enqueued right before the
        # start event on the same stream: they run between the steps, and
        # while the GPU works on them the host enqueues the step, so the events
        # bracket the device's work for the step, not the host's launch latency
        # (which, with eight rank processes launching at once, also skews the
        # ranks' start times; the e2e figure below keeps every host cost).
        torch.cuda._sleep(HOLD_CYCLES)
        flush.fill_(i & 0xFF)
        starts[i].record(stream)
        attn(q, k, v, out=out)
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    rt.barrier()
    wall_ms = (time.perf_counter() - t_wall0) * 1e3
    clocks = sampler.stop() if rank == 0 else None
    attn.check()
    local = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    step_max = []
    for c in range(0, len(local), 16):
        step_max += rt.reduce_max(local[c:c + 16])
    ms_per_step = statistics.mean(step_max)
    value = flops_total / (ms_per_step * 1e-3) / 1e12

    # ---- end to end through the public call: H2D inputs, D2H output ----
    # Every step copies its Q/K/V from pinned host memory and reads its output
    # back.  The copies of step i+1 overlap the attention of step i (double-
    # buffered device inputs and outputs; host-to-device and device-to-host
    # copies on two streams, so both PCIe directions run at once), the way a
    # serving loop runs; the K-step loop is timed as a whole and divided by K.
    e2e = None
    if not args.no_e2e:
        q_h = q.cpu().pin_memory()
        k_h = k.cpu().pin_memory()
        v_h = v.cpu().pin_memory()
        outs_h = [torch.empty(q.shape, dtype=dtype).pin_memory() for _ in range(2)]
        ins = [(torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)) for _ in range(2)]
        outs_d = [torch.empty_like(q) for _ in range(2)]
        cstream = torch.cuda.Stream(dev)  # host -> device
        ostream = torch.cuda.Stream(dev)  # device -> host

        def run_e2e(nsteps):
            ev_in = [torch.cuda.Event() for _ in range(nsteps)]
            ev_comp = [torch.cuda.Event() for _ in range(nsteps)]
            ev_out = [torch.cuda.Event() for _ in range(nsteps)]
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            cstream.wait_event(t0)
            ostream.wait_event(t0)

            def h2d(i):
                with torch.cuda.stream(cstream):
                    if i >= 2:
                        cstream.wait_event(ev_comp[i - 2])  # buffer i%2 is free again
                    bq, bk, bv = ins[i % 2]
                    bq.copy_(q_h, non_blocking=True)
                    bk.copy_(k_h, non_blocking=True)
                    bv.copy_(v_h, non_blocking=True)
                    ev_in[i].record(cstream)

            h2d(0)
            for i in range(nsteps):
                if i + 1 < nsteps:
                    h2d(i + 1)
                stream.wait_event(ev_in[i])
                if i >= 2:
                    stream.wait_event(ev_out[i - 2])  # outs_d[i % 2] was read back
                bq, bk, bv = ins[i % 2]
                attn(bq, bk, bv, out=outs_d[i % 2])
                ev_comp[i].record(stream)
                with torch.cuda.stream(ostream):
                    ostream.wait_event(ev_comp[i])
                    outs_h[i % 2].copy_(outs_d[i % 2], non_blocking=True)
                    ev_out[i].record(ostream)
            stream.wait_stream(cstream)
            stream.wait_stream(ostream)
            t1.record(stream)
            torch.cuda.synchronize(dev)
            return t0.elapsed_time(t1)

        run_e2e(args.warmup)
        rt.barrier()
        e2e_ms = rt.reduce_max([run_e2e(args.steps)])[0] / args.steps
        attn.check()
        ok = bool(torch.isfinite(outs_h[0]).all()) and bool(
            torch.allclose(outs_h[(args.steps - 1) % 2], out.cpu()))
        e2e = {"value": round(flops_total / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
               "ms_per_step": round(e2e_ms, 4),
               "h2d_bytes_per_step": int((q_h.numel() + k_h.numel() + v_h.numel())
                                         * q_h.element_size()),
               "d2h_bytes_per_step": int(outs_h[0].numel() * outs_h[0].element_size()),
               "output_matches_device_timed_run": ok,
               "schedule": "H2D of step i+1 and D2H of step i-1 overlap step i on two copy "
                           "streams; K-step loop timed as a whole, steps back to back with no "
                           "L2 flush or hold between them (each step's inputs arrive by H2D)"}

    # ---- output check: sampled rows of every rank vs a float64 recomputation ----
    # over the K/V of ALL ranks, regenerated from their seeds on this GPU (not
    # read through the ring), outside every timed region
    from ring_attention_benchmark_b200.utils.verify import ring_output_error

    def kv_of(r):
        if r == rank:
            return k, v
        y = gen(r)
        return y.k, y.v

    err_local = ring_output_error(out, q, rank, world, kv_of, x.scale, causal=causal,
                                  zigzag=causal, n_rows=256)
    max_err = rt.reduce_max([err_local])[0]
    tol = 2e-5 if dt == "fp32" else 2e-2
    check = {"max_abs_err": max_err, "tol": tol, "passed": bool(max_err <= tol),
             "rows_per_rank": 256, "heads": "all",
             "oracle": "float64 over all ranks' K/V regenerated from their seeds (max over ranks)"}

    # ---- overlap trace of one extra call (outside the timed regions) ----
    overlap = attn.overlap_trace(q, k, v, out=out) if world > 1 else None

    nsplit = attn.engine.nsplit
    # ring-format prep (fp32, one launch), the fused kernel, the merge pass (split or balanced)
    per_step = (1 if dt == "fp32" else 0) + 1 + attn.engine.merge_launches
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": dt,
            "data": "synthetic",
            "config": {
                "model": (f"ring attention fwd [{args.preset}], {heads} q heads / {heads_kv} kv "
                          f"heads, d={head_dim}, {'causal zigzag' if causal else 'non-causal'}, "
                          f"{'fp32 via 3xTF32 tensor-core products' if dt == 'fp32' else 'bf16, fp32 accumulation'}"),
                "global_batch": 1,
                "seq_len": total_tokens,
                "seq_per_rank": seq,
                "kv_block_elements_per_rank": seq * heads_kv * head_dim,
                "parallelism": f"cp{world} (ring over NVLink, fused in-kernel transfer, "
                               f"{args.ring_mode} mode)",
                "data_init": (f"iid N(0,1) x {mult} from the CUDA generator seeded "
                              f"{'rank' if seed is None else f'{seed}+rank'}, "
                              f"scale 1/sqrt({head_dim})"),
                "check": check,
                "overlap": overlap,
                "l2": "256 MiB buffer written before every timed step, enqueued on the same "
                      "stream just ahead of the start event (outside the events)",
                "step_start": "after a host barrier, a ~0.5 ms device-side hold and the L2 "
                              "flush, so the events time device work, not host launch latency",
                "host_affinity": host_affinity,
                "flops_per_step_total": flops_total,
                "wall_ms_bracketed_loop": round(wall_ms, 3),
                "nsplit": nsplit,
                "grid": attn.engine.grid,
            },
            "clocks": clocks,
            "e2e": e2e,
            "gpu_launches": per_step * args.steps,
        }
        print(json.dumps(line), flush=True)
        if not check["passed"]:
            print(f"bench.py: output check failed: max abs err {max_err:.3g} > {tol:g}",
                  file=sys.stderr)
    attn.close()
    return 0 if check["passed"] else 1


if __name__ == "__main__":
    sys.exit(main())
