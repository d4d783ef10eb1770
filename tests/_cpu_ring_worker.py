"""One gloo rank of the CPU ring-attention test (world 2,
per-rank [256, 1, 64] Q/K/V, N(0,1) from seed 0, non-causal, scale 1/sqrt(64);
plus a causal zigzag GQA case on 4 ranks)."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from ring_attention_benchmark_b200.models import oracle  # noqa: E402
from ring_attention_benchmark_b200.models.cpu_ring import ring_attention_cpu  # noqa: E402


def fault(case):
    """Injected on the host: rank 1 sends NaN K/V ("fault_nan") or leaves before
    the ring ("fault_exit"); the others must fail with a clear error, fast."""
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=8))
    rank, world = dist.get_rank(), dist.get_world_size()
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(64, 1, 32, generator=g) for _ in range(3))
    if rank == 1 and case == "fault_exit":
        print("rank 1 leaves before the ring", flush=True)
        os._exit(3)
    if rank == 1 and case == "fault_nan":
        k = torch.full_like(k, float("nan"))
    ring_attention_cpu(q, k, v)
    print(f"rank {rank} finished the ring", flush=True)


def main():
    case = sys.argv[1]
    if case.startswith("fault_"):
        return fault(case)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    g = torch.Generator().manual_seed(0)
    if case == "config1":
        seq, h, hk, d = 256, 1, 1, 64
        qs = [torch.randn(seq, h, d, generator=g) for _ in range(world)]
        ks = [torch.randn(seq, hk, d, generator=g) for _ in range(world)]
        vs = [torch.randn(seq, hk, d, generator=g) for _ in range(world)]
        out = ring_attention_cpu(qs[rank], ks[rank], vs[rank])
        full = oracle.full_attention(torch.cat(qs), torch.cat(ks), torch.cat(vs), d ** -0.5)
        ref = full[rank * seq:(rank + 1) * seq]
    else:  # causal zigzag GQA
        spr, h, hk, d = 64, 4, 2, 32
        total = world * spr
        q = torch.randn(total, h, d, generator=g)
        k = torch.randn(total, hk, d, generator=g)
        v = torch.randn(total, hk, d, generator=g)
        pos = lambda r: oracle.zigzag_positions(r, world, spr)  # noqa: E731
        out = ring_attention_cpu(oracle.zigzag_shard(q, rank, world),
                                 oracle.zigzag_shard(k, rank, world),
                                 oracle.zigzag_shard(v, rank, world), q_pos=pos(rank),
                                 pos_of_rank=pos)
        allpos = torch.arange(total)
        full = oracle.full_attention(q, k, v, d ** -0.5, allpos, allpos)
        ref = full[pos(rank)]
    err = (out.double() - ref).abs().max().item()
    dist.destroy_process_group()
    if not err < 1e-5:
        raise SystemExit(f"rank {rank}: {case} err {err}")
    print(f"rank {rank} {case} ok err={err:.2e}", flush=True)


if __name__ == "__main__":
    main()
