"""Output check of a ring-attention run against a float64 recomputation.

`ring_output_error` takes one rank's output, recomputes a sample of its query
rows (every head) over the keys of ALL ranks in float64, and returns the
largest absolute difference.  The other ranks' K/V blocks are regenerated on
this rank's GPU from their seeds (`inputs.normal_inputs_device`), never read
through the ring, so the check is independent of the transport it verifies.
The float64 products run as device GEMMs; memory stays at one block of one
head at a time.  Causal runs mask by global token position (zigzag or
contiguous sharding), like `oracle.full_attention`.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from ..models import oracle


def sample_rows(seq: int, n: int = 256) -> torch.Tensor:
    """`n` query rows spread evenly over [0, seq), first and last included."""
    n = min(n, seq)
    return torch.linspace(0, seq - 1, n).round().long().unique()


def _positions(rank: int, world: int, seq: int, zigzag: bool) -> torch.Tensor:
    if zigzag:
        return oracle.zigzag_positions(rank, world, seq)
    return torch.arange(rank * seq, (rank + 1) * seq)


@torch.no_grad()
def ring_output_error(out: torch.Tensor, q: torch.Tensor, rank: int, world: int,
                      kv_of: Callable[[int], "tuple[torch.Tensor, torch.Tensor]"],
                      scale: float, causal: bool = False, zigzag: bool = False,
                      n_rows: int = 256, rows: Optional[torch.Tensor] = None) -> float:
    """max |out - reference| over the sampled rows of this rank.

    out, q: this rank's [seq, heads, d] output and queries (on its GPU);
    kv_of(r): rank r's (k, v) [seq, heads_kv, d] on the same GPU, in the
    precision the kernel consumed.
    """
    dev = out.device
    seq, heads, d = q.shape
    rows = sample_rows(seq, n_rows) if rows is None else rows
    rows_d = rows.to(dev)
    q64 = q.index_select(0, rows_d).double()  # [R, H, D]
    qpos = _positions(rank, world, seq, zigzag).index_select(0, rows).to(dev) if causal else None
    R = rows.numel()
    m = torch.full((heads, R), float("-inf"), dtype=torch.float64, device=dev)
    l = torch.zeros(heads, R, dtype=torch.float64, device=dev)
    acc = torch.zeros(heads, R, d, dtype=torch.float64, device=dev)
    for src in oracle.ring_block_order(rank, world):
        k, v = kv_of(src)
        hk = k.shape[1]
        group = heads // hk
        kpos = _positions(src, world, seq, zigzag).to(dev) if causal else None
        for kh in range(hk):
            kk = k[:, kh].double()  # [S, D]
            vv = v[:, kh].double()
            for h in range(kh * group, (kh + 1) * group):
                s = (q64[:, h] @ kk.T) * scale  # [R, S]
                if causal:
                    s = s.masked_fill(kpos.view(1, -1) > qpos.view(-1, 1), float("-inf"))
                mb = s.amax(dim=1)
                mn = torch.maximum(m[h], mb)
                safe = torch.where(torch.isinf(mn), torch.zeros_like(mn), mn)
                a = torch.exp(m[h] - safe)
                w = torch.exp(s - safe.view(-1, 1))
                l[h] = l[h] * a + w.sum(dim=1)
                acc[h] = acc[h] * a.view(-1, 1) + w @ vv
                m[h] = mn
    ref = (acc / l.unsqueeze(-1)).transpose(0, 1)  # [R, H, D]
    got = out.index_select(0, rows_d).double()
    return float((got - ref).abs().max().item())
