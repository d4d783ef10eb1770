"""Ring attention on CPU ranks over torch.distributed (gloo), in fp32.

A plain restatement of the reference's algorithm without any GPU: every rank
keeps its queries, folds its own K/V block first, then passes the block it
holds to rank r+1 and receives the next one from rank r-1 (world-1 exchanges),
merging each block's partial (acc, m, l) into a running state and normalising
once at the end (``src/attention/ring_attention_nccl_gpu_bench.cu`` lines
331-394).  Used to test the host-side plumbing and the merge arithmetic with
real processes, and as the CPU baseline of the BASELINE config with two ranks.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def partial_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                 mask: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, ...]:
    """(acc, m, l) of one block in fp32; q [sq,h,d], k/v [sk,hk,d]."""
    h, hk = q.shape[1], k.shape[1]
    if hk != h:
        k = k.repeat_interleave(h // hk, dim=1)
        v = v.repeat_interleave(h // hk, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), k.float()) * scale
    if mask is not None:
        s = s.masked_fill(~mask.unsqueeze(0), float("-inf"))
    m = s.amax(-1)
    m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    w = torch.exp(s - m_safe.unsqueeze(-1))
    return torch.einsum("hqk,khd->qhd", w, v.float()), m.t().contiguous(), w.sum(-1).t().contiguous()


def merge_fp32(run, new):
    acc_r, m_r, l_r = run
    acc_n, m_n, l_n = new
    m = torch.maximum(m_r, m_n)
    m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    a = torch.where(torch.isinf(m_r), torch.zeros_like(m_r), torch.exp(m_r - m_safe))
    b = torch.where(torch.isinf(m_n), torch.zeros_like(m_n), torch.exp(m_n - m_safe))
    return a.unsqueeze(-1) * acc_r + b.unsqueeze(-1) * acc_n, m, a * l_r + b * l_n


class RingDataError(RuntimeError):
    """A block received over the ring is not finite (a corrupt or NaN shard)."""


def ring_attention_cpu(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       scale: Optional[float] = None,
                       q_pos: Optional[torch.Tensor] = None,
                       pos_of_rank=None, group=None, check_finite: bool = True) -> torch.Tensor:
    """Every rank calls this with its own shard; returns its normalised output.

    For causal masking pass this rank's global query positions `q_pos` and
    `pos_of_rank(r)` giving rank r's key positions.  With `check_finite` every
    received block is checked and a non-finite one raises `RingDataError`
    naming the rank it came from and the step.  A peer that stops taking part
    makes the exchange fail within the process group's timeout.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    sq, h, d = q.shape
    state = (torch.zeros(sq, h, d), torch.full((sq, h), float("-inf")), torch.zeros(sq, h))
    cur_k, cur_v = k.contiguous().float(), v.contiguous().float()
    right, left = (rank + 1) % world, (rank - 1) % world
    for step in range(world):
        src = (rank - step) % world
        mask = None
        if q_pos is not None:
            mask = pos_of_rank(src).view(1, -1) <= q_pos.view(-1, 1)
        state = merge_fp32(state, partial_fp32(q, cur_k, cur_v, scale, mask))
        if step < world - 1:
            nk, nv = torch.empty_like(cur_k), torch.empty_like(cur_v)
            ops = [dist.P2POp(dist.isend, cur_k, right, group), dist.P2POp(dist.isend, cur_v, right, group),
                   dist.P2POp(dist.irecv, nk, left, group), dist.P2POp(dist.irecv, nv, left, group)]
            for req in dist.batch_isend_irecv(ops):
                req.wait()
            if check_finite and not (torch.isfinite(nk).all() and torch.isfinite(nv).all()):
                origin = (rank - step - 1) % world
                raise RingDataError(
                    f"rank {rank}: K/V block of rank {origin} received from rank {left} at ring "
                    f"step {step + 1} is not finite")
            cur_k, cur_v = nk, nv
    acc, _, l = state
    return acc / l.unsqueeze(-1)
