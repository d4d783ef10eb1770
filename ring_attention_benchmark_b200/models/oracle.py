"""Float64 CPU oracle for (ring) attention.

`partial_attention` and `merge_online_softmax` restate the reference's CPU
statement of its two kernels (``src/attention/ring_attention_staged_gpu_bench.cu``
lines 41-77 and 152-170): an unnormalised accumulator ``acc = sum_j w_j V_j``
with ``w_j = exp(s_j - m)``, the row max ``m`` and the row sum ``l``, merged
across ring steps by rescaling both sides to the common max.  `ring_attention`
runs the ring in the reference's block order (own block first, then the blocks
of ranks r-1, r-2, ...; ``src/attention/ring_attention_nccl_gpu_bench.cu``
lines 331-376) and `full_attention` is the independent check: softmax over the
concatenated sequence.

Tensors are ``[seq, heads, dim]``.  Grouped-query attention maps query head
``h`` to key/value head ``h // (heads // heads_kv)``.  Causal masks are given in
global token positions so zigzag-sharded ranks can be checked against the
unsharded sequence.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import torch

NEG_INF = float("-inf")


def _expand_kv(k: torch.Tensor, heads: int) -> torch.Tensor:
    hk = k.shape[1]
    if hk == heads:
        return k
    if heads % hk:
        raise ValueError(f"heads={heads} is not a multiple of heads_kv={hk}")
    return k.repeat_interleave(heads // hk, dim=1)


def scores(q: torch.Tensor, k: torch.Tensor, scale: float) -> torch.Tensor:
    """[heads, seq_q, seq_k] float64 scores."""
    q64 = q.double()
    k64 = _expand_kv(k.double(), q.shape[1])
    s = torch.einsum("qhd,khd->hqk", q64, k64)
    if scale != 1.0:
        s = s * scale
    return s


def _mask(s: torch.Tensor, q_pos: Optional[torch.Tensor], k_pos: Optional[torch.Tensor]):
    if q_pos is None:
        return s
    allowed = k_pos.view(1, 1, -1) <= q_pos.view(1, -1, 1)
    return s.masked_fill(~allowed, NEG_INF)


def partial_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float = 1.0,
    q_pos: Optional[torch.Tensor] = None,
    k_pos: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Unnormalised block attention: returns (acc [sq,h,d], m [sq,h], l [sq,h]).

    Rows that see no key (fully masked) get m = -inf, l = 0, acc = 0.
    """
    s = _mask(scores(q, k, scale), q_pos, k_pos)
    m = s.amax(dim=-1)  # [h, sq]
    m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    w = torch.exp(s - m_safe.unsqueeze(-1))
    l = w.sum(dim=-1)
    v64 = _expand_kv(v.double(), q.shape[1])
    acc = torch.einsum("hqk,khd->qhd", w, v64)
    return acc, m.transpose(0, 1).contiguous(), l.transpose(0, 1).contiguous()


def merge_online_softmax(
    run: Tuple[torch.Tensor, torch.Tensor, torch.Tensor],
    new: Tuple[torch.Tensor, torch.Tensor, torch.Tensor],
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Merge (acc, m, l) states; both accumulators stay unnormalised."""
    acc_r, m_r, l_r = run
    acc_n, m_n, l_n = new
    m = torch.maximum(m_r, m_n)
    m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    a = torch.exp(m_r - m_safe)
    b = torch.exp(m_n - m_safe)
    a = torch.where(torch.isinf(m_r) & (m_r < 0), torch.zeros_like(a), a)
    b = torch.where(torch.isinf(m_n) & (m_n < 0), torch.zeros_like(b), b)
    acc = a.unsqueeze(-1) * acc_r + b.unsqueeze(-1) * acc_n
    return acc, m, a * l_r + b * l_n


def empty_state(seq_q: int, heads: int, dim: int):
    return (
        torch.zeros(seq_q, heads, dim, dtype=torch.float64),
        torch.full((seq_q, heads), NEG_INF, dtype=torch.float64),
        torch.zeros(seq_q, heads, dtype=torch.float64),
    )


def normalize(state) -> torch.Tensor:
    acc, _, l = state
    return acc / l.unsqueeze(-1)


def lse(state) -> torch.Tensor:
    _, m, l = state
    return m + torch.log(l)


def full_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float = 1.0,
    q_pos: Optional[torch.Tensor] = None,
    k_pos: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Softmax attention over the whole key sequence (float64)."""
    s = _mask(scores(q, k, scale), q_pos, k_pos)
    p = torch.softmax(s, dim=-1)
    v64 = _expand_kv(v.double(), q.shape[1])
    return torch.einsum("hqk,khd->qhd", p, v64)


def ring_block_order(rank: int, world: int) -> List[int]:
    """Ranks whose K/V block rank `rank` consumes at ring steps 0..world-1."""
    return [(rank - s) % world for s in range(world)]


def ring_attention(
    qs: Sequence[torch.Tensor],
    ks: Sequence[torch.Tensor],
    vs: Sequence[torch.Tensor],
    scale: float = 1.0,
    positions: Optional[Sequence[torch.Tensor]] = None,
) -> List[torch.Tensor]:
    """Reference ring: every rank folds blocks in ring order, normalises once."""
    world = len(qs)
    outs = []
    for r in range(world):
        state = empty_state(qs[r].shape[0], qs[r].shape[1], vs[r].shape[2])
        for src in ring_block_order(r, world):
            qp = positions[r] if positions is not None else None
            kp = positions[src] if positions is not None else None
            state = merge_online_softmax(
                state, partial_attention(qs[r], ks[src], vs[src], scale, qp, kp)
            )
        outs.append(normalize(state))
    return outs


# ---------------------------------------------------------------------------
# zigzag sharding for causal ring attention
# ---------------------------------------------------------------------------
def zigzag_positions(rank: int, world: int, seq_per_rank: int) -> torch.Tensor:
    """Global token positions held by `rank`: chunks r and 2*world-1-r.

    The global sequence of world*seq_per_rank tokens is cut into 2*world equal
    chunks; pairing an early chunk with a late one gives every rank the same
    causal work.
    """
    if seq_per_rank % 2:
        raise ValueError("zigzag sharding needs an even number of tokens per rank")
    c = seq_per_rank // 2
    first = torch.arange(rank * c, (rank + 1) * c)
    j = 2 * world - 1 - rank
    second = torch.arange(j * c, (j + 1) * c)
    return torch.cat([first, second])


def zigzag_shard(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Take rank's zigzag shard of a [seq_total, ...] tensor."""
    pos = zigzag_positions(rank, world, x.shape[0] // world)
    return x[pos]


def zigzag_unshard(shards: Sequence[torch.Tensor]) -> torch.Tensor:
    world = len(shards)
    spr = shards[0].shape[0]
    out = torch.empty((world * spr,) + tuple(shards[0].shape[1:]), dtype=shards[0].dtype)
    for r, s in enumerate(shards):
        out[zigzag_positions(r, world, spr)] = s
    return out


def attention_flops(seq_q: int, seq_k: int, heads: int, dim: int, causal_fraction: float = 1.0):
    """Forward FLOPs of softmax attention: 2 GEMMs of 2*sq*sk*d each per head."""
    return 4.0 * seq_q * seq_k * dim * heads * causal_fraction


def default_scale(dim: int) -> float:
    return 1.0 / math.sqrt(dim)
