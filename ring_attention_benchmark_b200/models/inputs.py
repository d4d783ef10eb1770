"""Synthetic inputs.

Two families:

* ``ref_compat``: exactly the reference benchmark's data.  One K/V buffer per
  rank with ``kv[i] = rank*1000 + i`` over the flat ``[seq, 64]`` index, used as
  both K and V (``src/attention/ring_attention_staged_gpu_bench.cu`` lines
  271-273 and 362-366), and ``Q[i] = (rank*500 + (i % 64)*0.01) * 0.001``
  (lines 278-280), so every query row on a rank is identical.  No softmax scale.
* ``normal``: i.i.d. N(0, 1) Q/K/V from a seeded generator (seed = rank unless
  given), scale 1/sqrt(d), optionally multiplied by a constant and cast.

The comm-only benchmark fills its shard with ``rank*1000 + i`` like the
reference's loops (``src/loop/ring_loop_staged.cu`` lines 111-117).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class AttnInputs:
    q: torch.Tensor  # [seq, heads, d]
    k: torch.Tensor  # [seq, heads_kv, d]
    v: torch.Tensor  # [seq, heads_kv, d]
    scale: float
    kv_shared: bool  # K and V are the same buffer (reference-compatible data)


def ref_compat_kv(rank: int, seq: int, dim: int = 64) -> torch.Tensor:
    n = seq * dim
    idx = torch.arange(n, dtype=torch.float32)
    return (rank * 1000.0 + idx).view(seq, 1, dim)


def ref_compat_q(rank: int, seq: int, dim: int = 64) -> torch.Tensor:
    col = torch.arange(seq * dim) % dim
    q = (rank * 500.0 + col.to(torch.float32) * 0.01) * 0.001
    return q.to(torch.float32).view(seq, 1, dim)


def ref_compat_inputs(rank: int, seq: int, dim: int = 64) -> AttnInputs:
    kv = ref_compat_kv(rank, seq, dim)
    return AttnInputs(q=ref_compat_q(rank, seq, dim), k=kv, v=kv, scale=1.0, kv_shared=True)


def normal_inputs(
    rank: int,
    seq: int,
    heads: int = 1,
    dim: int = 64,
    heads_kv: Optional[int] = None,
    seed: Optional[int] = None,
    mult: float = 1.0,
    dtype: torch.dtype = torch.float32,
) -> AttnInputs:
    hk = heads if heads_kv is None else heads_kv
    g = torch.Generator(device="cpu").manual_seed(rank if seed is None else seed)
    q = torch.randn(seq, heads, dim, generator=g) * mult
    k = torch.randn(seq, hk, dim, generator=g) * mult
    v = torch.randn(seq, hk, dim, generator=g) * mult
    return AttnInputs(
        q=q.to(dtype), k=k.to(dtype), v=v.to(dtype), scale=dim ** -0.5, kv_shared=False
    )


def comm_init(rank: int, n_floats: int) -> torch.Tensor:
    return rank * 1000.0 + torch.arange(n_floats, dtype=torch.float32)


def size_to_seq(kv_size_bytes: int, dim: int = 64, elem_bytes: int = 4) -> int:
    """Tokens per rank for a K/V shard of `kv_size_bytes` (reference CLI units)."""
    if kv_size_bytes <= 0 or kv_size_bytes % (dim * elem_bytes):
        raise ValueError(f"kv_size_bytes must be a positive multiple of {dim * elem_bytes}")
    return kv_size_bytes // (dim * elem_bytes)


def normal_inputs_device(
    rank: int,
    seq: int,
    heads: int = 1,
    dim: int = 64,
    heads_kv: Optional[int] = None,
    seed: Optional[int] = None,
    mult: float = 1.0,
    dtype: torch.dtype = torch.float32,
    device="cuda",
) -> AttnInputs:
    """`normal_inputs` drawn on the GPU from a seeded ``torch.Generator`` of
    that device (Philox; the same values on every GPU for the same seed), so
    any rank can regenerate any other rank's inputs in milliseconds - the
    benchmark's output check rebuilds the whole ring's K/V this way.  Values
    differ from the CPU generator's for the same seed."""
    hk = heads if heads_kv is None else heads_kv
    g = torch.Generator(device=device).manual_seed(rank if seed is None else seed)
    q = torch.randn(seq, heads, dim, generator=g, device=device) * mult
    k = torch.randn(seq, hk, dim, generator=g, device=device) * mult
    v = torch.randn(seq, hk, dim, generator=g, device=device) * mult
    return AttnInputs(
        q=q.to(dtype), k=k.to(dtype), v=v.to(dtype), scale=dim ** -0.5, kv_shared=False
    )
