"""Python surface of the attention kernels (sm_100a).

* `flash_attention`: tcgen05 flash forward over K/V blocks that are already on
  this GPU (ring order), bf16 or fp32 (3xTF32) - the kernel the fused ring
  backend runs, here without the in-kernel NVLink transfer.
* `partial_attention`: one ring step of the unfused baselines - unnormalised
  accumulator plus row max / row sum (the reference's C16 kernel contract,
  ``src/attention/ring_attention_staged_gpu_bench.cu`` lines 78-143), on the
  tensor cores or on the exact-order CUDA-core kernel.
* `merge_lse`, `normalize`: the reference's C17 merge and C19 normalisation as
  device kernels.

All tensors are ``[seq, heads, dim]`` and must live on the GPU.  Every call goes
to the native extension; there is no PyTorch fallback.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from .._ext import load

PREC_BF16 = 0
PREC_FP32 = 1  # fp32 storage, 3xTF32 tensor-core products


def prec_of(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return PREC_BF16
    if dtype == torch.float32:
        return PREC_FP32
    raise ValueError(f"unsupported dtype {dtype}; use bfloat16 or float32")


def new_status(device) -> torch.Tensor:
    return torch.zeros(8, dtype=torch.int32, device=device)


class DeviceTimeout(RuntimeError):
    """A bounded device-side wait ran out (status word set by a kernel)."""


WAIT_SITES = {
    1: "q_full", 2: "k_full", 3: "v_full", 4: "k_empty", 5: "v_empty", 6: "s_full",
    7: "p_full", 8: "o_ready", 9: "block_ready", 10: "peer_ready", 11: "peer_consumed",
    12: "copy_slice", 13: "ring_flag", 14: "test", 15: "pv_done", 16: "item_queue",
}


def check_status(status: torch.Tensor, what: str = "kernel") -> None:
    s = status.tolist()
    if s[0] != 0:
        site = WAIT_SITES.get(s[1], str(s[1]))
        raise DeviceTimeout(
            f"{what}: device status code={s[0]} site={site} block={s[2]} detail={s[3]} "
            f"errors={s[4]}"
        )


def ring_slots(ks: Sequence[torch.Tensor], vs: Sequence[torch.Tensor]) -> torch.Tensor:
    """Pack K/V blocks into consecutive ring-format slots (uint8 buffer)."""
    C = load()
    k0 = ks[0]
    prec = prec_of(k0.dtype)
    skv, hkv, d = k0.shape
    bb = C.ring_block_bytes(prec, skv, hkv, d)
    slots = torch.empty(bb * len(ks), dtype=torch.uint8, device=k0.device)
    for i, (k, v) in enumerate(zip(ks, vs)):
        C.ring_format(prec, k.contiguous(), v.contiguous(), slots[i * bb:(i + 1) * bb])
    return slots


def flash_attention(
    q: torch.Tensor,
    ks: Sequence[torch.Tensor],
    vs: Sequence[torch.Tensor],
    scale: Optional[float] = None,
    causal: bool = False,
    zigzag: bool = False,
    world: int = 1,
    rank: int = 0,
    nsplit: int = 0,
    out_dtype: Optional[torch.dtype] = None,
    return_lse: bool = False,
    slots: Optional[torch.Tensor] = None,
    timeout_s: float = 10.0,
):
    """Attention of `q` over the blocks `ks`/`vs` (block i = ring step i).

    With ``causal`` the mask uses global positions: block i comes from rank
    ``(rank - i) % world``; ``zigzag`` selects the balanced sharding in which
    rank r holds global chunks r and 2*world-1-r.

    ``nsplit`` picks the work schedule of the persistent kernel: 0 lets the
    planner choose, n > 0 splits every 128-row query tile's KV range into n
    equal chunks, -1 forces the balanced schedule (each CTA takes an equal
    share of all (query tile, KV tile) pairs; needs ``causal=False``).
    """
    C = load()
    prec = prec_of(q.dtype)
    sq, hq, d = q.shape
    skv, hkv, _ = ks[0].shape
    if scale is None:
        scale = d ** -0.5
    if slots is None:
        slots = ring_slots(ks, vs)
    out = torch.empty(sq, hq, d, dtype=out_dtype or q.dtype, device=q.device)
    lse = torch.empty(sq, hq, dtype=torch.float32, device=q.device) if return_lse else None
    status = new_status(q.device)
    C.flash_fwd(prec, q.contiguous(), slots, len(ks), skv, hkv, out=out, lse=lse, scale=scale,
                causal=causal, zigzag=zigzag, world=world, rank=rank, nsplit=nsplit,
                status=status, timeout_s=timeout_s)
    check_status(status, "flash_fwd")
    return (out, lse) if return_lse else out


def partial_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float = 1.0,
    kernel: str = "tcgen05",
    out: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
    nsplit: int = 0,
):
    """One ring step: returns (acc unnormalised, m natural-log row max, l row sum).

    ``nsplit`` selects the work schedule as in :func:`flash_attention`.
    """
    C = load()
    sq, hq, d = q.shape
    if out is None:
        out = (
            torch.empty(sq, hq, d, dtype=torch.float32, device=q.device),
            torch.empty(sq, hq, dtype=torch.float32, device=q.device),
            torch.empty(sq, hq, dtype=torch.float32, device=q.device),
        )
    acc, m, l = out
    if kernel == "simt":
        C.simt_partial_attention(q.contiguous(), k.contiguous(), v.contiguous(), acc, m, l, scale,
                                 -1, False)
        return acc, m, l
    prec = prec_of(q.dtype)
    slots = ring_slots([k], [v])
    status = new_status(q.device)
    C.flash_fwd(prec, q.contiguous(), slots, 1, k.shape[0], k.shape[1], scale=scale, acc=acc,
                m=m, l=l, status=status, nsplit=nsplit)
    check_status(status, "flash_fwd(partial)")
    return acc, m, l


def merge_lse(run, new) -> None:
    """In-place online-softmax merge of `new` (acc, m, l) into `run`."""
    acc_r, m_r, l_r = run
    acc_n, m_n, l_n = new
    load().merge_lse(m_r, l_r, acc_r, m_n, l_n, acc_n)


def normalize(acc, m, l, out_dtype=torch.float32, want_lse=False):
    C = load()
    out = torch.empty(acc.shape, dtype=out_dtype, device=acc.device)
    lse = torch.empty(m.shape, dtype=torch.float32, device=acc.device) if want_lse else None
    C.normalize(acc, m, l, out, lse)
    return (out, lse) if want_lse else out
