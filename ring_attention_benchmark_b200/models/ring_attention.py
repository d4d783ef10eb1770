"""Public API: ring attention over all ranks of the job, fused on B200.

    from ring_attention_benchmark_b200 import RingAttention
    attn = RingAttention(seq_per_rank=16384, heads=1, head_dim=64, dtype=torch.float32)
    out = attn(q, k, v)          # q [S, H, D], k/v [S, Hkv, D] on this rank's GPU

Every rank calls it with its own sequence shard.  The whole ring (all
world-size key/value blocks, in the reference's order: own block first, then
the blocks of ranks r-1, r-2, ...) runs in one persistent sm_100a kernel per
call: the K/V blocks of the other ranks are pulled over NVLink into this
rank's ring slots inside the kernel while the tensor cores already work on the
blocks that are present, and the online-softmax state never leaves the chip.

* fp32 inputs are computed with 3xTF32 tensor-core products (fp32-level
  accuracy); bf16 inputs with bf16 products and fp32 accumulation.
* ``causal=True`` masks by global token position; ``zigzag=True`` (default for
  causal) expects the balanced sharding in which rank r holds the global chunks
  r and 2*world-1-r (see `oracle.zigzag_shard`).
* GQA: ``heads_kv`` divides ``heads``; only the ``heads_kv`` heads rotate.
* ``ring_mode="chain"`` forwards each block along the ring (rank r copies block
  s from rank r-1's slot s-1) instead of reading it from its origin.

The engine allocates its ring slots once (``world`` blocks in the symmetric,
IPC-mapped arena).  Writing K and V straight into slot 0 (``kv_slot()``) skips
the per-call copy for bf16 inputs.

CUDA graphs: a call is a fixed sequence of launches on the current stream, but
with more than one rank the fused kernel's launch parameters carry the call's
epoch (the flag values it waits for).  ``graph_safe=True`` moves the epoch into
a call counter in device memory that the kernel itself advances, so a call
captured once (``capture()``, or any ``torch.cuda.graph`` region) can be
replayed; every rank must capture and replay in step, one replay being one
ring call, with the same input and output tensors each time.
"""
from __future__ import annotations

from typing import Optional

import torch

from .._ext import load
from ..parallel.dist import RingRuntime

_DTYPES = {torch.float32: "fp32", torch.bfloat16: "bf16"}


class RingAttention:
    def __init__(self, seq_per_rank: int, heads: int = 1, head_dim: int = 64,
                 heads_kv: Optional[int] = None, dtype: torch.dtype = torch.float32,
                 causal: bool = False, zigzag: Optional[bool] = None, ring_mode: str = "direct",
                 runtime: Optional[RingRuntime] = None, timeout_s: float = 10.0,
                 graph_safe: bool = False):
        if dtype not in _DTYPES:
            raise ValueError("dtype must be torch.float32 or torch.bfloat16")
        if ring_mode not in ("direct", "chain"):
            raise ValueError("ring_mode must be 'direct' or 'chain'")
        C = load()
        self.seq = seq_per_rank
        self.heads = heads
        self.heads_kv = heads if heads_kv is None else heads_kv
        self.head_dim = head_dim
        self.dtype = dtype
        self.causal = causal
        self.zigzag = causal if zigzag is None else zigzag
        prec = _DTYPES[dtype]
        self._own_runtime = runtime is None
        if runtime is None:
            from ..parallel.dist import detect_ranks

            world = detect_ranks().world
            runtime = RingRuntime(C.FusedRing.arena_bytes(prec, seq_per_rank, self.heads_kv,
                                                          head_dim, world))
        self.runtime = runtime
        self.engine = C.FusedRing(runtime.ctx, prec, seq_per_rank, heads, self.heads_kv, head_dim,
                                  causal, self.zigzag, ring_mode == "chain", timeout_s,
                                  graph_safe)
        self.graph_safe = graph_safe
        # the per-call checks compare against these (built once: a call's host
        # path is on the critical path of a step that starts from an idle GPU)
        self._dev = torch.device("cuda", runtime.device)
        self._shape_q = torch.Size((seq_per_rank, heads, head_dim))
        self._shape_kv = torch.Size((seq_per_rank, self.heads_kv, head_dim))
        self._default_scale = head_dim ** -0.5

    @property
    def rank(self) -> int:
        return self.runtime.rank

    @property
    def world(self) -> int:
        return self.runtime.world

    def _check_inputs(self, q, k, v, out=None):
        dev, dt = self._dev, self.dtype
        for name, t, shape in (("q", q, self._shape_q), ("k", k, self._shape_kv),
                               ("v", v, self._shape_kv)):
            if t.shape != shape or t.dtype != dt or t.device != dev:
                raise ValueError(f"{name}: expected {dt} tensor of shape {tuple(shape)} on {dev}, "
                                 f"got {t.dtype} {tuple(t.shape)} on {t.device}")
        if out is not None and (out.shape != self._shape_q or out.device != dev
                                or out.dtype not in (torch.float32, torch.bfloat16)
                                or not out.is_contiguous()):
            raise ValueError(f"out: expected a contiguous float32/bfloat16 tensor of shape "
                             f"{tuple(self._shape_q)} on {dev}, got {out.dtype} {tuple(out.shape)} "
                             f"on {out.device}")

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 scale: Optional[float] = None, return_lse: bool = False,
                 out: Optional[torch.Tensor] = None, check: bool = False):
        """Attention of this rank's queries over the whole ring; stream-ordered.

        With ``check=True`` the call synchronises and raises if a bounded
        device-side wait ran out (e.g. a peer rank never arrived).
        """
        self._check_inputs(q, k, v, out)
        if scale is None:
            scale = self._default_scale
        if out is None:
            out = torch.empty_like(q)
        lse = (torch.empty(self.seq, self.heads, dtype=torch.float32, device=q.device)
               if return_lse else None)
        self.engine.forward(q.contiguous(), k.contiguous(), v.contiguous(), out, lse, float(scale))
        if check:
            self.engine.check()
        return (out, lse) if return_lse else out

    forward = __call__

    def __enter__(self) -> "RingAttention":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def check(self) -> None:
        self.engine.check()

    def overlap_trace(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      out: Optional[torch.Tensor] = None) -> dict:
        """One call with the kernel's overlap trace on (per CTA: when each ring
        block was first waited for and when it was present); returns the
        summary of `utils.overlap.summarize`.  Synchronises; every rank of the
        job must call it together, like any other call."""
        from ..utils.overlap import summarize

        self.engine.set_trace(True)
        try:
            self(q, k, v, out=out, check=True)
            torch.cuda.synchronize(q.device)
            stamps = self.engine.read_trace()
        finally:
            self.engine.set_trace(False)
        return summarize(stamps, self.world)

    def capture(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                out: Optional[torch.Tensor] = None, scale: Optional[float] = None):
        """Capture one call into a CUDA graph and return ``(graph, out)``:
        ``graph.replay()`` reruns the whole ring call on the same ``q``, ``k``,
        ``v`` (refill them in place between replays) into ``out``.  Needs
        ``graph_safe=True`` when the ring has more than one rank; every rank
        captures together and replays in step.  Runs one eager call first (it
        loads the kernels and sets their attributes outside the capture)."""
        if self.world > 1 and not self.graph_safe:
            raise RuntimeError("capture() with more than one rank needs "
                               "RingAttention(..., graph_safe=True)")
        if out is None:
            out = torch.empty_like(q)
        self(q, k, v, scale=scale, out=out, check=True)  # eager warm-up call
        torch.cuda.synchronize(q.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self(q, k, v, scale=scale, out=out)
        return graph, out

    def close(self) -> None:
        self.engine = None
        if self._own_runtime and self.runtime is not None:
            self.runtime.close()
            self.runtime = None
