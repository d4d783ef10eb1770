"""B200-native ring attention benchmark framework.

Re-creates the capabilities of the ring-attention-benchmark suite (comm-only
ring rotation and full ring attention across ranks, one GPU per rank) on
NVIDIA B200: hand-written sm_100a kernels (tcgen05 / TMEM / TMA), a native C++
ring runtime (shared-memory control plane, CUDA IPC peer mapping, NCCL), and a
fused backend that moves K/V shards over NVLink from inside the attention
kernel.
"""

__version__ = "0.1.0"

from ._ext import available as extension_available  # noqa: F401


def __getattr__(name):
    # torch-dependent public classes load on first use
    if name == "RingAttention":
        from .models.ring_attention import RingAttention

        return RingAttention
    if name == "RingRuntime":
        from .parallel.dist import RingRuntime

        return RingRuntime
    raise AttributeError(name)
