"""Two ranks run fused ring-attention steps; rank 1 then leaves between steps
with nothing in flight.  Rank 0 must learn of it on the host (its next barrier
names the missing rank) and must not launch another fused kernel."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from ring_attention_benchmark_b200 import RingAttention, _ext  # noqa: E402


def main():
    attn = RingAttention(512, 1, 64, dtype=torch.float32, timeout_s=3.0)
    rt = attn.runtime
    dev = torch.device("cuda", rt.device)
    q = torch.randn(512, 1, 64, device=dev)
    for _ in range(2):
        attn(q, q, q, check=True)
    torch.cuda.synchronize(dev)
    rt.barrier()
    if rt.rank == 1:
        os._exit(0)  # leaves between steps, no kernel in flight
    try:
        rt.barrier()  # the host learns about the missing rank here
    except _ext.load().RankFailure as e:
        print(f"rank 0 detected: {e}", flush=True)
        os._exit(0)
    attn(q, q, q, check=True)  # not reached
    raise SystemExit("missing rank not detected")


if __name__ == "__main__":
    main()
