"""One rank of the CPU-only host control-plane tests (no GPU): barrier,
max-reduction, fragment-mailbox ring exchange, failure detection."""
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from ring_attention_benchmark_b200 import _ext  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    name = sys.argv[1]
    case = sys.argv[2]
    C = _ext.load()
    frag = 64 * 1024
    if rank == 0:
        h = C.HostComm(name, rank, world, True, frag, 3.0)
    else:
        deadline = time.time() + 10
        while True:
            try:
                h = C.HostComm(name, rank, world, False, frag, 3.0)
                break
            except RuntimeError:
                if time.time() > deadline:
                    raise
                time.sleep(0.05)
    h.barrier()
    if rank == 0:
        h.unlink()
    if case == "ok":
        for it in range(3):
            mx = h.reduce_max([float(rank), float(-rank), float(it * world + rank)])
            assert mx == [world - 1.0, 0.0, float(it * world + world - 1)], mx
        for n in (4, 1000, frag, 5 * frag + 12, 3 * 1024 * 1024):
            send = (torch.arange(n, dtype=torch.int64) % 251 + rank * 7).to(torch.uint8)
            recv = torch.zeros(n, dtype=torch.uint8)
            h.ring_sendrecv(send, recv)
            left = (rank - 1) % world
            exp = (torch.arange(n, dtype=torch.int64) % 251 + left * 7).to(torch.uint8)
            assert torch.equal(recv, exp), f"rank {rank} n {n}"
        h.barrier()
        print(f"rank {rank} ok", flush=True)
    elif case == "dead_rank":
        # the last rank leaves between steps without joining the barrier
        if rank == world - 1:
            sys.exit(0)
        try:
            h.barrier()
        except C.RankFailure as e:
            msg = str(e)
            assert "missing ranks" in msg or "aborted" in msg, msg
            print(f"rank {rank} detected: {msg}", flush=True)
            sys.exit(0)
        raise SystemExit("barrier did not fail")
    elif case == "abort":
        if rank == 1:
            h.abort("injected failure on rank 1")
            sys.exit(0)
        try:
            h.barrier()
        except C.RankFailure as e:
            assert "injected failure" in str(e) or "missing" in str(e), str(e)
            print(f"rank {rank} saw abort: {e}", flush=True)
            sys.exit(0)
        raise SystemExit("barrier did not fail")
    elif case == "dropped_message":
        # rank 0 never sends: its right neighbour's receive must time out
        if rank == 0:
            time.sleep(5)
            sys.exit(0)
        try:
            send = torch.zeros(1000, dtype=torch.uint8)
            recv = torch.zeros(1000, dtype=torch.uint8)
            h.ring_sendrecv(send, recv)
        except C.RankFailure as e:
            print(f"rank {rank} timed out: {e}", flush=True)
            sys.exit(0)
        if rank != 1:  # ranks further along may still finish their exchange
            sys.exit(0)
        raise SystemExit("receive did not time out")


if __name__ == "__main__":
    main()
