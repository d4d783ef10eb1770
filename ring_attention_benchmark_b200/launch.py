"""Local multi-process launcher (the `LAUNCHER=local` path of the scripts).

    python -m ring_attention_benchmark_b200.launch -np 4 [--timeout S] prog [args...]

Starts `np` copies of `prog` on this node with RANK / WORLD_SIZE / LOCAL_RANK /
LOCAL_WORLD_SIZE / MASTER_ADDR=127.0.0.1 / MASTER_PORT set, like mpirun or
torchrun would.  Watchdog: when one rank exits non-zero (or the optional
timeout passes) every other rank is terminated and the launcher returns that
rank's exit code, so a failed rank never leaves the others waiting.
"""
from __future__ import annotations

import argparse
import os
import signal
import socket
import subprocess
import sys
import time


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(np: int, cmd, timeout: float = 0.0, env=None) -> int:
    port = free_port()
    procs = []
    base = dict(os.environ if env is None else env)
    for r in range(np):
        e = dict(base)
        e.update(RANK=str(r), WORLD_SIZE=str(np), LOCAL_RANK=str(r), LOCAL_WORLD_SIZE=str(np),
                 MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        procs.append(subprocess.Popen(cmd, env=e, start_new_session=True))
    t0 = time.time()
    rc = 0
    try:
        while True:
            alive = False
            for r, p in enumerate(procs):
                code = p.poll()
                if code is None:
                    alive = True
                elif code != 0 and rc == 0:
                    rc = code
                    print(f"[launch] rank {r} exited with {code}; stopping the other ranks",
                          file=sys.stderr, flush=True)
            if rc != 0 or not alive:
                break
            if timeout > 0 and time.time() - t0 > timeout:
                print(f"[launch] timeout after {timeout:.0f} s; stopping all ranks",
                      file=sys.stderr, flush=True)
                rc = 124
                break
            time.sleep(0.05)
    finally:
        for p in procs:
            if p.poll() is None:
                try:
                    os.killpg(p.pid, signal.SIGTERM)
                except ProcessLookupError:
                    pass
        deadline = time.time() + 10
        for p in procs:
            while p.poll() is None and time.time() < deadline:
                time.sleep(0.05)
            if p.poll() is None:
                try:
                    os.killpg(p.pid, signal.SIGKILL)
                except ProcessLookupError:
                    pass
                p.wait()
    return rc


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("-np", "--np", type=int, required=True)
    ap.add_argument("--timeout", type=float, default=0.0)
    ap.add_argument("cmd", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cmd = a.cmd[1:] if a.cmd and a.cmd[0] == "--" else a.cmd
    if not cmd:
        ap.error("missing program")
    if os.path.exists(cmd[0]) and not os.access(cmd[0], os.X_OK):
        cmd = [sys.executable] + cmd
    return launch(a.np, cmd, a.timeout)


if __name__ == "__main__":
    sys.exit(main())
