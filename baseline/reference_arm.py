#!/usr/bin/env python3
"""The reference arm of ``bench.py``: the UNMODIFIED reference programs, built
with their own Makefile and run one process per GPU.

    python baseline/reference_arm.py install      # copy + build into baseline/_ref
    python baseline/reference_arm.py mpirun -np N PROGRAM [ARGS...]

The reference (``3429495086/ring-attention-benchmark``) is a set of MPI
programs; no MPI is installed on the machines this framework targets, so the
programs are linked against ``baseline/minimpi`` (an implementation of the MPI
subset they call: shared-memory channels for host buffers, CUDA IPC for
device buffers, as an intra-node CUDA-aware MPI moves them).  NCCL is the copy
that ships with torch.  The sources are copied verbatim into
``baseline/_ref/reference`` and built there with the reference's own Makefile
(``make all``) with ``MPI_HOME`` and ``NCCL_HOME`` pointed at those libraries
and ``NVCCFLAGS="-O3 -gencode arch=compute_100a,code=sm_100a"``; nothing of
this framework's kernels or engine is on that path.

`run_attention` runs one reference attention program as rank RANK of
WORLD_SIZE (the torchrun environment), with a job name shared through a gloo
broadcast, and returns rank 0's two summary lines.  A world of one rank runs
the program too: the reference rejects it itself.
"""
from __future__ import annotations

import os
import re
import shutil
import subprocess
import sys
import uuid
from typing import Dict, List, Optional, Tuple

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
REF_SRC_DIR = os.path.join(REF_DIR, "reference")
MINIMPI_SRC = os.path.join(HERE, "minimpi")
MINIMPI_DIR = os.path.join(REF_DIR, "minimpi")
ORIGINAL_SOURCE = "/root/reference"  # read only by `install`
NVCCFLAGS = "-O3 -gencode arch=compute_100a,code=sm_100a"


def cuda_home() -> str:
    return os.environ.get("CUDA_HOME") or "/usr/local/cuda"


def nccl_home() -> str:
    import nvidia.nccl  # the NCCL that ships with torch

    base = (os.path.dirname(nvidia.nccl.__file__) if nvidia.nccl.__file__
            else list(nvidia.nccl.__path__)[0])
    return base


def build_minimpi(dest: str = MINIMPI_DIR) -> str:
    """Build libmpi.so (+ mpi.h) into dest/{lib,include}; returns dest."""
    os.makedirs(os.path.join(dest, "lib"), exist_ok=True)
    os.makedirs(os.path.join(dest, "include"), exist_ok=True)
    shutil.copy2(os.path.join(MINIMPI_SRC, "mpi.h"), os.path.join(dest, "include", "mpi.h"))
    out = os.path.join(dest, "lib", "libmpi.so")
    subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-Wall",
                    f"-I{os.path.join(cuda_home(), 'include')}",
                    os.path.join(MINIMPI_SRC, "minimpi.cpp"), "-o", out, "-ldl"], check=True)
    return dest


def runtime_env(env: Optional[Dict[str, str]] = None) -> Dict[str, str]:
    env = dict(os.environ if env is None else env)
    libs = [os.path.join(MINIMPI_DIR, "lib"), os.path.join(nccl_home(), "lib")]
    old = env.get("LD_LIBRARY_PATH", "")
    env["LD_LIBRARY_PATH"] = ":".join(libs + ([old] if old else []))
    return env


def install(source: str = ORIGINAL_SOURCE, jobs: int = 8) -> List[str]:
    """Copy the reference verbatim and build every program; returns the built paths."""
    if not os.path.isdir(REF_SRC_DIR):
        if not os.path.isdir(source):
            raise FileNotFoundError(f"reference sources not found at {source}")
        shutil.copytree(source, REF_SRC_DIR)
    build_minimpi()
    cmd = ["make", "-C", REF_SRC_DIR, f"-j{jobs}", "CONFIG=/dev/null",
           f"MPI_HOME={MINIMPI_DIR}", f"NCCL_HOME={nccl_home()}",
           f"NVCC={os.path.join(cuda_home(), 'bin', 'nvcc')}", f"NVCCFLAGS={NVCCFLAGS}", "all"]
    subprocess.run(cmd, check=True)
    bindir = os.path.join(REF_SRC_DIR, "bin")
    return sorted(os.path.join(bindir, f) for f in os.listdir(bindir))


def program(name: str) -> str:
    return os.path.join(REF_SRC_DIR, "bin", name)


def rank_env(rank: int, world: int, local_rank: int, job: str,
             env: Optional[Dict[str, str]] = None) -> Dict[str, str]:
    """Launcher variables the reference (and minimpi) read: Open MPI's names."""
    e = runtime_env(env)
    e.update({"OMPI_COMM_WORLD_RANK": str(rank), "OMPI_COMM_WORLD_SIZE": str(world),
              "OMPI_COMM_WORLD_LOCAL_RANK": str(local_rank), "MINIMPI_JOB": job})
    return e


def mpirun(np_: int, argv: List[str], timeout: Optional[float] = None) -> int:
    """Start np_ ranks of argv on this node; the first non-zero exit code wins."""
    job = uuid.uuid4().hex[:16]
    procs = [subprocess.Popen(argv, env=rank_env(r, np_, r, job)) for r in range(np_)]
    rc = 0
    for p in procs:
        try:
            code = p.wait(timeout=timeout)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            return 124
        rc = rc or code
    return rc


_AVG = re.compile(r"avg_total=([0-9.]+) ms")


def parse_avg_total_ms(text: str) -> Optional[float]:
    m = _AVG.search(text)
    return float(m.group(1)) if m else None


def run_attention(backend: str, kv_bytes: int, warmup: int, iters: int, workdir: str,
                  timeout: float = 1500.0) -> Tuple[int, str, str]:
    """Run bin/ring_attention_<backend>_gpu_bench as this torchrun rank.

    Every rank calls this; returns (exit code, stdout, stderr) of this rank's
    process.  The job name comes from rank 0 through a gloo broadcast, so no
    two runs share shared-memory names.
    """
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    job = uuid.uuid4().hex[:16]
    if world > 1:
        import torch.distributed as dist

        if not dist.is_initialized():
            import datetime

            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=timeout + 120))
        box = [job]
        dist.broadcast_object_list(box, src=0)
        job = box[0]
    exe = program(f"ring_attention_{backend}_gpu_bench")
    os.makedirs(workdir, exist_ok=True)
    try:
        p = subprocess.run([exe, str(kv_bytes), str(warmup), str(iters)], cwd=workdir,
                           env=rank_env(rank, world, local, job), capture_output=True,
                           text=True, timeout=timeout)
        rc, out, err = p.returncode, p.stdout, p.stderr
    except subprocess.TimeoutExpired as e:
        rc, out, err = 124, e.stdout or "", (e.stderr or "") + "\n(timed out)"
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    return rc, out, err


def main(argv: List[str]) -> int:
    if argv[:1] == ["install"]:
        for p in install():
            print(p)
        return 0
    if argv[:1] == ["mpirun"] and len(argv) >= 4 and argv[1] == "-np":
        return mpirun(int(argv[2]), argv[3:])
    print(__doc__.split("\n\n")[1], file=sys.stderr)
    return 2


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
