"""Rank discovery, device selection and bootstrap of the native ring runtime.

Rank / size / local rank come from the launcher's environment, in the order
torchrun, Open MPI, MVAPICH, Slurm, PMI, PALS (the reference reads the same
local-rank variables, ``src/common/device_utils.cuh`` lines 9-28).  The device is
``local_rank % device_count``; more ranks than devices is an error unless
``ALLOW_GPU_OVERSUBSCRIBE`` is set (reference lines 60-66).

Bootstrap: a gloo process group (host only) exchanges the shared-memory segment
name, the CUDA IPC handle of every rank's device arena, the device UUIDs and the
NCCL unique id.  After that the native runtime needs no Python: barriers,
reductions, host transfers and flag words go through the shared-memory segment,
device transfers through the peer-mapped arenas or NCCL.
"""
from __future__ import annotations

import datetime
import os
import uuid
from dataclasses import dataclass
from typing import Optional

import torch

from .._ext import load

_RANK_VARS = ("RANK", "OMPI_COMM_WORLD_RANK", "PMIX_RANK", "PMI_RANK", "MV2_COMM_WORLD_RANK",
              "SLURM_PROCID")
_SIZE_VARS = ("WORLD_SIZE", "OMPI_COMM_WORLD_SIZE", "PMIX_SIZE", "PMI_SIZE", "MV2_COMM_WORLD_SIZE",
              "SLURM_NTASKS")
_LOCAL_VARS = ("LOCAL_RANK", "OMPI_COMM_WORLD_LOCAL_RANK", "MV2_COMM_WORLD_LOCAL_RANK",
               "SLURM_LOCALID", "MPI_LOCALRANKID", "PMI_LOCAL_RANK", "PALS_LOCAL_RANK")


def _first_int(names, default=None):
    for n in names:
        v = os.environ.get(n)
        if v not in (None, ""):
            return int(v)
    return default


@dataclass
class RankInfo:
    rank: int
    world: int
    local_rank: int


def detect_ranks() -> RankInfo:
    rank = _first_int(_RANK_VARS, 0)
    world = _first_int(_SIZE_VARS, 1)
    local = _first_int(_LOCAL_VARS, rank)
    return RankInfo(rank, world, local)


def select_device(local_rank: int) -> int:
    n = torch.cuda.device_count()
    if n <= 0:
        raise RuntimeError("No CUDA devices found.")
    if local_rank >= n and not os.environ.get("ALLOW_GPU_OVERSUBSCRIBE"):
        raise RuntimeError(
            f"local_rank {local_rank}: only {n} CUDA device(s) are visible. "
            "Reduce ranks per node or set ALLOW_GPU_OVERSUBSCRIBE=1.")
    dev = local_rank % n
    torch.cuda.set_device(dev)
    return dev


def _pg_timeout() -> datetime.timedelta:
    return datetime.timedelta(seconds=float(os.environ.get("RAB_PG_TIMEOUT_S", "120")))


def init_process_group_if_needed(info: RankInfo):
    import torch.distributed as dist

    if info.world <= 1:
        return None
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29517")
        dist.init_process_group("gloo", rank=info.rank, world_size=info.world,
                                timeout=_pg_timeout())
    return dist


def _all_gather(dist, obj):
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


class RingRuntime:
    """One rank's view of the ring: native RingContext plus bootstrap state."""

    def __init__(self, arena_bytes: int, need_nccl: bool = False, frag_bytes: int = 1 << 20,
                 timeout_s: Optional[float] = None, info: Optional[RankInfo] = None):
        C = load()
        self.info = info or detect_ranks()
        self.device = select_device(self.info.local_rank)
        self.timeout_s = float(timeout_s if timeout_s is not None
                               else os.environ.get("RAB_TIMEOUT_S", "60"))
        self.dist = init_process_group_if_needed(self.info)
        rank, world = self.info.rank, self.info.world
        name = f"/rab_{os.getpid()}_{uuid.uuid4().hex[:12]}"
        if self.dist is not None:
            name = _all_gather(self.dist, name)[0]
        if rank == 0:
            self.ctx = C.RingContext(rank, world, self.device, name, True, frag_bytes,
                                     int(arena_bytes), self.timeout_s)
        if self.dist is not None:
            self.dist.barrier()
        if rank != 0:
            self.ctx = C.RingContext(rank, world, self.device, name, False, frag_bytes,
                                     int(arena_bytes), self.timeout_s)
        self.devices_unique = True
        if self.dist is not None:
            uuids = _all_gather(self.dist, str(torch.cuda.get_device_properties(self.device).uuid))
            self.devices_unique = len(set(uuids)) == len(uuids)
            self.ctx.set_devices_unique(self.devices_unique)
            handles = _all_gather(self.dist, self.ctx.ipc_handle())
            self.ctx.open_peers(handles)
            if need_nccl:
                uid = C.RingContext.nccl_unique_id() if rank == 0 else None
                uid = _all_gather(self.dist, uid)[0]
                self.ctx.init_nccl(uid)
        elif need_nccl:
            self.ctx.init_nccl(C.RingContext.nccl_unique_id())
        self.ctx.barrier()
        if rank == 0:
            self.ctx.unlink_shm()  # the mapping stays; nothing is left in /dev/shm

    @property
    def rank(self) -> int:
        return self.info.rank

    @property
    def world(self) -> int:
        return self.info.world

    def barrier(self):
        self.ctx.barrier()

    def reduce_max(self, vals):
        return self.ctx.reduce_max(list(vals))

    def close(self):
        ctx = getattr(self, "ctx", None)
        if ctx is not None:
            torch.cuda.synchronize(self.device)
            ctx.barrier()
            del self.ctx
        if self.dist is not None and self.dist.is_initialized():
            self.dist.destroy_process_group()
            self.dist = None
