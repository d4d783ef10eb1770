"""The MPI subset library used to build and run the unmodified reference
programs (baseline/minimpi), on CPU with host buffers: a ring of Sendrecv
larger than the shared-memory channel, Isend/Irecv with Testall, Reduce /
Allreduce, Bcast, Comm_split_type; and MPI_Abort in one rank ending every
rank with its code (no rank waits forever)."""
import os
import subprocess
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "baseline"))
import reference_arm  # noqa: E402


@pytest.fixture(scope="module")
def selftest(tmp_path_factory):
    d = tmp_path_factory.mktemp("minimpi")
    mpi = reference_arm.build_minimpi(str(d / "minimpi"))
    exe = str(d / "selftest")
    subprocess.run(["gcc", "-O2", "-std=c11", os.path.join(ROOT, "tests", "data",
                                                           "minimpi_selftest.c"),
                    f"-I{mpi}/include", f"-L{mpi}/lib", "-lmpi", f"-Wl,-rpath,{mpi}/lib", "-o",
                    exe], check=True)
    return exe


def _run(exe, np_, *args, timeout=120):
    job = f"t{os.getpid()}_{np_}_{time.time_ns() % 10**9}"
    procs = []
    for r in range(np_):
        env = dict(os.environ, OMPI_COMM_WORLD_RANK=str(r), OMPI_COMM_WORLD_SIZE=str(np_),
                   MINIMPI_JOB=job, MINIMPI_TIMEOUT_S="60")
        procs.append(subprocess.Popen([exe, *args], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    res = [(p.wait(timeout=timeout), p.stdout.read(), p.stderr.read()) for p in procs]
    left = [f for f in os.listdir("/dev/shm") if f.startswith(f"mmpi_{job}")]
    assert not left, f"shared-memory segments left behind: {left}"
    return res


@pytest.mark.parametrize("np_", [1, 2, 3])
def test_minimpi_selftest(selftest, np_):
    res = _run(selftest, np_)
    for r, (rc, out, err) in enumerate(res):
        assert rc == 0, err
        assert out.strip() == f"ok {r}", (out, err)


def test_minimpi_abort_ends_every_rank(selftest):
    t0 = time.time()
    res = _run(selftest, 3, "abort")
    assert time.time() - t0 < 30
    assert [rc for rc, _, _ in res] == [7, 7, 7], [e for _, _, e in res]
    assert "MPI_Abort(7)" in res[2][2]
