"""Failure detection on the GPU without a GPU fault.

* A bounded device-side wait on a flag that nothing sets gives up after its
  limit, records the timeout in the status word and returns; the host reads the
  status and the same CUDA context keeps working.
* On 2 GPUs, a rank that leaves between ring steps (none of its kernels in
  flight) is detected on the host at the survivor's next barrier, before it
  launches another fused kernel.  NVLS is off in every library used.
"""
import os
import subprocess
import sys
import time

import pytest
import torch

from ring_attention_benchmark_b200.ops import attention as A

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def test_device_wait_times_out_and_context_survives(ext, cuda_device):
    flag = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    status = torch.zeros(8, dtype=torch.int32, device=cuda_device)
    t0 = time.time()
    ext.wait_selftest(flag, 1, 0.5, status)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    s = status.tolist()
    assert s[0] == 1 and A.WAIT_SITES[s[1]] == "test", s
    assert 0.4 < elapsed < 10
    with pytest.raises(A.DeviceTimeout):
        A.check_status(status, "selftest")
    # the context is still usable: a normal kernel runs and is correct
    x = torch.randn(1024, device=cuda_device)
    y = torch.empty(1024, device=cuda_device, dtype=torch.bfloat16)
    ext.cast(x, y)
    torch.cuda.synchronize()
    assert torch.equal(y, x.to(torch.bfloat16))
    # a wait whose flag is set returns without an error
    flag.fill_(5)
    status.zero_()
    ext.wait_selftest(flag, 3, 0.5, status)
    torch.cuda.synchronize()
    assert status[0].item() == 0


def test_rank_leaving_between_steps_is_detected():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", RAB_TIMEOUT_S="3")
    cmd = [sys.executable, "-m", "ring_attention_benchmark_b200.launch", "-np", "2",
           "--timeout", "120", sys.executable, os.path.join(ROOT, "tests", "_leave_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=180)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "rank 0 detected" in r.stdout, r.stdout
