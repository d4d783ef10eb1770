"""The allocation-free C entry point `rab_flash_attention_noalloc` (for callers
that may not allocate device memory where they run attention, e.g. a plugin
inside another runtime's execute callback with a fixed memory budget).

Called through its exported C symbols with ctypes:
* two calls in a row with different inputs (so a call that read the previous
  call's leftovers in the shared scratch array would show up), each checked
  against the float64 oracle and against the regular entry point
  (`flash_attention`, whose split workspace comes from the caller's
  allocator), non-causal and causal, with and without a KV split;
* the status word of every call is read back through
  `rab_flash_attention_noalloc_status` and must be clean;
* free device memory is the same before and after the second call (the first
  call may load kernels lazily);
* a bounded device-side wait that runs out surfaces as RAB_NOALLOC_ERR_DEVICE
  through the status call, and the next attention call is clean again;
* an oversized problem is refused with a clear message.
This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

from ring_attention_benchmark_b200 import _ext
from ring_attention_benchmark_b200.models import oracle
from ring_attention_benchmark_b200.ops import attention as A

pytestmark = pytest.mark.gpu

HQ, HKV, D = 4, 2, 128
TOO_LARGE, DEVICE_ERROR = -2, -4
TOL = 2e-2  # bf16 output


def _lib():
    lib = ctypes.CDLL(_ext.load().__file__)
    fn = lib.rab_flash_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_void_p] + [ctypes.c_int] * 5 + [
        ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p,
        ctypes.c_size_t]
    st = lib.rab_flash_attention_noalloc_status
    st.restype = ctypes.c_int
    st.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint), ctypes.c_char_p,
                   ctypes.c_size_t]
    wt = lib.rab_flash_attention_noalloc_wait_selftest
    wt.restype = ctypes.c_int
    wt.argtypes = [ctypes.c_double, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    return fn, st, wt


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _call(fn, q, k, v, out, lse, nsplit, causal, sq, skv, hq=HQ, hkv=HKV, d=D):
    err = ctypes.create_string_buffer(512)
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
            lse.data_ptr() if lse is not None else None, sq, skv, hq, hkv, d, d ** -0.5,
            int(causal), nsplit, _stream(), err, len(err))
    return rc, err.value.decode()


def _status(st):
    err = ctypes.create_string_buffer(512)
    info = (ctypes.c_uint * 4)()
    rc = st(_stream(), info, err, len(err))
    return rc, list(info), err.value.decode()


@pytest.mark.parametrize("causal,sq,skv,nsplit", [
    (False, 512, 4096, 4), (False, 512, 4096, 0), (True, 1024, 1024, 1), (True, 1024, 1024, 4)])
def test_noalloc_matches_oracle_and_regular_entry_point(cuda_device, causal, sq, skv, nsplit):
    fn, st, _ = _lib()
    g = torch.Generator(device="cpu").manual_seed(7 + nsplit + 100 * int(causal))
    pos = torch.arange(sq) if causal else None
    free_before = None
    for call in range(2):  # two calls in a row share the scratch array
        q = torch.randn(sq, HQ, D, generator=g).to(cuda_device, torch.bfloat16)
        k = torch.randn(skv, HKV, D, generator=g).to(cuda_device, torch.bfloat16)
        v = torch.randn(skv, HKV, D, generator=g).to(cuda_device, torch.bfloat16)
        out = torch.full((sq, HQ, D), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        lse = torch.full((sq, HQ), float("nan"), device=cuda_device)
        torch.cuda.synchronize()
        if call == 1:
            free_before = torch.cuda.mem_get_info(cuda_device)[0]
        rc, msg = _call(fn, q, k, v, out, lse, nsplit, causal, sq, skv)
        assert rc == 0, msg
        rc, info, msg = _status(st)  # waits for the stream
        assert rc == 0 and info[0] == 0, (msg, info)
        if call == 1:
            assert torch.cuda.mem_get_info(cuda_device)[0] == free_before, \
                "free device memory changed across an allocation-free call"
        qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
        ref = oracle.full_attention(qc, kc, vc, D ** -0.5, pos, pos)
        assert torch.isfinite(out.float()).all(), f"call {call}"
        err = (out.cpu().double() - ref).abs().max().item()
        assert err < TOL, f"call {call}: max abs err vs float64 oracle {err}"
        # natural-log LSE against the oracle's
        s = oracle._mask(oracle.scores(qc, kc, D ** -0.5), pos, pos)
        ref_lse = torch.logsumexp(s, dim=-1).transpose(0, 1)
        assert (lse.cpu().double() - ref_lse).abs().max().item() < TOL, f"call {call}"
        regular = A.flash_attention(q, [k], [v], causal=causal, nsplit=nsplit or 0)
        torch.cuda.synchronize()
        assert (out.float() - regular.float()).abs().max().item() < TOL, f"call {call}"


def test_noalloc_device_timeout_surfaces_through_status(cuda_device):
    fn, st, wt = _lib()
    err = ctypes.create_string_buffer(512)
    assert wt(0.05, _stream(), err, len(err)) == 0, err.value.decode()
    rc, info, msg = _status(st)
    assert rc == DEVICE_ERROR, (rc, msg)
    assert info[0] == 1 and A.WAIT_SITES[info[1]] == "test", info
    assert "timed out" in msg
    # the context and the entry point keep working, and the next call starts clean
    sq, skv = 256, 1024
    q = torch.randn(sq, HQ, D, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(skv, HKV, D, device=cuda_device).to(torch.bfloat16)
    v = torch.randn(skv, HKV, D, device=cuda_device).to(torch.bfloat16)
    out = torch.empty_like(q)
    rc, msg = _call(fn, q, k, v, out, None, 0, False, sq, skv)
    assert rc == 0, msg
    rc, info, msg = _status(st)
    assert rc == 0 and info[0] == 0, (msg, info)
    ref = oracle.full_attention(q.cpu(), k.cpu(), v.cpu(), D ** -0.5)
    assert (out.cpu().double() - ref).abs().max().item() < TOL


def test_noalloc_rejects_oversized_problem(cuda_device):
    fn, _, _ = _lib()
    sq, skv, hq = 16384, 16384, 32
    q = torch.empty(1, device=cuda_device, dtype=torch.bfloat16)  # never touched
    rc, msg = _call(fn, q, q, q, q, None, 8, False, sq, skv, hq=hq, hkv=hq, d=128)
    assert rc == TOO_LARGE
    assert "static scratch array holds" in msg
