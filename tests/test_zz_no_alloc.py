"""The allocation-free C entry point `rab_flash_attention_noalloc` (for callers
that may not allocate device memory where they run attention, e.g. a plugin
inside another runtime's execute callback with a fixed memory budget).

Called through its exported C symbol with ctypes and compared with the regular
entry point (`flash_attention`, whose split workspace comes from the caller's
allocator) on two calls in a row with different inputs, so a call that read
the previous call's leftovers in the shared scratch array would show up.  Also
checks that an oversized problem is refused with a clear message.  This file
is collected last on purpose.
"""
import ctypes

import pytest
import torch

from ring_attention_benchmark_b200 import _ext
from ring_attention_benchmark_b200.ops import attention as A

pytestmark = pytest.mark.gpu

SQ, SKV, HQ, HKV, D = 512, 4096, 4, 2, 128
TOO_LARGE = -2


def _entry():
    lib = ctypes.CDLL(_ext.load().__file__)
    fn = lib.rab_flash_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_void_p] + [ctypes.c_int] * 5 + [
        ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p,
        ctypes.c_size_t]
    return fn


def _call(fn, q, k, v, out, lse, nsplit, sq=SQ, skv=SKV, hq=HQ, hkv=HKV, d=D):
    err = ctypes.create_string_buffer(512)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
            lse.data_ptr() if lse is not None else None, sq, skv, hq, hkv, d, d ** -0.5, 0,
            nsplit, stream, err, len(err))
    return rc, err.value.decode()


@pytest.mark.parametrize("nsplit", [4, 0])
def test_noalloc_matches_regular_entry_point(cuda_device, nsplit):
    fn = _entry()
    g = torch.Generator(device="cpu").manual_seed(7 + nsplit)
    for call in range(2):  # two calls in a row share the scratch array
        q = torch.randn(SQ, HQ, D, generator=g).to(cuda_device, torch.bfloat16)
        k = torch.randn(SKV, HKV, D, generator=g).to(cuda_device, torch.bfloat16)
        v = torch.randn(SKV, HKV, D, generator=g).to(cuda_device, torch.bfloat16)
        out = torch.full((SQ, HQ, D), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        lse = torch.full((SQ, HQ), float("nan"), device=cuda_device)
        rc, msg = _call(fn, q, k, v, out, lse, nsplit)
        assert rc == 0, msg
        ref, ref_lse = A.flash_attention(q, [k], [v], nsplit=nsplit or 0, return_lse=True)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all(), f"call {call}"
        assert (out.float() - ref.float()).abs().max().item() < 2e-2, f"call {call}"
        assert (lse - ref_lse).abs().max().item() < 2e-2, f"call {call}"


def test_noalloc_rejects_oversized_problem(cuda_device):
    fn = _entry()
    sq, skv, hq = 16384, 16384, 32
    q = torch.empty(1, device=cuda_device, dtype=torch.bfloat16)  # never touched
    rc, msg = _call(fn, q, q, q, q, None, 8, sq=sq, skv=skv, hq=hq, hkv=hq, d=128)
    assert rc == TOO_LARGE
    assert "static scratch array holds" in msg
