"""Public RingAttention API on one GPU: results against the oracle, caller-owned
outputs, and the input/output checks of the Python layer and of the native
binding (bad shapes and dtypes are refused before anything is launched)."""
import pytest
import torch

from ring_attention_benchmark_b200 import RingAttention
from ring_attention_benchmark_b200.models import inputs, oracle

pytestmark = pytest.mark.gpu


def test_single_rank_api_and_io_checks(cuda_device):
    x = inputs.normal_inputs(0, 256, 2, 64)
    ref = oracle.full_attention(x.q, x.k, x.v, x.scale)
    q, k, v = x.q.to(cuda_device), x.k.to(cuda_device), x.v.to(cuda_device)
    with RingAttention(256, heads=2, head_dim=64, dtype=torch.float32) as attn:
        out, lse = attn(q, k, v, return_lse=True, check=True)
        torch.cuda.synchronize()
        assert (out.cpu().double() - ref).abs().max().item() < 1e-4
        assert lse.shape == (256, 2) and bool(torch.isfinite(lse).all())
        # a caller-owned bf16 output from the fp32 engine
        o16 = torch.empty(256, 2, 64, dtype=torch.bfloat16, device=cuda_device)
        attn(q, k, v, out=o16, check=True)
        torch.cuda.synchronize()
        assert (o16.float().cpu().double() - ref).abs().max().item() < 2e-2
        # Python-layer checks
        with pytest.raises(ValueError, match="out"):
            attn(q, k, v, out=torch.empty(128, 2, 64, device=cuda_device))
        with pytest.raises(ValueError, match="k:"):
            attn(q, k[:128], v)
        with pytest.raises(ValueError, match="q:"):
            attn(q.cpu(), k, v)
        # native binding checks (called directly, past the Python layer)
        with pytest.raises(RuntimeError, match="elements"):
            attn.engine.forward(q, k, v, torch.empty(10, device=cuda_device), None, 0.125)
        with pytest.raises(RuntimeError, match="dtype"):
            attn.engine.forward(q.bfloat16(), k, v, torch.empty_like(q), None, 0.125)
        with pytest.raises(RuntimeError, match="lse"):
            attn.engine.forward(q, k, v, torch.empty_like(q),
                                torch.empty(3, device=cuda_device), 0.125)
        # still usable after the refused calls
        out2 = attn(q, k, v, check=True)
        torch.cuda.synchronize()
        assert torch.equal(out2, out)
    assert attn.engine is None and attn.runtime is None


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_capture_and_replay_one_rank(cuda_device, dtype):
    """A call captured into a CUDA graph replays the whole ring call: refill the
    captured inputs in place, replay, and the output matches an eager call on
    the same inputs (bit for bit: same kernels, same schedule)."""
    d = 64 if dtype == torch.float32 else 128  # the fp32 (3xTF32) path is d=64
    shape = (512, 4, d)
    with RingAttention(512, heads=4, head_dim=d, dtype=dtype, causal=True,
                       graph_safe=True) as attn:
        g = torch.Generator(device="cpu").manual_seed(3)
        q, k, v = (torch.randn(shape, generator=g).to(cuda_device, dtype) for _ in range(3))
        graph, out = attn.capture(q, k, v)
        for step in range(3):
            for t in (q, k, v):
                t.copy_(torch.randn(shape, generator=g).to(dtype))
            graph.replay()
            eager = attn(q, k, v, check=True)
            torch.cuda.synchronize()
            assert torch.equal(out, eager), step
            pos = torch.arange(512)
            ref = oracle.full_attention(q.cpu(), k.cpu(), v.cpu(), d ** -0.5, pos, pos)
            tol = 2e-5 if dtype == torch.float32 else 2e-2
            assert (out.cpu().double() - ref).abs().max().item() < tol, step
        attn.check()
