"""CUDA-core kernels vs the float64 oracle: exact-order fp32 partial attention,
online-softmax merge, normalisation, casts and the tf32 split."""
import pytest
import torch

from ring_attention_benchmark_b200.models import inputs, oracle

pytestmark = pytest.mark.gpu


def _partial(ext, dev, q, k, v, scale, causal_offset=-1, normalize=False):
    sq, h, d = q.shape
    acc = torch.empty(sq, h, d, device=dev)
    m = torch.empty(sq, h, device=dev)
    l = torch.empty(sq, h, device=dev)
    ext.simt_partial_attention(q.to(dev), k.to(dev), v.to(dev), acc, m, l, scale,
                               causal_offset, normalize)
    torch.cuda.synchronize()
    return acc.cpu(), m.cpu(), l.cpu()


@pytest.mark.parametrize("seq,heads,hk,d", [(256, 1, 1, 64), (300, 4, 2, 64), (128, 2, 2, 128)])
def test_simt_partial_normal(ext, cuda_device, seq, heads, hk, d):
    x = inputs.normal_inputs(0, seq, heads, d, heads_kv=hk)
    acc, m, l = _partial(ext, cuda_device, x.q, x.k, x.v, x.scale)
    racc, rm, rl = oracle.partial_attention(x.q, x.k, x.v, x.scale)
    assert torch.allclose(m.double(), rm, rtol=1e-5, atol=1e-5)
    assert torch.allclose(l.double(), rl, rtol=1e-4, atol=1e-4)
    assert torch.allclose(acc.double(), racc, rtol=1e-4, atol=1e-4)


def test_simt_causal(ext, cuda_device):
    x = inputs.normal_inputs(1, 192, 2, 64)
    acc, m, l = _partial(ext, cuda_device, x.q, x.k, x.v, x.scale, causal_offset=0, normalize=True)
    pos = torch.arange(192)
    ref = oracle.full_attention(x.q, x.k, x.v, x.scale, pos, pos)
    assert torch.allclose(acc.double(), ref, rtol=1e-4, atol=1e-5)


def test_simt_ref_compat_matches_fp32_sequential(ext, cuda_device):
    # the reference data: scores ~1e7, neighbouring keys 1.3 apart
    seq = 256
    q = inputs.ref_compat_q(1, seq)
    kv = inputs.ref_compat_kv(0, seq)
    acc, m, l = _partial(ext, cuda_device, q, kv, kv, 1.0)
    # CPU fp32 statement with the same fma order (torch.addcmul keeps fp32)
    q0 = q[0, 0]
    s = torch.zeros(seq, dtype=torch.float32)
    for d in range(64):
        s = torch.addcmul(s, kv[:, 0, d], q0[d].expand(seq))
    assert torch.allclose(m[:, 0], s.max().expand(seq), rtol=2e-7, atol=0)
    out = acc / l.unsqueeze(-1)
    ref = oracle.normalize(oracle.partial_attention(q, kv, kv, 1.0))
    rel = ((out.double() - ref).abs() / ref.abs().clamp_min(1e-12)).max().item()
    assert rel < 1e-5


def test_merge_and_normalize(ext, cuda_device):
    dev = cuda_device
    seq, h, d = 200, 3, 64
    a = inputs.normal_inputs(0, seq, h, d)
    b = inputs.normal_inputs(1, seq, h, d)
    st1 = oracle.partial_attention(a.q, a.k, a.v, a.scale)
    st2 = oracle.partial_attention(a.q, b.k, b.v, a.scale)
    acc = st1[0].float().to(dev).contiguous()
    m = st1[1].float().to(dev).contiguous()
    l = st1[2].float().to(dev).contiguous()
    ext.merge_lse(m, l, acc, st2[1].float().to(dev).contiguous(),
                  st2[2].float().to(dev).contiguous(), st2[0].float().to(dev).contiguous())
    out = torch.empty(seq, h, d, device=dev)
    lse = torch.empty(seq, h, device=dev)
    ext.normalize(acc, m, l, out, lse)
    out_bf = torch.empty(seq, h, d, device=dev, dtype=torch.bfloat16)
    ext.normalize(acc, m, l, out_bf, None)
    torch.cuda.synchronize()
    ref_state = oracle.merge_online_softmax(st1, st2)
    ref = oracle.normalize(ref_state)
    assert torch.allclose(out.cpu().double(), ref, rtol=1e-5, atol=1e-6)
    assert torch.allclose(lse.cpu().double(), oracle.lse(ref_state), rtol=1e-5, atol=1e-5)
    assert torch.allclose(out_bf.cpu().double(), ref, rtol=1e-2, atol=1e-2)


def test_cast_and_split(ext, cuda_device):
    x = torch.randn(4096, device=cuda_device) * 3
    bf = torch.empty(4096, device=cuda_device, dtype=torch.bfloat16)
    ext.cast(x, bf)
    back = torch.empty(4096, device=cuda_device)
    ext.cast(bf, back)
    assert torch.equal(bf, x.to(torch.bfloat16))
    assert torch.equal(back, bf.float())
    big = torch.empty_like(x)
    small = torch.empty_like(x)
    ext.split_tf32(x, big, small)
    torch.cuda.synchronize()
    assert ((big.view(torch.int32) & 0x1FFF) == 0).all()
    assert ((small.view(torch.int32) & 0x1FFF) == 0).all()
    err = ((big.double() + small.double()) - x.double()).abs() / x.double().abs().clamp_min(1e-30)
    assert err.max().item() < 2 ** -21
