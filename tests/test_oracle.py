"""CPU oracle: ring order + online-softmax merge equals full softmax attention
(world_size 2, seq 256, 1 head, d 64, N(0,1) seed 0, scale 1/sqrt(64)), and
zigzag causal sharding equals the unsharded causal attention."""
import torch

from ring_attention_benchmark_b200.models import inputs, oracle


def test_ring_equals_full_world2():
    world, seq, d = 2, 256, 64
    g = torch.Generator().manual_seed(0)
    q = [torch.randn(seq, 1, d, generator=g) for _ in range(world)]
    k = [torch.randn(seq, 1, d, generator=g) for _ in range(world)]
    v = [torch.randn(seq, 1, d, generator=g) for _ in range(world)]
    scale = d ** -0.5
    outs = oracle.ring_attention(q, k, v, scale)
    full = oracle.full_attention(torch.cat(q), torch.cat(k), torch.cat(v), scale)
    assert torch.allclose(torch.cat(outs), full, atol=1e-12, rtol=1e-10)


def test_block_order():
    assert oracle.ring_block_order(0, 4) == [0, 3, 2, 1]
    assert oracle.ring_block_order(2, 4) == [2, 1, 0, 3]


def test_zigzag_causal_gqa():
    world, spr, h, hk, d = 4, 32, 4, 2, 16
    g = torch.Generator().manual_seed(3)
    total = world * spr
    q = torch.randn(total, h, d, generator=g)
    k = torch.randn(total, hk, d, generator=g)
    v = torch.randn(total, hk, d, generator=g)
    pos = torch.arange(total)
    full = oracle.full_attention(q, k, v, 0.25, pos, pos)
    qs = [oracle.zigzag_shard(q, r, world) for r in range(world)]
    ks = [oracle.zigzag_shard(k, r, world) for r in range(world)]
    vs = [oracle.zigzag_shard(v, r, world) for r in range(world)]
    ps = [oracle.zigzag_positions(r, world, spr) for r in range(world)]
    outs = oracle.ring_attention(qs, ks, vs, 0.25, ps)
    assert torch.allclose(oracle.zigzag_unshard(outs), full, atol=1e-12)


def test_ref_compat_inputs_shape_and_values():
    x = inputs.ref_compat_inputs(1, 1024)
    assert x.q.shape == (1024, 1, 64) and x.k is x.v
    assert x.k[0, 0, 0].item() == 1000.0 and x.k[1, 0, 0].item() == 1064.0
    assert abs(x.q[5, 0, 3].item() - (500 + 3 * 0.01) * 0.001) < 1e-7
    assert inputs.size_to_seq(262144) == 1024
