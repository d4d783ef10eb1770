"""The bf16 d=128 flash kernel on CTA pairs (tcgen05 cta_group::2: each CTA of
a cluster of two loads half of every K/V tile, the leader issues M=256 MMAs
for both) against the float64 oracle: one block and ring blocks, GQA, KV
splits, causal with contiguous and zigzag sharding, dynamic claiming, the
reference's partial-output contract, and the fused ring path in loopback.
The kernel is selected with RAB_FLASH_2SM=1; each test checks that the
planner picked its 512-row units."""
import pytest
import torch

from ring_attention_benchmark_b200.models import inputs, oracle
from ring_attention_benchmark_b200.ops import attention as A

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def pair_kernel(monkeypatch):
    monkeypatch.setenv("RAB_FLASH_2SM", "1")


def _blocks(world, spr, h, hk, seed):
    g = torch.Generator().manual_seed(seed)
    mk = lambda n: [torch.randn(spr, n, 128, generator=g).to(torch.bfloat16)  # noqa: E731
                    for _ in range(world)]
    return mk(h), mk(hk), mk(hk)


def _positions(world, spr, causal, zigzag):
    if not causal:
        return None
    return [oracle.zigzag_positions(r, world, spr) if zigzag
            else torch.arange(r * spr, (r + 1) * spr) for r in range(world)]


def _check(ext, dev, world, spr, h, hk, causal=False, zigzag=False, nsplit=0, seed=0):
    qs, ks, vs = _blocks(world, spr, h, hk, seed)
    pos = _positions(world, spr, causal, zigzag)
    for rank in range(world):
        info = ext.flash_plan_info(A.PREC_BF16, spr, spr, world, h, hk, 128, causal=causal,
                                   zigzag=zigzag, world=world, rank=rank, nsplit=nsplit)
        assert info["rows_per_unit"] == 512, info
        order = oracle.ring_block_order(rank, world)
        out, lse = A.flash_attention(qs[rank].to(dev), [ks[s].to(dev) for s in order],
                                     [vs[s].to(dev) for s in order], causal=causal,
                                     zigzag=zigzag, world=world, rank=rank, nsplit=nsplit,
                                     return_lse=True)
        state = oracle.empty_state(spr, h, 128)
        for s in order:
            state = oracle.merge_online_softmax(state, oracle.partial_attention(
                qs[rank], ks[s], vs[s], 128 ** -0.5, pos[rank] if pos else None,
                pos[s] if pos else None))
        ref, rlse = oracle.normalize(state), oracle.lse(state)
        err = (out.float().cpu().double() - ref).abs().max().item()
        assert err < 2e-2, (rank, info, err)
        assert (lse.cpu().double() - rlse).abs().max().item() < 2e-2, (rank, info)


@pytest.mark.parametrize("nsplit", [1, 0])
def test_pair_single_block_gqa(ext, cuda_device, nsplit):
    _check(ext, cuda_device, 1, 1024, 4, 2, nsplit=nsplit, seed=1)


@pytest.mark.parametrize("nsplit", [1, 3])
def test_pair_ring_blocks(ext, cuda_device, nsplit):
    _check(ext, cuda_device, 3, 512, 2, 2, nsplit=nsplit, seed=2)


def test_pair_causal_contiguous(ext, cuda_device):
    _check(ext, cuda_device, 2, 1024, 2, 1, causal=True, seed=3)


@pytest.mark.parametrize("nsplit", [0, 2])
def test_pair_causal_zigzag(ext, cuda_device, nsplit):
    _check(ext, cuda_device, 2, 1024, 4, 2, causal=True, zigzag=True, nsplit=nsplit, seed=4)


def test_pair_many_units(ext, cuda_device):
    # more work items than resident pairs: every pair loops over several units
    _check(ext, cuda_device, 1, 4096, 16, 4, nsplit=1, seed=5)


def test_pair_partial_outputs(ext, cuda_device):
    g = torch.Generator().manual_seed(6)
    q = torch.randn(512, 2, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1024, 2, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1024, 2, 128, generator=g).to(torch.bfloat16)
    acc, m, l = A.partial_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                    scale=128 ** -0.5)
    racc, rm, rl = oracle.partial_attention(q, k, v, 128 ** -0.5)
    # the kernel's natural-log m may differ from the oracle's exact row max by the
    # lazy-rescale slack; compare the scale-free quantities
    got = acc.cpu().double() / l.cpu().double().unsqueeze(-1)
    ref = racc / rl.unsqueeze(-1)
    assert (got - ref).abs().max().item() < 2e-2
    lse = m.cpu().double() + torch.log(l.cpu().double())
    assert (lse - (rm + torch.log(rl))).abs().max().item() < 2e-2


def test_pair_fused_loopback(ext, cuda_device):
    world, seq, h, hk = 4, 1024, 2, 2
    xs = [inputs.normal_inputs(r, seq, h, 128, heads_kv=hk, seed=70 + r) for r in range(world)]
    glob = [torch.cat([x.q for x in xs]), torch.cat([x.k for x in xs]),
            torch.cat([x.v for x in xs])]
    shard = [[oracle.zigzag_shard(t, r, world).to(torch.bfloat16) for t in glob]
             for r in range(world)]
    blocks = A.ring_slots([s[1].to(cuda_device) for s in shard],
                          [s[2].to(cuda_device) for s in shard])
    rank = 2
    q = shard[rank][0].to(cuda_device).contiguous()
    out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device=cuda_device)
    status = A.new_status(cuda_device)
    plan = ext.flash_fused_loopback(A.PREC_BF16, q, blocks, world, rank, seq, hk, out,
                                    scale=128 ** -0.5, causal=True, zigzag=True, status=status,
                                    timeout_s=5.0)
    A.check_status(status, "pair loopback")
    assert plan[3] == 512, plan
    order = oracle.ring_block_order(rank, world)
    ref = oracle.full_attention(
        shard[rank][0], torch.cat([shard[r][1] for r in order]),
        torch.cat([shard[r][2] for r in order]), 128 ** -0.5,
        oracle.zigzag_positions(rank, world, seq),
        torch.cat([oracle.zigzag_positions(r, world, seq) for r in order]))
    assert (out.float().cpu().double() - ref).abs().max().item() < 2e-2
