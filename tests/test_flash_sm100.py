"""tcgen05 flash forward vs the float64 oracle: bf16 and fp32 (3xTF32), one
and several ring blocks, GQA, KV splitting, zigzag causal masks and the
reference's partial-output contract (acc, m, l)."""
import pytest
import torch

from ring_attention_benchmark_b200.models import inputs, oracle
from ring_attention_benchmark_b200.ops import attention as A

pytestmark = pytest.mark.gpu


def _blocks(world, spr, h, hk, d, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    qs, ks, vs = [], [], []
    for _ in range(world):
        qs.append(torch.randn(spr, h, d, generator=g))
        ks.append(torch.randn(spr, hk, d, generator=g))
        vs.append(torch.randn(spr, hk, d, generator=g))
    cast = lambda xs: [x.to(dtype) for x in xs]  # noqa: E731
    return cast(qs), cast(ks), cast(vs)


def _run_rank(dev, qs, ks, vs, rank, world, causal=False, zigzag=False, nsplit=0):
    order = oracle.ring_block_order(rank, world)
    out, lse = A.flash_attention(
        qs[rank].to(dev), [ks[s].to(dev) for s in order], [vs[s].to(dev) for s in order],
        causal=causal, zigzag=zigzag, world=world, rank=rank, nsplit=nsplit, return_lse=True)
    torch.cuda.synchronize()
    return out.float().cpu(), lse.cpu()


def _oracle_rank(qs, ks, vs, rank, world, causal=False, zigzag=False):
    d = qs[0].shape[-1]
    scale = d ** -0.5
    spr = qs[0].shape[0]
    if causal:
        pos = [oracle.zigzag_positions(r, world, spr) if zigzag
               else torch.arange(r * spr, (r + 1) * spr) for r in range(world)]
    else:
        pos = None
    state = oracle.empty_state(spr, qs[0].shape[1], d)
    for s in oracle.ring_block_order(rank, world):
        state = oracle.merge_online_softmax(state, oracle.partial_attention(
            qs[rank], ks[s], vs[s], scale, pos[rank] if pos else None, pos[s] if pos else None))
    return oracle.normalize(state), oracle.lse(state)


@pytest.mark.parametrize("d", [64, 128])
def test_bf16_single_block(cuda_device, d):
    qs, ks, vs = _blocks(1, 256, 2, 2, d, torch.bfloat16)
    out, lse = _run_rank(cuda_device, qs, ks, vs, 0, 1)
    ref, rlse = _oracle_rank(qs, ks, vs, 0, 1)
    assert (out.double() - ref).abs().max().item() < 2e-2
    assert (lse.double() - rlse).abs().max().item() < 2e-2


def test_fp32_3xtf32_single_block(cuda_device):
    qs, ks, vs = _blocks(1, 512, 1, 1, 64, torch.float32, seed=1)
    out, lse = _run_rank(cuda_device, qs, ks, vs, 0, 1, nsplit=1)
    ref, rlse = _oracle_rank(qs, ks, vs, 0, 1)
    err = (out.double() - ref).abs().max().item()
    assert err < 2e-5, err  # fp32-level, far below a tf32-only product (~1e-3)
    assert (lse.double() - rlse).abs().max().item() < 2e-5


@pytest.mark.parametrize("dtype,d", [(torch.bfloat16, 128), (torch.float32, 64)])
@pytest.mark.parametrize("nsplit", [1, 3])
def test_ring_blocks_gqa(cuda_device, dtype, d, nsplit):
    world = 3
    qs, ks, vs = _blocks(world, 256, 4, 2, d, dtype, seed=2)
    for rank in range(world):
        out, _ = _run_rank(cuda_device, qs, ks, vs, rank, world, nsplit=nsplit)
        ref, _ = _oracle_rank(qs, ks, vs, rank, world)
        tol = 2e-2 if dtype == torch.bfloat16 else 2e-5
        assert (out.double() - ref).abs().max().item() < tol


@pytest.mark.parametrize("dtype,d,spr,heads,world", [
    (torch.float32, 64, 2048, 1, 3),     # 16 query tiles on every SM: many CTAs per tile
    (torch.bfloat16, 128, 4096, 8, 1),   # 256 query tiles: whole tiles plus cut ones per CTA
    (torch.bfloat16, 64, 384, 3, 2),     # fewer (tile, KV tile) pairs than CTAs: empty ranges
    (torch.bfloat16, 64, 512, 37, 1),    # 148 query tiles: one whole wave on a 148-SM B200
    (torch.float32, 64, 128, 1, 9),      # one query tile cut into 18 one-tile pieces (> 16)
])
def test_balanced_schedule(cuda_device, dtype, d, spr, heads, world):
    """Balanced schedule (nsplit=-1): whole waves of query tiles, then equal
    (query tile, KV tile) shares of the rest per CTA, cut query tiles merged
    from the CTAs' partial records."""
    qs, ks, vs = _blocks(world, spr, heads, 1, d, dtype, seed=6)
    for rank in range(world):
        out, lse = _run_rank(cuda_device, qs, ks, vs, rank, world, nsplit=-1)
        ref, rlse = _oracle_rank(qs, ks, vs, rank, world)
        tol = 2e-2 if dtype == torch.bfloat16 else 2e-5
        assert (out.double() - ref).abs().max().item() < tol
        assert (lse.double() - rlse).abs().max().item() < tol


def test_balanced_schedule_partial_contract(cuda_device):
    x = inputs.normal_inputs(0, 1024, 2, 64)
    y = inputs.normal_inputs(1, 1024, 2, 64)
    dev = cuda_device
    acc, m, l = A.partial_attention(x.q.to(dev), y.k.to(dev), y.v.to(dev), x.scale, nsplit=-1)
    torch.cuda.synchronize()
    racc, rm, rl = oracle.partial_attention(x.q, y.k, y.v, x.scale)
    out = acc.cpu().double() / l.cpu().double().unsqueeze(-1)
    assert torch.allclose(out, racc / rl.unsqueeze(-1), atol=2e-5)
    assert torch.allclose(m.cpu().double() + torch.log(l.cpu().double()), rm + torch.log(rl),
                          atol=2e-5)


def test_balanced_schedule_rejects_causal(cuda_device):
    qs, ks, vs = _blocks(1, 256, 1, 1, 64, torch.bfloat16)
    with pytest.raises(RuntimeError, match="balanced"):
        _run_rank(cuda_device, qs, ks, vs, 0, 1, causal=True, nsplit=-1)


@pytest.mark.parametrize("dtype,d", [(torch.bfloat16, 128), (torch.float32, 64)])
def test_dynamic_schedule_reuses_status(cuda_device, dtype, d):
    """Causal launches claim work items from a counter in the status block; the
    last CTA resets it, so back-to-back launches on one status block stay exact
    and leave the counter words at zero."""
    C = A.load()
    world = 2
    qs, ks, vs = _blocks(world, 1024, 3, 1, d, dtype, seed=7)
    dev = cuda_device
    status = A.new_status(dev)
    for rank in range(world):
        order = oracle.ring_block_order(rank, world)
        slots = A.ring_slots([ks[s].to(dev) for s in order], [vs[s].to(dev) for s in order])
        q = qs[rank].to(dev)
        ref, _ = _oracle_rank(qs, ks, vs, rank, world, causal=True, zigzag=True)
        for _ in range(3):
            out = torch.empty_like(q)
            C.flash_fwd(A.prec_of(dtype), q, slots, world, 1024, 1, out=out, scale=d ** -0.5,
                        causal=True, zigzag=True, world=world, rank=rank, status=status)
            torch.cuda.synchronize()
            A.check_status(status)
            assert status.tolist()[5:7] == [0, 0]
            tol = 2e-2 if dtype == torch.bfloat16 else 2e-5
            assert (out.float().cpu().double() - ref).abs().max().item() < tol


@pytest.mark.parametrize("dtype,d", [(torch.bfloat16, 128), (torch.float32, 64)])
def test_zigzag_causal(cuda_device, dtype, d):
    world = 2
    qs, ks, vs = _blocks(world, 512, 2, 1, d, dtype, seed=3)
    for rank in range(world):
        out, lse = _run_rank(cuda_device, qs, ks, vs, rank, world, causal=True, zigzag=True)
        ref, rlse = _oracle_rank(qs, ks, vs, rank, world, causal=True, zigzag=True)
        tol = 2e-2 if dtype == torch.bfloat16 else 2e-5
        assert (out.double() - ref).abs().max().item() < tol
        assert (lse.double() - rlse).abs().max().item() < tol


def test_partial_contract_fp32(cuda_device):
    x = inputs.normal_inputs(0, 256, 2, 64)
    y = inputs.normal_inputs(1, 256, 2, 64)
    dev = cuda_device
    acc, m, l = A.partial_attention(x.q.to(dev), y.k.to(dev), y.v.to(dev), x.scale)
    torch.cuda.synchronize()
    racc, rm, rl = oracle.partial_attention(x.q, y.k, y.v, x.scale)
    # the kernel may keep a reference max up to 2^8 below the row max (lazy
    # rescaling); compare the invariant quantities acc/l and m + log l
    out = acc.cpu().double() / l.cpu().double().unsqueeze(-1)
    assert torch.allclose(out, racc / rl.unsqueeze(-1), atol=2e-5)
    assert torch.allclose(m.cpu().double() + torch.log(l.cpu().double()), rm + torch.log(rl),
                          atol=2e-5)


@pytest.mark.parametrize("causal", [False, True])
def test_two_tile_bf16_kernel(cuda_device, monkeypatch, causal):
    """The opt-in two-query-tile bf16 kernel (RAB_FLASH_2Q=1) against the oracle."""
    monkeypatch.setenv("RAB_FLASH_2Q", "1")
    world = 2
    qs, ks, vs = _blocks(world, 512, 4, 2, 128, torch.bfloat16, seed=5)
    for rank in range(world):
        out, lse = _run_rank(cuda_device, qs, ks, vs, rank, world, causal=causal, zigzag=causal)
        ref, rlse = _oracle_rank(qs, ks, vs, rank, world, causal=causal, zigzag=causal)
        assert (out.double() - ref).abs().max().item() < 2e-2
        assert (lse.double() - rlse).abs().max().item() < 2e-2
