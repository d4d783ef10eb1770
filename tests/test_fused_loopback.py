"""The fused ring path on ONE GPU: the fused kernel runs as one rank of an
emulated 4-rank ring whose peers' slots and flag words are regions of the same
GPU's memory (`flash_fused_loopback`).  The copy warps pull blocks 1..3 from
those "peer" slots into the rank's own ring slots, bump the per-block arrival
counters, and the TMA thread waits on them (with the generic->async proxy
fence) before it loads the copied tiles - the code path of a real multi-GPU
launch, checked here against the float64 oracle over the whole ring, without
needing a second GPU.
"""
import pytest
import torch

from ring_attention_benchmark_b200.models import inputs, oracle
from ring_attention_benchmark_b200.ops import attention as A

pytestmark = pytest.mark.gpu

WORLD = 4


def _run(ext, dev, rank, seq, heads, heads_kv, d, dtype, causal):
    prec = A.prec_of(dtype)
    xs = [inputs.normal_inputs(r, seq, heads, d, heads_kv=heads_kv, seed=50 + r)
          for r in range(WORLD)]
    if causal:  # zigzag shards of one global sequence
        glob = [torch.cat([x.q for x in xs]), torch.cat([x.k for x in xs]),
                torch.cat([x.v for x in xs])]
        shard = [[oracle.zigzag_shard(t, r, WORLD) for t in glob] for r in range(WORLD)]
    else:
        shard = [[x.q, x.k, x.v] for x in xs]
    shard = [[t.to(dtype) for t in s] for s in shard]
    blocks = A.ring_slots([s[1].to(dev) for s in shard], [s[2].to(dev) for s in shard])
    q = shard[rank][0].to(dev).contiguous()
    out = torch.full(q.shape, float("nan"), dtype=dtype, device=dev)
    lse = torch.full((seq, heads), float("nan"), device=dev)
    status = A.new_status(dev)
    plan = ext.flash_fused_loopback(prec, q, blocks, WORLD, rank, seq, heads_kv, out, lse,
                                    scale=d ** -0.5, causal=causal, zigzag=causal,
                                    status=status, timeout_s=5.0)
    A.check_status(status, "fused loopback")
    # oracle: this rank's queries over every rank's keys, in global positions
    order = oracle.ring_block_order(rank, WORLD)
    k_all = torch.cat([shard[r][1] for r in order])
    v_all = torch.cat([shard[r][2] for r in order])
    q_pos = k_pos = None
    if causal:
        q_pos = oracle.zigzag_positions(rank, WORLD, seq)
        k_pos = torch.cat([oracle.zigzag_positions(r, WORLD, seq) for r in order])
    ref = oracle.full_attention(shard[rank][0], k_all, v_all, d ** -0.5, q_pos, k_pos)
    s = oracle._mask(oracle.scores(shard[rank][0], k_all, d ** -0.5), q_pos, k_pos)
    ref_lse = torch.logsumexp(s, dim=-1).transpose(0, 1)
    return plan, out.cpu().double(), ref, lse.cpu().double(), ref_lse


@pytest.mark.parametrize("rank", [0, 3])
def test_loopback_fp32(ext, cuda_device, rank):
    plan, out, ref, lse, ref_lse = _run(ext, cuda_device, rank, 512, 2, 2, 64, torch.float32,
                                        False)
    assert torch.isfinite(out).all()
    assert (out - ref).abs().max().item() < 2e-5, plan
    assert (lse - ref_lse).abs().max().item() < 2e-5, plan


@pytest.mark.parametrize("rank", [1, 2])
def test_loopback_bf16_causal_zigzag_gqa(ext, cuda_device, rank):
    plan, out, ref, lse, ref_lse = _run(ext, cuda_device, rank, 1024, 4, 2, 128, torch.bfloat16,
                                        True)
    assert torch.isfinite(out).all()
    assert (out - ref).abs().max().item() < 2e-2, plan
    assert (lse - ref_lse).abs().max().item() < 2e-2, plan


def test_loopback_bf16_two_tile_kernel(ext, cuda_device, monkeypatch):
    monkeypatch.setenv("RAB_FLASH_2Q", "1")  # the two-query-tile kernel on a small shape
    plan, out, ref, lse, ref_lse = _run(ext, cuda_device, 2, 512, 2, 1, 128, torch.bfloat16,
                                        False)
    assert plan[3] == 256, plan  # 256-row units: the two-tile kernel ran
    assert (out - ref).abs().max().item() < 2e-2, plan
    assert (lse - ref_lse).abs().max().item() < 2e-2, plan
