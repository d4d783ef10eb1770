"""Host planner of the flash kernel, on the CPU (no GPU: the SM count is given).

* The causal planner's closed-form visible tile ranges against a brute-force
  classification of every (query tile, KV tile) pair by global position, with
  contiguous and zigzag sharding, several ranks and ring block offsets.
* The schedule choices the kernel relies on: the balanced schedule for the
  headline 16384 x 1 head fp32 workload, equal split for many heads, dynamic
  claiming with a split for long causal rows, and the forced modes.
"""
import pytest

from ring_attention_benchmark_b200._ext import load
from ring_attention_benchmark_b200.models import oracle

F32, BF16 = 1, 0


@pytest.fixture(scope="module")
def C():
    try:
        return load()
    except Exception as e:  # pragma: no cover - extension not built
        pytest.skip(f"extension not built: {e}")


def _brute_visible(prec, sq, skv, nblk, zigzag, world, rank, blk_offset, q0):
    kN = 64 if prec == F32 else 128
    tpb = skv // kN

    def pos(owner, n, i):
        if zigzag:
            return int(oracle.zigzag_positions(owner, world, n)[i])
        return owner * n + i

    q_hi = pos(rank, sq, q0 + 127)
    vis = set()
    for s in range(nblk):
        owner = (rank - blk_offset - s) % world
        for t in range(tpb):
            if pos(owner, skv, t * kN) <= q_hi:
                vis.add(s * tpb + t)
    return vis


@pytest.mark.parametrize("prec", [F32, BF16])
@pytest.mark.parametrize("zigzag", [False, True])
@pytest.mark.parametrize("world,rank,blk_offset", [(1, 0, 0), (2, 1, 0), (4, 2, 0), (4, 3, 1)])
def test_visible_ranges_match_bruteforce(C, prec, zigzag, world, rank, blk_offset):
    sq = skv = 1024
    nblk = world - blk_offset
    for q0 in range(0, sq, 128):
        ranges = C.flash_visible_ranges(prec, sq, skv, nblk, zigzag, world, rank, blk_offset, q0)
        got = set()
        for a, b in ranges:
            assert a < b
            got.update(range(a, b))
        assert got == _brute_visible(prec, sq, skv, nblk, zigzag, world, rank, blk_offset, q0), \
            (q0, ranges)


def test_plan_headline_is_balanced(C, monkeypatch):
    monkeypatch.delenv("RAB_FLASH_2Q", raising=False)
    # 16384 tokens x 1 head: 128 query tiles would leave 20 of 148 SMs idle
    pl = C.flash_plan_info(F32, 16384, 16384, 1, 1, 1, 64, sms=148)
    assert pl["balanced"] == 1 and pl["grid"] == 148 and pl["n_items"] == 148
    assert pl["full_waves"] == 0 and pl["dynamic"] == 0
    # two partial records (acc [128][64] + m + l) per CTA
    assert pl["workspace_bytes"] == 2 * 148 * 128 * (64 + 2) * 4
    # eight ring blocks: still balanced, every CTA also copies its slice
    pl8 = C.flash_plan_info(F32, 16384, 16384, 8, 1, 1, 64, sms=148, fused=True)
    assert pl8["balanced"] == 1 and pl8["grid"] == 148


def test_plan_many_heads_two_tile(C, monkeypatch):
    monkeypatch.delenv("RAB_FLASH_2Q", raising=False)
    # non-causal bf16 with >= two waves of 256-row units: the two-query-tile kernel
    pl = C.flash_plan_info(BF16, 16384, 16384, 1, 32, 32, 128, sms=148)
    assert pl["rows_per_unit"] == 256 and pl["balanced"] == 0 and pl["nsplit"] == 1
    assert pl["n_items"] == 2048 and pl["grid"] == 148 and pl["workspace_bytes"] == 0
    # disabled: one-tile kernel, equal split
    monkeypatch.setenv("RAB_FLASH_2Q", "0")
    pl = C.flash_plan_info(BF16, 16384, 16384, 1, 32, 32, 128, sms=148)
    assert pl["rows_per_unit"] == 128 and pl["nsplit"] == 1 and pl["n_items"] == 4096
    monkeypatch.delenv("RAB_FLASH_2Q")
    # too few non-causal 256-row units (64 < 2 waves): one-tile kernel; causal: the
    # two-tile kernel with dynamic claiming, whatever the size
    assert C.flash_plan_info(BF16, 16384, 16384, 1, 1, 1, 128, sms=148)["rows_per_unit"] == 128
    pc = C.flash_plan_info(BF16, 16384, 16384, 1, 32, 32, 128, causal=True, sms=148)
    assert pc["rows_per_unit"] == 256 and pc["dynamic"] == 1
    assert C.flash_plan_info(BF16, 1024, 1024, 1, 1, 1, 128, causal=True,
                             sms=148)["rows_per_unit"] == 256
    # the balanced schedule is never combined with the two-tile kernel, even when forced
    monkeypatch.setenv("RAB_FLASH_2Q", "1")
    assert C.flash_plan_info(BF16, 4096, 4096, 1, 8, 8, 128, nsplit=-1,
                             sms=148)["rows_per_unit"] == 128
    monkeypatch.delenv("RAB_FLASH_2Q")
    # fp32 never
    assert C.flash_plan_info(F32, 16384, 16384, 1, 32, 32, 64, sms=148)["rows_per_unit"] == 128


def test_plan_causal_is_dynamic(C, monkeypatch):
    monkeypatch.delenv("RAB_FLASH_2Q", raising=False)
    # long causal rows on one head: a split shortens the longest query tile
    pl = C.flash_plan_info(F32, 16384, 16384, 1, 1, 1, 64, causal=True, sms=148)
    assert pl["dynamic"] == 1 and pl["balanced"] == 0 and pl["nsplit"] == 2
    # many heads: enough items without a split
    pl = C.flash_plan_info(BF16, 16384, 16384, 1, 32, 32, 128, causal=True, sms=148)
    assert pl["dynamic"] == 1 and pl["nsplit"] == 1


def test_plan_fused_causal_follows_ring_blocks(C, monkeypatch):
    """In a fused ring launch every item walks its chunk's ring blocks in order
    and waits for each to land; when the blocks arrive slower than the items
    use them (16k tokens x 32 heads per rank: 268 MB blocks), the causal split
    cuts the ring at block boundaries so the early items run on the blocks
    already present.  Long GQA rows use each block for longer than it takes to
    arrive and keep (nearly) whole items."""
    monkeypatch.delenv("RAB_FLASH_2Q", raising=False)
    for world in (2, 4, 8):
        for rank in (0, world - 1):
            pl = C.flash_plan_info(BF16, 16384, 16384, world, 32, 32, 128, causal=True,
                                   zigzag=True, world=world, rank=rank, sms=148, fused=True)
            ns = pl["nsplit"]
            assert pl["dynamic"] == 1 and ns >= max(2, world // 2), (world, rank, ns)
            assert world % ns == 0, (world, rank, ns)  # chunks made of whole ring blocks
        gqa = C.flash_plan_info(BF16, 65536, 65536, world, 32, 8, 128, causal=True, zigzag=True,
                                world=world, rank=0, sms=148, fused=True)
        assert gqa["nsplit"] <= 2, (world, gqa["nsplit"])
    # the same shape on one GPU (no ring) keeps whole items
    one = C.flash_plan_info(BF16, 16384, 16384, 1, 32, 32, 128, causal=True, zigzag=True,
                            sms=148)
    assert one["nsplit"] == 1
    # without a mask too (two-tile kernel, static item order): block-aligned chunks
    for world in (4, 8):
        nc = C.flash_plan_info(BF16, 16384, 16384, world, 32, 32, 128, world=world, sms=148,
                               fused=True)
        assert nc["rows_per_unit"] == 256 and nc["balanced"] == 0 and nc["dynamic"] == 0
        assert nc["nsplit"] >= world // 2 and world % nc["nsplit"] == 0, (world, nc["nsplit"])
    # the fp32 headline keeps its balanced schedule at every ring size
    for world in (1, 2, 8):
        hl = C.flash_plan_info(F32, 16384, 16384, world, 1, 1, 64, world=world, sms=148,
                               fused=world > 1)
        assert hl["balanced"] == 1


def test_plan_forced_modes(C, monkeypatch):
    monkeypatch.delenv("RAB_FLASH_2Q", raising=False)
    pl = C.flash_plan_info(BF16, 4096, 4096, 1, 8, 8, 128, nsplit=-1, sms=148)
    assert pl["balanced"] == 1 and pl["full_waves"] == 1  # 256 units: one whole wave first
    pl = C.flash_plan_info(BF16, 4096, 4096, 1, 8, 8, 128, nsplit=3, sms=148)
    assert pl["balanced"] == 0 and pl["nsplit"] == 3 and pl["n_items"] == 768
    with pytest.raises(RuntimeError, match="balanced"):
        C.flash_plan_info(BF16, 4096, 4096, 1, 8, 8, 128, causal=True, nsplit=-1, sms=148)


def test_pair_kernel_plan(monkeypatch):
    """RAB_FLASH_2SM=1 selects the CTA-pair kernel (512-row units, an even grid
    of pairs) for bf16 d=128 shapes that split into 512-row units, and nothing
    else."""
    from ring_attention_benchmark_b200 import _ext

    C = _ext.load()
    monkeypatch.setenv("RAB_FLASH_2SM", "1")
    info = C.flash_plan_info(0, 4096, 4096, 2, 8, 8, 128, causal=True, zigzag=True, world=2,
                             rank=0, sms=148)
    assert info["rows_per_unit"] == 512 and info["grid"] % 2 == 0 and info["grid"] <= 148
    assert info["dynamic"] == 1
    fused = C.flash_plan_info(0, 4096, 4096, 2, 8, 8, 128, world=2, sms=148, fused=True)
    assert fused["rows_per_unit"] == 512 and fused["grid"] == 148
    # d=64, fp32, a zigzag half that is not a multiple of 512 rows: not the pair kernel
    assert C.flash_plan_info(0, 4096, 4096, 1, 8, 8, 64, sms=148)["rows_per_unit"] != 512
    assert C.flash_plan_info(1, 4096, 4096, 1, 1, 1, 64, sms=148)["rows_per_unit"] == 128
    assert C.flash_plan_info(0, 1536, 1536, 2, 8, 8, 128, causal=True, zigzag=True, world=2,
                             sms=148)["rows_per_unit"] != 512
    monkeypatch.setenv("RAB_FLASH_2SM", "0")
    assert C.flash_plan_info(0, 4096, 4096, 1, 8, 8, 128, sms=148)["rows_per_unit"] != 512


def test_plan_split_invariants(C, monkeypatch):
    """Whatever split the planner picks, the plan is self-consistent: items =
    units x split, the grid never exceeds the SMs (fused launches use every SM,
    each CTA also copies a slice), the split never exceeds the tiles of a unit,
    and the workspace holds one partial record per item when there is a split."""
    monkeypatch.delenv("RAB_FLASH_2Q", raising=False)
    for prec, d in ((BF16, 128), (BF16, 64), (F32, 64)):
        for causal in (False, True):
            for world in (1, 2, 3, 8):
                for seq, heads in ((1024, 4), (4096, 8), (16384, 1)):
                    pl = C.flash_plan_info(prec, seq, seq, world, heads, heads, d, causal=causal,
                                           zigzag=causal, world=world, rank=world - 1, sms=148,
                                           fused=world > 1)
                    kn = 64 if prec == F32 else 128
                    tiles = world * seq // kn
                    assert 1 <= pl["grid"] <= 148
                    if pl["balanced"]:
                        assert pl["n_items"] == pl["grid"] and not causal
                        continue
                    ns = pl["nsplit"]
                    assert 1 <= ns <= max(1, tiles), pl
                    assert pl["n_items"] == pl["n_units"] * ns
                    assert pl["n_units"] == heads * seq // pl["rows_per_unit"]
                    if world > 1:
                        assert pl["grid"] == 148
                    rec = pl["n_items"] * pl["rows_per_unit"] * (d + 2) * 4
                    assert pl["workspace_bytes"] == (rec if ns > 1 else 0)
                    assert pl["merge_kernel"] == (1 if ns > 1 else 0)
