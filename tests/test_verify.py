"""The benchmark's output check (`utils.verify.ring_output_error`) on CPU
tensors: the float64 oracle ring's own outputs pass at rounding level, a
perturbed row is caught, causal zigzag and GQA included."""
import pytest
import torch

from ring_attention_benchmark_b200.models import inputs, oracle
from ring_attention_benchmark_b200.utils.verify import ring_output_error, sample_rows


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_ring_passes_and_perturbation_is_caught(causal):
    world, seq, h, hk, d = 3, 64, 4, 2, 16
    xs = [inputs.normal_inputs(r, seq, h, d, heads_kv=hk) for r in range(world)]
    pos = [oracle.zigzag_positions(r, world, seq) for r in range(world)] if causal else None
    outs = oracle.ring_attention([x.q for x in xs], [x.k for x in xs], [x.v for x in xs],
                                 xs[0].scale, positions=pos)
    for r in range(world):
        err = ring_output_error(outs[r], xs[r].q, r, world, lambda s: (xs[s].k, xs[s].v),
                                xs[0].scale, causal=causal, zigzag=causal, n_rows=16)
        assert err < 1e-12
    rows = sample_rows(seq, 16)
    bad = outs[1].clone()
    bad[rows[5], 2, 3] += 1e-3
    err = ring_output_error(bad, xs[1].q, 1, world, lambda s: (xs[s].k, xs[s].v), xs[0].scale,
                            causal=causal, zigzag=causal, n_rows=16)
    assert abs(err - 1e-3) < 1e-9


def test_sample_rows_cover_the_ends():
    r = sample_rows(16384, 256)
    assert r[0] == 0 and r[-1] == 16383 and r.numel() == 256
    assert sample_rows(100, 256).numel() == 100
