"""Summary of the fused kernel's overlap trace (utils.overlap) on synthetic
stamps: per-block waits, arrival times and the TMA wait fraction."""
import torch

from ring_attention_benchmark_b200.utils.overlap import summarize


def test_summary_of_synthetic_stamps():
    grid, slots = 4, 64
    s = torch.zeros(grid, slots, 2, dtype=torch.int64)
    for c in range(grid):
        s[c, 0] = torch.tensor([1000 + c, 101000])  # 100 us of TMA role
    s[0, 1] = torch.tensor([20000, 30000])  # CTA 0 waited 10 us for block 1
    s[1, 1] = torch.tensor([25000, 25000])  # CTA 1 found it present
    out = summarize(s, world=3)
    assert out["ctas"] == 4 and abs(out["kernel_tma_span_us"] - 100.0) < 1e-6
    b1, b2 = out["blocks"]
    assert b1["ctas_waited"] == 2 and b1["wait_us_max"] == 10.0 and b1["wait_us_median"] == 0.0
    assert b2["ctas_waited"] == 0
    assert abs(out["tma_wait_fraction_max"] - 0.1) < 1e-3
    assert summarize(torch.zeros(2, slots, 2, dtype=torch.int64), 2) == {"ctas": 0}
