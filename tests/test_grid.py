"""Host logic of the (batch, n) grid sweep: regime classification, summary and
table (the GPU run itself is python -m gpumode_qr_b200.grid)."""

from __future__ import annotations

import math

from gpumode_qr_b200 import grid

PEAKS = {"hbm_gbs": 6553.0, "source": "test"}


def test_regime_bounds_follow_the_roofline_crossover():
    small = grid.regime(4096, 32, 0.0225, PEAKS)
    assert small["path"] == "fused" and small["bound"] == "hbm"
    assert math.isclose(small["floor_ms"], 2 * 4096 * 32 * 32 * 4 / 6553e9 * 1e3)
    assert 0.2 < small["roofline_frac"] < 0.25 and small["achieved_unit"] == "GB/s"
    big = grid.regime(8, 4096, 30.0, PEAKS)
    assert big["path"] == "blocked" and big["bound"] == "flop"
    assert grid.regime(8, 64, 0.035, PEAKS)["path"] == "fused_cta"
    assert grid.regime(1024, 96, 0.27, PEAKS)["path"] == "blocked"
    flops = 4 / 3 * 4096**3 * 8
    assert math.isclose(big["achieved"], flops / 0.030 / 1e12)
    assert math.isclose(big["roofline_frac"], flops / (grid.FP32_FFMA_TFLOPS * 1e12) * 1e3 / 30.0)


def _row(b, n, ms, sp, passed=True):
    return {"shape": {"batch": b, "n": n, "cond": 1}, "name": f"b{b}_n{n}_cond1",
            "correctness": {"passed": passed}, "b200_geqrf": {"median_ms": ms},
            "regime": grid.regime(b, n, ms, PEAKS), "speedup_vs_torch_cuda": sp}


def test_summary_and_table():
    rows = [_row(2, 32, 0.01, 4.0), _row(2, 64, 0.05, 9.0), _row(8, 32, 0.01, 16.0, passed=False)]
    s = grid.summarize(rows)
    assert s["n_points"] == 3 and s["gate_failures"] == ["b8_n32_cond1"]
    assert math.isclose(s["speedup_vs_torch_cuda"]["geomean"], (4 * 9 * 16) ** (1 / 3))
    md = grid.markdown(rows)
    lines = md.splitlines()
    assert lines[0].startswith("| batch \\ n | 32 | 64 |")
    assert len(lines) == 4 and "16x" in lines[3] and lines[3].endswith("|  |")
