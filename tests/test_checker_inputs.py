"""The FP64 gate restatement and the seeded input generators (CPU)."""

from __future__ import annotations

import json

import pytest
import torch
from conftest import GOLDEN, load_golden

from gpumode_qr_b200 import checker, inputs


def _ref_checker():
    return json.loads((GOLDEN / "ref_checker.json").read_text())


def test_checker_reproduces_reference_values():
    ref = _ref_checker()
    lap = load_golden("lapack.npz")
    fused = load_golden("ref_fused.npz")
    blocked = load_golden("ref_blocked.npz")
    A1, H1, t1 = (torch.from_numpy(lap[f"cfg1_{s}"]) for s in ("A", "H", "tau"))
    Hbad = H1.clone()
    Hbad[:, 5, 2] += 1e-2
    cases = {
        "cfg1_geqrf": (A1, H1, t1),
        "cfg1_perturbed": (A1, Hbad, t1),
        "fused_n33": tuple(torch.from_numpy(fused[f"n33_{s}"]) for s in ("A", "H", "tau")),
        "blocked_n100": tuple(torch.from_numpy(blocked[f"n100_w32_{s}"]) for s in ("A", "H", "tau")),
    }
    for name, (A, H, tau) in cases.items():
        got = checker.check(A, H, tau).as_dict()
        want = ref[name]
        for key in ("factor_residual", "orth_residual", "leakage", "reconstruction"):
            assert got[key] == pytest.approx(want[key], rel=1e-6, abs=1e-12), (name, key)
        for key in ("factor_threshold", "orth_threshold", "passed", "factor_pass", "orth_pass", "n", "batch"):
            assert got[key] == want[key], (name, key)
    assert not ref["cfg1_perturbed"]["passed"]


def test_checker_chunking_matches_single_slice(monkeypatch):
    g = torch.Generator().manual_seed(0)
    A = torch.randn(5, 20, 20, generator=g)
    H, tau = torch.geqrf(A)
    whole = checker.check(A, H, tau)
    monkeypatch.setattr(checker, "_auto_batch_chunk", lambda b, n, max_bytes=0: 2)
    chunked = checker.check(A, H, tau)
    assert whole.factor_residual == pytest.approx(chunked.factor_residual)
    assert whole.orth_residual == pytest.approx(chunked.orth_residual)


def test_parity_metric():
    g = torch.Generator().manual_seed(1)
    A = torch.randn(3, 16, 16, generator=g)
    H, tau = torch.geqrf(A)
    p = checker.parity(H, tau, H, tau)
    assert p.h_rel == 0 and p.tau_rel == 0 and p.ok()
    H2 = H.clone()
    H2[1, 3, 3] += 0.1 * H.abs().max()
    assert not checker.parity(H2, tau, H, tau).ok()


def test_config_table_matches_workload_spec():
    got = [(c.batch, c.n, c.kind, c.seed, c.log10_cond) for c in inputs.CONFIGS]
    assert got == [(8, 64, "iid", 0, 0.0), (4096, 32, "iid", 1, 0.0), (640, 512, "haar", 2, 2.0),
                   (64, 1024, "haar", 3, 4.0), (8, 4096, "iid", 4, 0.0)]
    assert inputs.config(2).bytes == 33_554_432
    assert inputs.config(3).flops == pytest.approx(114.53e9, rel=1e-3)
    assert [c.parity for c in inputs.CONFIGS] == [True, True, True, False, True]


def test_input_checksums_pinned():
    sums = json.loads((GOLDEN / "input_checksums.json").read_text())
    for cfg in inputs.CONFIGS:
        if cfg.n >= 4096:
            continue  # 537 MB draw; pinned by the same generator path as cfg1/cfg2
        want = sums[cfg.name]
        A = inputs.make_config_input(cfg, batch=want["batch"]).double()
        assert A.sum().item() == pytest.approx(want["sum"], rel=1e-9, abs=1e-6)
        assert (A * A).sum().item() == pytest.approx(want["sumsq"], rel=1e-9)
        assert A.reshape(-1)[:4].tolist() == pytest.approx(want["first"], rel=1e-12)


def test_haar_inputs_have_requested_spectrum():
    cfg = inputs.Config(9, 2, 48, "haar", 7, 2.0)
    A = inputs.make_config_input(cfg).double()
    s = torch.linalg.svdvals(A)
    want = torch.logspace(0, 2, 48, dtype=torch.float64).flip(0)
    assert torch.allclose(s, want.expand_as(s), rtol=1e-5)


def test_stress_cases_structure():
    cases = inputs.stress_cases(32, batch=4)
    assert [c.name for c in cases] == [
        f"{k}_n32" for k in ("dense_cond1", "dense_cond4", "rank_deficient", "near_rank_deficient",
                             "banded", "row_scaled", "near_collinear", "upper_triangular",
                             "clustered_scale")]
    assert all(c.tensor.shape == (4, 32, 32) and c.tensor.dtype == torch.float32 for c in cases)
    rd = cases[2].tensor.double()
    assert int(torch.linalg.matrix_rank(rd[0], rtol=1e-5)) == 16  # rank n/2 up to fp32 rounding
    ut = cases[7].tensor
    assert torch.equal(ut, torch.triu(ut))


def test_benchmark_shapes_are_the_reference_shapes():
    assert [(s["batch"], s["n"], s["cond"]) for s in inputs.BENCHMARK_SHAPES] == [
        (20, 32, 1), (40, 176, 1), (40, 352, 1), (640, 512, 2), (60, 1024, 2), (8, 2048, 1), (2, 4096, 1)]
    p = inputs.make_benchmark_problem(inputs.BENCHMARK_SHAPES[0])
    assert p.name == "b20_n32_cond1" and p.tensor.shape == (20, 32, 32)
