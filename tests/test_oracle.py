"""Pin the CPU oracle against golden vectors made by the reference itself.

Goldens (tests/golden/make_golden.py): the reference's Triton kernels run by
Triton's CPU interpreter (fused QR, panel + T, blocked driver, champion
dispatch) and the reference's oracle CPU torch.geqrf. Tolerances are FP32
rounding-level (summation order differs); rank-deficient inputs have
non-unique reflectors and are pinned through the FP64 gates instead.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_cases

import oracle
from gpumode_qr_b200 import checker

RTOL = 2e-5  # FP32 vs FP32 (different summation order), relative to max|H|
NON_UNIQUE = {"rank4"}  # rank-deficient: reflectors of the null space are arbitrary


def _rel(x, ref):
    return float(np.abs(x - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("f64", [False, True])
def test_oracle_fused_matches_reference_kernel(ref_fused, f64):
    for case in golden_cases(ref_fused):
        A = ref_fused[f"{case}_A"]
        H, tau = oracle.geqr2(A, f64=f64)
        gate = checker.check(torch.from_numpy(A).double().float(), torch.from_numpy(H), torch.from_numpy(tau))
        assert gate.passed, (case, gate.as_dict())
        if case in NON_UNIQUE:
            continue
        assert _rel(H, ref_fused[f"{case}_H"]) < RTOL, case
        assert np.abs(tau - ref_fused[f"{case}_tau"]).max() < 1e-5, case


def test_oracle_panel_matches_reference_kernel(ref_panel):
    for case in golden_cases(ref_panel):
        P = ref_panel[f"{case}_P"]
        H, V, tau, T = oracle.panel(P, f64=False)
        assert _rel(H, ref_panel[f"{case}_H"]) < RTOL, case
        assert np.abs(V - ref_panel[f"{case}_V"]).max() < 1e-5, case
        assert np.abs(tau - ref_panel[f"{case}_tau"]).max() < 1e-5, case
        assert np.abs(T - ref_panel[f"{case}_T"]).max() < 1e-5, case


def test_oracle_panel_algebra():
    # Q^T = I - V T^T V^T applied to the panel reproduces triu(H), Q orthonormal
    # (the isolation checks of scripts/hh_panel_isolation.py:33-71).
    g = torch.Generator().manual_seed(11)
    P = torch.randn(3, 70, 32, generator=g).numpy()
    H, V, tau, T = oracle.panel(P, f64=True)
    Vd, Td, Pd = V.astype(np.float64), T.astype(np.float64), P.astype(np.float64)
    R = Pd - Vd @ (Td.transpose(0, 2, 1) @ (Vd.transpose(0, 2, 1) @ Pd))
    assert np.abs(R[:, :32] - np.triu(H[:, :32])).max() < 1e-5
    assert np.abs(np.tril(R[:, :32], -1)).max() < 1e-5 and np.abs(R[:, 32:]).max() < 1e-5
    Q = np.eye(70) - Vd @ Td @ Vd.transpose(0, 2, 1)
    assert np.abs(Q.transpose(0, 2, 1) @ Q - np.eye(70)).max() < 1e-6


def test_oracle_blocked_matches_reference_driver(ref_blocked):
    for case in golden_cases(ref_blocked):
        A = ref_blocked[f"{case}_A"]
        w = int(case.split("_w")[1]) if "_w" in case else 32
        H, tau = oracle.blocked_geqrf(A, w=w, f64=False)
        assert _rel(H, ref_blocked[f"{case}_H"]) < RTOL, case
        assert np.abs(tau - ref_blocked[f"{case}_tau"]).max() < 2e-5, case


def test_oracle_matches_lapack(lapack_golden):
    # the reference's oracle (CPU torch.geqrf): parity for full-rank cases,
    # FP64 gates for all (rank-deficient reflectors are not unique).
    for case in golden_cases(lapack_golden):
        A = lapack_golden[f"{case}_A"]
        H, tau = oracle.geqr2(A, f64=True)
        gate = checker.check(torch.from_numpy(A), torch.from_numpy(H), torch.from_numpy(tau))
        assert gate.passed, (case, gate.as_dict())
        if "rank_deficient" in case or "collinear" in case:
            continue
        par = checker.parity(H, tau, lapack_golden[f"{case}_H"], lapack_golden[f"{case}_tau"])
        assert par.ok(1e-4), (case, par)


def test_oracle_larfb_matches_dense_formula():
    g = torch.Generator().manual_seed(3)
    for r, k, c in ((40, 8, 13), (64, 32, 70), (33, 32, 1)):
        V = torch.randn(2, r, k, generator=g)
        V = torch.tril(V, -1) + torch.eye(r, k)
        T = torch.triu(torch.randn(2, k, k, generator=g))
        C = torch.randn(2, r, c, generator=g)
        out = oracle.larfb(V.numpy(), T.numpy(), C.numpy(), f64=True)
        ref = (C.double() - V.double() @ (T.double().transpose(1, 2) @ (V.double().transpose(1, 2) @ C.double())))
        assert _rel(out, ref.numpy()) < 1e-6  # output rounded to fp32


def test_oracle_f32_f64_consistent():
    g = torch.Generator().manual_seed(5)
    A = torch.randn(3, 96, 96, generator=g).numpy()
    H32, t32 = oracle.blocked_geqrf(A, 32, f64=False)
    H64, t64 = oracle.blocked_geqrf(A, 32, f64=True)
    assert _rel(H32, H64) < 1e-5
    Hu, tu = oracle.geqr2(A, f64=True)
    assert _rel(H64, Hu) < 1e-6  # blocked == unblocked in exact-ish arithmetic


def test_oracle_edge_cases():
    # zero matrix: every tau 0, H == A; 1x1: tau 0; identity: R = -I? (alpha>=0 -> beta=-|x|)
    Z = np.zeros((2, 5, 5), np.float32)
    H, tau = oracle.geqr2(Z)
    assert (H == 0).all() and (tau == 0).all()
    one = np.array([[[3.0]]], np.float32)
    H, tau = oracle.geqr2(one)
    assert H[0, 0, 0] == 3.0 and tau[0, 0] == 0.0
    eye = np.eye(4, dtype=np.float32)[None]
    H, tau = oracle.geqr2(eye)
    # sigma == 0 for every column of I: identity reflectors, R = I
    assert (tau == 0).all() and np.array_equal(H, eye)
