"""GPU parity of each kernel family through the C ABI against the oracle.

Tolerances: H and tau within 1e-4 of the reference's outputs relative to
max|H| (FP32 rounding-level; the north-star bar is 1e-3), T within 1e-4
absolute, trailing update within 1e-5 relative to max|C| of the FP64 oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_cases

import oracle
from gpumode_qr_b200 import _lib, api, checker

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
RTOL = 1e-4


def _rel(x, ref):
    x = x.detach().cpu().numpy() if hasattr(x, "detach") else x
    return float(np.abs(x - ref).max() / max(np.abs(ref).max(), 1e-30))


def test_fused_kernel_matches_reference_kernel(ref_fused):
    for case in golden_cases(ref_fused):
        A = torch.from_numpy(ref_fused[f"{case}_A"])
        if A.shape[-1] > api.fused_max_n():
            continue
        H, tau = api.hh_fused_qr(A.to(DEV))
        gate = checker.check(A, H.cpu(), tau.cpu())
        assert gate.passed, (case, gate.as_dict())
        if case == "rank4":
            continue  # reflectors of a rank-deficient matrix are not unique
        assert _rel(H, ref_fused[f"{case}_H"]) < RTOL, case
        assert np.abs(tau.cpu().numpy() - ref_fused[f"{case}_tau"]).max() < RTOL, case


@pytest.mark.parametrize("n", list(range(1, 33)))
def test_fused_kernel_every_small_n(n):
    A = torch.randn(37, n, n, generator=torch.Generator().manual_seed(n))
    H, tau = api.hh_fused_qr(A.to(DEV))
    Ho, to = oracle.geqr2(A.numpy(), f64=True)
    par = checker.parity(H.cpu(), tau.cpu(), Ho, to)
    assert par.ok(RTOL), (n, par)
    assert checker.check(A, H.cpu(), tau.cpu()).passed
    if n == 1:
        assert (tau == 0).all()
    assert (tau[:, -1] == 0).all()


@pytest.mark.parametrize("n", [33, 40, 64, 65, 96, 97, 127, 128])
def test_fused_operator_covers_the_reference_cap(n):
    # hh_fused_qr serves every n <= 128, as the reference's make_hh_fused_smalln
    # (src/qrbench/variants.py:698, :741); above 32 one CTA factors one matrix.
    A = torch.randn(5, n, n, generator=torch.Generator().manual_seed(1000 + n))
    H, tau = api.hh_fused_qr(A.to(DEV))
    Ho, to = oracle.geqr2(A.numpy(), f64=True)
    par = checker.parity(H.cpu(), tau.cpu(), Ho, to)
    assert par.ok(RTOL), (n, par)
    assert checker.check(A, H.cpu(), tau.cpu()).passed
    Hg, tg = api.geqrf(A.to(DEV))  # the champion route runs the same kernel here
    assert torch.equal(Hg, H) and torch.equal(tg, tau)


def test_fused_operator_refuses_n_above_128():
    with pytest.raises(ValueError, match="n <= 128"):
        api.hh_fused_qr(torch.zeros(1, 129, 129, device=DEV))


@pytest.mark.parametrize("n", [1, 5, 8, 9, 16, 17, 31, 32])
@pytest.mark.parametrize("b", [1, 3, 5, 6, 7, 37, 4736, 4737])
def test_fused_kernel_two_and_four_matrices_per_warp_agree(n, b):
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(b * 33 + n)).to(DEV)
    outs = {}
    try:
        for cpl in (2, 4, 0):
            _lib.set_config("fused_cpl", cpl)
            outs[cpl] = api.hh_fused_qr(A)
    finally:
        _lib.set_config("fused_cpl", 0)
    for cpl in (4, 0):
        assert torch.equal(outs[cpl][0], outs[2][0]) and torch.equal(outs[cpl][1], outs[2][1])
    if b <= 37:
        assert checker.check(A.cpu(), outs[2][0].cpu(), outs[2][1].cpu()).passed


def test_panel_kernel_matches_reference_kernel(ref_panel):
    for case in golden_cases(ref_panel):
        P = torch.from_numpy(ref_panel[f"{case}_P"])
        H, V, tau, T = api.hh_panel_qr(P.to(DEV))
        assert _rel(H, ref_panel[f"{case}_H"]) < RTOL, case
        assert np.abs(V.cpu().numpy() - ref_panel[f"{case}_V"]).max() < RTOL, case
        assert np.abs(tau.cpu().numpy() - ref_panel[f"{case}_tau"]).max() < RTOL, case
        assert np.abs(T.cpu().numpy() - ref_panel[f"{case}_T"]).max() < RTOL, case


@pytest.mark.parametrize("r,w", [(32, 32), (33, 32), (64, 32), (257, 32), (512, 32), (513, 32),
                                 (1024, 32), (1500, 32), (2048, 32), (3000, 32), (4096, 32),
                                 (8192, 32), (100, 7), (2049, 16), (40, 1)])
def test_panel_kernel_shapes_and_clusters(r, w):
    b = 3 if r <= 4096 else 1
    P = torch.randn(b, r, w, generator=torch.Generator().manual_seed(r + w))
    H, V, tau, T = api.hh_panel_qr(P.to(DEV))
    Ho, Vo, to, To = oracle.panel(P.numpy(), f64=True)
    assert _rel(H, Ho) < RTOL
    assert np.abs(V.cpu().numpy() - Vo).max() < RTOL
    assert np.abs(tau.cpu().numpy() - to).max() < RTOL
    assert np.abs(T.cpu().numpy() - To).max() < 5 * RTOL
    # algebra: Q^T P reproduces triu(H) and Q = I - V T V^T is orthonormal on V's span
    Vd, Td, Pd = V.double().cpu(), T.double().cpu(), P.double()
    R = Pd - Vd @ (Td.transpose(1, 2) @ (Vd.transpose(1, 2) @ Pd))
    assert (R[:, :w] - torch.triu(H.double().cpu()[:, :w])).abs().max() < 1e-4 * Pd.abs().max()
    if r > w:
        assert R[:, w:].abs().max() < 1e-4 * Pd.abs().max()


@pytest.fixture(params=[0, 1, 2], ids=["ffma", "tcgen05", "ffma_tcgen05"])
def larfb_kind(request):
    old = _lib.get_config("larfb_kind")
    _lib.set_config("larfb_kind", request.param)
    yield request.param
    _lib.set_config("larfb_kind", old)


@pytest.mark.parametrize("r,k,c", [(64, 32, 64), (64, 32, 1), (100, 32, 36), (512, 32, 480),
                                   (4096, 32, 200), (33, 32, 4), (50, 8, 13), (129, 31, 70),
                                   (300, 1, 3), (129, 32, 260), (1000, 32, 132)])
def test_larfb_kernel_matches_fp64(r, k, c, larfb_kind):
    g = torch.Generator().manual_seed(r * 7 + k + c)
    b = 3
    Vfull = torch.randn(b, r, k, generator=g)
    Vexp = torch.tril(Vfull, -1) + torch.eye(r, k)
    T = torch.triu(torch.randn(b, k, k, generator=g)) * 0.5
    C = torch.randn(b, r, c, generator=g)
    want = oracle.larfb(Vexp.numpy(), T.numpy(), C.numpy(), f64=True)
    # V is passed with garbage on and above the diagonal: only the strict lower part is read
    Cd = C.to(DEV)
    api.larfb(Vfull.to(DEV), T.to(DEV), Cd)
    # FFMA: FP32 rounding. Tensor cores in 3xTF32: each product carries ~2^-21
    # relative error (the dropped lo*lo term) instead of 2^-24.
    tol = 1e-5 if larfb_kind == 0 else 4e-5
    assert _rel(Cd, want) < tol


@pytest.mark.parametrize("r,c", [(64, 4), (65, 64), (100, 36), (512, 448), (1000, 132),
                                 (4096, 64), (2049, 200)])
def test_larfb_two_level_block_matches_fp64(r, c):
    # k = 64: the two-level block (two panels' reflectors in one update)
    g = torch.Generator().manual_seed(r + 3 * c)
    b, k = 3, 64
    Vfull = torch.randn(b, r, k, generator=g)
    Vexp = torch.tril(Vfull, -1) + torch.eye(r, k)
    T = torch.triu(torch.randn(b, k, k, generator=g)) * 0.25
    C = torch.randn(b, r, c, generator=g)
    want = oracle.larfb(Vexp.numpy(), T.numpy(), C.numpy(), f64=True)
    Cd = C.to(DEV)
    api.larfb(Vfull.to(DEV), T.to(DEV), Cd)
    assert _rel(Cd, want) < 1e-5


def test_larfb_two_level_block_needs_aligned_operands():
    V = torch.randn(2, 100, 64, device=DEV)
    T = torch.randn(2, 64, 64, device=DEV)
    C = torch.randn(2, 100, 6, device=DEV)  # c % 4 != 0
    with pytest.raises(_lib.QRBError):
        api.larfb(V, T, C)


def test_larfb_strided_views_inside_a_matrix(larfb_kind):
    # V and C as views into one packed matrix, as the blocked driver uses them
    g = torch.Generator().manual_seed(9)
    n, j0 = 200, 64
    Hm = torch.randn(2, n, n, generator=g)
    V = Hm[:, j0:, j0:j0 + 32]
    C = Hm[:, j0:, j0 + 32:]
    T = torch.triu(torch.randn(2, 32, 32, generator=g)) * 0.3
    Vexp = torch.tril(V, -1) + torch.eye(n - j0, 32)
    want = oracle.larfb(Vexp.numpy(), T.numpy(), C.numpy(), f64=True)
    Hd = Hm.to(DEV)
    api.larfb(Hd[:, j0:, j0:j0 + 32], T.to(DEV), Hd[:, j0:, j0 + 32:])
    got = Hd[:, j0:, j0 + 32:].cpu().numpy()
    assert np.abs(got - want).max() / np.abs(want).max() < 1e-5
    # everything outside C untouched
    mask = torch.ones(2, n, n, dtype=torch.bool)
    mask[:, j0:, j0 + 32:] = False
    assert torch.equal(Hd.cpu()[mask], Hm[mask])


@pytest.fixture
def blocked_route():
    """Run n <= 128 through the blocked panel route instead of the fused CTA kernel."""
    old = _lib.get_config("mid_fused")
    _lib.set_config("mid_fused", 0)
    yield
    _lib.set_config("mid_fused", old)


def test_launch_counter_counts_kernels(blocked_route):
    A = torch.randn(4, 96, 96, device=DEV)
    torch.cuda.synchronize()
    groups = _lib.get_config("groups")
    try:
        # (setting, groups used): 0 = automatic (2 below n = 1024); at most batch / 2
        for g, used in ((1, 1), (2, 2), (0, 2), (4, 2)):
            _lib.set_config("groups", g)
            _lib.set_config("launches", 0)
            H, tau = api.geqrf(A)
            torch.cuda.synchronize()
            # per batch group: 3 panels + 2 trailing updates
            assert _lib.get_config("launches") == 5 * used
            assert checker.check(A, H, tau).passed
    finally:
        _lib.set_config("groups", groups)


@pytest.mark.parametrize("n", [96, 200, 512, 1000])
def test_geqrf_same_with_ffma_and_tensor_core_updates(n, blocked_route):
    A = torch.randn(4, n, n, generator=torch.Generator().manual_seed(n)).to(DEV)
    old = _lib.get_config("larfb_kind")
    try:
        out = {}
        for kind in (0, 1, 2, 3):
            _lib.set_config("larfb_kind", kind)
            out[kind] = api.geqrf(A)
            torch.cuda.synchronize()
            assert checker.check(A, *out[kind]).passed, kind
    finally:
        _lib.set_config("larfb_kind", old)
    for kind in (1, 2, 3):
        par = checker.parity(out[kind][0].cpu(), out[kind][1].cpu(), out[0][0].cpu(),
                             out[0][1].cpu())
        assert par.ok(RTOL), (kind, par)
    assert _lib.get_config("device_error") == 0


@pytest.mark.parametrize("n", [33, 40, 47, 63, 64, 65, 80, 96, 100, 127, 128])
@pytest.mark.parametrize("b", [1, 3, 200, 593])
def test_fused_cta_kernel_mid_n(n, b):
    # 32 < n <= 128: one launch of the CTA-per-matrix kernel; parity with the
    # FP64 oracle, FP64 gates, and agreement with the blocked route.
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(b * 131 + n))
    Ad = A.to(DEV)
    _lib.set_config("launches", 0)
    H, tau = api.geqrf(Ad)
    torch.cuda.synchronize()
    fused = n <= 64 or n > 96 or b <= 592  # the dispatch rule for the CTA kernel
    assert (_lib.get_config("launches") == 1) == fused
    k = min(b, 16)
    Ho, to = oracle.geqr2(A[:k].numpy(), f64=True)
    assert checker.parity(H[:k].cpu(), tau[:k].cpu(), Ho, to).ok(RTOL), n
    assert checker.check(A[:k], H[:k].cpu(), tau[:k].cpu()).passed
    assert (tau[:, -1] == 0).all()
    old = _lib.get_config("mid_fused")
    try:
        _lib.set_config("mid_fused", 0)
        Hb, tb = api.geqrf(Ad)
        torch.cuda.synchronize()
    finally:
        _lib.set_config("mid_fused", old)
    # both routes against FP64 at the parity bar; with each other (two FP32
    # algorithms, every matrix of the batch) H within 1e-4, tau within 2e-4
    assert checker.parity(Hb[:k].cpu(), tb[:k].cpu(), Ho, to).ok(RTOL), n
    assert _rel(H, Hb.cpu().numpy()) < RTOL
    assert (tau - tb).abs().max() < 2 * RTOL


def test_fused_cta_kernel_in_place_and_strided():
    n = 72
    A = torch.randn(6, n, n, generator=torch.Generator().manual_seed(3)).to(DEV)
    H, tau = api.geqrf(A)
    big = torch.zeros(6, n, n + 8, device=DEV)
    big[:, :, :n] = A
    H2, tau2 = api.geqrf(big[:, :, :n])  # row stride n + 8
    M = A.clone()
    t3 = api.geqrf_out(M, M, torch.empty(6, n, device=DEV))[1]
    torch.cuda.synchronize()
    assert torch.equal(H, H2) and torch.equal(tau, tau2)
    assert torch.equal(M, H) and torch.equal(t3, tau)


@pytest.mark.parametrize("n", [129, 200, 512, 1000, 1100])
@pytest.mark.parametrize("groups", [1, 2])
def test_panel_lookahead_gives_identical_results(n, groups):
    # the look-ahead only reorders independent column updates across two
    # streams: H and tau must be bit-identical; a one-factor workspace runs
    # without it.
    b = 4
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(n + groups)).to(DEV)
    old = {k: _lib.get_config(k) for k in ("lookahead", "groups", "larfb_kind")}
    outs = {}
    try:
        _lib.set_config("groups", groups)
        _lib.set_config("larfb_kind", 0)  # the FFMA update, which a one-factor workspace also runs
        for la in (0, 1):
            _lib.set_config("lookahead", la)
            outs[la] = api.geqrf(A)
        torch.cuda.synchronize()
        # minimal workspace: one factor per matrix, look-ahead requested but unavailable
        ws_one = b * 32 * 32 * 4
        ws = torch.empty(ws_one, dtype=torch.uint8, device=DEV)
        H = torch.empty_like(A)
        tau = torch.empty(b, n, device=DEV)
        rc = _lib.lib().qrb_geqrf_f32(A.data_ptr(), n * n, n, H.data_ptr(), tau.data_ptr(), b, n,
                                      ws.data_ptr(), ws_one, torch.cuda.current_stream().cuda_stream)
        _lib.check(rc)
        torch.cuda.synchronize()
    finally:
        for k, v in old.items():
            _lib.set_config(k, v)
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(H, outs[0][0]) and torch.equal(tau, outs[0][1])
    assert checker.check(A.cpu(), outs[1][0].cpu(), outs[1][1].cpu()).passed


@pytest.mark.parametrize("n", [129, 130, 200, 256, 512, 1000, 1100])
@pytest.mark.parametrize("groups", [1, 2])
def test_two_level_blocking_matches_one_level(n, groups):
    # Two panels combined into one 64-reflector update: the same factorization
    # up to FP32 rounding (different summation order), FP64 gates passing.
    # n % 4 != 0 takes the aligned-operand fallback (two 32-wide updates).
    b = 4
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(2 * n + groups)).to(DEV)
    old = {k: _lib.get_config(k) for k in ("two_level", "groups", "mid_fused", "larfb_kind")}
    outs = {}
    try:
        _lib.set_config("groups", groups)
        _lib.set_config("mid_fused", 0)
        _lib.set_config("larfb_kind", 0)  # two-level blocking runs on the FFMA update
        for tl in (0, 1):
            _lib.set_config("two_level", tl)
            outs[tl] = api.geqrf(A)
            torch.cuda.synchronize()
        # a two-factor workspace cannot hold the 64 x 64 factor: one-level route
        ws_two = 2 * b * 32 * 32 * 4
        ws = torch.empty(ws_two, dtype=torch.uint8, device=DEV)
        H = torch.empty_like(A)
        tau = torch.empty(b, n, device=DEV)
        rc = _lib.lib().qrb_geqrf_f32(A.data_ptr(), n * n, n, H.data_ptr(), tau.data_ptr(), b, n,
                                      ws.data_ptr(), ws_two, torch.cuda.current_stream().cuda_stream)
        _lib.check(rc)
        torch.cuda.synchronize()
    finally:
        for k, v in old.items():
            _lib.set_config(k, v)
    assert checker.check(A.cpu(), outs[1][0].cpu(), outs[1][1].cpu()).passed
    # each route within 1e-4 of FP64 LAPACK; with each other H within 1e-4,
    # tau within 2e-4 (two summation orders)
    H64, t64 = torch.geqrf(A.cpu().double())
    for tl in (0, 1):
        pf = checker.parity(outs[tl][0].cpu(), outs[tl][1].cpu(), H64.float(), t64.float())
        assert pf.ok(RTOL), (tl, pf)
    par = checker.parity(outs[1][0].cpu(), outs[1][1].cpu(), outs[0][0].cpu(), outs[0][1].cpu())
    assert par.h_rel < RTOL and par.col_rel < RTOL and par.tau_rel < 2 * RTOL, par
    assert torch.equal(H, outs[0][0]) and torch.equal(tau, outs[0][1])


def test_two_level_blocking_against_lapack():
    # elementwise against CPU LAPACK geqrf on a well-conditioned problem
    # (column scales 1 .. 1e-2, the benchmark's cond 1e2 family)
    from gpumode_qr_b200 import inputs
    prob = inputs.make_benchmark_problem({"batch": 3, "n": 640, "cond": 2})
    A = prob.tensor
    old = _lib.get_config("two_level")
    try:
        _lib.set_config("two_level", 1)
        H, tau = api.geqrf(A.to(DEV))
        torch.cuda.synchronize()
    finally:
        _lib.set_config("two_level", old)
    Hr, tr = torch.geqrf(A)
    par = checker.parity(H.cpu(), tau.cpu(), Hr, tr)
    assert par.ok(1e-3), par


@pytest.mark.parametrize("rpt", [1, 2, 4])
@pytest.mark.parametrize("n", [160, 512, 1100, 2100])
def test_panel_rows_per_thread_variants(rpt, n):
    # rows per thread of the panel kernel changes the reduction grouping only
    b = 2
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(n + rpt)).to(DEV)
    H0, t0 = api.geqrf(A)
    old = _lib.get_config("panel_rpt")
    try:
        _lib.set_config("panel_rpt", rpt)
        H, tau = api.geqrf(A)
        torch.cuda.synchronize()
    finally:
        _lib.set_config("panel_rpt", old)
    assert checker.check(A.cpu(), H.cpu(), tau.cpu()).passed
    # a Gaussian matrix of n = 2100 has cond ~ 1e4: the trailing tau move by a
    # few 1e-4 under a different summation order; the north-star bar is 1e-3
    assert checker.parity(H.cpu(), tau.cpu(), H0.cpu(), t0.cpu()).ok(1e-3)
