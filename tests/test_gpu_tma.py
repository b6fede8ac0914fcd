"""The TMA-fed tcgen05 (3xTF32) trailing update inside the blocked route.

Parity: every factorization passes the FP64 gates; H and tau agree with the
FP64 oracle within 1e-4 of max|H|, the bar of the other kernel tests, and with
CPU LAPACK within the north-star 1e-3; against FP64 LAPACK the tensor-core
route stays within 1e-4 (H) as the FFMA route does. The look-ahead split and
the batch groups leave the bits unchanged, the route falls back to FFMA where
the update cannot run (n % 4 != 0, too little workspace), and the bounded
device-side waits time out into an error status, not a hang.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gpumode_qr_b200 import _lib, api, checker

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
RTOL = 1e-4


def _hooks(**kv):
    old = {k: _lib.get_config(k) for k in kv}
    for k, v in kv.items():
        _lib.set_config(k, v)
    return old


def _restore(old):
    for k, v in old.items():
        _lib.set_config(k, v)


@pytest.mark.parametrize("b,n", [(3, 160), (2, 256), (5, 300), (3, 512), (2, 1024)])
def test_tma_route_matches_the_fp64_oracle(b, n):
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(7 * n + b))
    assert "tcgen05_tma" in api.route(b, n)
    H, tau = api.geqrf(A.to(DEV))
    torch.cuda.synchronize()
    assert checker.check(A, H.cpu(), tau.cpu()).passed
    k = min(b, 2)
    Ho, to = oracle.geqr2(A[:k].numpy(), f64=True)
    par = checker.parity(H[:k].cpu(), tau[:k].cpu(), Ho, to)
    assert par.ok(RTOL), par
    assert (tau[:, -1] == 0).all()
    assert _lib.get_config("device_error") == 0


@pytest.mark.parametrize("n", [132, 256, 384, 640, 1000, 1028, 2048])
def test_tma_route_agrees_with_ffma(n):
    # Both FP32 routes against FP64 LAPACK on the same inputs: the tensor-core
    # route stays within 1e-4 of max|H| (and tau within 5e-4) of FP64, as
    # FFMA does; the two agree with each other in H within 1e-4. tau of the
    # last columns is the most rounding-sensitive output at large n (FFMA
    # itself sits ~1e-4 from LAPACK there), so their mutual tau bar is the
    # north-star 1e-3.
    b = 4 if n <= 1028 else 2
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(n)).to(DEV)
    old = _hooks(larfb_kind=0)
    try:
        Hf, tf = api.geqrf(A)
        _lib.set_config("larfb_kind", 3)
        Ht, tt = api.geqrf(A)
        torch.cuda.synchronize()
    finally:
        _restore(old)
    assert checker.check(A, Ht, tt).passed
    H64, t64 = torch.geqrf(A.cpu().double())
    pf = checker.parity(Hf.cpu(), tf.cpu(), H64.float(), t64.float())
    pt = checker.parity(Ht.cpu(), tt.cpu(), H64.float(), t64.float())
    print(f"n={n}: tensor-core route vs FP64 {pt}; FFMA vs FP64 {pf}")
    assert pf.h_rel < RTOL and pt.h_rel < RTOL and pt.col_rel < RTOL, (n, pt, pf)
    assert pt.tau_rel < 5e-4, (n, pt, pf)
    par = checker.parity(Ht.cpu(), tt.cpu(), Hf.cpu(), tf.cpu())
    assert par.h_rel < RTOL and par.col_rel < RTOL and par.tau_rel < 1e-3, (n, par)


def test_tma_route_matches_lapack_on_config_3_shape():
    # config 3's matrix type (Haar, cond 1e2) on a slice of its batch
    from gpumode_qr_b200 import inputs

    cfg = inputs.config(3)
    A = inputs.make_config_input(cfg, 16)
    H, tau = api.geqrf(A.to(DEV))
    Hl, tl = oracle.lapack_geqrf(A)
    par = checker.parity(H.cpu(), tau.cpu(), torch.from_numpy(Hl), torch.from_numpy(tl))
    assert par.ok(), par
    assert checker.check(A, H.cpu(), tau.cpu()).passed


def test_tma_groups_leave_bits_unchanged_and_lookahead_agrees():
    # the batch groups change no bits, with or without the look-ahead; the
    # look-ahead updates the next panel's columns with the narrow FFMA kernel
    # instead of the tensor-core one, so it agrees within the parity bar
    A = torch.randn(8, 512, 512, generator=torch.Generator().manual_seed(3)).to(DEV)
    outs = {}
    old = _hooks(lookahead=0, groups=1)
    try:
        for la, g in ((0, 1), (1, 1), (0, 4), (1, 4), (1, 2), (0, 2)):
            _lib.set_config("lookahead", la)
            _lib.set_config("groups", g)
            assert "tcgen05_tma" in api.route(8, 512)
            outs[la, g] = api.geqrf(A)
        torch.cuda.synchronize()
    finally:
        _restore(old)
    for (la, g), (H, tau) in outs.items():
        H0, t0 = outs[la, 1]
        assert torch.equal(H, H0) and torch.equal(tau, t0), (la, g)
    par = checker.parity(outs[1, 1][0].cpu(), outs[1, 1][1].cpu(), outs[0, 1][0].cpu(),
                         outs[0, 1][1].cpu())
    assert par.h_rel < RTOL and par.col_rel < RTOL and par.tau_rel < 1e-3, par


def test_tma_route_in_place_and_strided_inputs():
    n = 256
    g = torch.Generator().manual_seed(11)
    A = torch.randn(3, n, n, generator=g).to(DEV)
    H_ref, t_ref = api.geqrf(A)
    # in place: H is A itself
    Ai = A.clone()
    tau = torch.empty(3, n, device=DEV)
    api.geqrf_out(Ai, Ai, tau)
    assert torch.equal(Ai, H_ref) and torch.equal(tau, t_ref)
    # A viewed with a larger batch stride (the copy into H runs per matrix)
    big = torch.zeros(3, n + 8, n, device=DEV)
    big[:, :n] = A
    H2, t2 = api.geqrf(big[:, :n])
    assert torch.equal(H2, H_ref) and torch.equal(t2, t_ref)
    # a row stride larger than n
    wide = torch.zeros(3, n, n + 4, device=DEV)
    wide[:, :, :n] = A
    H3, t3 = api.geqrf(wide[:, :, :n])
    assert torch.equal(H3, H_ref) and torch.equal(t3, t_ref)


@pytest.mark.parametrize("n", [130, 258])
def test_rows_not_16_byte_aligned_use_ffma(n):
    assert "ffma" in api.route(3, n)
    A = torch.randn(3, n, n, generator=torch.Generator().manual_seed(n))
    H, tau = api.geqrf(A.to(DEV))
    assert checker.check(A, H.cpu(), tau.cpu()).passed


def test_too_little_workspace_uses_ffma():
    b, n = 2, 256
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(5)).to(DEV)
    H_ref, t_ref = api.geqrf(A)
    small = 4 * b * 32 * 32 * 4  # the T factors only
    assert "ffma" in api.route(b, n, small)
    H = torch.empty_like(A)
    tau = torch.empty(b, n, device=DEV)
    ws = torch.empty(small, dtype=torch.uint8, device=DEV)
    _lib.check(_lib.lib().qrb_geqrf_f32(A.data_ptr(), A.stride(0), A.stride(1), H.data_ptr(),
                                        tau.data_ptr(), b, n, ws.data_ptr(), small,
                                        torch.cuda.current_stream().cuda_stream))
    par = checker.parity(H.cpu(), tau.cpu(), H_ref.cpu(), t_ref.cpu())
    assert par.ok(RTOL), par


def test_tma_many_tiles_per_cta():
    # more tiles than SMs: each persistent CTA walks several (matrix, column
    # tile) items, including the column-limited tiles of the look-ahead
    b, n = 400, 512  # 1600 tiles in the first update, over at most 148 CTAs
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(12))
    old = _hooks(lookahead=1, groups=1)
    try:
        H, tau = api.geqrf(A.to(DEV))
        torch.cuda.synchronize()
    finally:
        _restore(old)
    assert checker.check(A[:4], H[:4].cpu(), tau[:4].cpu()).passed
    Hl, tl = oracle.lapack_geqrf(A[:4])
    par = checker.parity(H[:4].cpu(), tau[:4].cpu(), torch.from_numpy(Hl), torch.from_numpy(tl))
    assert par.ok(), par
    assert _lib.get_config("device_error") == 0


def test_bounded_wait_probe_times_out_into_the_error_flag():
    _lib.set_config("device_error", 0)
    _lib.set_config("wait_probe", 2_000_000)  # ~1 ms; nothing completes the barrier
    assert _lib.get_config("device_error") == 1
    _lib.set_config("device_error", 0)
    A = torch.randn(2, 256, 256, generator=torch.Generator().manual_seed(1))
    H, tau = api.geqrf(A.to(DEV))  # the context is still usable
    assert checker.check(A, H.cpu(), tau.cpu()).passed


def test_tma_update_abandons_a_call_whose_waits_run_out():
    # the update withholds its MMAs: its bounded waits run out, it sets the
    # error flag, waits for its own copies, frees TMEM and returns; with
    # sync_check the call reports QRB_ERR_DEVICE_WAIT, and the next call works
    A = torch.randn(2, 256, 256, generator=torch.Generator().manual_seed(2)).to(DEV)
    _lib.set_config("device_error", 0)
    old = _hooks(wait_limit=2_000_000, test_skip_mma=1, sync_check=1)
    try:
        with pytest.raises(_lib.QRBError) as exc:
            api.geqrf(A)
        assert exc.value.status == 7
    finally:
        _restore(old)
    assert _lib.get_config("device_error") == 1
    _lib.set_config("device_error", 0)
    H, tau = api.geqrf(A)
    torch.cuda.synchronize()
    assert checker.check(A, H, tau).passed
    assert _lib.get_config("device_error") == 0


def test_tma_route_nan_input_propagates():
    A = torch.randn(2, 256, 256, generator=torch.Generator().manual_seed(4))
    A[1, 100, 7] = float("nan")
    H, tau = api.geqrf(A.to(DEV))
    torch.cuda.synchronize()
    assert torch.isfinite(H[0]).all()
    assert not torch.isfinite(H[1]).all()
    assert np.isfinite(tau[0].cpu().numpy()).all()
    assert _lib.get_config("device_error") == 0


@pytest.mark.parametrize("b,n,groups", [(3, 160, 1), (4, 300, 2), (3, 512, 1), (8, 640, 4),
                                        (2, 1028, 1), (2, 2048, 2)])
def test_two_level_tensor_core_route(b, n, groups):
    # two 32-column panels per 64-reflector block (T 64 x 64 from the panels'
    # factors and their cross block), the 64-reflector update on the tensor
    # cores: FP64 gates, and within 1e-4 of FP64 LAPACK like the one-level route
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(17 * n + b))
    old = _hooks(two_level=1, lookahead=0, groups=groups)
    try:
        route = api.route(b, n)
        H, tau = api.geqrf(A.to(DEV))
        torch.cuda.synchronize()
    finally:
        _restore(old)
    assert "tcgen05_tma" in route and "two_level" in route and "lookahead" not in route, route
    assert checker.check(A, H.cpu(), tau.cpu()).passed
    H64, t64 = torch.geqrf(A.double())
    par = checker.parity(H.cpu(), tau.cpu(), H64.float(), t64.float())
    assert par.h_rel < RTOL and par.col_rel < RTOL and par.tau_rel < 5e-4, par
    assert _lib.get_config("device_error") == 0


def test_narrow_update_agrees_with_the_tma_kernel():
    # the next panel's 32 columns by the narrow cluster kernel (default) or by
    # the TMA-fed kernel: both within 1e-4 of each other and of FP64 LAPACK
    b, n = 4, 768
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(21)).to(DEV)
    old = _hooks(narrow_update=1, lookahead=1)
    try:
        Hn, tn = api.geqrf(A)
        _lib.set_config("narrow_update", 0)
        Ht, tt = api.geqrf(A)
        torch.cuda.synchronize()
    finally:
        _restore(old)
    H64, t64 = torch.geqrf(A.cpu().double())
    for H, tau in ((Hn, tn), (Ht, tt)):
        par = checker.parity(H.cpu(), tau.cpu(), H64.float(), t64.float())
        assert par.h_rel < RTOL and par.col_rel < RTOL and par.tau_rel < 5e-4, par
    par = checker.parity(Hn.cpu(), tn.cpu(), Ht.cpu(), tt.cpu())
    assert par.h_rel < RTOL and par.col_rel < RTOL, par
    assert _lib.get_config("device_error") == 0


def test_tall_panels_stage_the_narrow_update_in_chunks():
    # n = 4160: up to 4128 rows for the narrow update, 544 per cluster rank,
    # staged in two chunks (512 rows at most per chunk)
    n = 4160
    A = torch.randn(1, n, n, generator=torch.Generator().manual_seed(5)).to(DEV)
    assert "tcgen05_tma" in api.route(1, n)
    old = _hooks(lookahead=1)
    try:
        H, tau = api.geqrf(A)
        _lib.set_config("larfb_kind", 0)
        Hf, tf = api.geqrf(A)
        torch.cuda.synchronize()
    finally:
        _lib.set_config("larfb_kind", -1)
        _restore(old)
    assert checker.check(A, H, tau).passed
    par = checker.parity(H.cpu(), tau.cpu(), Hf.cpu(), tf.cpu())
    assert par.h_rel < RTOL and par.col_rel < RTOL and par.tau_rel < 1e-3, par
    assert _lib.get_config("device_error") == 0


@pytest.mark.parametrize("depth", [1, 2])
@pytest.mark.parametrize("b,n,groups", [(3, 160, 1), (2, 196, 1), (4, 300, 2), (3, 512, 1),
                                        (8, 640, 4), (2, 1028, 1), (2, 2048, 2)])
def test_two_level_lookahead_route(b, n, groups, depth):
    # two-level blocking with the look-ahead: per 64 columns panel 1, the
    # narrow update of the next 64 columns, panel 2, the narrow update of the
    # next 32; t64 and the 64-reflector update of the rest on the other
    # stream. FP64 gates, within 1e-4 of FP64 LAPACK, and the batch groups
    # leave the bits unchanged
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(29 * n + b))
    # depth 2: the priority stream also applies both panels' reflectors to the
    # next block's second 32 columns, and the wide update starts at j0 + 128
    old = _hooks(two_level=1, lookahead=1, groups=groups, lookahead_depth=depth)
    try:
        route = api.route(b, n)
        H, tau = api.geqrf(A.to(DEV))
        _lib.set_config("groups", 1)
        H1, t1 = api.geqrf(A.to(DEV))
        torch.cuda.synchronize()
    finally:
        _restore(old)
    assert "two_level" in route and "lookahead" in route and "tcgen05_tma" in route, route
    assert ("depth2" in route) == (depth == 2), route
    assert torch.equal(H, H1) and torch.equal(tau, t1)
    assert checker.check(A, H.cpu(), tau.cpu()).passed
    H64, t64 = torch.geqrf(A.double())
    par = checker.parity(H.cpu(), tau.cpu(), H64.float(), t64.float())
    assert par.h_rel < RTOL and par.col_rel < RTOL and par.tau_rel < 5e-4, par
    assert _lib.get_config("device_error") == 0


@pytest.mark.parametrize("b,n,two_level,la,groups", [(3, 160, 0, 0, 1), (5, 300, 0, 0, 1),
                                                     (8, 512, 0, 0, 4), (2, 1024, 1, 1, 1),
                                                     (4, 1028, 1, 0, 2), (1, 2048, 1, 1, 1)])
def test_row_split_tiles(b, n, two_level, la, groups):
    # every update over more than 128 rows sums V^T C in two row halves: one
    # CTA per tile keeping both, or a 2-CTA cluster per tile (one half each,
    # the partials added through distributed shared memory) give the same
    # bits, as do the batch groups; FP64 gates, within 1e-4 of FP64 LAPACK and
    # of the update without halves
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(31 * n + b)).to(DEV)
    old = _hooks(tma_split_rows=129, tma_pair=2, two_level=two_level, lookahead=la,
                 groups=groups)
    try:
        assert "tcgen05_tma" in api.route(b, n)
        Hs, ts = api.geqrf(A)
        _lib.set_config("tma_pair", 1)
        Hp, tp = api.geqrf(A)
        _lib.set_config("tma_pair", 0)
        _lib.set_config("groups", 1)
        Hs1, ts1 = api.geqrf(A)
        _lib.set_config("tma_split_rows", 0)
        Hu, tu = api.geqrf(A)
        torch.cuda.synchronize()
    finally:
        _restore(old)
    assert torch.equal(Hs, Hp) and torch.equal(ts, tp)
    assert torch.equal(Hs, Hs1) and torch.equal(ts, ts1)
    assert checker.check(A, Hs, ts).passed
    H64, t64 = torch.geqrf(A.cpu().double())
    par = checker.parity(Hs.cpu(), ts.cpu(), H64.float(), t64.float())
    assert par.h_rel < RTOL and par.col_rel < RTOL and par.tau_rel < 5e-4, par
    par = checker.parity(Hs.cpu(), ts.cpu(), Hu.cpu(), tu.cpu())
    assert par.h_rel < RTOL and par.col_rel < RTOL and par.tau_rel < 2 * RTOL, par
    assert _lib.get_config("device_error") == 0


def test_row_split_update_abandons_a_call_whose_waits_run_out():
    # as the unsplit case: both CTAs of each cluster time out (the one whose
    # MMAs are withheld, and its peer waiting for the partial W), set the error
    # flag, meet at the closing cluster barrier and free their TMEM
    A = torch.randn(2, 256, 256, generator=torch.Generator().manual_seed(2)).to(DEV)
    _lib.set_config("device_error", 0)
    old = _hooks(wait_limit=2_000_000, test_skip_mma=1, sync_check=1, tma_split_rows=129,
                 tma_pair=2)
    try:
        with pytest.raises(_lib.QRBError) as exc:
            api.geqrf(A)
        assert exc.value.status == 7
    finally:
        _restore(old)
    assert _lib.get_config("device_error") == 1
    _lib.set_config("device_error", 0)
    old = _hooks(tma_split_rows=129, tma_pair=2)
    try:
        H, tau = api.geqrf(A)
        torch.cuda.synchronize()
    finally:
        _restore(old)
    assert checker.check(A, H, tau).passed
    assert _lib.get_config("device_error") == 0


@pytest.mark.parametrize("b,n,groups", [(3, 160, 1), (5, 300, 1), (2, 1000, 1), (8, 640, 4),
                                        (320, 512, 2)])
def test_two_ctas_per_sm_give_the_same_bits(b, n, groups):
    # the 32-reflector update with two CTAs per SM (4 worker warps, 2 pass-1
    # stages, one pass-2 accumulator, the epilogue in two column halves) runs
    # the same FP32 operations in the same order as one CTA per SM
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(37 * n + b)).to(DEV)
    old = _hooks(tma_dual=2, two_level=0, lookahead=0, groups=groups)
    try:
        assert "tcgen05_tma" in api.route(b, n)
        Hd, td = api.geqrf(A)
        _lib.set_config("tma_dual", 1)
        H1, t1 = api.geqrf(A)
        _lib.set_config("tma_dual", 0)
        Ha, ta = api.geqrf(A)
        torch.cuda.synchronize()
    finally:
        _restore(old)
    assert torch.equal(Hd, H1) and torch.equal(td, t1)
    assert torch.equal(Ha, H1) and torch.equal(ta, t1)
    k = min(b, 8)
    assert checker.check(A[:k], Hd[:k], td[:k]).passed
    H64, t64 = torch.geqrf(A[:k].cpu().double())
    par = checker.parity(Hd[:k].cpu(), td[:k].cpu(), H64.float(), t64.float())
    assert par.h_rel < RTOL and par.col_rel < RTOL and par.tau_rel < 5e-4, par
    assert _lib.get_config("device_error") == 0


def test_two_ctas_per_sm_abandon_a_call_whose_waits_run_out():
    A = torch.randn(2, 256, 256, generator=torch.Generator().manual_seed(2)).to(DEV)
    _lib.set_config("device_error", 0)
    old = _hooks(wait_limit=2_000_000, test_skip_mma=1, sync_check=1, tma_dual=2,
                 two_level=0, lookahead=0)
    try:
        with pytest.raises(_lib.QRBError) as exc:
            api.geqrf(A)
        assert exc.value.status == 7
    finally:
        _restore(old)
    assert _lib.get_config("device_error") == 1
    _lib.set_config("device_error", 0)
    old = _hooks(tma_dual=2, two_level=0, lookahead=0)
    try:
        H, tau = api.geqrf(A)
        torch.cuda.synchronize()
    finally:
        _restore(old)
    assert checker.check(A, H, tau).passed
    assert _lib.get_config("device_error") == 0
