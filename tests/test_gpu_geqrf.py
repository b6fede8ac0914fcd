"""Full-path parity and gates of qrb_geqrf_f32 (through the C ABI via the
Python API) on the GPU.

Bars: every factorization passes the reference's FP64 gates (factor residual
<= 20 n eps32, orthogonality <= 100 n eps32); for well-conditioned inputs H and
tau agree with the oracle within 1e-4 relative (PARITY_RTOL below; the
north-star bar is 1e-3) — rank-deficient inputs have non-unique reflectors
and are gated only.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch
from conftest import golden_cases

import oracle
from gpumode_qr_b200 import _lib, api, checker, inputs

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
PARITY_RTOL = 1e-4


def _gpu_qr(A_cpu):
    H, tau = api.geqrf(A_cpu.to(DEV))
    torch.cuda.synchronize()
    return H.cpu(), tau.cpu()


@pytest.mark.parametrize("n", [1, 2, 3, 7, 16, 31, 32, 33, 40, 63, 64, 65, 96, 100, 127, 128, 129,
                               160, 176, 200, 255, 256, 257, 300, 352, 511, 512, 513, 700])
def test_geqrf_matches_oracle(n):
    b = 5 if n <= 256 else 2
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(1000 + n))
    H, tau = _gpu_qr(A)
    Ho, to = oracle.blocked_geqrf(A.numpy(), 32, f64=True)
    par = checker.parity(H, tau, Ho, to)
    assert par.ok(PARITY_RTOL), (n, par)
    gate = checker.check(A, H, tau)
    assert gate.passed, (n, gate.as_dict())


def test_geqrf_matches_reference_driver_and_champion(ref_blocked):
    for case in golden_cases(ref_blocked):
        A = torch.from_numpy(ref_blocked[f"{case}_A"])
        H, tau = _gpu_qr(A)
        par = checker.parity(H, tau, ref_blocked[f"{case}_H"], ref_blocked[f"{case}_tau"])
        assert par.ok(PARITY_RTOL), (case, par)


def test_geqrf_matches_lapack_goldens(lapack_golden):
    for case in golden_cases(lapack_golden):
        A = torch.from_numpy(lapack_golden[f"{case}_A"])
        H, tau = _gpu_qr(A)
        gate = checker.check(A, H, tau)
        assert gate.passed, (case, gate.as_dict())
        if "rank_deficient" in case or "collinear" in case:
            continue
        par = checker.parity(H, tau, lapack_golden[f"{case}_H"], lapack_golden[f"{case}_tau"])
        assert par.ok(PARITY_RTOL), (case, par)


@pytest.mark.parametrize("n", [32, 176, 512])
def test_stress_suite(n):
    # the reference's 27-case --stress suite (scripts/run_baseline.py:66-82)
    for prob in inputs.stress_cases(n, batch=4):
        H, tau = _gpu_qr(prob.tensor)
        gate = checker.check(prob.tensor, H, tau)
        assert gate.passed, (prob.name, gate.as_dict())
        assert torch.isfinite(H).all() and torch.isfinite(tau).all()


@pytest.mark.parametrize("shape", inputs.BENCHMARK_SHAPES, ids=lambda s: f"b{s['batch']}_n{s['n']}")
def test_reference_benchmark_shapes(shape):
    prob = inputs.make_benchmark_problem(shape)
    A = prob.tensor
    if A.shape[-1] >= 2048:
        A = A[:1]  # one matrix is enough to gate the shape
    H, tau = _gpu_qr(A)
    gate = checker.check(A, H, tau)
    assert gate.passed, (prob.name, gate.as_dict())


def test_edge_cases():
    # empty batch / empty matrices
    H, tau = api.geqrf(torch.empty(0, 8, 8, device=DEV))
    assert H.shape == (0, 8, 8) and tau.shape == (0, 8)
    H, tau = api.geqrf(torch.empty(3, 0, 0, device=DEV))
    assert H.shape == (3, 0, 0) and tau.shape == (3, 0)
    # zero matrices: identity reflectors, H == 0, tau == 0
    for n in (5, 32, 70):
        H, tau = api.geqrf(torch.zeros(2, n, n, device=DEV))
        assert (H == 0).all() and (tau == 0).all()
    # identity: R = I with tau = 0 (nothing below the diagonal)
    for n in (8, 40):
        eye = torch.eye(n, device=DEV).expand(2, n, n).contiguous()
        H, tau = api.geqrf(eye)
        assert torch.equal(H, eye) and (tau == 0).all()
    # upper triangular input keeps R = A, tau = 0
    U = torch.triu(torch.randn(2, 50, 50, generator=torch.Generator().manual_seed(2)))
    H, tau = _gpu_qr(U)
    assert torch.equal(H, U) and (tau == 0).all()
    # a zero column in the middle
    Z = torch.randn(2, 48, 48, generator=torch.Generator().manual_seed(3))
    Z[:, :, 20] = 0
    H, tau = _gpu_qr(Z)
    assert checker.check(Z, H, tau).passed


def test_nan_input_propagates_without_hanging():
    for n in (16, 80):
        A = torch.randn(2, n, n, device=DEV)
        A[1, 3, 2] = float("nan")
        H, tau = api.geqrf(A)
        torch.cuda.synchronize()
        assert torch.isfinite(H[0]).all()  # the clean matrix is unaffected
        assert torch.isnan(H[1]).any()


def test_non_contiguous_and_batched_views():
    g = torch.Generator().manual_seed(4)
    base = torch.randn(6, 70, 70, generator=g)
    # transposed matrices (column stride != 1) and a strided batch slice
    for view in (base.transpose(1, 2), base[::2], base[:, :, :]):
        H, tau = _gpu_qr(view)
        Ho, to = oracle.geqr2(view.contiguous().numpy(), f64=True)
        assert checker.parity(H, tau, Ho, to).ok(PARITY_RTOL)
    # row-strided input consumed directly (no copy): a column sub-block
    wide = torch.randn(3, 64, 100, generator=g)
    A = wide[:, :, 10:74]
    H, tau = _gpu_qr(A)
    Ho, to = oracle.geqr2(A.contiguous().numpy(), f64=True)
    assert checker.parity(H, tau, Ho, to).ok(PARITY_RTOL)
    # extra leading batch dims
    A4 = torch.randn(2, 3, 40, 40, generator=g)
    H, tau = _gpu_qr(A4)
    assert H.shape == A4.shape and tau.shape == (2, 3, 40)
    Ho, to = oracle.geqr2(A4.reshape(6, 40, 40).numpy(), f64=True)
    assert checker.parity(H.reshape(6, 40, 40), tau.reshape(6, 40), Ho, to).ok(PARITY_RTOL)
    # the input is never modified
    A = torch.randn(2, 90, 90, device=DEV)
    keep = A.clone()
    api.geqrf(A)
    torch.cuda.synchronize()
    assert torch.equal(A, keep)


def test_in_place_mode_through_the_c_abi():
    g = torch.Generator().manual_seed(6)
    for n in (30, 130):
        A = torch.randn(3, n, n, generator=g)
        want_H, want_tau = _gpu_qr(A)
        Ad = A.to(DEV)
        tau = torch.empty(3, n, device=DEV)
        ws_n = api.workspace_bytes(3, n)
        ws = torch.empty(max(ws_n, 16), dtype=torch.uint8, device=DEV)
        rc = _lib.lib().qrb_geqrf_f32(Ad.data_ptr(), n * n, n, Ad.data_ptr(), tau.data_ptr(), 3, n,
                                      ws.data_ptr(), ws_n, torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.equal(Ad.cpu(), want_H) and torch.equal(tau.cpu(), want_tau)


def test_deterministic_and_stream_ordered():
    A = torch.randn(16, 200, 200, device=DEV)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        H1, t1 = api.geqrf(A)
        H2, t2 = api.geqrf(A)
    s.synchronize()
    assert torch.equal(H1, H2) and torch.equal(t1, t2)
    H3, t3 = api.geqrf(A)
    torch.cuda.synchronize()
    assert torch.equal(H1, H3)


def test_large_batch_grid_chunking():
    # more matrices than one grid dimension of the trailing update holds
    b, n = 65537, 36
    A = torch.randn(b, n, n, device=DEV)
    H, tau = api.geqrf(A)
    idx = torch.tensor([0, 1, 65535, 65536])
    Ho, to = oracle.geqr2(A[idx].cpu().numpy(), f64=True)
    assert checker.parity(H[idx].cpu(), tau[idx].cpu(), Ho, to).ok(PARITY_RTOL)


def test_max_n_and_beyond():
    n = api.max_n()
    A = torch.randn(1, n, n, device=DEV)
    H, tau = api.geqrf(A)
    gate = checker.check(A, H, tau)
    assert gate.passed, gate.as_dict()
    with pytest.raises(ValueError):
        api.geqrf(torch.empty(1, n + 1, n + 1, device=DEV))


def test_error_paths_raise():
    A = torch.randn(2, 40, 40, device=DEV)
    _lib.set_config("fail_next", 1)
    with pytest.raises(_lib.QRBError, match="injected"):
        api.geqrf(A)
    H, tau = api.geqrf(A)  # the next call works again
    torch.cuda.synchronize()
    assert checker.check(A, H, tau).passed
    _lib.set_config("sync_check", 1)
    try:
        H2, _ = api.geqrf(A)
        assert torch.equal(H, H2)
    finally:
        _lib.set_config("sync_check", 0)
    with pytest.raises(ValueError):
        api.geqrf(torch.randn(2, 4, 5, device=DEV))
    with pytest.raises(ValueError):
        api.hh_fused_qr(torch.randn(2, 129, 129, device=DEV))


@pytest.mark.parametrize("b,n,chunks", [(10, 48, 3), (4096, 32, 0), (7, 100, 64), (5, 33, 1),
                                         (600, 64, 0), (3, 256, 2), (8, 512, 0), (3, 1024, 0),
                                         (8, 1024, 0), (6, 130, 0), (5, 2048, 0)])
def test_host_buffer_api_matches_device_api(b, n, chunks):
    # the blocked route with the automatic depth streams its batch groups
    # (host path 4): each group's copy gates only that group's kernels
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(b * 1000 + n))
    Ah = A.pin_memory()
    H, tau = _gpu_qr(A)
    for host_groups in ((8, 0, 3) if n > 128 and chunks == 0 else (8,)):
        _lib.set_config("host_groups", host_groups)
        try:
            Hh = torch.empty_like(Ah).pin_memory()
            th = torch.empty(b, n).pin_memory()
            api.geqrf_host(Ah, Hh, th, device=DEV, chunks=chunks)
            torch.cuda.synchronize()
        finally:
            _lib.set_config("host_groups", 8)
        if n > 128 and chunks == 0:
            assert _lib.get_config("host_path") == 4
        assert torch.equal(Hh, H) and torch.equal(th, tau), host_groups


@pytest.mark.parametrize("b,n", [(4096, 32), (9, 17), (1, 1), (3, 32)])
def test_host_direct_path_is_taken_and_matches(b, n):
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(b + n))
    H, tau = _gpu_qr(A)
    Ah = A.pin_memory()
    mode0 = _lib.get_config("host_direct")
    for mode, blocks, ramp in ((1, 0, 1), (1, 1, 1), (1, 3, 1), (2, 0, 1), (3, 0, 0), (3, 0, 1),
                               (0, 0, 0), (0, 0, 1)):
        _lib.set_config("host_direct", mode)
        _lib.set_config("direct_blocks", blocks)
        _lib.set_config("host_ramp", ramp)
        try:
            Hh = torch.full_like(Ah, float("nan")).pin_memory()
            th = torch.full((b, n), float("nan")).pin_memory()
            api.geqrf_host(Ah, Hh, th, device=DEV, chunks=3)
            torch.cuda.synchronize()
            assert _lib.get_config("host_path") == mode
            assert torch.equal(Hh, H) and torch.equal(th, tau)
        finally:
            _lib.set_config("host_direct", mode0)
            _lib.set_config("direct_blocks", 0)
            _lib.set_config("host_ramp", 0)
    # in place, on mapped memory
    M = A.clone().pin_memory()
    th = torch.empty(b, n).pin_memory()
    api.geqrf_host(M, M, th, device=DEV)
    torch.cuda.synchronize()
    assert _lib.get_config("host_path") == mode0
    assert torch.equal(M, H) and torch.equal(th, tau)


def test_host_direct_path_not_taken_for_pageable_buffers():
    A = torch.randn(8, 32, 32)
    H, tau = _gpu_qr(A)
    mode0 = _lib.get_config("host_direct")
    try:
        for mode in (1, 2, 3):
            _lib.set_config("host_direct", mode)
            # pageable H: H is copied; the pinned tau is still written directly
            Hh = torch.empty_like(A)
            th = torch.empty(8, 32).pin_memory()
            api.geqrf_host(A.pin_memory(), Hh, th, device=DEV)
            torch.cuda.synchronize()
            assert _lib.get_config("host_path") == 3
            assert torch.equal(Hh, H) and torch.equal(th, tau)
            # everything pageable: copies only
            Hh = torch.empty_like(A)
            th = torch.empty(8, 32)
            api.geqrf_host(A, Hh, th, device=DEV)
            torch.cuda.synchronize()
            assert _lib.get_config("host_path") == 0
            assert torch.equal(Hh, H) and torch.equal(th, tau)
    finally:
        _lib.set_config("host_direct", mode0)


def test_host_buffer_api_in_place_pageable_and_caller_workspace():
    A = torch.randn(9, 40, 40, generator=torch.Generator().manual_seed(5))
    H, tau = _gpu_qr(A)
    M = A.clone()  # pageable, factored in place
    th = torch.empty(9, 40)
    ws = torch.empty(api.host_workspace_bytes(9, 40), dtype=torch.uint8, device=DEV)
    api.geqrf_host(M, M, th, device=DEV, chunks=4, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(M, H) and torch.equal(th, tau)
    with pytest.raises(ValueError):
        api.geqrf_host(M, M, th, device=DEV, workspace=ws[:100])


def test_host_buffer_api_injected_failure_enqueues_nothing():
    A = torch.randn(4, 64, 64).pin_memory()
    Hh = torch.full_like(A, 7.0).pin_memory()
    th = torch.full((4, 64), 7.0).pin_memory()
    _lib.set_config("fail_next", 1)
    with pytest.raises(_lib.QRBError):
        api.geqrf_host(A, Hh, th, device=DEV)
    torch.cuda.synchronize()
    assert bool((Hh == 7.0).all()) and bool((th == 7.0).all())
    api.geqrf_host(A, Hh, th, device=DEV)
    torch.cuda.synchronize()
    H, tau = _gpu_qr(A)
    assert torch.equal(Hh, H) and torch.equal(th, tau)


def test_registered_variant_callable():
    from gpumode_qr_b200 import variants

    A = torch.randn(3, 64, 64, device=DEV)
    H, tau = variants.VARIANTS[variants.CHAMPION](A)
    torch.cuda.synchronize()
    assert checker.check(A, H, tau).passed


def test_second_device_if_present():
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU visible")
    d1 = torch.device("cuda", 1)
    A = torch.randn(4, 100, 100)
    H1, t1 = api.geqrf(A.to(d1))
    H0, t0 = _gpu_qr(A)
    torch.cuda.synchronize(d1)
    assert torch.equal(H1.cpu(), H0) and torch.equal(t1.cpu(), t0)
    assert ctypes is not None


@pytest.mark.parametrize("scale", [1e-18, 1e-12, 1e12, 1e18])
@pytest.mark.parametrize("n", [24, 100])
def test_tiny_and_huge_entries(scale, n):
    # alpha^2 + sigma outside (1e-30, 1e30) takes the plain IEEE reflector
    # formulas; inside, the reciprocal-square-root form. Both must give the
    # same factorization up to scaling.
    A = torch.randn(3, n, n, generator=torch.Generator().manual_seed(n)) * scale
    H, tau = _gpu_qr(A)
    Ho, to = oracle.geqr2(A.numpy(), f64=True)
    par = checker.parity(H, tau, Ho, to)
    assert par.ok(PARITY_RTOL), (scale, n, par)
    assert checker.check(A, H, tau).passed


def test_no_device_wait_timed_out():
    # every bounded device-side wait in the kernels completed during this run
    torch.cuda.synchronize()
    assert _lib.get_config("device_error") == 0


@pytest.mark.parametrize("b,n", [(4096, 32), (8, 64), (200, 100), (64, 512), (8, 4096)])
def test_cuda_graph_capture_and_replay(b, n):
    # The whole call (including the batch-group streams and the panel
    # look-ahead, which fork from and join back into the capturing stream)
    # captures into one CUDA graph; replays give the eager results bit for bit.
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(b + n)).to(DEV)
    H = torch.empty_like(A)
    tau = torch.empty(b, n, device=DEV)
    step = api.geqrf_into_fn(A, H, tau)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # warm-up outside capture (first-call attribute setup)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for seed in (1, 2):
        A.copy_(torch.randn(b, n, n, generator=torch.Generator().manual_seed(seed)).to(DEV))
        g.replay()
        torch.cuda.synchronize()
        He, te = api.geqrf(A)
        torch.cuda.synchronize()
        assert torch.equal(H, He) and torch.equal(tau, te)
    del g


@pytest.mark.parametrize("b,n", [(8, 512), (2, 4096), (64, 1024), (3, 300)])
def test_repeated_calls_replay_a_cached_graph(b, n):
    # The second call with the same arguments is captured into a CUDA graph
    # and later calls replay it: the bits of the eager call, and the same
    # launch count per call; a qrb_set_config change drops the match.
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(3 * n + b)).to(DEV)
    H = torch.empty_like(A)
    tau = torch.empty(b, n, device=DEV)
    step = api.geqrf_into_fn(A, H, tau)
    _lib.set_config("graph_cache", 0)
    try:
        step()
        torch.cuda.synchronize()
        He, te = H.clone(), tau.clone()
        _lib.set_config("graph_cache", 1)
        counts = []
        for k in range(5):
            if k == 3:
                _lib.set_config("lookahead", _lib.get_config("lookahead"))  # new generation
            H.fill_(float("nan"))
            tau.fill_(float("nan"))
            _lib.set_config("launches", 0)
            step()
            torch.cuda.synchronize()
            counts.append(_lib.get_config("launches"))
            assert torch.equal(H, He) and torch.equal(tau, te), k
        assert _lib.get_config("graph_cache_entries") >= 1
        assert len(set(counts)) == 1 and counts[0] > 0, counts
    finally:
        _lib.set_config("graph_cache", 1)
    assert checker.check(A, H, tau).passed
    assert _lib.get_config("device_error") == 0
