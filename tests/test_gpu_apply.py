"""GPU forming and applying of Q from a factorization (qrb_orgqr_f32 /
qrb_ormqr_f32) against CPU LAPACK (torch.linalg.householder_product /
torch.ormqr, the calls the reference makes at src/qrbench/checker.py:129 and
src/qrbench/variants.py:165) and against the C oracle's LARFT.

Tolerances: Q and Q C agree with LAPACK within 1e-5 * max(n, 8) relative to
max |Q| (both are FP32 products of k reflectors); Q is orthogonal within
20 * n * eps32 and reproduces A = Q R within 20 * n * eps32 relative.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gpumode_qr_b200 import _lib, api

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
EPS32 = 2.0**-23


def _factor(b, n, seed):
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(seed))
    H, tau = api.geqrf(A.to(DEV))
    torch.cuda.synchronize()
    return A, H, tau


def _tol(n):
    return 1e-5 * max(n, 8)


@pytest.mark.parametrize("n", [1, 2, 5, 31, 32, 33, 64, 100, 257, 512])
def test_householder_product_matches_lapack_and_is_orthogonal(n):
    b = 3
    A, H, tau = _factor(b, n, n)
    Q = api.householder_product(H, tau)
    torch.cuda.synchronize()
    Qc = Q.cpu().double()
    want = torch.from_numpy(oracle.lapack_householder_product(H.cpu().numpy(), tau.cpu().numpy()))
    assert (Qc - want.double()).abs().max() <= _tol(n)
    eye = torch.eye(n, dtype=torch.float64)
    assert (Qc.transpose(1, 2) @ Qc - eye).abs().max() <= 20 * n * EPS32 + 1e-6
    R = torch.triu(H.cpu().double())
    resid = (Qc @ R - A.double()).abs().max() / A.double().abs().max()
    assert resid <= 20 * n * EPS32 + 1e-6


@pytest.mark.parametrize("n,k", [(64, 1), (64, 20), (100, 33), (130, 64), (40, 0)])
def test_householder_product_fewer_reflectors(n, k):
    A, H, tau = _factor(2, n, 7 * n + k)
    tk = tau[:, :k].contiguous()
    Q = api.householder_product(H, tk)
    torch.cuda.synchronize()
    want = torch.linalg.householder_product(H.cpu(), tk.cpu())
    assert (Q.cpu() - want).abs().max() <= _tol(n)


@pytest.mark.parametrize("n,m", [(32, 5), (33, 64), (200, 17), (512, 96), (1000, 40)])
@pytest.mark.parametrize("transpose", [False, True])
def test_ormqr_matches_lapack(n, m, transpose):
    A, H, tau = _factor(2, n, n + m)
    C = torch.randn(2, n, m, generator=torch.Generator().manual_seed(m))
    out = api.ormqr(H, tau, C.to(DEV), transpose=transpose)
    torch.cuda.synchronize()
    want = torch.from_numpy(oracle.lapack_ormqr(H.cpu().numpy(), tau.cpu().numpy(), C.numpy(),
                                                transpose=transpose))
    scale = max(float(C.abs().max()), 1.0)
    assert (out.cpu() - want).abs().max() / scale <= _tol(n)


def test_ormqr_round_trip_and_identity():
    n = 96
    A, H, tau = _factor(3, n, 5)
    C = torch.randn(3, n, 50, device=DEV)
    back = api.ormqr(H, tau, api.ormqr(H, tau, C, transpose=True), transpose=False)
    torch.cuda.synchronize()
    assert (back - C).abs().max() / C.abs().max() <= 50 * n * EPS32
    eye = torch.eye(n, device=DEV).expand(3, n, n).contiguous()
    Q1 = api.ormqr(H, tau, eye)
    Q2 = api.householder_product(H, tau)
    torch.cuda.synchronize()
    assert (Q1 - Q2).abs().max() <= 10 * n * EPS32
    # Q^T A = R (upper triangle of H)
    R = api.ormqr(H, tau, A.to(DEV), transpose=True)
    torch.cuda.synchronize()
    assert (R.cpu() - torch.triu(H.cpu())).abs().max() / A.abs().max() <= 20 * n * EPS32


def test_orgqr_launch_count_and_strided_input():
    n = 100  # four reflector blocks: identity + 4 x (larft + larfb)
    A, H, tau = _factor(2, n, 11)
    _lib.set_config("launches", 0)
    Q = api.householder_product(H, tau)
    torch.cuda.synchronize()
    assert _lib.get_config("launches") == 1 + 2 * 4
    # a non-contiguous H (every other matrix of a larger batch) gives the same Q
    big = torch.empty(4, n, n, device=DEV)
    big[::2] = H
    Q2 = api.householder_product(big[::2], tau)
    torch.cuda.synchronize()
    assert torch.equal(Q, Q2)


def test_larft_inside_orgqr_matches_oracle():
    # One block (n <= 32): Q = I - V T V^T with T from the oracle's LARFT.
    n = 29
    A, H, tau = _factor(4, n, 3)
    Q = api.householder_product(H, tau).cpu().double().numpy()
    Hn, tn = H.cpu().numpy(), tau.cpu().numpy()
    T = oracle.larft(Hn, tn, f64=True).astype(np.float64)
    V = np.tril(Hn.astype(np.float64), -1) + np.eye(n)
    want = np.eye(n) - V @ T @ np.transpose(V, (0, 2, 1))
    assert np.abs(Q - want).max() <= _tol(n)


def test_apply_errors_raise():
    H = torch.randn(2, 8, 8, device=DEV)
    with pytest.raises(ValueError):
        api.householder_product(H, torch.randn(2, 9, device=DEV))
    with pytest.raises(ValueError):
        api.ormqr(H, torch.randn(2, 8, device=DEV), torch.randn(2, 7, 3, device=DEV))
    with pytest.raises(NotImplementedError):
        api.ormqr(H, torch.randn(2, 8, device=DEV), torch.randn(2, 8, 3, device=DEV), left=False)
    _lib.set_config("fail_next", 1)
    with pytest.raises(_lib.QRBError):
        api.householder_product(H, torch.randn(2, 8, device=DEV))
