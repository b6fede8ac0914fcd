"""GPU parity of the Gram step (S = G G^T) and of Gram + factorization.

The Gram kernel is FP32 arithmetic (FMA, no TF32); it is compared with the
FP64 product of the same FP32 inputs. Tolerance: max |S - S64| <= 2e-5 max|S64|
(a k-term FP32 dot product carries about sqrt(k) * 2^-24 relative error; 2e-5
covers k = 4096 with margin). The factorization of S is the library's own
geqrf, so gram_geqrf must equal geqrf(gram(G)) bit for bit, pass the FP64
gates against S, and agree with CPU LAPACK on S within the north-star 1e-3.
"""

from __future__ import annotations

import pytest
import torch

from gpumode_qr_b200 import _lib, api, checker

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TOL = 2e-5


def _gram64(G: torch.Tensor) -> torch.Tensor:
    g = G.double().cpu()
    return g @ g.transpose(-1, -2)


@pytest.fixture(params=[0, 64, 128], ids=["auto", "tile64", "tile128"])
def gram_tile(request):
    old = _lib.get_config("gram_tile")
    _lib.set_config("gram_tile", request.param)
    yield request.param
    _lib.set_config("gram_tile", old)


@pytest.mark.parametrize("b,n,k", [(3, 64, 64), (2, 100, 37), (4, 512, 512), (2, 130, 1000),
                                   (1, 32, 4096), (5, 1, 7), (3, 200, 4), (2, 65, 33),
                                   (64, 32, 128), (1, 1000, 96), (2, 129, 64), (1, 257, 40)])
def test_gram_matches_fp64(b, n, k, gram_tile):
    G = torch.randn(b, n, k, generator=torch.Generator().manual_seed(b * 1000 + n + k))
    S = api.gram(G.to(DEV))
    torch.cuda.synchronize()
    want = _gram64(G)
    got = S.double().cpu()
    assert (got - want).abs().max() <= TOL * want.abs().max()
    assert torch.equal(S, S.transpose(-1, -2))  # both triangles from one tile


def test_gram_strided_and_batched_views():
    g = torch.Generator().manual_seed(5)
    wide = torch.randn(3, 96, 200, generator=g).to(DEV)
    G = wide[:, :, 8:136]  # row stride 200, k = 128
    S = api.gram(G)
    S2 = api.gram(G.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(S, S2)
    G4 = torch.randn(2, 3, 40, 50, generator=g).to(DEV)  # leading dimensions
    S4 = api.gram(G4)
    torch.cuda.synchronize()
    assert S4.shape == (2, 3, 40, 40)
    assert torch.equal(S4.reshape(6, 40, 40), api.gram(G4.reshape(6, 40, 50)))


def test_gram_empty_contraction():
    G = torch.empty(2, 48, 0, device=DEV)
    S = api.gram(G)
    H, tau = api.gram_geqrf(G)
    torch.cuda.synchronize()
    assert torch.count_nonzero(S) == 0
    assert torch.count_nonzero(H) == 0 and torch.count_nonzero(tau) == 0


@pytest.mark.parametrize("b,n,k", [(16, 32, 96), (8, 64, 256), (6, 200, 600), (4, 512, 1024),
                                   (2, 1030, 2100)])
def test_gram_geqrf_equals_geqrf_of_gram_and_passes_gates(b, n, k):
    G = torch.randn(b, n, k, generator=torch.Generator().manual_seed(n + k)).to(DEV)
    H, tau = api.gram_geqrf(G)
    S = api.gram(G)
    H2, tau2 = api.geqrf(S)
    torch.cuda.synchronize()
    assert torch.equal(H, H2) and torch.equal(tau, tau2)
    assert checker.check(S, H, tau).passed


def test_gram_geqrf_against_lapack():
    # k = 4 n: cond(S) = cond(G)^2 stays small, so elementwise parity is meaningful
    G = torch.randn(3, 256, 1024, generator=torch.Generator().manual_seed(11)).to(DEV)
    H, tau = api.gram_geqrf(G)
    S = api.gram(G).cpu()
    torch.cuda.synchronize()
    Hr, tr = torch.geqrf(S)
    par = checker.parity(H.cpu(), tau.cpu(), Hr, tr)
    assert par.ok(1e-3), par
