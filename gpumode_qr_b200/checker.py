"""FP64 correctness gates and the elementwise parity metric.

The gates restate the reference's checker (``src/qrbench/checker.py:79-158``):
``Q = householder_product(H, tau)`` formed in FP32 and then cast to FP64,
``R = triu(H)``, factor residual ``||R - Q^T A||_1 / ||A||_1 <= 20 n eps32``
and orthogonality ``||Q^T Q - I||_1 <= 100 n eps32`` with the induced 1-norm
(max absolute column sum), reduced as the max over the batch; the FP64
workspace is chunked to stay under 2 GB (``checker.py:71-76``). Lower-triangle
leakage and the reconstruction residual are diagnostics, as there.

:func:`parity` is the elementwise agreement used against a reference
factorization (CPU ``torch.geqrf``) for well-conditioned inputs.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

import torch

EPS32 = 2.0**-23


@dataclass
class CheckResult:
    n: int
    batch: int
    factor_residual: float
    factor_threshold: float
    factor_pass: bool
    orth_residual: float
    orth_threshold: float
    orth_pass: bool
    leakage: float
    reconstruction: float

    @property
    def passed(self) -> bool:
        return bool(self.factor_pass and self.orth_pass)

    def as_dict(self) -> dict:
        d = asdict(self)
        d["passed"] = self.passed
        return d


def _l1(x: torch.Tensor) -> torch.Tensor:
    return torch.linalg.matrix_norm(x, ord=1)


def _auto_batch_chunk(batch: int, n: int, max_bytes: int = 2_000_000_000) -> int:
    per_item = 4 * n * n * 8
    return max(1, min(batch, max_bytes // max(per_item, 1)))


def _check_slice(A, H, tau, eye):
    A64 = A.double()
    Q = torch.linalg.householder_product(H, tau).double()
    R = torch.triu(H).double()
    QtA = Q.transpose(-2, -1) @ A64
    a_norm = _l1(A64).clamp_min(torch.finfo(torch.float64).tiny)
    factor = (_l1(R - QtA) / a_norm).max().item()
    orth = _l1(Q.transpose(-2, -1) @ Q - eye).max().item()
    leak = (_l1(torch.tril(QtA, diagonal=-1)) / a_norm).max().item()
    recon = (_l1(Q @ R - A64) / a_norm).max().item()
    return factor, orth, leak, recon


def check(A: torch.Tensor, H: torch.Tensor, tau: torch.Tensor) -> CheckResult:
    """Validate a compact (H, tau) factorization of A ([b, n, n]); FP64 residuals."""
    n = A.shape[-1]
    batch = A.shape[0]
    factor_thr = 20.0 * n * EPS32
    orth_thr = 100.0 * n * EPS32
    eye = torch.eye(n, device=A.device, dtype=torch.float64)
    chunk = _auto_batch_chunk(batch, n)
    f = o = lk = rc = 0.0
    for s in range(0, batch, chunk):
        e = min(s + chunk, batch)
        f2, o2, l2, r2 = _check_slice(A[s:e], H[s:e], tau[s:e], eye)
        f, o, lk, rc = max(f, f2), max(o, o2), max(lk, l2), max(rc, r2)
    return CheckResult(
        n=n,
        batch=batch,
        factor_residual=f,
        factor_threshold=factor_thr,
        factor_pass=f <= factor_thr,
        orth_residual=o,
        orth_threshold=orth_thr,
        orth_pass=o <= orth_thr,
        leakage=lk,
        reconstruction=rc,
    )


PARITY_RTOL = 1e-3


@dataclass
class Parity:
    h_rel: float  # max over matrices of max|H - H_ref| / max|H_ref|
    tau_rel: float  # max over matrices of max|tau - tau_ref| / max(1, max|tau_ref|)
    col_rel: float  # max over columns of max_i |dH_ij| / ||H_ref[:, j]||_2

    def ok(self, rtol: float = PARITY_RTOL) -> bool:
        return self.h_rel <= rtol and self.tau_rel <= rtol and self.col_rel <= rtol


def parity(H, tau, H_ref, tau_ref) -> Parity:
    """Normwise elementwise agreement of (H, tau) with a reference factorization."""
    H = torch.as_tensor(H).double().cpu()
    tau = torch.as_tensor(tau).double().cpu()
    Hr = torch.as_tensor(H_ref).double().cpu()
    tr = torch.as_tensor(tau_ref).double().cpu()
    b = Hr.shape[0]
    dH = (H - Hr).abs().reshape(b, -1).amax(1)
    hmax = Hr.abs().reshape(b, -1).amax(1).clamp_min(1e-300)
    dt = (tau - tr).abs().amax(1)
    tmax = tr.abs().amax(1).clamp_min(1.0)
    coln = Hr.norm(dim=1).clamp_min(1e-300)  # [b, n]: 2-norm of each column
    dcol = (H - Hr).abs().amax(1) / coln
    return Parity(
        h_rel=(dH / hmax).max().item(),
        tau_rel=(dt / tmax).max().item(),
        col_rel=dcol.max().item(),
    )
