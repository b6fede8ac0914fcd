"""CPU oracle for the batched compact-Householder QR path.

TEST INFRASTRUCTURE ONLY: this package is the checker the GPU library is
compared against. Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import it; the product package
``gpumode_qr_b200`` never does, and nothing here is on the product path.

Two oracles live here:

* :func:`lapack_geqrf` — the reference's own oracle, ``torch.geqrf`` on the CPU
  (``src/qrbench/reference.py:18-20``), i.e. LAPACK ``sgeqrf`` from the MKL
  build that ships with torch (third-party; its version is reported by
  :func:`lapack_provenance`).
* the C restatement ``hhqr_oracle.c`` of the reference's Householder kernels
  (fused QR ``src/qrbench/triton_kernels.py:641-720``, panel + LARFT
  ``:787-910``, blocked driver ``src/qrbench/variants.py:761-805``), compiled
  with gcc into ``oracle/_build/libhhqr_oracle.so`` by :func:`build`.

Both are pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``: the reference's Triton kernels executed by
Triton's CPU interpreter, and CPU ``torch.geqrf``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
SRC = ORACLE_DIR / "hhqr_oracle.c"
BUILD_DIR = ORACLE_DIR / "_build"
LIB = BUILD_DIR / "libhhqr_oracle.so"

_lib = None


def build(force: bool = False) -> Path:
    """Compile the C oracle with gcc (-O2, OpenMP over the batch)."""
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    BUILD_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = ["gcc", "-O2", "-fopenmp", "-shared", "-fPIC", "-std=c11", str(SRC), "-o", str(tmp), "-lm"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"gcc failed on the oracle:\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIB))
        i64, i32, fp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        lib.oracle_geqr2.argtypes = [i64, i32, i32, fp, i64, i64, fp, fp, i32]
        lib.oracle_panel.argtypes = [i64, i32, i32, fp, fp, fp, fp, fp, i32]
        lib.oracle_larfb.argtypes = [i64, i32, i32, i32, fp, fp, fp, i32]
        lib.oracle_blocked_geqrf.argtypes = [i64, i32, fp, i64, i64, fp, fp, i32, i32]
        lib.oracle_larft.argtypes = [i64, i32, i32, fp, i64, i64, fp, i64, fp, i32]
        for f in ("oracle_geqr2", "oracle_panel", "oracle_larfb", "oracle_blocked_geqrf",
                  "oracle_larft"):
            getattr(lib, f).restype = None
        _lib = lib
    return _lib


def _f32(x) -> np.ndarray:
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    return np.ascontiguousarray(x, dtype=np.float32)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def geqr2(A, f64: bool = True):
    """Unblocked Householder QR of a batch ``[b, rows, cols]`` -> (H, tau)."""
    a = _f32(A)
    if a.ndim == 2:
        a = a[None]
    b, rows, cols = a.shape
    H = np.empty_like(a)
    tau = np.empty((b, cols), np.float32)
    _load().oracle_geqr2(b, rows, cols, _ptr(a), rows * cols, cols, _ptr(H), _ptr(tau), int(f64))
    return H, tau


def panel(P, f64: bool = True):
    """Panel factorization ``[b, r, w]`` -> (H, V, tau, T), as hh_panel_qr."""
    p = _f32(P)
    b, r, w = p.shape
    H = np.empty_like(p)
    V = np.empty_like(p)
    tau = np.empty((b, w), np.float32)
    T = np.empty((b, w, w), np.float32)
    _load().oracle_panel(b, r, w, _ptr(p), _ptr(H), _ptr(V), _ptr(tau), _ptr(T), int(f64))
    return H, V, tau, T


def larfb(V, T, C, f64: bool = True) -> np.ndarray:
    """Return ``C - V (T^T (V^T C))`` for explicit V ``[b,r,k]``, T ``[b,k,k]``."""
    v = _f32(V)
    t = _f32(T)
    c = _f32(C).copy()
    b, r, k = v.shape
    _load().oracle_larfb(b, r, k, c.shape[2], _ptr(v), _ptr(t), _ptr(c), int(f64))
    return c


def larft(H, tau, f64: bool = True) -> np.ndarray:
    """T ``[b,k,k]`` of the packed reflector block ``H [b,r,k]`` (strictly lower
    part, unit diagonal) with coefficients ``tau [b,k]``."""
    h = _f32(H)
    t = _f32(tau)
    b, r, k = h.shape
    T = np.empty((b, k, k), np.float32)
    _load().oracle_larft(b, r, k, _ptr(h), r * k, k, _ptr(t), k, _ptr(T), int(f64))
    return T


def blocked_geqrf(A, w: int = 32, f64: bool = True):
    """Blocked Householder QR with panel width ``w`` -> (H, tau)."""
    a = _f32(A)
    b, n, _ = a.shape
    H = np.empty_like(a)
    tau = np.empty((b, n), np.float32)
    _load().oracle_blocked_geqrf(b, n, _ptr(a), n * n, n, _ptr(H), _ptr(tau), int(w), int(f64))
    return H, tau


def lapack_geqrf(A):
    """The reference's oracle: CPU ``torch.geqrf`` (LAPACK sgeqrf) -> numpy."""
    import torch

    t = torch.as_tensor(_f32(A))
    H, tau = torch.geqrf(t)
    return H.numpy(), tau.numpy()


def lapack_householder_product(H, tau):
    """Q from (H, tau) with CPU ``torch.linalg.householder_product`` (LAPACK
    sorgqr), as the reference's checker forms it (src/qrbench/checker.py:129)."""
    import torch

    return torch.linalg.householder_product(torch.as_tensor(_f32(H)), torch.as_tensor(_f32(tau))).numpy()


def lapack_ormqr(H, tau, C, transpose: bool = False):
    """Q C (or Q^T C) with CPU ``torch.ormqr`` (LAPACK sormqr), left side."""
    import torch

    return torch.ormqr(torch.as_tensor(_f32(H)), torch.as_tensor(_f32(tau)), torch.as_tensor(_f32(C)),
                       left=True, transpose=transpose).numpy()


def lapack_provenance() -> dict:
    import torch

    cfg = torch.__config__.show()
    mkl = [ln.strip() for ln in cfg.splitlines() if "MKL" in ln or "LAPACK" in ln]
    return {"torch": torch.__version__, "lapack": mkl[:3]}
