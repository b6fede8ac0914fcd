"""Python entry points over libqrb200, shaped like the reference's operators.

* :func:`geqrf` / :func:`impl` — ``impl(A: [b, n, n] fp32) -> (H, tau)`` with
  ``torch.geqrf`` semantics: the reference's registered callable type
  (``src/qrbench/reference.py:15``) and its champion dispatch
  (``src/qrbench/variants.py:876-917``).
* :func:`hh_fused_qr` — the fused small-n kernel
  (``src/qrbench/triton_kernels.py:722-755``).
* :func:`hh_panel_qr` — panel factorization + compact-WY T
  (``src/qrbench/triton_kernels.py:912-967``).
* :func:`larfb` — the trailing block-reflector update
  (``src/qrbench/variants.py:800-804``).
* :func:`gram`, :func:`gram_geqrf` — the statistics ``G @ G.mT`` that the
  reference's workload factors, alone or followed by the factorization.

Every function runs the CUDA library on the caller's current stream. Inputs
that the library cannot take (CPU tensors, other dtypes, non-square shapes)
raise; nothing falls back to another implementation. ``A`` is never modified.
"""

from __future__ import annotations

import math

import torch

from . import _lib


def _require_cuda_f32(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32, got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (libqrb200 has no CPU path)")


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _as_rowmajor_batch(A: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """View A as [b, rows, cols] with unit column stride (copying only if needed)."""
    A3 = A.reshape(-1, rows, cols)
    if A3.stride(-1) != 1 or (A3.shape[0] > 1 and A3.stride(0) < rows * cols) or A3.stride(1) < cols:
        A3 = A3.contiguous()
    return A3


def workspace_bytes(batch: int, n: int) -> int:
    return int(_lib.lib().qrb_workspace_bytes(int(batch), int(n)))


# Trailing-update kinds of the blocked route (qrb_set_config("larfb_kind")).
LARFB_KINDS = {0: "ffma", 1: "tcgen05_staged_3xtf32", 2: "ffma_then_tcgen05",
               3: "tcgen05_tma_3xtf32"}
_ROUTES = {1: "fused_warp", 2: "fused_cta", 3: "blocked"}


def route(batch: int, n: int, workspace: int | None = None) -> str:
    """The route ``qrb_geqrf_f32`` takes for ``(batch, n)`` with ``workspace``
    bytes (default: :func:`workspace_bytes`), as text, e.g.
    ``"blocked:ffma,groups=4,lookahead"`` (``qrb_route``)."""
    ws = workspace_bytes(batch, n) if workspace is None else int(workspace)
    code = int(_lib.lib().qrb_route(int(batch), int(n), ws))
    base = _ROUTES.get(code & 0xF)
    if base is None:
        return "none"
    if base != "blocked":
        return base
    parts = [LARFB_KINDS.get((code >> 4) & 0xF, f"kind{(code >> 4) & 0xF}"),
             f"groups={(code >> 12) & 0xF}"]
    if code & (1 << 8):
        parts.append("lookahead")
    if code & (1 << 9):
        parts.append("two_level")
    if code & (1 << 10):
        parts.append("depth2")
    return base + ":" + ",".join(parts)


def max_n() -> int:
    return int(_lib.lib().qrb_max_n())


def fused_max_n() -> int:
    return int(_lib.lib().qrb_fused_max_n())


def geqrf(A: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Batched FP32 compact-Householder QR: returns ``(H, tau)`` as ``torch.geqrf``.

    ``A`` is ``[..., n, n]`` float32 on a CUDA device (any strides). ``H`` has
    A's shape (contiguous) and ``tau`` is ``[..., n]``; both are new tensors.
    """
    _require_cuda_f32("A", A)
    if A.dim() < 2 or A.shape[-1] != A.shape[-2]:
        raise ValueError(f"A must be [..., n, n] (square), got {tuple(A.shape)}")
    n = A.shape[-1]
    lead = A.shape[:-2]
    H = torch.empty(A.shape, dtype=A.dtype, device=A.device)
    tau = torch.empty((*lead, n), dtype=A.dtype, device=A.device)
    if H.numel() == 0:
        return H, tau
    if n > max_n():
        raise ValueError(f"n={n} exceeds the supported maximum {max_n()}")
    A3 = _as_rowmajor_batch(A, n, n)
    b = A3.shape[0]
    L = _lib.lib()
    with torch.cuda.device(A.device):
        ws_n = workspace_bytes(b, n)
        ws = torch.empty(max(ws_n, 16), dtype=torch.uint8, device=A.device)
        rc = L.qrb_geqrf_f32(
            A3.data_ptr(), A3.stride(0), A3.stride(1), H.data_ptr(), tau.data_ptr(),
            b, n, ws.data_ptr(), ws_n, _stream(A.device),
        )
    _lib.check(rc)
    return H, tau


def impl(A: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The registered variant callable (``QRImpl``): identical to :func:`geqrf`."""
    return geqrf(A)


def _check_out(A3: torch.Tensor, H: torch.Tensor, tau: torch.Tensor) -> None:
    b, n, _ = A3.shape
    for nm, t, shape in (("H", H, (b, n, n)), ("tau", tau, (b, n))):
        _require_cuda_f32(nm, t)
        if tuple(t.shape) != shape or not t.is_contiguous() or t.device != A3.device:
            raise ValueError(f"{nm} must be a contiguous {shape} tensor on {A3.device}")


def geqrf_into_fn(A: torch.Tensor, H: torch.Tensor, tau: torch.Tensor):
    """Return a no-argument callable that factors ``A`` into preallocated (H, tau).

    Shapes, strides and the workspace are resolved once, so each call is a
    single C-ABI call on the then-current stream of A's device (the lowest
    host overhead per factorization; used by the benchmark and repeated
    solves of same-shape batches). ``H`` may be ``A`` itself (in-place) when A
    is contiguous.
    """
    _require_cuda_f32("A", A)
    if A.dim() != 3 or A.shape[1] != A.shape[2]:
        raise ValueError(f"A must be (B, n, n), got {tuple(A.shape)}")
    b, n, _ = A.shape
    A3 = _as_rowmajor_batch(A, n, n)
    if A3.data_ptr() != A.data_ptr():
        raise ValueError("A must have unit column stride")
    _check_out(A3, H, tau)
    ws_n = workspace_bytes(b, n)
    ws = torch.empty(max(ws_n, 16), dtype=torch.uint8, device=A.device)
    L = _lib.lib()
    args = (A3.data_ptr(), A3.stride(0), A3.stride(1), H.data_ptr(), tau.data_ptr(), b, n,
            ws.data_ptr(), ws_n)
    dev = A.device

    def run() -> None:
        _lib.check(L.qrb_geqrf_f32(*args, torch.cuda.current_stream(dev).cuda_stream))

    run.buffers = (A3, H, tau, ws)  # type: ignore[attr-defined]  # keep the buffers alive
    return run


def geqrf_out(A: torch.Tensor, H: torch.Tensor, tau: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """:func:`geqrf` into caller-provided contiguous ``H [b,n,n]`` and ``tau [b,n]``."""
    geqrf_into_fn(A, H, tau)()
    return H, tau


def host_workspace_bytes(batch: int, n: int) -> int:
    """Device staging bytes :func:`geqrf_host` needs (``qrb_host_workspace_bytes``)."""
    return int(_lib.lib().qrb_host_workspace_bytes(batch, n))


def geqrf_host(A_host: torch.Tensor, H_host: torch.Tensor, tau_host: torch.Tensor,
               device: torch.device | int | str = "cuda", chunks: int = 0,
               workspace: torch.Tensor | None = None) -> None:
    """Factor a host-resident batch end to end: host -> device -> QR -> host.

    ``A_host`` ``[b, n, n]``, ``H_host`` ``[b, n, n]`` (may be ``A_host``) and
    ``tau_host`` ``[b, n]`` are contiguous float32 CPU tensors, ideally pinned
    (then the two copy directions overlap each other and the factorization).
    One call of ``qrb_geqrf_f32_host``. For n <= 32 with pinned (mapped) buffers
    the fused kernel reads and writes host memory directly in one launch;
    otherwise the batch is cut into ``chunks`` pieces (0 = 4) pipelined over
    copy-in, compute and copy-out streams inside the library. Either way the
    work is ordered after, and joined back into, the device's current stream;
    synchronise that stream before reading the outputs.
    ``workspace`` (optional) is a device uint8 tensor of at least
    :func:`host_workspace_bytes` bytes; by default one is taken from the torch
    caching allocator for the call.
    """
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("device must be a CUDA device")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    for nm, t in (("A_host", A_host), ("H_host", H_host), ("tau_host", tau_host)):
        if t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError(f"{nm} must be a contiguous float32 CPU tensor")
    if A_host.dim() != 3 or A_host.shape[1] != A_host.shape[2]:
        raise ValueError(f"A_host must be (B, n, n), got {tuple(A_host.shape)}")
    b, n, _ = A_host.shape
    if tuple(H_host.shape) != (b, n, n) or tuple(tau_host.shape) != (b, n):
        raise ValueError("H_host / tau_host shapes do not match A_host")
    if b == 0 or n == 0:
        return
    L = _lib.lib()
    need = int(L.qrb_host_workspace_bytes(b, n))
    with torch.cuda.device(dev):
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        elif (not workspace.is_cuda or workspace.device != dev
              or workspace.numel() * workspace.element_size() < need):
            raise ValueError(f"workspace must be a device tensor of >= {need} bytes on {dev}")
        rc = L.qrb_geqrf_f32_host(
            A_host.data_ptr(), H_host.data_ptr(), tau_host.data_ptr(), b, n,
            workspace.data_ptr(), workspace.numel() * workspace.element_size(), int(chunks),
            torch.cuda.current_stream(dev).cuda_stream,
        )
        _lib.check(rc)


def _gram_input(G: torch.Tensor) -> torch.Tensor:
    _require_cuda_f32("G", G)
    if G.dim() < 2:
        raise ValueError(f"G must be [..., n, k], got {tuple(G.shape)}")
    n, k = G.shape[-2], G.shape[-1]
    if n > max_n():
        raise ValueError(f"n={n} exceeds the supported maximum {max_n()}")
    if k == 0:  # nothing to read: S = 0
        return G.new_empty((math.prod(G.shape[:-2]), n, 0))
    return _as_rowmajor_batch(G, n, k)


def gram(G: torch.Tensor) -> torch.Tensor:
    """``S = G @ G.mT`` in FP32 (no TF32) for ``G [..., n, k]``: the statistics
    the reference's workload factors (its task statement, ``AGENTS.md:27``).
    ``S`` is ``[..., n, n]``, exactly symmetric, a new tensor."""
    G3 = _gram_input(G)
    n, k = G.shape[-2], G.shape[-1]
    S = torch.empty((*G.shape[:-2], n, n), dtype=G.dtype, device=G.device)
    if S.numel() == 0:
        return S
    with torch.cuda.device(G.device):
        rc = _lib.lib().qrb_gram_f32(G3.data_ptr(), G3.stride(0), G3.stride(1), S.data_ptr(),
                                     G3.shape[0], n, k, _stream(G.device))
    _lib.check(rc)
    return S


def gram_geqrf(G: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``geqrf(G @ G.mT)`` in one library call: ``(H, tau)`` of the Gram matrix
    of ``G [..., n, k]``, with ``torch.geqrf`` semantics as :func:`geqrf`."""
    G3 = _gram_input(G)
    n, k = G.shape[-2], G.shape[-1]
    lead = G.shape[:-2]
    H = torch.empty((*lead, n, n), dtype=G.dtype, device=G.device)
    tau = torch.empty((*lead, n), dtype=G.dtype, device=G.device)
    if H.numel() == 0:
        return H, tau
    b = G3.shape[0]
    with torch.cuda.device(G.device):
        ws_n = workspace_bytes(b, n)
        ws = torch.empty(max(ws_n, 16), dtype=torch.uint8, device=G.device)
        rc = _lib.lib().qrb_gram_geqrf_f32(G3.data_ptr(), G3.stride(0), G3.stride(1),
                                           H.data_ptr(), tau.data_ptr(), b, n, k, ws.data_ptr(),
                                           ws_n, _stream(G.device))
    _lib.check(rc)
    return H, tau


def hh_fused_qr(A: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused one-launch QR for small n (``n <= fused_max_n()``), as hh_fused_qr."""
    _require_cuda_f32("A", A)
    if A.dim() != 3 or A.shape[1] != A.shape[2]:
        raise ValueError(f"A must be (B, n, n), got {tuple(A.shape)}")
    b, n, _ = A.shape
    if n > fused_max_n():
        raise ValueError(f"hh_fused_qr handles n <= {fused_max_n()}, got n={n}")
    H = torch.empty((b, n, n), dtype=A.dtype, device=A.device)
    tau = torch.empty((b, n), dtype=A.dtype, device=A.device)
    if H.numel() == 0:
        return H, tau
    A3 = _as_rowmajor_batch(A, n, n)
    with torch.cuda.device(A.device):
        rc = _lib.lib().qrb_fused_qr_f32(
            A3.data_ptr(), A3.stride(0), A3.stride(1), H.data_ptr(), tau.data_ptr(), b, n,
            _stream(A.device),
        )
    _lib.check(rc)
    return H, tau


def hh_panel_qr(panel: torch.Tensor, num_warps: int | None = None, num_stages: int = 1):
    """Panel factorization of ``[B, r, w]`` (w <= 32, r >= w) -> ``(H, V, tau, T)``.

    Same outputs as the reference's ``hh_panel_qr``: packed H, unit-lower V,
    tau and the upper compact-WY factor T with ``Q^T C = C - V (T^T (V^T C))``.
    ``num_warps`` / ``num_stages`` are accepted for signature compatibility; they
    were launch knobs of the Triton kernel and have no meaning here.
    """
    del num_warps, num_stages
    _require_cuda_f32("panel", panel)
    if panel.dim() != 3:
        raise ValueError(f"panel must be (B, r, w), got {tuple(panel.shape)}")
    b, r, w = panel.shape
    if w > 32 or r < w:
        raise ValueError(f"panel needs w <= 32 and r >= w, got r={r}, w={w}")
    dev = panel.device
    H = torch.empty((b, r, w), dtype=torch.float32, device=dev)
    V = torch.empty((b, r, w), dtype=torch.float32, device=dev)
    tau = torch.empty((b, w), dtype=torch.float32, device=dev)
    T = torch.empty((b, w, w), dtype=torch.float32, device=dev)
    if H.numel() == 0:
        return H, V, tau, T
    P = _as_rowmajor_batch(panel, r, w)
    with torch.cuda.device(dev):
        rc = _lib.lib().qrb_panel_qr_f32(
            P.data_ptr(), P.stride(0), P.stride(1), H.data_ptr(), V.data_ptr(), tau.data_ptr(),
            T.data_ptr(), b, r, w, _stream(dev),
        )
    _lib.check(rc)
    return H, V, tau, T


def _reflectors(H: torch.Tensor, tau: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _require_cuda_f32("H", H)
    _require_cuda_f32("tau", tau)
    if H.dim() != 3 or H.shape[1] != H.shape[2]:
        raise ValueError(f"H must be (B, n, n), got {tuple(H.shape)}")
    b, n, _ = H.shape
    if tau.dim() != 2 or tau.shape[0] != b or tau.shape[1] > n:
        raise ValueError(f"tau must be (B, k) with k <= n, got {tuple(tau.shape)}")
    if tau.device != H.device:
        raise ValueError("H and tau must be on the same device")
    return _as_rowmajor_batch(H, n, n), tau.contiguous()


def householder_product(H: torch.Tensor, tau: torch.Tensor) -> torch.Tensor:
    """Q = H_0 H_1 ... H_{k-1} from a factorization, as
    ``torch.linalg.householder_product(H, tau)`` for square ``H [B,n,n]`` and
    ``tau [B,k]`` (k <= n); the reference's checker forms Q this way
    (src/qrbench/checker.py:129). One call of ``qrb_orgqr_f32``."""
    H3, t = _reflectors(H, tau)
    b, n, _ = H3.shape
    k = t.shape[1]
    Q = torch.empty((b, n, n), dtype=torch.float32, device=H.device)
    if Q.numel() == 0:
        return Q
    L = _lib.lib()
    ws_n = int(L.qrb_orgqr_workspace_bytes(b, n))
    ws = torch.empty(max(ws_n, 16), dtype=torch.uint8, device=H.device)
    with torch.cuda.device(H.device):
        rc = L.qrb_orgqr_f32(H3.data_ptr(), H3.stride(0), H3.stride(1), t.data_ptr(), k,
                             Q.data_ptr(), b, n, ws.data_ptr(), ws_n, _stream(H.device))
    _lib.check(rc)
    return Q


def ormqr(H: torch.Tensor, tau: torch.Tensor, C: torch.Tensor, left: bool = True,
          transpose: bool = False) -> torch.Tensor:
    """``Q C`` (or ``Q^T C`` with ``transpose``) as ``torch.ormqr(H, tau, C,
    left=True, transpose=...)`` for square ``H [B,n,n]``, ``tau [B,k]`` and
    ``C [B,n,m]``; returns a new tensor. Only ``left=True`` is supported.
    One call of ``qrb_ormqr_f32`` (src/qrbench/variants.py:165 is the
    reference's use of torch.ormqr)."""
    if not left:
        raise NotImplementedError("ormqr: only left=True (Q applied from the left) is supported")
    H3, t = _reflectors(H, tau)
    _require_cuda_f32("C", C)
    b, n, _ = H3.shape
    if C.dim() != 3 or C.shape[0] != b or C.shape[1] != n:
        raise ValueError(f"C must be (B, n, m) = ({b}, {n}, m), got {tuple(C.shape)}")
    out = C.contiguous().clone()
    if out.numel() == 0 or t.shape[1] == 0:
        return out
    L = _lib.lib()
    ws_n = int(L.qrb_orgqr_workspace_bytes(b, n))
    ws = torch.empty(max(ws_n, 16), dtype=torch.uint8, device=H.device)
    m = out.shape[2]
    with torch.cuda.device(H.device):
        rc = L.qrb_ormqr_f32(H3.data_ptr(), H3.stride(0), H3.stride(1), t.data_ptr(), t.shape[1],
                             out.data_ptr(), out.stride(0), out.stride(1), b, n, m,
                             1 if transpose else 0, ws.data_ptr(), ws_n, _stream(H.device))
    _lib.check(rc)
    return out


def larfb(V: torch.Tensor, T: torch.Tensor, C: torch.Tensor) -> torch.Tensor:
    """In-place ``C -= V (T^T (V^T C))`` for ``V [B,r,k]``, ``T [B,k,k]``, ``C [B,r,c]``.

    Only the strictly lower part of V is read (unit diagonal implied), so V may
    be a view into a packed H. Returns C.
    """
    for nm, t in (("V", V), ("T", T), ("C", C)):
        _require_cuda_f32(nm, t)
        if t.dim() != 3:
            raise ValueError(f"{nm} must be 3-D, got {tuple(t.shape)}")
    b, r, k = V.shape
    if T.shape != (b, k, k) or C.shape[0] != b or C.shape[1] != r:
        raise ValueError(f"shape mismatch V{tuple(V.shape)} T{tuple(T.shape)} C{tuple(C.shape)}")
    if C.stride(-1) != 1:
        raise ValueError("C must have unit column stride (it is updated in place)")
    c = C.shape[2]
    if C.numel() == 0 or k == 0:
        return C
    Vv = V if V.stride(-1) == 1 else V.contiguous()
    Tc = T.contiguous()
    with torch.cuda.device(C.device):
        rc = _lib.lib().qrb_larfb_f32(
            Vv.data_ptr(), Vv.stride(0), Vv.stride(1), Tc.data_ptr(), C.data_ptr(), C.stride(0),
            C.stride(1), b, r, k, c, _stream(C.device),
        )
    _lib.check(rc)
    return C
