"""gpumode_qr_b200 — B200-native (sm_100a) batched FP32 compact-Householder QR.

``impl(A: [b, n, n] fp32) -> (H, tau)`` with ``torch.geqrf`` semantics, backed
by the CUDA library ``libqrb200.so`` (C ABI in ``include/qrb200.h``). The
callables and the registry are importable without a GPU; the library is loaded
on first use and its absence is an error, never a fallback.
"""

from __future__ import annotations

__all__ = [
    "geqrf",
    "impl",
    "hh_fused_qr",
    "hh_panel_qr",
    "larfb",
    "householder_product",
    "ormqr",
    "geqrf_host",
    "gram",
    "gram_geqrf",
    "VARIANTS",
    "VARIANT_INFO",
    "CHAMPION",
    "EPS32",
]

EPS32 = 2.0**-23

from .variants import CHAMPION, VARIANT_INFO, VARIANTS  # noqa: E402


def __getattr__(name):  # lazy: keep `import gpumode_qr_b200` torch-free
    if name in ("geqrf", "impl", "hh_fused_qr", "hh_panel_qr", "larfb", "householder_product",
                "ormqr", "geqrf_host", "gram", "gram_geqrf"):
        from . import api

        return getattr(api, name)
    raise AttributeError(name)
