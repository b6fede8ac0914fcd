"""Variant registry and the drop-in registration into the reference's harness.

The reference looks implementations up by name in
``REGISTRY = {**reference.REGISTRY, **variants.VARIANTS}``
(``scripts/run_baseline.py:38-40``), with one-line metadata in
``variants.VARIANT_INFO`` (``src/qrbench/variants.py:1186``) used by ``--list``.
This module exposes the same names for this library (``VARIANTS``,
``VARIANT_INFO``, ``CHAMPION``, ``describe_variants``) and
:func:`register_into_qrbench`, which inserts them into an imported reference
``qrbench.variants`` module so its harness runs them unchanged.

Importing this module needs neither torch nor a GPU (the reference's ``--list``
path is torch-free too, ``src/qrbench/variants.py:97-100``); the callables load
the CUDA library on first use.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

CHAMPION = "b200_geqrf"


def _geqrf(A):
    from .api import geqrf

    return geqrf(A)


def _fused(A):
    from .api import hh_fused_qr

    return hh_fused_qr(A)


VARIANTS: dict[str, Callable] = {
    "b200_geqrf": _geqrf,
    "b200_fused_smalln": _fused,
}


@dataclass(frozen=True)
class VariantInfo:
    description: str
    status: str  # active | experimental | killed | baseline


VARIANT_INFO: dict[str, VariantInfo] = {
    "b200_geqrf": VariantInfo(
        "B200 sm_100a: fused warp kernel (n<=32), fused CTA kernel (n<=128, size permitting), "
        "else cluster panel + larft + FFMA larfb",
        "active",
    ),
    "b200_fused_smalln": VariantInfo(
        "B200 sm_100a fused whole-matrix QR, 2 or 4 matrices per warp (n<=32 only)",
        "experimental",
    ),
}


def describe_variants() -> list[tuple[str, VariantInfo, bool]]:
    order = {"active": 0, "experimental": 1, "killed": 2, "baseline": 3}
    names = sorted(VARIANTS, key=lambda n: (n != CHAMPION, order[VARIANT_INFO[n].status], n))
    return [(n, VARIANT_INFO[n], n == CHAMPION) for n in names]


def register_into_qrbench(variants_module) -> list[str]:
    """Insert this library's variants into a reference ``qrbench.variants`` module.

    Entries are added to ``VARIANTS`` and, using that module's own
    ``VariantInfo`` type, to ``VARIANT_INFO``. The reference's ``CHAMPION`` is
    left untouched. Returns the names added.
    """
    ref_info_type = getattr(variants_module, "VariantInfo", None)
    added = []
    for name, fn in VARIANTS.items():
        variants_module.VARIANTS[name] = fn
        if ref_info_type is not None and hasattr(variants_module, "VARIANT_INFO"):
            info = VARIANT_INFO[name]
            variants_module.VARIANT_INFO[name] = ref_info_type(info.description, info.status)
        added.append(name)
    return added
