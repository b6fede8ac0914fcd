"""Host-side API behaviour and the drop-in registration (CPU only)."""

from __future__ import annotations

import importlib
import subprocess
import sys
import types

import pytest
import torch
from conftest import REPO, reference_checkout

import gpumode_qr_b200 as pkg
from gpumode_qr_b200 import api, variants

REFERENCE = reference_checkout()


def test_import_is_torch_free():
    code = (
        "import sys; import gpumode_qr_b200, gpumode_qr_b200.variants as v; "
        "assert 'torch' not in sys.modules, 'torch imported'; print(v.CHAMPION)"
    )
    out = subprocess.run([sys.executable, "-c", code], cwd=REPO, capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "b200_geqrf"


def test_api_rejects_what_it_cannot_run():
    A = torch.randn(2, 8, 8)
    with pytest.raises(ValueError, match="CUDA"):
        api.geqrf(A)  # no CPU path, no fallback
    with pytest.raises(TypeError, match="float32"):
        api.geqrf(A.double())
    with pytest.raises(TypeError):
        api.geqrf(A.numpy())
    with pytest.raises(ValueError, match="CUDA"):
        api.hh_fused_qr(A)
    with pytest.raises(ValueError, match="CUDA"):
        api.hh_panel_qr(torch.randn(2, 8, 4))


def test_host_api_validates_buffers():
    A = torch.randn(2, 8, 8)
    with pytest.raises(ValueError):
        api.geqrf_host(A, torch.empty(2, 8, 7), torch.empty(2, 8), device="cuda:0")
    with pytest.raises(ValueError):
        api.geqrf_host(A, torch.empty(2, 8, 8), torch.empty(2, 8), device="cpu")


def test_registry_shape():
    assert variants.CHAMPION in variants.VARIANTS
    assert set(variants.VARIANT_INFO) == set(variants.VARIANTS)
    rows = variants.describe_variants()
    assert rows[0][0] == variants.CHAMPION and rows[0][2]
    assert pkg.VARIANTS is variants.VARIANTS
    assert callable(pkg.impl) and callable(pkg.geqrf)


def test_register_into_fake_qrbench():
    class VariantInfo:  # stand-in for qrbench.variants.VariantInfo
        def __init__(self, description, status):
            self.description, self.status = description, status

    fake = types.SimpleNamespace(VARIANTS={"x": None}, VARIANT_INFO={}, VariantInfo=VariantInfo,
                                 CHAMPION="x")
    added = variants.register_into_qrbench(fake)
    assert set(added) == set(variants.VARIANTS)
    assert fake.VARIANTS["b200_geqrf"] is variants.VARIANTS["b200_geqrf"]
    assert isinstance(fake.VARIANT_INFO["b200_geqrf"], VariantInfo)
    assert fake.CHAMPION == "x"


@pytest.mark.skipif(REFERENCE is None, reason="reference checkout absent")
def test_register_into_reference_qrbench_and_list():
    code = f"""
import sys
sys.path.insert(0, {str(REFERENCE / 'src')!r})
sys.path.insert(0, {str(REPO)!r})
from qrbench import variants as rv
from gpumode_qr_b200 import variants
variants.register_into_qrbench(rv)
assert 'b200_geqrf' in rv.VARIANTS
txt = rv.format_variant_list()
assert 'b200_geqrf' in txt, txt
print('ok')
"""
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip().endswith("ok")


@pytest.mark.skipif(REFERENCE is None, reason="reference checkout absent")
def test_harness_shim_lists_our_variant():
    out = subprocess.run(
        [sys.executable, "-m", "gpumode_qr_b200.harness", "--reference", str(REFERENCE), "--list"],
        cwd=REPO, capture_output=True, text=True,
    )
    assert out.returncode == 0, out.stderr
    assert "b200_geqrf" in out.stdout


def test_lazy_attribute_error():
    with pytest.raises(AttributeError):
        importlib.import_module("gpumode_qr_b200").__getattr__("nope")
