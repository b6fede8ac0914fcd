"""The C ABI loads, exports what include/qrb200.h declares, and validates its
arguments on the host (no GPU work is enqueued by anything in this file)."""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest
from conftest import REPO

from gpumode_qr_b200 import _lib, api
from gpumode_qr_b200.build import LIB_PATH

HEADER = REPO / "include" / "qrb200.h"
FAKE = ctypes.c_void_p(0x1000)  # never dereferenced: every call below fails or returns early


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"QRB_API\s+[\w\s\*]+?\b(qrb_\w+)\s*\(", text)


def test_header_declares_the_expected_entry_points():
    assert set(declared_symbols()) == {
        "qrb_version", "qrb_status_string", "qrb_max_n", "qrb_workspace_bytes", "qrb_geqrf_f32",
        "qrb_geqrf_f32_noalloc", "qrb_host_workspace_bytes", "qrb_geqrf_f32_host", "qrb_fused_qr_f32",
        "qrb_fused_max_n", "qrb_panel_qr_f32", "qrb_larfb_f32", "qrb_orgqr_workspace_bytes",
        "qrb_orgqr_f32", "qrb_ormqr_f32", "qrb_gram_f32", "qrb_gram_geqrf_f32",
        "qrb_set_config", "qrb_get_config", "qrb_route",
    }


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True, text=True)
    exported = set(re.findall(r"\b(qrb_\w+)\b", out.stdout))
    for name in declared_symbols():
        assert name in exported, name
        assert hasattr(L, name)
        assert name in _lib.SIGNATURES
    # nothing else leaks out of the library with a qrb_ prefix
    assert exported == set(declared_symbols())


def test_status_strings_and_constants():
    L = _lib.lib()
    assert L.qrb_version() >= 100
    for code in range(8):
        s = _lib.status_string(code)
        assert s.startswith("qrb:")
    assert "unknown" in _lib.status_string(99)
    assert L.qrb_max_n() == 8192
    assert L.qrb_fused_max_n() == 128


def test_workspace_bytes():
    L = _lib.lib()
    assert L.qrb_workspace_bytes(4096, 32) == 0
    unit = 8 * 32 * 32 * 4  # one 32 x 32 factor per matrix
    assert L.qrb_workspace_bytes(8, 64) == 8 * unit
    assert L.qrb_workspace_bytes(0, 512) == 0
    # from n = 129 with n % 4 == 0: plus four buffers of split reflectors
    # (two V buffers x hi and lo, n x 64 each) for the tensor-core update
    assert L.qrb_workspace_bytes(8, 128) == 8 * unit
    assert L.qrb_workspace_bytes(8, 130) == 8 * unit
    assert L.qrb_workspace_bytes(8, 4096) == 8 * unit + 4 * 8 * 4096 * 64 * 4


def test_host_entry_workspace_and_validation_without_gpu():
    L = _lib.lib()
    mats, taus = 8 * 64 * 64 * 4, 8 * 64 * 4
    up = lambda x: (x + 255) // 256 * 256
    assert L.qrb_host_workspace_bytes(8, 64) == up(mats) + up(taus) + 8 * 8 * 32 * 32 * 4
    assert L.qrb_host_workspace_bytes(4096, 32) == up(4096 * 32 * 32 * 4) + up(4096 * 32 * 4)
    assert L.qrb_host_workspace_bytes(0, 64) == 0
    assert L.qrb_host_workspace_bytes(4, 8193) == 0
    need = L.qrb_host_workspace_bytes(8, 64)
    ws = ctypes.c_void_p(0x100000)
    # empty problems succeed without touching memory
    assert L.qrb_geqrf_f32_host(None, None, None, 0, 64, None, 0, 0, None) == 0
    # null host pointers, negative sizes, chunks outside 0..64
    assert L.qrb_geqrf_f32_host(None, FAKE, FAKE, 8, 64, ws, need, 0, None) == 1
    assert L.qrb_geqrf_f32_host(FAKE, FAKE, FAKE, -1, 64, ws, need, 0, None) == 1
    assert L.qrb_geqrf_f32_host(FAKE, FAKE, FAKE, 8, 64, ws, need, 65, None) == 1
    assert L.qrb_geqrf_f32_host(FAKE, FAKE, FAKE, 8, 64, ws, need, -1, None) == 1
    # too large, missing / short / misaligned workspace
    assert L.qrb_geqrf_f32_host(FAKE, FAKE, FAKE, 1, 8193, ws, 1 << 30, 0, None) == 2
    assert L.qrb_geqrf_f32_host(FAKE, FAKE, FAKE, 8, 64, None, need, 0, None) == 3
    assert L.qrb_geqrf_f32_host(FAKE, FAKE, FAKE, 8, 64, ws, need - 1, 0, None) == 3
    assert L.qrb_geqrf_f32_host(FAKE, FAKE, FAKE, 8, 64, ctypes.c_void_p(0x100010), need, 0,
                                None) == 1


def test_gram_validation_without_gpu():
    # every call here returns before anything is enqueued
    L = _lib.lib()
    ws = ctypes.c_void_p(0x100000)
    need = L.qrb_workspace_bytes(2, 64)
    # empty problems
    assert L.qrb_gram_f32(None, 0, 0, None, 0, 64, 64, None) == 0
    assert L.qrb_gram_f32(None, 0, 0, None, 2, 0, 64, None) == 0
    assert L.qrb_gram_geqrf_f32(None, 0, 0, None, None, 0, 64, 64, None, 0, None) == 0
    # negative sizes, null pointers, row stride < k, overlapping matrices, too large
    assert L.qrb_gram_f32(FAKE, 64 * 80, 80, FAKE, -1, 64, 80, None) == 1
    assert L.qrb_gram_f32(None, 64 * 80, 80, FAKE, 2, 64, 80, None) == 1
    assert L.qrb_gram_f32(FAKE, 64 * 80, 80, None, 2, 64, 80, None) == 1
    assert L.qrb_gram_f32(FAKE, 64 * 80, 79, FAKE, 2, 64, 80, None) == 1
    assert L.qrb_gram_f32(FAKE, 64 * 80 - 1, 80, FAKE, 2, 64, 80, None) == 1
    assert L.qrb_gram_f32(FAKE, 0, 80, FAKE, 1, 8193, 80, None) == 2
    # gram + geqrf: null tau, short / missing / misaligned workspace
    assert L.qrb_gram_geqrf_f32(FAKE, 64 * 80, 80, FAKE, None, 2, 64, 80, ws, need, None) == 1
    assert L.qrb_gram_geqrf_f32(FAKE, 64 * 80, 80, FAKE, FAKE, 2, 64, 80, ws, need // 8 - 1,
                                None) == 3
    assert L.qrb_gram_geqrf_f32(FAKE, 64 * 80, 80, FAKE, FAKE, 2, 64, 80, None, need, None) == 3
    assert L.qrb_gram_geqrf_f32(FAKE, 64 * 80, 80, FAKE, FAKE, 2, 64, 80,
                                ctypes.c_void_p(0x100004), need, None) == 1
    assert L.qrb_gram_geqrf_f32(FAKE, 64 * 80, 79, FAKE, FAKE, 2, 64, 80, ws, need, None) == 1


def test_orgqr_ormqr_validation_without_gpu():
    L = _lib.lib()
    assert L.qrb_orgqr_workspace_bytes(8, 64) == 8 * 32 * 32 * 4
    assert L.qrb_orgqr_workspace_bytes(8, 16) == 8 * 32 * 32 * 4
    assert L.qrb_orgqr_workspace_bytes(0, 16) == 0
    ws = ctypes.c_void_p(0x100000)
    need = L.qrb_orgqr_workspace_bytes(2, 64)
    # empty problems
    assert L.qrb_orgqr_f32(None, 0, 0, None, 0, None, 0, 64, None, 0, None) == 0
    assert L.qrb_ormqr_f32(None, 0, 0, None, 0, None, 0, 0, 2, 64, 0, 1, None, 0, None) == 0
    # bad arguments: k > n, null pointers, overlapping rows, short workspace, too large
    assert L.qrb_orgqr_f32(FAKE, 4096, 64, FAKE, 65, FAKE, 2, 64, ws, need, None) == 1
    assert L.qrb_orgqr_f32(None, 4096, 64, FAKE, 64, FAKE, 2, 64, ws, need, None) == 1
    assert L.qrb_orgqr_f32(FAKE, 4096, 32, FAKE, 64, FAKE, 2, 64, ws, need, None) == 1
    assert L.qrb_orgqr_f32(FAKE, 4096, 64, FAKE, 64, FAKE, 2, 64, ws, need - 1, None) == 3
    assert L.qrb_orgqr_f32(FAKE, 8193 * 8193, 8193, FAKE, 8193, FAKE, 1, 8193, ws, 1 << 30,
                           None) == 2
    assert L.qrb_ormqr_f32(FAKE, 4096, 64, FAKE, 64, FAKE, 640, 9, 2, 64, 10, 1, ws, need,
                           None) == 1
    assert L.qrb_ormqr_f32(FAKE, 4096, 64, FAKE, 64, FAKE, 640, 10, 2, 64, 10, 1, None, 0,
                           None) == 3


def test_argument_validation_without_gpu():
    L = _lib.lib()
    ws = ctypes.c_void_p(0x2000)
    # empty problems succeed without touching memory
    assert L.qrb_geqrf_f32(None, 0, 0, None, None, 0, 64, None, 0, None) == 0
    assert L.qrb_geqrf_f32(None, 0, 0, None, None, 4, 0, None, 0, None) == 0
    # negative sizes, null pointers, overlapping strides
    assert L.qrb_geqrf_f32(FAKE, 4096, 64, FAKE, FAKE, -1, 64, ws, 1 << 20, None) == 1
    assert L.qrb_geqrf_f32(None, 4096, 64, FAKE, FAKE, 1, 64, ws, 1 << 20, None) == 1
    assert L.qrb_geqrf_f32(FAKE, 4096, 63, FAKE, FAKE, 1, 64, ws, 1 << 20, None) == 1
    assert L.qrb_geqrf_f32(FAKE, 100, 64, FAKE, FAKE, 2, 64, ws, 1 << 20, None) == 1
    # too large
    assert L.qrb_geqrf_f32(FAKE, 8193 * 8193, 8193, FAKE, FAKE, 1, 8193, ws, 1 << 30, None) == 2
    # blocked path needs workspace
    assert L.qrb_geqrf_f32(FAKE, 4096, 64, FAKE, FAKE, 2, 64, None, 0, None) == 3
    assert L.qrb_geqrf_f32(FAKE, 4096, 64, FAKE, FAKE, 2, 64, ws, 100, None) == 3
    # in-place requires a contiguous A
    assert L.qrb_geqrf_f32(FAKE, 8192, 128, FAKE, FAKE, 2, 64, ws, 1 << 20, None) == 1
    # kernel-level entry points
    assert L.qrb_fused_qr_f32(FAKE, 129 * 129, 129, FAKE, FAKE, 1, 129, None) == 2
    assert L.qrb_panel_qr_f32(FAKE, 100 * 33, 33, FAKE, None, FAKE, FAKE, 1, 100, 33, None) == 2
    assert L.qrb_panel_qr_f32(FAKE, 100, 10, FAKE, None, FAKE, FAKE, 1, 5, 10, None) == 2
    assert L.qrb_larfb_f32(FAKE, 64 * 8, 8, None, FAKE, 64 * 8, 8, 1, 64, 8, 8, None) == 1
    assert L.qrb_larfb_f32(FAKE, 64 * 40, 40, FAKE, FAKE, 64 * 8, 8, 1, 64, 40, 8, None) == 2


def test_fault_injection_is_host_side():
    # "fail_next" makes the next compute call fail before anything is enqueued.
    L = _lib.lib()
    ws = ctypes.c_void_p(0x2000)
    _lib.set_config("fail_next", 2)
    assert _lib.get_config("fail_next") == 2
    assert L.qrb_geqrf_f32(FAKE, 4096, 64, FAKE, FAKE, 2, 64, ws, 1 << 20, None) == 6
    assert L.qrb_fused_qr_f32(FAKE, 32 * 32, 32, FAKE, FAKE, 2, 32, None) == 6
    assert _lib.get_config("fail_next") == 0
    with pytest.raises(_lib.QRBError) as ei:
        _lib.check(6)
    assert ei.value.status == 6 and "injected" in str(ei.value)


def test_config_keys():
    assert _lib.get_config("sync_check") == 0
    _lib.set_config("sync_check", 1)
    assert _lib.get_config("sync_check") == 1
    _lib.set_config("sync_check", 0)
    _lib.set_config("launches", 0)
    assert _lib.get_config("launches") == 0
    assert _lib.get_config("larfb_kind") == -1  # automatic
    for v in (0, 1, 2, 3, -1):
        _lib.set_config("larfb_kind", v)
        assert _lib.get_config("larfb_kind") == v
    for bad in (4, -2):
        with pytest.raises(_lib.QRBError):
            _lib.set_config("larfb_kind", bad)
    assert _lib.get_config("wait_limit") == 2_000_000_000
    _lib.set_config("wait_limit", 5000)
    assert _lib.get_config("wait_limit") == 5000
    _lib.set_config("wait_limit", 2_000_000_000)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("wait_limit", 10)
    assert _lib.get_config("test_skip_mma") == 0
    with pytest.raises(_lib.QRBError):
        _lib.set_config("test_skip_mma", 2)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("wait_probe", 10)
    assert _lib.get_config("host_groups") == 8
    _lib.set_config("host_groups", 0)
    assert _lib.get_config("host_groups") == 0
    _lib.set_config("host_groups", 8)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("host_groups", 9)
    assert _lib.get_config("tma_split_rows") == 1024
    _lib.set_config("tma_split_rows", 0)
    assert _lib.get_config("tma_split_rows") == 0
    _lib.set_config("tma_split_rows", 1024)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("tma_split_rows", -1)
    assert _lib.get_config("tma_pair") == 0
    for v in (1, 2, 0):
        _lib.set_config("tma_pair", v)
        assert _lib.get_config("tma_pair") == v
    with pytest.raises(_lib.QRBError):
        _lib.set_config("tma_pair", 3)
    assert _lib.get_config("graph_cache") == 1
    _lib.set_config("graph_cache", 0)
    assert _lib.get_config("graph_cache") == 0
    assert _lib.get_config("graph_cache_entries") == 0
    _lib.set_config("graph_cache", 1)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("graph_cache", 2)
    assert _lib.get_config("lookahead_depth") == 0
    for v in (1, 2, 0):
        _lib.set_config("lookahead_depth", v)
        assert _lib.get_config("lookahead_depth") == v
    with pytest.raises(_lib.QRBError):
        _lib.set_config("lookahead_depth", 3)
    assert _lib.get_config("tma_dual") == 0
    for v in (1, 2, 0):
        _lib.set_config("tma_dual", v)
        assert _lib.get_config("tma_dual") == v
    with pytest.raises(_lib.QRBError):
        _lib.set_config("tma_dual", 3)
    assert _lib.get_config("tma_ctas") == 0
    _lib.set_config("tma_ctas", 96)
    assert _lib.get_config("tma_ctas") == 96
    _lib.set_config("tma_ctas", 0)
    for key in ("narrow_update", "panel_priority"):
        assert _lib.get_config(key) == 1
        _lib.set_config(key, 0)
        assert _lib.get_config(key) == 0
        _lib.set_config(key, 1)
        with pytest.raises(_lib.QRBError):
            _lib.set_config(key, 2)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("tma_ctas", -1)
    assert _lib.get_config("host_direct") in (0, 1, 2, 3)
    _lib.set_config("host_direct", 0)
    assert _lib.get_config("host_direct") == 0
    _lib.set_config("host_direct", 2)
    assert _lib.get_config("host_direct") == 2
    _lib.set_config("host_direct", 1)
    assert _lib.get_config("host_direct") == 1
    _lib.set_config("host_direct", 3)  # the default
    with pytest.raises(_lib.QRBError):
        _lib.set_config("host_direct", 4)
    assert _lib.get_config("host_ramp") == 0
    _lib.set_config("host_ramp", 1)
    assert _lib.get_config("host_ramp") == 1
    _lib.set_config("host_ramp", 0)
    assert _lib.get_config("groups") == 0
    _lib.set_config("groups", 3)
    assert _lib.get_config("groups") == 3
    _lib.set_config("groups", 0)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("groups", 9)
    assert _lib.get_config("lookahead") == 2
    _lib.set_config("lookahead", 1)
    assert _lib.get_config("lookahead") == 1
    _lib.set_config("lookahead", 2)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("lookahead", 3)
    assert _lib.get_config("two_level") == 2  # automatic
    for v in (0, 1, 2):
        _lib.set_config("two_level", v)
        assert _lib.get_config("two_level") == v
    with pytest.raises(_lib.QRBError):
        _lib.set_config("two_level", 3)
    assert _lib.get_config("panel_rpt") == 0
    for v in (1, 2, 4, 0):
        _lib.set_config("panel_rpt", v)
        assert _lib.get_config("panel_rpt") == v
    with pytest.raises(_lib.QRBError):
        _lib.set_config("panel_rpt", 3)
    assert _lib.get_config("gram_tile") == 0
    for v in (64, 128, 0):
        _lib.set_config("gram_tile", v)
        assert _lib.get_config("gram_tile") == v
    with pytest.raises(_lib.QRBError):
        _lib.set_config("gram_tile", 32)
    assert _lib.get_config("mid_fused") == 1
    _lib.set_config("mid_fused", 0)
    assert _lib.get_config("mid_fused") == 0
    _lib.set_config("mid_fused", 2)
    assert _lib.get_config("mid_fused") == 2
    _lib.set_config("mid_fused", 1)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("mid_fused", 3)
    assert _lib.get_config("fused_cpl") == 0
    _lib.set_config("fused_cpl", 4)
    assert _lib.get_config("fused_cpl") == 4
    _lib.set_config("fused_cpl", 0)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("fused_cpl", 3)
    assert _lib.get_config("direct_blocks") > 0
    _lib.set_config("direct_blocks", 7)
    assert _lib.get_config("direct_blocks") == 7
    _lib.set_config("direct_blocks", 0)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("direct_blocks", -1)
    assert _lib.get_config("host_path") in (-1, 0, 1, 2, 3, 4)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("host_path", 1)  # read-only
    with pytest.raises(_lib.QRBError):
        _lib.set_config("no_such_key", 1)
    with pytest.raises(_lib.QRBError):
        _lib.set_config("sync_check", 7)
    with pytest.raises(_lib.QRBError):
        _lib.get_config("no_such_key")



def test_route_is_a_function_of_batch_n_and_workspace():
    # with every hook at its default the route depends on (batch, n, workspace)
    # only; the reference's champion dispatch routes by n alone
    L = _lib.lib()
    assert L.qrb_route(4096, 32, 0) & 0xF == 1
    assert L.qrb_route(8, 64, 0) & 0xF == 2
    assert L.qrb_route(8, 128, 0) & 0xF == 2
    assert L.qrb_route(0, 64, 0) == 0 and L.qrb_route(4, 9000, 0) == 0
    ws = L.qrb_workspace_bytes(8, 4096)
    assert L.qrb_route(8, 4096, 0) == 0  # the blocked route needs workspace
    code = L.qrb_route(8, 4096, ws)
    assert code & 0xF == 3 and code & (1 << 8)  # blocked, with the look-ahead
    # the tensor-core update needs the split-reflector part of the workspace
    # (and, on a machine without a CUDA driver, the TMA encoder: FFMA then)
    kind = (code >> 4) & 0xF
    assert kind in (0, 3)
    assert (code >> 12) & 0xF == 4
    big = L.qrb_route(64, 4096, L.qrb_workspace_bytes(64, 4096))
    small = L.qrb_route(640, 512, L.qrb_workspace_bytes(640, 512))
    assert not small & (3 << 8)
    if kind == 3:  # two-level from n = 1024, with the look-ahead up to batch * n = 2^16
        assert code & (1 << 9)
        assert big & (1 << 9) and not big & (1 << 8)
    else:  # FFMA: the look-ahead from n = 4096, no two-level blocking
        assert not code & (1 << 9)
        assert big & (1 << 8) and not big & (1 << 9)
    assert (L.qrb_route(8, 4096, 4 * 8 * 32 * 32 * 4) >> 4) & 0xF == 0
    assert (L.qrb_route(8, 130, L.qrb_workspace_bytes(8, 130)) >> 4) & 0xF == 0
    assert L.qrb_route(8, 4096, ws) == code  # no hidden state between queries
    assert api.route(640, 512).startswith("blocked:")
    assert api.route(4096, 32) == "fused_warp"
