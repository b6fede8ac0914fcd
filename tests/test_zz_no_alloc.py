"""qrb_geqrf_f32_noalloc: the batched QR for callers that cannot allocate.

Callers with no way to obtain device memory (a budget reserved up front, a
host application that owns the only allocator, a runtime that forbids
cudaMalloc after start-up) use this entry point; its scratch is an array built
into the library. These tests call it through the C ABI and compare it with
qrb_geqrf_f32 given ordinary workspace, on two calls in a row (the second call
finds the first call's leftovers in the shared array). The file is named to be
collected last, and each test builds every buffer it uses, so it passes alone
in a fresh process and after the rest of the suite.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from gpumode_qr_b200 import _lib, checker

pytestmark = pytest.mark.gpu
PARITY_RTOL = 1e-4  # the tolerance the other parity tests use


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _with_workspace(A):
    b, n, _ = A.shape
    H = torch.empty_like(A)
    tau = torch.empty(b, n, device=A.device)
    nbytes = _lib.lib().qrb_workspace_bytes(b, n)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=A.device)
    rc = _lib.lib().qrb_geqrf_f32(A.data_ptr(), A.stride(0), A.stride(1), H.data_ptr(), tau.data_ptr(),
                                  b, n, ws.data_ptr(), nbytes, _stream())
    assert rc == 0, _lib.status_string(rc)
    return H, tau


def _no_alloc(A):
    b, n, _ = A.shape
    H = torch.empty_like(A)
    tau = torch.empty(b, n, device=A.device)
    rc = _lib.lib().qrb_geqrf_f32_noalloc(A.data_ptr(), A.stride(0), A.stride(1), H.data_ptr(),
                                          tau.data_ptr(), b, n, _stream())
    assert rc == 0, _lib.status_string(rc)
    return H, tau


@pytest.mark.parametrize("b,n", [(640, 512), (1024, 96), (8, 64), (2, 1000), (4096, 32)])
def test_no_alloc_matches_workspace_entry_point_twice(b, n):
    # The built-in scratch holds the T factors only, so this entry point runs
    # the FFMA trailing update; qrb_geqrf_f32 with its full workspace would
    # pick the tensor-core update, a different (equally valid) rounding. The
    # comparison therefore pins both to the FFMA update, where the two entry
    # points run the same kernels and must agree bit for bit.
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(b + n)
    old = _lib.get_config("larfb_kind")
    try:
        _lib.set_config("larfb_kind", 0)
        for call in range(2):  # two calls in a row share the built-in scratch
            A = torch.randn(b, n, n, generator=g).to(dev)
            H_ref, t_ref = _with_workspace(A)
            H, tau = _no_alloc(A)
            torch.cuda.synchronize()
            assert torch.equal(H, H_ref) and torch.equal(tau, t_ref), (b, n, call)
            par = checker.parity(H.cpu(), tau.cpu(), H_ref.cpu(), t_ref.cpu())
            assert par.ok(PARITY_RTOL), (b, n, call, par)
            k = min(b, 16)
            assert checker.check(A[:k], H[:k], tau[:k]).passed
    finally:
        _lib.set_config("larfb_kind", old)


def test_no_alloc_call_allocates_no_device_memory():
    # After one warm call (library loaded, scratch address looked up), further
    # calls leave the device's free memory unchanged.
    dev = torch.device("cuda", 0)
    b, n = 640, 512
    A = torch.randn(b, n, n, generator=torch.Generator().manual_seed(3)).to(dev)
    H = torch.empty_like(A)
    tau = torch.empty(b, n, device=dev)
    L = _lib.lib()

    def call():
        rc = L.qrb_geqrf_f32_noalloc(A.data_ptr(), A.stride(0), A.stride(1), H.data_ptr(),
                                     tau.data_ptr(), b, n, _stream())
        assert rc == 0, _lib.status_string(rc)

    call()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(dev)
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0
    assert checker.check(A[:8], H[:8], tau[:8]).passed


def test_no_alloc_rejects_batches_beyond_its_scratch():
    # 1025 matrices of n > 32 need more than the 4 MiB built-in scratch: refused
    # on the host with QRB_ERR_UNSUPPORTED before anything touches the pointers.
    fake = ctypes.c_void_p(0x1000)
    rc = _lib.lib().qrb_geqrf_f32_noalloc(fake, 64 * 64, 64, fake, fake, 1025, 64, None)
    assert rc == 2 and "unsupported" in _lib.status_string(rc)
    assert _lib.lib().qrb_geqrf_f32_noalloc(None, 0, 0, None, None, 0, 64, None) == 0
