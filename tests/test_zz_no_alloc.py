"""GPU: the allocation-free factorisation entry point (qrb_geqrf_f32_noalloc).

Callers that cannot allocate device memory -- a plugin host that passes only raw
input and output pointers, or a path that must not enter the allocator -- use
this entry point; its scratch is a static device array inside the library.  The
test calls it through the C ABI twice in a row (the second call sees the scratch
the first one left behind) and compares each result with the regular
qrb_geqrf_f32.  The two run different fp32 trailing updates (SIMT here, the
tensor-core split kernels there), so their rounding differs like two LAPACK
builds': the H/tau tolerance of the other parity tests, 5e-5, is scaled by n/256
beyond n = 256 (rounding differences grow with the number of panels).  This file
sorts last so a stop-at-first-failure run has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_H = 5e-5   # same H / tau tolerance as tests/test_gpu_parity.py


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import build
    build.build()
    from qr_b200 import _lib
    return _lib.lib()


def _regular(lib, A):
    batch, n, _ = A.shape
    H = torch.empty_like(A)
    tau = torch.empty(batch, n, device=A.device)
    nb = lib.qrb_workspace_size(batch, n)
    ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=A.device)
    st = lib.qrb_geqrf_f32(A.data_ptr(), H.data_ptr(), tau.data_ptr(), batch, n, ws.data_ptr(), nb,
                           torch.cuda.current_stream().cuda_stream)
    assert st == 0
    return H, tau


def _noalloc(lib, A):
    batch, n, _ = A.shape
    H = torch.empty_like(A)
    tau = torch.empty(batch, n, device=A.device)
    st = lib.qrb_geqrf_f32_noalloc(A.data_ptr(), H.data_ptr(), tau.data_ptr(), batch, n,
                                   torch.cuda.current_stream().cuda_stream)
    assert st == 0
    return H, tau


@pytest.mark.parametrize("batch,n", [(16, 200), (3, 1100), (64, 48)])
def test_noalloc_matches_regular_twice(lib, batch, n):
    g = torch.Generator(device="cuda").manual_seed(n)
    for call in range(2):
        A = torch.randn(batch, n, n, device="cuda", generator=g)
        H_ref, tau_ref = _regular(lib, A)
        H, tau = _noalloc(lib, A)
        torch.cuda.synchronize()
        scale = A.abs().max().item()
        tol = TOL_H * max(1.0, n / 256)
        assert (H - H_ref).abs().max().item() <= tol * scale, call
        assert (tau - tau_ref).abs().max().item() <= tol, call


def test_noalloc_rejects_batch_beyond_scratch(lib):
    A = torch.empty(1, 128, 128, device="cuda")
    # 2049 matrices need more than the 8 MiB of T scratch; rejected before any launch.
    st = lib.qrb_geqrf_f32_noalloc(A.data_ptr(), A.data_ptr(), A.data_ptr(), 2049, 128,
                                   torch.cuda.current_stream().cuda_stream)
    assert st == 2
    # Batches whose T scratch size would wrap a 64-bit product, and batches beyond the
    # 2^31 cap the other entry points enforce (n <= 64 too), are rejected the same way
    # and leave a message in qrb_last_error.
    for batch, n in ((1 << 62, 128), ((1 << 31) + 1, 32), ((1 << 31) + 1, 128)):
        st = lib.qrb_geqrf_f32_noalloc(A.data_ptr(), A.data_ptr(), A.data_ptr(), batch, n,
                                       torch.cuda.current_stream().cuda_stream)
        assert st == 2, (batch, n)
        buf = ctypes.create_string_buffer(256)
        assert lib.qrb_last_error(buf, len(buf)) == 2
        assert b"batch" in buf.value
