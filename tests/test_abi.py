"""CPU: the C-ABI library loads, exports what include/qrb200.h declares, and
validates arguments on the host before touching a device."""
import ctypes
import re
from pathlib import Path

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "qrb200.h"


@pytest.fixture(scope="module")
def lib():
    import build  # linalg-gpu-comp_b200/build.py
    build.build()
    from qr_b200 import _lib
    return _lib.lib()


def declared_symbols():
    text = HEADER.read_text()
    return re.findall(r"QRB_API\s+[\w\s\*]+?\b(qrb_\w+)\s*\(", text)


def test_header_declares_the_api():
    assert set(declared_symbols()) == {
        "qrb_version", "qrb_status_string", "qrb_last_error", "qrb_workspace_size",
        "qrb_geqrf_f32", "qrb_orgqr_f32", "qrb_qr_f32", "qrb_geqrf_f32_noalloc", "qrb_device_error",
        "qrb_host_workspace_size", "qrb_qr_f32_host", "qrb_kernel_launches", "qrb_kernel_timing",
        "qrb_kernel_timing_report", "qrb_selftest_bounded_wait"}


def test_library_exports_every_declared_symbol(lib):
    from qr_b200 import _lib
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, name


def test_version_and_status_strings(lib):
    assert lib.qrb_version() >= 100
    assert lib.qrb_status_string(0) == b"ok"
    assert b"workspace" in lib.qrb_status_string(3)
    assert lib.qrb_status_string(99) == b"unknown status"


def _wide_floats(batch, n, sms=148):
    """Wide-path scratch (csrc/qrb_wide.cu wide_ws_floats): block T factors, two V and two
    W2 piece arrays, and the Y partials of the largest row-chunk split."""
    al = lambda x: (x + 63) // 64 * 64
    nblk = (n + 127) // 128
    ymax = 0
    for K in range(0, n, 128):
        m = n - K
        bw = min(128, n - K)
        for cend in (n, K + bw):        # full-width product and the Gram-only one
            nstrips = (cend - K + 127) // 128
            ns = max(1, min(-(-2 * sms // (nstrips * batch)), (m + 511) // 512, 8))
            chunk = (-(-m // ns) + 31) // 32 * 32
            ns = -(-m // chunk)
            ymax = max(ymax, ns * batch * nblk * 128 * 128)
    return al(nblk * batch * 128 * 128) + 4 * al(batch * n * 128) + al(ymax)


def _ws(batch, n):
    al = lambda x: (x + 255) // 256 * 256
    t = -(-n // 32) * batch * 4096
    if n <= 64:
        return 0
    b = t
    if n % 4 == 0:
        b = al(b) + (batch * n * 32 + 8 * batch * (-(-n // 64)) * 64 * 32) * 4
    if n % 4 == 0 and n >= 256:
        b = al(b) + _wide_floats(batch, n) * 4
    return b


@pytest.mark.parametrize("batch,n,expect", [
    (10, 1, 0), (10, 64, 0), (10, 65, 3 * 10 * 32 * 32 * 4),
    # T factors + (n % 4 == 0) W2 (fp32) + 8 row-chunk W^T partials
    (7, 128, 4 * 7 * 4096 + (1 + 8) * 7 * 128 * 32 * 4),
    (3, 100, 4 * 3 * 4096 + (3 * 100 * 32 + 8 * 3 * 128 * 32) * 4),
    # n >= 256, n % 4 == 0: plus the wide-block scratch
    (7, 512, _ws(7, 512)), (32, 2048, _ws(32, 2048)), (2, 260, _ws(2, 260)), (2, 258, _ws(2, 258)),
    (1, 4097, _ws(1, 4097)), (1, 8192, _ws(1, 8192)), (1, 8193, 0), (-1, 100, 0)])
def test_workspace_size(lib, batch, n, expect):
    assert lib.qrb_workspace_size(batch, n) == expect


def test_wide_workspace_components():
    # b32_n2048: 16 blocks of T (8 MiB each... 2 MiB per block at batch 32), V/W2 pieces 32 MiB each
    assert _wide_floats(32, 2048) >= 16 * 32 * 128 * 128 + 4 * 32 * 2048 * 128
    assert _ws(2, 258) == 9 * 2 * 4096          # n % 4 != 0: T factors only (SIMT update)


def _err(lib):
    buf = ctypes.create_string_buffer(256)
    st = lib.qrb_last_error(buf, 256)
    return st, buf.value.decode()


FAKE = 0x10000  # a 256-byte aligned non-null address; never dereferenced (checks fail first or batch == 0)


def test_argument_errors_are_statuses(lib):
    # null pointers
    assert lib.qrb_geqrf_f32(None, FAKE, FAKE, 4, 32, None, 0, None) == 1
    assert "A is null" in _err(lib)[1]
    assert lib.qrb_qr_f32(FAKE, FAKE, FAKE, None, 4, 32, None, 0, None) == 1
    # bad sizes
    assert lib.qrb_geqrf_f32(FAKE, FAKE, FAKE, 4, 0, None, 0, None) == 1
    assert lib.qrb_geqrf_f32(FAKE, FAKE, FAKE, -1, 8, None, 0, None) == 1
    assert lib.qrb_geqrf_f32(FAKE, FAKE, FAKE, 4, 8200, None, 0, None) == 2
    assert "QRB_MAX_N" in _err(lib)[1]
    # workspace
    assert lib.qrb_geqrf_f32(FAKE, FAKE, FAKE, 4, 128, None, 0, None) == 3
    assert lib.qrb_orgqr_f32(FAKE, FAKE, FAKE + 256, 4, 128, FAKE, 16, None) == 3
    assert lib.qrb_geqrf_f32(FAKE, FAKE, FAKE, 4, 128, FAKE + 16, 1 << 20, None) == 1
    # alignment of matrices
    assert lib.qrb_geqrf_f32(FAKE + 4, FAKE, FAKE, 4, 32, None, 0, None) == 1
    assert "aligned" in _err(lib)[1]
    # aliasing
    assert lib.qrb_qr_f32(FAKE, FAKE, FAKE, FAKE, 4, 32, None, 0, None) == 1
    assert lib.qrb_orgqr_f32(FAKE, FAKE, FAKE, 4, 32, None, 0, None) == 1
    st, msg = _err(lib)
    assert st == 1 and "alias" in msg


def test_empty_batch_is_a_no_op(lib):
    # batch == 0 returns before any CUDA call, so it succeeds without a device.
    assert lib.qrb_geqrf_f32(FAKE, FAKE, FAKE, 0, 32, None, 0, None) == 0
    assert lib.qrb_qr_f32(FAKE, FAKE, FAKE, FAKE + 256, 0, 300, None, 0, None) == 0


def test_kernel_launch_count(lib):
    """qrb_kernel_launches mirrors the dispatch: one fused kernel for n <= 64; otherwise a
    panel per 32 columns and, per block update, wpart + update (+ w2 when the W^T
    reduction is split over row chunks, i.e. blocks taller than 512 rows at small batch),
    or one SIMT launch when n % 4 != 0."""
    assert lib.qrb_kernel_launches(4096, 64, 1) == 1
    assert lib.qrb_kernel_launches(7, 1, 0) == 1
    assert lib.qrb_kernel_launches(1, 256, 1) == 8 + (7 + 8) * 2
    assert lib.qrb_kernel_launches(1, 256, 0) == 8 + 7 * 2
    assert lib.qrb_kernel_launches(1, 258, 1) == 9 + 8 + 9
    n32 = lib.qrb_kernel_launches(32, 2048, 1)
    assert 64 + 127 * 2 < n32 <= 64 + 127 * 3
    assert lib.qrb_kernel_launches(4096, 2048, 1) == 64 + 127 * 2   # wide batch: no split
    assert lib.qrb_kernel_launches(0, 256, 1) == 0
    assert lib.qrb_kernel_launches(1, 8200, 1) == 0


def test_kernel_launch_count_bounds(lib):
    """For every n the count is one fused launch (n <= 64) or np panels plus 1 (SIMT),
    2 or 3 (tensor core) launches per block update; geqrf alone has np - 1 updates."""
    for n in range(1, 4097):
        for batch in (1, 7, 64, 640, 4096):
            full, geqrf = lib.qrb_kernel_launches(batch, n, 1), lib.qrb_kernel_launches(batch, n, 0)
            if n <= 64:
                assert full == geqrf == 1
                continue
            np_ = (n + 31) // 32
            lo, hi = (1, 1) if n % 4 else (2, 3)
            assert np_ + lo * (2 * np_ - 1) <= full <= np_ + hi * (2 * np_ - 1), (batch, n, full)
            assert np_ + lo * (np_ - 1) <= geqrf <= np_ + hi * (np_ - 1), (batch, n, geqrf)
            assert geqrf < full


def test_compiled_call_path_loads():
    """The compiled torch call path (qr_b200/_entry.cpp) is built next to the library,
    links it, and exposes the two hot calls (no GPU needed to load it)."""
    from qr_b200 import ops
    assert ops._entry is not None, "qr_b200/_entry is not built"
    assert callable(ops._fast().geqrf) and callable(ops._fast().qr)


def test_python_ops_reject_cpu_and_wrong_dtype():
    import torch
    from qr_b200 import custom_kernel, form_q
    with pytest.raises(ValueError, match="CUDA"):
        custom_kernel(torch.randn(2, 8, 8))
    with pytest.raises(TypeError):
        custom_kernel(torch.randn(2, 8, 8, dtype=torch.float64).to("meta"))
    with pytest.raises(ValueError):
        form_q(torch.randn(2, 8, 8), torch.randn(2, 8))


def test_host_pipeline_workspace_and_argument_checks(lib):
    """qrb_qr_f32_host: chunked workspace sizing and the checks made before any CUDA call."""
    def slot(cb, n, with_q):
        a = lambda x: (x + 255) // 256 * 256
        mat = a(cb * n * n * 4)
        return mat + a(cb * n * 4) + (mat if with_q else 0) + a(lib.qrb_workspace_size(cb, n))
    # n <= 128: 8 chunks; 3 device slots of one chunk each.
    assert lib.qrb_host_workspace_size(4096, 64, 1) == 3 * slot(512, 64, True)
    assert lib.qrb_host_workspace_size(4096, 64, 0) == 3 * slot(512, 64, False)
    assert lib.qrb_host_workspace_size(512, 256, 1) == 3 * slot(128, 256, True)      # 4 chunks
    assert lib.qrb_host_workspace_size(256, 512, 1) == 3 * slot(64, 512, True)
    assert lib.qrb_host_workspace_size(32, 2048, 1) == 3 * slot(16, 2048, True)      # 2 chunks
    assert lib.qrb_host_workspace_size(3, 64, 1) == 3 * slot(1, 64, True)            # batch < chunks
    assert lib.qrb_host_workspace_size(0, 64, 1) == 0
    assert lib.qrb_host_workspace_size(4, 0, 1) == 0
    assert lib.qrb_qr_f32_host(FAKE, FAKE, FAKE, None, 0, 64, None, 0, None) == 0   # empty batch
    assert lib.qrb_qr_f32_host(None, FAKE, FAKE, None, 4, 64, None, 0, None) == 1
    assert lib.qrb_qr_f32_host(FAKE, FAKE, FAKE, FAKE, 4, 64, None, 0, None) == 1   # Q aliases A
    assert lib.qrb_qr_f32_host(FAKE, FAKE + 64, FAKE + 128, None, 4, 8200, None, 0, None) == 2
    need = lib.qrb_host_workspace_size(4, 64, 0)
    assert lib.qrb_qr_f32_host(FAKE, FAKE, FAKE + 64, None, 4, 64, FAKE, need - 1, None) == 3
    assert lib.qrb_qr_f32_host(FAKE, FAKE, FAKE + 64, None, 4, 64, FAKE + 16, need, None) == 1
    st, msg = _err(lib)
    assert "256-byte" in msg


def test_qr_host_rejects_device_and_bad_shapes():
    import torch
    from qr_b200 import qr_host
    with pytest.raises(ValueError):
        qr_host(torch.randn(2, 8, 7))
    with pytest.raises(ValueError):
        qr_host(torch.randn(2, 8, 8, dtype=torch.float64))
