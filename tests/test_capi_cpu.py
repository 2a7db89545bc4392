"""The C-ABI library without a GPU: it loads, exports every entry point the
header declares, and its argument checks fail cleanly before any device work."""

from __future__ import annotations

import ctypes
import re

import pytest

from repercep_runtime_b200 import _lib


@pytest.fixture(scope="module")
def lib():
    from repercep_runtime_b200 import build

    build.build()  # no-op when up to date; nvcc cross-compiles without a GPU
    return _lib.load()


def _declared_symbols() -> set[str]:
    text = _lib.HEADER_PATH.read_text()
    return set(re.findall(r"^\s*(?:int|float|const char\*)\s+(rp_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_expected_entry_points():
    syms = _declared_symbols()
    for name in ("rp_quant_fp8_e4m3", "rp_quant_fp8_e4m3_ex", "rp_quant_fp8_e4m3_noalloc",
                 "rp_attn_fp8_fwd", "rp_attn_fp8_fwd_ex", "rp_attn_fp8_fwd_chunked",
                 "rp_attn_fp8_prefix_decode", "rp_last_error", "rp_attn_rescale_tau"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    for name in sorted(_declared_symbols()):
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_abi_version(lib):
    assert lib.rp_abi_version() == _lib.ABI_VERSION


def test_workspace_size_is_host_only(lib):
    n = ctypes.c_size_t(0)
    assert lib.rp_quant_workspace_bytes(3, 2, 32, 8192, 128, 0, ctypes.byref(n)) == 0
    assert n.value == 3 * 2 * 32 * 64 * 4
    assert lib.rp_quant_workspace_bytes(3, 2, 32, 8192, 128, 1, ctypes.byref(n)) == 0
    assert n.value == 0
    assert lib.rp_quant_workspace_bytes(3, 2, 32, 8192, 128, 7, ctypes.byref(n)) == -1


def test_argument_errors_are_reported_not_thrown(lib):
    strides = _lib.i64_array([0, 0, 0, 1])
    ptrs = _lib.ptr_array([0])
    rc = lib.rp_quant_fp8_e4m3(4, ptrs, strides, 1, 1, 1, 128, 0, ptrs, ptrs, None, 0, None)
    assert rc == -1 and b"num_tensors" in lib.rp_last_error()
    rc = lib.rp_quant_fp8_e4m3(1, ptrs, strides, 1, 1, 1, 96, 0, ptrs, ptrs, None, 0, None)
    assert rc == -2 and b"head_dim" in lib.rp_last_error()
    out_strides = _lib.i64_array([1, 1, 1, 1])
    rc = lib.rp_attn_fp8_fwd(None, None, None, None, None, None, 0, 1, 1, 128, 128, 128, 0.0, 0, 0,
                             None, out_strides, None)
    assert rc == -1 and b"null" in lib.rp_last_error()
    dummy = 1 << 20
    rc = lib.rp_attn_fp8_fwd(dummy, dummy, dummy, dummy, dummy, dummy, 0, 1, 1, 128, 128, 64, 0.0, 0,
                             0, dummy, out_strides, None)
    assert rc == -2 and b"head_dim" in lib.rp_last_error()
    rc = lib.rp_attn_fp8_prefix_decode(*([dummy] * 10), 4, 3, 512, 32, 128, 0.0, 0, dummy,
                                       _lib.i64_array([1, 1, 1]), None)
    assert rc == -2 and b"divide 128" in lib.rp_last_error()


def test_native_error_carries_the_message(lib):
    with pytest.raises(_lib.NativeError, match="RP_ERR_INVALID"):
        _lib.check("rp_quant_workspace_bytes",
                   lib.rp_quant_workspace_bytes(0, 1, 1, 1, 1, 0, ctypes.byref(ctypes.c_size_t())))


def test_extended_entry_points_check_dtype_rows_and_head_dim(lib):
    dummy = 1 << 20
    strides = _lib.i64_array([0, 0, 0, 1])
    ptrs = _lib.ptr_array([dummy])
    # quantizer: unknown input dtype, rows narrower than D or not a multiple of 16
    rc = lib.rp_quant_fp8_e4m3_ex(1, ptrs, strides, 1, 1, 1, 64, 7, 0, ptrs, 64, ptrs, None, 0, None)
    assert rc == -2 and b"dtype" in lib.rp_last_error()
    rc = lib.rp_quant_fp8_e4m3_ex(1, ptrs, strides, 1, 1, 1, 64, 1, 0, ptrs, 32, ptrs, None, 0, None)
    assert rc == -1 and b"out_row_bytes" in lib.rp_last_error()
    rc = lib.rp_quant_fp8_e4m3_ex(1, ptrs, strides, 1, 1, 1, 64, 1, 0, ptrs, 136, ptrs, None, 0, None)
    assert rc == -1 and b"out_row_bytes" in lib.rp_last_error()
    out_strides = _lib.i64_array([1024, 1024, 64, 1])
    args = [dummy] * 6

    def attn(D, row, dtype):  # type: ignore[no-untyped-def]
        return lib.rp_attn_fp8_fwd_ex(*args, 0, 1, 1, 128, 128, D, row, 0.0, 0, 0, dummy,
                                      out_strides, dtype, None)

    assert attn(96, 128, 0) == -2 and b"head_dim" in lib.rp_last_error()
    assert attn(64, 64, 0) == -2 and b"128 bytes" in lib.rp_last_error()   # D <= 128 reads 128-byte rows
    assert attn(256, 128, 0) == -2 and b"256 bytes" in lib.rp_last_error()
    assert attn(128, 128, 5) == -2 and b"dtype" in lib.rp_last_error()
    # the plain entry point still takes only D = 128
    rc = lib.rp_attn_fp8_fwd(*args, 0, 1, 1, 128, 128, 256, 0.0, 0, 0, dummy, out_strides, None)
    assert rc == -2 and b"_ex" in lib.rp_last_error()


def test_gemm_entry_points_check_shapes_and_pitches(lib):
    dummy = 1 << 20
    # the reference-compatible entry point needs 16-byte rows (K, N multiples of 16)
    assert lib.rp_fp8_gemm(dummy, dummy, dummy, 1.0, 1.0, 16, 16, 40, None) == -3
    assert b"multiples of 16" in lib.rp_last_error()

    def ex(lda, ldb, layout, out_dtype=0, M=16, N=16, K=32, a=dummy):  # type: ignore[no-untyped-def]
        return lib.rp_fp8_gemm_ex(a, lda, dummy, ldb, layout, None, 0, 1.0, None, 0, 1.0, None,
                                  dummy, N, out_dtype, M, N, K, None)

    assert ex(32, 32, 2) == -1 and b"b_layout" in lib.rp_last_error()
    assert ex(32, 32, 0, out_dtype=4) == -2 and b"dtype" in lib.rp_last_error()
    assert ex(16, 32, 1) == -1 and b"shorter" in lib.rp_last_error()      # lda < K
    assert ex(40, 48, 1) == -3 and b"16 bytes" in lib.rp_last_error()     # lda % 16
    assert ex(32, 32, 0, a=None) == -1 and b"non-null" in lib.rp_last_error()
    assert ex(32, 32, 0, M=-1) == -1
    assert ex(32, 32, 0, M=0) == 0  # empty output: nothing to launch
    big = 2**31 - 1
    rc = lib.rp_fp8_gemm_ex(dummy, 16, dummy, 16, 1, None, 0, 1.0, None, 0, 1.0, None, dummy, big, 0,
                            big, big, 16, None)
    assert rc == -2 and b"too large" in lib.rp_last_error()
    # row quantizer
    assert lib.rp_quant_fp8_rows(dummy, 16, 0, 4, 12, dummy, 16, dummy, None) == -2  # cols % 8
    assert lib.rp_quant_fp8_rows(dummy, 16, 3, 4, 16, dummy, 16, dummy, None) == -2  # dtype
    assert lib.rp_quant_fp8_rows(dummy + 8, 16, 0, 4, 16, dummy, 16, dummy, None) == -3
    assert lib.rp_quant_fp8_rows(dummy, 16, 0, 4, 16, dummy + 4, 16, dummy, None) == -3
    assert lib.rp_quant_fp8_rows(dummy, 16, 0, 0, 16, dummy, 16, dummy, None) == 0


def test_rescale_threshold_default(lib, monkeypatch):
    # read once per process from REPERCEP_B200_RESCALE_TAU; the default is 1
    import os

    if "REPERCEP_B200_RESCALE_TAU" not in os.environ:
        assert lib.rp_attn_rescale_tau() == 1.0


def test_wait_selftest_limit_is_bounded(lib):
    # checked before any device work: no limit above the kernels' own, none <= 0
    assert lib.rp_selftest_wait_timeout(0, None) == -1
    assert lib.rp_selftest_wait_timeout(10**12, None) == -1 and b"limit_cycles" in lib.rp_last_error()
