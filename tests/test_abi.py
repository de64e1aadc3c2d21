"""The C-ABI library loads and exports what include/specdecode_cuda.h
declares.  CPU only: these calls validate arguments and return before any
device work."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from specdecode_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "specdecode_cuda.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"SDC_API\s+[\w\s\*]+?\b(sdc_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return _lib.load_library()


def test_header_declares_the_loader_symbol_list():
    assert declared_symbols() == sorted(_lib.EXPORTED_SYMBOLS)


def test_every_declared_symbol_is_exported(lib):
    for name in declared_symbols():
        assert hasattr(lib.handle, name), name


def test_no_undeclared_sdc_symbols_are_exported(lib):
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", lib.path], capture_output=True, text=True, check=True)
    exported = sorted({line.split()[-1] for line in out.stdout.splitlines() if " T sdc_" in line})
    assert exported == declared_symbols()


def test_abi_version_and_status_strings(lib):
    assert lib.handle.sdc_abi_version() == _lib.ABI_VERSION == 0x00020003
    assert lib.status_string(0) == "ok"
    assert lib.status_string(3) == "non-finite value"
    assert lib.status_string(10) == "invalid quantization scale"
    assert lib.status_string(999) == "unknown status"


def test_host_validation_rejects_before_device_work(lib):
    h = lib.handle
    # reference conventions: null arguments and empty vectors are rejected first
    assert h.sdc_quantize_symmetric_int8_f64(None, 4, None, None) == _lib.STATUS_NULL_ARGUMENT
    values = (ctypes.c_double * 1)(1.0)
    out = (ctypes.c_int8 * 1)()
    scale = ctypes.c_double()
    assert h.sdc_quantize_symmetric_int8_f64(values, 0, out, ctypes.byref(scale)) == _lib.STATUS_INVALID_SIZE
    codes = (ctypes.c_int8 * 1)(1)
    dq = (ctypes.c_double * 1)(8.0)
    assert h.sdc_dequantize_symmetric_int8_f64(codes, 1, 0.0, dq) == _lib.STATUS_INVALID_SCALE
    assert dq[0] == 8.0  # untouched on error
    assert h.sdc_dequantize_symmetric_int8_f64(codes, 1, -1.0, dq) == _lib.STATUS_INVALID_SCALE
    assert h.sdc_quantize_append(None, 0, 1, None, None, 0, 0, 0, 0, 0, None, None, None, 0) == \
        _lib.STATUS_NULL_ARGUMENT
    pool = _lib.PagePool(16, 16, 16, 16, 4, 2, 1, 1, 24, 48, 48, 48, 2, 2, 2)
    status = ctypes.c_int32()
    assert h.sdc_rollback(ctypes.byref(pool), None, 0, None, ctypes.byref(status), 0) == _lib.STATUS_UNSUPPORTED
    # the attention wait test hook takes only stall 0 or 1; (0, 0) restores the defaults
    assert h.sdc_test_attention_waits(0, 2) == _lib.STATUS_INVALID_ARGUMENT
    assert h.sdc_test_attention_waits(0, 0) == _lib.STATUS_OK


def test_workspace_sizing_is_host_only(lib):
    size = ctypes.c_size_t()
    assert lib.handle.sdc_paged_attention_workspace_size(32, 32, 8, 128, 5, 8192, ctypes.byref(size)) == 0
    assert size.value > 0
    assert lib.handle.sdc_paged_attention_workspace_size(1, 6, 4, 128, 5, 100, ctypes.byref(size)) == \
        _lib.STATUS_INVALID_ARGUMENT
    assert lib.handle.sdc_paged_attention_workspace_size(1, 8, 8, 128, 9, 8, ctypes.byref(size)) == \
        _lib.STATUS_INVALID_SIZE


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(_lib.NativeLibraryNotFound):
        _lib.load_library(tmp_path / "does-not-exist.so")


def test_sampling_entry_points_validate_on_the_host(lib):
    """Null pointers, sizes, dtypes and strides are refused before any launch."""
    h = lib.handle
    buf = ctypes.c_void_p(16)  # never dereferenced: every call below fails validation first
    assert h.sdc_sample_categorical_rows(None, _lib.DTYPE_F64, 1, 4, 4, buf, buf, None, 0) == \
        _lib.STATUS_NULL_ARGUMENT
    assert h.sdc_sample_categorical_rows(buf, _lib.DTYPE_BF16, 1, 4, 4, buf, buf, None, 0) == \
        _lib.STATUS_UNSUPPORTED
    assert h.sdc_sample_categorical_rows(buf, _lib.DTYPE_F64, 0, 4, 4, buf, buf, None, 0) == \
        _lib.STATUS_INVALID_SIZE
    assert h.sdc_sample_categorical_rows(buf, _lib.DTYPE_F64, 1, 4, 3, buf, buf, None, 0) == \
        _lib.STATUS_INVALID_SIZE
    assert h.sdc_sample_categorical_rows(buf, _lib.DTYPE_F64, 1, (1 << 21) + 1, 1 << 22, buf, buf, None, 0) == \
        _lib.STATUS_UNSUPPORTED
    assert h.sdc_normalize_rows(buf, _lib.DTYPE_F32, 2, 8, 8, None, 8, None, 0) == _lib.STATUS_NULL_ARGUMENT
    assert h.sdc_residual_weights_rows(buf, None, _lib.DTYPE_F32, 2, 8, 8, 8, buf, 8, None, 0) == \
        _lib.STATUS_NULL_ARGUMENT
    assert h.sdc_acceptance_probabilities_rows(buf, buf, _lib.DTYPE_F32, 2, 8, 8, 8, None, buf, None, 0) == \
        _lib.STATUS_NULL_ARGUMENT
    assert h.sdc_first_rejection_rows(buf, buf, 0, 4, 4, buf, None, 0) == _lib.STATUS_INVALID_SIZE
    assert h.sdc_first_rejection_rows(buf, buf, 2, 4, 3, buf, None, 0) == _lib.STATUS_INVALID_SIZE
    out = ctypes.c_void_p(16)
    assert h.sdc_speculative_verify(None, out, out, out, None, None, 0) == _lib.STATUS_NULL_ARGUMENT
    # target sequence stride too small for proposals + 1 rows
    batch = _lib.VerifyBatch(16, 16, _lib.DTYPE_F32, 2, 3, 100, 300, 100, 300, 100, 16, 3, 16, 4, None, None)
    assert h.sdc_speculative_verify(ctypes.byref(batch), out, out, out, None, None, 0) == _lib.STATUS_INVALID_SIZE
    # uniform stride must hold proposals + 1 draws
    batch = _lib.VerifyBatch(16, 16, _lib.DTYPE_F32, 2, 3, 100, 400, 100, 300, 100, 16, 3, 16, 3, None, None)
    assert h.sdc_speculative_verify(ctypes.byref(batch), out, out, out, None, None, 0) == _lib.STATUS_INVALID_SIZE
    assert lib.status_string(_lib.STATUS_INVALID_UNIFORM) == "uniform must be finite and in [0, 1)"
    assert lib.status_string(_lib.STATUS_ZERO_MASS) == "zero probability mass"


def test_page_allocator_entry_points_validate_on_the_host(lib):
    h = lib.handle
    size = ctypes.c_size_t()
    assert h.sdc_pages_append_workspace_size(4, 100, 16, ctypes.byref(size)) == 0 and size.value > 0
    assert h.sdc_pages_append_workspace_size(0, 100, 16, ctypes.byref(size)) == _lib.STATUS_INVALID_SIZE
    assert h.sdc_pages_append_workspace_size(1025, 100, 16, ctypes.byref(size)) == _lib.STATUS_INVALID_SIZE
    alloc = _lib.PageAllocator(None, 16, 16, 16, 16, 16, 16, 64, 16, 4, 8)
    buf = ctypes.c_void_p(16)
    assert h.sdc_pages_append(ctypes.byref(alloc), None, buf, buf, 1, 1, buf, buf, 64, None, 0) == \
        _lib.STATUS_NULL_ARGUMENT
    assert h.sdc_pages_truncate(ctypes.byref(alloc), None, buf, buf, 1, 1, None, 0) == _lib.STATUS_NULL_ARGUMENT
    assert h.sdc_pages_fork(ctypes.byref(alloc), buf, buf, 1, None, 0) == _lib.STATUS_NULL_ARGUMENT
    alloc = _lib.PageAllocator(16, 16, 16, 16, 16, 16, 16, 0, 16, 4, 8)
    assert h.sdc_pages_fork(ctypes.byref(alloc), buf, buf, 1, None, 0) == _lib.STATUS_INVALID_SIZE


def test_head_gather_entry_points_validate_on_the_host(lib):
    """The fused head gather refuses bad rank / world / epoch and null
    destination arrays before any device work; the peer-buffer helpers
    refuse null and short arguments."""
    h = lib.handle
    pool = _lib.PagePool(16, 16, 16, 16, 4, 2, 1, 1, 128, 2048, 2048, 2048, 16, 16, 16)
    buf = ctypes.c_void_p(256)  # never dereferenced
    outs = (ctypes.c_void_p * 2)(256, 512)
    flags = (ctypes.c_void_p * 2)(1024, 2048)
    status = ctypes.c_void_p(4096)

    def call(outs_, flags_, world, rank, epoch):
        return h.sdc_paged_verify_attention_gather(ctypes.byref(pool), 0, buf, _lib.DTYPE_BF16, 1, 4, 1, buf, 1,
                                                   buf, 16, outs_, flags_, world, rank, epoch, buf, 1 << 20,
                                                   status, 0)

    assert call(None, flags, 2, 0, 1) == _lib.STATUS_NULL_ARGUMENT
    assert call(outs, None, 2, 0, 1) == _lib.STATUS_NULL_ARGUMENT
    assert call(outs, flags, 9, 0, 1) == _lib.STATUS_INVALID_ARGUMENT
    assert call(outs, flags, 0, 0, 1) == _lib.STATUS_INVALID_ARGUMENT
    assert call(outs, flags, 2, 2, 1) == _lib.STATUS_INVALID_ARGUMENT
    assert call(outs, flags, 2, -1, 1) == _lib.STATUS_INVALID_ARGUMENT
    assert call(outs, flags, 2, 0, 0) == _lib.STATUS_INVALID_ARGUMENT
    misaligned = (ctypes.c_void_p * 2)(256, 520)
    assert call(misaligned, flags, 2, 0, 1) == _lib.STATUS_MISALIGNED
    ptr = ctypes.c_void_p()
    assert h.sdc_peer_buffer_alloc(64, None) == _lib.STATUS_NULL_ARGUMENT
    assert h.sdc_peer_buffer_alloc(0, ctypes.byref(ptr)) == _lib.STATUS_INVALID_SIZE
    handle = (ctypes.c_char * _lib.PEER_HANDLE_BYTES)()
    assert h.sdc_peer_buffer_export(None, handle, len(handle)) == _lib.STATUS_NULL_ARGUMENT
    assert h.sdc_peer_buffer_export(buf, handle, 8) == _lib.STATUS_INVALID_SIZE
    assert h.sdc_peer_buffer_open(handle, 8, ctypes.byref(ptr)) == _lib.STATUS_INVALID_SIZE
    assert h.sdc_peer_buffer_open(None, len(handle), ctypes.byref(ptr)) == _lib.STATUS_NULL_ARGUMENT
    assert h.sdc_peer_buffer_free(None) == _lib.STATUS_OK
    assert h.sdc_peer_buffer_close(None) == _lib.STATUS_OK


COMPAT_HEADER = Path(__file__).resolve().parents[1] / "include" / "specdecode_native_compat.h"


def test_reference_native_symbols_are_exported(lib):
    """The nine sd_* names the reference's loader binds (native.py:93-153)
    are declared in the compatibility header and exported, and no others."""
    import subprocess

    declared = sorted(set(re.findall(r"SDC_API\s+[\w\s\*]+?\b(sd_\w+)\s*\(", COMPAT_HEADER.read_text())))
    assert len(declared) == 9
    out = subprocess.run(["nm", "-D", "--defined-only", lib.path], capture_output=True, text=True, check=True)
    exported = sorted({line.split()[-1] for line in out.stdout.splitlines() if " T sd_" in line})
    assert exported == declared
    h = ctypes.CDLL(lib.path)
    h.sd_abi_version.restype = ctypes.c_uint32
    assert h.sd_abi_version() == 0x00010001


def test_reference_loader_accepts_the_library(lib):
    """The reference's own ctypes loader (its _NativeLibrary, unchanged from
    oracle/_ref) loads libspecdecode_cuda.so, checks its ABI version and
    binds every function; its status strings equal the reference library's,
    and the checks that need no device give the reference's statuses."""
    from oracle.reference_runs import ReferenceUnavailable, reference_package

    try:
        reference_package()
    except ReferenceUnavailable as error:
        pytest.skip(str(error))
    from specdecode import native as ref_native

    ours = ref_native._NativeLibrary(lib.path)
    theirs = ref_native._NativeLibrary(str(Path(ref_native.__file__).resolve().parents[1] /
                                           "libspecdecode_native.so"))
    for status in range(12):
        assert ours.handle.sd_status_string(status) == theirs.handle.sd_status_string(status), status
    d = (ctypes.c_double * 3)(0.2, 0.3, 0.5)
    token = ctypes.c_uint64()
    for h in (ours.handle, theirs.handle):
        assert h.sd_sample_categorical_f64(d, 3, 0.5, None) == 1
        assert h.sd_sample_categorical_f64(d, 3, 1.0, ctypes.byref(token)) == 7
        assert h.sd_sample_categorical_f64(d, 0, 0.5, ctypes.byref(token)) == 2
        assert h.sd_normalize_f64(d, 3, None) == 1
        tok = (ctypes.c_uint64 * 1)(0)
        assert h.sd_acceptance_probabilities_f64(d, d, tok, 0, 3, d) == 2
        accepted, index = ctypes.c_size_t(9), ctypes.c_size_t(9)
        assert h.sd_first_rejection_f64(None, None, 0, ctypes.byref(accepted), ctypes.byref(index)) == 0
        assert (accepted.value, index.value) == (0, 0)
