"""ctypes loader for libspecdecode_cuda.so (include/specdecode_cuda.h).

Search order, after the pattern of the reference's loader
(src/specdecode/native.py:57-74): an explicit path, then the
``SPECDECODE_CUDA_LIBRARY`` environment variable, then the library built
in-tree beside this file.  The ABI version must match exactly
(src/specdecode/native.py:87-91).  A missing library raises
``NativeLibraryNotFound``; there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

ABI_VERSION = 0x00020003
PEER_HANDLE_BYTES = 64  # SDC_PEER_HANDLE_BYTES
LIBRARY_NAME = "libspecdecode_cuda.so"
_ENV = "SPECDECODE_CUDA_LIBRARY"

STATUS_OK = 0
STATUS_NULL_ARGUMENT = 1
STATUS_INVALID_SIZE = 2
STATUS_NONFINITE_VALUE = 3
STATUS_NEGATIVE_PROBABILITY = 4
STATUS_ZERO_MASS = 5
STATUS_TOKEN_OUT_OF_RANGE = 6
STATUS_INVALID_UNIFORM = 7
STATUS_OVERFLOW = 8
STATUS_INTERNAL_ERROR = 9
STATUS_INVALID_SCALE = 10
STATUS_CUDA_ERROR = 11
STATUS_UNSUPPORTED = 12
STATUS_MISALIGNED = 13
STATUS_DEVICE_FAULT = 14
STATUS_INVALID_ARGUMENT = 15
STATUS_SCRATCH_EXCEEDED = 16

FAULT_NONFINITE_VALUE = 0x01
FAULT_INVALID_SCALE = 0x02
FAULT_SLOT_RANGE = 0x04
FAULT_BLOCK_RANGE = 0x08
FAULT_CONTEXT_RANGE = 0x10
FAULT_WAIT_TIMEOUT = 0x20
FAULT_TABLE_RANGE = 0x40
FAULT_NEGATIVE_WEIGHT = 0x80
FAULT_ZERO_MASS = 0x100
FAULT_TOKEN_RANGE = 0x200
FAULT_INVALID_UNIFORM = 0x400
FAULT_PROPOSAL_COUNT = 0x800
FAULT_CAPACITY = 0x1000

FAULT_NAMES = {
    FAULT_NONFINITE_VALUE: "non-finite value",
    FAULT_INVALID_SCALE: "quantization scale outside float32",
    FAULT_SLOT_RANGE: "slot outside the page pool",
    FAULT_BLOCK_RANGE: "block id outside the page pool",
    FAULT_CONTEXT_RANGE: "context length outside the block table",
    FAULT_WAIT_TIMEOUT: "a pipeline wait gave up",
    FAULT_TABLE_RANGE: "block-table edit outside the table",
    FAULT_NEGATIVE_WEIGHT: "negative probability",
    FAULT_ZERO_MASS: "zero probability mass",
    FAULT_TOKEN_RANGE: "token out of range",
    FAULT_INVALID_UNIFORM: "uniform must be finite and in [0, 1)",
    FAULT_PROPOSAL_COUNT: "proposal count outside [1, proposals]",
    FAULT_CAPACITY: "the page pool is short of free blocks",
}

# The reference's status for the input a sampling fault bit reports, in the
# order its functions check (native/src/native.cpp:29-41, 113-118, 209-225).
FAULT_STATUS = (
    (FAULT_INVALID_UNIFORM, STATUS_INVALID_UNIFORM),
    (FAULT_TOKEN_RANGE, STATUS_TOKEN_OUT_OF_RANGE),
    (FAULT_NONFINITE_VALUE, STATUS_NONFINITE_VALUE),
    (FAULT_NEGATIVE_WEIGHT, STATUS_NEGATIVE_PROBABILITY),
    (FAULT_ZERO_MASS, STATUS_ZERO_MASS),
    (FAULT_PROPOSAL_COUNT, STATUS_INVALID_SIZE),
)

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2
DTYPE_F64 = 3

EXPORTED_SYMBOLS = (
    "sdc_abi_version",
    "sdc_status_string",
    "sdc_quantize_symmetric_int8_f64",
    "sdc_dequantize_symmetric_int8_f64",
    "sdc_quantize_rows",
    "sdc_quantize_append",
    "sdc_rollback",
    "sdc_paged_attention_workspace_size",
    "sdc_paged_verify_attention",
    "sdc_gather_dequantize",
    "sdc_paged_verify_attention_no_alloc",
    "sdc_paged_verify_attention_gather",
    "sdc_peer_buffer_alloc",
    "sdc_peer_buffer_free",
    "sdc_peer_buffer_export",
    "sdc_peer_buffer_open",
    "sdc_peer_buffer_close",
    "sdc_test_attention_waits",
    "sdc_normalize_rows",
    "sdc_sample_categorical_rows",
    "sdc_residual_weights_rows",
    "sdc_acceptance_probabilities_rows",
    "sdc_first_rejection_rows",
    "sdc_speculative_verify",
    "sdc_pages_append_workspace_size",
    "sdc_pages_append",
    "sdc_pages_truncate",
    "sdc_pages_fork",
)


class NativeLibraryNotFound(OSError):
    """Raised when the CUDA library cannot be located or loaded."""


class NativeBackendError(RuntimeError):
    """Raised when the C ABI rejects a call or a kernel reports a fault."""

    def __init__(self, message: str, *, status: int | None = None, faults: int = 0) -> None:
        super().__init__(message)
        self.status = status
        self.faults = faults


class PagePool(ctypes.Structure):
    _fields_ = [
        ("keys", ctypes.c_void_p),
        ("values", ctypes.c_void_p),
        ("key_scales", ctypes.c_void_p),
        ("value_scales", ctypes.c_void_p),
        ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int64),
        ("num_layers", ctypes.c_int64),
        ("num_heads", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("code_block_stride", ctypes.c_int64),
        ("code_layer_stride", ctypes.c_int64),
        ("code_head_stride", ctypes.c_int64),
        ("scale_block_stride", ctypes.c_int64),
        ("scale_layer_stride", ctypes.c_int64),
        ("scale_head_stride", ctypes.c_int64),
    ]


class TableEdits(ctypes.Structure):
    _fields_ = [
        ("block_tables", ctypes.c_void_p),
        ("table_stride", ctypes.c_int64),
        ("table_rows", ctypes.c_int64),
        ("context_lens", ctypes.c_void_p),
        ("entries", ctypes.c_void_p),
        ("num_entries", ctypes.c_int64),
        ("lengths", ctypes.c_void_p),
        ("num_lengths", ctypes.c_int64),
    ]


class VerifyBatch(ctypes.Structure):
    _fields_ = [
        ("target_rows", ctypes.c_void_p),
        ("draft_rows", ctypes.c_void_p),
        ("dtype", ctypes.c_int),
        ("sequences", ctypes.c_int64),
        ("proposals", ctypes.c_int64),
        ("vocab", ctypes.c_int64),
        ("target_sequence_stride", ctypes.c_int64),
        ("target_row_stride", ctypes.c_int64),
        ("draft_sequence_stride", ctypes.c_int64),
        ("draft_row_stride", ctypes.c_int64),
        ("proposed_tokens", ctypes.c_void_p),
        ("token_stride", ctypes.c_int64),
        ("uniforms", ctypes.c_void_p),
        ("uniform_stride", ctypes.c_int64),
        ("proposal_counts", ctypes.c_void_p),
        ("bonus_allowed", ctypes.c_void_p),
    ]


class PageAllocator(ctypes.Structure):
    _fields_ = [
        ("free_bits", ctypes.c_void_p),
        ("refcount", ctypes.c_void_p),
        ("high_water", ctypes.c_void_p),
        ("block_order", ctypes.c_void_p),
        ("heap_of", ctypes.c_void_p),
        ("block_tables", ctypes.c_void_p),
        ("context_lens", ctypes.c_void_p),
        ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int64),
        ("table_rows", ctypes.c_int64),
        ("table_stride", ctypes.c_int64),
    ]


def fault_message(bits: int) -> str:
    names = [name for bit, name in FAULT_NAMES.items() if bits & bit]
    return ", ".join(names) if names else f"fault bits 0x{bits:x}"


def resolve_library_path(path: str | os.PathLike[str] | None = None) -> str:
    explicit = path or os.environ.get(_ENV)
    if explicit:
        candidate = Path(explicit).expanduser().resolve()
        if not candidate.is_file():
            raise NativeLibraryNotFound(f"CUDA library does not exist: {candidate}")
        return str(candidate)
    candidate = Path(__file__).resolve().parent / LIBRARY_NAME
    if candidate.is_file():
        return str(candidate)
    raise NativeLibraryNotFound(
        f"{LIBRARY_NAME} was not found; build it with "
        "`python llm-inference-accelerator_b200/csrc/build.py` or set " + _ENV)


class CudaLibrary:
    """The loaded C ABI with argument types configured and the ABI checked."""

    def __init__(self, path: str) -> None:
        try:
            self.handle = ctypes.CDLL(path)
        except OSError as error:
            raise NativeLibraryNotFound(f"could not load CUDA library {path}: {error}") from error
        self.path = path
        self._configure()
        version = int(self.handle.sdc_abi_version())
        if version != ABI_VERSION:
            raise NativeBackendError(
                f"CUDA library ABI mismatch: expected 0x{ABI_VERSION:08x}, received 0x{version:08x}")

    def _configure(self) -> None:
        h = self.handle
        vp, i64, u = ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64
        h.sdc_abi_version.argtypes = []
        h.sdc_abi_version.restype = ctypes.c_uint32
        h.sdc_status_string.argtypes = [ctypes.c_int]
        h.sdc_status_string.restype = ctypes.c_char_p
        h.sdc_quantize_symmetric_int8_f64.argtypes = [
            ctypes.POINTER(ctypes.c_double), ctypes.c_size_t, ctypes.POINTER(ctypes.c_int8),
            ctypes.POINTER(ctypes.c_double)]
        h.sdc_quantize_symmetric_int8_f64.restype = ctypes.c_int
        h.sdc_dequantize_symmetric_int8_f64.argtypes = [
            ctypes.POINTER(ctypes.c_int8), ctypes.c_size_t, ctypes.c_double,
            ctypes.POINTER(ctypes.c_double)]
        h.sdc_dequantize_symmetric_int8_f64.restype = ctypes.c_int
        h.sdc_quantize_rows.argtypes = [vp, ctypes.c_int, i64, i64, vp, vp, vp, u]
        h.sdc_quantize_rows.restype = ctypes.c_int
        h.sdc_quantize_append.argtypes = [
            ctypes.POINTER(PagePool), i64, i64, vp, vp, ctypes.c_int, i64, i64, i64, i64, vp,
            ctypes.POINTER(TableEdits), vp, u]
        h.sdc_quantize_append.restype = ctypes.c_int
        h.sdc_rollback.argtypes = [ctypes.POINTER(PagePool), vp, i64, ctypes.POINTER(TableEdits), vp, u]
        h.sdc_rollback.restype = ctypes.c_int
        h.sdc_paged_attention_workspace_size.argtypes = [i64, i64, i64, i64, i64, i64,
                                                         ctypes.POINTER(ctypes.c_size_t)]
        h.sdc_paged_attention_workspace_size.restype = ctypes.c_int
        h.sdc_paged_verify_attention.argtypes = [
            ctypes.POINTER(PagePool), i64, vp, ctypes.c_int, i64, i64, i64, vp, i64, vp, i64, vp, vp,
            ctypes.c_size_t, vp, u]
        h.sdc_paged_verify_attention.restype = ctypes.c_int
        h.sdc_paged_verify_attention_no_alloc.argtypes = [
            ctypes.POINTER(PagePool), i64, vp, ctypes.c_int, i64, i64, i64, vp, i64, vp, i64, vp, vp, u]
        h.sdc_paged_verify_attention_no_alloc.restype = ctypes.c_int
        h.sdc_paged_verify_attention_gather.argtypes = [
            ctypes.POINTER(PagePool), i64, vp, ctypes.c_int, i64, i64, i64, vp, i64, vp, i64,
            ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.c_int32, ctypes.c_int32, ctypes.c_uint32, vp,
            ctypes.c_size_t, vp, u]
        h.sdc_paged_verify_attention_gather.restype = ctypes.c_int
        h.sdc_peer_buffer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
        h.sdc_peer_buffer_alloc.restype = ctypes.c_int
        h.sdc_peer_buffer_free.argtypes = [vp]
        h.sdc_peer_buffer_free.restype = ctypes.c_int
        h.sdc_peer_buffer_export.argtypes = [vp, vp, ctypes.c_size_t]
        h.sdc_peer_buffer_export.restype = ctypes.c_int
        h.sdc_peer_buffer_open.argtypes = [vp, ctypes.c_size_t, ctypes.POINTER(vp)]
        h.sdc_peer_buffer_open.restype = ctypes.c_int
        h.sdc_peer_buffer_close.argtypes = [vp]
        h.sdc_peer_buffer_close.restype = ctypes.c_int
        h.sdc_test_attention_waits.argtypes = [i64, ctypes.c_int32]
        h.sdc_test_attention_waits.restype = ctypes.c_int
        h.sdc_gather_dequantize.argtypes = [
            ctypes.POINTER(PagePool), i64, i64, vp, i64, vp, vp, ctypes.c_int, i64, i64, i64, vp, u]
        h.sdc_gather_dequantize.restype = ctypes.c_int
        h.sdc_normalize_rows.argtypes = [vp, ctypes.c_int, i64, i64, i64, vp, i64, vp, u]
        h.sdc_normalize_rows.restype = ctypes.c_int
        h.sdc_sample_categorical_rows.argtypes = [vp, ctypes.c_int, i64, i64, i64, vp, vp, vp, u]
        h.sdc_sample_categorical_rows.restype = ctypes.c_int
        h.sdc_residual_weights_rows.argtypes = [vp, vp, ctypes.c_int, i64, i64, i64, i64, vp, i64, vp, u]
        h.sdc_residual_weights_rows.restype = ctypes.c_int
        h.sdc_acceptance_probabilities_rows.argtypes = [vp, vp, ctypes.c_int, i64, i64, i64, i64, vp, vp, vp, u]
        h.sdc_acceptance_probabilities_rows.restype = ctypes.c_int
        h.sdc_first_rejection_rows.argtypes = [vp, vp, i64, i64, i64, vp, vp, u]
        h.sdc_first_rejection_rows.restype = ctypes.c_int
        h.sdc_speculative_verify.argtypes = [ctypes.POINTER(VerifyBatch), vp, vp, vp, vp, vp, u]
        h.sdc_speculative_verify.restype = ctypes.c_int
        h.sdc_pages_append_workspace_size.argtypes = [i64, i64, i64, ctypes.POINTER(ctypes.c_size_t)]
        h.sdc_pages_append_workspace_size.restype = ctypes.c_int
        h.sdc_pages_append.argtypes = [ctypes.POINTER(PageAllocator), ctypes.POINTER(PagePool), vp, vp, i64, i64, vp,
                                       vp, ctypes.c_size_t, vp, u]
        h.sdc_pages_append.restype = ctypes.c_int
        h.sdc_pages_truncate.argtypes = [ctypes.POINTER(PageAllocator), ctypes.POINTER(PagePool), vp, vp, i64, i64,
                                         vp, u]
        h.sdc_pages_truncate.restype = ctypes.c_int
        h.sdc_pages_fork.argtypes = [ctypes.POINTER(PageAllocator), vp, vp, i64, vp, u]
        h.sdc_pages_fork.restype = ctypes.c_int

    def status_string(self, status: int) -> str:
        raw = self.handle.sdc_status_string(int(status))
        return raw.decode("utf-8") if raw else f"status {status}"

    def check(self, status: int, operation: str) -> None:
        if status == STATUS_OK:
            return
        raise NativeBackendError(f"CUDA {operation} failed: {self.status_string(status)}", status=status)


_LOCK = threading.Lock()
_CACHED: dict[str, CudaLibrary] = {}


def load_library(path: str | os.PathLike[str] | None = None) -> CudaLibrary:
    resolved = resolve_library_path(path)
    with _LOCK:
        library = _CACHED.get(resolved)
        if library is None:
            library = CudaLibrary(resolved)
            _CACHED[resolved] = library
        return library
