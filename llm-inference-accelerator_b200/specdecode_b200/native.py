"""``NativeKVQuantizer`` over the CUDA library's C ABI.

Keeps the reference's quantizer binding surface (src/specdecode/native.py:
175-219): ``name == "native"``, ``load(path)``, ``library_path``,
``quantize(values) -> QuantizedVector``, ``dequantize(vector) -> tuple``, and
``NativeBackendError`` carrying the ABI status on rejection.  The arithmetic
runs on the GPU through ``sdc_quantize_symmetric_int8_f64`` /
``sdc_dequantize_symmetric_int8_f64``, which take the reference's exact
host-buffer signatures (native/include/specdecode/native.h:93-106).

``quantize_batch`` is an additive device-tensor form: many rows in one launch
with no host round trip.
"""

from __future__ import annotations

import ctypes
import os
from collections.abc import Sequence

from . import _lib
from ._lib import ABI_VERSION, NativeBackendError, NativeLibraryNotFound
from .kv_cache import QuantizedVector

__all__ = ["ABI_VERSION", "NativeBackendError", "NativeLibraryNotFound", "NativeKVQuantizer"]


class NativeKVQuantizer:
    """Per-vector symmetric INT8 quantization executed by the CUDA library."""

    name = "native"

    def __init__(self, library: _lib.CudaLibrary) -> None:
        self._library = library

    @classmethod
    def load(cls, path: str | os.PathLike[str] | None = None) -> "NativeKVQuantizer":
        return cls(_lib.load_library(path))

    @property
    def library_path(self) -> str:
        return self._library.path

    def quantize(self, values: Sequence[float]) -> QuantizedVector:
        source = tuple(values)
        if any(isinstance(value, bool) for value in source):
            raise TypeError("KV values must be real numbers, not booleans")
        inputs = (ctypes.c_double * len(source))(*(float(v) for v in source))
        output = (ctypes.c_int8 * max(1, len(source)))()
        scale = ctypes.c_double()
        status = self._library.handle.sdc_quantize_symmetric_int8_f64(
            inputs, len(source), output, ctypes.byref(scale))
        self._library.check(status, "INT8 quantization")
        return QuantizedVector(tuple(int(v) for v in output[: len(source)]), scale.value)

    def dequantize(self, vector: QuantizedVector) -> tuple[float, ...]:
        if not isinstance(vector, QuantizedVector):
            raise TypeError("dequantization requires a QuantizedVector")
        inputs = (ctypes.c_int8 * len(vector.values))(*vector.values)
        output = (ctypes.c_double * len(vector.values))()
        status = self._library.handle.sdc_dequantize_symmetric_int8_f64(
            inputs, len(vector.values), vector.scale, output)
        self._library.check(status, "INT8 dequantization")
        return tuple(output)

    def quantize_batch(self, rows):
        """Quantize every row of a device tensor ``[n, count]`` (f32/bf16/f16/f64).

        Returns ``(codes int8 [n, count], scales float32 [n], status int32 [n])``
        on the same device; ``status`` uses the reference's status numbers and
        rows with a non-zero status hold unspecified codes.
        """
        import torch

        from .kv_cache import _dtype_code

        if rows.dim() != 2:
            raise ValueError("rows must be a 2-D tensor")
        if rows.device.type != "cuda":
            raise ValueError("rows must be on a CUDA device")
        rows = rows.contiguous()
        n, count = rows.shape
        codes = torch.empty((n, count), dtype=torch.int8, device=rows.device)
        scales = torch.empty((n,), dtype=torch.float32, device=rows.device)
        status = torch.empty((n,), dtype=torch.int32, device=rows.device)
        stream = torch.cuda.current_stream(rows.device)
        self._library.check(self._library.handle.sdc_quantize_rows(
            rows.data_ptr(), _dtype_code(rows.dtype), n, count, codes.data_ptr(), scales.data_ptr(),
            status.data_ptr(), stream.cuda_stream), "row quantization")
        return codes, scales, status
