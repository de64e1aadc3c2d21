"""ORACLE — per-head symmetric INT8 quantizer restated on the CPU.

Test infrastructure only.  Three forms of the same rule:

* ``quantize_vector`` / ``dequantize_vector`` — scalar Python, following
  src/specdecode/kv_cache.py:130-151 (the reference's PythonKVQuantizer) and
  native/src/native.cpp:275-353.  Rounding is half away from zero, as the
  reference's C++ ``std::round`` does (native.cpp:311); the reference's Python
  form ``floor(v + 0.5)`` (kv_cache.py:119-122) agrees with it on every
  quotient of two float32 values.
* ``quantize_rows`` — numpy float64, vectorised over rows.
* ``CQuantizer`` — the C restatement in oracle/quantize_oracle.c, loaded with
  ctypes (built by ``make -C oracle``).

Statuses use the reference's numbering (native/include/specdecode/native.h:25-37).
"""

from __future__ import annotations

import ctypes
import math
import struct
from pathlib import Path

import numpy as np

STATUS_OK = 0
STATUS_NULL_ARGUMENT = 1
STATUS_INVALID_SIZE = 2
STATUS_NONFINITE_VALUE = 3
STATUS_INVALID_SCALE = 10

_HERE = Path(__file__).resolve().parent


def _to_float32(value: float) -> float:
    return struct.unpack("=f", struct.pack("=f", value))[0]


def _round_half_away(value: float) -> int:
    # Exact: floor() and the fractional part of a double are both exact.
    magnitude = abs(value)
    whole = math.floor(magnitude)
    rounded = whole + (1 if magnitude - whole >= 0.5 else 0)
    return int(rounded) if value >= 0.0 else -int(rounded)


def quantize_vector(values) -> tuple[tuple[int, ...], float]:
    """kv_cache.py:130-146 / native.cpp:275-319 for one head vector."""
    source = [float(v) for v in values]
    if not source:
        raise ValueError("a KV head vector cannot be empty")
    if not all(math.isfinite(v) for v in source):
        raise ValueError("KV values must be finite")
    maximum = max(abs(v) for v in source)
    if maximum == 0.0:
        return (0,) * len(source), 0.0
    try:
        scale = _to_float32(maximum / 127.0)
    except OverflowError as error:  # pragma: no cover - float input cannot overflow
        raise ValueError("quantization scale is outside the float32 range") from error
    if not math.isfinite(scale) or scale == 0.0:
        raise ValueError("quantization scale is outside the float32 range")
    codes = tuple(max(-127, min(127, _round_half_away(v / scale))) for v in source)
    return codes, scale


def dequantize_vector(codes, scale: float) -> tuple[float, ...]:
    """kv_cache.py:148-151 / native.cpp:321-353."""
    return tuple(int(c) * float(scale) for c in codes)


def quantize_rows(x: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Quantize every length-D row of ``x`` (``[..., D]``).

    Returns ``(codes int8 [..., D], scales float32 [...], status int32 [...])``.
    Rows with a non-OK status get zero codes and a zero scale here; the
    reference writes nothing for them.
    """
    x = np.asarray(x, dtype=np.float64)
    finite = np.isfinite(x).all(axis=-1)
    safe = np.where(np.isfinite(x), x, 0.0)
    maximum = np.abs(safe).max(axis=-1)
    with np.errstate(over="ignore", under="ignore"):
        scale32 = (maximum / 127.0).astype(np.float32)
    zero = maximum == 0.0
    bad_scale = ~zero & (~np.isfinite(scale32) | (scale32 == 0.0))
    ok = finite & ~bad_scale
    divisor = np.where(ok & ~zero, scale32.astype(np.float64), 1.0)
    y = safe / divisor[..., None]
    magnitude = np.abs(y)
    whole = np.floor(magnitude)
    rounded = whole + (magnitude - whole >= 0.5)
    rounded = np.minimum(rounded, 127.0)
    codes = np.where(y < 0, -rounded, rounded)
    codes = np.where((ok & ~zero)[..., None], codes, 0.0).astype(np.int8)
    scales = np.where(ok & ~zero, scale32, np.float32(0.0)).astype(np.float32)
    status = np.where(~finite, STATUS_NONFINITE_VALUE,
                      np.where(bad_scale, STATUS_INVALID_SCALE, STATUS_OK)).astype(np.int32)
    return codes, scales, status


class CQuantizer:
    """ctypes handle on oracle/_build/liboracle_quant.so (the C restatement)."""

    def __init__(self, path: str | Path | None = None) -> None:
        library = Path(path) if path is not None else _HERE / "_build" / "liboracle_quant.so"
        if not library.is_file():
            raise FileNotFoundError(f"{library} is missing; run `make -C oracle`")
        self.handle = ctypes.CDLL(str(library))
        i8p = ctypes.POINTER(ctypes.c_int8)
        f64p = ctypes.POINTER(ctypes.c_double)
        self.handle.oracle_quantize_f64.argtypes = [f64p, ctypes.c_size_t, i8p, f64p]
        self.handle.oracle_quantize_f64.restype = ctypes.c_int
        self.handle.oracle_dequantize_f64.argtypes = [i8p, ctypes.c_size_t, ctypes.c_double, f64p]
        self.handle.oracle_dequantize_f64.restype = ctypes.c_int
        for name in ("oracle_quantize_rows_f64", "oracle_quantize_rows_f32"):
            fn = getattr(self.handle, name)
            fn.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                           ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
            fn.restype = None

    def quantize(self, values) -> tuple[int, tuple[int, ...], float]:
        source = (ctypes.c_double * len(values))(*[float(v) for v in values])
        out = (ctypes.c_int8 * max(1, len(values)))()
        scale = ctypes.c_double(-1.0)
        status = self.handle.oracle_quantize_f64(source, len(values), out, ctypes.byref(scale))
        return status, tuple(int(v) for v in out[: len(values)]), scale.value

    def quantize_rows(self, x: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        x = np.ascontiguousarray(x)
        if x.dtype == np.float32:
            fn = self.handle.oracle_quantize_rows_f32
        else:
            x = np.ascontiguousarray(x, dtype=np.float64)
            fn = self.handle.oracle_quantize_rows_f64
        count = x.shape[-1]
        rows = x.size // count if count else 0
        codes = np.empty(x.shape, dtype=np.int8)
        scales = np.empty(x.shape[:-1], dtype=np.float32)
        status = np.empty(x.shape[:-1], dtype=np.int32)
        fn(x.ctypes.data, rows, count, codes.ctypes.data, scales.ctypes.data, status.ctypes.data)
        return codes, scales, status


def bits_f32(values: np.ndarray) -> np.ndarray:
    """Bit patterns of float32 values, for bit-exact comparisons."""
    return np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
