"""Device-resident acceptance and sampling for speculative decoding.

The reference's sampling backend (src/specdecode/backends.py:23-51, its
native form src/specdecode/native.py:222-345 over native/src/native.cpp:84-273)
on the kernels of csrc/sampling.cu:

* batched functions over device tensors -- ``normalize_rows``,
  ``sample_rows``, ``residual_rows``, ``acceptance_rows``,
  ``first_rejection_rows`` -- and ``verify_batch``, one verification round of
  the reference decoder (src/specdecode/decoder.py:206-257) for every
  sequence of a batch in two launches;
* ``DeviceSamplingBackend``, the reference's ``SamplingBackend`` protocol
  (same method names, arguments, results and error type as
  ``NativeSamplingBackend``) over the same kernels, one call per row set.

Weights are float32 or float64 device rows; they need not be normalised.
Faults the kernels find (a negative or non-finite weight, a zero-mass row, a
token outside the vocabulary, a uniform outside [0, 1)) are OR-ed into a
device status word.  The batched functions leave that word to the caller
(``status=``), so a decoding loop reads it once per round;
``DeviceSamplingBackend`` reads it after every call and raises
``NativeBackendError`` with the reference's status and message.  There is no
CPU fallback: a missing library raises ``NativeLibraryNotFound``.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence
from dataclasses import dataclass
from typing import Any

from . import _lib

__all__ = [
    "DeviceSamplingBackend",
    "VerificationResult",
    "acceptance_rows",
    "first_rejection_rows",
    "normalize_rows",
    "residual_rows",
    "sample_rows",
    "verify_batch",
]


@dataclass(frozen=True, slots=True)
class VerificationResult:
    """src/specdecode/backends.py:15-20."""

    accepted_count: int
    rejection_index: int | None


def _dtype(t) -> int:
    import torch

    if t.dtype == torch.float32:
        return _lib.DTYPE_F32
    if t.dtype == torch.float64:
        return _lib.DTYPE_F64
    raise TypeError(f"probability rows must be float32 or float64, not {t.dtype}")


def _rows(t, name: str):
    """A 2-D row batch on a CUDA device with unit element stride (rows may be
    strided)."""
    if t.dim() != 2:
        raise ValueError(f"{name} must be [rows, vocab]")
    _on_cuda(t, name)
    if t.stride(1) != 1:
        t = t.contiguous()
    return t


def _on_cuda(t, name: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be on a CUDA device")


def _aux(t, device, dtype):
    """A small per-row input (uniforms, tokens, counts) as a contiguous
    tensor of ``dtype`` on the rows' device (copied there if it is not)."""
    return t.to(device=device, dtype=dtype).contiguous()


def _out(t, shape, dtype, device, name: str):
    """A caller-provided output: exactly the shape, dtype and device the
    launch writes, contiguous."""
    if tuple(t.shape) != tuple(shape) or t.dtype != dtype or t.device != device or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous {dtype} tensor of shape {tuple(shape)} on {device}")
    return t


def _stride(t, dim: int, span: int) -> int:
    """t.stride(dim), or ``span`` where the dimension has one element (its
    stride is then arbitrary, and numpy's added axes give it 0)."""
    return t.stride(dim) if t.shape[dim] > 1 else span


def _status(status, device):
    import torch

    if status is None:
        return torch.zeros(1, dtype=torch.int32, device=device)
    if status.dtype != torch.int32 or status.device != device or status.numel() < 1:
        raise ValueError(f"the status word must be an int32 tensor on {device}")
    return status


def _stream(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def _library(library):
    return library if library is not None else _lib.load_library()


def normalize_rows(weights, *, status=None, library=None):
    """out[r] = weights[r] / sum(weights[r]) in float64 (sd_normalize_f64)."""
    import torch

    lib = _library(library)
    w = _rows(weights, "weights")
    out = torch.empty(w.shape, dtype=torch.float64, device=w.device)
    st = _status(status, w.device)
    lib.check(lib.handle.sdc_normalize_rows(w.data_ptr(), _dtype(w), w.shape[0], w.shape[1],
                                            _stride(w, 0, w.shape[1]), out.data_ptr(), w.shape[1], st.data_ptr(),
                                            _stream(w.device)),
              "row normalisation")
    return out


def sample_rows(weights, uniforms, *, out=None, status=None, library=None):
    """int64 [rows]: per row, the first index whose running weight sum exceeds
    uniform * total (sd_sample_categorical_f64); -1 for a faulted row."""
    import torch

    lib = _library(library)
    w = _rows(weights, "weights")
    u = _aux(uniforms, w.device, torch.float64)
    if u.numel() != w.shape[0]:
        raise ValueError("one uniform per row is required")
    if out is None:
        out = torch.empty(w.shape[0], dtype=torch.int64, device=w.device)
    else:
        out = _out(out, (w.shape[0],), torch.int64, w.device, "out")
    st = _status(status, w.device)
    lib.check(lib.handle.sdc_sample_categorical_rows(w.data_ptr(), _dtype(w), w.shape[0], w.shape[1],
                                                     _stride(w, 0, w.shape[1]), u.data_ptr(), out.data_ptr(),
                                                     st.data_ptr(), _stream(w.device)),
              "categorical sampling")
    return out


def _pair(target, draft):
    t = _rows(target, "target")
    d = _rows(draft, "draft")
    if t.shape != d.shape or t.device != d.device:
        raise ValueError("target and draft rows must have the same shape and device")
    if t.dtype != d.dtype:
        raise TypeError("target and draft rows must have the same dtype")
    return t, d


def residual_rows(target, draft, *, status=None, library=None):
    """float64 [rows, vocab]: max(0, target/sum - draft/sum), or the normalised
    target where that has mass <= 1e-15 (sd_residual_weights_f64)."""
    import torch

    lib = _library(library)
    t, d = _pair(target, draft)
    out = torch.empty(t.shape, dtype=torch.float64, device=t.device)
    st = _status(status, t.device)
    lib.check(lib.handle.sdc_residual_weights_rows(t.data_ptr(), d.data_ptr(), _dtype(t), t.shape[0], t.shape[1],
                                                   _stride(t, 0, t.shape[1]), _stride(d, 0, d.shape[1]),
                                                   out.data_ptr(), t.shape[1],
                                                   st.data_ptr(), _stream(t.device)),
              "residual construction")
    return out


def acceptance_rows(target, draft, tokens, *, status=None, library=None):
    """float64 [rows]: min(1, p(token) / q(token)) per row, 1 where q(token) is 0
    (sd_acceptance_probabilities_f64); NaN for a faulted row."""
    import torch

    lib = _library(library)
    t, d = _pair(target, draft)
    tok = _aux(tokens, t.device, torch.int64)
    if tok.numel() != t.shape[0]:
        raise ValueError("one proposed token per row is required")
    out = torch.empty(t.shape[0], dtype=torch.float64, device=t.device)
    st = _status(status, t.device)
    lib.check(lib.handle.sdc_acceptance_probabilities_rows(t.data_ptr(), d.data_ptr(), _dtype(t), t.shape[0],
                                                           t.shape[1], _stride(t, 0, t.shape[1]),
                                                           _stride(d, 0, d.shape[1]), tok.data_ptr(),
                                                           out.data_ptr(), st.data_ptr(), _stream(t.device)),
              "acceptance verification")
    return out


def first_rejection_rows(probabilities, uniforms, *, status=None, library=None):
    """int64 [sequences]: the first i with !(u[i] < p[i]), else the proposal
    count (sd_first_rejection_f64); -1 for a faulted row."""
    import torch

    lib = _library(library)
    _on_cuda(probabilities, "probabilities")
    p = probabilities.to(dtype=torch.float64).contiguous()
    u = _aux(uniforms, p.device, torch.float64)
    if p.dim() != 2 or p.shape != u.shape:
        raise ValueError("probabilities and uniforms must both be [sequences, proposals]")
    out = torch.empty(p.shape[0], dtype=torch.int64, device=p.device)
    st = _status(status, p.device)
    lib.check(lib.handle.sdc_first_rejection_rows(p.data_ptr(), u.data_ptr(), p.shape[0], p.shape[1], p.shape[1],
                                                  out.data_ptr(), st.data_ptr(), _stream(p.device)),
              "first-rejection verification")
    return out


def verify_batch(target, draft, tokens, uniforms, *, proposal_counts=None, bonus_allowed=None, status=None,
                 out_accepted=None, out_tokens=None, out_probabilities=None, reuse_row_sums=True, library=None):
    """One verification round for every sequence of a batch.

    ``target`` [S, k + 1, V] and ``draft`` [S, k, V] (float32 or float64, unit
    stride along V) are the distributions at the proposal positions, the
    target's with the bonus position; ``tokens`` [S, k] the proposals;
    ``uniforms`` [S, >= k + 1] float64 the sequence's draws in the reference
    decoder's order: draw i decides proposal i, draw j + 1 samples the
    correction after a rejection at j, draw n the bonus after a full
    acceptance of n proposals.  ``proposal_counts`` [S] (int64, 1..k) makes
    the windows ragged; ``bonus_allowed`` [S] (uint8) 0 ends a full
    acceptance without a bonus.

    Returns (accepted [S] int64, token [S] int64, probabilities [S, k]
    float64); token is the correction or bonus, -1 after a full acceptance
    without a bonus; a faulted sequence gets -1 in both.  With
    ``reuse_row_sums`` the deciding launch takes the row sums from the first
    through a small scratch tensor instead of summing the rows again."""
    import torch

    lib = _library(library)
    if target.dim() != 3 or draft.dim() != 3:
        raise ValueError("target must be [S, k + 1, V] and draft [S, k, V]")
    S, k1, V = target.shape
    k = k1 - 1
    if k < 1 or tuple(draft.shape) != (S, k, V):
        raise ValueError("target must be [S, k + 1, V] and draft [S, k, V] with k >= 1")
    if target.dtype != draft.dtype:
        raise TypeError("target and draft rows must have the same dtype")
    _on_cuda(target, "target")
    if draft.device != target.device:
        raise ValueError("target and draft rows must be on the same device")
    dev = target.device
    if target.stride(2) != 1:
        target = target.contiguous()
    if draft.stride(2) != 1:
        draft = draft.contiguous()
    tok = tokens.to(device=dev, dtype=torch.int64)
    if tok.dim() != 2 or tuple(tok.shape) != (S, k):
        raise ValueError("tokens must be [S, k]")
    if tok.stride(1) != 1:
        tok = tok.contiguous()
    u = uniforms
    if u.dtype != torch.float64 or u.device != dev or u.dim() != 2 or u.shape[0] != S or u.shape[1] < k + 1 or \
            u.stride(1) != 1:
        u = uniforms.to(device=dev, dtype=torch.float64).contiguous()
        if u.dim() != 2 or u.shape[0] != S or u.shape[1] < k + 1:
            raise ValueError("uniforms must be [S, >= k + 1]")
    counts = None
    if proposal_counts is not None:
        counts = _aux(proposal_counts, dev, torch.int64)
        if counts.numel() != S:
            raise ValueError("proposal_counts must hold one count per sequence")
    bonus = None
    if bonus_allowed is not None:
        bonus = _aux(bonus_allowed, dev, torch.uint8)
        if bonus.numel() != S:
            raise ValueError("bonus_allowed must hold one flag per sequence")
    accepted = torch.empty(S, dtype=torch.int64, device=dev) if out_accepted is None else \
        _out(out_accepted, (S,), torch.int64, dev, "out_accepted")
    final = torch.empty(S, dtype=torch.int64, device=dev) if out_tokens is None else \
        _out(out_tokens, (S,), torch.int64, dev, "out_tokens")
    probs = torch.empty((S, k), dtype=torch.float64, device=dev) if out_probabilities is None else \
        _out(out_probabilities, (S, k), torch.float64, dev, "out_probabilities")
    st = _status(status, dev)
    sums = torch.empty((S, k, 4), dtype=torch.float64, device=dev) if reuse_row_sums else None
    t_row = target.stride(1)
    d_row = _stride(draft, 1, V)
    batch = _lib.VerifyBatch(
        target.data_ptr(), draft.data_ptr(), _dtype(target), S, k, V, _stride(target, 0, (k + 1) * t_row), t_row,
        _stride(draft, 0, k * d_row), d_row, tok.data_ptr(), _stride(tok, 0, k), u.data_ptr(),
        _stride(u, 0, u.shape[1]),
        counts.data_ptr() if counts is not None else None, bonus.data_ptr() if bonus is not None else None)
    lib.check(lib.handle.sdc_speculative_verify(ctypes.byref(batch), probs.data_ptr(), accepted.data_ptr(),
                                                final.data_ptr(), sums.data_ptr() if sums is not None else None,
                                                st.data_ptr(), _stream(dev)),
              "speculative verification")
    return accepted, final, probs


def raise_for_status(status, operation: str) -> None:
    """Reads a status word and raises NativeBackendError carrying the
    reference's status code and message for the first fault found, in the
    order the reference checks its inputs."""
    bits = int(status.item())
    if bits == 0:
        return
    lib = _lib.load_library()
    for bit, code in _lib.FAULT_STATUS:
        if bits & bit:
            raise _lib.NativeBackendError(f"CUDA {operation} failed: {lib.status_string(code)}", status=code,
                                          faults=bits)
    raise _lib.NativeBackendError(f"CUDA {operation} failed: {_lib.fault_message(bits)}",
                                  status=_lib.STATUS_DEVICE_FAULT, faults=bits)


class DeviceSamplingBackend:
    """The reference's sampling backend protocol on the device kernels.

    Method for method the reference's ``NativeSamplingBackend``
    (src/specdecode/native.py:222-345): the same inputs (Python sequences of
    floats), results and ``NativeBackendError`` on invalid input.  Each call
    copies its rows to the device, launches, and reads the result back, so
    it serves a per-token decoding loop; batched callers use the functions
    of this module on device tensors instead."""

    name = "cuda"

    def __init__(self, device: Any = None, library: _lib.CudaLibrary | None = None) -> None:
        import torch

        self.device = torch.device(device if device is not None else "cuda")
        self._library = _library(library)
        self._status = torch.zeros(1, dtype=torch.int32, device=self.device)

    @property
    def library_path(self) -> str:
        return self._library.path

    def _tensor(self, values, dtype=None):
        import torch

        return torch.tensor(values, dtype=dtype or torch.float64, device=self.device)

    def _finish(self, operation: str) -> None:
        try:
            raise_for_status(self._status, operation)
        finally:
            self._status.zero_()

    def normalize(self, weights: Sequence[float]) -> tuple[float, ...]:
        if len(weights) == 0:
            raise _lib.NativeBackendError("CUDA normalization failed: invalid size", status=_lib.STATUS_INVALID_SIZE)
        out = normalize_rows(self._tensor([list(weights)]), status=self._status, library=self._library)
        self._finish("normalization")
        return tuple(out[0].tolist())

    def categorical(self, probabilities: Sequence[float], uniform: float) -> int:
        if len(probabilities) == 0:
            raise _lib.NativeBackendError("CUDA categorical sampling failed: invalid size",
                                          status=_lib.STATUS_INVALID_SIZE)
        out = sample_rows(self._tensor([list(probabilities)]), self._tensor([float(uniform)]), status=self._status,
                          library=self._library)
        self._finish("categorical sampling")
        return int(out.item())

    def residual_weights(self, target_probabilities: Sequence[float],
                         draft_probabilities: Sequence[float]) -> tuple[float, ...]:
        if len(target_probabilities) != len(draft_probabilities):
            raise _lib.NativeBackendError("native residual inputs must have equal sizes")
        if len(target_probabilities) == 0:
            raise _lib.NativeBackendError("CUDA residual construction failed: invalid size",
                                          status=_lib.STATUS_INVALID_SIZE)
        out = residual_rows(self._tensor([list(target_probabilities)]), self._tensor([list(draft_probabilities)]),
                            status=self._status, library=self._library)
        self._finish("residual construction")
        return tuple(out[0].tolist())

    def acceptance_probabilities(self, target_rows: Sequence[Sequence[float]],
                                 draft_rows: Sequence[Sequence[float]],
                                 token_ids: Sequence[int]) -> tuple[float, ...]:
        import torch

        if not (len(target_rows) == len(draft_rows) == len(token_ids)):
            raise _lib.NativeBackendError("native acceptance inputs must have equal row counts")
        if not target_rows:
            raise _lib.NativeBackendError("native acceptance requires at least one proposal")
        vocabulary_size = len(target_rows[0])
        if vocabulary_size == 0:
            raise _lib.NativeBackendError("native acceptance vocabulary cannot be empty")
        if any(len(row) != vocabulary_size for row in target_rows):
            raise _lib.NativeBackendError("native target rows must have equal vocabulary sizes")
        if any(len(row) != vocabulary_size for row in draft_rows):
            raise _lib.NativeBackendError("native draft rows must have equal vocabulary sizes")
        if any(isinstance(t, bool) or not isinstance(t, int) or t < 0 for t in token_ids):
            raise _lib.NativeBackendError("native proposed token IDs must be non-negative integers")
        out = acceptance_rows(self._tensor([list(r) for r in target_rows]), self._tensor([list(r) for r in draft_rows]),
                              self._tensor(list(token_ids), torch.int64), status=self._status,
                              library=self._library)
        self._finish("acceptance verification")
        return tuple(out.tolist())

    def first_rejection(self, acceptance_probabilities: Sequence[float],
                        uniforms: Sequence[float]) -> VerificationResult:
        if len(acceptance_probabilities) != len(uniforms):
            raise _lib.NativeBackendError("native acceptance probabilities and uniforms must have equal sizes")
        n = len(acceptance_probabilities)
        if n == 0:
            return VerificationResult(0, None)
        out = first_rejection_rows(self._tensor([list(acceptance_probabilities)]), self._tensor([list(uniforms)]),
                                   status=self._status, library=self._library)
        self._finish("first-rejection verification")
        index = int(out.item())
        return VerificationResult(index, None if index == n else index)
