"""Stream, event and buffer plumbing for the device path.

Keeps the surface of the reference's ``CudaExecutionRuntime``
(src/specdecode/cuda.py:34-369): three streams by role (draft, target,
transfer), ``submit*`` returning a ``CudaTask`` whose completion event other
submissions can wait on, NVTX ranges per submission, optional timing events,
power-of-two-grown reusable device workspaces and pinned host buffers,
pinned non-blocking host-to-device copies, memory snapshots and environment
metadata.  The paged-cache kernels launch on whatever stream is current, so
a submission scopes them to its role's stream.

``torch_module`` can be injected for tests on machines without a GPU.
"""

from __future__ import annotations

import os
import platform
import sys
from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass
from math import prod
from numbers import Integral
from typing import Any, Generic, TypeVar


class CudaDependencyError(ImportError):
    """Raised when PyTorch is not importable."""


class CudaUnavailableError(RuntimeError):
    """Raised when CUDA execution is requested without a usable device."""


def _require_torch() -> Any:
    try:
        import torch
    except ImportError as error:  # pragma: no cover - torch is part of the image
        raise CudaDependencyError("the device path requires PyTorch") from error
    return torch


@dataclass(frozen=True, slots=True)
class CudaRuntimeConfig:
    device: str = "cuda:0"
    enable_timing: bool = True
    enable_nvtx: bool = True

    def __post_init__(self) -> None:
        if not isinstance(self.device, str) or not self.device.startswith("cuda"):
            raise ValueError("CUDA runtime device must be a CUDA device string")


@dataclass(frozen=True, slots=True)
class CudaRuntimeStats:
    workspace_allocations: int
    workspace_reuses: int
    pinned_allocations: int
    pinned_reuses: int
    submitted_draft_tasks: int
    submitted_target_tasks: int
    submitted_transfer_tasks: int


@dataclass(frozen=True, slots=True)
class CudaMemorySnapshot:
    allocated_bytes: int
    reserved_bytes: int
    peak_allocated_bytes: int
    peak_reserved_bytes: int


ResultT = TypeVar("ResultT")


@dataclass(slots=True)
class CudaTask(Generic[ResultT]):
    """An asynchronously submitted operation, its result and completion event."""

    result: ResultT
    completion_event: Any
    start_event: Any | None
    _timing_enabled: bool

    def wait(self) -> ResultT:
        self.completion_event.synchronize()
        return self.result

    def elapsed_ms(self) -> float | None:
        if not self._timing_enabled or self.start_event is None:
            return None
        self.completion_event.synchronize()
        return float(self.start_event.elapsed_time(self.completion_event))


def _normalized_shape(shape: Sequence[int]) -> tuple[int, ...]:
    if any(isinstance(d, bool) or not isinstance(d, Integral) for d in shape):
        raise ValueError("buffer dimensions must be integers")
    dims = tuple(int(d) for d in shape)
    if not dims or any(d < 1 for d in dims):
        raise ValueError("buffer shape must contain positive dimensions")
    return dims


class _GrowingBuffers:
    """Named flat buffers grown to the next power of two and handed out as views."""

    def __init__(self, factory: Callable[[int, Any], Any]) -> None:
        self._factory = factory
        self._buffers: dict[tuple[str, str], Any] = {}
        self.allocations = 0
        self.reuses = 0

    def acquire(self, name: str, shape: Sequence[int], dtype: Any) -> Any:
        dims = _normalized_shape(shape)
        need = prod(dims)
        key = (name, str(dtype))
        buffer = self._buffers.get(key)
        if buffer is not None and int(buffer.numel()) >= need:
            self.reuses += 1
        else:
            buffer = self._factory(1 << (need - 1).bit_length(), dtype)
            self._buffers[key] = buffer
            self.allocations += 1
        return buffer[:need].view(dims)


class CudaExecutionRuntime:
    """Reusable streams, events, device workspaces and pinned buffers for one device."""

    _ROLES = ("draft", "target", "transfer")

    def __init__(self, config: CudaRuntimeConfig | None = None, *, torch_module: Any | None = None) -> None:
        self.config = config or CudaRuntimeConfig()
        self._torch = torch_module if torch_module is not None else _require_torch()
        self._cuda = self._torch.cuda
        if not bool(self._cuda.is_available()):
            raise CudaUnavailableError("PyTorch reports that CUDA is unavailable")
        self.device = self._torch.device(self.config.device)
        if getattr(self.device, "type", "cuda") != "cuda":
            raise ValueError("CUDA runtime resolved a non-CUDA device")
        self._streams = {role: self._cuda.Stream(device=self.device) for role in self._ROLES}
        torch = self._torch
        self._workspaces = _GrowingBuffers(lambda n, dtype: torch.empty((n,), dtype=dtype, device=self.device))
        self._pinned = _GrowingBuffers(
            lambda n, dtype: torch.empty((n,), dtype=dtype, device="cpu", pin_memory=True))
        self._submitted = {role: 0 for role in self._ROLES}

    @property
    def streams(self) -> Mapping[str, Any]:
        return dict(self._streams)

    @property
    def torch_module(self) -> Any:
        return self._torch

    def acquire_workspace(self, name: str, shape: Sequence[int], *, dtype: Any) -> Any:
        return self._workspaces.acquire(name, shape, dtype)

    def acquire_pinned_buffer(self, name: str, shape: Sequence[int], *, dtype: Any) -> Any:
        return self._pinned.acquire(name, shape, dtype)

    def _nvtx(self, label: str) -> bool:
        if not self.config.enable_nvtx:
            return False
        push = getattr(getattr(self._cuda, "nvtx", None), "range_push", None)
        if push is None:
            return False
        push(label)
        return True

    def _nvtx_pop(self) -> None:
        pop = getattr(getattr(self._cuda, "nvtx", None), "range_pop", None)
        if pop is not None:
            pop()

    def submit(self, role: str, operation: Callable[[], ResultT], *, wait_for: Sequence[CudaTask[Any]] = (),
               label: str | None = None) -> CudaTask[ResultT]:
        if role not in self._streams:
            raise ValueError(f"unknown CUDA stream role: {role}")
        stream = self._streams[role]
        timing = self.config.enable_timing
        start = self._cuda.Event(enable_timing=True) if timing else None
        done = self._cuda.Event(enable_timing=timing)
        with self._cuda.stream(stream):
            for dependency in wait_for:
                stream.wait_event(dependency.completion_event)
            if start is not None:
                start.record(stream)
            pushed = self._nvtx(label or f"specdecode.{role}")
            try:
                result = operation()
            finally:
                if pushed:
                    self._nvtx_pop()
            done.record(stream)
        self._submitted[role] += 1
        return CudaTask(result=result, completion_event=done, start_event=start, _timing_enabled=timing)

    def submit_draft(self, operation, *, wait_for=(), label: str = "specdecode.draft"):
        return self.submit("draft", operation, wait_for=wait_for, label=label)

    def submit_target(self, operation, *, wait_for=(), label: str = "specdecode.target"):
        return self.submit("target", operation, wait_for=wait_for, label=label)

    def submit_transfer(self, operation, *, wait_for=(), label: str = "specdecode.transfer"):
        return self.submit("transfer", operation, wait_for=wait_for, label=label)

    def copy_to_device(self, name: str, source: Any, *, wait_for: Sequence[CudaTask[Any]] = ()) -> CudaTask[Any]:
        shape = tuple(int(d) for d in source.shape)
        pinned = self.acquire_pinned_buffer(name, shape, dtype=source.dtype)
        pinned.copy_(source, non_blocking=False)
        workspace = self.acquire_workspace(name, shape, dtype=source.dtype)
        return self.submit_transfer(lambda: workspace.copy_(pinned, non_blocking=True), wait_for=wait_for,
                                    label=f"specdecode.transfer.{name}")

    def stage_token_ids(self, name: str, token_ids: Sequence[int]) -> CudaTask[Any]:
        if not token_ids:
            raise ValueError("token_ids cannot be empty")
        source = self._torch.tensor([list(token_ids)], dtype=self._torch.long, device="cpu")
        return self.copy_to_device(name, source)

    def run_speculative_round(self, draft_operation, target_operation):
        draft = self.submit_draft(draft_operation)
        target = self.submit_target(lambda: target_operation(draft.result), wait_for=(draft,))
        return draft, target

    def synchronize(self) -> None:
        self._cuda.synchronize(self.device)

    def reset_peak_memory(self) -> None:
        self._cuda.reset_peak_memory_stats(self.device)

    def memory_snapshot(self) -> CudaMemorySnapshot:
        return CudaMemorySnapshot(
            allocated_bytes=int(self._cuda.memory_allocated(self.device)),
            reserved_bytes=int(self._cuda.memory_reserved(self.device)),
            peak_allocated_bytes=int(self._cuda.max_memory_allocated(self.device)),
            peak_reserved_bytes=int(self._cuda.max_memory_reserved(self.device)))

    def stats(self) -> CudaRuntimeStats:
        return CudaRuntimeStats(
            workspace_allocations=self._workspaces.allocations, workspace_reuses=self._workspaces.reuses,
            pinned_allocations=self._pinned.allocations, pinned_reuses=self._pinned.reuses,
            submitted_draft_tasks=self._submitted["draft"], submitted_target_tasks=self._submitted["target"],
            submitted_transfer_tasks=self._submitted["transfer"])

    def environment(self) -> dict[str, Any]:
        driver = getattr(self._cuda, "driver_version", None)
        return {
            "python": sys.version.split()[0],
            "python_compiler": platform.python_compiler(),
            "platform": platform.platform(),
            "cxx": os.environ.get("CXX"),
            "torch": str(getattr(self._torch, "__version__", "unknown")),
            "torch_cuda": getattr(getattr(self._torch, "version", None), "cuda", None),
            "cuda_driver": driver() if callable(driver) else None,
            "device": str(self.device),
            "device_name": self._cuda.get_device_name(self.device),
            "compute_capability": list(self._cuda.get_device_capability(self.device)),
        }
