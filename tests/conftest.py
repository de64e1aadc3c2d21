"""Shared test configuration.

Tests marked ``gpu`` need a CUDA device and the in-tree library; everything
else runs on a CPU-only machine.  ``oracle/`` is imported only here in
tests, as the checker.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PACKAGE_ROOT = REPO / "llm-inference-accelerator_b200"
for path in (str(REPO), str(PACKAGE_ROOT)):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libspecdecode_cuda.so")


def cuda_available() -> bool:
    try:
        import torch

        return bool(torch.cuda.is_available())
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


@pytest.fixture(scope="session")
def oracle_c():
    """The C restatement, built by `make -C oracle` if missing."""
    import subprocess

    from oracle.quant import CQuantizer

    library = REPO / "oracle" / "_build" / "liboracle_quant.so"
    if not library.is_file():
        subprocess.run(["make", "-C", str(REPO / "oracle"), "all"], check=True, capture_output=True)
    return CQuantizer(library)


@pytest.fixture(scope="session")
def device():
    if not cuda_available():
        pytest.skip("no CUDA device")
    import torch

    return torch.device("cuda", 0)
