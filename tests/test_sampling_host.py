"""Host-side logic of the device sampling path, on the CPU: the batched
driver's adaptive window (the reference's rule, src/specdecode/decoder.py:47-60)
and the mapping of device fault bits to the reference's status codes and
messages (native/src/native.cpp:52-80)."""

from __future__ import annotations

import pytest

from specdecode_b200 import _lib
from specdecode_b200.sampling import raise_for_status
from specdecode_b200.speculative import DraftWindow


def test_window_follows_the_reference_rule():
    w = DraftWindow(size=4, min_size=1, max_size=8)
    w.observe(4, 4)
    assert w.size == 5  # full acceptance grows by one
    w.observe(2, 5)
    assert w.size == 2  # under half halves
    w.observe(1, 2)
    assert w.size == 1  # otherwise shrinks by one, floored at the minimum
    w.observe(0, 0)
    assert w.size == 1  # no proposals: unchanged
    fixed = DraftWindow(size=4, dynamic=False)
    fixed.observe(4, 4)
    assert fixed.size == 4


@pytest.mark.parametrize("bits,status", [
    (_lib.FAULT_INVALID_UNIFORM | _lib.FAULT_NEGATIVE_WEIGHT, _lib.STATUS_INVALID_UNIFORM),
    (_lib.FAULT_TOKEN_RANGE | _lib.FAULT_ZERO_MASS, _lib.STATUS_TOKEN_OUT_OF_RANGE),
    (_lib.FAULT_NONFINITE_VALUE | _lib.FAULT_ZERO_MASS, _lib.STATUS_NONFINITE_VALUE),
    (_lib.FAULT_NEGATIVE_WEIGHT | _lib.FAULT_ZERO_MASS, _lib.STATUS_NEGATIVE_PROBABILITY),
    (_lib.FAULT_ZERO_MASS, _lib.STATUS_ZERO_MASS),
    (_lib.FAULT_PROPOSAL_COUNT, _lib.STATUS_INVALID_SIZE),
    (_lib.FAULT_SLOT_RANGE, _lib.STATUS_DEVICE_FAULT),
])
def test_fault_bits_map_to_the_reference_status(bits, status):
    """The first fault in the reference's order of checks decides the status
    and its message (the reference's status strings)."""
    import torch

    with pytest.raises(_lib.NativeBackendError) as err:
        raise_for_status(torch.tensor([bits], dtype=torch.int32), "sampling")
    assert err.value.status == status
    assert err.value.faults == bits
    if status != _lib.STATUS_DEVICE_FAULT:
        assert _lib.load_library().status_string(status) in str(err.value)


def test_no_fault_raises_nothing():
    import torch

    raise_for_status(torch.zeros(1, dtype=torch.int32), "sampling")
