"""The kernels' bounded waits, exercised on a real GPU without a fault.

Every bulk-copy completion wait in the pipelined kernels gives up after a time
limit, records bit 0 of the device fault word, waits (with the same limit) for
the copies it had already issued, and lets the kernel return. Here a
diagnostic kernel runs that path on a two-slot ring: one slot's copy is issued
only after its wait has expired, so the wait must give up; the drain must then
see both copies land (bit 1 clear), the host must read the fault bit, and the
context must still run the library's kernels correctly afterwards.
"""
import pytest
import torch

import bloth_b200
import oracle
from bloth_b200 import _lib
from oracle.reference_path import seeded_normal, seeded_weight, tolerance_ok

pytestmark = pytest.mark.gpu


def test_expired_wait_sets_the_fault_bit_and_the_context_stays_usable(cuda):
    lib = _lib.load()
    bloth_b200.device_fault(reset=True)  # start clean
    stream = _lib.stream_of(torch.empty(1, device=cuda))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    assert lib.bloth_selftest_wait_expiry(50, stream) == 0
    e1.record()
    torch.cuda.synchronize()
    assert e0.elapsed_time(e1) >= 45.0  # it did wait for its limit
    # bit 0: the expired copy wait; bit 1 clear: the drain saw every issued
    # copy land before the kernel returned
    assert bloth_b200.device_fault(reset=True) == 1
    assert bloth_b200.device_fault() == 0
    # the context still runs the kernels correctly
    x = seeded_normal((257, 4096), torch.bfloat16, 1)
    w = seeded_weight(4096, torch.bfloat16, 2)
    y = bloth_b200.rms_norm(x.to(cuda), w.to(cuda), 1e-5)
    ok, worst = tolerance_ok(y.cpu(), oracle.rms_norm(x, w, 1e-5)[0], torch.bfloat16)
    assert ok, worst
    assert bloth_b200.device_fault() == 0


def test_fault_checking_mode_raises_on_the_next_call(cuda, monkeypatch):
    lib = _lib.load()
    bloth_b200.device_fault(reset=True)
    monkeypatch.setattr(_lib, "_CHECK_FAULTS", True)
    x = seeded_normal((64, 512), torch.bfloat16, 3).to(cuda)
    w = seeded_weight(512, torch.bfloat16, 4).to(cuda)
    bloth_b200.rms_norm(x, w, 1e-5)  # no fault: no error
    assert lib.bloth_selftest_wait_expiry(5, _lib.stream_of(x)) == 0
    with pytest.raises(bloth_b200.BlothDeviceFault):
        bloth_b200.rms_norm(x, w, 1e-5)
    assert bloth_b200.device_fault(reset=True) == 1
    bloth_b200.rms_norm(x, w, 1e-5)
