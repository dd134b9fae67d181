"""The kernels' bounded waits, exercised on a real GPU without a fault.

Every bulk-copy completion wait in the pipelined kernels gives up after a time
limit, records bit 0 of the device fault word and lets the kernel return. Here
a diagnostic kernel waits on a barrier nothing completes (no copy is issued),
so its wait must expire; the host must then read the fault bit, and the
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
    lib.bloth_device_fault(1)  # start clean
    stream = _lib.stream_of(torch.empty(1, device=cuda))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    assert lib.bloth_selftest_wait_expiry(50, stream) == 0
    e1.record()
    torch.cuda.synchronize()
    assert e0.elapsed_time(e1) >= 45.0  # it did wait for its limit
    assert lib.bloth_device_fault(1) == 1  # bit 0: an expired copy wait; cleared
    assert lib.bloth_device_fault(0) == 0
    # the context still runs the kernels correctly
    x = seeded_normal((257, 4096), torch.bfloat16, 1)
    w = seeded_weight(4096, torch.bfloat16, 2)
    y = bloth_b200.rms_norm(x.to(cuda), w.to(cuda), 1e-5)
    ok, worst = tolerance_ok(y.cpu(), oracle.rms_norm(x, w, 1e-5)[0], torch.bfloat16)
    assert ok, worst
    assert lib.bloth_device_fault(0) == 0
