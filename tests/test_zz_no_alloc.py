"""The allocation-free RMSNorm backward (bloth_rmsnorm_bwd_noalloc).

Some callers cannot allocate device memory: an operator interface that hands
a kernel only its inputs and outputs (the host framework owns the memory plan,
so there is nowhere to get a workspace from), or a process whose device memory
another allocator has already reserved. This entry point serves them by
keeping the weight-gradient partial sums in a library-owned static device
array instead of a caller workspace. These tests call it through the C ABI and
check it against the workspace entry point, bloth_rmsnorm_bwd, on the same
inputs, twice in a row (the array keeps the previous call's contents), plus
the rejection of a call that needs more partial-sum space than the array
holds. This file is collected last so that a run stopping at its first failure
has already run every other test.
"""
import pytest
import torch

from bloth_b200 import _lib
from oracle.reference_path import seeded_normal, seeded_weight, tolerance_ok

pytestmark = pytest.mark.gpu

SCRATCH = 16 * 1024 * 1024  # BLOTH_NOALLOC_SCRATCH_BYTES


def _backward(dy, x, w, rstd, noalloc: bool):
    lib = _lib.load()
    M, N = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(N, dtype=w.dtype, device=x.device)
    code, wcode = _lib.dtype_code(x.dtype), _lib.dtype_code(w.dtype)
    stream = _lib.stream_of(x)
    if noalloc:
        rc = lib.bloth_rmsnorm_bwd_noalloc(_lib.ptr(dy), N, _lib.ptr(x), N, _lib.ptr(w), 0.0,
                                           _lib.ptr(rstd), _lib.ptr(dx), N, _lib.ptr(dw), M, N,
                                           code, wcode, stream)
    else:
        ws_bytes = lib.bloth_rmsnorm_bwd_workspace_bytes(M, N, code)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        rc = lib.bloth_rmsnorm_bwd(_lib.ptr(dy), N, _lib.ptr(x), N, _lib.ptr(w), 0.0,
                                   _lib.ptr(rstd), _lib.ptr(dx), N, _lib.ptr(dw), M, N, code, wcode,
                                   _lib.ptr(ws), ws_bytes, stream)
    torch.cuda.synchronize()
    assert rc == 0, lib.bloth_strerror(rc)
    return dx, dw


def _inputs(M, N, dtype, seed, dev):
    x = seeded_normal((M, N), dtype, seed).to(dev)
    w = seeded_weight(N, dtype, seed + 1).to(dev)
    dy = seeded_normal((M, N), dtype, seed + 2).to(dev)
    from bloth_b200.kernels.rms_norm import rmsnorm_forward
    _, rstd = rmsnorm_forward(x, w, 1e-5)
    return dy, x, w, rstd


@pytest.mark.parametrize("dtype,N", [(torch.bfloat16, 4096), (torch.float32, 1024)])
def test_noalloc_matches_workspace_entry_point_twice(cuda, dtype, N):
    for call, (M, seed) in enumerate(((4096, 10), (1500, 20))):
        dy, x, w, rstd = _inputs(M, N, dtype, seed, cuda)
        ref_dx, ref_dw = _backward(dy, x, w, rstd, noalloc=False)
        dx, dw = _backward(dy, x, w, rstd, noalloc=True)
        ok, worst = tolerance_ok(dx.cpu(), ref_dx.cpu(), dtype)
        assert ok, f"call {call}: dx off by {worst}"
        ok, worst = tolerance_ok(dw.cpu(), ref_dw.cpu(), dtype, scale_with_magnitude=True)
        assert ok, f"call {call}: dw off by {worst}"


def test_noalloc_rejects_calls_beyond_the_scratch(cuda):
    lib = _lib.load()
    M, N = 1 << 16, 65536  # bf16 rows of 64K: partial sums far beyond 16 MiB
    need = lib.bloth_rmsnorm_bwd_workspace_bytes(M, N, _lib.BF16)
    assert need > SCRATCH
    # rejected during argument checks, before any kernel is launched
    one = torch.zeros(16, dtype=torch.bfloat16, device=cuda)
    rc = lib.bloth_rmsnorm_bwd_noalloc(_lib.ptr(one), N, _lib.ptr(one), N, _lib.ptr(one), 0.0,
                                       _lib.ptr(one), _lib.ptr(one), N, _lib.ptr(one), M, N,
                                       _lib.BF16, _lib.BF16, _lib.stream_of(one))
    assert rc == 4  # BLOTH_ERR_WORKSPACE
