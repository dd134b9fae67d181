"""The allocation-free RMSNorm backward (bloth_rmsnorm_bwd_noalloc).

Some callers cannot allocate device memory: an operator interface that hands
a kernel only its inputs and outputs (the host framework owns the memory plan,
so there is nowhere to get a workspace from), or a process whose device memory
another allocator has already reserved. This entry point serves them by
keeping the weight-gradient partial sums in a library-owned static device
array instead of a caller workspace. It runs the same kernels with the same
partial-sum layout and the same fixed-order reduce as the workspace entry
point, bloth_rmsnorm_bwd, so its results must be bit-identical to it. These
tests call both through the C ABI on the same inputs, twice in a row (the
array keeps the previous call's contents, so a partial row read from a stale
call would show), on the vector path, on the scalar path of unaligned rows,
and at a size whose partial sums fill most of the array; plus the rejection of
a call that needs more than the array holds. This file is collected last so
that a run stopping at its first failure has already run every other test.
"""
import pytest
import torch

from bloth_b200 import _lib
from bloth_b200.kernels.rms_norm import rmsnorm_forward

pytestmark = pytest.mark.gpu

SCRATCH = 16 * 1024 * 1024  # BLOTH_NOALLOC_SCRATCH_BYTES


def _backward(dy, x, w, rstd, noalloc: bool):
    """dx, dw of rows x [M, N] (row stride x.stride(0), the same for dy and dx)."""
    lib = _lib.load()
    M, N = x.shape
    ld = x.stride(0)
    dx = torch.full_like(x, float("nan"))
    dw = torch.full((N,), float("nan"), dtype=w.dtype, device=x.device)
    code, wcode = _lib.dtype_code(x.dtype), _lib.dtype_code(w.dtype)
    stream = _lib.stream_of(x)
    if noalloc:
        rc = lib.bloth_rmsnorm_bwd_noalloc(_lib.ptr(dy), dy.stride(0), _lib.ptr(x), ld,
                                           _lib.ptr(w), 0.0, _lib.ptr(rstd), _lib.ptr(dx),
                                           dx.stride(0), _lib.ptr(dw), M, N, code, wcode, stream)
    else:
        ws_bytes = lib.bloth_rmsnorm_bwd_workspace_bytes(M, N, code)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        rc = lib.bloth_rmsnorm_bwd(_lib.ptr(dy), dy.stride(0), _lib.ptr(x), ld, _lib.ptr(w), 0.0,
                                   _lib.ptr(rstd), _lib.ptr(dx), dx.stride(0), _lib.ptr(dw), M, N,
                                   code, wcode, _lib.ptr(ws), ws_bytes, stream)
    torch.cuda.synchronize()
    assert rc == 0, lib.bloth_strerror(rc)
    return dx, dw


def _rows(M, N, ld, dtype, gen, dev):
    """[M, N] rows with row stride ld (a view into an [M, ld] buffer)."""
    buf = torch.randn(M, ld, generator=gen, device=dev, dtype=torch.float32).to(dtype)
    return buf[:, :N]


def _inputs(M, N, dtype, seed, dev, ld=None):
    ld = ld or N
    gen = torch.Generator(device=dev).manual_seed(seed)
    x = _rows(M, N, ld, dtype, gen, dev)
    dy = _rows(M, N, ld, dtype, gen, dev)
    w = (1 + 0.1 * torch.randn(N, generator=gen, device=dev)).to(dtype)
    _, rstd = rmsnorm_forward(x, w, 1e-5)
    return dy, x, w, rstd


def _equal_twice(cases, dev):
    for call, (M, N, dtype, seed, ld) in enumerate(cases):
        dy, x, w, rstd = _inputs(M, N, dtype, seed, dev, ld)
        ref_dx, ref_dw = _backward(dy, x, w, rstd, noalloc=False)
        dx, dw = _backward(dy, x, w, rstd, noalloc=True)
        assert torch.equal(dx, ref_dx), f"call {call}: dx differs from bloth_rmsnorm_bwd"
        assert torch.equal(dw, ref_dw), f"call {call}: dw differs from bloth_rmsnorm_bwd"


@pytest.mark.parametrize("dtype,N", [(torch.bfloat16, 4096), (torch.float32, 1024)])
def test_noalloc_matches_workspace_entry_point_twice(cuda, dtype, N):
    # the second call has fewer rows: a partial row left over from the first
    # call in the shared array must not leak into its result
    _equal_twice([(4096, N, dtype, 10, None), (1500, N, dtype, 20, None)], cuda)


def test_noalloc_scalar_path_of_unaligned_rows_twice(cuda):
    # a row stride that is not a multiple of 16 bytes takes the scalar kernels
    _equal_twice([(700, 1000, torch.bfloat16, 30, 1003), (333, 1000, torch.bfloat16, 40, 1003)],
                 cuda)


def test_noalloc_near_the_scratch_limit(cuda):
    lib = _lib.load()
    best = None
    for dtype in (torch.bfloat16, torch.float32):
        for N in (1024, 2048, 3072, 4096, 6144, 8192, 12288, 16384):
            need = lib.bloth_rmsnorm_bwd_workspace_bytes(1 << 14, N, _lib.dtype_code(dtype))
            if need <= SCRATCH and (best is None or need > best[0]):
                best = (need, N, dtype)
    need, N, dtype = best
    # the largest launch-time partial-sum need that fits fills most of the array
    assert need >= SCRATCH // 2, best
    _equal_twice([(1 << 14, N, dtype, 50, None), (1 << 14, N, dtype, 60, None)], cuda)


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
