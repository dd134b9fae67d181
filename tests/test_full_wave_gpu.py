"""Row backward kernels at sizes that fill a whole wave of CTAs.

Each CTA of a row backward kernel writes one partial weight-gradient row into
the caller's workspace, so the size that bloth_*_bwd_workspace_bytes reports
must cover the largest grid any kernel for that row width can launch: the
staged-table kernel, the generic table kernel, the register fallbacks.
Small parity cases launch fewer CTAs than one wave and cannot show an
undersized query; these cases launch a full wave (148 SMs x resident CTAs,
up to 32 rows each) through the library's own workspace query and check the
results against the oracle, evaluated in float64 on the GPU. The table cases
cover cos/sin rows that are staged in one copy per block (contiguous), one
copy per row (strided, 16-byte aligned) and read from global memory
(strided, misaligned). Staged tables on fully rotated rows, and on 16-bit
rows rotated on their first half, take the paired layout (a thread holds a
column and its rotation partner), with 2 to 32 threads per row over these
widths. Tolerances are the path's (see
oracle.tolerance_ok).
"""
import pytest
import torch

import bloth_b200
import oracle
from bloth_b200.kernels.fused_norm_qkv_rope import norm_rope_backward, norm_rope_forward
from oracle.reference_path import seeded_normal, seeded_weight, tolerance_ok

pytestmark = pytest.mark.gpu

FULL_WAVE_ROWS = 148 * 8 * 32 + 77  # more rows than any narrow-row wave holds
DTYPES = [torch.bfloat16, torch.float16, torch.float32]


def _check(got, ref, dtype, what, scale=None):
    ok, worst = tolerance_ok(got.detach(), ref, dtype, scale_with_magnitude=True, scale=scale)
    assert ok, f"{what}: worst excess over tolerance {worst:.3e}"


def _rows(N):
    return FULL_WAVE_ROWS if N <= 512 else 4096 + 77


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("N", [32, 64, 128, 256, 512])
@pytest.mark.parametrize("layout", ["contiguous", "strided", "misaligned"])
def test_table_rope_backward_full_wave(cuda, dtype, N, layout):
    M, h, eps = _rows(N), N // 2, 1e-6
    x = seeded_normal((M, N), dtype, 1).to(cuda)
    w = seeded_weight(N, dtype, 2).to(cuda)
    dy = seeded_normal((M, N), dtype, 3).to(cuda)
    pad = {"contiguous": 0, "strided": 8, "misaligned": 1}[layout]
    ang = seeded_normal((M, h + pad), torch.float32, 4).to(cuda) * 3.0
    cs_dtype = torch.float32 if dtype == torch.float32 else dtype
    cos = ang.cos().to(cs_dtype)[:, :h]
    sin = ang.sin().to(cs_dtype)[:, :h]
    if layout == "contiguous":
        cos, sin = cos.contiguous(), sin.contiguous()
    assert cos.stride(0) == h + pad
    y, rstd = norm_rope_forward(x, w, cos, sin, eps)
    dx, dw = norm_rope_backward(dy, x, w, cos, sin, rstd)
    torch.cuda.synchronize()
    ry, _, rdx, rdw = oracle.norm_rope_table_fwd_bwd(x, w, cos, sin, dy, eps)
    _check(y, ry, dtype, f"{layout} y")
    _check(dx, rdx, dtype, f"{layout} dx")
    _check(dw, rdw, dtype, f"{layout} dw", oracle.norm_rope_table_dw_scale(x, cos, sin, dy, eps))
    assert bloth_b200._lib.load().bloth_device_fault(0) == 0


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("N", [128, 256, 512])
@pytest.mark.parametrize("layout", ["contiguous", "strided"])
def test_half_rotated_table_rope_backward_full_wave(cuda, dtype, N, layout):
    # rotation on the first half of each row (half = N / 4; the paired layout
    # with two more vectors per thread when the tables are staged)
    M, h, eps = _rows(N), N // 4, 1e-6
    x = seeded_normal((M, N), dtype, 5).to(cuda)
    w = seeded_weight(N, dtype, 6).to(cuda)
    dy = seeded_normal((M, N), dtype, 7).to(cuda)
    pad = {"contiguous": 0, "strided": 8}[layout]
    ang = seeded_normal((M, h + pad), torch.float32, 8).to(cuda) * 3.0
    cs_dtype = torch.float32 if dtype == torch.float32 else dtype
    cos = ang.cos().to(cs_dtype)[:, :h]
    sin = ang.sin().to(cs_dtype)[:, :h]
    if layout == "contiguous":
        cos, sin = cos.contiguous(), sin.contiguous()
    y, rstd = norm_rope_forward(x, w, cos, sin, eps)
    dx, dw = norm_rope_backward(dy, x, w, cos, sin, rstd)
    torch.cuda.synchronize()
    ry, _, rdx, rdw = oracle.norm_rope_table_fwd_bwd(x, w, cos, sin, dy, eps)
    _check(y, ry, dtype, f"{layout} y")
    _check(dx, rdx, dtype, f"{layout} dx")
    _check(dw, rdw, dtype, f"{layout} dw", oracle.norm_rope_table_dw_scale(x, cos, sin, dy, eps))
    assert bloth_b200._lib.load().bloth_device_fault(0) == 0


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("N", [64, 128, 256, 512, 4096])
def test_rmsnorm_backward_full_wave(cuda, dtype, N):
    M, eps = _rows(N), 1e-6
    x = seeded_normal((M, N), dtype, 5).to(cuda).requires_grad_(True)
    w = seeded_weight(N, dtype, 6).to(cuda).requires_grad_(True)
    g = seeded_normal((M, N), dtype, 7).to(cuda)
    y = bloth_b200.rms_norm(x, w, eps)
    y.backward(g)
    torch.cuda.synchronize()
    ry, _, rdx, rdw = oracle.rms_norm_fwd_bwd(x.detach(), w.detach(), g, eps)
    _check(y, ry, dtype, "y")
    _check(x.grad, rdx, dtype, "dx")
    _check(w.grad, rdw, dtype, "dw", oracle.rms_norm_dw_scale(x.detach(), g, eps))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("N", [64, 128, 256, 512, 4096])
def test_add_rmsnorm_backward_full_wave(cuda, dtype, N):
    M, eps = _rows(N), 1e-6
    x = seeded_normal((M, N), dtype, 8).to(cuda).requires_grad_(True)
    r = seeded_normal((M, N), dtype, 9).to(cuda).requires_grad_(True)
    w = seeded_weight(N, dtype, 10).to(cuda).requires_grad_(True)
    gy = seeded_normal((M, N), dtype, 11).to(cuda)
    gz = seeded_normal((M, N), dtype, 12).to(cuda)
    y, z = bloth_b200.fused_add_rms_norm(x, r, w, eps)
    torch.autograd.backward([y, z], [gy, gz])
    torch.cuda.synchronize()
    ry, rz, _, rdz, rdw = oracle.add_rms_norm_fwd_bwd(x.detach(), r.detach(), w.detach(), gy,
                                                      gz, eps)
    _check(y, ry, dtype, "y")
    assert torch.equal(z, rz)
    _check(x.grad, rdz, dtype, "dx")
    _check(r.grad, rdz, dtype, "dr")
    _check(w.grad, rdw, dtype, "dw", oracle.rms_norm_dw_scale(z.detach(), gy, eps))
