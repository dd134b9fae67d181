"""Weight-gradient workspaces at every base alignment the C ABI accepts.

The backward kernels store one partial row of accumulators per CTA into the
caller's workspace: as 16-byte vectors when its base is 16-byte aligned,
value by value otherwise. Both paths must give bit-identical dx and dweight
(the partial rows and the fixed-order reduce are the same), and a base that
is not aligned to the accumulator (4 bytes for 16-bit tensors, 8 for fp32)
must be rejected with BLOTH_ERR_ALIGN before anything is launched.
"""
import ctypes

import pytest
import torch

import bloth_b200
from bloth_b200 import _lib
from bloth_b200.kernels.rms_norm import rmsnorm_forward

pytestmark = pytest.mark.gpu

ERR_ALIGN = 3


def _rms_bwd(dy, x, w, rstd, offset):
    """bloth_rmsnorm_bwd with the workspace base `offset` bytes past a
    256-byte aligned allocation; returns (rc, dx, dw)."""
    lib = _lib.load()
    M, N = x.shape
    code = _lib.dtype_code(x.dtype)
    need = lib.bloth_rmsnorm_bwd_workspace_bytes(M, N, code)
    buf = torch.empty(need + 64, dtype=torch.uint8, device=x.device)
    dx = torch.full_like(x, float("nan"))
    dw = torch.full((N,), float("nan"), dtype=w.dtype, device=x.device)
    rc = lib.bloth_rmsnorm_bwd(_lib.ptr(dy), dy.stride(0), _lib.ptr(x), x.stride(0), _lib.ptr(w),
                               0.0, _lib.ptr(rstd), _lib.ptr(dx), dx.stride(0), _lib.ptr(dw), M, N,
                               code, code, ctypes.c_void_p(buf.data_ptr() + offset), need,
                               _lib.stream_of(x))
    torch.cuda.synchronize()
    return rc, dx, dw


# rows of 4096 (pipelined kernel), 65536 bf16 (register kernel), 1000 with a
# row stride of 1003 (scalar kernel)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("M,N,ld", [(1500, 4096, 4096), (6, 65536, 65536), (333, 1000, 1003)])
def test_rmsnorm_bwd_bit_identical_at_every_accepted_alignment(cuda, dtype, M, N, ld):
    if dtype == torch.float32 and N > 32768:
        pytest.skip("fp32 rows are limited to 32768")
    g = torch.Generator(device=cuda).manual_seed(M + N)
    x = torch.randn(M, ld, generator=g, device=cuda).to(dtype)[:, :N]
    dy = torch.randn(M, ld, generator=g, device=cuda).to(dtype)[:, :N]
    w = (1 + 0.1 * torch.randn(N, generator=g, device=cuda)).to(dtype)
    _, rstd = rmsnorm_forward(x, w, 1e-5)
    rc, ref_dx, ref_dw = _rms_bwd(dy, x, w, rstd, 0)
    assert rc == 0
    acc = 8 if dtype == torch.float32 else 4
    for offset in (4, 8, 16, 24):
        rc, dx, dw = _rms_bwd(dy, x, w, rstd, offset)
        if offset % acc:
            assert rc == ERR_ALIGN, offset
            continue
        assert rc == 0, offset
        assert torch.equal(dx, ref_dx), f"dx differs at workspace offset {offset}"
        assert torch.equal(dw, ref_dw), f"dw differs at workspace offset {offset}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_qk_bwd_bit_identical_at_every_accepted_alignment(cuda, monkeypatch, dtype):
    B, S, Hq, Hk, D = 2, 300, 8, 4, 128
    g = torch.Generator(device=cuda).manual_seed(7)
    q = torch.randn(B, S, Hq, D, generator=g, device=cuda).to(dtype)
    k = torch.randn(B, S, Hk, D, generator=g, device=cuda).to(dtype)
    wq = (1 + 0.1 * torch.randn(D, generator=g, device=cuda)).to(dtype)
    wk = (1 + 0.1 * torch.randn(D, generator=g, device=cuda)).to(dtype)
    gq, gk = torch.randn_like(q), torch.randn_like(k)
    pos = torch.arange(S, device=cuda).expand(B, S)
    inv = 1.0 / (1e4 ** (torch.arange(0, D // 2, dtype=torch.float32, device=cuda) / (D // 2)))

    def grads():
        leaves = [t.clone().requires_grad_(True) for t in (q, k, wq, wk)]
        out = bloth_b200.fused_qk_norm_rope(*leaves, pos, inv, 1e-6)
        torch.autograd.backward(out, (gq, gk))
        torch.cuda.synchronize()
        return [t.grad for t in leaves]

    ref = grads()
    # the op allocates its workspace; give it 64 bytes more and move the base
    # the kernels receive by `offset`
    ws_bytes, call = _lib.workspace_bytes, _lib.call
    acc = 8 if dtype == torch.float32 else 4
    for offset in (4, 8, 16, 24):
        def shifted_call(name, *args, _off=offset):
            if name == "bloth_qk_norm_rope_bwd":
                args = list(args)
                args[-3] = ctypes.c_void_p(args[-3].value + _off)  # workspace pointer
            return call(name, *args)

        monkeypatch.setattr(_lib, "workspace_bytes", lambda e, d, *a: ws_bytes(e, d, *a) + 64)
        monkeypatch.setattr(_lib, "call", shifted_call)
        if offset % acc:
            with pytest.raises(RuntimeError):
                grads()
            continue
        got = grads()
        for name, a, b in zip(("dq", "dk", "dwq", "dwk"), got, ref):
            assert torch.equal(a, b), f"{name} differs at workspace offset {offset}"
