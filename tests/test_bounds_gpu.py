"""Out-of-bounds write detection without a sanitizer.

Each output of a C-ABI call is placed inside a larger buffer whose every
other byte holds a guard pattern: 4 KiB before and after the tensor, and the
gaps between rows when the row stride is wider than the row. After the call,
every guard byte must be unchanged, i.e. the kernels wrote only the elements
of their outputs. Shapes are chosen to hit partial chunks, partial row blocks,
ragged widths (the scalar path), single rows and odd head counts. Inputs are
ordinary tensors; correctness of the values is the parity tests' job.
"""
import pytest
import torch

import bloth_b200
from bloth_b200 import _lib

pytestmark = pytest.mark.gpu

GUARD = 4096
PATTERN = 0xA5


class Guarded:
    """A [rows, cols] view with row stride `ld` (elements) inside a guarded
    byte buffer."""

    def __init__(self, rows, cols, ld, dtype, dev):
        es = torch.tensor([], dtype=dtype).element_size()
        self.span = ((rows - 1) * ld + cols) * es if rows else 0
        # 16-byte aligned start inside the buffer, as the kernels require
        self.buf = torch.full((GUARD + self.span + GUARD + 16,), PATTERN, dtype=torch.uint8,
                              device=dev)
        off = GUARD + (-(self.buf.data_ptr() + GUARD) % 16)
        self.off = off
        flat = self.buf[off:off + self.span].view(dtype) if rows else \
            torch.empty(0, dtype=dtype, device=dev)
        self.t = torch.as_strided(flat, (rows, cols), (ld, 1)) if rows else \
            torch.empty(0, cols, dtype=dtype, device=dev)
        mask = torch.ones(self.buf.numel(), dtype=torch.bool, device=dev)
        if rows:
            starts = off + torch.arange(rows, device=dev) * (ld * es)
            idx = starts[:, None] + torch.arange(cols * es, device=dev)[None, :]
            mask[idx.reshape(-1)] = False
        self.mask = mask

    def intact(self) -> bool:
        if self.buf.is_cuda:
            torch.cuda.synchronize()
        return bool((self.buf[self.mask] == PATTERN).all())


def _rows_in(M, N, dtype, dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randn(M, N, generator=g, device=dev, dtype=torch.float32).to(dtype)


ROW_SHAPES = [(1, 64), (3, 1000), (17, 8), (130, 4096), (5, 4100), (257, 2048), (2, 65536)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("M,N", ROW_SHAPES)
@pytest.mark.parametrize("pad", [0, 24])
def test_rmsnorm_writes_stay_in_bounds(cuda, dtype, M, N, pad):
    if dtype == torch.float32 and N > 32768:
        pytest.skip("fp32 rows are limited to 32768")
    lib = _lib.load()
    code = _lib.dtype_code(dtype)
    x = _rows_in(M, N, dtype, cuda)
    dy = _rows_in(M, N, dtype, cuda, 1)
    w = torch.ones(N, dtype=dtype, device=cuda)
    ld = N + pad
    y = Guarded(M, N, ld, dtype, cuda)
    rstd = Guarded(1, M, M, torch.float32, cuda)
    rc = lib.bloth_rmsnorm_fwd(_lib.ptr(x), N, _lib.ptr(w), 0.0, _lib.ptr(y.t), ld,
                               _lib.ptr(rstd.t), M, N, 1e-6, code, code, _lib.stream_of(x))
    assert rc == 0
    assert y.intact() and rstd.intact()
    dx = Guarded(M, N, ld, dtype, cuda)
    dw = Guarded(1, N, N, dtype, cuda)
    ws_bytes = lib.bloth_rmsnorm_bwd_workspace_bytes(M, N, code)
    ws = Guarded(1, max(ws_bytes, 1), max(ws_bytes, 1), torch.uint8, cuda)
    rc = lib.bloth_rmsnorm_bwd(_lib.ptr(dy), N, _lib.ptr(x), N, _lib.ptr(w), 0.0,
                               _lib.ptr(rstd.t), _lib.ptr(dx.t), ld, _lib.ptr(dw.t), M, N, code,
                               code, _lib.ptr(ws.t), ws_bytes, _lib.stream_of(x))
    assert rc == 0
    assert dx.intact() and dw.intact() and ws.intact()


@pytest.mark.parametrize("M,N", [(1, 64), (97, 4096), (5, 4100), (300, 1024)])
def test_add_rmsnorm_writes_stay_in_bounds(cuda, M, N):
    lib = _lib.load()
    dtype = torch.bfloat16
    code = _lib.dtype_code(dtype)
    x, r = _rows_in(M, N, dtype, cuda), _rows_in(M, N, dtype, cuda, 1)
    dy, dzo = _rows_in(M, N, dtype, cuda, 2), _rows_in(M, N, dtype, cuda, 3)
    w = torch.ones(N, dtype=dtype, device=cuda)
    z, y = Guarded(M, N, N + 8, dtype, cuda), Guarded(M, N, N, dtype, cuda)
    rstd = Guarded(1, M, M, torch.float32, cuda)
    rc = lib.bloth_add_rmsnorm_fwd(_lib.ptr(x), N, _lib.ptr(r), N, _lib.ptr(z.t), N + 8,
                                   _lib.ptr(w), 1.0, _lib.ptr(y.t), N, _lib.ptr(rstd.t), M, N,
                                   1e-6, code, code, _lib.stream_of(x))
    assert rc == 0 and z.intact() and y.intact() and rstd.intact()
    dz, dw = Guarded(M, N, N, dtype, cuda), Guarded(1, N, N, dtype, cuda)
    ws_bytes = lib.bloth_add_rmsnorm_bwd_workspace_bytes(M, N, code)
    ws = Guarded(1, max(ws_bytes, 1), max(ws_bytes, 1), torch.uint8, cuda)
    rc = lib.bloth_add_rmsnorm_bwd(_lib.ptr(dy), N, _lib.ptr(dzo), N, _lib.ptr(z.t), N + 8,
                                   _lib.ptr(w), 1.0, _lib.ptr(rstd.t), _lib.ptr(dz.t), N,
                                   _lib.ptr(dw.t), M, N, code, code, _lib.ptr(ws.t), ws_bytes,
                                   _lib.stream_of(x))
    assert rc == 0 and dz.intact() and dw.intact() and ws.intact()


@pytest.mark.parametrize("B,S,Hq,Hk,D", [(1, 1, 1, 1, 64), (2, 37, 5, 3, 128),
                                         (3, 129, 32, 8, 128), (1, 9, 7, 0, 256),
                                         (2, 1000, 2, 1, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_qk_norm_rope_writes_stay_in_bounds(cuda, B, S, Hq, Hk, D, dtype):
    lib = _lib.load()
    code = _lib.dtype_code(dtype)
    g = torch.Generator(device=cuda).manual_seed(0)

    def heads(H, seed):
        return torch.randn(B, S, H, D, generator=g, device=cuda).to(dtype)

    q, gq = heads(Hq, 1), heads(Hq, 2)
    k, gk = (heads(Hk, 3), heads(Hk, 4)) if Hk else (None, None)
    w = torch.ones(D, dtype=dtype, device=cuda)
    inv = (1.0 / (1e4 ** (torch.arange(0, D // 2, device=cuda, dtype=torch.float32) / (D // 2))))
    pos = torch.arange(S, device=cuda).expand(B, S).contiguous()
    # outputs with a head stride wider than D (gaps are guarded too)
    qo = Guarded(B * S * Hq, D, D + 16, dtype, cuda)
    ko = Guarded(B * S * Hk, D, D + 16, dtype, cuda) if Hk else None
    rq = Guarded(1, B * S * Hq, B * S * Hq, torch.float32, cuda)
    rk = Guarded(1, B * S * Hk, B * S * Hk, torch.float32, cuda) if Hk else None

    def st4(H):
        return _lib.strides((S * H * (D + 16), H * (D + 16), D + 16))

    def st(t):
        return None if t is None else _lib.strides(t.stride()[:3])

    P = _lib.ptr
    pos_st = _lib.strides((S, 1))
    rc = lib.bloth_qk_norm_rope_fwd(
        P(q), st(q), P(k), st(k), P(w), P(w) if Hk else None, 0.0, P(qo.t), st4(Hq),
        P(ko.t) if Hk else None, st4(Hk) if Hk else None, P(rq.t), P(rk.t) if Hk else None,
        P(pos), pos_st, _lib.I64, P(inv), None, None, None, 0, 0, 1.0, B, S, Hq, Hk, D, 1e-6,
        code, code, _lib.stream_of(q))
    assert rc == 0
    assert qo.intact() and rq.intact() and (not Hk or (ko.intact() and rk.intact()))
    dq = Guarded(B * S * Hq, D, D + 16, dtype, cuda)
    dk = Guarded(B * S * Hk, D, D + 16, dtype, cuda) if Hk else None
    dwq, dwk = Guarded(1, D, D, dtype, cuda), Guarded(1, D, D, dtype, cuda)
    ws_bytes = lib.bloth_qk_norm_rope_bwd_workspace_bytes(B, S, D, code)
    ws = Guarded(1, max(ws_bytes, 1), max(ws_bytes, 1), torch.uint8, cuda)
    rc = lib.bloth_qk_norm_rope_bwd(
        P(gq), st(gq), P(gk), st(gk), P(q), st(q), P(k), st(k), P(w), P(w) if Hk else None, 0.0,
        P(rq.t), P(rk.t) if Hk else None, P(dq.t), st4(Hq), P(dk.t) if Hk else None,
        st4(Hk) if Hk else None, P(dwq.t), P(dwk.t) if Hk else None, P(pos), pos_st, _lib.I64,
        P(inv), None, None, None, 0, 0, 1.0, B, S, Hq, Hk, D, code, code, P(ws.t), ws_bytes,
        _lib.stream_of(q))
    assert rc == 0
    assert dq.intact() and dwq.intact() and ws.intact()
    assert not Hk or (dk.intact() and dwk.intact())
    assert lib.bloth_device_fault(0) == 0
