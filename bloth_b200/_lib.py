"""ctypes binding of ``libbloth_b200.so`` (the C ABI in include/bloth_b200.h).

The library is loaded on first use. There is no fallback: if the shared
library is missing, or a tensor is not on a CUDA device, the call raises.
Launches go to the current torch CUDA stream of the tensors' device; outputs
and workspaces are allocated by the callers through torch's caching
allocator, never inside the library.
"""
from __future__ import annotations

import ctypes
import os
import threading
from collections import OrderedDict
from contextlib import contextmanager

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libbloth_b200.so")

F32, BF16, F16, I32, I64 = 0, 1, 2, 3, 4
ERR_ALIGN = 3

_DTYPE_CODE = {
    torch.float32: F32,
    torch.bfloat16: BF16,
    torch.float16: F16,
    torch.int32: I32,
    torch.int64: I64,
}

_lib = None
_lock = threading.Lock()

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t
_i64p = ctypes.POINTER(ctypes.c_int64)

_SIGNATURES = {
    "bloth_version": (_int, []),
    "bloth_strerror": (ctypes.c_char_p, [_int]),
    "bloth_last_cuda_error": (_int, []),
    "bloth_device_fault": (_int, [_int]),
    "bloth_selftest_wait_expiry": (_int, [_int, _vp]),
    "bloth_kernel_launch_count": (_i64, []),
    "bloth_rmsnorm_fwd": (_int, [_vp, _i64, _vp, _f32, _vp, _i64, _vp, _i64, _i64, _f32, _int,
                                 _int, _vp]),
    "bloth_rmsnorm_bwd_workspace_bytes": (_sz, [_i64, _i64, _int]),
    "bloth_rmsnorm_bwd": (_int, [_vp, _i64, _vp, _i64, _vp, _f32, _vp, _vp, _i64, _vp, _i64, _i64,
                                 _int, _int, _vp, _sz, _vp]),
    "bloth_rmsnorm_bwd_noalloc": (_int, [_vp, _i64, _vp, _i64, _vp, _f32, _vp, _vp, _i64, _vp,
                                         _i64, _i64, _int, _int, _vp]),
    "bloth_add_rmsnorm_fwd": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _f32, _vp, _i64, _vp,
                                     _i64, _i64, _f32, _int, _int, _vp]),
    "bloth_add_rmsnorm_bwd_workspace_bytes": (_sz, [_i64, _i64, _int]),
    "bloth_add_rmsnorm_bwd": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _f32, _vp, _vp, _i64,
                                     _vp, _i64, _i64, _int, _int, _vp, _sz, _vp]),
    "bloth_norm_rope_fwd": (_int, [_vp, _i64, _vp, _f32, _vp, _vp, _i64, _int, _i64, _vp, _i64,
                                   _vp, _i64, _i64, _f32, _int, _int, _vp]),
    "bloth_norm_rope_bwd_workspace_bytes": (_sz, [_i64, _i64, _int]),
    "bloth_norm_rope_bwd": (_int, [_vp, _i64, _vp, _i64, _vp, _f32, _vp, _vp, _i64, _int, _i64,
                                   _vp, _vp, _i64, _vp, _i64, _i64, _int, _int, _vp, _sz, _vp]),
    "bloth_qk_norm_rope_fwd": (_int, [_vp, _i64p, _vp, _i64p, _vp, _vp, _f32, _vp, _i64p, _vp,
                                      _i64p, _vp, _vp, _vp, _i64p, _int, _vp, _vp, _vp, _i64p,
                                      _i64, _int, _f32, _i64, _i64, _i64, _i64, _i64, _f32, _int,
                                      _int, _vp]),
    "bloth_qk_norm_rope_bwd_workspace_bytes": (_sz, [_i64, _i64, _i64, _int]),
    "bloth_qk_norm_rope_bwd": (_int, [_vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _vp,
                                      _f32, _vp, _vp, _vp, _i64p, _vp, _i64p, _vp, _vp, _vp,
                                      _i64p, _int, _vp, _vp, _vp, _i64p, _i64, _int, _f32, _i64,
                                      _i64, _i64, _i64, _i64, _int, _int, _vp, _sz, _vp]),
    "bloth_rope": (_int, [_vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _int, _vp,
                          _vp, _vp, _i64p, _i64, _int, _f32, _i64, _i64, _i64, _i64, _i64, _int,
                          _int, _vp]),
}


def load() -> ctypes.CDLL:
    """Loads the shared library (once) and declares every entry point."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"[Bloth] CUDA extension {LIB_PATH} is not built; run "
                    "`python -m bloth_b200.build` (nvcc, sm_100a)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"[Bloth] unsupported dtype {dt}") from None


class BlothError(RuntimeError):
    """A status code returned by the C ABI."""

    def __init__(self, status: int, what: str):
        lib = load()
        msg = lib.bloth_strerror(status).decode()
        if status == 6:
            msg += f" (cudaError {lib.bloth_last_cuda_error()})"
        super().__init__(f"[Bloth] {what}: {msg}")
        self.status = status


def check(status: int, what: str) -> None:
    if status != 0:
        raise BlothError(status, what)


def require_cuda(*tensors: torch.Tensor) -> None:
    """The reference's convention (fused_norm_qkv_rope.py:133): CUDA tensors only."""
    for t in tensors:
        if t is not None:
            assert t.is_cuda, "[Bloth] CUDA GPU required"


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def strides(vals) -> ctypes.Array:
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def stream_of(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


_WS_CACHE_MAX = 4096
_ws_cache: OrderedDict = OrderedDict()
_ws_lock = threading.Lock()


def workspace_bytes(entry: str, device: torch.device, *args) -> int:
    """Size reported by the C ABI's `entry` (a *_workspace_bytes function) on
    `device`, cached (it depends only on the sizes and the device) in a
    least-recently-used table of bounded size, so that shapes that vary from
    step to step (packed batches) do not grow it without limit."""
    key = (entry, device.index, args)
    with _ws_lock:
        v = _ws_cache.get(key)
        if v is not None:
            _ws_cache.move_to_end(key)
            return v
    with torch.cuda.device(device):
        v = int(getattr(load(), entry)(*args))
    with _ws_lock:
        _ws_cache[key] = v
        while len(_ws_cache) > _WS_CACHE_MAX:
            _ws_cache.popitem(last=False)
    return v


def aligned16(t: torch.Tensor) -> torch.Tensor:
    """t itself when its data is 16-byte aligned, else an aligned copy."""
    return t if t.data_ptr() % 16 == 0 else t.clone()


# ------------------------------------------------------------- launch timer
class LaunchTimer:
    """Records a CUDA event pair around every C-ABI launch, on the launching
    stream, grouped by entry point. Used by bench.py to time individual
    kernels inside its timed region. With ``external=True`` the events are
    created so that a CUDA-graph capture turns their records into event-record
    nodes, which re-record on every replay of the graph."""

    def __init__(self, external: bool = False, only=None):
        self.pairs: dict[str, list] = {}
        self.external = external
        self.only = None if only is None else set(only)

    def _event(self):
        if self.external:
            return torch.cuda.Event(enable_timing=True, external=True)
        return torch.cuda.Event(enable_timing=True)

    def wrap(self, name: str, t: torch.Tensor, fn):
        if self.only is not None and name not in self.only:
            return fn()
        s = torch.cuda.current_stream(t.device)
        a = self._event()
        b = self._event()
        a.record(s)
        rc = fn()
        b.record(s)
        self.pairs.setdefault(name, []).append((a, b))
        return rc

    def summary(self) -> dict[str, dict]:
        out = {}
        for name, evs in self.pairs.items():
            ms = [a.elapsed_time(b) for a, b in evs]
            out[name] = {"launches": len(ms), "total_ms": sum(ms), "mean_ms": sum(ms) / len(ms)}
        return out


# Process-wide, not per thread: autograd runs backward on its own engine
# thread, whose launches the timer must see too. One timing owner at a time.
_timer: LaunchTimer | None = None


@contextmanager
def timing_launches(external: bool = False, only=None):
    """Times every C-ABI launch made inside the block (or only those of the
    entry points named in `only`)."""
    global _timer
    prev, _timer = _timer, LaunchTimer(external, only)
    try:
        yield _timer
    finally:
        _timer = prev


class BlothDeviceFault(RuntimeError):
    """A kernel recorded a fault on the device (see :func:`device_fault`)."""


def device_fault(reset: bool = False, device=None) -> int:
    """Fault bits the library's kernels recorded on `device` (default: the
    current CUDA device) since the last reset; 0 when every call completed.

    Bit 0: a kernel gave up waiting for one of its bulk copies (after 2 s)
    and returned early, after waiting for the copies it had already issued;
    the results of that call are invalid. Bit 1: one of those waits gave up
    too. Reading synchronises with the device; ``reset=True`` clears the bits.
    The kernels never check this word themselves: read it after a step whose
    results must be valid (or set BLOTH_CHECK_FAULTS=1 to have every call
    check it, at the cost of a device synchronisation per call)."""
    lib = load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else \
        torch.device(device)
    with torch.cuda.device(dev):
        v = int(lib.bloth_device_fault(1 if reset else 0))
    if v < 0:
        raise BlothError(-v, "reading the device fault word")
    return v


def kernel_launch_count() -> int:
    """Kernels this library has launched (or recorded into a capturing
    stream) in this process."""
    return int(load().bloth_kernel_launch_count())


# BLOTH_CHECK_FAULTS=1: every call outside stream capture reads the device
# fault word afterwards (a synchronisation per call) and raises on a fault.
_CHECK_FAULTS = os.environ.get("BLOTH_CHECK_FAULTS", "") not in ("", "0")


def _after_call(name: str, rc: int) -> int:
    if rc == 0 and _CHECK_FAULTS and not torch.cuda.is_current_stream_capturing():
        fault = int(load().bloth_device_fault(0))
        if fault != 0:
            raise BlothDeviceFault(
                f"[Bloth] {name}: device fault word {fault:#x} (a bulk-copy wait expired; "
                "this call's results are invalid)")
    return rc


def call(name: str, t: torch.Tensor, *args) -> int:
    """Calls entry point `name` with `t`'s device current (the C ABI launches
    on the calling thread's current device)."""
    fn = getattr(load(), name)
    if t.device.index != torch.cuda.current_device():
        with torch.cuda.device(t.device):
            return call(name, t, *args)
    if _timer is None:
        return _after_call(name, fn(*args))
    return _after_call(name, _timer.wrap(name, t, lambda: fn(*args)))
