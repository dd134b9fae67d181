"""The C-ABI library loads without a GPU and exports every declared entry
point; host-side argument handling raises the reference's errors. CPU only:
no kernel is launched here."""
import ctypes
import os
import re

import pytest
import torch

import bloth_b200
from bloth_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "bloth_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bloth_\w+)\s*\(", text)))


def declared_prototypes():
    """{name: (return type, [argument types])} of every prototype in the header,
    types as written in C with the parameter names removed."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = "\n".join(ln for ln in text.splitlines() if not ln.lstrip().startswith("#"))
    out = {}
    for ret, name, args in re.findall(r"([\w\s\*]+?)\s*\b(bloth_\w+)\s*\(([^)]*)\)\s*;", text):
        types = []
        for arg in args.split(","):
            arg = " ".join(arg.split())
            if arg in ("", "void"):
                continue
            m = re.match(r"(.*?[\s\*])(\w+)$", arg)
            types.append(m.group(1).replace(" ", "").replace("const", "const "))
        out[name] = (" ".join(ret.split()), types)
    return out


_CTYPES_OF = {
    "int": ctypes.c_int, "int64_t": ctypes.c_int64, "float": ctypes.c_float,
    "size_t": ctypes.c_size_t, "const char*": ctypes.c_char_p,
    "const int64_t*": ctypes.POINTER(ctypes.c_int64),
}


def ctypes_of(ctype: str):
    if ctype in _CTYPES_OF:
        return _CTYPES_OF[ctype]
    assert ctype.endswith("*"), ctype
    return ctypes.c_void_p  # data pointers and cudaStream_t


def test_library_built_and_loads():
    assert os.path.exists(_lib.LIB_PATH), "run python -m bloth_b200.build"
    lib = _lib.load()
    assert lib.bloth_version() == (0 << 16) | (2 << 8) | 0


def test_ctypes_signatures_match_the_header():
    protos = declared_prototypes()
    assert sorted(protos) == declared_symbols()
    for name, (ret, args) in protos.items():
        res, argtypes = _lib._SIGNATURES[name]
        assert res is ctypes_of(ret.replace(" *", "*")), name
        assert len(argtypes) == len(args), (name, len(argtypes), len(args))
        for i, (got, want) in enumerate(zip(argtypes, args)):
            assert got is ctypes_of(want), (name, i, want)


def test_every_declared_symbol_is_exported_and_bound():
    syms = declared_symbols()
    assert len(syms) >= 12
    lib = _lib.load()
    for s in syms:
        assert hasattr(lib, s), s
    assert sorted(_lib.exported_symbols()) == syms


def test_strerror_texts():
    lib = _lib.load()
    for code in range(0, 8):
        assert lib.bloth_strerror(code)
    assert lib.bloth_strerror(999) == b"unknown status"


def test_validation_errors_without_gpu():
    # argument checks run before any CUDA call, so they answer on a CPU host
    lib = _lib.load()
    fwd = lib.bloth_rmsnorm_fwd
    assert fwd(None, 0, None, 0.0, None, 0, None, 1, 70000, 1e-6, 1, 1, None) == 2
    assert fwd(None, 0, None, 0.0, None, 0, None, 1, 40000, 1e-6, 0, 0, None) == 2
    assert fwd(None, 0, None, 0.0, None, 0, None, 1, 64, 1e-6, 7, 1, None) == 1
    assert fwd(None, 0, None, 1.0, None, 0, None, 4, 64, 1e-6, 1, 1, None) == 5
    # M == 0 is a no-op
    assert fwd(None, 0, None, 0.0, None, 0, None, 0, 64, 1e-6, 1, 1, None) == 0
    # rotated part wider than the row
    assert lib.bloth_norm_rope_fwd(None, 0, None, 0.0, None, None, 0, 0, 40, None, 0, None, 4,
                                   64, 1e-6, 1, 1, None) == 2
    # head_dim outside {64, 128, 256}
    st = _lib.strides((0, 0, 0))
    assert lib.bloth_rope(None, st, None, st, None, None, None, None, None, None, 0, None, None,
                          None, None, 0, 0, 1.0, 1, 1, 1, 0, 96, 0, 1, None) == 2
    # no heads at all
    assert lib.bloth_rope(None, st, None, st, None, None, None, None, None, None, 0, None, None,
                          None, None, 0, 0, 1.0, 1, 1, 0, 0, 64, 0, 1, None) == 2
    # both a table and inv_freq
    dummy = _lib.ptr(torch.zeros(1))
    assert lib.bloth_rope(None, st, None, st, None, None, None, None, None, None, 0, dummy, dummy,
                          dummy, st, 1, 0, 1.0, 1, 1, 1, 0, 64, 0, 1, None) == 7


def test_cpu_tensors_raise_like_the_reference():
    x = torch.randn(4, 64)
    w = torch.ones(64)
    with pytest.raises(AssertionError, match="CUDA GPU required"):
        bloth_b200.kernels.fused_norm_rope(x, w, torch.ones(4, 32), torch.zeros(4, 32))
    with pytest.raises(AssertionError, match="CUDA GPU required"):
        bloth_b200.rms_norm(x, w)
    with pytest.raises(AssertionError, match="CUDA GPU required"):
        bloth_b200.fused_qk_norm_rope(torch.randn(1, 2, 2, 64), None, w, None)


def test_row_limit_error_like_the_reference():
    from bloth_b200.kernels.rms_norm import _check_row
    with pytest.raises(RuntimeError, match="exceeds max"):
        _check_row(65537, torch.bfloat16)
    with pytest.raises(RuntimeError, match="exceeds max"):
        _check_row(32769, torch.float32)
    _check_row(65536, torch.bfloat16)


def test_reference_name_surface():
    for name in ("rms_norm", "BlothRMSNorm", "fused_norm_qkv", "BlothFusedNormQKV",
                 "rope_embedding", "BlothRoPE", "patch_model", "FastModel"):
        assert hasattr(bloth_b200, name), name
    k = bloth_b200.kernels
    assert k.bloth_rms_norm is k.rms_norm
    for name in ("rms_norm", "bloth_rms_norm", "fused_norm_rope", "rope_embedding"):
        assert hasattr(k, name), name


def test_position_and_table_parsing():
    from bloth_b200.kernels.fused_norm_qkv_rope import _positions, _tables
    p, st = _positions(torch.arange(16), 3, 16)
    assert list(st) == [0, 1] and p.dtype == torch.int64
    p, st = _positions(torch.arange(32, dtype=torch.int32).view(2, 16), 2, 16)
    assert list(st) == [16, 1] and p.dtype == torch.int32
    with pytest.raises(ValueError):
        _positions(torch.arange(15), 1, 16)
    c = torch.randn(100, 64)
    _, _, st, rows, tok = _tables(c, c.clone(), 2, 16, 128)
    assert list(st) == [0, 64] and rows == 100 and not tok
    c = torch.randn(2, 16, 128)
    _, _, st, rows, tok = _tables(c, c.clone(), 2, 16, 128)
    assert list(st) == [16 * 128, 128] and rows == 16 and tok
    c = torch.randn(1, 16, 128)
    _, _, st, rows, tok = _tables(c, c.clone(), 4, 16, 128)
    assert list(st) == [0, 128] and tok
    with pytest.raises(ValueError):
        _tables(torch.randn(16, 48), torch.randn(16, 48), 1, 16, 128)


def test_patch_model_swaps_norms_and_shares_weights():
    transformers = pytest.importorskip("transformers")
    cfg = transformers.Qwen3Config(vocab_size=64, hidden_size=64, intermediate_size=128,
                                   num_hidden_layers=2, num_attention_heads=4,
                                   num_key_value_heads=2, head_dim=16)
    model = transformers.Qwen3ForCausalLM(cfg)
    before = {n: m.weight for n, m in model.named_modules()
              if type(m).__name__ == "Qwen3RMSNorm"}
    keys = set(model.state_dict())
    bloth_b200.patch_model(model, verbose=False)
    after = {n: m for n, m in model.named_modules() if type(m).__name__ == "BlothRMSNorm"}
    # 2 layers x (input, post-attention, q_norm, k_norm) + final norm
    assert len(before) == len(after) == 9
    for n, m in after.items():
        assert m.weight is before[n]
    assert set(model.state_dict()) == keys


def test_workspace_size_cache_is_bounded(monkeypatch):
    calls = []

    class FakeLib:
        def fake_ws(self, *args):
            calls.append(args)
            return 64 * args[0]

    monkeypatch.setattr(_lib, "load", lambda: FakeLib())
    monkeypatch.setattr(_lib, "_WS_CACHE_MAX", 8)
    monkeypatch.setattr(_lib, "_ws_cache", _lib.OrderedDict())
    monkeypatch.setattr(torch.cuda, "device", lambda d: __import__("contextlib").nullcontext())
    dev = torch.device("cpu")
    for m in range(20):
        assert _lib.workspace_bytes("fake_ws", dev, m, 4096, 1) == 64 * m
    assert len(_lib._ws_cache) == 8
    n = len(calls)
    assert _lib.workspace_bytes("fake_ws", dev, 19, 4096, 1) == 64 * 19  # cached
    assert len(calls) == n


def test_wait_expiry_selftest_validates_its_limit_without_gpu():
    lib = _lib.load()
    assert lib.bloth_selftest_wait_expiry(0, None) == 7
    assert lib.bloth_selftest_wait_expiry(5000, None) == 7


def test_launch_counter_and_fault_reader_without_gpu():
    # the launch counter is host-side: no launch has happened in this process
    assert bloth_b200.kernel_launch_count() == 0
    assert isinstance(bloth_b200.kernel_launch_count(), int)
    # the fault reader needs a device; without one it raises instead of
    # returning a stale value
    if not torch.cuda.is_available():
        with pytest.raises(Exception):
            bloth_b200.device_fault()
