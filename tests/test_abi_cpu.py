"""CPU checks of the C-ABI library: it loads, exports every symbol the header declares, and
its host-side argument checks work without a GPU (no compute is launched here)."""
import ctypes
import os
import re

import pytest

import vxg_b200
from vxg_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    names = []
    inc = os.path.join(ROOT, "include")
    for fn in sorted(os.listdir(inc)):
        if fn.endswith(".h"):
            src = open(os.path.join(inc, fn)).read()
            names += re.findall(r"VXG_ATTN_API[^;(]*?\b(vxg_attn_cuda_\w+)\s*\(", src)
    return names


def test_library_exports_every_declared_symbol():
    names = header_symbols()
    assert len(names) >= 25
    L = _lib.lib()
    for n in names:
        assert hasattr(L, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_rust_binding_declares_every_declared_symbol():
    """The committed Rust binding (include/vxg_attn_cuda.rs) declares every entry point of the
    header, each once, and nothing the header does not declare."""
    rs = open(os.path.join(ROOT, "include", "vxg_attn_cuda.rs")).read()
    missing = [n for n in header_symbols() if f"fn {n}(" not in rs]
    assert not missing, missing
    declared = re.findall(r"\bfn (vxg_attn_cuda_\w+)\(", rs)
    assert len(declared) == len(set(declared)), "an entry point is declared twice"
    assert set(declared) <= set(header_symbols()), set(declared) - set(header_symbols())


def test_version():
    assert b"sm_100a" in _lib.lib().vxg_attn_cuda_version()


def test_null_handles_are_rejected():
    L = _lib.lib()
    err = _lib.ErrBuf()
    rc = L.vxg_attn_cuda_q8_decode(None, None, 1, 16, None, None, None, None, None, None,
                                   ctypes.c_float(0.0625), 0, None, 0, None, err.buf, err.cap)
    assert rc == _lib.ERR_NULL_PTR and "null context" in err.text
    rc = L.vxg_attn_cuda_deltanet_step(None, 1, 1, 1, 128, 128, *([None] * 7),
                                       ctypes.c_float(1.0), ctypes.c_float(1e-6), None, None, 0,
                                       None, err.buf, err.cap)
    assert rc == _lib.ERR_NULL_PTR
    assert L.vxg_attn_cuda_kv_bytes(None) == 0
    assert L.vxg_attn_cuda_sm_count(None) == 0
    L.vxg_attn_cuda_destroy(None)
    L.vxg_attn_cuda_kv_destroy(None)


def test_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(vxg_b200.VxgError):
        vxg_b200.Context()
