"""ctypes binding of ``libvxg_attn_cuda.so`` (the C ABI in include/vxg_attn_cuda.h).

There is no fallback: if the library is missing or no sm_100 device is present, calls raise.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
# VXG_ATTN_LIB selects another build of the same library (A/B comparisons of builds).
LIB_PATH = os.environ.get("VXG_ATTN_LIB") or os.path.join(HERE, "libvxg_attn_cuda.so")

OK = 0
WARN_NONFINITE = 1
ERR_NULL_PTR = -1
ERR_INVALID_OPTION = -2
ERR_BUFFER_TOO_SMALL = -3
ERR_UNSUPPORTED = -6
ERR_INTERNAL = -7
MEM_HOST = 0
MEM_DEVICE = 1

_P = ctypes.c_void_p
_I = ctypes.c_int
_U = ctypes.c_uint32
_F = ctypes.c_float
_S = ctypes.c_size_t
_C = ctypes.c_char_p

# name -> (restype, argtypes); every symbol declared in include/vxg_attn_cuda.h
SIGNATURES = {
    "vxg_attn_cuda_version": (ctypes.c_char_p, []),
    "vxg_attn_cuda_create": (_P, [_C, _S]),
    "vxg_attn_cuda_destroy": (None, [_P]),
    "vxg_attn_cuda_sync": (_I, [_P, _P, _C, _S]),
    "vxg_attn_cuda_sm_count": (_I, [_P]),
    "vxg_attn_cuda_set_timing": (_I, [_P, _I]),
    "vxg_attn_cuda_last_split_ms": (ctypes.c_double, [_P]),
    "vxg_attn_cuda_force_generic": (_I, [_P, _I]),
    "vxg_attn_cuda_malloc": (_P, [_P, _S, _C, _S]),
    "vxg_attn_cuda_free": (None, [_P, _P]),
    "vxg_attn_cuda_host_alloc": (_P, [_P, _S, _C, _S]),
    "vxg_attn_cuda_host_free": (None, [_P, _P]),
    "vxg_attn_cuda_memcpy": (_I, [_P, _P, _P, _S, _I, _C, _S]),
    "vxg_attn_cuda_kv_create": (_P, [_P, _U, _U, _U, _U, _C, _S]),
    "vxg_attn_cuda_kv_destroy": (None, [_P]),
    "vxg_attn_cuda_kv_bytes": (_S, [_P]),
    "vxg_attn_cuda_kv_capacity": (_U, [_P]),
    "vxg_attn_cuda_kv_reserve": (_I, [_P, _U, _C, _S]),
    "vxg_attn_cuda_kv_device_ptrs": (_I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P),
                                          ctypes.POINTER(_S)]),
    "vxg_attn_cuda_kv_import": (_I, [_P, _P, _U, _U, _U, _P, _P, _I, _C, _S]),
    "vxg_attn_cuda_kv_export": (_I, [_P, _P, _U, _U, _U, _P, _P, _I, _C, _S]),
    "vxg_attn_cuda_q8_append": (_I, [_P, _P, _U, _U, _P, _P, _P, _P, _I, _P, _C, _S]),
    "vxg_attn_cuda_q8_decode": (_I, [_P, _P, _U, _U, _P, _P, _P, _P, _P, _P, _F, _U, _P, _I, _P,
                                     _C, _S]),
    "vxg_attn_cuda_q8_decode_host_async": (_I, [_P, _P, _U, _U, _P, _P, _P, _P, _P, _P, _F, _U,
                                                _P, _P, _C, _S]),
    "vxg_attn_cuda_ticket_wait": (_I, [_P, ctypes.c_uint64, _C, _S]),
    "vxg_attn_cuda_peer_buffer_bytes": (_S, [_U, _U, _U]),
    "vxg_attn_cuda_peer_alloc": (_P, [_P, _U, _U, _U, _P, _C, _S]),
    "vxg_attn_cuda_peer_open": (_P, [_P, _P, _C, _S]),
    "vxg_attn_cuda_peer_close": (None, [_P, _P]),
    "vxg_attn_cuda_peer_free": (None, [_P, _P]),
    "vxg_attn_cuda_peer_step": (_I, [_P, _P, _U, _U, _U, _U, _P, _P, _P, _P, _C, _S]),
    "vxg_attn_cuda_q8_decode_noalloc": (_I, [_P, _P, _U, _U, _U, _U, _U, _U, _P, _P, _P, _P, _P,
                                             _P, _F, _P, _P, _C, _S]),
    "vxg_attn_cuda_kv_create_f32": (_P, [_P, _U, _U, _U, _U, _C, _S]),
    "vxg_attn_cuda_f32_append": (_I, [_P, _P, _U, _U, _P, _P, _P, _P, _I, _P, _C, _S]),
    "vxg_attn_cuda_f32_decode": (_I, [_P, _P, _U, _U, _P, _P, _P, _P, _P, _P, _F, _U, _P, _I, _P,
                                      _C, _S]),
    "vxg_attn_cuda_step_full_gqa": (_I, [_P, _P, _U, _P, _P, _P, _P, _P, _I, _U, _U, _U, _U, _U,
                                         _F, _I, _F, _P, _C, _S]),
    "vxg_attn_cuda_q8_prefill": (_I, [_P, _P, _U, _U, _U, _P, _P, _P, _P, _P, _P, _I, _F, _U, _P,
                                      _I, _P, _C, _S]),
    "vxg_attn_cuda_q8_decode_partial": (_I, [_P, _P, _U, _U, _P, _P, _P, _P, _F, _U, _P, _P, _P,
                                             _I, _P, _C, _S]),
    "vxg_attn_cuda_lse_combine": (_I, [_P, _U, _U, _U, _P, _P, _P, _P, _P, _I, _P, _C, _S]),
    "vxg_attn_cuda_state_checkpoint": (_I, [_P, _U, _P, _P, _P, _U, _P, _C, _S]),
    "vxg_attn_cuda_lse_combine_packed": (_I, [_P, _U, _U, _U, _P, _P, _P, _I, _P, _C, _S]),
    "vxg_attn_cuda_step_full_gqa_q8": (_I, [_P, _P, _U, _P, _P, _P, _P, _P, _I, _U, _U, _U, _U,
                                            _U, _U, _F, _I, _F, _P, _C, _S]),
    "vxg_attn_cuda_deltanet_step": (_I, [_P, _U, _U, _U, _U, _U, _P, _P, _P, _P, _P, _P, _P, _F,
                                         _F, _P, _P, _I, _P, _C, _S]),
    "vxg_attn_cuda_deltanet_prefill": (_I, [_P, _U, _U, _U, _U, _U, _U, _P, _P, _P, _P, _P, _P,
                                            _P, _F, _F, _P, _P, _I, _P, _C, _S]),
    "vxg_attn_cuda_step_deltanet_recurrent": (_I, [_P, _U, _P, _U, _P, _P, _P, _P, _P, _P, _P, _P,
                                                   _P, _U, _U, _U, _U, _U, _F, _P, _I, _P, _C,
                                                   _S]),
}

_lock = threading.Lock()
_lib = None


class VxgError(RuntimeError):
    """A negative status from the C ABI (code = include/vxg.h class)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m vxg_b200.build` "
                    "(the CUDA backend has no CPU fallback)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


class ErrBuf:
    """Message buffer passed as (err, cap)."""

    def __init__(self, n: int = 512):
        self.buf = ctypes.create_string_buffer(n)
        self.cap = n

    @property
    def text(self) -> str:
        return self.buf.value.decode(errors="replace")


def check(rc: int, err: ErrBuf) -> int:
    if rc < 0:
        raise VxgError(rc, err.text)
    return rc
