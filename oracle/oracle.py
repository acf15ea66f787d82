"""TEST INFRASTRUCTURE ONLY: ctypes/numpy front end of the C restatement in ``vxg_oracle.c``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
use this module, and only as the checker or the timed CPU baseline.  The product package
``vxg_b200`` never imports it.

Every function here forwards to a C function that restates one reference function; the C
file's comments give the reference file:line for each.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libvxg_oracle.so")
_lock = threading.Lock()
_lib = None

BLK = 34  # bytes per KvQ8Block (crates/vxg-tensor/src/llm_prefill.rs:17-24)

_f = ctypes.c_float
_sz = ctypes.c_size_t
_p = ctypes.c_void_p


def build(force: bool = False) -> str:
    """Compile the restatement with its Makefile (gcc); returns the .so path."""
    src = os.path.join(_HERE, "vxg_oracle.c")
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_SO)
            L.vxo_f16_to_f32.restype = _f
            L.vxo_f16_to_f32.argtypes = [ctypes.c_uint16]
            L.vxo_f32_to_f16.restype = ctypes.c_uint16
            L.vxo_f32_to_f16.argtypes = [_f]
            L.vxo_q8_quantize_rows.argtypes = [_p, _sz, _p]
            L.vxo_q8_dot.restype = _f
            L.vxo_q8_dot.argtypes = [_p, _p]
            L.vxo_q8_append.argtypes = [_p, _p, _sz, _sz, _sz, _p, _p]
            L.vxo_q8_attend.argtypes = [_p, _p, _p, _p, _sz, _sz, _sz, _sz, _f, _p, _p]
            L.vxo_f32_attend.argtypes = [_p, _p, _p, _p, _sz, _sz, _sz, _sz, _f, _p, _p]
            L.vxo_step_full_gqa.argtypes = [_p, _p, _p, _p, _p, ctypes.c_int, _sz, _sz, _sz, _sz,
                                            _sz, _f, ctypes.c_int, _f, _p, _p, _p]
            L.vxo_step_full_gqa_q8.argtypes = [
                _p, _p, _p, _p, _p, ctypes.c_int, _sz, _sz, _sz, _sz, _sz, _sz, _f,
                ctypes.c_int, _f, _p, _p, _p]
            L.vxo_deltanet_core.argtypes = [_p, _p, _p, _p, _p, _p, _p, _sz, _sz, _sz, _sz,
                                            _f, _f, _p, _p]
            L.vxo_step_deltanet_recurrent.argtypes = [
                _p, _sz, _p, _p, _p, _p, _p, _p, _p, _p, _p, _sz, _sz, _sz, _sz, _sz, _f, _p]
            L.vxo_batch_decode_q8.argtypes = [
                _sz, _p, _p, _p, _p, _p, _p, _p, _p, _sz, _sz, _sz, _sz, _f, ctypes.c_int, _p,
                ctypes.c_int]
            L.vxo_batch_deltanet.argtypes = [
                _sz, _p, _p, _p, _p, _p, _p, _p, _sz, _sz, _sz, _sz, _f, _f, _p, _p,
                ctypes.c_int]
            L.vxo_rms_norm.argtypes = [_p, _p, _f, _p, _sz]
            L.vxo_apply_rope.argtypes = [_p, _sz, _sz, _sz, _f, ctypes.c_int]
            _lib = L
    return _lib


def _ptr(a):
    if a is None:
        return None
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- fp16 (fp16.rs:6-77)
def f32_to_f16(x: float) -> int:
    return int(lib().vxo_f32_to_f16(_f(x)))


def f16_to_f32(bits: int) -> float:
    return float(lib().vxo_f16_to_f32(ctypes.c_uint16(bits)))


# ---------------------------------------------------------------- Q8 blocks (llm_prefill.rs:26-63)
def q8_quantize(x: np.ndarray) -> np.ndarray:
    """Quantise ``x`` (..., 32k) f32 into KvQ8Block bytes (..., k, 34) uint8."""
    x = _f32(x)
    assert x.shape[-1] % 32 == 0
    rows = x.size // 32
    out = np.empty(rows * BLK, dtype=np.uint8)
    lib().vxo_q8_quantize_rows(_ptr(x), rows, _ptr(out))
    return out.reshape(x.shape[:-1] + (x.shape[-1] // 32, BLK))


def q8_dequantize(blocks: np.ndarray) -> np.ndarray:
    """(..., 34) uint8 -> (..., 32) f32 values code * f16(d) (exact in f32)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    d = b[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    qs = b[..., 2:34].view(np.int8).astype(np.float32)
    return qs * d[..., None]


def q8_append(k_cur, v_cur, n_kv, hd, pos, k_cache, v_cache):
    """llm_prefill.rs:311-324 in place on k_cache / v_cache (uint8 arrays, >= pos+1 tokens)."""
    k_cur, v_cur = _f32(k_cur), _f32(v_cur)
    lib().vxo_q8_append(_ptr(k_cur), _ptr(v_cur), n_kv, hd, pos, _ptr(k_cache), _ptr(v_cache))


def q8_attend(q_heads, k_cache, v_cache, n_head, n_kv, hd, seq_len, scale=None, gates=None):
    """llm_prefill.rs:326-369: attention of prepared queries over tokens [0, seq_len)."""
    q_heads = _f32(q_heads)
    out = np.zeros(n_head * hd, dtype=np.float32)
    if scale is None:
        scale = 1.0 / np.sqrt(np.float32(hd))
    g = _f32(gates) if gates is not None else None
    lib().vxo_q8_attend(_ptr(q_heads), _ptr(g), _ptr(k_cache), _ptr(v_cache), n_head, n_kv, hd,
                        seq_len, _f(scale), _ptr(out), None)
    return out.reshape(n_head, hd)


def step_full_gqa_q8(q_raw, k_cur, v_cur, q_norm, k_norm, gated_q, n_head, n_head_kv, head_dim,
                     pos, rope_pos, rope_dim, rope_freq_base, rope_neox, eps, k_q8, v_q8):
    """Whole llm_prefill.rs:259-370.  k_cur is updated in place (as in the reference);
    k_q8 / v_q8 are uint8 caches of at least (pos+1) tokens.  Returns attn_out [n_head*hd]."""
    out = np.zeros(n_head * head_dim, dtype=np.float32)
    qn = _f32(q_norm) if q_norm is not None else None
    kn = _f32(k_norm) if k_norm is not None else None
    lib().vxo_step_full_gqa_q8(_ptr(_f32(q_raw)), _ptr(k_cur), _ptr(_f32(v_cur)), _ptr(qn),
                               _ptr(kn), int(bool(gated_q)), n_head, n_head_kv, head_dim, pos,
                               rope_pos, rope_dim, _f(rope_freq_base), int(bool(rope_neox)),
                               _f(eps), _ptr(k_q8), _ptr(v_q8), _ptr(out))
    return out


def batch_decode_q8(seq_ids, pos, q, k_new, v_new, k_pool, v_pool, cap, n_head, n_kv, hd,
                    scale=None, gates=None, do_append=True, n_threads=1):
    """Batched decode step over the device-pool layout [n_seq][cap][n_kv][hd/32] blocks."""
    seq_ids = np.ascontiguousarray(seq_ids, dtype=np.int32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    B = seq_ids.shape[0]
    out = np.zeros((B, n_head, hd), dtype=np.float32)
    if scale is None:
        scale = 1.0 / np.sqrt(np.float32(hd))
    q = _f32(q)
    kn = _f32(k_new) if k_new is not None else None
    vn = _f32(v_new) if v_new is not None else None
    g = _f32(gates) if gates is not None else None
    lib().vxo_batch_decode_q8(B, _ptr(seq_ids), _ptr(pos), _ptr(q), _ptr(kn), _ptr(vn), _ptr(g),
                              _ptr(k_pool), _ptr(v_pool), cap, n_head, n_kv, hd, _f(scale),
                              int(bool(do_append)), _ptr(out), int(n_threads))
    return out


def f32_attend(q_heads, k_cache, v_cache, n_head, n_kv, hd, seq_len, scale=None, gates=None):
    """llm_ops.rs:255-299: attention over fp32 caches [t][n_kv][hd] for tokens [0, seq_len)."""
    q_heads = _f32(q_heads)
    out = np.zeros(n_head * hd, dtype=np.float32)
    if scale is None:
        scale = 1.0 / np.sqrt(np.float32(hd))
    g = _f32(gates) if gates is not None else None
    lib().vxo_f32_attend(_ptr(q_heads), _ptr(g), _ptr(_f32(k_cache)), _ptr(_f32(v_cache)), n_head,
                         n_kv, hd, seq_len, _f(scale), _ptr(out), None)
    return out.reshape(n_head, hd)


def step_full_gqa(q_raw, k_cur, v_cur, q_norm, k_norm, gated_q, n_head, n_head_kv, head_dim, pos,
                  rope_dim, rope_freq_base, rope_neox, eps, k_cache, v_cache):
    """Whole llm_ops.rs:196-300.  k_cur is updated in place; k_cache / v_cache are f32 arrays of
    at least (pos+1) rows of [n_kv][hd], row pos written.  Returns att_cat [n_head*hd]."""
    out = np.zeros(n_head * head_dim, dtype=np.float32)
    qn = _f32(q_norm) if q_norm is not None else None
    kn = _f32(k_norm) if k_norm is not None else None
    lib().vxo_step_full_gqa(_ptr(_f32(q_raw)), _ptr(k_cur), _ptr(_f32(v_cur)), _ptr(qn), _ptr(kn),
                            int(bool(gated_q)), n_head, n_head_kv, head_dim, pos, rope_dim,
                            _f(rope_freq_base), int(bool(rope_neox)), _f(eps), _ptr(k_cache),
                            _ptr(v_cache), _ptr(out))
    return out


def prefill_q8(seq_ids, pos, q, k_new, v_new, k_pool, v_pool, cap, n_head, n_kv, hd,
               scale=None, gates=None, n_threads=1):
    """The reference's prefill attention: prompt token ti runs step_full_gqa_q8 at position
    pos + ti, appending its K/V and attending over [0, pos + ti] (llm_prefill.rs:497-517), in
    token order.  q [B][N][n_head][hd], k_new / v_new [B][N][n_kv][hd] f32; returns
    out [B][N][n_head][hd]; the pools are updated in place."""
    q, k_new, v_new = _f32(q), _f32(k_new), _f32(v_new)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    B, N = q.shape[0], q.shape[1]
    out = np.zeros((B, N, n_head, hd), dtype=np.float32)
    for ti in range(N):
        g = None if gates is None else gates[:, ti]
        out[:, ti] = batch_decode_q8(seq_ids, pos + ti, q[:, ti], k_new[:, ti], v_new[:, ti],
                                     k_pool, v_pool, cap, n_head, n_kv, hd, scale=scale, gates=g,
                                     n_threads=n_threads)
    return out


# ---------------------------------------------------------------- gated DeltaNet (llm_ops.rs)
def deltanet_core(q, k, v, beta_raw, alpha_raw, ssm_a, dt_bias, n_kh, n_vh, dk, dv, eps,
                  q_scale, state):
    """llm_ops.rs:139-184 for one sequence; ``state`` [n_vh, dv, dk] f32 updated in place."""
    o = np.zeros(n_vh * dv, dtype=np.float32)
    lib().vxo_deltanet_core(_ptr(_f32(q)), _ptr(_f32(k)), _ptr(_f32(v)), _ptr(_f32(beta_raw)),
                            _ptr(_f32(alpha_raw)), _ptr(_f32(ssm_a)), _ptr(_f32(dt_bias)), n_kh,
                            n_vh, dk, dv, _f(eps), _f(q_scale), _ptr(state), _ptr(o))
    return o.reshape(n_vh, dv)


def batch_deltanet(q, k, v, beta_raw, alpha_raw, ssm_a, dt_bias, n_kh, n_vh, dk, dv, eps,
                   q_scale, state, n_threads=1):
    """Batched core step: q,k [B,n_kh,dk], v [B,n_vh,dv], state [B,n_vh,dv,dk] in place."""
    B = state.shape[0]
    o = np.zeros((B, n_vh, dv), dtype=np.float32)
    lib().vxo_batch_deltanet(B, _ptr(_f32(q)), _ptr(_f32(k)), _ptr(_f32(v)), _ptr(_f32(beta_raw)),
                             _ptr(_f32(alpha_raw)), _ptr(_f32(ssm_a)), _ptr(_f32(dt_bias)), n_kh,
                             n_vh, dk, dv, _f(eps), _f(q_scale), _ptr(state), _ptr(o),
                             int(n_threads))
    return o


def step_deltanet_recurrent(qkv_mixed, z, alpha_raw, beta_raw, ssm_conv1d, ssm_a, ssm_dt_bias,
                            ssm_norm, conv_state, ssm_state, n_kh, n_vh, dk, dv, k_sz, eps):
    """Whole llm_ops.rs:103-193; conv_state / ssm_state updated in place; returns y_concat."""
    qkv = _f32(qkv_mixed)
    y = np.zeros(n_vh * dv, dtype=np.float32)
    lib().vxo_step_deltanet_recurrent(
        _ptr(qkv), qkv.size, _ptr(_f32(z)), _ptr(_f32(alpha_raw)), _ptr(_f32(beta_raw)),
        _ptr(_f32(ssm_conv1d)), _ptr(_f32(ssm_a)), _ptr(_f32(ssm_dt_bias)), _ptr(_f32(ssm_norm)),
        _ptr(conv_state), _ptr(ssm_state), n_kh, n_vh, dk, dv, k_sz, _f(eps), _ptr(y))
    return y
