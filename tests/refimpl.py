"""Independent numpy restatements used only to cross-check the C oracle on the CPU.

They follow the same reference functions as oracle/vxg_oracle.c but are written separately
(vectorised numpy, float64 where the reference's summation order does not matter), so a
mistake in one restatement shows up as a disagreement.
"""
import numpy as np

F32 = np.float32


def quantize(x):
    """KvQ8Block::quantize (crates/vxg-tensor/src/llm_prefill.rs:27-42), rows of 32 -> (d bits, codes)."""
    x = np.asarray(x, dtype=F32)
    ax = np.abs(x)
    ax = np.where(np.isnan(ax), F32(0), ax)          # f32::max ignores NaN
    amax = np.maximum(F32(0), ax.max(axis=-1))
    with np.errstate(over="ignore"):
        d16 = (amax / F32(127)).astype(np.float16)   # IEEE binary16 RNE
    df = d16.astype(F32)
    with np.errstate(divide="ignore", over="ignore"):
        inv = np.where(df > 0, F32(1) / np.where(df > 0, df, F32(1)), F32(0)).astype(F32)
    with np.errstate(invalid="ignore", over="ignore"):
        r = np.rint(x * inv[..., None])
    r = np.where(np.isnan(r), 0, np.clip(r, -127, 127)).astype(np.int8)
    return d16.view(np.uint16), r


def to_blocks(d_bits, codes):
    """(d u16 [...], codes i8 [..., 32]) -> uint8 [..., 34] KvQ8Block bytes."""
    out = np.empty(d_bits.shape + (34,), np.uint8)
    out[..., 0:2] = d_bits[..., None].view(np.uint8).reshape(d_bits.shape + (2,))
    out[..., 2:] = codes.view(np.uint8)
    return out


def dequant(blocks):
    b = np.ascontiguousarray(blocks)
    d = b[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float64)
    return b[..., 2:].view(np.int8).astype(np.float64) * d[..., None]


def attend(q, k_blocks, v_blocks, scale, gates=None):
    """Softmax attention in float64 over dequantised blocks.
    q [H, hd]; k/v_blocks [T, n_kv, nb, 34]."""
    T, n_kv, nb, _ = k_blocks.shape
    H, hd = q.shape
    K = dequant(k_blocks).reshape(T, n_kv, hd)
    V = dequant(v_blocks).reshape(T, n_kv, hd)
    G = H // n_kv
    out = np.empty((H, hd))
    for h in range(H):
        kh = h // G
        s = (K[:, kh, :] @ q[h].astype(np.float64)) * float(scale)
        p = np.exp(s - s.max())
        out[h] = (p @ V[:, kh, :]) / p.sum()
        if gates is not None:
            out[h] *= 1.0 / (1.0 + np.exp(-gates[h].astype(np.float64)))
    return out


def deltanet_core(q, k, v, beta_raw, alpha_raw, ssm_a, dt_bias, eps, q_scale, state):
    """llm_ops.rs:139-184 in float64; q,k [n_kh, dk], v [n_vh, dv], state [n_vh, dv, dk]."""
    n_kh, dk = q.shape
    n_vh, dv = v.shape
    S = state.astype(np.float64).copy()
    o = np.empty((n_vh, dv))
    for h in range(n_vh):
        hk = h // (n_vh // n_kh)
        qh = q[hk].astype(np.float64)
        kk = k[hk].astype(np.float64)
        qh = qh * q_scale / np.sqrt((qh * qh).sum() + eps)
        kk = kk / np.sqrt((kk * kk).sum() + eps)
        beta = 1.0 / (1.0 + np.exp(-float(beta_raw[h])))
        x = float(alpha_raw[h]) + float(dt_bias[h])
        sp = x if x > 20 else (np.exp(x) if x < -20 else np.log1p(np.exp(x)))
        decay = np.exp(sp * float(ssm_a[h]))
        Sh = S[h] * decay
        sk = Sh @ kk
        d = (v[h].astype(np.float64) - sk) * beta
        Sh = Sh + np.outer(d, kk)
        S[h] = Sh
        o[h] = Sh @ qh
    return o, S
