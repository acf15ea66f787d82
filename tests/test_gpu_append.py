"""GPU parity: fused Q8 quantise-and-append is bit-exact with the reference quantiser
(KvQ8Block::quantize, crates/vxg-tensor/src/llm_prefill.rs:27-42, layout :311-324)."""
import numpy as np
import pytest

import vxg_b200
from oracle import oracle

pytestmark = pytest.mark.gpu


def edge_tokens(n_kv, hd):
    rng = np.random.default_rng(11)
    rows = []
    specials = [np.zeros(hd, np.float32), np.full(hd, 1e-9, np.float32),
                np.full(hd, 7e-6, np.float32), np.full(hd, 3e38, np.float32),
                (np.arange(hd, dtype=np.float32) % 32 - 16) * np.float32(0.5),
                np.tile(np.linspace(-127, 127, 32, dtype=np.float32), hd // 32)]
    for s in specials:
        rows.append(np.stack([s] * n_kv))
    r = rng.standard_normal((n_kv, hd)).astype(np.float32)
    r[0, 3] = np.nan
    r[1, 40] = np.inf
    r[1, 100] = -np.inf
    rows.append(r)
    return np.stack(rows)


def test_append_bit_exact(ctx):
    rng = np.random.default_rng(12)
    n_seq, n_kv, hd, cap = 5, 2, 256, 64
    pool = vxg_b200.KvQ8Pool(ctx, n_seq, n_kv, hd, cap)
    for trial in range(3):
        B = 4
        seq = rng.choice(n_seq, B, replace=False).astype(np.int32)
        pos = rng.integers(0, cap - 4, B).astype(np.int32)
        T = 3
        k = (rng.standard_normal((B, T, n_kv, hd)) * rng.choice([1e-4, 1.0, 8.0, 300.0])).astype(np.float32)
        v = rng.standard_normal((B, T, n_kv, hd)).astype(np.float32)
        pool.append(seq, pos, k, v, n_tok=T)
        for b in range(B):
            kb, vb = pool.export_blocks(int(seq[b]), int(pos[b]), T)
            assert np.array_equal(kb, oracle.q8_quantize(k[b])), (trial, b)
            assert np.array_equal(vb, oracle.q8_quantize(v[b])), (trial, b)


def test_append_edge_values_bit_exact(ctx):
    n_kv, hd = 2, 256
    toks = edge_tokens(n_kv, hd)
    T = toks.shape[0]
    pool = vxg_b200.KvQ8Pool(ctx, 1, n_kv, hd, T)
    seq = np.zeros(1, np.int32)
    pos = np.zeros(1, np.int32)
    pool.append(seq, pos, toks[None], toks[None][:, ::-1].copy(), n_tok=T)
    kb, vb = pool.export_blocks(0, 0, T)
    assert np.array_equal(kb, oracle.q8_quantize(toks))
    assert np.array_equal(vb, oracle.q8_quantize(toks[::-1].copy()))


@pytest.mark.parametrize("n_kv,hd,T", [(3, 96, 7), (1, 32, 1), (5, 160, 13)])
def test_append_odd_shapes_bit_exact(ctx, n_kv, hd, T):
    """Blocks per token and tokens per entry that are not powers of two (the append divides
    block indices by both), and blocks whose scale rounds down to a binary16 subnormal, where
    |x / scale| exceeds 127.5 and the codes clamp at +-127."""
    rng = np.random.default_rng(13 + n_kv)
    n_seq, cap, B = 6, 40, 5
    pool = vxg_b200.KvQ8Pool(ctx, n_seq, n_kv, hd, cap)
    seq = rng.choice(n_seq, B, replace=False).astype(np.int32)
    pos = rng.integers(0, cap - T, B).astype(np.int32)
    k = rng.standard_normal((B, T, n_kv, hd)).astype(np.float32)
    v = rng.standard_normal((B, T, n_kv, hd)).astype(np.float32)
    # max |x| / 127 = 8.9e-8 rounds to the subnormal 5.96e-8: codes of -amax would be -190
    tiny = np.linspace(-1.1303e-5, 2e-6, 32, dtype=np.float32)
    k[0, 0, 0, :32] = tiny
    v[-1, -1, -1, -32:] = -tiny[::-1]
    pool.append(seq, pos, k, v, n_tok=T)
    for b in range(B):
        kb, vb = pool.export_blocks(int(seq[b]), int(pos[b]), T)
        assert np.array_equal(kb, oracle.q8_quantize(k[b])), b
        assert np.array_equal(vb, oracle.q8_quantize(v[b])), b
    pool.close()


def test_append_rejects_out_of_range(ctx):
    pool = vxg_b200.KvQ8Pool(ctx, 2, 2, 256, 8)
    k = np.zeros((1, 1, 2, 256), np.float32)
    with pytest.raises(vxg_b200.VxgError) as e:
        pool.append(np.array([2], np.int32), np.array([0], np.int32), k, k)
    assert e.value.code == -2
    with pytest.raises(vxg_b200.VxgError) as e:
        pool.append(np.array([0], np.int32), np.array([8], np.int32), k, k)
    assert e.value.code == -3


def test_import_export_roundtrip_and_reserve(ctx):
    rng = np.random.default_rng(13)
    pool = vxg_b200.KvQ8Pool(ctx, 3, 2, 128, 16)
    kb = oracle.q8_quantize(rng.standard_normal((10, 2, 128)).astype(np.float32))
    vb = oracle.q8_quantize(rng.standard_normal((10, 2, 128)).astype(np.float32))
    pool.import_blocks(1, 3, kb, vb)
    k2, v2 = pool.export_blocks(1, 3, 10)
    assert np.array_equal(k2, kb) and np.array_equal(v2, vb)
    assert pool.nbytes == 2 * 3 * 16 * 2 * 4 * 34
    pool.reserve(100)
    assert pool.capacity >= 100
    k3, v3 = pool.export_blocks(1, 3, 10)
    assert np.array_equal(k3, kb) and np.array_equal(v3, vb)
    z, _ = pool.export_blocks(1, 20, 5)
    assert not z.any()


def _amax_for_scale(x):
    """A float32 block maximum m with fl32(m / 127) == x, so the quantiser's scale rounding sees
    exactly x (the reference's f32_to_f16(amax / 127), llm_prefill.rs:30-31)."""
    a = np.float32(x) * np.float32(127)
    for _ in range(8):
        for cand in (a, np.nextafter(a, np.float32(np.inf)), np.nextafter(a, np.float32(0))):
            if np.float32(cand) / np.float32(127) == np.float32(x):
                return np.float32(cand)
        a = np.nextafter(a, np.float32(0))
    return None


def test_append_scale_rounding_on_reference_f16_cases(ctx):
    """The reference's f16 known-answer cases (fp16.rs:89-108) run through the GPU quantiser:
    one block per case whose amax / 127 is that case's f32 value, so the block scale passes
    through every subnormal and half-ULP boundary of the test.  The scale bits written by the
    GPU must equal the reference's expected f16 bits, and the whole block must equal the
    oracle's bytes."""
    import json
    import os
    kat = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "fp16_kat.json")))
    rng = np.random.default_rng(14)
    blocks, expect = [], []
    for c in kat["cases"]:
        x = np.array([c["f32_bits"]], np.uint32).view(np.float32)[0]
        if not np.isfinite(x) or np.signbit(x):
            continue                      # a block scale is |max| / 127: finite, non-negative
        m = _amax_for_scale(x)
        if m is None or not np.isfinite(m):
            continue
        blk = (rng.uniform(-1, 1, 32) * m * np.float32(0.99)).astype(np.float32)
        blk[rng.integers(32)] = m if rng.random() < 0.5 else -m
        blocks.append(blk)
        expect.append(c["f16_bits"])
    assert len(blocks) >= 8
    n_kv, hd = 2, 256
    per_tok = n_kv * hd // 32
    T = -(-len(blocks) // per_tok)
    flat = np.zeros((T * per_tok, 32), np.float32)
    flat[:len(blocks)] = np.stack(blocks)
    toks = flat.reshape(T, n_kv, hd)
    pool = vxg_b200.KvQ8Pool(ctx, 1, n_kv, hd, T)
    pool.append(np.zeros(1, np.int32), np.zeros(1, np.int32), toks[None], toks[None], n_tok=T)
    kb, vb = pool.export_blocks(0, 0, T)
    assert np.array_equal(kb, oracle.q8_quantize(toks))
    assert np.array_equal(vb, kb)
    d = kb.reshape(-1, 34)[:len(blocks), :2].copy().view(np.uint16)[:, 0]
    assert d.tolist() == expect
