"""CPU checks of the parity oracle (oracle/vxg_oracle.c): the reference's own f16 known-answer
test, then agreement with the independent numpy restatements in tests/refimpl.py."""
import json
import os

import numpy as np
import pytest

from oracle import oracle
from tests import refimpl

HERE = os.path.dirname(os.path.abspath(__file__))


def test_fp16_known_answers_from_reference():
    """crates/vxg-tensor/src/fp16.rs:89-108, both signs, via tests/golden/fp16_kat.json."""
    kat = json.load(open(os.path.join(HERE, "golden", "fp16_kat.json")))
    assert kat["source"].startswith("crates/vxg-tensor/src/fp16.rs")
    assert len(kat["cases"]) == 20
    for case in kat["cases"]:
        x = np.uint32(case["f32_bits"]).view(np.float32)
        assert oracle.f32_to_f16(float(x)) == case["f16_bits"], hex(case["f32_bits"])


def test_f16_to_f32_all_patterns():
    """fp16.rs:6-29 over all 65536 bit patterns equals IEEE widening."""
    bits = np.arange(65536, dtype=np.uint32)
    want = bits.astype(np.uint16).view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(b)) for b in bits[::7]], dtype=np.float32)
    w = want[::7]
    nan = np.isnan(w)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), w[~nan].view(np.uint32))


def test_f32_to_f16_matches_ieee_rne():
    """fp16.rs:33-77 is IEEE round-to-nearest-even for finite values (what the GPU uses)."""
    rng = np.random.default_rng(1)
    xs = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 5, 4000),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e30, -1e30, 6.1e-5, 5.96e-8, 2.98e-8,
                  np.inf, -np.inf], dtype=np.float32)])
    for x in xs:
        with np.errstate(over="ignore"):
            want = int(np.float32(x).astype(np.float16).view(np.uint16))
        assert oracle.f32_to_f16(float(x)) == want, repr(x)


def _edge_rows():
    rows = [np.zeros(32, np.float32), np.full(32, np.float32(1e-9)), np.full(32, np.float32(7e-6)),
            np.linspace(-127, 127, 32).astype(np.float32),      # exact codes
            (np.arange(32, dtype=np.float32) - 16) * np.float32(0.5),  # ties at .5 steps
            np.full(32, np.float32(3e38)), np.full(32, np.float32(-65504 * 127))]
    r = np.random.default_rng(2).standard_normal(32).astype(np.float32)
    r[3] = np.nan
    rows.append(r)
    r = np.random.default_rng(3).standard_normal(32).astype(np.float32)
    r[7] = np.inf
    rows.append(r)
    r = np.random.default_rng(4).standard_normal(32).astype(np.float32)
    r[0] = -np.inf
    r[1] = np.nan
    rows.append(r)
    rows.append(np.full(32, np.nan, np.float32))
    return np.stack(rows)


def test_quantize_matches_independent_restatement():
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal((3000, 32)).astype(np.float32),
                        (rng.standard_normal((500, 32)) * 8).astype(np.float32),
                        (rng.standard_normal((500, 32)) * 1e-4).astype(np.float32),
                        _edge_rows()])
    blk = oracle.q8_quantize(x).reshape(-1, 34)
    d, c = refimpl.quantize(x)
    assert np.array_equal(blk, refimpl.to_blocks(d, c))


def test_q8_footprint():
    """34 bytes per 32 floats: >= 3.5x smaller than f32 (vxt_roadmap_steps.rs:243-248)."""
    x = np.random.default_rng(0).standard_normal((10, 2, 256)).astype(np.float32)
    blk = oracle.q8_quantize(x)
    assert blk.nbytes * 3.5 <= x.nbytes


def test_attend_matches_float64():
    rng = np.random.default_rng(6)
    H, n_kv, hd, T = 16, 2, 256, 300
    k = rng.standard_normal((T, n_kv, hd)).astype(np.float32)
    v = rng.standard_normal((T, n_kv, hd)).astype(np.float32)
    q = rng.standard_normal((H, hd)).astype(np.float32)
    gates = rng.standard_normal((H, hd)).astype(np.float32)
    kb, vb = oracle.q8_quantize(k), oracle.q8_quantize(v)
    for g in (None, gates):
        got = oracle.q8_attend(q, kb, vb, H, n_kv, hd, T, gates=g)
        want = refimpl.attend(q, kb, vb, 1.0 / 16.0, gates=g)
        np.testing.assert_allclose(got, want, atol=2e-5, rtol=1e-4)


def test_append_layout():
    """llm_prefill.rs:311-324: token pos lands at pos*n_kv*nb + kh*nb + b."""
    rng = np.random.default_rng(7)
    n_kv, hd, cap = 2, 64, 5
    kc = np.zeros(cap * n_kv * (hd // 32) * 34, np.uint8)
    vc = np.zeros_like(kc)
    k = rng.standard_normal((n_kv, hd)).astype(np.float32)
    v = rng.standard_normal((n_kv, hd)).astype(np.float32)
    oracle.q8_append(k, v, n_kv, hd, 3, kc, vc)
    kc = kc.reshape(cap, n_kv, hd // 32, 34)
    assert np.array_equal(kc[3], oracle.q8_quantize(k))
    assert not kc[:3].any() and not kc[4].any()


def test_step_full_gqa_q8_prologue():
    """The whole step (gate split, q/k RMSNorm, NeoX RoPE) against numpy."""
    rng = np.random.default_rng(8)
    H, n_kv, hd, pos = 4, 2, 64, 6
    cap = pos + 1
    q_raw = rng.standard_normal(H * 2 * hd).astype(np.float32)
    k_cur = rng.standard_normal(n_kv * hd).astype(np.float32)
    v_cur = rng.standard_normal(n_kv * hd).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kc = np.zeros(cap * n_kv * (hd // 32) * 34, np.uint8)
    vc = np.zeros_like(kc)
    prev_k = rng.standard_normal((pos, n_kv, hd)).astype(np.float32)
    prev_v = rng.standard_normal((pos, n_kv, hd)).astype(np.float32)
    kc[: pos * n_kv * 2 * 34] = oracle.q8_quantize(prev_k).reshape(-1)
    vc[: pos * n_kv * 2 * 34] = oracle.q8_quantize(prev_v).reshape(-1)
    kk = k_cur.copy()
    out = oracle.step_full_gqa_q8(q_raw, kk, v_cur, qn, kn, True, H, n_kv, hd, pos, pos, hd,
                                  10000.0, True, 1e-6, kc, vc)

    def rms(x, w):
        return x / np.sqrt((x.astype(np.float64) ** 2).mean() + 1e-6) * w

    def rope(x):
        half = hd // 2
        i = np.arange(half)
        theta = pos * 10000.0 ** (-(2.0 * i) / hd)
        x0, x1 = x[:half].copy(), x[half:].copy()
        return np.concatenate([x0 * np.cos(theta) - x1 * np.sin(theta),
                               x0 * np.sin(theta) + x1 * np.cos(theta)])

    qh = np.stack([rope(rms(q_raw[h * 2 * hd:h * 2 * hd + hd], qn)) for h in range(H)])
    gates = np.stack([q_raw[h * 2 * hd + hd:(h + 1) * 2 * hd] for h in range(H)])
    kr = np.concatenate([rope(rms(k_cur[j * hd:(j + 1) * hd], kn)) for j in range(n_kv)])
    np.testing.assert_allclose(kk, kr, atol=1e-4, rtol=1e-4)
    want = refimpl.attend(qh, kc.reshape(cap, n_kv, 2, 34), vc.reshape(cap, n_kv, 2, 34),
                          1 / np.sqrt(hd), gates=gates)
    np.testing.assert_allclose(out.reshape(H, hd), want, atol=1e-4, rtol=1e-3)


def test_deltanet_core_matches_float64():
    rng = np.random.default_rng(9)
    n_kh, n_vh, dk, dv = 2, 4, 128, 64
    state = (rng.standard_normal((n_vh, dv, dk)) * 0.02).astype(np.float32)
    for step in range(3):
        q = rng.standard_normal((n_kh, dk)).astype(np.float32)
        k = rng.standard_normal((n_kh, dk)).astype(np.float32)
        v = rng.standard_normal((n_vh, dv)).astype(np.float32)
        br = rng.standard_normal(n_vh).astype(np.float32)
        ar = rng.standard_normal(n_vh).astype(np.float32)
        A = -np.ones(n_vh, np.float32)
        dt = np.zeros(n_vh, np.float32)
        want_o, want_s = refimpl.deltanet_core(q, k, v, br, ar, A, dt, 1e-6, 1 / np.sqrt(dk), state)
        o = oracle.deltanet_core(q, k, v, br, ar, A, dt, n_kh, n_vh, dk, dv, 1e-6,
                                 1 / np.sqrt(dk), state)
        np.testing.assert_allclose(o, want_o, atol=1e-5, rtol=1e-4)
        np.testing.assert_allclose(state, want_s, atol=1e-5, rtol=1e-4)


def test_softplus_branches():
    """llm_ops.rs:158-164: the +-20 cut-offs of softplus."""
    n = 3
    state = np.zeros((n, 32, 64), np.float32)
    q = np.ones((1, 64), np.float32)
    k = np.ones((1, 64), np.float32)
    v = np.ones((n, 32), np.float32)
    ar = np.array([25.0, -25.0, 0.5], np.float32)
    o = oracle.deltanet_core(q, k, v, np.zeros(n, np.float32), ar, -np.full(n, 0.01, np.float32),
                             np.zeros(n, np.float32), 1, n, 64, 32, 1e-6, 0.125, state)
    want, _ = refimpl.deltanet_core(q, k, v, np.zeros(n), ar, -np.full(n, 0.01), np.zeros(n),
                                    1e-6, 0.125, np.zeros((n, 32, 64), np.float32))
    np.testing.assert_allclose(o, want, rtol=1e-5, atol=1e-6)


def test_batch_drivers_thread_invariant():
    """The threaded CPU-baseline drivers give the same bits with 1 and 4 threads."""
    rng = np.random.default_rng(10)
    n_seq, cap, n_kv, hd, H = 6, 40, 2, 64, 8
    k_pool = np.zeros(n_seq * cap * n_kv * 2 * 34, np.uint8)
    ks = rng.standard_normal((n_seq, cap, n_kv, hd)).astype(np.float32)
    vs = rng.standard_normal((n_seq, cap, n_kv, hd)).astype(np.float32)
    k_pool[:] = oracle.q8_quantize(ks).reshape(-1)
    v_pool = oracle.q8_quantize(vs).reshape(-1).copy()
    seq = np.arange(n_seq, dtype=np.int32)
    pos = rng.integers(5, cap, n_seq).astype(np.int32)
    q = rng.standard_normal((n_seq, H, hd)).astype(np.float32)
    o1 = oracle.batch_decode_q8(seq, pos, q, None, None, k_pool, v_pool, cap, H, n_kv, hd,
                                do_append=False, n_threads=1)
    o4 = oracle.batch_decode_q8(seq, pos, q, None, None, k_pool, v_pool, cap, H, n_kv, hd,
                                do_append=False, n_threads=4)
    assert np.array_equal(o1, o4)
