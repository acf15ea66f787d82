"""GPU parity of the fp32-KV path (KvCacheMode::Fp32, the reference's default cache mode):
the step_full_gqa operator (crates/vxg-tensor/src/llm_ops.rs:196-300) and its batched decode.
Tolerance: |gpu - ref| <= 1e-3 + 1e-3*|ref|; the keys written by the drop-in's norm + RoPE
prologue are compared bit for bit."""
import numpy as np
import pytest

import vxg_b200
from oracle import oracle

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3


def _pool(ctx, rng, lens, n_kv, hd, cap):
    pool = vxg_b200.KvF32Pool(ctx, len(lens), n_kv, hd, cap)
    kh = np.zeros((len(lens), cap, n_kv, hd), np.float32)
    vh = np.zeros_like(kh)
    for s, L in enumerate(lens):
        kh[s, :L] = rng.standard_normal((L, n_kv, hd))
        vh[s, :L] = rng.standard_normal((L, n_kv, hd))
        if L:
            pool.import_rows(s, 0, kh[s, :L], vh[s, :L])
    return pool, kh, vh


@pytest.mark.parametrize("n_head,n_kv,hd,device", [(16, 2, 256, False), (16, 2, 256, True),
                                                   (8, 8, 128, False), (32, 4, 64, False)])
def test_f32_decode_ragged(ctx, n_head, n_kv, hd, device):
    rng = np.random.default_rng(60 + hd)
    lens = [37, 0, 700, 3000]
    cap = 3010
    pool, kh, vh = _pool(ctx, rng, lens, n_kv, hd, cap)
    seq = np.array([2, 0, 3, 1], np.int32)
    pos = np.array([lens[s] for s in seq], np.int32)
    q = rng.standard_normal((4, n_head, hd)).astype(np.float32)
    kn = rng.standard_normal((4, n_kv, hd)).astype(np.float32)
    vn = rng.standard_normal((4, n_kv, hd)).astype(np.float32)
    gate = rng.standard_normal((4, n_head, hd)).astype(np.float32)
    if device:
        import torch
        d = lambda x: torch.from_numpy(x).cuda()
        out = pool.decode(d(seq), d(pos), d(q), d(kn), d(vn), q_gate=d(gate))
        assert ctx.sync() == 0
        out = out.cpu().numpy()
    else:
        out = pool.decode(seq, pos, q, kn, vn, q_gate=gate)
    for b, s in enumerate(seq):
        kh[s, pos[b]] = kn[b]
        vh[s, pos[b]] = vn[b]
        want = oracle.f32_attend(q[b], kh[s], vh[s], n_head, n_kv, hd, pos[b] + 1, gates=gate[b])
        np.testing.assert_allclose(out[b], want, atol=ATOL, rtol=RTOL)
        assert np.abs(out[b] - want).max() < 2e-5
    k_back, v_back = pool.export_rows(3, 0, pos[2] + 1)
    assert np.array_equal(k_back, kh[3, :pos[2] + 1]) and np.array_equal(v_back, vh[3, :pos[2] + 1])
    pool.close()


@pytest.mark.parametrize("gated,norms", [(True, True), (False, False)])
def test_step_full_gqa_dropin(ctx, gated, norms):
    """Drop-in for step_full_gqa: same arguments, k_cur rewritten in place (bit-exact), output
    within the bar, over several consecutive positions."""
    rng = np.random.default_rng(61)
    n_head, n_kv, hd, rope_dim = 16, 2, 256, 64
    cap = 64
    pool = vxg_b200.KvF32Pool(ctx, 2, n_kv, hd, cap)
    kc = np.zeros((cap, n_kv, hd), np.float32)
    vc = np.zeros_like(kc)
    qn = (rng.standard_normal(hd) * 0.1 + 1).astype(np.float32) if norms else None
    knorm = (rng.standard_normal(hd) * 0.1 + 1).astype(np.float32) if norms else None
    for pos in range(12):
        q_raw = rng.standard_normal(n_head * hd * (2 if gated else 1)).astype(np.float32)
        k_cur = rng.standard_normal(n_kv * hd).astype(np.float32)
        v_cur = rng.standard_normal(n_kv * hd).astype(np.float32)
        k_ref = k_cur.copy()
        out = np.zeros(n_head * hd, np.float32)
        vxg_b200.step_full_gqa(ctx, pool, 1, q_raw, k_cur, v_cur, qn, knorm, gated, n_head, n_kv,
                               hd, pos, rope_dim, 1e7, True, 1e-6, out)
        want = oracle.step_full_gqa(q_raw, k_ref, v_cur, qn, knorm, gated, n_head, n_kv, hd, pos,
                                    rope_dim, 1e7, True, 1e-6, kc, vc)
        assert np.array_equal(k_cur, k_ref), f"k_cur differs at pos {pos}"
        np.testing.assert_allclose(out, want, atol=ATOL, rtol=RTOL)
    pool.close()


def test_pool_kinds_are_checked(ctx):
    q8 = vxg_b200.KvQ8Pool(ctx, 1, 2, 256, 16)
    f32 = vxg_b200.KvF32Pool(ctx, 1, 2, 256, 16)
    assert f32.nbytes == 2 * 16 * 2 * 256 * 4
    q = np.zeros((1, 16, 256), np.float32)
    with pytest.raises(vxg_b200.VxgError) as e:
        q8.__class__.decode(f32, np.zeros(1, np.int32), np.zeros(1, np.int32), q)
    assert e.value.code == -2
    with pytest.raises(vxg_b200.VxgError) as e:
        f32.__class__.decode(q8, np.zeros(1, np.int32), np.zeros(1, np.int32), q)
    assert e.value.code == -2
    q8.close()
    f32.close()
