"""GPU parity of the step_full_gqa_q8 drop-in (crates/vxg-tensor/src/llm_prefill.rs:259-370):
the same host buffers in and out as the reference, token after token.  The prologue (gate
split, q/k RMSNorm, RoPE) is bit-exact, so the normed/RoPE'd K written back into k_cur and the
Q8 cache bytes must match the oracle exactly; attn_out within 1e-3 + 1e-3*|ref|."""
import numpy as np
import pytest

import vxg_b200
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,n_kv,hd,gated,norm,neox,rope_dim", [
    (16, 2, 256, True, True, True, 64),     # Qwen3.5 full-attention layer (partial RoPE)
    (4, 2, 64, False, False, False, 64),    # the reference test model's GQA layer shape
    (8, 2, 128, True, False, True, 128),
])
def test_step_sequence(ctx, H, n_kv, hd, gated, norm, neox, rope_dim):
    rng = np.random.default_rng(40)
    steps = 40
    cap = 64
    pool = vxg_b200.KvQ8Pool(ctx, 2, n_kv, hd, cap)
    nb = hd // 32
    kc = np.zeros(cap * n_kv * nb * 34, np.uint8)
    vc = np.zeros_like(kc)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if norm else None
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if norm else None
    for pos in range(steps):
        q_raw = rng.standard_normal(H * (2 if gated else 1) * hd).astype(np.float32)
        k_cur = rng.standard_normal(n_kv * hd).astype(np.float32)
        v_cur = rng.standard_normal(n_kv * hd).astype(np.float32)
        k_ref = k_cur.copy()
        want = oracle.step_full_gqa_q8(q_raw, k_ref, v_cur, qn, kn, gated, H, n_kv, hd, pos,
                                       pos + 3, rope_dim, 1e6, neox, 1e-6, kc, vc)
        out = np.zeros(H * hd, np.float32)
        vxg_b200.step_full_gqa_q8(ctx, pool, 1, q_raw, k_cur, v_cur, qn, kn, gated, H, n_kv, hd,
                                  pos, pos + 3, rope_dim, 1e6, neox, 1e-6, out)
        assert np.array_equal(k_cur.view(np.uint32), k_ref.view(np.uint32)), pos
        np.testing.assert_allclose(out, want, atol=1e-3, rtol=1e-3)
    kb, vb = pool.export_blocks(1, 0, steps)
    assert np.array_equal(kb.reshape(-1), kc[: steps * n_kv * nb * 34])
    assert np.array_equal(vb.reshape(-1), vc[: steps * n_kv * nb * 34])
