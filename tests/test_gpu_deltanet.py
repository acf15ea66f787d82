"""GPU parity of the gated-DeltaNet decode step against the oracle (llm_ops.rs:139-184).
Tolerance: |gpu - ref| <= 1e-3 + 1e-3*|ref| on outputs and states."""
import numpy as np
import pytest

import vxg_b200
from oracle import oracle

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3


def inputs(rng, B, n_kh, n_vh, dk, dv):
    q = rng.standard_normal((B, n_kh, dk)).astype(np.float32)
    k = rng.standard_normal((B, n_kh, dk)).astype(np.float32)
    v = rng.standard_normal((B, n_vh, dv)).astype(np.float32)
    br = rng.standard_normal((B, n_vh)).astype(np.float32)
    ar = rng.standard_normal((B, n_vh)).astype(np.float32)
    return q, k, v, br, ar


@pytest.mark.parametrize("B,n_kh,n_vh,dk,dv,steps", [
    (64, 32, 32, 128, 128, 3),     # BASELINE config 4 shape
    (3, 2, 4, 64, 32, 5),          # grouped k heads (h / (n_vh / n_kh))
    (2, 4, 8, 256, 64, 3),
    (2, 16, 32, 128, 128, 64),     # drift over many steps
])
def test_deltanet_steps(ctx, B, n_kh, n_vh, dk, dv, steps):
    rng = np.random.default_rng(30)
    state = (rng.standard_normal((B, n_vh, dv, dk)) * 0.02).astype(np.float32)
    ref_state = state.copy()
    A = -np.exp(rng.standard_normal(n_vh) * 0.3).astype(np.float32)
    dt = (rng.standard_normal(n_vh) * 0.1).astype(np.float32)
    qs = 1.0 / np.sqrt(dk)
    for _ in range(steps):
        q, k, v, br, ar = inputs(rng, B, n_kh, n_vh, dk, dv)
        o = vxg_b200.deltanet_step(ctx, q, k, v, br, ar, A, dt, state, q_scale=qs, eps=1e-6)
        ro = oracle.batch_deltanet(q, k, v, br, ar, A, dt, n_kh, n_vh, dk, dv, 1e-6, qs,
                                   ref_state, n_threads=8)
        np.testing.assert_allclose(o, ro, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(state, ref_state, atol=ATOL, rtol=RTOL)


def test_deltanet_device_resident_state(ctx):
    """State kept in device memory across steps (torch tensors) matches the host path."""
    import torch
    rng = np.random.default_rng(31)
    B, H, dk, dv = 4, 8, 128, 128
    state = (rng.standard_normal((B, H, dv, dk)) * 0.02).astype(np.float32)
    dstate = torch.from_numpy(state.copy()).cuda()
    A = -np.ones(H, np.float32)
    dt = np.zeros(H, np.float32)
    dA, ddt = torch.from_numpy(A).cuda(), torch.from_numpy(dt).cuda()
    for _ in range(4):
        q, k, v, br, ar = inputs(rng, B, H, H, dk, dv)
        o_h = vxg_b200.deltanet_step(ctx, q, k, v, br, ar, A, dt, state)
        o_d = vxg_b200.deltanet_step(ctx, *[torch.from_numpy(x).cuda() for x in (q, k, v, br, ar)],
                                     dA, ddt, dstate)
        ctx.sync()
        np.testing.assert_array_equal(o_d.cpu().numpy(), o_h)
    np.testing.assert_array_equal(dstate.cpu().numpy(), state)


def test_deltanet_rejects_bad_shapes(ctx):
    rng = np.random.default_rng(32)
    state = np.zeros((1, 4, 32, 96), np.float32)
    q, k, v, br, ar = inputs(rng, 1, 4, 4, 96, 32)
    with pytest.raises(vxg_b200.VxgError) as e:
        vxg_b200.deltanet_step(ctx, q, k, v, br, ar, np.ones(4, np.float32),
                               np.zeros(4, np.float32), state)
    assert e.value.code == -6
