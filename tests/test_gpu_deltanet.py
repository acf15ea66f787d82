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


def test_state_checkpoint_restore_rolls_back_a_step(ctx):
    """vxg_attn_cuda_state_checkpoint (native/metal_cb4_fast.mm:531-570): save the ssm and conv
    states, run a step, restore; the states are bit-identical to the saved ones and a replayed
    step reproduces the first output exactly."""
    import torch
    rng = np.random.default_rng(33)
    B, H, dk, dv = 2, 4, 128, 128
    state = torch.from_numpy((rng.standard_normal((B, H, dv, dk)) * 0.02).astype(np.float32)).cuda()
    conv = torch.from_numpy(rng.standard_normal((B, 3, 1024)).astype(np.float32)).cuda()
    saved = [state.clone(), conv.clone()]
    bak = [torch.empty_like(state), torch.empty_like(conv)]
    A = -torch.ones(H, device="cuda")
    dt = torch.zeros(H, device="cuda")
    q, k, v, br, ar = [torch.from_numpy(x).cuda() for x in inputs(rng, B, H, H, dk, dv)]
    assert ctx.checkpoint([state, conv], bak) == 0
    o1 = vxg_b200.deltanet_step(ctx, q, k, v, br, ar, A, dt, state).clone()
    conv.add_(1.0)
    assert not torch.equal(state, saved[0])
    assert ctx.checkpoint([state, conv], bak, restore=True) == 0
    ctx.sync()
    assert torch.equal(state, saved[0]) and torch.equal(conv, saved[1])
    o2 = vxg_b200.deltanet_step(ctx, q, k, v, br, ar, A, dt, state)
    ctx.sync()
    assert torch.equal(o1, o2)


def test_deltanet_rejects_bad_shapes(ctx):
    rng = np.random.default_rng(32)
    state = np.zeros((1, 4, 32, 96), np.float32)
    q, k, v, br, ar = inputs(rng, 1, 4, 4, 96, 32)
    with pytest.raises(vxg_b200.VxgError) as e:
        vxg_b200.deltanet_step(ctx, q, k, v, br, ar, np.ones(4, np.float32),
                               np.zeros(4, np.float32), state)
    assert e.value.code == -6


def seq_inputs(rng, B, T, n_kh, n_vh, dk, dv):
    q = rng.standard_normal((B, T, n_kh, dk)).astype(np.float32)
    k = rng.standard_normal((B, T, n_kh, dk)).astype(np.float32)
    v = rng.standard_normal((B, T, n_vh, dv)).astype(np.float32)
    br = rng.standard_normal((B, T, n_vh)).astype(np.float32)
    ar = rng.standard_normal((B, T, n_vh)).astype(np.float32)
    return q, k, v, br, ar


@pytest.mark.parametrize("B,T,n_kh,n_vh,dk,dv", [
    (2, 96, 4, 8, 128, 128),
    (3, 40, 2, 4, 64, 64),
    (1, 33, 2, 2, 256, 96),
])
def test_deltanet_prefill_matches_token_by_token_oracle(ctx, B, T, n_kh, n_vh, dk, dv):
    """The reference prefill applies the step token by token (llm_prefill.rs:470-480)."""
    rng = np.random.default_rng(33)
    state = (rng.standard_normal((B, n_vh, dv, dk)) * 0.02).astype(np.float32)
    ref = state.copy()
    A = -np.exp(rng.standard_normal(n_vh) * 0.3).astype(np.float32)
    dt = (rng.standard_normal(n_vh) * 0.1).astype(np.float32)
    q, k, v, br, ar = seq_inputs(rng, B, T, n_kh, n_vh, dk, dv)
    o = vxg_b200.deltanet_prefill(ctx, q, k, v, br, ar, A, dt, state)
    for t in range(T):
        ro = oracle.batch_deltanet(q[:, t], k[:, t], v[:, t], br[:, t], ar[:, t], A, dt, n_kh,
                                   n_vh, dk, dv, 1e-6, 1 / np.sqrt(dk), ref, n_threads=8)
        np.testing.assert_allclose(o[:, t], ro, atol=ATOL, rtol=RTOL, err_msg=f"token {t}")
    np.testing.assert_allclose(state, ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("B,T,n_kh,n_vh,dv,generic", [
    (2, 300, 2, 4, 64, False),      # chunked (WY) mma.sync kernel: 5 chunks, the last partial
    (2, 300, 2, 4, 128, False),     # chunked tcgen05 kernel (dv 128): GQA, the last chunk partial
    (1, 4096, 2, 2, 128, False),    # config-5b prompt length, 64 chunks (tcgen05 kernel)
    (2, 300, 2, 4, 64, True),       # the sequential kernel on the same shapes
])
def test_deltanet_prefill_chunked_matches_sequential_oracle(ctx, B, T, n_kh, n_vh, dv, generic):
    """dk = 128 prompts run the chunked (WY) form; it must match the token-by-token fp32
    recurrence of the reference (llm_prefill.rs:470-480) within the bar, outputs and state."""
    rng = np.random.default_rng(34 + T)
    dk = 128
    state = (rng.standard_normal((B, n_vh, dv, dk)) * 0.02).astype(np.float32)
    ref = state.copy()
    A = -np.exp(rng.standard_normal(n_vh) * 0.3).astype(np.float32)
    dt = (rng.standard_normal(n_vh) * 0.1).astype(np.float32)
    q, k, v, br, ar = seq_inputs(rng, B, T, n_kh, n_vh, dk, dv)
    ctx.force_generic(generic)
    try:
        o = vxg_b200.deltanet_prefill(ctx, q, k, v, br, ar, A, dt, state)
    finally:
        ctx.force_generic(False)
    worst = 0.0
    for t in range(T):
        ro = oracle.batch_deltanet(q[:, t], k[:, t], v[:, t], br[:, t], ar[:, t], A, dt, n_kh,
                                   n_vh, dk, dv, 1e-6, 1 / np.sqrt(dk), ref, n_threads=8)
        np.testing.assert_allclose(o[:, t], ro, atol=ATOL, rtol=RTOL, err_msg=f"token {t}")
        worst = max(worst, float((np.abs(o[:, t] - ro) / (ATOL + RTOL * np.abs(ro))).max()))
    np.testing.assert_allclose(state, ref, atol=ATOL, rtol=RTOL)
    assert worst < 0.25, worst


def test_deltanet_prefill_equals_decode_steps_long(ctx):
    """Config-5b-like length: the on-chip recurrence over 2048 tokens equals 2048 decode steps
    (both on the GPU; size-independent property)."""
    import torch
    rng = np.random.default_rng(34)
    B, T, H, D = 2, 2048, 8, 128
    q, k, v, br, ar = [torch.from_numpy(x).cuda() for x in seq_inputs(rng, B, T, H, H, D, D)]
    s0 = torch.from_numpy((rng.standard_normal((B, H, D, D)) * 0.02).astype(np.float32)).cuda()
    A = -torch.ones(H, device="cuda")
    dt = torch.zeros(H, device="cuda")
    s1 = s0.clone()
    o1 = vxg_b200.deltanet_prefill(ctx, q, k, v, br, ar, A, dt, s1)
    s2 = s0.clone()
    o2 = torch.empty_like(o1)
    for t in range(T):
        o2[:, t] = vxg_b200.deltanet_step(ctx, q[:, t].contiguous(), k[:, t].contiguous(),
                                          v[:, t].contiguous(), br[:, t].contiguous(),
                                          ar[:, t].contiguous(), A, dt, s2)
    ctx.sync()
    torch.testing.assert_close(o1, o2, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(s1, s2, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("n_kh,n_vh,dk,dv,k_sz", [(2, 4, 128, 128, 4), (1, 2, 64, 32, 3)])
def test_step_deltanet_recurrent_dropin(ctx, n_kh, n_vh, dk, dv, k_sz):
    """The whole reference step (conv1d + SiLU, core, RMSNorm * SiLU(z)) for several tokens."""
    rng = np.random.default_rng(35)
    B = 3
    conv_ch = 2 * n_kh * dk + n_vh * dv
    w = (rng.standard_normal((conv_ch, k_sz)) * 0.5).astype(np.float32)
    A = -np.exp(rng.standard_normal(n_vh) * 0.3).astype(np.float32)
    dt = (rng.standard_normal(n_vh) * 0.1).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(dv)).astype(np.float32)
    conv_state = (rng.standard_normal((B, k_sz - 1, conv_ch))).astype(np.float32)
    ssm_state = (rng.standard_normal((B, n_vh, dv, dk)) * 0.02).astype(np.float32)
    ref_conv = conv_state.copy()
    ref_ssm = ssm_state.copy()
    for step in range(5):
        x = rng.standard_normal((B, conv_ch)).astype(np.float32)
        z = rng.standard_normal((B, n_vh * dv)).astype(np.float32)
        ar = rng.standard_normal((B, n_vh)).astype(np.float32)
        br = rng.standard_normal((B, n_vh)).astype(np.float32)
        y = vxg_b200.step_deltanet_recurrent(ctx, x, z, ar, br, w, A, dt, norm_w, conv_state,
                                             ssm_state, n_kh, n_vh, dk, dv, k_sz, 1e-6)
        for b in range(B):
            ry = oracle.step_deltanet_recurrent(x[b], z[b], ar[b], br[b], w, A, dt, norm_w,
                                                ref_conv[b], ref_ssm[b], n_kh, n_vh, dk, dv,
                                                k_sz, 1e-6)
            np.testing.assert_allclose(y[b], ry, atol=ATOL, rtol=RTOL, err_msg=f"step {step}")
        assert np.array_equal(conv_state, ref_conv)   # the rolling history is a pure copy
        np.testing.assert_allclose(ssm_state, ref_ssm, atol=ATOL, rtol=RTOL)
