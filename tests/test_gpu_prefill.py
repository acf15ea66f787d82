"""GPU parity of the chunked causal prefill (vxg_attn_cuda_q8_prefill) against the reference's
token-by-token prefill: prompt token ti runs step_full_gqa_q8 at pos + ti, appending its K/V
and attending over [0, pos + ti] (crates/vxg-tensor/src/llm_prefill.rs:497-517, :311-369).

Appended Q8 codes and scales are compared bit for bit.  Outputs: |gpu - ref| <= 1e-3 +
1e-3*|ref| element-wise.  The tensor-core path forms every product from f16 hi/lo operand
splits with f32 accumulation, so it sits far inside that bar (checked below at 2% of it).
"""
import numpy as np
import pytest

import vxg_b200
from oracle import oracle

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3


def _bf16_bits(x):
    """float32 -> bf16 bit patterns (round to nearest even) as uint16."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def _bf16_to_f32(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _prefilled_pools(ctx, rng, n_seq, n_kv, hd, cap, prior):
    """Pools (device and oracle host copy) with `prior[s]` random tokens already cached."""
    nb = hd // 32
    pool = vxg_b200.KvQ8Pool(ctx, n_seq, n_kv, hd, cap)
    k_host = np.zeros((n_seq, cap, n_kv, nb, 34), np.uint8)
    v_host = np.zeros_like(k_host)
    for s, L in enumerate(prior):
        if L == 0:
            continue
        k_host[s, :L] = oracle.q8_quantize(rng.standard_normal((L, n_kv, hd)).astype(np.float32))
        v_host[s, :L] = oracle.q8_quantize(rng.standard_normal((L, n_kv, hd)).astype(np.float32))
        pool.import_blocks(s, 0, k_host[s, :L], v_host[s, :L])
    return pool, k_host, v_host


def _run_case(ctx, rng, n_head, n_kv, hd, prior, seq, n_tok, gated=False, bf16=False,
              device=False, cap=None, generic=False):
    n_seq = len(prior)
    B = len(seq)
    cap = cap or (max(prior) + n_tok + 3)
    pool, kh, vh = _prefilled_pools(ctx, rng, n_seq, n_kv, hd, cap, prior)
    seq = np.asarray(seq, np.int32)
    pos = np.asarray([prior[s] for s in seq], np.int32)
    q = rng.standard_normal((B, n_tok, n_head, hd)).astype(np.float32)
    k = rng.standard_normal((B, n_tok, n_kv, hd)).astype(np.float32)
    v = rng.standard_normal((B, n_tok, n_kv, hd)).astype(np.float32)
    g = rng.standard_normal((B, n_tok, n_head, hd)).astype(np.float32) if gated else None
    if bf16:
        qb, kb, vb = _bf16_bits(q), _bf16_bits(k), _bf16_bits(v)
        gb = _bf16_bits(g) if gated else None
        q, k, v = _bf16_to_f32(qb), _bf16_to_f32(kb), _bf16_to_f32(vb)
        g = _bf16_to_f32(gb) if gated else None
        args = (qb, kb, vb, gb)
    else:
        args = (q, k, v, g)
    ctx.force_generic(generic)
    if device:
        import torch

        def dev(x):
            if x is None:
                return None
            if x.dtype == np.uint16:
                return torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
            return torch.from_numpy(x).cuda()
        out = pool.prefill(torch.from_numpy(seq).cuda(), torch.from_numpy(pos).cuda(),
                           *[dev(x) for x in args[:3]], q_gate=dev(args[3]))
        assert ctx.sync() == 0
        out = out.cpu().numpy()
    else:
        out = pool.prefill(seq, pos, *args[:3], q_gate=args[3])
        assert pool.last_rc == 0
    ctx.force_generic(False)
    want = oracle.prefill_q8(seq, pos, q, k, v, kh.reshape(-1), vh.reshape(-1), cap, n_head,
                             n_kv, hd, gates=g, n_threads=8)
    np.testing.assert_allclose(out, want, atol=ATOL, rtol=RTOL)
    for s in set(seq.tolist()):
        kd, vd = pool.export_blocks(s, 0, cap)
        assert np.array_equal(kd.reshape(kh[s].shape), kh[s]), f"K blocks of seq {s}"
        assert np.array_equal(vd.reshape(vh[s].shape), vh[s]), f"V blocks of seq {s}"
    pool.close()
    return out, want


def test_prefill_f32_host_ragged(ctx):
    """Qwen-style GQA 16/2/256; prompts continue caches of 0, 37 and 130 tokens; n_tok not a
    multiple of the 16-token query block; sequence ids permuted."""
    rng = np.random.default_rng(50)
    out, want = _run_case(ctx, rng, 16, 2, 256, prior=[37, 0, 130], seq=[2, 0, 1], n_tok=150)
    # split operands: only accumulation-order rounding remains, also for the first tokens
    ratio = np.abs(out - want) / (ATOL + RTOL * np.abs(want))
    assert ratio.max() < 0.02


@pytest.mark.parametrize("generic", [False, True])
def test_prefill_bf16_device_gated(ctx, generic):
    """bf16 inputs: the tcgen05/TMEM kernel (generic=False) and the mma.sync kernel."""
    rng = np.random.default_rng(51)
    out, want = _run_case(ctx, rng, 16, 2, 256, prior=[5, 64], seq=[1, 0], n_tok=97, gated=True,
                          bf16=True, device=True, generic=generic)
    ratio = np.abs(out - want) / (ATOL + RTOL * np.abs(want))
    assert ratio.max() < 0.02


@pytest.mark.parametrize("n_head,n_kv", [(16, 2), (32, 2), (8, 2), (4, 4)])
def test_prefill_bf16_tensor_memory_kernel(ctx, n_head, n_kv):
    """The tcgen05 kernel at head_dim 256 over query groups of 16, 8, 4 and 1 heads per kv head,
    prompts continuing cached contexts (0, 33 and 300 tokens; n_tok not a multiple of the
    query block or the 32-key tile)."""
    rng = np.random.default_rng(57 + n_head)
    out, want = _run_case(ctx, rng, n_head, n_kv, 256, prior=[33, 0, 300], seq=[2, 1, 0],
                          n_tok=75, bf16=True, device=True)
    ratio = np.abs(out - want) / (ATOL + RTOL * np.abs(want))
    assert ratio.max() < 0.02


@pytest.mark.parametrize("n_head,n_kv,hd", [(8, 2, 128), (4, 4, 64), (32, 2, 128), (4, 1, 256)])
def test_prefill_other_shapes(ctx, n_head, n_kv, hd):
    rng = np.random.default_rng(52 + n_head + hd)
    _run_case(ctx, rng, n_head, n_kv, hd, prior=[3, 70], seq=[0, 1], n_tok=45)


def test_prefill_single_token_equals_decode(ctx):
    """n_tok = 1 is one decode step: the same result as vxg_attn_cuda_q8_decode (whose f16
    P x V rounding leaves it ~1e-4 from the reference, inside the bar) and as the oracle."""
    rng = np.random.default_rng(53)
    n_kv, hd, n_head, cap = 2, 256, 16, 600
    pool, kh, vh = _prefilled_pools(ctx, rng, 2, n_kv, hd, cap, [500, 17])
    q = rng.standard_normal((2, 1, n_head, hd)).astype(np.float32)
    k = rng.standard_normal((2, 1, n_kv, hd)).astype(np.float32)
    v = rng.standard_normal((2, 1, n_kv, hd)).astype(np.float32)
    seq = np.array([0, 1], np.int32)
    pos = np.array([500, 17], np.int32)
    a = pool.prefill(seq, pos, q, k, v)
    b = pool.decode(seq, pos, q[:, 0], k[:, 0], v[:, 0])  # re-appends the same token
    np.testing.assert_allclose(a[:, 0], b, atol=ATOL, rtol=RTOL)
    kh[0, 500] = oracle.q8_quantize(k[0, 0])
    vh[0, 500] = oracle.q8_quantize(v[0, 0])
    kh[1, 17] = oracle.q8_quantize(k[1, 0])
    vh[1, 17] = oracle.q8_quantize(v[1, 0])
    want = oracle.batch_decode_q8(seq, pos, q[:, 0], None, None, kh.reshape(-1), vh.reshape(-1),
                                  cap, n_head, n_kv, hd, do_append=False)
    ratio = np.abs(a[:, 0] - want) / (ATOL + RTOL * np.abs(want))
    assert ratio.max() < 0.02
    pool.close()


def test_prefill_long_prompt(ctx):
    """One 1100-token prompt (many 64-key tiles, causal diagonal at every block)."""
    rng = np.random.default_rng(54)
    _run_case(ctx, rng, 16, 2, 256, prior=[0], seq=[0], n_tok=1100)


def test_prefill_rejects_positions_beyond_capacity(ctx):
    rng = np.random.default_rng(55)
    pool = vxg_b200.KvQ8Pool(ctx, 1, 2, 256, 64)
    q = rng.standard_normal((1, 10, 16, 256)).astype(np.float32)
    k = rng.standard_normal((1, 10, 2, 256)).astype(np.float32)
    with pytest.raises(vxg_b200.VxgError) as e:
        pool.prefill(np.array([0], np.int32), np.array([60], np.int32), q, k, k)
    assert e.value.code == -3
    pool.close()


def test_prefill_config5a_shape_sampled(ctx):
    """BASELINE config 5a shape at reduced batch: 2 x 8192-token bf16 prompts, 16/2/256.  All
    appended blocks are checked bit for bit against the oracle quantiser; attention outputs are
    checked against the oracle at sampled tokens (first, tile edges, middle, last)."""
    import torch
    B, N, H, KV, HD = 2, 8192, 16, 2, 256
    g = torch.Generator(device="cuda").manual_seed(56)
    q = torch.randn(B, N, H, HD, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, N, KV, HD, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, N, KV, HD, device="cuda", generator=g).to(torch.bfloat16)
    pool = vxg_b200.KvQ8Pool(ctx, B, KV, HD, N)
    seq = torch.arange(B, dtype=torch.int32, device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = pool.prefill(seq, pos, q, k, v)
    assert ctx.sync() == 0
    out = out.cpu().numpy()
    kf = k.float().cpu().numpy()
    vf = v.float().cpu().numpy()
    qf = q.float().cpu().numpy()
    for s in range(B):
        kd, vd = pool.export_blocks(s, 0, N)
        kq = oracle.q8_quantize(kf[s])
        vq = oracle.q8_quantize(vf[s])
        assert np.array_equal(kd.reshape(kq.shape), kq)
        assert np.array_equal(vd.reshape(vq.shape), vq)
        for t in [0, 1, 15, 16, 63, 64, 65, 4095, 4096, 8190, 8191]:
            want = oracle.q8_attend(qf[s, t], kq.reshape(-1), vq.reshape(-1), H, KV, HD, t + 1)
            np.testing.assert_allclose(out[s, t], want, atol=ATOL, rtol=RTOL)
    pool.close()
