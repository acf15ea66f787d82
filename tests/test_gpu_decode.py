"""GPU parity of split-KV Q8 decode attention against the oracle (the attention half of
step_full_gqa_q8, crates/vxg-tensor/src/llm_prefill.rs:326-369).

Tolerance (floating point, from the build's acceptance bar): |gpu - ref| <= 1e-3 + 1e-3*|ref|
element-wise.  Q8 codes / scales written by the append are compared bit for bit.
"""
import numpy as np
import pytest

import vxg_b200
from oracle import oracle

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3


def make_pool(ctx, rng, ctx_lens, n_kv, hd, cap=None, outlier_frac=0.0, n_seq=None):
    """Random N(0,1) K/V quantised by the oracle and imported into a device pool."""
    n_seq = n_seq or len(ctx_lens)
    cap = cap or (max(ctx_lens) + 1)
    pool = vxg_b200.KvQ8Pool(ctx, n_seq, n_kv, hd, cap)
    nb = hd // 32
    k_host = np.zeros((n_seq, cap, n_kv, nb, 34), np.uint8)
    v_host = np.zeros_like(k_host)
    for s, L in enumerate(ctx_lens):
        k = rng.standard_normal((L, n_kv, hd)).astype(np.float32)
        v = rng.standard_normal((L, n_kv, hd)).astype(np.float32)
        if outlier_frac:
            m = rng.random((L, n_kv)) < outlier_frac
            k[m] *= 8.0
        k_host[s, :L] = oracle.q8_quantize(k)
        v_host[s, :L] = oracle.q8_quantize(v)
        pool.import_blocks(s, 0, k_host[s, :L], v_host[s, :L])
    return pool, k_host, v_host, cap


def oracle_decode(k_host, v_host, cap, seq, pos, q, n_kv, hd, gates=None, threads=8):
    H = q.shape[1]
    return oracle.batch_decode_q8(seq, pos, q, None, None, k_host.reshape(-1), v_host.reshape(-1),
                                  cap, H, n_kv, hd, gates=gates, do_append=False,
                                  n_threads=threads)


@pytest.mark.parametrize("generic", [False, True])
def test_config1_shape(ctx, generic):
    """B=1, 16 q heads / 2 kv heads, hd 256, ctx 2048."""
    rng = np.random.default_rng(20)
    pool, kh, vh, cap = make_pool(ctx, rng, [2048], 2, 256)
    q = rng.standard_normal((1, 16, 256)).astype(np.float32)
    seq = np.zeros(1, np.int32)
    pos = np.array([2047], np.int32)
    ctx.force_generic(generic)
    try:
        out = pool.decode(seq, pos, q)
    finally:
        ctx.force_generic(False)
    want = oracle_decode(kh, vh, cap, seq, pos, q, 2, 256)
    np.testing.assert_allclose(out, want, atol=ATOL, rtol=RTOL)
    assert np.abs(out - want).max() < 1e-4


@pytest.mark.parametrize("generic", [False, True])
def test_ragged_batch_with_gate(ctx, generic):
    rng = np.random.default_rng(21)
    lens = [1, 2, 63, 64, 65, 127, 128, 129, 700, 1000, 17, 333]
    pool, kh, vh, cap = make_pool(ctx, rng, lens, 2, 256)
    order = rng.permutation(len(lens)).astype(np.int32)
    pos = np.array([lens[s] - 1 for s in order], np.int32)
    q = rng.standard_normal((len(lens), 16, 256)).astype(np.float32)
    gate = rng.standard_normal((len(lens), 16, 256)).astype(np.float32)
    ctx.force_generic(generic)
    try:
        out = pool.decode(order, pos, q, q_gate=gate)
    finally:
        ctx.force_generic(False)
    want = oracle_decode(kh, vh, cap, order, pos, q, 2, 256, gates=gate)
    np.testing.assert_allclose(out, want, atol=ATOL, rtol=RTOL)


def test_decode_with_append_matches_reference_step(ctx):
    """Append-then-attend of step_full_gqa_q8; appended blocks bit-exact."""
    rng = np.random.default_rng(22)
    lens = [5, 100, 257, 64]
    pool, kh, vh, cap = make_pool(ctx, rng, lens, 2, 256, cap=300)
    seq = np.arange(4, dtype=np.int32)
    pos = np.array(lens, np.int32)              # the new token goes at index len
    q = rng.standard_normal((4, 16, 256)).astype(np.float32)
    kn = rng.standard_normal((4, 2, 256)).astype(np.float32)
    vn = rng.standard_normal((4, 2, 256)).astype(np.float32)
    out = pool.decode(seq, pos, q, k_new=kn, v_new=vn)
    kpool, vpool = kh.reshape(-1).copy(), vh.reshape(-1).copy()
    want = oracle.batch_decode_q8(seq, pos, q, kn, vn, kpool, vpool, cap, 16, 2, 256,
                                  do_append=True, n_threads=4)
    np.testing.assert_allclose(out, want, atol=ATOL, rtol=RTOL)
    kp = kpool.reshape(4, cap, 2, 8, 34)
    for b in range(4):
        kb, vb = pool.export_blocks(b, 0, lens[b] + 1)
        assert np.array_equal(kb, kp[b, :lens[b] + 1])
        assert np.array_equal(vb, vpool.reshape(4, cap, 2, 8, 34)[b, :lens[b] + 1])


@pytest.mark.parametrize("H,n_kv,hd", [(4, 2, 64), (8, 8, 128), (32, 2, 128), (12, 4, 96),
                                       (16, 2, 256)])
def test_other_shapes(ctx, H, n_kv, hd):
    """Shapes outside the fast path go through the portable kernel (the reference's own test
    model uses 4 q heads / 2 kv heads / hd 64, llm_gpu_cpu_parity.rs:31-55)."""
    rng = np.random.default_rng(23)
    lens = [1, 40, 513, 1100]
    pool, kh, vh, cap = make_pool(ctx, rng, lens, n_kv, hd)
    seq = np.arange(len(lens), dtype=np.int32)
    pos = np.array(lens, np.int32) - 1
    q = rng.standard_normal((len(lens), H, hd)).astype(np.float32)
    out = pool.decode(seq, pos, q)
    want = oracle_decode(kh, vh, cap, seq, pos, q, n_kv, hd)
    np.testing.assert_allclose(out, want, atol=ATOL, rtol=RTOL)


def test_partials_combine_equal_full(ctx):
    """KV-range split into 3 partials + LSE combine == one full pass (the multi-GPU split)."""
    rng = np.random.default_rng(24)
    L = 5000
    pool, kh, vh, cap = make_pool(ctx, rng, [L], 2, 256, outlier_frac=0.01)
    q = rng.standard_normal((1, 16, 256)).astype(np.float32)
    seq = np.zeros(1, np.int32)
    cuts = [0, 1234, 1235, L]
    ms, ls, os_ = [], [], []
    for a, b in zip(cuts[:-1], cuts[1:]):
        m, l, o = pool.decode_partial(seq, np.array([a], np.int32), np.array([b], np.int32), q)
        ms.append(m[0]), ls.append(l[0]), os_.append(o[0])
    empty = pool.decode_partial(seq, np.array([7], np.int32), np.array([7], np.int32), q)
    assert np.all(np.isneginf(empty[0])) and not empty[1].any() and not empty[2].any()
    ms.append(empty[0][0]), ls.append(empty[1][0]), os_.append(empty[2][0])
    out = vxg_b200.lse_combine(ctx, np.stack(ms), np.stack(ls), np.stack(os_))
    full = pool.decode(seq, np.array([L - 1], np.int32), q)[0]
    np.testing.assert_allclose(out, full, atol=1e-5, rtol=1e-4)
    # the all-gather layout: per part [m | l | o] packed back to back
    packed = np.stack([np.concatenate([m_, l_, o_.reshape(-1)]) for m_, l_, o_ in
                       zip(ms, ls, os_)]).astype(np.float32)
    out_p = vxg_b200.lse_combine_packed(ctx, packed, len(ms), 16, 256)
    np.testing.assert_array_equal(out_p, out)
    want = oracle_decode(kh, vh, cap, seq, np.array([L - 1], np.int32), q, 2, 256)[0]
    np.testing.assert_allclose(out, want, atol=ATOL, rtol=RTOL)


def test_outlier_rows_long_context(ctx):
    """Config-3 distribution (1% of K rows x8) at 16k tokens, fast vs oracle."""
    rng = np.random.default_rng(25)
    L = 16384
    pool, kh, vh, cap = make_pool(ctx, rng, [L], 2, 256, outlier_frac=0.01)
    q = rng.standard_normal((1, 16, 256)).astype(np.float32)
    seq = np.zeros(1, np.int32)
    pos = np.array([L - 1], np.int32)
    out = pool.decode(seq, pos, q)
    want = oracle_decode(kh, vh, cap, seq, pos, q, 2, 256)
    np.testing.assert_allclose(out, want, atol=ATOL, rtol=RTOL)


def test_device_tensors_and_torch_stream(ctx):
    """Device-memory calls on torch's stream equal host-memory calls."""
    import torch
    rng = np.random.default_rng(26)
    lens = [300, 90]
    pool, kh, vh, cap = make_pool(ctx, rng, lens, 2, 256, cap=400)
    q = rng.standard_normal((2, 16, 256)).astype(np.float32)
    seq = np.arange(2, dtype=np.int32)
    pos = np.array(lens, np.int32) - 1
    host = pool.decode(seq, pos, q)
    dev = pool.decode(torch.from_numpy(seq).cuda(), torch.from_numpy(pos).cuda(),
                      torch.from_numpy(q).cuda())
    ctx.sync()
    np.testing.assert_array_equal(dev.cpu().numpy(), host)


def test_decode_steps_replayed_from_cuda_graph(ctx):
    """Append + attend steps captured once in a CUDA graph and replayed give the eager results
    (the append, split and combine kernels of a step are chained by programmatic dependent
    launch, which a capture must keep in order)."""
    import torch
    rng = np.random.default_rng(29)
    lens = [700, 2100, 64]
    pool, kh, vh, cap = make_pool(ctx, rng, lens, 2, 256, cap=2200)
    n, steps = len(lens), 3
    seq = torch.arange(n, dtype=torch.int32, device="cuda")
    pos = [torch.tensor(lens, dtype=torch.int32, device="cuda") + i for i in range(steps)]
    q = [torch.from_numpy(rng.standard_normal((n, 16, 256)).astype(np.float32)).cuda()
         for _ in range(steps)]
    kn = [torch.from_numpy(rng.standard_normal((n, 2, 256)).astype(np.float32)).cuda()
          for _ in range(steps)]
    vn = [torch.from_numpy(rng.standard_normal((n, 2, 256)).astype(np.float32)).cuda()
          for _ in range(steps)]
    outs = [torch.empty((n, 16, 256), device="cuda") for _ in range(steps)]
    for i in range(steps):
        pool.decode(seq, pos[i], q[i], kn[i], vn[i], out=outs[i], max_ctx=cap)
    torch.cuda.synchronize()
    eager = [o.cpu().numpy().copy() for o in outs]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(steps):
            # the appends rewrite the same positions with the same K/V on every replay
            pool.decode(seq, pos[i], q[i], kn[i], vn[i], out=outs[i], max_ctx=cap)
    for rep in range(2):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for i in range(steps):
            np.testing.assert_allclose(outs[i].cpu().numpy(), eager[i], atol=ATOL, rtol=RTOL,
                                       err_msg=f"replay {rep} step {i}")
    del g
    assert ctx.sync() == 0


def test_back_to_back_calls_on_gpu_computed_positions(ctx):
    """Decode calls issued back to back on one stream, each right after a torch kernel that
    computes its positions, without append: every call sees its own positions and the previous
    call's combine is done with the shared scratch before the next split reuses it."""
    import torch
    rng = np.random.default_rng(31)
    lens = [1500, 333, 2900, 64, 777]
    pool, kh, vh, cap = make_pool(ctx, rng, lens, 2, 256, cap=3000)
    n, calls = len(lens), 5
    seq_np = np.arange(n, dtype=np.int32)
    qs = rng.standard_normal((calls, n, 16, 256)).astype(np.float32)
    seq = torch.from_numpy(seq_np).cuda()
    p = torch.tensor(lens, dtype=torch.int32, device="cuda") - 1
    q_dev = torch.from_numpy(qs).cuda()
    torch.cuda.synchronize()
    outs = []
    for i in range(calls):
        p = p - 3 * (i + 1)  # a kernel on the same stream right before the call
        outs.append(pool.decode(seq, p, q_dev[i]))
    torch.cuda.synchronize()
    assert ctx.sync() == 0
    pos = np.array(lens, np.int32) - 1
    for i in range(calls):
        pos = pos - 3 * (i + 1)
        want = pool.decode(seq_np, pos, qs[i])
        np.testing.assert_allclose(outs[i].cpu().numpy(), want, atol=ATOL, rtol=RTOL,
                                   err_msg=f"call {i}")


def test_nonfinite_query_reports_warning(ctx):
    rng = np.random.default_rng(27)
    pool, kh, vh, cap = make_pool(ctx, rng, [50], 2, 256)
    q = rng.standard_normal((1, 16, 256)).astype(np.float32)
    q[0, 3, 7] = np.nan
    out = pool.decode(np.zeros(1, np.int32), np.array([49], np.int32), q)
    assert pool.last_rc == 1
    assert np.isnan(out[0, 3]).all() and np.isfinite(np.delete(out[0], 3, axis=0)).all()


def test_overlapped_host_steps_match_synchronous_steps(ctx):
    """vxg_attn_cuda_q8_decode_host_async: a run of appended decode steps whose copies overlap
    the neighbouring steps' kernels gives, step for step, the bytes of the synchronous
    host-memory call on an identical pool; the appended Q8 blocks are identical too."""
    rng = np.random.default_rng(77)
    lens = [500, 3, 1200, 64, 900]
    H, n_kv, hd, steps = 16, 2, 256, 7
    cap = max(lens) + steps + 1
    pool_a, k_host, v_host, _ = make_pool(ctx, rng, lens, n_kv, hd, cap=cap)
    pool_b = vxg_b200.KvQ8Pool(ctx, len(lens), n_kv, hd, cap)
    for s, L in enumerate(lens):
        pool_b.import_blocks(s, 0, k_host[s, :L], v_host[s, :L])
    B = len(lens)
    seq = ctx.pinned_empty((B,), np.int32)
    seq[...] = np.array([3, 0, 4, 2, 1], np.int32)
    pos = ctx.pinned_empty((steps, B), np.int32)
    q = ctx.pinned_empty((steps, B, H, hd), np.float32)
    kn = ctx.pinned_empty((steps, B, n_kv, hd), np.float32)
    vn = ctx.pinned_empty((steps, B, n_kv, hd), np.float32)
    gate = ctx.pinned_empty((steps, B, H, hd), np.float32)
    for i in range(steps):
        pos[i] = np.array([lens[s] for s in seq], np.int32) + i
    q[...] = rng.standard_normal(q.shape)
    kn[...] = rng.standard_normal(kn.shape)
    vn[...] = rng.standard_normal(vn.shape)
    gate[...] = rng.standard_normal(gate.shape)
    outs = [ctx.pinned_empty((B, H, hd), np.float32) for _ in range(steps)]
    tickets = []
    for i in range(steps):
        tickets.append(pool_b.decode_host_async(seq, pos[i], q[i], kn[i], vn[i], q_gate=gate[i],
                                                out=outs[i], max_ctx=cap))
    assert tickets == sorted(tickets) and len(set(tickets)) == steps
    assert [ctx.wait(t) for t in reversed(tickets)] == [0] * steps
    assert ctx.wait(tickets[0]) == 0  # waited before
    for i in range(steps):
        want = pool_a.decode(np.array(seq), np.array(pos[i]), np.array(q[i]), np.array(kn[i]),
                             np.array(vn[i]), q_gate=np.array(gate[i]), max_ctx=cap)
        assert np.array_equal(outs[i], want), f"step {i}"
    for s, L in enumerate(lens):
        ka, va = pool_a.export_blocks(s, 0, L + steps)
        kb, vb = pool_b.export_blocks(s, 0, L + steps)
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)
    pool_a.close()
    pool_b.close()


def test_overlapped_host_step_rejects_bad_positions(ctx):
    pool = vxg_b200.KvQ8Pool(ctx, 2, 2, 256, 16)
    q = np.zeros((1, 16, 256), np.float32)
    with pytest.raises(vxg_b200.VxgError) as e:
        pool.decode_host_async(np.array([0], np.int32), np.array([16], np.int32), q)
    assert e.value.code == -3  # VXG_ATTN_ERR_BUFFER_TOO_SMALL: position beyond the capacity
    with pytest.raises(vxg_b200.VxgError):
        ctx.wait(10 ** 9)
    pool.close()


@pytest.mark.parametrize("with_gate", [True, False])
def test_wide_batch_single_pass_combine(ctx, with_gate):
    """Batches of >= 32 entries take the single-pass combine (one CTA per entry and 16-dim
    chunk): ragged lengths from 1 token to several split segments, repeated sequence ids, with
    and without the sigmoid gate."""
    rng = np.random.default_rng(131)
    lens = [int(x) for x in rng.integers(1, 2500, 40)] + [2, 1, 96, 97, 5000]
    pool, kh, vh, cap = make_pool(ctx, rng, lens, 2, 256)
    B = 48
    seq = np.concatenate([rng.permutation(len(lens)), rng.integers(0, len(lens), B - len(lens))])
    seq = seq.astype(np.int32)
    pos = np.array([lens[s] - 1 for s in seq], np.int32)
    q = rng.standard_normal((B, 16, 256)).astype(np.float32)
    gate = rng.standard_normal((B, 16, 256)).astype(np.float32) if with_gate else None
    out = pool.decode(seq, pos, q, q_gate=gate, max_ctx=cap)
    want = oracle_decode(kh, vh, cap, seq, pos, q, 2, 256, gates=gate)
    np.testing.assert_allclose(out, want, atol=ATOL, rtol=RTOL)
    pool.close()


def test_entry_over_more_slots_than_one_combine_chunk(ctx):
    """A 32-entry batch (single-level combine) whose last entry holds most of the units, so it
    is spread over more split CTAs than the combine stages in one chunk (128 slots): the
    chunks' running maximum is rescaled between them.  1% of K rows x8 make the per-chunk
    maxima differ."""
    rng = np.random.default_rng(141)
    lens = [96] * 31 + [28800]
    pool, kh, vh, cap = make_pool(ctx, rng, lens, 2, 256, outlier_frac=0.01)
    seq = np.arange(32, dtype=np.int32)
    pos = np.array([L - 1 for L in lens], np.int32)
    q = rng.standard_normal((32, 16, 256)).astype(np.float32)
    out = pool.decode(seq, pos, q, max_ctx=cap)
    want = oracle_decode(kh, vh, cap, seq, pos, q, 2, 256)
    np.testing.assert_allclose(out, want, atol=ATOL, rtol=RTOL)
    pool.close()


def test_misaligned_device_arrays_are_rejected(ctx):
    """Device arrays are accessed with 16-byte vectors and bulk copies: a view that starts one
    float into an allocation is refused on the host, before any launch."""
    import torch
    pool = vxg_b200.KvQ8Pool(ctx, 1, 2, 256, 16)
    seq = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    qbuf = torch.zeros(16 * 256 + 1, device="cuda")
    q = qbuf[1:].view(1, 16, 256)
    with pytest.raises(vxg_b200.VxgError) as e:
        pool.decode(seq, pos, q)
    assert e.value.code == -2 and "aligned" in str(e.value)
    ok = pool.decode(seq, pos, qbuf[:-1].view(1, 16, 256))
    assert ctx.sync() == 0 and torch.isfinite(ok).all()
    pool.close()
