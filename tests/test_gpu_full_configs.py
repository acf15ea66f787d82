"""GPU parity of the five benchmark configurations at their full sizes, against the oracle.

Each test runs the CUDA path through the C ABI on seeded inputs with a configuration's shapes
and value distributions and compares every output with the oracle (the C restatement of the
reference's CPU operators) on the same inputs:

* config 2: 64 sequences with contexts U[1024, 32768], eight append + attend steps, every output
  and every appended Q8 block (llm_prefill.rs:311-369);
* config 2 again with heavy-tailed queries: a few channels of every head at x30 to x1000, the
  shape of post-q_norm / RoPE queries with outlier channels;
* config 3: 262144 tokens with 1% of K rows x8, one append + attend step;
* config 4: 256 DeltaNet steps over 64 sequences x 32 heads, every output and the final state
  (llm_ops.rs:150-184);
* config 5a: one 8192-token prompt, 64 evenly spaced tokens (llm_prefill.rs:497-527);
* config 5b: one 8192-token prompt x 32 heads, every output and the final state against the
  token-by-token recurrence (llm_prefill.rs:470-480).

Bar (floating point): |gpu - ref| <= 1e-3 + 1e-3 |ref| element-wise; each test also asserts
the worst ratio to that bar below a margin taken from measurements, so that a drift shows
before it fails the bar.  Q8 codes and scales are compared byte for byte.  Run with -s to see
the per-configuration ratios.
"""
import os

import numpy as np
import pytest

import vxg_b200
from oracle import oracle
from vxg_b200 import workloads as wl

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3
CORES = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def ratio(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float((np.abs(got - want) / (ATOL + RTOL * np.abs(want))).max())


def report(name, r):
    print(f"\n[parity] {name}: worst / bar = {r:.4f}", flush=True)


def _config2_pool(ctx, seed):
    batch = wl.DecodeBatch(seed=seed)
    lens = batch.ctx_lens()
    n = batch.n_seq
    steps = 8
    cap = int(lens.max()) + steps + 1
    pool = vxg_b200.KvQ8Pool(ctx, n, wl.HKV, wl.HD, cap)
    wl.fill_pool_device(pool, lens, seed=seed + 6)
    kp = np.zeros((n, cap, wl.HKV, wl.HD // 32, 34), np.uint8)
    vp = np.zeros_like(kp)
    for s in range(n):
        kp[s, :lens[s]], vp[s, :lens[s]] = pool.export_blocks(s, 0, int(lens[s]))
    return pool, lens, n, steps, cap, kp, vp


def heavy_tailed(rng, shape, mults):
    """N(0,1) queries with 4 channels of every head scaled by that head's multiplier."""
    q = rng.standard_normal(shape).astype(np.float32)
    B, H, D = shape
    for b in range(B):
        for h in range(H):
            idx = rng.choice(D, 4, replace=False)
            q[b, h, idx] *= mults[(b * H + h) % len(mults)]
    return q


@pytest.mark.parametrize("queries", ["normal", "heavy_tailed"])
def test_config2_full_batch_eight_steps(ctx, queries):
    """64 ragged sequences, 8 consecutive append + attend steps; outputs within the bar at every
    step, appended blocks bit-exact."""
    rng = np.random.default_rng(201 if queries == "normal" else 202)
    pool, lens, n, steps, cap, kp, vp = _config2_pool(ctx, seed=1 if queries == "normal" else 2)
    kf, vf = kp.reshape(-1), vp.reshape(-1)
    seq = rng.permutation(n).astype(np.int32)
    worst = 0.0
    for i in range(steps):
        if queries == "normal":
            q = rng.standard_normal((n, wl.HQ, wl.HD)).astype(np.float32)
        else:
            q = heavy_tailed(rng, (n, wl.HQ, wl.HD), [1.0, 30.0, 100.0, 300.0, 1000.0])
        kn = rng.standard_normal((n, wl.HKV, wl.HD)).astype(np.float32)
        vn = rng.standard_normal((n, wl.HKV, wl.HD)).astype(np.float32)
        pos = (lens[seq] + i).astype(np.int32)
        got = pool.decode(seq, pos, q, kn, vn, max_ctx=cap)
        want = oracle.batch_decode_q8(seq, pos, q, kn, vn, kf, vf, cap, wl.HQ, wl.HKV, wl.HD,
                                      do_append=True, n_threads=CORES)
        np.testing.assert_allclose(got, want, atol=ATOL, rtol=RTOL, err_msg=f"step {i}")
        worst = max(worst, ratio(got, want))
    for s in range(n):
        kg, vg = pool.export_blocks(s, int(lens[s]), steps)
        assert np.array_equal(kg, kp[s, lens[s]:lens[s] + steps]), f"K blocks of seq {s}"
        assert np.array_equal(vg, vp[s, lens[s]:lens[s] + steps]), f"V blocks of seq {s}"
    report(f"config 2, {queries} queries (64 seqs x 8 steps)", worst)
    assert worst < (0.1 if queries == "normal" else 0.3)   # measured 0.03 / 0.19
    pool.close()


@pytest.mark.parametrize("mult", [1.0, 30.0, 100.0, 1000.0])
def test_heavy_tailed_queries_short_and_long_contexts(ctx, mult):
    """Queries with outlier channels against contexts from one token to 20k, fast kernel; mult
    1 is plain N(0,1) queries, whose short contexts give the most peaked softmax."""
    rng = np.random.default_rng(203)
    lens = [1, 2, 17, 96, 300, 2048, 20000]
    n_kv, hd = 2, 256
    cap = max(lens) + 1
    pool = vxg_b200.KvQ8Pool(ctx, len(lens), n_kv, hd, cap)
    kp = np.zeros((len(lens), cap, n_kv, hd // 32, 34), np.uint8)
    vp = np.zeros_like(kp)
    for s, L in enumerate(lens):
        kp[s, :L] = oracle.q8_quantize(rng.standard_normal((L, n_kv, hd)).astype(np.float32))
        vp[s, :L] = oracle.q8_quantize(rng.standard_normal((L, n_kv, hd)).astype(np.float32))
        pool.import_blocks(s, 0, kp[s, :L], vp[s, :L])
    seq = np.arange(len(lens), dtype=np.int32)
    pos = np.array(lens, np.int32) - 1
    worst = 0.0
    for trial in range(3):
        q = heavy_tailed(rng, (len(lens), 16, hd), [mult])
        got = pool.decode(seq, pos, q)
        want = oracle.batch_decode_q8(seq, pos, q, None, None, kp.reshape(-1), vp.reshape(-1),
                                      cap, 16, n_kv, hd, do_append=False, n_threads=CORES)
        np.testing.assert_allclose(got, want, atol=ATOL, rtol=RTOL)
        worst = max(worst, ratio(got, want))
    report(f"queries with channels x{mult:g}, contexts 1..20000", worst)
    # plain queries take the two-digit path with P rounded once to f16, whose error shows on the
    # one- and two-token contexts (measured 0.35); outlier heads take the three-digit path, whose
    # error still grows with the outlier (measured 0.02 at x30 / x100, 0.16 at x1000)
    assert worst < (0.5 if mult == 1.0 else 0.3)
    pool.close()


def test_config3_full_context_one_step(ctx):
    """262144 tokens, 1% of K rows x8, a new outlier K row appended, attend over all of it."""
    rng = np.random.default_rng(204)
    L = 262144
    pool = vxg_b200.KvQ8Pool(ctx, 1, wl.HKV, wl.HD, L + 2)
    wl.fill_pool_device(pool, [L], seed=3, outlier_frac=0.01)
    kp = np.zeros((1, L + 2, wl.HKV, wl.HD // 32, 34), np.uint8)
    vp = np.zeros_like(kp)
    kp[0, :L], vp[0, :L] = pool.export_blocks(0, 0, L)
    q = rng.standard_normal((1, wl.HQ, wl.HD)).astype(np.float32)
    kn = (rng.standard_normal((1, wl.HKV, wl.HD)) * 8).astype(np.float32)
    vn = rng.standard_normal((1, wl.HKV, wl.HD)).astype(np.float32)
    seq, pos = np.zeros(1, np.int32), np.array([L], np.int32)
    got = pool.decode(seq, pos, q, kn, vn, max_ctx=L + 2)
    want = oracle.batch_decode_q8(seq, pos, q, kn, vn, kp.reshape(-1), vp.reshape(-1), L + 2,
                                  wl.HQ, wl.HKV, wl.HD, do_append=True)
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=RTOL)
    kg, vg = pool.export_blocks(0, L, 1)
    assert np.array_equal(kg[0], kp[0, L]) and np.array_equal(vg[0], vp[0, L])
    r = ratio(got, want)
    report("config 3 (ctx 262144, 1% outlier K rows)", r)
    # N(0,1) queries take the two-digit path; the x8 K rows scale its score error by 8 and, with
    # scores of std 8 on those rows, the softmax peaks on them (measured 0.64)
    assert r < 0.8
    pool.close()


def test_config4_256_steps(ctx):
    """64 sequences x 32 heads, dk = dv = 128, 256 consecutive steps: every step's output and the
    final state within the bar."""
    import torch
    B, H, D, T = 64, 32, 128, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(205)
    state = torch.randn((B, H, D, D), generator=g, device="cuda") * 0.02
    st_host = state.cpu().numpy().copy()
    q = torch.randn((T, B, H, D), generator=g, device="cuda")
    k = torch.randn((T, B, H, D), generator=g, device="cuda")
    v = torch.randn((T, B, H, D), generator=g, device="cuda")
    br = torch.randn((T, B, H), generator=g, device="cuda")
    ar = torch.randn((T, B, H), generator=g, device="cuda")
    A, dt = -torch.ones(H, device="cuda"), torch.zeros(H, device="cuda")
    outs = torch.empty((T, B, H, D), device="cuda")
    for t in range(T):
        vxg_b200.deltanet_step(ctx, q[t], k[t], v[t], br[t], ar[t], A, dt, state, o=outs[t])
    assert ctx.sync() == 0
    hq, hk, hv, hb, ha = (x.cpu().numpy() for x in (q, k, v, br, ar))
    An, dtn = A.cpu().numpy(), dt.cpu().numpy()
    got = outs.cpu().numpy()
    worst = 0.0
    for t in range(T):
        want = oracle.batch_deltanet(hq[t], hk[t], hv[t], hb[t], ha[t], An, dtn, H, H, D, D, 1e-6,
                                     1.0 / np.sqrt(D), st_host, n_threads=CORES)
        np.testing.assert_allclose(got[t], want, atol=ATOL, rtol=RTOL, err_msg=f"step {t}")
        worst = max(worst, ratio(got[t], want))
    st_got = state.cpu().numpy()
    np.testing.assert_allclose(st_got, st_host, atol=ATOL, rtol=RTOL)
    rs = ratio(st_got, st_host)
    report("config 4, outputs of 256 steps", worst)
    report("config 4, state after 256 steps", rs)
    assert worst < 0.05 and rs < 0.05


def test_config5a_prompt_8192(ctx):
    """One 8192-token bf16 prompt of config 5a: the cache equals the oracle quantiser's output
    byte for byte, and 64 evenly spaced tokens (the first one included) equal the reference's
    per-token step."""
    import torch
    N, H, KV, HD = 8192, 16, 2, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(206)
    q = torch.randn((1, N, H, HD), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((1, N, KV, HD), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((1, N, KV, HD), generator=g, device="cuda").to(torch.bfloat16)
    pool = vxg_b200.KvQ8Pool(ctx, 1, KV, HD, N)
    seq = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = pool.prefill(seq, pos, q, k, v, max_ctx=N)
    assert ctx.sync() == 0
    kb, vb = pool.export_blocks(0, 0, N)
    assert np.array_equal(kb, oracle.q8_quantize(k[0].float().cpu().numpy()))
    assert np.array_equal(vb, oracle.q8_quantize(v[0].float().cpu().numpy()))
    t_idx = ((np.arange(64) + 0.5) * N / 64).astype(np.int64)
    t_idx[0] = 0
    qs = q[0, torch.as_tensor(t_idx, device="cuda")].float().cpu().numpy()
    want = oracle.batch_decode_q8(np.zeros(64, np.int32), t_idx.astype(np.int32), qs, None, None,
                                  kb.reshape(-1), vb.reshape(-1), N, H, KV, HD, do_append=False,
                                  n_threads=CORES)
    got = out[0, torch.as_tensor(t_idx, device="cuda")].cpu().numpy()
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=RTOL)
    r = ratio(got, want)
    report("config 5a (8192-token prompt, 64 tokens)", r)
    assert r < 0.02
    pool.close()


def test_config5b_prompt_8192_all_heads(ctx):
    """One 8192-token prompt x 32 heads of config 5b (chunked WY kernel): every output and the
    final state against the token-by-token recurrence."""
    import torch
    T, H, D = 8192, 32, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(207)
    q, k, v = (torch.randn((1, T, H, D), generator=g, device="cuda") for _ in range(3))
    br, ar = (torch.randn((1, T, H), generator=g, device="cuda") for _ in range(2))
    A, dt = -torch.ones(H, device="cuda"), torch.zeros(H, device="cuda")
    state = torch.randn((1, H, D, D), generator=g, device="cuda") * 0.02
    st = state.cpu().numpy().copy()
    o = vxg_b200.deltanet_prefill(ctx, q, k, v, br, ar, A, dt, state)
    assert ctx.sync() == 0
    hq, hk, hv, hb, ha = (x.cpu().numpy() for x in (q, k, v, br, ar))
    An, dtn = A.cpu().numpy(), dt.cpu().numpy()
    want = np.zeros((T, H, D), np.float32)
    sth = np.ascontiguousarray(st[0].reshape(H, 1, D, D))   # heads as one-head batch entries
    for t in range(T):
        want[t] = oracle.batch_deltanet(hq[0, t].reshape(H, 1, D), hk[0, t].reshape(H, 1, D),
                                        hv[0, t].reshape(H, 1, D), hb[0, t].reshape(H, 1),
                                        ha[0, t].reshape(H, 1), An, dtn, 1, 1, D, D, 1e-6,
                                        1.0 / np.sqrt(D), sth, n_threads=CORES).reshape(H, D)
    got = o[0].cpu().numpy()
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=RTOL)
    st_got = state[0].cpu().numpy()
    np.testing.assert_allclose(st_got, sth.reshape(H, D, D), atol=ATOL, rtol=RTOL)
    ro, rs = ratio(got, want), ratio(st_got, sth.reshape(H, D, D))
    report("config 5b, outputs (8192 tokens x 32 heads)", ro)
    report("config 5b, final state", rs)
    assert ro < 0.1 and rs < 0.05
