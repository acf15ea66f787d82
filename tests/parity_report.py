"""Parity report of the five benchmark configurations against the oracle (needs a B200).

    python tests/parity_report.py

For each configuration the CUDA path runs on seeded inputs of the configuration's shapes and
distributions and is compared with the oracle (the C restatement of the reference's CPU
operators) on the same inputs.  Printed per row: max |gpu - ref|, max |gpu - ref| / |ref| over
elements with |ref| >= 1e-2, and the worst ratio to the acceptance bar
|gpu - ref| <= 1e-3 + 1e-3 |ref| (pass: ratio <= 1); Q8 codes and scales written by the GPU
append are compared byte for byte.  Where the oracle cannot finish a configuration in seconds
the comparison uses a stated sample of it.
"""
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

import vxg_b200  # noqa: E402
from oracle import oracle  # noqa: E402
from vxg_b200 import workloads as wl  # noqa: E402

ATOL, RTOL = 1e-3, 1e-3
CORES = os.cpu_count() or 1


def stats(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    d = np.abs(got - want)
    big = np.abs(want) >= 1e-2
    rel = float((d[big] / np.abs(want[big])).max()) if big.any() else 0.0
    return float(d.max()), rel, float((d / (ATOL + RTOL * np.abs(want))).max())


def row(name, sample, s, q8=None):
    a, r, b = s
    q8s = "—" if q8 is None else ("bit-exact" if q8 else "MISMATCH")
    print(f"| {name} | {sample} | {a:.2e} | {r:.2e} | {b:.3f} | {q8s} |", flush=True)


def config_1_2_3(ctx):
    # config 1: B=1, ctx 2048, attend (no append)
    rng = np.random.default_rng(101)
    L = 2048
    pool = vxg_b200.KvQ8Pool(ctx, 1, wl.HKV, wl.HD, L + 1)
    k = oracle.q8_quantize(rng.standard_normal((L, wl.HKV, wl.HD)).astype(np.float32))
    v = oracle.q8_quantize(rng.standard_normal((L, wl.HKV, wl.HD)).astype(np.float32))
    pool.import_blocks(0, 0, k, v)
    q = rng.standard_normal((1, wl.HQ, wl.HD)).astype(np.float32)
    seq = np.zeros(1, np.int32)
    pos = np.array([L - 1], np.int32)
    got = pool.decode(seq, pos, q)
    kp = np.zeros((1, L + 1) + k.shape[1:], np.uint8)
    vp = np.zeros_like(kp)
    kp[0, :L], vp[0, :L] = k, v
    want = oracle.batch_decode_q8(seq, pos, q, None, None, kp.reshape(-1), vp.reshape(-1), L + 1,
                                  wl.HQ, wl.HKV, wl.HD, do_append=False)
    row("1", "full (B=1, ctx 2048)", stats(got, want))
    pool.close()

    # config 2: 64 ragged sequences, one append + attend step (device-filled caches)
    batch = wl.DecodeBatch(seed=1)
    lens = batch.ctx_lens()
    n = batch.n_seq
    cap = int(lens.max()) + 2
    pool = vxg_b200.KvQ8Pool(ctx, n, wl.HKV, wl.HD, cap)
    wl.fill_pool_device(pool, lens, seed=7)
    kp = np.zeros((n, cap, wl.HKV, wl.HD // 32, 34), np.uint8)
    vp = np.zeros_like(kp)
    for s in range(n):
        kp[s, :lens[s]], vp[s, :lens[s]] = pool.export_blocks(s, 0, int(lens[s]))
    q = rng.standard_normal((n, wl.HQ, wl.HD)).astype(np.float32)
    kn = rng.standard_normal((n, wl.HKV, wl.HD)).astype(np.float32)
    vn = rng.standard_normal((n, wl.HKV, wl.HD)).astype(np.float32)
    seq = np.arange(n, dtype=np.int32)
    pos = lens.astype(np.int32)
    got = pool.decode(seq, pos, q, kn, vn, max_ctx=cap)
    kf, vf = kp.reshape(-1), vp.reshape(-1)
    want = oracle.batch_decode_q8(seq, pos, q, kn, vn, kf, vf, cap, wl.HQ, wl.HKV, wl.HD,
                                  do_append=True, n_threads=CORES)
    same = True
    for s in range(n):
        kg, vg = pool.export_blocks(s, int(lens[s]), 1)
        same &= np.array_equal(kg[0], kp[s, lens[s]]) and np.array_equal(vg[0], vp[s, lens[s]])
    row("2", f"full step (64 seqs, mean ctx {lens.mean():.0f})", stats(got, want), same)
    pool.close()

    # config 3: ctx 262144 with 1% outlier K rows, one append + attend step
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
    kg, vg = pool.export_blocks(0, L, 1)
    same = np.array_equal(kg[0], kp[0, L]) and np.array_equal(vg[0], vp[0, L])
    row("3", "full step (1 GPU, ctx 262144, outlier new K row)", stats(got, want), same)
    pool.close()


def config_4(ctx):
    B, H, D = 64, 32, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    state = torch.randn((B, H, D, D), generator=g, device="cuda") * 0.02
    q, k, v = (torch.randn((B, H, D), generator=g, device="cuda") for _ in range(3))
    br, ar = (torch.randn((B, H), generator=g, device="cuda") for _ in range(2))
    A, dt = -torch.ones(H, device="cuda"), torch.zeros(H, device="cuda")
    st_host = state.cpu().numpy().copy()
    o = vxg_b200.deltanet_step(ctx, q, k, v, br, ar, A, dt, state)
    ctx.sync()
    h = lambda x: x.cpu().numpy()
    want_o = oracle.batch_deltanet(h(q), h(k), h(v), h(br), h(ar), h(A), h(dt), H, H, D, D, 1e-6,
                                   1.0 / np.sqrt(D), st_host, n_threads=CORES)
    row("4", "one step, output o (64 seqs x 32 heads)", stats(h(o), want_o))
    row("4", "one step, state S", stats(h(state), st_host))


def config_5(ctx):
    # 5a: one 8192-token prompt of the config; outputs of 64 evenly spaced tokens against the
    # reference's per-token step over the cache the GPU wrote, and the cache against the oracle
    # quantiser of the same bf16 inputs
    N, H, KV, HD = 8192, 16, 2, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    q = torch.randn((1, N, H, HD), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((1, N, KV, HD), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((1, N, KV, HD), generator=g, device="cuda").to(torch.bfloat16)
    pool = vxg_b200.KvQ8Pool(ctx, 1, KV, HD, N)
    seq = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = pool.prefill(seq, pos, q, k, v, max_ctx=N)
    ctx.sync()
    kb, vb = pool.export_blocks(0, 0, N)
    same = (np.array_equal(kb, oracle.q8_quantize(k[0].float().cpu().numpy()))
            and np.array_equal(vb, oracle.q8_quantize(v[0].float().cpu().numpy())))
    t_idx = ((np.arange(64) + 0.5) * N / 64).astype(np.int64)
    kp, vp = kb.reshape(1, N, KV, HD // 32, 34), vb.reshape(1, N, KV, HD // 32, 34)
    qs = q[0, torch.as_tensor(t_idx, device="cuda")].float().cpu().numpy()
    want = oracle.batch_decode_q8(np.zeros(64, np.int32), t_idx.astype(np.int32), qs, None, None,
                                  kp.reshape(-1), vp.reshape(-1), N, H, KV, HD, do_append=False,
                                  n_threads=CORES)
    got = out[0, torch.as_tensor(t_idx, device="cuda")].cpu().numpy()
    row("5a", "1 of 8 prompts (8192 tokens), 64 evenly spaced tokens", stats(got, want), same)
    pool.close()

    # 5b: one 8192-token prompt, 32 heads, all outputs and the final state against the
    # token-by-token recurrence
    T, H, D = 8192, 32, 128
    g.manual_seed(11)
    q, k, v = (torch.randn((1, T, H, D), generator=g, device="cuda") for _ in range(3))
    br, ar = (torch.randn((1, T, H), generator=g, device="cuda") for _ in range(2))
    A, dt = -torch.ones(H, device="cuda"), torch.zeros(H, device="cuda")
    state = torch.randn((1, H, D, D), generator=g, device="cuda") * 0.02
    st = state.cpu().numpy().copy()
    o = vxg_b200.deltanet_prefill(ctx, q, k, v, br, ar, A, dt, state)
    ctx.sync()
    hq, hk, hv, hb, ha = (x.cpu().numpy() for x in (q, k, v, br, ar))
    An, dtn = A.cpu().numpy(), dt.cpu().numpy()
    want = np.zeros((T, H, D), np.float32)
    # heads are independent: run them on separate threads as B = H one-head "sequences"
    sth = np.ascontiguousarray(st[0].reshape(H, 1, D, D))  # one-head batch entries
    for t in range(T):
        want[t] = oracle.batch_deltanet(hq[0, t].reshape(H, 1, D), hk[0, t].reshape(H, 1, D),
                                        hv[0, t].reshape(H, 1, D), hb[0, t].reshape(H, 1),
                                        ha[0, t].reshape(H, 1), An, dtn, 1, 1, D, D, 1e-6,
                                        1.0 / np.sqrt(D), sth, n_threads=CORES).reshape(H, D)
    row("5b", "1 of 8 prompts (8192 tokens x 32 heads), all outputs", stats(o[0].cpu().numpy(), want))
    row("5b", "same prompt, final state", stats(state[0].cpu().numpy(), sth.reshape(H, D, D)))


def main():
    ctx = vxg_b200.Context()
    print(f"device {ctx.device_name}, oracle threads {CORES}")
    print("| config | sample | max abs err | max rel err (|ref| >= 1e-2) | worst / bar | Q8 |")
    print("|---|---|---:|---:|---:|---|")
    t0 = time.time()
    config_1_2_3(ctx)
    config_4(ctx)
    config_5(ctx)
    print(f"({time.time() - t0:.0f} s)")
    ctx.close()


if __name__ == "__main__":
    main()
