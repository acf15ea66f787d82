"""Host-side multi-rank logic on CPU with the gloo backend (world size 2): sequence sharding,
KV-range ownership, and the all-gather + log-sum-exp merge of split-KV partials.  The merge is
checked against a single softmax over the whole range (numpy float64)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vxg_b200 import dist as vdist


def test_shard_sequences_cover_exactly():
    for n, w in [(64, 1), (64, 8), (10, 3), (3, 4)]:
        ids = [i for r in range(w) for i in vdist.shard_sequences(n, w, r)]
        assert ids == list(range(n))


def test_kv_range_ownership():
    r = [vdist.KvRange(262144 + 9, 4, k) for k in range(4)]
    assert sum(x.local_len(262144) for x in r) == 262144
    for pos in [0, 65538, 65539, 262144]:
        o = r[0].owner(pos)
        assert r[o].begin <= pos < r[o].begin + r[o].span
        assert r[0].local_pos(pos) == pos - r[o].begin


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, scores, values, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # this rank's token range and its partial (log2 domain, like the device kernels)
        n = scores.shape[1]
        kr = vdist.KvRange(n, world, rank)
        lo, hi = kr.begin, kr.begin + kr.local_len(n)
        s2 = scores[:, lo:hi] * np.log2(np.e)
        if hi > lo:
            m = s2.max(axis=1)
            p = np.exp2(s2 - m[:, None])
            l = p.sum(axis=1)
            o = np.einsum("rt,rtd->rd", p, values[:, lo:hi])
        else:
            m = np.full(scores.shape[0], -np.inf)
            l = np.zeros(scores.shape[0])
            o = np.zeros((scores.shape[0], values.shape[2]))
        t = lambda x: torch.tensor(x, dtype=torch.float64)
        M, L, O = vdist.all_gather_partials(t(m), t(l), t(o))
        # log-sum-exp merge, as the device combine does it
        Mx = M.max(dim=0).values
        f = torch.where(torch.isinf(M), torch.zeros_like(M), torch.exp2(M - Mx))
        out = (O * f[..., None]).sum(0) / (L * f).sum(0)[:, None]
        out_q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_tok", [1000, 3])   # 3 tokens over 2 ranks: one rank nearly empty
def test_all_gather_partials_merge_matches_full_softmax(n_tok):
    rng = np.random.default_rng(3)
    rows, hd, world = 16, 8, 2
    scores = rng.standard_normal((rows, n_tok)) * 3
    values = rng.standard_normal((rows, n_tok, hd))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scores, values, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    p_full = np.exp(scores - scores.max(1, keepdims=True))
    want = np.einsum("rt,rtd->rd", p_full, values) / p_full.sum(1)[:, None]
    for r in range(world):
        np.testing.assert_allclose(res[r], want, rtol=1e-10, atol=1e-12)
