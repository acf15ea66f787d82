"""Seeded synthetic workloads with the shapes and value distributions of the five benchmark
configurations (N(0,1) queries / keys / values quantised by the reference quantiser, ragged
context lengths, outlier key rows, DeltaNet state N(0, 0.02^2)).  No dataset is involved: these
stand in for the reference's model activations.

Device-side generation uses torch's CUDA generator (plumbing only); caches are filled through
the library's own bit-exact quantise-and-append kernel.
"""
from __future__ import annotations

import dataclasses

import numpy as np

HQ, HKV, HD = 16, 2, 256          # Qwen3.5-style full-attention layer shape of all configs
TOKEN_BYTES = 2 * HKV * (HD // 32) * 34   # K + V bytes of one token in the Q8 cache (1088)


@dataclasses.dataclass
class DecodeBatch:
    """Config 2: 64 sequences, ragged contexts U[1024, 32768], append + attend per step."""
    n_seq: int = 64
    ctx_lo: int = 1024
    ctx_hi: int = 32768
    seed: int = 0

    def ctx_lens(self) -> np.ndarray:
        rng = np.random.default_rng(self.seed)
        return rng.integers(self.ctx_lo, self.ctx_hi + 1, self.n_seq).astype(np.int32)

    def kv_bytes_per_step(self, step: int) -> int:
        """Algorithmic bytes of one step: KV read over ctx+1 tokens (after the append)."""
        return int(((self.ctx_lens().astype(np.int64) + step + 1) * TOKEN_BYTES).sum())


def fill_pool_device(pool, ctx_lens, seed: int, outlier_frac: float = 0.0, chunk: int = 8192,
                     offset: int = 0):
    """Fill sequence s of ``pool`` with ctx_lens[s] tokens of N(0,1) K/V (device RNG), quantised
    by the library's append kernel, at positions [offset, offset + ctx_lens[s]).  With
    outlier_frac, that fraction of (token, kv head) K rows is scaled x8 before quantisation.
    The tokens depend only on the seed and the lengths, not on the offset, so one rank's slice
    of a split sequence can be rebuilt inside a whole-sequence pool."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    for s, L in enumerate(ctx_lens):
        L = int(L)
        for t0 in range(0, L, chunk):
            n = min(chunk, L - t0)
            k = torch.randn((1, n, pool.n_head_kv, pool.head_dim), generator=g, device="cuda")
            v = torch.randn((1, n, pool.n_head_kv, pool.head_dim), generator=g, device="cuda")
            if outlier_frac:
                m = torch.rand((1, n, pool.n_head_kv, 1), generator=g, device="cuda") < outlier_frac
                k = torch.where(m, k * 8.0, k)
            seq = torch.tensor([s], dtype=torch.int32, device="cuda")
            pos = torch.tensor([t0 + offset], dtype=torch.int32, device="cuda")
            pool.append(seq, pos, k.contiguous(), v.contiguous(), n_tok=n)
    pool.ctx.sync()


def decode_step_inputs_device(n_seq: int, steps: int, seed: int):
    """Per-step q [n_seq,16,256], k_new / v_new [n_seq,2,256] (N(0,1)), resident on the device."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn((steps, n_seq, HQ, HD), generator=g, device="cuda")
    k = torch.randn((steps, n_seq, HKV, HD), generator=g, device="cuda")
    v = torch.randn((steps, n_seq, HKV, HD), generator=g, device="cuda")
    return q, k, v


def decode_step_inputs_host(n_seq: int, steps: int, seed: int):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((steps, n_seq, HQ, HD), dtype=np.float32)
    k = rng.standard_normal((steps, n_seq, HKV, HD), dtype=np.float32)
    v = rng.standard_normal((steps, n_seq, HKV, HD), dtype=np.float32)
    return q, k, v
