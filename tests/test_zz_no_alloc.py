"""GPU test of vxg_attn_cuda_q8_decode_noalloc, the decode entry point that allocates nothing.

It exists for callers that cannot call cudaMalloc: engines whose device memory belongs to a
budgeted pool or to another framework's caching allocator, and decode loops that must not stall
on the allocator.  Such a caller owns every buffer (here torch allocates them, standing in for
the caller's allocator); the entry point keeps its split-KV scratch in a fixed built-in device
array.  The test calls it through the C ABI twice in a row with different inputs, so the second
call runs on the scratch the first one left behind, and compares each result with the
allocating entry point vxg_attn_cuda_q8_decode at the tolerance of the other decode tests.
This file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

import vxg_b200
from vxg_b200 import _lib
from oracle import oracle

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3


def _noalloc(pool, seq, pos, q, out, n_head, gate=None):
    """Call the no-alloc entry point on torch device tensors (NULL stream: synchronous)."""
    k_ptr, v_ptr, _ = pool.device_ptrs()
    err = _lib.ErrBuf()
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    return _lib.lib().vxg_attn_cuda_q8_decode_noalloc(
        ctypes.c_void_p(k_ptr), ctypes.c_void_p(v_ptr), pool.n_seq, pool.capacity,
        pool.n_head_kv, pool.head_dim, seq.numel(), n_head, p(seq), p(pos), p(q), None, None,
        p(gate), ctypes.c_float(1.0 / np.sqrt(pool.head_dim)), p(out), None, err.buf,
        err.cap), err.text


@pytest.mark.parametrize("n_head,n_kv,hd", [(16, 2, 256), (4, 2, 64)])
def test_noalloc_matches_allocating_entry_point(n_head, n_kv, hd):
    import torch
    torch.cuda.set_device(0)
    rng = np.random.default_rng(70)
    lens = [1, 65, 700, 2049, 5000, 64, 130]
    cap = max(lens) + 1
    ctx = vxg_b200.Context()
    pool = vxg_b200.KvQ8Pool(ctx, len(lens), n_kv, hd, cap)
    for s, L in enumerate(lens):
        kb = oracle.q8_quantize(rng.standard_normal((L, n_kv, hd)).astype(np.float32))
        vb = oracle.q8_quantize(rng.standard_normal((L, n_kv, hd)).astype(np.float32))
        pool.import_blocks(s, 0, kb, vb)
    for call, subset in enumerate([[0, 1, 2, 3, 4, 5, 6], [4, 2, 6]]):
        seq = np.array(subset, np.int32)
        pos = np.array([lens[s] - 1 for s in subset], np.int32)
        q = rng.standard_normal((len(subset), n_head, hd)).astype(np.float32)
        gate = rng.standard_normal((len(subset), n_head, hd)).astype(np.float32) if call else None
        want = pool.decode(seq, pos, q, q_gate=gate)          # allocating entry point
        dq = torch.from_numpy(q).cuda()
        dg = torch.from_numpy(gate).cuda() if gate is not None else None
        out = torch.full((len(subset), n_head, hd), float("nan"), device="cuda")
        rc, msg = _noalloc(pool, torch.from_numpy(seq).cuda(), torch.from_numpy(pos).cuda(), dq,
                           out, n_head, dg)
        assert rc == 0, msg
        np.testing.assert_allclose(out.cpu().numpy(), want, atol=ATOL, rtol=RTOL)
    pool.close()
    ctx.close()


SCRATCH_BYTES = 32 << 20      # the built-in array, less the 256-byte status word below
STATUS_BYTES = 256


def _scratch_bytes_16_2_256(n, sm_count):
    """Split-KV scratch of one call at 16 q / 2 kv heads, head_dim 256 (the fast kernel): six
    (m, l, o) slots per (CTA, entry) boundary, a second level of slots when the combine splits
    a small batch, and the unit prefix plus CTA ranges."""
    grid = min(sm_count, 512)
    floats = (grid + n) * 6 * 16 * 258
    per = n * (8 if n < 32 else 4)  # combine CTAs per split level (32- or 64-dim chunks)
    splits = max(1, min(32, -(-128 // per)))
    if splits > 1:
        floats += n * splits * 16 * 258
    return 4 * (1056 + floats + n + grid + 64)  # + the split pass's state (rates per CTA)


def _largest_batch(sm_count):
    n = 1
    while _scratch_bytes_16_2_256(n + 1, sm_count) + STATUS_BYTES <= SCRATCH_BYTES:
        n += 1
    return n


def test_noalloc_batch_limit_boundary():
    """The largest batch that fits the array runs and matches the allocating entry point; one
    entry more is rejected before anything is launched."""
    import torch
    torch.cuda.set_device(0)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    n = _largest_batch(sms)
    assert n >= 64, f"a 64-sequence batch should fit on {sms} SMs"
    rng = np.random.default_rng(71)
    n_seq, L = 8, 300
    ctx = vxg_b200.Context()
    pool = vxg_b200.KvQ8Pool(ctx, n_seq, 2, 256, L)
    for s in range(n_seq):
        kb = oracle.q8_quantize(rng.standard_normal((L, 2, 256)).astype(np.float32))
        vb = oracle.q8_quantize(rng.standard_normal((L, 2, 256)).astype(np.float32))
        pool.import_blocks(s, 0, kb, vb)
    seq = (np.arange(n) % n_seq).astype(np.int32)
    pos = rng.integers(0, L, n).astype(np.int32)
    q = rng.standard_normal((n, 16, 256)).astype(np.float32)
    want = pool.decode(seq, pos, q)
    out = torch.full((n, 16, 256), float("nan"), device="cuda")
    rc, msg = _noalloc(pool, torch.from_numpy(seq).cuda(), torch.from_numpy(pos).cuda(),
                       torch.from_numpy(q).cuda(), out, 16)
    assert rc == 0, msg
    np.testing.assert_allclose(out.cpu().numpy(), want, atol=ATOL, rtol=RTOL)
    m = n + 1
    seq1 = torch.zeros(m, dtype=torch.int32, device="cuda")
    out1 = torch.zeros((m, 16, 256), device="cuda")
    rc, msg = _noalloc(pool, seq1, seq1.clone(), torch.zeros((m, 16, 256), device="cuda"), out1,
                       16)
    assert rc == _lib.ERR_BUFFER_TOO_SMALL and "scratch" in msg
    assert not out1.any()                       # rejected before any launch
    pool.close()
    ctx.close()


def test_noalloc_rejects_batches_beyond_its_scratch():
    import torch
    torch.cuda.set_device(0)
    ctx = vxg_b200.Context()
    pool = vxg_b200.KvQ8Pool(ctx, 1, 2, 256, 16)
    n = 400                                     # well past the limit at this shape
    seq = torch.zeros(n, dtype=torch.int32, device="cuda")
    pos = torch.zeros(n, dtype=torch.int32, device="cuda")
    q = torch.zeros((n, 16, 256), device="cuda")
    out = torch.zeros((n, 16, 256), device="cuda")
    rc, msg = _noalloc(pool, seq, pos, q, out, 16)
    assert rc == _lib.ERR_BUFFER_TOO_SMALL and "scratch" in msg
    pool.close()
    ctx.close()
