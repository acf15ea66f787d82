"""Failure detection on the GPU without a GPU fault: a bounded device-side wait that runs out.

A two-rank peer-exchange step is issued on one GPU with both exchange buffers local and rank 1
never pushing, so rank 0's combine kernel waits for a flag that nothing sets.  The wait gives up
after its 2 s limit, the kernel returns, and the host reads the timeout from the status word:
the call fails with VXG_ATTN_ERR_INTERNAL, the library context refuses further work, and the
device stays usable (a new context decodes normally).  Only one kernel waits and nothing waits
on it, so no kernels wait on one another."""
import ctypes
import time

import numpy as np
import pytest

import vxg_b200
from vxg_b200._lib import ErrBuf, lib
from oracle import oracle

pytestmark = pytest.mark.gpu


def test_peer_wait_runs_out_and_is_reported():
    import torch
    ctx = vxg_b200.Context()
    L = lib()
    err = ErrBuf()
    rows, hd, world = 16, 256, 2
    handles = [(ctypes.c_uint8 * 64)() for _ in range(world)]
    bufs = [L.vxg_attn_cuda_peer_alloc(ctx.h, world, rows, hd, handles[r], err.buf, err.cap)
            for r in range(world)]
    assert all(bufs), err.text
    table = (ctypes.c_void_p * world)(*bufs)
    send = torch.zeros(rows * (hd + 2), device="cuda")
    out = torch.empty((rows, hd), device="cuda")
    t0 = time.time()
    rc = L.vxg_attn_cuda_peer_step(ctx.h, table, world, 0, rows, hd,
                                   ctypes.c_void_p(send.data_ptr()), None,
                                   ctypes.c_void_p(out.data_ptr()), None, err.buf, err.cap)
    waited = time.time() - t0
    assert rc == -7 and "bounded wait" in err.text, (rc, err.text)
    assert 1.5 < waited < 30, waited
    assert torch.count_nonzero(out).item() == 0  # the rows of a failed step are zeroed
    # the library context is poisoned: every later call fails fast
    rc2 = L.vxg_attn_cuda_peer_step(ctx.h, table, world, 0, rows, hd,
                                    ctypes.c_void_p(send.data_ptr()), None,
                                    ctypes.c_void_p(out.data_ptr()), None, err.buf, err.cap)
    assert rc2 == -7 and "poisoned" in err.text
    for b in bufs:
        L.vxg_attn_cuda_peer_free(ctx.h, b)
    ctx.close()
    # the device itself is fine: a fresh context runs a decode step against the oracle
    ctx2 = vxg_b200.Context()
    rng = np.random.default_rng(3)
    pool = vxg_b200.KvQ8Pool(ctx2, 1, 2, 256, 64)
    k = oracle.q8_quantize(rng.standard_normal((40, 2, 256)).astype(np.float32))
    v = oracle.q8_quantize(rng.standard_normal((40, 2, 256)).astype(np.float32))
    pool.import_blocks(0, 0, k, v)
    q = rng.standard_normal((1, 16, 256)).astype(np.float32)
    got = pool.decode(np.zeros(1, np.int32), np.array([39], np.int32), q)
    kp = np.zeros((1, 64, 2, 8, 34), np.uint8)
    vp = np.zeros_like(kp)
    kp[0, :40], vp[0, :40] = k, v
    want = oracle.batch_decode_q8(np.zeros(1, np.int32), np.array([39], np.int32), q, None, None,
                                  kp.reshape(-1), vp.reshape(-1), 64, 16, 2, 256, do_append=False)
    np.testing.assert_allclose(got, want, atol=1e-3, rtol=1e-3)
    pool.close()
    ctx2.close()
