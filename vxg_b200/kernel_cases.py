"""Small cases that run each kernel of the library through the public API (one GPU).

Each case is a few calls on seeded synthetic inputs, sized so that its main kernel reads or
writes more than the 126 MB L2 where the kernel is memory-bound, and finishes in about a
second.  The cases are the workloads of the per-kernel ncu summaries (a summary names its
command, e.g. ``ncu ... -k regex:^deltanet_conv_kernel python -m vxg_b200.kernel_cases
dnet_recurrent``) and a quick way to exercise every launch path:

    python -m vxg_b200.kernel_cases [case ...]        (no case: all of them)

case              kernels
append_bf16       q8_append_kernel<bf16> (8 prompts x 8192 tokens, via the causal prefill)
decode_small      q8_append_kernel<float>, decode_fast_split, decode_fast_combine(_final)
decode_generic    decode_generic_split, decode_combine (16 q / 4 kv heads, head_dim 128)
f32kv             f32_append_kernel, decode_generic_split over fp32 K/V, decode_combine
lse               lse_combine_kernel (packed partials of 8 parts)
peer              peer_push_kernel, peer_combine_kernel (a one-rank exchange)
gqa_step          gqa_prep_kernel (the step_full_gqa_q8 drop-in)
dnet_recurrent    deltanet_conv_kernel, deltanet_step_persistent with the fused epilogue
dnet_step_d256    deltanet_step_kernel (dk = dv = 256, outside the persistent kernel's shapes)
dnet_prefill      deltanet_prep_vec_kernel, deltanet_chunk_kernel (2 prompts x 4096 tokens)
dnet_prefill_seq  deltanet_prep_vec_kernel, deltanet_prefill_kernel (dk 64: the sequential kernel)
prefill_f32       q8_dequant_f16_kernel, prefill_attn_kernel (f32 q/k/v)
"""
from __future__ import annotations

import ctypes
import sys

import numpy as np


def _t():
    import torch
    torch.cuda.set_device(0)
    return torch


def append_bf16(ctx):
    torch = _t()
    import vxg_b200
    B, N, H, KV, HD = 8, 8192, 16, 2, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    q = torch.randn((B, N, H, HD), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((B, N, KV, HD), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((B, N, KV, HD), generator=g, device="cuda").to(torch.bfloat16)
    pool = vxg_b200.KvQ8Pool(ctx, B, KV, HD, N)
    seq = torch.arange(B, dtype=torch.int32, device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    pool.prefill(seq, pos, q, k, v, max_ctx=N)
    pool.close()


def decode_small(ctx):
    torch = _t()
    import vxg_b200
    from vxg_b200 import workloads as wl
    n = 8                                   # < 32 entries: the combine splits its slots
    lens = np.random.default_rng(2).integers(1024, 16384, n).astype(np.int32)
    cap = int(lens.max()) + 8
    pool = vxg_b200.KvQ8Pool(ctx, n, wl.HKV, wl.HD, cap)
    wl.fill_pool_device(pool, lens, seed=3)
    q, kn, vn = wl.decode_step_inputs_device(n, 3, seed=4)
    seq = torch.arange(n, dtype=torch.int32, device="cuda")
    for i in range(3):
        pos = torch.from_numpy(lens + i).cuda()
        pool.decode(seq, pos, q[i], kn[i], vn[i], max_ctx=cap)
    pool.close()


def decode_generic(ctx):
    torch = _t()
    import vxg_b200
    n, H, KV, HD, L = 64, 16, 4, 128, 4096
    pool = vxg_b200.KvQ8Pool(ctx, n, KV, HD, L + 4)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    for t0 in range(0, L, 1024):
        k = torch.randn((n, 1024, KV, HD), generator=g, device="cuda")
        pool.append(torch.arange(n, dtype=torch.int32, device="cuda"),
                    torch.full((n,), t0, dtype=torch.int32, device="cuda"), k, k, n_tok=1024)
    q = torch.randn((n, H, HD), generator=g, device="cuda")
    pos = torch.full((n,), L - 1, dtype=torch.int32, device="cuda")
    for _ in range(3):
        pool.decode(torch.arange(n, dtype=torch.int32, device="cuda"), pos, q, max_ctx=L + 4)
    pool.close()


def f32kv(ctx):
    torch = _t()
    import vxg_b200
    n, H, KV, HD, L = 16, 16, 2, 256, 4096
    pool = vxg_b200.KvF32Pool(ctx, n, KV, HD, L + 4)
    g = torch.Generator(device="cuda")
    g.manual_seed(6)
    seq = torch.arange(n, dtype=torch.int32, device="cuda")
    k = torch.randn((n, L, KV, HD), generator=g, device="cuda")
    pool.append(seq, torch.zeros(n, dtype=torch.int32, device="cuda"), k, k, n_tok=L)
    q = torch.randn((n, H, HD), generator=g, device="cuda")
    pos = torch.full((n,), L - 1, dtype=torch.int32, device="cuda")
    for _ in range(3):
        pool.decode(seq, pos, q, max_ctx=L + 4)
    pool.close()


def lse(ctx):
    torch = _t()
    import vxg_b200
    parts, rows, hd = 8, 16 * 64, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    packed = torch.randn((parts, rows * (hd + 2)), generator=g, device="cuda")
    for _ in range(3):
        vxg_b200.lse_combine_packed(ctx, packed, parts, rows, hd)


def peer(ctx):
    torch = _t()
    from vxg_b200._lib import ErrBuf, lib
    rows, hd = 16, 256
    err = ErrBuf()
    handle = (ctypes.c_uint8 * 64)()
    own = lib().vxg_attn_cuda_peer_alloc(ctx.h, 1, rows, hd, handle, err.buf, err.cap)
    assert own, err.text
    bufs = (ctypes.c_void_p * 1)(own)
    send = torch.randn(rows * (hd + 2), device="cuda")
    send[:rows] = 0.0
    out = torch.empty((rows, hd), device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        rc = lib().vxg_attn_cuda_peer_step(ctx.h, bufs, 1, 0, rows, hd,
                                           ctypes.c_void_p(send.data_ptr()), None,
                                           ctypes.c_void_p(out.data_ptr()), stream, err.buf,
                                           err.cap)
        assert rc == 0, err.text
    torch.cuda.synchronize()
    lib().vxg_attn_cuda_peer_free(ctx.h, own)


def gqa_step(ctx):
    import vxg_b200
    rng = np.random.default_rng(8)
    H, KV, HD, cap = 16, 2, 256, 64
    pool = vxg_b200.KvQ8Pool(ctx, 1, KV, HD, cap)
    qn = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
    out = np.zeros(H * HD, np.float32)
    for pos in range(4):
        q_raw = rng.standard_normal(2 * H * HD).astype(np.float32)
        k_cur = rng.standard_normal(KV * HD).astype(np.float32)
        v_cur = rng.standard_normal(KV * HD).astype(np.float32)
        vxg_b200.step_full_gqa_q8(ctx, pool, 0, q_raw, k_cur, v_cur, qn, kn, True, H, KV, HD,
                                  pos, pos, 64, 1e7, True, 1e-6, out)
    pool.close()


def dnet_recurrent(ctx):
    torch = _t()
    import vxg_b200
    B, n_kh, n_vh, dk, dv, k_sz = 64, 16, 32, 128, 128, 4
    conv_ch = 2 * n_kh * dk + n_vh * dv
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    qkv = torch.randn((B, conv_ch), generator=g, device="cuda")
    z = torch.randn((B, n_vh * dv), generator=g, device="cuda")
    ar = torch.randn((B, n_vh), generator=g, device="cuda")
    br = torch.randn((B, n_vh), generator=g, device="cuda")
    w = torch.randn((conv_ch, k_sz), generator=g, device="cuda") * 0.3
    A = -torch.ones(n_vh, device="cuda")
    dt = torch.zeros(n_vh, device="cuda")
    norm = torch.ones(dv, device="cuda")
    conv_state = torch.zeros((B, k_sz - 1, conv_ch), device="cuda")
    state = torch.randn((B, n_vh, dv, dk), generator=g, device="cuda") * 0.02
    for _ in range(3):
        vxg_b200.step_deltanet_recurrent(ctx, qkv, z, ar, br, w, A, dt, norm, conv_state, state,
                                         n_kh, n_vh, dk, dv, k_sz, 1e-6)


def dnet_step_d256(ctx):
    torch = _t()
    import vxg_b200
    B, H, D = 32, 16, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(10)
    state = torch.randn((B, H, D, D), generator=g, device="cuda") * 0.02
    q, k, v = (torch.randn((B, H, D), generator=g, device="cuda") for _ in range(3))
    br, ar = (torch.randn((B, H), generator=g, device="cuda") for _ in range(2))
    A, dt = -torch.ones(H, device="cuda"), torch.zeros(H, device="cuda")
    for _ in range(3):
        vxg_b200.deltanet_step(ctx, q, k, v, br, ar, A, dt, state)


def dnet_prefill(ctx):
    torch = _t()
    import vxg_b200
    B, T, H, D = 2, 4096, 32, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    q, k, v = (torch.randn((B, T, H, D), generator=g, device="cuda") for _ in range(3))
    br, ar = (torch.randn((B, T, H), generator=g, device="cuda") for _ in range(2))
    A, dt = -torch.ones(H, device="cuda"), torch.zeros(H, device="cuda")
    state = torch.randn((B, H, D, D), generator=g, device="cuda") * 0.02
    vxg_b200.deltanet_prefill(ctx, q, k, v, br, ar, A, dt, state)


def dnet_prefill_seq(ctx):
    torch = _t()
    import vxg_b200
    B, T, H, D = 8, 1024, 16, 64
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    q, k, v = (torch.randn((B, T, H, D), generator=g, device="cuda") for _ in range(3))
    br, ar = (torch.randn((B, T, H), generator=g, device="cuda") for _ in range(2))
    A, dt = -torch.ones(H, device="cuda"), torch.zeros(H, device="cuda")
    state = torch.randn((B, H, D, D), generator=g, device="cuda") * 0.02
    vxg_b200.deltanet_prefill(ctx, q, k, v, br, ar, A, dt, state)


def prefill_f32(ctx):
    torch = _t()
    import vxg_b200
    B, N, H, KV, HD = 2, 4096, 16, 2, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(13)
    q = torch.randn((B, N, H, HD), generator=g, device="cuda")
    k = torch.randn((B, N, KV, HD), generator=g, device="cuda")
    v = torch.randn((B, N, KV, HD), generator=g, device="cuda")
    pool = vxg_b200.KvQ8Pool(ctx, B, KV, HD, N)
    seq = torch.arange(B, dtype=torch.int32, device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    pool.prefill(seq, pos, q, k, v, max_ctx=N)
    pool.close()


CASES = {f.__name__: f for f in (append_bf16, decode_small, decode_generic, f32kv, lse, peer,
                                 gqa_step, dnet_recurrent, dnet_step_d256, dnet_prefill,
                                 dnet_prefill_seq, prefill_f32)}


def main(argv):
    import vxg_b200
    names = argv or list(CASES)
    unknown = [n for n in names if n not in CASES]
    if unknown:
        raise SystemExit(f"unknown case(s) {unknown}; cases: {', '.join(CASES)}")
    _t()
    ctx = vxg_b200.Context()
    for name in names:
        CASES[name](ctx)
        rc = ctx.sync()
        if rc < 0:
            raise SystemExit(f"{name}: device status {rc}")
        print(f"{name}: ok", flush=True)
    ctx.close()


if __name__ == "__main__":
    main(sys.argv[1:])
