#!/usr/bin/env python
"""Benchmark of the B200 Q8-KV decode attention hot path (one JSON line on rank 0).

Default workload: per GPU, 64 sequences with context lengths U[1024, 32768]
(seeded), 16 query / 2 KV heads, head_dim 256, Q8_0 KV.  One step = quantise-and-append one new
N(0,1) K/V token per sequence, then split-KV attention of each sequence's query over its whole
cache.  Inputs are synthetic (device RNG; see vxg_b200/workloads.py).  Multi-GPU: one process
per GPU, each with its own 64 sequences of the same context lengths (weak scaling, no data-path
collective); time = max over ranks of the device-timed region.  After the config-2 line is
measured, the same run times config 3 (one 262144-token context: split-KV over the SMs on one
GPU, KV-range split with an exchange of the (m, l, o) partials on N GPUs) and reports it under
"long_context" (--no-long skips it).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|long|deltanet|prefill|dnet_prefill]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q8-KV decode attn: HBM GB/s (% of peak) and seq-steps/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary (profiles/*.json)."""
    p = os.path.join(ROOT, "profiles", name)
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("traffic_bytes_per_launch")
        except Exception:
            return None
    return None


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# --------------------------------------------------------------------------- clocks (NVML)
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
            0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
            0x100: "display_clock_setting"}


class ClockSampler:
    """Polls SM clock and clock-event reasons of this process's GPU every ~2 ms."""

    def __init__(self, torch_device: int):
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            import torch
            props = torch.cuda.get_device_properties(torch_device)
            h = None
            try:
                bus = "%08X:%02X:%02X.0" % (props.pci_domain_id, props.pci_bus_id,
                                           props.pci_device_id)
                h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[torch_device]) if vis else torch_device
                h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.h = h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # pragma: no cover - no NVML
            self.err = str(e)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        if self.h is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread:
            self._stop.set()
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [s[0] for s in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= int(r)
        reasons = [n for b, n in _REASONS.items() if bits & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz)}


# --------------------------------------------------------------------------- distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def barrier_max(torch, dist, world, value: float) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier_min(torch, dist, world, value: float) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return float(t.item())


def barrier(torch, dist, world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


# --------------------------------------------------------------------------- our arm
def run_decode(args, world, rank, local):
    import torch
    import torch.distributed as dist
    import vxg_b200
    from vxg_b200 import workloads as wl

    K, W = args.steps, args.warmup
    ctx = vxg_b200.Context()
    # every rank decodes the same context lengths (its own K/V data and queries), so the
    # max-over-ranks step time measures the GPUs, not a per-rank workload imbalance
    batch = wl.DecodeBatch(n_seq=args.seqs, ctx_hi=args.ctx_max, seed=1)
    lens = batch.ctx_lens()
    n = batch.n_seq
    E2E_W = 2
    cap = int(lens.max()) + W + K + E2E_W + K + 8
    pool = vxg_b200.KvQ8Pool(ctx, n, wl.HKV, wl.HD, cap)
    wl.fill_pool_device(pool, lens, seed=7 + rank)
    q, kn, vn = wl.decode_step_inputs_device(n, W + K, seed=11 + rank)
    seq = torch.arange(n, dtype=torch.int32, device="cuda")
    pos = [torch.from_numpy(lens + i).to(torch.int32).cuda() for i in range(W + K)]
    out = torch.empty((n, wl.HQ, wl.HD), dtype=torch.float32, device="cuda")
    for i in range(W):
        pool.decode(seq, pos[i], q[i], kn[i], vn[i], out=out, max_ctx=cap)
    ctx.sync()
    sampler = ClockSampler(local)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(torch, dist, world)
    sampler.start()
    e0.record()
    for i in range(W, W + K):
        pool.decode(seq, pos[i], q[i], kn[i], vn[i], out=out, max_ctx=cap)
    e1.record()
    torch.cuda.synchronize()
    sampler.stop()
    rc = ctx.sync()
    ms = e0.elapsed_time(e1)
    # the same steps again with events around each split launch, for the roofline (the events
    # sit between the kernels, so this pass is not the one timed for the step)
    ctx.set_timing(True)
    for i in range(W, W + K):
        pool.decode(seq, pos[i], q[i], kn[i], vn[i], out=out, max_ctx=cap)
    torch.cuda.synchronize()
    split_ms = ctx.split_ms_total() / K
    ctx.set_timing(False)
    rc |= ctx.sync()
    ms_max = barrier_max(torch, dist, world, ms)
    split_ms_max = barrier_max(torch, dist, world, split_ms)
    barrier(torch, dist, world)

    # ---- end to end through the public API with pinned host buffers ---------------------------
    qh = ctx.pinned_empty((E2E_W + K, n, wl.HQ, wl.HD), np.float32)
    kh = ctx.pinned_empty((E2E_W + K, n, wl.HKV, wl.HD), np.float32)
    vh = ctx.pinned_empty((E2E_W + K, n, wl.HKV, wl.HD), np.float32)
    hq, hk, hv = wl.decode_step_inputs_host(n, E2E_W + K, seed=13 + rank)
    qh[...] = hq
    kh[...] = hk
    vh[...] = hv
    # one output buffer per staging slot: step i's result lands in outh[i % 2] and stays valid
    # until step i + 2 is queued
    outh = ctx.pinned_empty((2, n, wl.HQ, wl.HD), np.float32)
    seq_h = ctx.pinned_empty((n,), np.int32)
    seq_h[...] = np.arange(n, dtype=np.int32)
    base = lens + W + K
    pos_h = ctx.pinned_empty((E2E_W + K, n), np.int32)
    for i in range(E2E_W + K):
        pos_h[i] = base + i
    for i in range(E2E_W):
        ctx.wait(pool.decode_host_async(seq_h, pos_h[i], qh[i], kh[i], vh[i], out=outh[i % 2],
                                        max_ctx=cap))
    barrier(torch, dist, world)
    t0 = time.perf_counter()
    tickets = [pool.decode_host_async(seq_h, pos_h[i], qh[i], kh[i], vh[i], out=outh[i % 2],
                                      max_ctx=cap) for i in range(E2E_W, E2E_W + K)]
    e2e_rc = [ctx.wait(t) for t in tickets]
    e2e_s = time.perf_counter() - t0
    e2e_s = barrier_max(torch, dist, world, e2e_s)
    h2d = seq_h.nbytes + pos_h[0].nbytes + qh[0].nbytes + kh[0].nbytes + vh[0].nbytes
    d2h = outh[0].nbytes

    # ---- algorithmic bytes of the split-KV pass ---------------------------------------------
    kv_bytes = np.mean([batch.kv_bytes_per_step(i) for i in range(W, W + K)])
    q_bytes = n * wl.HQ * wl.HD * 4
    alg_bytes = kv_bytes + q_bytes
    peak, peak_kind = measured_peaks()
    # each rank's own bytes over its own split time; the slowest rank's figure is reported
    achieved = barrier_min(torch, dist, world, alg_bytes / (split_ms * 1e-3) / 1e9)
    step_bytes = alg_bytes + n * (wl.HQ * wl.HD * 4 + 2 * wl.HKV * wl.HD * 4 + 1088)

    res = {
        "metric": METRIC,
        "value": n * world * K / (ms_max * 1e-3),
        "unit": "seq-steps/s",
        "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_max / K,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {
            "workload": f"config2: batched decode + Q8 append, {n} seqs per GPU, ctx U[1024,"
                        f"{batch.ctx_hi}], 16 q / 2 kv heads, head_dim 256, Q8_0 KV (34-B blocks)",
            "seqs_per_gpu": n, "mean_ctx": float(lens.mean()), "parallelism": f"seq-shard x{world}",
            "l2": "inputs larger than L2 (%.2f GB of KV read per step)" % (kv_bytes / 1e9),
            "hbm_gbs_whole_step": step_bytes / (ms_max / K * 1e-3) / 1e9,
        },
        "roofline": {
            "kernel": "decode_fast_split",
            "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_kind": peak_kind,
            "split_ms_per_launch": split_ms_max,
            "algorithmic_bytes_per_launch": alg_bytes,
            "traffic": profile_traffic("decode_fast_split_config2.json"),
        },
        "e2e": {"value": n * world * K / e2e_s, "unit": "seq-steps/s",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "api": "KvQ8Pool.decode_host_async / vxg_attn_cuda_q8_decode_host_async: pinned "
                       "host buffers, each step's upload and download overlap the neighbouring "
                       "steps' kernels; host wall clock from the first call to the last wait",
                "status": max(e2e_rc)},
        "gpu_launches": 3 * K,
        "clocks": sampler.summary(),
        "device_status": rc,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_decode(pool, lens, n)
    pool.close()
    del q, kn, vn
    torch.cuda.empty_cache()
    if not args.no_long:
        # config 3 on the same GPUs (one GPU: split-KV over its SMs; N GPUs: KV-range split)
        barrier(torch, dist, world)
        lr = measure_long(args, world, rank, local, ctx, K, W, check=world > 1)
        pool_l = lr.pop("_pool", None)
        lr.pop("_inputs", None)
        if pool_l is not None:
            pool_l.close()
        res["long_context"] = lr
    return res


def cpu_sample_size(n, cores):
    """Sequences per CPU step: one per host thread (at least 4, at most the batch), so every
    thread of the oracle has a sequence; the reference arm uses the same first sequences."""
    return int(min(n, max(4, cores)))


def cpu_baseline_decode(pool, lens, n, budget_s=12.0):
    """The oracle port on this host's cores over a bounded sample: the first
    cpu_sample_size() sequences of the batch (their real caches, exported from the device), one
    append+attend step each, repeated until ~budget_s of wall time."""
    from oracle import oracle
    from vxg_b200 import workloads as wl
    rng = np.random.default_rng(99)
    n_sample = cpu_sample_size(n, host_cores())
    pick = np.arange(n_sample)
    cap = int(lens[pick].max()) + 2
    kpool = np.zeros((n_sample, cap, wl.HKV, wl.HD // 32, 34), np.uint8)
    vpool = np.zeros_like(kpool)
    for j, s in enumerate(pick):
        k, v = pool.export_blocks(int(s), 0, int(lens[s]))
        kpool[j, :lens[s]] = k
        vpool[j, :lens[s]] = v
    cores = host_cores()
    q = rng.standard_normal((n_sample, wl.HQ, wl.HD), dtype=np.float32)
    kn = rng.standard_normal((n_sample, wl.HKV, wl.HD), dtype=np.float32)
    vn = rng.standard_normal((n_sample, wl.HKV, wl.HD), dtype=np.float32)
    seq = np.arange(n_sample, dtype=np.int32)
    pos = lens[pick].astype(np.int32)
    kflat, vflat = kpool.reshape(-1), vpool.reshape(-1)
    reps = 0
    t0 = time.perf_counter()
    while True:
        oracle.batch_decode_q8(seq, pos, q, kn, vn, kflat, vflat, cap, wl.HQ, wl.HKV, wl.HD,
                               do_append=True, n_threads=cores)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    return {"value": n_sample * reps / el, "unit": "seq-steps/s", "cores": cores, "kind": "port",
            "sample": f"the first {n_sample} of the 64 sequences (mean ctx "
                      f"{lens[pick].mean():.0f}), one append+attend step each, {cores} threads, "
                      f"x{reps} repetitions, {el:.1f} s"}


def _timed_reps(fn, budget_s, max_reps=1000):
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= max_reps:
            return reps, el


def cpu_baseline_long(pool, L, q, kn, vn, budget_s=10.0):
    """Config 3 on the oracle port: append + attend of the 262144-token sequence (its real cache,
    exported from the device), one thread as in the reference's per-sequence step."""
    from oracle import oracle
    from vxg_b200 import workloads as wl
    k, v = pool.export_blocks(0, 0, L)
    cap = L + 1
    kp = np.zeros((1, cap, wl.HKV, wl.HD // 32, 34), np.uint8)
    vp = np.zeros_like(kp)
    kp[0, :L], vp[0, :L] = k, v
    kf, vf = kp.reshape(-1), vp.reshape(-1)
    seq, pos = np.zeros(1, np.int32), np.array([L], np.int32)
    qh, kh, vh = (x.reshape(1, -1, wl.HD) for x in (q, kn, vn))
    reps, el = _timed_reps(lambda: oracle.batch_decode_q8(seq, pos, qh, kh, vh, kf, vf, cap,
                                                           wl.HQ, wl.HKV, wl.HD, do_append=True,
                                                           n_threads=1), budget_s)
    return {"value": reps / el, "unit": "seq-steps/s", "cores": 1, "kind": "port",
            "sample": f"the full step (ctx {L}), x{reps} repetitions, {el:.1f} s"}


def cpu_baseline_deltanet(q, k, v, br, ar, A, dt, state, budget_s=10.0):
    """Config 4 on the oracle port: the batched core step over all 64 sequences x 32 heads (the
    bench's own state and inputs), sequences spread over the host's cores."""
    from oracle import oracle
    B, H, D, _ = state.shape
    cores = host_cores()
    st = np.ascontiguousarray(state, dtype=np.float32)
    reps, el = _timed_reps(lambda: oracle.batch_deltanet(q, k, v, br, ar, A, dt, H, H, D, D, 1e-6,
                                                         1.0 / np.sqrt(D), st, n_threads=cores),
                           budget_s)
    return {"value": B * reps / el, "unit": "seq-steps/s", "cores": cores, "kind": "port",
            "sample": f"all {B} sequences x {H} heads per step, x{reps} steps, {el:.1f} s"}


def cpu_baseline_prefill(pool, q, B, N, H, KV, HD, budget_s=12.0, per_prompt=16):
    """Config 5a on the oracle port: the reference runs prompt token t as one decode step over
    the cache [0, t] (llm_prefill.rs:497-517).  Sample: per prompt, `per_prompt` tokens at
    evenly spaced positions (their mean cost is the prompt's mean cost), attending over the real
    Q8 cache the GPU prefill wrote; all host cores over the sampled tokens."""
    from oracle import oracle
    cores = host_cores()
    kp = np.zeros((B, N, KV, HD // 32, 34), np.uint8)
    vp = np.zeros_like(kp)
    for b in range(B):
        kp[b], vp[b] = pool.export_blocks(b, 0, N)
    kf, vf = kp.reshape(-1), vp.reshape(-1)
    t_idx = ((np.arange(per_prompt) + 0.5) * N / per_prompt).astype(np.int64)
    seq = np.repeat(np.arange(B, dtype=np.int32), per_prompt)
    pos = np.tile(t_idx, B).astype(np.int32)
    import torch
    qs = q[:, torch.as_tensor(t_idx, device=q.device)].float().cpu().numpy()
    qs = qs.reshape(B * per_prompt, H, HD)
    reps, el = _timed_reps(lambda: oracle.batch_decode_q8(seq, pos, qs, None, None, kf, vf, N, H,
                                                           KV, HD, do_append=False,
                                                           n_threads=cores), budget_s)
    n = B * per_prompt
    return {"value": n * reps / el, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{per_prompt} evenly spaced tokens of each of {B} prompts, attend over "
                      f"their prefix, x{reps} repetitions, {el:.1f} s"}


def cpu_baseline_dnet_prefill(q, k, v, br, ar, A, dt, state0, budget_s=10.0, n_tok=64):
    """Config 5b on the oracle port: the reference's token-by-token recurrence
    (llm_prefill.rs:470-480) over the first `n_tok` tokens of every prompt, all heads, prompts
    spread over the host's cores."""
    from oracle import oracle
    B, H, D, _ = state0.shape
    cores = host_cores()
    qh, kh, vh = (x[:, :n_tok].cpu().numpy() for x in (q, k, v))
    bh, ah = br[:, :n_tok].cpu().numpy(), ar[:, :n_tok].cpu().numpy()
    An, dtn = A.cpu().numpy(), dt.cpu().numpy()

    def run():
        st = state0.cpu().numpy().copy()
        for t in range(n_tok):
            oracle.batch_deltanet(qh[:, t], kh[:, t], vh[:, t], bh[:, t], ah[:, t], An, dtn, H, H,
                                  D, D, 1e-6, 1.0 / np.sqrt(D), st, n_threads=cores)

    reps, el = _timed_reps(run, budget_s)
    return {"value": B * n_tok * reps / el, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"the first {n_tok} tokens of each of {B} prompts, all {H} heads, "
                      f"x{reps} repetitions, {el:.1f} s"}


def run_deltanet(args, world, rank, local):
    """64 seqs x 32 heads, dk = dv = 128, state R+W per step."""
    import torch
    import torch.distributed as dist
    import vxg_b200
    K, W = args.steps, args.warmup
    ctx = vxg_b200.Context()
    B, H, D = 64, 32, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(5 + rank)
    state = torch.randn((B, H, D, D), generator=g, device="cuda") * 0.02
    T = W + K
    q = torch.randn((T, B, H, D), generator=g, device="cuda")
    k = torch.randn((T, B, H, D), generator=g, device="cuda")
    v = torch.randn((T, B, H, D), generator=g, device="cuda")
    br = torch.randn((T, B, H), generator=g, device="cuda")
    ar = torch.randn((T, B, H), generator=g, device="cuda")
    A = -torch.ones(H, device="cuda")
    dt = torch.zeros(H, device="cuda")
    o = torch.empty((B, H, D), device="cuda")
    for i in range(W):
        vxg_b200.deltanet_step(ctx, q[i], k[i], v[i], br[i], ar[i], A, dt, state, o=o)
    ctx.sync()
    sampler = ClockSampler(local)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(torch, dist, world)
    sampler.start()
    e0.record()
    for i in range(W, T):
        vxg_b200.deltanet_step(ctx, q[i], k[i], v[i], br[i], ar[i], A, dt, state, o=o)
    e1.record()
    torch.cuda.synchronize()
    sampler.stop()
    ms = barrier_max(torch, dist, world, e0.elapsed_time(e1))
    alg = 2 * B * H * D * D * 4 + B * H * 4 * D * 4
    peak, peak_kind = measured_peaks()
    ach = alg / (ms / K * 1e-3) / 1e9
    res = {
        "metric": "gated-DeltaNet decode step: HBM GB/s and seq-steps/s",
        "value": B * world * K / (ms * 1e-3), "unit": "seq-steps/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config4: DeltaNet decode, 64 seqs x 32 heads, dk=dv=128, fp32 "
                               "state N(0,0.02^2) read+written every step",
                   "l2": "state larger than L2 (268 MB per step)"},
        "roofline": {"kernel": "deltanet_step_persistent", "bound": "hbm", "achieved": ach,
                     "peak": peak, "unit": "GB/s", "frac": ach / peak, "peak_kind": peak_kind,
                     "traffic": profile_traffic("deltanet_step_config4.json")},
        "gpu_launches": K, "clocks": sampler.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        i = W
        res["cpu_baseline"] = cpu_baseline_deltanet(
            q[i].cpu().numpy(), k[i].cpu().numpy(), v[i].cpu().numpy(), br[i].cpu().numpy(),
            ar[i].cpu().numpy(), A.cpu().numpy(), dt.cpu().numpy(), state.cpu().numpy())
    return res


def measure_long(args, world, rank, local, ctx, K, W, check=False):
    """B=1, ctx 262144, 1% of K rows x8.  One GPU: split-KV across its SMs.
    N GPUs: the KV range is split across ranks (vxg_b200.dist.LongContextDecoder): append on the
    owning rank, per-rank split-KV partial, exchange of (m, l, o) (NVLink peer memory or one
    NCCL all-gather), LSE combine.  A step is ~0.1 ms of device work, so on N GPUs the K timed
    steps are captured once into a CUDA graph and replayed, after one untimed step (a graph of
    its own, replayed first) that absorbs the skew between the ranks' replay launches; the split
    time per launch comes from an eager pass of K further steps.  With ``check``, the first step's merged output is compared
    on rank 0 with a one-GPU decode of the same whole cache, before anything is timed."""
    import torch
    import torch.distributed as dist
    import vxg_b200
    from vxg_b200 import workloads as wl
    L = 262144
    n_in = 2 + W + 2 * K
    cap = L + n_in + 8
    q, kn, vn = wl.decode_step_inputs_device(1, n_in, seed=4)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    dec = pool = None
    check_err = None
    if world == 1:
        pool = vxg_b200.KvQ8Pool(ctx, 1, wl.HKV, wl.HD, cap)
        wl.fill_pool_device(pool, [L], seed=3, outlier_frac=0.01)
        seq = torch.zeros(1, dtype=torch.int32, device="cuda")
        pos = [torch.tensor([L + i], dtype=torch.int32, device="cuda") for i in range(n_in)]
        out = torch.empty((1, wl.HQ, wl.HD), device="cuda")
        step = lambda i: pool.decode(seq, pos[i], q[i], kn[i], vn[i], out=out, max_ctx=cap)
    else:
        from vxg_b200.dist import KvRange, LongContextDecoder
        dec = LongContextDecoder(ctx, cap, wl.HQ, wl.HKV, wl.HD, world, rank,
                                 exchange=args.exchange)
        mine = dec.range.local_len(L)
        wl.fill_pool_device(dec.pool, [mine], seed=3 + rank, outlier_frac=0.01)
        step = lambda i: dec.step(L + i, q[i], kn[i], vn[i])
        if check:
            got = step(0).clone()
            torch.cuda.synchronize()
            if rank == 0:
                # the whole sequence on this GPU alone: every rank's slice rebuilt from its seed
                full = vxg_b200.KvQ8Pool(ctx, 1, wl.HKV, wl.HD, L + 1)
                for r in range(world):
                    kr = KvRange(cap, world, r)
                    wl.fill_pool_device(full, [kr.local_len(L)], seed=3 + r, outlier_frac=0.01,
                                        offset=kr.begin)
                one = full.decode(torch.zeros(1, dtype=torch.int32, device="cuda"),
                                  torch.tensor([L], dtype=torch.int32, device="cuda"), q[0],
                                  kn[0], vn[0], max_ctx=L + 1)
                check_err = float((one[0] - got.reshape(one[0].shape)).abs().max())
                full.close()
                del one
            barrier(torch, dist, world)
    first = 1 if (world > 1 and check) else 0
    for i in range(first, first + W):
        step(i)
    ctx.sync()
    t0 = first + W
    graph = align = None
    if world > 1:
        # One untimed step in a graph of its own is replayed first: the ranks' replays start at
        # different host times, and that step's exchange (each rank waits for every rank's
        # partials) absorbs the skew, so the events around the second graph time K steps of
        # aligned ranks.
        align = torch.cuda.CUDAGraph()
        with torch.cuda.graph(align):
            step(t0)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(t0 + 1, t0 + 1 + K):
                step(i)
        align.replay()
        graph.replay()
        torch.cuda.synchronize()
        t0 += 1
    # split-pass timing (events between the kernels) on steps of their own, before the timed ones
    barrier(torch, dist, world)
    ctx.set_timing(True)
    n_split = min(n_in, t0 + 2 * K) - (t0 + K)
    for i in range(t0 + K, t0 + K + n_split):
        step(i)
    torch.cuda.synchronize()
    split_local = ctx.split_ms_total() / max(1, n_split)
    split = barrier_max(torch, dist, world, split_local)
    ctx.set_timing(False)
    barrier(torch, dist, world)
    sampler = ClockSampler(local)
    sampler.start()
    if graph is not None:
        align.replay()
        e0.record()
        graph.replay()
        e1.record()
    else:
        e0.record()
        for i in range(t0, t0 + K):
            step(i)
        e1.record()
    torch.cuda.synchronize()
    sampler.stop()
    rc = ctx.sync()
    ms = barrier_max(torch, dist, world, e0.elapsed_time(e1))
    del graph, align
    torch.cuda.synchronize()
    # algorithmic bytes of this rank's split launches: its own share of the mean context
    mean_ctx = L + t0 + K // 2
    alg = float((mean_ctx if dec is None else dec.range.local_len(mean_ctx)) * wl.TOKEN_BYTES)
    if dec is not None:
        dec.close()
        dec.pool.close()
    peak, peak_kind = measured_peaks()
    ach = barrier_min(torch, dist, world, alg / (split_local * 1e-3) / 1e9)
    res = {"workload": "config3: B=1 ctx 262144, 1% K rows x8, split-KV over SMs"
                       + (f" and {world} GPUs (KV-range split, partials "
                          + ("through NVLink peer memory" if args.exchange == "peer"
                             else "by one NCCL all-gather")
                          + ", LSE combine, CUDA graph of the K steps)" if world > 1 else ""),
           "value": K / (ms * 1e-3), "unit": "seq-steps/s", "scaling": "strong",
           "ms_per_step": ms / K, "split_ms_per_launch": split,
           "exchange_and_merge_ms": max(0.0, ms / K - split),
           "exchange": (args.exchange if world > 1 else "none (one GPU)"),
           "roofline": {"kernel": "decode_fast_split", "bound": "hbm", "achieved": ach,
                        "peak": peak, "unit": "GB/s", "frac": ach / peak,
                        "peak_kind": peak_kind, "note": "slowest rank: its own bytes over its "
                        "own split time", "algorithmic_bytes_per_launch": alg},
           "gpu_launches": (3 if world == 1 else 4) * K, "clocks": sampler.summary(),
           "device_status": rc}
    if check_err is not None:
        res["check_vs_one_gpu_max_abs_err"] = check_err
    if pool is not None:
        res["_pool"] = pool
        res["_inputs"] = (L + t0 + K, q[n_in - 1], kn[n_in - 1], vn[n_in - 1])
    return res


def run_long(args, world, rank, local):
    """BASELINE config 3 as the main line (``--workload long``)."""
    import vxg_b200
    ctx = vxg_b200.Context()
    K, W = args.steps, args.warmup
    lr = measure_long(args, world, rank, local, ctx, K, W, check=world > 1)
    pool = lr.pop("_pool", None)
    inputs = lr.pop("_inputs", None)
    res = {"metric": METRIC, "value": lr["value"], "unit": "seq-steps/s", "n_gpus": world,
           "steps": K, "warmup": W, "ms_per_step": lr["ms_per_step"], "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": lr["workload"],
                      "l2": "inputs larger than L2 (285 MB of KV per step)"},
           "roofline": dict(lr["roofline"], split_ms_per_launch=lr["split_ms_per_launch"]),
           "long_context": {k: v for k, v in lr.items()
                            if k in ("exchange", "exchange_and_merge_ms",
                                     "check_vs_one_gpu_max_abs_err")},
           "gpu_launches": lr["gpu_launches"], "clocks": lr["clocks"]}
    if rank == 0 and world == 1 and not args.no_cpu_baseline and pool is not None:
        L, qi, ki, vi = inputs
        res["cpu_baseline"] = cpu_baseline_long(pool, L, qi.cpu().numpy(), ki.cpu().numpy(),
                                                vi.cpu().numpy())
    if pool is not None:
        pool.close()
    return res


def measured_tensor_peak(sustained=False):
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops_sustained" if sustained else "bf16_tflops"]), "measured"
    return (1400.0 if sustained else 1590.0), "fallback"


def run_prefill(args, world, rank, local):
    """BASELINE config 5a: per GPU 8 prompts of 8192 tokens, 16 q / 2 kv heads, head_dim 256,
    bf16 q/k/v from N(0,1).  One step = vxg_attn_cuda_q8_prefill over all 8 prompts: Q8 append
    of every prompt token, dequantisation of the cache, causal attention on tensor cores."""
    import torch
    import torch.distributed as dist
    import vxg_b200
    K, W = args.steps, args.warmup
    B, N, H, KV, HD = args.prompts, 8192, 16, 2, 256
    ctx = vxg_b200.Context()
    g = torch.Generator(device="cuda")
    g.manual_seed(7 + rank)
    q = torch.randn((B, N, H, HD), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((B, N, KV, HD), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((B, N, KV, HD), generator=g, device="cuda").to(torch.bfloat16)
    pool = vxg_b200.KvQ8Pool(ctx, B, KV, HD, N)
    seq = torch.arange(B, dtype=torch.int32, device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.empty((B, N, H, HD), device="cuda")
    step = lambda: pool.prefill(seq, pos, q, k, v, out=out, max_ctx=N)
    for _ in range(W):
        step()
    assert ctx.sync() == 0
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(torch, dist, world)
    sampler = ClockSampler(local)
    ctx.set_timing(True)
    sampler.start()
    e0.record()
    for _ in range(K):
        step()
    e1.record()
    torch.cuda.synchronize()
    sampler.stop()
    ms = barrier_max(torch, dist, world, e0.elapsed_time(e1))
    attn = barrier_max(torch, dist, world, ctx.split_ms_total() / K)
    flop = 4.0 * B * H * HD * N * (N + 1) / 2
    peak, peak_kind = measured_tensor_peak(sustained=True)
    ach = flop / (attn * 1e-3) / 1e12
    res = {
        "metric": "causal GQA prefill over the Q8 cache: prompt tokens/s and tensor TFLOP/s",
        "value": B * N * world * K / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 in, f16 x f16 -> f32 mma",
        "data": "synthetic",
        "config": {"workload": f"config5a: {B} prompts x 8192 tokens per GPU, 16 q / 2 kv heads, "
                               "head_dim 256, bf16 N(0,1) q/k/v, K/V appended to the Q8 cache",
                   "l2": "inputs larger than L2 (1.1 GB of q/k/v/out per step)"},
        "roofline": {"kernel": "prefill_tc_kernel", "bound": "tensor", "achieved": ach,
                     "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                     "peak_kind": peak_kind + " (sustained bf16)",
                     "flop_per_launch": flop, "attn_ms_per_launch": attn},
        "gpu_launches": 3 * K, "clocks": sampler.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_prefill(pool, q, B, N, H, KV, HD)
    pool.close()
    ctx.close()
    return res


def run_dnet_prefill(args, world, rank, local):
    """BASELINE config 5b: gated-DeltaNet prefill of 8 prompts x 8192 tokens per GPU, 32 heads,
    dk = dv = 128, the decode config's distributions (q, k, v N(0,1), beta = sigmoid(N(0,1)),
    decay exp(-softplus(N(0,1)))).  One step = vxg_attn_cuda_deltanet_prefill over all prompts
    (chunked WY form, 64-token chunks, one tcgen05 kernel with the state in tensor memory)."""
    import torch
    import torch.distributed as dist
    import vxg_b200
    K, W = args.steps, args.warmup
    B, T, H, D = args.prompts, 8192, 32, 128
    ctx = vxg_b200.Context()
    g = torch.Generator(device="cuda")
    g.manual_seed(11 + rank)
    q = torch.randn((B, T, H, D), generator=g, device="cuda")
    k = torch.randn((B, T, H, D), generator=g, device="cuda")
    v = torch.randn((B, T, H, D), generator=g, device="cuda")
    br = torch.randn((B, T, H), generator=g, device="cuda")
    ar = torch.randn((B, T, H), generator=g, device="cuda")
    A = -torch.ones(H, device="cuda")
    dt = torch.zeros(H, device="cuda")
    state0 = torch.randn((B, H, D, D), generator=g, device="cuda") * 0.02
    state = state0.clone()
    o = torch.empty((B, T, H, D), device="cuda")
    step = lambda: vxg_b200.deltanet_prefill(ctx, q, k, v, br, ar, A, dt, state, o=o)
    for _ in range(W):
        step()
    assert ctx.sync() == 0
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(torch, dist, world)
    sampler = ClockSampler(local)
    sampler.start()
    e0.record()
    for _ in range(K):
        step()
    e1.record()
    torch.cuda.synchronize()
    sampler.stop()
    ms = barrier_max(torch, dist, world, e0.elapsed_time(e1))
    C = 64
    mac = (5 * C * C * D + 3 * C * D * D) * (T // C) * B * H   # chunked (WY) form per call
    peak, peak_kind = measured_tensor_peak(sustained=True)
    ach = 2 * mac / (ms / K * 1e-3) / 1e12
    res = {
        "metric": "gated-DeltaNet prefill: prompt tokens/s",
        "value": B * T * world * K / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config5b: DeltaNet prefill, {B} prompts x 8192 tokens per GPU, "
                               "32 heads, dk=dv=128, state N(0,0.02^2) on chip",
                   "l2": "inputs larger than L2 (4.3 GB of q/k/v/o per step)"},
        "roofline": {"kernel": "deltanet_chunk_tc_kernel", "bound": "tensor", "achieved": ach,
                     "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                     "peak_kind": peak_kind + " (sustained bf16)",
                     "flop_per_launch": 2 * mac,
                     "note": "FLOPs of the chunked (WY, C=64) algorithm, counted once; the "
                             "kernel runs its products on tcgen05 (f16, bf16 and hi/lo-split "
                             "bf16, so up to 3x these FLOPs on the tensor pipe) and forms the "
                             "norms, gates and the triangular inverse on chip"},
        "gpu_launches": K, "clocks": sampler.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_dnet_prefill(q, k, v, br, ar, A, dt, state0)
    ctx.close()
    return res


# --------------------------------------------------------------------------- reference arm
def run_reference(args, world, rank):
    """The reference algorithm (the C restatement of the Rust CPU operators; the Rust crate
    cannot be built here) on this host's cores, on a bounded sample of the same workload."""
    from oracle import oracle
    from vxg_b200 import workloads as wl
    K, W = args.steps, args.warmup
    cores = host_cores()
    batch = wl.DecodeBatch(seed=1)
    lens = batch.ctx_lens()
    S = cpu_sample_size(batch.n_seq, cores)
    lens = lens[:S]
    rng = np.random.default_rng(17)
    cap = int(lens.max()) + W + K + 1
    nb = wl.HD // 32
    kpool = np.zeros((S, cap, wl.HKV, nb, 34), np.uint8)
    vpool = np.zeros_like(kpool)
    for s in range(S):
        for t0 in range(0, int(lens[s]), 4096):
            n = min(4096, int(lens[s]) - t0)
            kpool[s, t0:t0 + n] = oracle.q8_quantize(
                rng.standard_normal((n, wl.HKV, wl.HD), dtype=np.float32))
            vpool[s, t0:t0 + n] = oracle.q8_quantize(
                rng.standard_normal((n, wl.HKV, wl.HD), dtype=np.float32))
    kflat, vflat = kpool.reshape(-1), vpool.reshape(-1)
    seq = np.arange(S, dtype=np.int32)

    def step(i):
        q = rng.standard_normal((S, wl.HQ, wl.HD), dtype=np.float32)
        kn = rng.standard_normal((S, wl.HKV, wl.HD), dtype=np.float32)
        vn = rng.standard_normal((S, wl.HKV, wl.HD), dtype=np.float32)
        t = time.perf_counter()
        oracle.batch_decode_q8(seq, (lens + i).astype(np.int32), q, kn, vn, kflat, vflat, cap,
                               wl.HQ, wl.HKV, wl.HD, do_append=True, n_threads=cores)
        return time.perf_counter() - t

    for i in range(W):
        step(i)
    el = sum(step(W + i) for i in range(K))
    v = S * K / el
    sample = (f"{S} of the 64 config-2 sequences (mean ctx {lens.mean():.0f}) per step, one "
              f"append+attend each, {cores} threads")
    return {"metric": METRIC, "value": v, "unit": "seq-steps/s", "impl": "reference",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": el / K * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "config2: batched decode + Q8 append, 64 seqs per GPU, ctx "
                                   "U[1024,32768], 16 q / 2 kv heads, head_dim 256, Q8_0 KV "
                                   "(34-B blocks)", "seqs_per_step_sampled": S},
            "cpu_baseline": {"value": v, "unit": "seq-steps/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": v, "unit": "seq-steps/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "long", "deltanet", "prefill", "dnet_prefill"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-long", action="store_true",
                    help="decode workload: skip the config-3 long-context leg")
    ap.add_argument("--seqs", type=int, default=64, help="sequences per GPU (profiling runs)")
    ap.add_argument("--ctx-max", type=int, default=32768, help="context upper bound (profiling)")
    ap.add_argument("--prompts", type=int, default=8, help="prefill prompts per GPU (profiling)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="config 3 on N GPUs: partials through NVLink peer memory or NCCL")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, world, rank)), flush=True)
        return
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        fn = {"decode": run_decode, "deltanet": run_deltanet, "long": run_long,
              "prefill": run_prefill, "dnet_prefill": run_dnet_prefill}[args.workload]
        res = fn(args, world, rank, local)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
