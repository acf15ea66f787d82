"""Two-GPU KV-range split of one long context: LongContextDecoder on 2 ranks, with the partials
exchanged by NCCL or through NVLink peer memory, equals the single-GPU decode of the same cache,
also when the peer steps are replayed from a CUDA graph.  Skipped with fewer than 2 GPUs."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import os, sys, datetime, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, os.environ["ROOT"])
import vxg_b200
from vxg_b200.dist import LongContextDecoder
from oracle import oracle
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                        device_id=torch.device("cuda", rank))
rng = np.random.default_rng(5)
L, cap = 3000, 3100
k = rng.standard_normal((L + 8, 2, 256)).astype(np.float32)
v = rng.standard_normal((L + 8, 2, 256)).astype(np.float32)
kb, vb = oracle.q8_quantize(k), oracle.q8_quantize(v)
ctx = vxg_b200.Context()
dec = LongContextDecoder(ctx, cap, 16, 2, 256, world, rank, exchange=os.environ["EXCHANGE"])
lo = dec.range.begin; n = dec.range.local_len(L)
if n: dec.pool.import_blocks(0, 0, kb[lo:lo + n], vb[lo:lo + n])
full = vxg_b200.KvQ8Pool(ctx, 1, 2, 256, cap)
full.import_blocks(0, 0, kb[:L], vb[:L])
worst = 0.0
for i in range(4):
    q = rng.standard_normal((16, 256)).astype(np.float32)
    out = dec.step(L + i, torch.from_numpy(q).cuda(), torch.from_numpy(k[L + i]).cuda(),
                   torch.from_numpy(v[L + i]).cuda())
    want = full.decode(np.zeros(1, np.int32), np.array([L + i], np.int32), q[None],
                       k_new=k[L + i][None], v_new=v[L + i][None])[0]
    worst = max(worst, float(np.abs(out.cpu().numpy() - want).max()))
ctx.sync()
if dec.peer is not None:
    # the same steps captured once and replayed: the device-side step counter keeps the flags
    # of both ranks in step across replays
    qs = [torch.from_numpy(rng.standard_normal((16, 256)).astype(np.float32)).cuda()
          for _ in range(3)]
    kn = [torch.from_numpy(k[L + 4 + i]).cuda() for i in range(3)]
    vn = [torch.from_numpy(v[L + 4 + i]).cuda() for i in range(3)]
    outs = [torch.empty((16, 256), device="cuda") for _ in range(3)]
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(3):
            # appends go to fixed positions: replaying rewrites the same tokens
            outs[i].copy_(dec.step(L + 4 + i, qs[i], kn[i], vn[i]))
    for rep in range(2):
        g.replay()
        torch.cuda.synchronize()
        for i in range(3):
            want = full.decode(np.zeros(1, np.int32), np.array([L + 4 + i], np.int32),
                               qs[i].cpu().numpy()[None], k_new=k[L + 4 + i][None],
                               v_new=v[L + 4 + i][None])[0]
            worst = max(worst, float(np.abs(outs[i].cpu().numpy() - want).max()))
    del g
    assert ctx.sync() == 0
dec.close()
print(f"rank {rank} max|diff| {worst:.3e}", flush=True)
dist.destroy_process_group()
assert worst < 1e-4
"""


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_long_context_split_two_gpus(tmp_path, exchange):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "w.py"
    script.write_text(WORKER)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, ROOT=ROOT, NCCL_NVLS_ENABLE="0", EXCHANGE=exchange)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port",
           str(port), str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
