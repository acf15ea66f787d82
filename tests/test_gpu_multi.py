"""Two-GPU KV-range split of one long context (NCCL): LongContextDecoder on 2 ranks equals the
single-GPU decode of the same cache.  Skipped on machines with fewer than 2 GPUs."""
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
k = rng.standard_normal((L + 4, 2, 256)).astype(np.float32)
v = rng.standard_normal((L + 4, 2, 256)).astype(np.float32)
kb, vb = oracle.q8_quantize(k), oracle.q8_quantize(v)
ctx = vxg_b200.Context()
dec = LongContextDecoder(ctx, cap, 16, 2, 256, world, rank)
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
print(f"rank {rank} max|diff| {worst:.3e}", flush=True)
dist.destroy_process_group()
assert worst < 1e-4
"""


def test_long_context_split_two_gpus(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "w.py"
    script.write_text(WORKER)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, ROOT=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port",
           str(port), str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
