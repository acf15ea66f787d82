"""Multi-GPU layouts of the decode path (one process per GPU, torch.distributed plumbing).

* Sequence sharding (batched decode, DeltaNet): each rank owns whole sequences; no collective
  on the data path.  ``shard_sequences`` gives a rank's contiguous share.
* KV-range split of one long context: rank r owns tokens [r*span, (r+1)*span) of the sequence
  in its own KV pool.  A decode step appends the new token on the rank that owns its
  position, every rank computes the split-KV partial (m, l, o) of the query over its range,
  the partials are all-gathered (NCCL over NVLink on GPUs; any backend works for the host
  logic), and every rank merges them with the log-sum-exp combine.  The exchanged data is
  n_head * (head_dim + 2) floats per rank, so the collective is latency-bound.  With
  ``exchange="peer"`` the partials travel through NVLink peer memory instead (PeerExchange:
  plain stores into every rank's IPC-mapped buffer, a step flag, a bounded wait and the merge,
  two kernels and no collective per step).
"""
from __future__ import annotations

import math

import numpy as np


def shard_sequences(n_seq: int, world: int, rank: int) -> range:
    """Contiguous, balanced share of sequence ids for ``rank``."""
    base, extra = divmod(n_seq, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


class KvRange:
    """Token-range ownership of one sequence split over ``world`` ranks."""

    def __init__(self, capacity: int, world: int, rank: int):
        self.world, self.rank = world, rank
        self.span = int(math.ceil(capacity / world))
        self.begin = rank * self.span

    def owner(self, pos: int) -> int:
        return min(pos // self.span, self.world - 1)

    def local_pos(self, pos: int) -> int:
        return pos - self.owner(pos) * self.span

    def local_len(self, ctx_len: int) -> int:
        """Tokens of [0, ctx_len) that live on this rank."""
        return int(max(0, min(self.span, ctx_len - self.begin)))


def pack_partials(m, l, o):
    """(m [R], l [R], o [R][hd]) -> one flat tensor [R*(hd+2)] for a single collective."""
    import torch
    return torch.cat([m.reshape(-1), l.reshape(-1), o.reshape(-1)])


def unpack_partials(buf, world: int, rows: int, hd: int):
    """[world * rows*(hd+2)] -> m, l [world][rows], o [world][rows][hd]."""
    per = rows * (hd + 2)
    b = buf.reshape(world, per)
    return (b[:, :rows].contiguous(), b[:, rows:2 * rows].contiguous(),
            b[:, 2 * rows:].reshape(world, rows, hd).contiguous())


def all_gather_partials(m, l, o, group=None):
    """All-gather this rank's partials; returns m, l [world][R], o [world][R][hd]."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rows, hd = o.reshape(-1, o.shape[-1]).shape
    send = pack_partials(m, l, o)
    recv = torch.empty(world * send.numel(), dtype=send.dtype, device=send.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    return unpack_partials(recv, world, rows, hd)


class PeerExchange:
    """Exchange + log-sum-exp merge of packed partials through NVLink peer memory
    (vxg_attn_cuda_peer_*): every rank maps every other rank's exchange buffer once (CUDA IPC
    handles passed with all_gather_object), then each ``step`` is two kernels on the caller's
    stream and no collective.  Collective over the group: every rank constructs it, steps it
    the same number of times and closes it."""

    def __init__(self, ctx, world: int, rank: int, n_rows: int, head_dim: int, group=None):
        import ctypes
        import torch.distributed as dist
        from ._lib import ErrBuf, VxgError, lib
        self.ctx, self.world, self.rank = ctx, world, rank
        self.n_rows, self.head_dim, self.group = n_rows, head_dim, group
        err = ErrBuf()
        handle = (ctypes.c_uint8 * 64)()
        self._own = lib().vxg_attn_cuda_peer_alloc(ctx.h, world, n_rows, head_dim, handle,
                                                   err.buf, err.cap)
        if not self._own:
            raise VxgError(-7, "vxg_attn_cuda_peer_alloc: " + err.text)
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._mapped = []
        ptrs = []
        for r in range(world):
            if r == rank:
                ptrs.append(self._own)
                continue
            hb = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
            p = lib().vxg_attn_cuda_peer_open(ctx.h, hb, err.buf, err.cap)
            if not p:
                raise VxgError(-7, f"vxg_attn_cuda_peer_open(rank {r}): " + err.text)
            self._mapped.append(p)
            ptrs.append(p)
        self._bufs = (ctypes.c_void_p * world)(*ptrs)
        dist.barrier(group=group)  # every buffer mapped everywhere before the first push

    def step(self, send, out, gate=None, stream=None):
        """Pushes this rank's packed partials `send` and writes the merged rows to `out`."""
        import ctypes
        import torch
        from ._lib import ErrBuf, check, lib
        from .attn import _stream_handle
        s = _stream_handle(stream if stream is not None else torch.cuda.current_stream())
        err = ErrBuf()
        check(lib().vxg_attn_cuda_peer_step(
            self.ctx.h, self._bufs, self.world, self.rank, self.n_rows, self.head_dim,
            ctypes.c_void_p(send.data_ptr()),
            ctypes.c_void_p(gate.data_ptr()) if gate is not None else None,
            ctypes.c_void_p(out.data_ptr()), s, err.buf, err.cap), err)
        return out

    def close(self):
        """After every rank's last step: unmap the peers' buffers and free the own one."""
        import torch
        import torch.distributed as dist
        from ._lib import lib
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no rank still writes into any buffer
        for p in self._mapped:
            lib().vxg_attn_cuda_peer_close(self.ctx.h, p)
        self._mapped = []
        dist.barrier(group=self.group)  # every mapping of the own buffer is gone
        lib().vxg_attn_cuda_peer_free(self.ctx.h, self._own)
        self._own = None


class LongContextDecoder:
    """One long sequence split by KV range across the ranks of the default process group.

    Owns this rank's slice as a one-sequence KvQ8Pool; ``step`` appends the new token where it
    belongs and returns the merged attention output (every rank gets it).  Per step: the split
    kernels write this rank's (m, l, o) straight into a packed send buffer, one NCCL
    all_gather_into_tensor exchanges n_head*(head_dim+2) floats per rank, and the packed
    log-sum-exp combine merges them; all buffers are allocated once."""

    def __init__(self, ctx, capacity: int, n_head: int, n_head_kv: int, head_dim: int,
                 world: int, rank: int, group=None, exchange: str = "nccl"):
        from .attn import KvQ8Pool
        import torch
        self.ctx = ctx
        self.range = KvRange(capacity, world, rank)
        self.pool = KvQ8Pool(ctx, 1, n_head_kv, head_dim, self.range.span)
        self.n_head, self.head_dim, self.world = n_head, head_dim, world
        self.group = group
        dev = torch.device("cuda", torch.cuda.current_device())
        self._seq = torch.zeros(1, dtype=torch.int32, device=dev)
        self._begin = torch.zeros(1, dtype=torch.int32, device=dev)
        # one-element views of a constant 0 .. span table stand for this step's local position
        # and length: no kernel to set them (a captured step replays with its own views)
        self._ar = torch.arange(self.range.span + 1, dtype=torch.int32, device=dev)
        per = n_head * (head_dim + 2)
        self._send = torch.empty(per, dtype=torch.float32, device=dev)
        self._recv = torch.empty(world * per, dtype=torch.float32, device=dev)
        self._out = torch.empty((n_head, head_dim), dtype=torch.float32, device=dev)
        self._m = self._send[:n_head].view(1, n_head)
        self._l = self._send[n_head:2 * n_head].view(1, n_head)
        self._o = self._send[2 * n_head:].view(1, n_head, head_dim)
        if exchange not in ("nccl", "peer"):
            raise ValueError("exchange must be 'nccl' or 'peer'")
        self.peer = PeerExchange(ctx, world, rank, n_head, head_dim, group) \
            if exchange == "peer" else None

    def close(self):
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def step(self, pos: int, q, k_new, v_new, scale=None):
        """Append (k_new, v_new) at ``pos`` (on its owner) and attend q over [0, pos]."""
        import torch.distributed as dist
        from .attn import lse_combine_packed
        r = self.range
        if r.owner(pos) == r.rank:
            lp = r.local_pos(pos)
            self.pool.append(self._seq, self._ar[lp:lp + 1], k_new.reshape(1, 1, -1, self.head_dim),
                             v_new.reshape(1, 1, -1, self.head_dim))
        le = r.local_len(pos + 1)
        self.pool.decode_partial(self._seq, self._begin, self._ar[le:le + 1],
                                 q.reshape(1, self.n_head, self.head_dim), scale=scale,
                                 out=(self._m, self._l, self._o))
        if self.peer is not None:
            return self.peer.step(self._send, self._out)
        dist.all_gather_into_tensor(self._recv, self._send, group=self.group)
        return lse_combine_packed(self.ctx, self._recv, self.world, self.n_head, self.head_dim,
                                  out=self._out)
