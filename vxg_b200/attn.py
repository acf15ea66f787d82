"""Python host layer over the C ABI: the vxg-tensor attention operators on B200.

Mirrors the reference's operator surface for the Q8-KV attention / gated-DeltaNet path:

* ``KvQ8Block`` -- the 34-byte block dtype (crates/vxg-tensor/src/llm_prefill.rs:17-24).
* ``KvQ8Pool`` -- the per-layer K/V caches of ``LlmState`` (llm.rs:36-41) as device pools,
  one per attention layer, ``n_seq`` sequences each.
* ``step_full_gqa_q8`` -- drop-in for llm_prefill.rs:259-370 (same arguments, same in-place
  behaviour on ``k_cur`` and ``attn_out``; the cache argument is a ``KvQ8Pool`` + sequence id).
* ``KvQ8Pool.append`` / ``.decode`` / ``.decode_partial`` / ``lse_combine`` -- batched forms.
* ``deltanet_step`` -- the gated-DeltaNet core, llm_ops.rs:139-184, batched over sequences.

Arrays are numpy (host memory: the call copies in/out and is synchronous) or torch CUDA tensors
(device memory: the call is enqueued on torch's current stream, or ``stream``, and is
asynchronous; ``Context.sync()`` collects the device status word).
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from ._lib import (MEM_DEVICE, MEM_HOST, ErrBuf, VxgError, check, lib)

KvQ8Block = np.dtype([("d", "<u2"), ("qs", "i1", (32,))])
assert KvQ8Block.itemsize == 34


# cudaStreamLegacy: torch reports its default stream as handle 0, which the C ABI would read as
# "no stream" (synchronous, on the context's own stream); name the legacy default stream instead.
_CUDA_STREAM_LEGACY = 1


def _stream_handle(s):
    h = int(s.cuda_stream)
    return ctypes.c_void_p(h if h != 0 else _CUDA_STREAM_LEGACY)


def _is_torch(x) -> bool:
    return type(x).__module__.startswith("torch")


class _Args:
    """Collects pointer arguments of one call, all host (numpy) or all device (torch)."""

    def __init__(self, like):
        self.device = _is_torch(like) and like.is_cuda
        self.keep = []

    def ptr(self, x, dtype, shape=None, name="array", writable=False):
        if x is None:
            return None
        if self.device:
            import torch
            if not (_is_torch(x) and x.is_cuda):
                raise TypeError(f"{name}: expected a CUDA tensor (the call uses device memory)")
            tdt = {np.float32: torch.float32, np.int32: torch.int32, np.uint8: torch.uint8,
                   "bf16": torch.bfloat16}[dtype]
            if x.dtype != tdt:
                raise TypeError(f"{name}: dtype {x.dtype}, expected {tdt}")
            if not x.is_contiguous():
                raise ValueError(f"{name}: must be contiguous")
            if shape is not None and x.numel() != int(np.prod(shape)):
                raise ValueError(f"{name}: {x.numel()} elements, expected shape {shape}")
            return ctypes.c_void_p(x.data_ptr())
        if _is_torch(x):
            raise TypeError(f"{name}: expected a numpy array (the call uses host memory)")
        if dtype == "bf16":
            # host bf16 travels as its raw 16-bit patterns
            if not (isinstance(x, np.ndarray) and x.dtype == np.uint16):
                raise TypeError(f"{name}: host bf16 data must be a uint16 numpy array of bits")
            dtype = np.uint16
        if writable:
            if not (isinstance(x, np.ndarray) and x.dtype == dtype and x.flags.c_contiguous):
                raise TypeError(f"{name}: must be a C-contiguous {np.dtype(dtype)} numpy array")
            a = x
        else:
            a = np.ascontiguousarray(x, dtype=dtype)
        if shape is not None and a.size != int(np.prod(shape)):
            raise ValueError(f"{name}: {a.size} elements, expected shape {shape}")
        self.keep.append(a)
        return a.ctypes.data_as(ctypes.c_void_p)

    @property
    def memkind(self):
        return MEM_DEVICE if self.device else MEM_HOST

    def stream(self, stream):
        if not self.device:
            return None
        import torch
        s = stream if stream is not None else torch.cuda.current_stream()
        return _stream_handle(s)


class Context:
    """One CUDA context handle (vxg_attn_cuda_create), bound to the current device."""

    def __init__(self):
        self._err = ErrBuf()
        self.h = lib().vxg_attn_cuda_create(self._err.buf, self._err.cap)
        if not self.h:
            raise VxgError(-7, "vxg_attn_cuda_create failed: " + self._err.text)
        self.device_name = self._err.text
        self.sm_count = lib().vxg_attn_cuda_sm_count(self.h)
        self._pinned = []
        self._inflight = {}  # ticket -> arrays an overlapped step still reads or writes

    def close(self):
        if self.h:
            for p in self._pinned:
                lib().vxg_attn_cuda_host_free(self.h, p)
            self._pinned = []
            lib().vxg_attn_cuda_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def sync(self, stream=None) -> int:
        s = None
        if stream is not None:
            s = _stream_handle(stream)
        else:
            try:
                import torch
                if torch.cuda.is_available():
                    s = _stream_handle(torch.cuda.current_stream())
            except ImportError:
                pass
        return check(lib().vxg_attn_cuda_sync(self.h, s, self._err.buf, self._err.cap), self._err)

    def set_timing(self, enable: bool):
        lib().vxg_attn_cuda_set_timing(self.h, int(enable))

    def split_ms_total(self) -> float:
        """Device ms summed over the split-KV passes since set_timing (waits for the last)."""
        return float(lib().vxg_attn_cuda_last_split_ms(self.h))

    def force_generic(self, enable: bool):
        lib().vxg_attn_cuda_force_generic(self.h, int(enable))

    def checkpoint(self, states, backups, restore: bool = False, stream=None):
        """Copy each device tensor of ``states`` into the matching one of ``backups`` (or back
        with restore=True): vxg_attn_cuda_state_checkpoint, asynchronous on the stream."""
        import torch
        n = len(states)
        if len(backups) != n:
            raise ValueError("states and backups differ in length")
        for s_, b_ in zip(states, backups):
            if s_.numel() * s_.element_size() != b_.numel() * b_.element_size():
                raise ValueError("state and backup sizes differ")
        src = (ctypes.c_void_p * n)(*[s_.data_ptr() for s_ in states])
        dst = (ctypes.c_void_p * n)(*[b_.data_ptr() for b_ in backups])
        nb = (ctypes.c_size_t * n)(*[s_.numel() * s_.element_size() for s_ in states])
        s = stream if stream is not None else torch.cuda.current_stream()
        err = ErrBuf()
        return check(lib().vxg_attn_cuda_state_checkpoint(
            self.h, n, ctypes.cast(src, ctypes.c_void_p), ctypes.cast(dst, ctypes.c_void_p),
            ctypes.cast(nb, ctypes.c_void_p), int(restore), _stream_handle(s), err.buf, err.cap),
            err)

    def host_alloc(self, nbytes: int):
        err = ErrBuf()
        p = lib().vxg_attn_cuda_host_alloc(self.h, nbytes, err.buf, err.cap)
        if not p:
            raise VxgError(-7, err.text)
        return p

    def host_free(self, p):
        lib().vxg_attn_cuda_host_free(self.h, p)

    def wait(self, ticket: int) -> int:
        """Waits for an overlapped host-memory step (KvQ8Pool.decode_host_async) and returns its
        status code; the step's input arrays are released."""
        rc = check(lib().vxg_attn_cuda_ticket_wait(self.h, ctypes.c_uint64(ticket), self._err.buf,
                                                   self._err.cap), self._err)
        self._inflight.pop(ticket, None)
        return rc

    def pinned_empty(self, shape, dtype):
        """numpy array in pinned host memory, freed when this context is closed."""
        dt = np.dtype(dtype)
        n = max(int(np.prod(shape)) * dt.itemsize, 1)
        p = self.host_alloc(n)
        self._pinned.append(p)
        buf = (ctypes.c_uint8 * n).from_address(p)
        return np.frombuffer(buf, dtype=np.uint8, count=n)[: int(np.prod(shape)) * dt.itemsize] \
            .view(dt).reshape(shape)


class KvQ8Pool:
    """Device K/V pools of KvQ8Block[n_seq][cap][n_head_kv][head_dim/32] (vxg_attn_cuda_kv_*)."""

    def __init__(self, ctx: Context, n_seq: int, n_head_kv: int, head_dim: int, cap_tokens: int):
        self.ctx = ctx
        err = ErrBuf()
        self.h = lib().vxg_attn_cuda_kv_create(ctx.h, n_seq, n_head_kv, head_dim, cap_tokens,
                                               err.buf, err.cap)
        if not self.h:
            raise VxgError(-2, "vxg_attn_cuda_kv_create failed: " + err.text)
        self.n_seq, self.n_head_kv, self.head_dim = n_seq, n_head_kv, head_dim
        self.nb = head_dim // 32

    def close(self):
        if self.h:
            lib().vxg_attn_cuda_kv_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def capacity(self) -> int:
        return int(lib().vxg_attn_cuda_kv_capacity(self.h))

    @property
    def nbytes(self) -> int:
        return int(lib().vxg_attn_cuda_kv_bytes(self.h))

    def reserve(self, cap_tokens: int):
        err = ErrBuf()
        check(lib().vxg_attn_cuda_kv_reserve(self.h, cap_tokens, err.buf, err.cap), err)

    def device_ptrs(self):
        k, v, s = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_size_t()
        check(lib().vxg_attn_cuda_kv_device_ptrs(self.h, ctypes.byref(k), ctypes.byref(v),
                                                 ctypes.byref(s)), ErrBuf())
        return k.value, v.value, s.value

    def import_blocks(self, seq: int, tok_begin: int, k_blocks, v_blocks):
        """k/v_blocks: (n_tok, n_head_kv, nb) KvQ8Block or (..., 34) uint8, host or device."""
        args = _Args(k_blocks)
        kb = k_blocks.view(np.uint8) if isinstance(k_blocks, np.ndarray) else k_blocks
        vb = v_blocks.view(np.uint8) if isinstance(v_blocks, np.ndarray) else v_blocks
        n_bytes = (kb.nbytes if isinstance(kb, np.ndarray) else kb.numel())
        per_tok = self.n_head_kv * self.nb * 34
        if n_bytes % per_tok:
            raise ValueError("block array is not a whole number of tokens")
        n_tok = n_bytes // per_tok
        err = ErrBuf()
        check(lib().vxg_attn_cuda_kv_import(self.ctx.h, self.h, seq, tok_begin, n_tok,
                                            args.ptr(kb, np.uint8, name="k_blocks"),
                                            args.ptr(vb, np.uint8, name="v_blocks"),
                                            args.memkind, err.buf, err.cap), err)

    def export_blocks(self, seq: int, tok_begin: int, n_tok: int):
        """Returns host (k, v) uint8 arrays of shape (n_tok, n_head_kv, nb, 34)."""
        shape = (n_tok, self.n_head_kv, self.nb, 34)
        k = np.empty(shape, np.uint8)
        v = np.empty(shape, np.uint8)
        err = ErrBuf()
        check(lib().vxg_attn_cuda_kv_export(self.ctx.h, self.h, seq, tok_begin, n_tok,
                                            k.ctypes.data_as(ctypes.c_void_p),
                                            v.ctypes.data_as(ctypes.c_void_p), MEM_HOST,
                                            err.buf, err.cap), err)
        return k, v

    # ---------------------------------------------------------------- ops
    def append(self, seq_ids, pos, k_new, v_new, n_tok: int = 1, stream=None) -> int:
        """Quantise-and-append k_new/v_new [B][n_tok][n_head_kv][head_dim] at pos[b] + t."""
        a = _Args(k_new)
        B = len(seq_ids) if not a.device else seq_ids.numel()
        shp = (B, n_tok, self.n_head_kv, self.head_dim)
        err = ErrBuf()
        return check(lib().vxg_attn_cuda_q8_append(
            self.ctx.h, self.h, B, n_tok, a.ptr(seq_ids, np.int32, (B,), "seq_ids"),
            a.ptr(pos, np.int32, (B,), "pos"), a.ptr(k_new, np.float32, shp, "k_new"),
            a.ptr(v_new, np.float32, shp, "v_new"), a.memkind, a.stream(stream), err.buf,
            err.cap), err)

    def decode(self, seq_ids, pos, q, k_new=None, v_new=None, q_gate=None, scale=None,
               max_ctx: int = 0, out=None, stream=None):
        """Append (if k_new) then attend over [0, pos[b]]: returns out [B][n_head][head_dim]."""
        a = _Args(q)
        B = len(seq_ids) if not a.device else seq_ids.numel()
        n_head = (q.size if not a.device else q.numel()) // (B * self.head_dim)
        qshape = (B, n_head, self.head_dim)
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if out is None:
            if a.device:
                import torch
                out = torch.empty(qshape, dtype=torch.float32, device=q.device)
            else:
                out = np.empty(qshape, np.float32)
        kshape = (B, self.n_head_kv, self.head_dim)
        err = ErrBuf()
        rc = check(lib().vxg_attn_cuda_q8_decode(
            self.ctx.h, self.h, B, n_head, a.ptr(seq_ids, np.int32, (B,), "seq_ids"),
            a.ptr(pos, np.int32, (B,), "pos"), a.ptr(q, np.float32, qshape, "q"),
            a.ptr(k_new, np.float32, kshape, "k_new"), a.ptr(v_new, np.float32, kshape, "v_new"),
            a.ptr(q_gate, np.float32, qshape, "q_gate"), ctypes.c_float(scale), max_ctx,
            a.ptr(out, np.float32, qshape, "out", writable=True), a.memkind, a.stream(stream),
            err.buf, err.cap), err)
        self.last_rc = rc
        return out

    def decode_host_async(self, seq_ids, pos, q, k_new=None, v_new=None, q_gate=None,
                          scale=None, max_ctx: int = 0, out=None) -> int:
        """decode() on numpy (ideally pinned) arrays, overlapped with the neighbouring steps
        (vxg_attn_cuda_q8_decode_host_async).  Returns a ticket; `out` is valid after
        ctx.wait(ticket).  The arrays must not change until then (references are kept)."""
        a = _Args(q)
        if a.device:
            raise TypeError("decode_host_async takes host (numpy) arrays")
        B = len(seq_ids)
        n_head = q.size // (B * self.head_dim)
        qshape = (B, n_head, self.head_dim)
        kshape = (B, self.n_head_kv, self.head_dim)
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if out is None:
            out = np.empty(qshape, np.float32)
        ptrs = [a.ptr(seq_ids, np.int32, (B,), "seq_ids"), a.ptr(pos, np.int32, (B,), "pos"),
                a.ptr(q, np.float32, qshape, "q"), a.ptr(k_new, np.float32, kshape, "k_new"),
                a.ptr(v_new, np.float32, kshape, "v_new"),
                a.ptr(q_gate, np.float32, qshape, "q_gate")]
        optr = a.ptr(out, np.float32, qshape, "out", writable=True)
        ticket = ctypes.c_uint64(0)
        err = ErrBuf()
        check(lib().vxg_attn_cuda_q8_decode_host_async(
            self.ctx.h, self.h, B, n_head, *ptrs, ctypes.c_float(scale), max_ctx, optr,
            ctypes.byref(ticket), err.buf, err.cap), err)
        if ticket.value:
            self.ctx._inflight[ticket.value] = (a.keep, out)
        return ticket.value

    def prefill(self, seq_ids, pos, q, k_new, v_new, q_gate=None, scale=None,
                max_ctx: int = 0, out=None, stream=None):
        """Append the prompt's K/V at pos[b] + t and attend each query token causally.

        q [B][n_tok][n_head][head_dim] and k_new / v_new [B][n_tok][n_head_kv][head_dim] are f32
        or bf16 (torch.bfloat16 on the device, uint16 bit patterns on the host).
        Returns out [B][n_tok][n_head][head_dim] f32."""
        a = _Args(q)
        if a.device:
            import torch
            bf16 = q.dtype == torch.bfloat16
        else:
            bf16 = isinstance(q, np.ndarray) and q.dtype == np.uint16
        dt = "bf16" if bf16 else np.float32
        B = len(seq_ids) if not a.device else seq_ids.numel()
        kv_el = (k_new.size if not a.device else k_new.numel())
        n_tok = kv_el // (B * self.n_head_kv * self.head_dim)
        n_head = (q.size if not a.device else q.numel()) // (B * n_tok * self.head_dim)
        qshape = (B, n_tok, n_head, self.head_dim)
        kshape = (B, n_tok, self.n_head_kv, self.head_dim)
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if out is None:
            if a.device:
                import torch
                out = torch.empty(qshape, dtype=torch.float32, device=q.device)
            else:
                out = np.empty(qshape, np.float32)
        err = ErrBuf()
        rc = check(lib().vxg_attn_cuda_q8_prefill(
            self.ctx.h, self.h, B, n_tok, n_head, a.ptr(seq_ids, np.int32, (B,), "seq_ids"),
            a.ptr(pos, np.int32, (B,), "pos"), a.ptr(q, dt, qshape, "q"),
            a.ptr(k_new, dt, kshape, "k_new"), a.ptr(v_new, dt, kshape, "v_new"),
            a.ptr(q_gate, dt, qshape, "q_gate"), int(bf16), ctypes.c_float(scale), max_ctx,
            a.ptr(out, np.float32, qshape, "out", writable=True), a.memkind, a.stream(stream),
            err.buf, err.cap), err)
        self.last_rc = rc
        return out

    def decode_partial(self, seq_ids, kv_begin, kv_end, q, scale=None, max_ctx: int = 0,
                       stream=None, out=None):
        """Per-(b, head) partial (m [log2 units], l, o unnormalised) over [kv_begin, kv_end).
        ``out`` = optional preallocated (m, l, o), e.g. views of one packed send buffer."""
        a = _Args(q)
        B = len(seq_ids) if not a.device else seq_ids.numel()
        n_head = (q.size if not a.device else q.numel()) // (B * self.head_dim)
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if out is not None:
            m, l, o = out
        elif a.device:
            import torch
            m = torch.empty((B, n_head), dtype=torch.float32, device=q.device)
            l = torch.empty((B, n_head), dtype=torch.float32, device=q.device)
            o = torch.empty((B, n_head, self.head_dim), dtype=torch.float32, device=q.device)
        else:
            m = np.empty((B, n_head), np.float32)
            l = np.empty((B, n_head), np.float32)
            o = np.empty((B, n_head, self.head_dim), np.float32)
        err = ErrBuf()
        check(lib().vxg_attn_cuda_q8_decode_partial(
            self.ctx.h, self.h, B, n_head, a.ptr(seq_ids, np.int32, (B,), "seq_ids"),
            a.ptr(kv_begin, np.int32, (B,), "kv_begin"), a.ptr(kv_end, np.int32, (B,), "kv_end"),
            a.ptr(q, np.float32, (B, n_head, self.head_dim), "q"), ctypes.c_float(scale),
            max_ctx, a.ptr(m, np.float32, writable=True), a.ptr(l, np.float32, writable=True),
            a.ptr(o, np.float32, writable=True), a.memkind, a.stream(stream), err.buf, err.cap),
            err)
        return m, l, o


class KvF32Pool:
    """Device fp32 K/V pools float[n_seq][cap][n_head_kv][head_dim] (KvCacheMode::Fp32, the
    reference's default cache mode; vxg_attn_cuda_kv_create_f32)."""

    def __init__(self, ctx: Context, n_seq: int, n_head_kv: int, head_dim: int, cap_tokens: int):
        self.ctx = ctx
        err = ErrBuf()
        self.h = lib().vxg_attn_cuda_kv_create_f32(ctx.h, n_seq, n_head_kv, head_dim, cap_tokens,
                                                   err.buf, err.cap)
        if not self.h:
            raise VxgError(-2, "vxg_attn_cuda_kv_create_f32 failed: " + err.text)
        self.n_seq, self.n_head_kv, self.head_dim = n_seq, n_head_kv, head_dim
        self.last_rc = 0

    close = KvQ8Pool.close
    __del__ = KvQ8Pool.__del__
    capacity = KvQ8Pool.capacity
    nbytes = KvQ8Pool.nbytes
    reserve = KvQ8Pool.reserve
    device_ptrs = KvQ8Pool.device_ptrs

    def import_rows(self, seq: int, tok_begin: int, k_rows, v_rows):
        """k/v_rows: float32 (n_tok, n_head_kv, head_dim), host."""
        k_rows = np.ascontiguousarray(k_rows, np.float32)
        v_rows = np.ascontiguousarray(v_rows, np.float32)
        n_tok = k_rows.size // (self.n_head_kv * self.head_dim)
        err = ErrBuf()
        check(lib().vxg_attn_cuda_kv_import(self.ctx.h, self.h, seq, tok_begin, n_tok,
                                            k_rows.ctypes.data_as(ctypes.c_void_p),
                                            v_rows.ctypes.data_as(ctypes.c_void_p), MEM_HOST,
                                            err.buf, err.cap), err)

    def export_rows(self, seq: int, tok_begin: int, n_tok: int):
        shape = (n_tok, self.n_head_kv, self.head_dim)
        k = np.empty(shape, np.float32)
        v = np.empty(shape, np.float32)
        err = ErrBuf()
        check(lib().vxg_attn_cuda_kv_export(self.ctx.h, self.h, seq, tok_begin, n_tok,
                                            k.ctypes.data_as(ctypes.c_void_p),
                                            v.ctypes.data_as(ctypes.c_void_p), MEM_HOST,
                                            err.buf, err.cap), err)
        return k, v

    def append(self, seq_ids, pos, k_new, v_new, n_tok: int = 1, stream=None) -> int:
        a = _Args(k_new)
        B = len(seq_ids) if not a.device else seq_ids.numel()
        kshape = (B, n_tok, self.n_head_kv, self.head_dim)
        err = ErrBuf()
        return check(lib().vxg_attn_cuda_f32_append(
            self.ctx.h, self.h, B, n_tok, a.ptr(seq_ids, np.int32, (B,), "seq_ids"),
            a.ptr(pos, np.int32, (B,), "pos"), a.ptr(k_new, np.float32, kshape, "k_new"),
            a.ptr(v_new, np.float32, kshape, "v_new"), a.memkind, a.stream(stream), err.buf,
            err.cap), err)

    def decode(self, seq_ids, pos, q, k_new=None, v_new=None, q_gate=None, scale=None,
               max_ctx: int = 0, out=None, stream=None):
        """Append (if k_new) then attend over [0, pos[b]]: returns out [B][n_head][head_dim]."""
        a = _Args(q)
        B = len(seq_ids) if not a.device else seq_ids.numel()
        n_head = (q.size if not a.device else q.numel()) // (B * self.head_dim)
        qshape = (B, n_head, self.head_dim)
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if out is None:
            if a.device:
                import torch
                out = torch.empty(qshape, dtype=torch.float32, device=q.device)
            else:
                out = np.empty(qshape, np.float32)
        kshape = (B, self.n_head_kv, self.head_dim)
        err = ErrBuf()
        self.last_rc = check(lib().vxg_attn_cuda_f32_decode(
            self.ctx.h, self.h, B, n_head, a.ptr(seq_ids, np.int32, (B,), "seq_ids"),
            a.ptr(pos, np.int32, (B,), "pos"), a.ptr(q, np.float32, qshape, "q"),
            a.ptr(k_new, np.float32, kshape, "k_new"), a.ptr(v_new, np.float32, kshape, "v_new"),
            a.ptr(q_gate, np.float32, qshape, "q_gate"), ctypes.c_float(scale), max_ctx,
            a.ptr(out, np.float32, qshape, "out", writable=True), a.memkind, a.stream(stream),
            err.buf, err.cap), err)
        return out


def step_full_gqa(ctx: Context, kv: KvF32Pool, seq: int, q_raw, k_cur, v_cur, q_norm, k_norm,
                  gated_q: bool, n_head: int, n_head_kv: int, head_dim: int, pos: int,
                  rope_dim: int, rope_freq_base: float, rope_neox: bool, eps: float,
                  att_cat) -> int:
    """Drop-in for step_full_gqa (llm_ops.rs:196-300), the fp32-KV operator, on host buffers:
    k_cur is overwritten with the normed / RoPE'd key and att_cat with the output."""
    a = _Args(q_raw)
    if a.device:
        raise TypeError("step_full_gqa takes host (numpy) buffers, as the reference does")
    err = ErrBuf()
    return check(lib().vxg_attn_cuda_step_full_gqa(
        ctx.h, kv.h, seq, a.ptr(q_raw, np.float32, name="q_raw"),
        a.ptr(k_cur, np.float32, (n_head_kv * head_dim,), "k_cur", writable=True),
        a.ptr(v_cur, np.float32, (n_head_kv * head_dim,), "v_cur"),
        a.ptr(q_norm, np.float32, (head_dim,), "q_norm"),
        a.ptr(k_norm, np.float32, (head_dim,), "k_norm"), int(bool(gated_q)), n_head, n_head_kv,
        head_dim, pos, rope_dim, ctypes.c_float(rope_freq_base), int(bool(rope_neox)),
        ctypes.c_float(eps), a.ptr(att_cat, np.float32, (n_head * head_dim,), "att_cat",
                                   writable=True), err.buf, err.cap), err)


def lse_combine(ctx: Context, m, l, o, gate=None, out=None, stream=None):
    """Merge partials m,l [P][R], o [P][R][hd] -> out [R][hd] (optional sigmoid gate)."""
    a = _Args(o)
    P, R, hd = tuple(o.shape)
    if out is None:
        if a.device:
            import torch
            out = torch.empty((R, hd), dtype=torch.float32, device=o.device)
        else:
            out = np.empty((R, hd), np.float32)
    err = ErrBuf()
    check(lib().vxg_attn_cuda_lse_combine(
        ctx.h, P, R, hd, a.ptr(m, np.float32, (P, R), "m"), a.ptr(l, np.float32, (P, R), "l"),
        a.ptr(o, np.float32, (P, R, hd), "o"), a.ptr(gate, np.float32, (R, hd), "gate"),
        a.ptr(out, np.float32, (R, hd), "out", writable=True), a.memkind, a.stream(stream),
        err.buf, err.cap), err)
    return out


def lse_combine_packed(ctx: Context, packed, n_parts: int, n_rows: int, head_dim: int,
                       gate=None, out=None, stream=None):
    """Merge packed partials packed[k] = [m (R) | l (R) | o (R*hd)] -> out [R][hd]."""
    a = _Args(packed)
    if out is None:
        if a.device:
            import torch
            out = torch.empty((n_rows, head_dim), dtype=torch.float32, device=packed.device)
        else:
            out = np.empty((n_rows, head_dim), np.float32)
    err = ErrBuf()
    check(lib().vxg_attn_cuda_lse_combine_packed(
        ctx.h, n_parts, n_rows, head_dim,
        a.ptr(packed, np.float32, (n_parts, n_rows * (head_dim + 2)), "packed"),
        a.ptr(gate, np.float32, (n_rows, head_dim), "gate"),
        a.ptr(out, np.float32, (n_rows, head_dim), "out", writable=True), a.memkind,
        a.stream(stream), err.buf, err.cap), err)
    return out


def deltanet_step(ctx: Context, q, k, v, beta_raw, alpha_raw, ssm_a, dt_bias, state,
                  q_scale=None, eps=1e-6, o=None, stream=None):
    """Gated-DeltaNet core step (llm_ops.rs:139-184), batched: q,k [B][n_kh][dk],
    v [B][n_vh][dv], beta_raw/alpha_raw [B][n_vh], state [B][n_vh][dv][dk] (in place).
    Returns o [B][n_vh][dv] (before the RMSNorm / SiLU(z) epilogue)."""
    a = _Args(state)
    B, n_vh, dv, dk = tuple(state.shape)
    n_kh = (q.size if not a.device else q.numel()) // (B * dk)
    if q_scale is None:
        q_scale = 1.0 / math.sqrt(dk)
    if o is None:
        if a.device:
            import torch
            o = torch.empty((B, n_vh, dv), dtype=torch.float32, device=state.device)
        else:
            o = np.empty((B, n_vh, dv), np.float32)
    err = ErrBuf()
    rc = check(lib().vxg_attn_cuda_deltanet_step(
        ctx.h, B, n_kh, n_vh, dk, dv, a.ptr(q, np.float32, (B, n_kh, dk), "q"),
        a.ptr(k, np.float32, (B, n_kh, dk), "k"), a.ptr(v, np.float32, (B, n_vh, dv), "v"),
        a.ptr(beta_raw, np.float32, (B, n_vh), "beta_raw"),
        a.ptr(alpha_raw, np.float32, (B, n_vh), "alpha_raw"),
        a.ptr(ssm_a, np.float32, (n_vh,), "ssm_a"), a.ptr(dt_bias, np.float32, (n_vh,), "dt_bias"),
        ctypes.c_float(q_scale), ctypes.c_float(eps),
        a.ptr(state, np.float32, (B, n_vh, dv, dk), "state", writable=True),
        a.ptr(o, np.float32, (B, n_vh, dv), "o", writable=True), a.memkind, a.stream(stream),
        err.buf, err.cap), err)
    ctx.last_rc = rc
    return o


def step_full_gqa_q8(ctx: Context, kv: KvQ8Pool, seq: int, q_raw, k_cur, v_cur, q_norm, k_norm,
                     gated_q: bool, n_head: int, n_head_kv: int, head_dim: int, pos: int,
                     rope_pos: int, rope_dim: int, rope_freq_base: float, rope_neox: bool,
                     eps: float, attn_out) -> int:
    """Drop-in for step_full_gqa_q8 (llm_prefill.rs:259-278) on host (numpy f32) buffers:
    k_cur is overwritten with the normed/RoPE'd key and attn_out with the attention output,
    exactly as the reference mutates its arguments; the token is appended to ``kv`` sequence
    ``seq`` at ``pos``."""
    a = _Args(q_raw)
    if a.device:
        raise TypeError("step_full_gqa_q8 takes host (numpy) buffers, as the reference does")
    err = ErrBuf()
    return check(lib().vxg_attn_cuda_step_full_gqa_q8(
        ctx.h, kv.h, seq, a.ptr(q_raw, np.float32, name="q_raw"),
        a.ptr(k_cur, np.float32, (n_head_kv * head_dim,), "k_cur", writable=True),
        a.ptr(v_cur, np.float32, (n_head_kv * head_dim,), "v_cur"),
        a.ptr(q_norm, np.float32, (head_dim,), "q_norm"),
        a.ptr(k_norm, np.float32, (head_dim,), "k_norm"), int(bool(gated_q)), n_head, n_head_kv,
        head_dim, pos, rope_pos, rope_dim, ctypes.c_float(rope_freq_base), int(bool(rope_neox)),
        ctypes.c_float(eps), a.ptr(attn_out, np.float32, (n_head * head_dim,), "attn_out",
                                   writable=True), err.buf, err.cap), err)


def deltanet_prefill(ctx: Context, q, k, v, beta_raw, alpha_raw, ssm_a, dt_bias, state,
                     q_scale=None, eps=1e-6, o=None, stream=None):
    """The DeltaNet recurrence over T tokens per sequence (the reference prefill applies the
    step token by token, llm_prefill.rs:470-480): q,k [B][T][n_kh][dk], v [B][T][n_vh][dv],
    beta_raw/alpha_raw [B][T][n_vh], state [B][n_vh][dv][dk] in place.  Returns o
    [B][T][n_vh][dv]."""
    a = _Args(state)
    B, n_vh, dv, dk = tuple(state.shape)
    T = (v.size if not a.device else v.numel()) // (B * n_vh * dv)
    n_kh = (q.size if not a.device else q.numel()) // (B * T * dk)
    if q_scale is None:
        q_scale = 1.0 / math.sqrt(dk)
    if o is None:
        if a.device:
            import torch
            o = torch.empty((B, T, n_vh, dv), dtype=torch.float32, device=state.device)
        else:
            o = np.empty((B, T, n_vh, dv), np.float32)
    err = ErrBuf()
    rc = check(lib().vxg_attn_cuda_deltanet_prefill(
        ctx.h, B, T, n_kh, n_vh, dk, dv, a.ptr(q, np.float32, (B, T, n_kh, dk), "q"),
        a.ptr(k, np.float32, (B, T, n_kh, dk), "k"), a.ptr(v, np.float32, (B, T, n_vh, dv), "v"),
        a.ptr(beta_raw, np.float32, (B, T, n_vh), "beta_raw"),
        a.ptr(alpha_raw, np.float32, (B, T, n_vh), "alpha_raw"),
        a.ptr(ssm_a, np.float32, (n_vh,), "ssm_a"), a.ptr(dt_bias, np.float32, (n_vh,), "dt_bias"),
        ctypes.c_float(q_scale), ctypes.c_float(eps),
        a.ptr(state, np.float32, (B, n_vh, dv, dk), "state", writable=True),
        a.ptr(o, np.float32, (B, T, n_vh, dv), "o", writable=True), a.memkind, a.stream(stream),
        err.buf, err.cap), err)
    ctx.last_rc = rc
    return o


def step_deltanet_recurrent(ctx: Context, qkv_mixed, z, alpha_raw, beta_raw, ssm_conv1d, ssm_a,
                            ssm_dt_bias, ssm_norm, conv_state, ssm_state, n_kh, n_vh, dk, dv,
                            k_sz, eps, y_concat=None, stream=None):
    """Drop-in for step_deltanet_recurrent (llm_ops.rs:103-121), batched: qkv_mixed [B][conv_ch],
    z [B][n_vh*dv], alpha_raw/beta_raw [B][n_vh]; conv_state [B][k_sz-1][conv_ch] and ssm_state
    [B][n_vh][dv][dk] are updated in place; returns y_concat [B][n_vh*dv]."""
    a = _Args(ssm_state)
    B = ssm_state.shape[0]
    conv_ch = 2 * n_kh * dk + n_vh * dv
    if y_concat is None:
        if a.device:
            import torch
            y_concat = torch.empty((B, n_vh * dv), dtype=torch.float32, device=ssm_state.device)
        else:
            y_concat = np.empty((B, n_vh * dv), np.float32)
    err = ErrBuf()
    rc = check(lib().vxg_attn_cuda_step_deltanet_recurrent(
        ctx.h, B, a.ptr(qkv_mixed, np.float32, (B, conv_ch), "qkv_mixed"), conv_ch,
        a.ptr(z, np.float32, (B, n_vh * dv), "z"), a.ptr(alpha_raw, np.float32, (B, n_vh), "alpha_raw"),
        a.ptr(beta_raw, np.float32, (B, n_vh), "beta_raw"),
        a.ptr(ssm_conv1d, np.float32, (conv_ch, k_sz), "ssm_conv1d"),
        a.ptr(ssm_a, np.float32, (n_vh,), "ssm_a"), a.ptr(ssm_dt_bias, np.float32, (n_vh,), "ssm_dt_bias"),
        a.ptr(ssm_norm, np.float32, (dv,), "ssm_norm"),
        a.ptr(conv_state, np.float32, (B, k_sz - 1, conv_ch), "conv_state", writable=True),
        a.ptr(ssm_state, np.float32, (B, n_vh, dv, dk), "ssm_state", writable=True),
        n_kh, n_vh, dk, dv, k_sz, ctypes.c_float(eps),
        a.ptr(y_concat, np.float32, (B, n_vh * dv), "y_concat", writable=True), a.memkind,
        a.stream(stream), err.buf, err.cap), err)
    ctx.last_rc = rc
    return y_concat
