"""One-shot all-reduce over NVLink peer memory for small bf16 messages.

The row-parallel layers sum [M, hidden] bf16 partials across tensor-parallel
ranks twice per layer; at decode sizes that is latency-bound.  ``CustomAllReduce``
runs the library's one-shot kernel (``w4a8_ar_*``: every rank reads every peer's
message once over CUDA IPC mappings and sums in fp32 in rank order, so all
ranks hold identical bits) for messages up to ``max_bytes`` and hands anything
else to NCCL -- the role of the reference's peer-read all-reduce
(npu_ops/python/peer_allreduce.py, npu_ops/kernel/peer_allreduce_f32.cpp:127-270),
which also loses to the library collective on large messages.

Every rank must call it in the same order with the same shapes (as with any
collective).  A wait for a peer is bounded in the kernel (1 s): ``check()``
raises if one ran out, instead of the GPU hanging.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch

from . import _lib

DEFAULT_MAX_BYTES = 1 << 20          # M <= 64 at hidden 5120 (640 KB) fits


def eligible(numel: int, dtype: torch.dtype, max_bytes: int) -> bool:
    """Whether a tensor takes the one-shot path (else the NCCL fallback).

    Only values every rank shares decide (the message's element count and
    dtype, and the group's byte limit): ranks that chose differently would
    wait on each other in two different collectives.  A tensor's own layout
    (strides, address) may differ between ranks, so it never decides the path;
    a tensor the kernel cannot take as it is goes through a staging buffer."""
    return dtype == torch.bfloat16 and numel > 0 and numel % 8 == 0 and numel * 2 <= max_bytes


def direct(t: torch.Tensor) -> bool:
    """Whether the kernel can reduce ``t`` in place (dense and 16-byte aligned)."""
    return t.is_contiguous() and t.data_ptr() % 16 == 0


class _Handle:
    def __init__(self, rank: int, world: int, max_bytes: int):
        L = _lib.lib()
        h = ctypes.c_void_p()
        _lib.check(L.w4a8_ar_create(rank, world, max_bytes, ctypes.byref(h)), "w4a8_ar_create")
        self.h = h
        self.rank, self.world, self.max_bytes = rank, world, max_bytes

    def ipc_handle(self) -> bytes:
        L = _lib.lib()
        buf = ctypes.create_string_buffer(L.w4a8_ar_ipc_handle_size())
        _lib.check(L.w4a8_ar_ipc_handle(self.h, ctypes.cast(buf, ctypes.c_void_p)), "w4a8_ar_ipc_handle")
        return buf.raw

    def open_peers(self, handles: List[bytes]) -> None:
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        _lib.check(_lib.lib().w4a8_ar_open_peers(self.h, ctypes.cast(buf, ctypes.c_void_p)), "w4a8_ar_open_peers")

    def open_local(self, peers: List["_Handle"]) -> None:
        arr = (ctypes.c_void_p * self.world)(*[p.h.value for p in peers])
        _lib.check(_lib.lib().w4a8_ar_open_local(self.h, ctypes.cast(arr, ctypes.c_void_p)), "w4a8_ar_open_local")

    def allreduce(self, inp: torch.Tensor, out: torch.Tensor) -> None:
        rc = _lib.lib().w4a8_ar_allreduce_bf16(self.h, inp.data_ptr(), out.data_ptr(), inp.numel(),
                                               torch.cuda.current_stream(inp.device).cuda_stream)
        _lib.check(rc, "w4a8_ar_allreduce_bf16")

    def status(self, reset: bool = True) -> int:
        return _lib.lib().w4a8_ar_status(self.h, 1 if reset else 0)

    def destroy(self) -> None:
        if self.h is not None and self.h.value:
            _lib.lib().w4a8_ar_destroy(self.h)
        self.h = None


class CustomAllReduce:
    """In-place bf16 sum over the ranks of ``group`` (one process per GPU).

    ``ar(t)`` reduces ``t`` in place: the one-shot kernel when ``t`` fits
    ``max_bytes``, ``torch.distributed.all_reduce`` otherwise."""

    def __init__(self, group=None, max_bytes: int = DEFAULT_MAX_BYTES, device: Optional[torch.device] = None):
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_bytes = max_bytes
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        with torch.cuda.device(self.device):
            self._h = _Handle(self.rank, self.world, max_bytes)
            handles: List[Optional[bytes]] = [None] * self.world
            dist.all_gather_object(handles, self._h.ipc_handle(), group=group)
            self._h.open_peers(handles)
        dist.barrier(group=group)
        # staging for eligible tensors the kernel cannot take in place (a view
        # with strides, or an address off the 16-byte grid); made here so that
        # calls inside CUDA graph capture allocate nothing
        self._stage = torch.empty(max_bytes // 2, dtype=torch.bfloat16, device=self.device)
        self.calls_custom = 0
        self.calls_staged = 0
        self.calls_fallback = 0
        self.calls_fused = 0

    def fits(self, t: torch.Tensor) -> bool:
        return eligible(t.numel(), t.dtype, self.max_bytes)

    def __call__(self, t: torch.Tensor) -> None:
        if self.world == 1:
            return
        if self.fits(t):
            if direct(t):
                self._h.allreduce(t, t)
            else:
                st = self._stage[:t.numel()]
                st.view(t.shape).copy_(t)
                self._h.allreduce(st, st)
                t.copy_(st.view(t.shape))
                self.calls_staged += 1
            self.calls_custom += 1
        else:
            import torch.distributed as dist
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            self.calls_fallback += 1

    def linear_prepared(self, x: torch.Tensor, pw, act: Optional[str] = None) -> torch.Tensor:
        """A row-parallel linear and its all-reduce: the sum over the ranks of
        ``ops.linear_prepared(x, pw, act=act)``, every rank calling with its own
        K shard (``w4a8_linear_prepared_allreduce``: the GEMM stores its output
        tiles straight into every rank's receive slot, one kernel then sums).
        Messages larger than ``max_bytes`` take the linear followed by NCCL.
        The same bits as the linear followed by ``self(y)``."""
        from . import ops
        K = pw.K
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        M, N = x2.shape[0], pw.N
        if self.world == 1 or not eligible(M * N, torch.bfloat16, self.max_bytes) or M == 0:
            y = ops.linear_prepared(x2, pw, act=act)
            self(y)
            return y.reshape(*x.shape[:-1], N)
        want = 2 * K if act == "swiglu" else K
        if x2.dtype != torch.bfloat16 or x2.shape[1] != want:
            raise RuntimeError(f"row-parallel linear: x must be bf16 [M, {want}]")
        y = torch.empty((M, N), dtype=torch.bfloat16, device=x2.device)
        ws, wsb = ops.workspace(ops._ws_bytes(M, N, K, pw.group_size), x2.device)
        rc = _lib.lib().w4a8_linear_prepared_allreduce(
            x2.data_ptr(), M, K, x2.stride(0), N, pw.group_size, pw.ptr(), pw.ws_dtype, 1 if pw.has_zero else 0,
            _lib.ACT_SWIGLU if act == "swiglu" else _lib.ACT_NONE, y.data_ptr(), ws, wsb, self._h.h,
            torch.cuda.current_stream(x2.device).cuda_stream)
        _lib.check(rc, "w4a8_linear_prepared_allreduce")
        self.calls_fused += 1
        return y.reshape(*x.shape[:-1], N)

    def check(self) -> None:
        """Raise if a kernel wait for a peer ran out (synchronises the device)."""
        torch.cuda.synchronize(self.device)
        rc = self._h.status(reset=True)
        _lib.check(rc, "custom all-reduce")

    def close(self) -> None:
        """Free the buffer once every rank's kernels are done with it (a peer
        may still be reading this rank's slots): synchronise, then a barrier."""
        if self._h is not None:
            import torch.distributed as dist
            torch.cuda.synchronize(self.device)
            if self.world > 1:
                dist.barrier(group=self.group)
            self._h.destroy()
            self._h = None
