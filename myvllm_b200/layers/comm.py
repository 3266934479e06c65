"""The tensor-parallel all-reduce of the row-parallel output projections.

The reference sums the partial outputs of ``RowParallelLinear`` with
``dist.all_reduce`` (``m/layers/linear.py:159-164``).  ``all_reduce`` below does the
same through NCCL unless a :class:`OneShotAllReduce` is enabled for the group: then
messages that fit its buffer (decode-size activations) are summed by the library's
one-shot kernel over NVLink peer memory (``mvb_allreduce_oneshot``), and larger ones
still go to NCCL.  With a :class:`FusedLinearAllReduce` enabled, ``RowParallelLinear``
runs its projection and the all-reduce as one kernel (``mvb_linear_allreduce``) for decode
batches.  Every rank of the group must make the same sequence of calls.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from .. import _lib


class _PeerBuffers:
    """One device buffer per rank of ``group``, mapped into every other rank's process
    through CUDA IPC; a collective to construct (every rank of the group calls it) and to
    :meth:`close`."""

    name = "peer buffers"

    def _open(self, group, buf_bytes: int):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if not 2 <= self.world <= _lib.AR_MAX_RANKS:
            raise ValueError(f"{self.name}: {self.world} ranks (2..{_lib.AR_MAX_RANKS} supported)")
        lib = _lib.load()
        self.buf_bytes = int(buf_bytes)
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.check(self.name, lib.mvb_ipc_alloc(self.buf_bytes, ctypes.byref(ptr), handle))
        self._own = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened = []
        peers = _lib.MvbAllReducePeers()
        peers.world, peers.rank, peers.buf_bytes = self.world, self.rank, self.buf_bytes
        for r, h in enumerate(handles):
            if r == self.rank:
                peers.bufs[r] = self._own
                continue
            p = ctypes.c_void_p()
            _lib.check(self.name, lib.mvb_ipc_open(h, ctypes.byref(p)))
            self._opened.append(p.value)
            peers.bufs[r] = p.value
        self.peers = peers
        # every rank has mapped every buffer before any kernel may store into a peer's flags
        dist.barrier(group=group)

    def check(self) -> None:
        """Raises if a launch since the last check gave up waiting for a peer.  Such a launch
        leaves a defined but wrong result and sets the library's device error word; reading
        the word synchronises the device, so call this at a point that already waits (end of
        a step, before :meth:`close`)."""
        status = _lib.device_status()
        if status != 0:
            raise RuntimeError(f"{self.name}: a peer did not answer within the wait limit "
                               f"(device status {status}); outputs since the last check are not the sums")

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's; collective (after the last use
        on every rank).  Raises, after releasing the buffers, if a launch gave up on a peer."""
        if self._own is None:
            return
        torch.cuda.synchronize()
        status = _lib.device_status()
        dist.barrier(group=self.group)
        lib = _lib.load()
        for p in self._opened:
            lib.mvb_ipc_close(p)
        dist.barrier(group=self.group)
        lib.mvb_ipc_free(self._own)
        self._own, self._opened = None, []
        if status != 0:
            raise RuntimeError(f"{self.name}: a peer did not answer within the wait limit "
                               f"(device status {status}); some outputs were not the sums")


class OneShotAllReduce(_PeerBuffers):
    """The one-shot all-reduce (``mvb_allreduce_oneshot``) for messages up to ``max_bytes``."""

    name = "OneShotAllReduce"

    def __init__(self, group=None, max_bytes: int = 4 << 20):
        self.max_bytes = int(max_bytes)
        self._open(group, int(_lib.load().mvb_allreduce_buffer_bytes(self.max_bytes)))

    def eligible(self, t: torch.Tensor) -> bool:
        nbytes = t.numel() * t.element_size()
        return (t.is_cuda and t.dtype in (torch.bfloat16, torch.float16) and t.is_contiguous()
                and nbytes <= self.max_bytes and nbytes % 16 == 0 and t.data_ptr() % 16 == 0)

    def __call__(self, t: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(t)
        _lib.call("allreduce_oneshot", "mvb_allreduce_oneshot", ctypes.byref(self.peers), _lib.desc(t),
                  _lib.desc(out), _lib.stream_of(t))
        return out


class FusedLinearAllReduce(_PeerBuffers):
    """Row-parallel projection fused with its all-reduce (``mvb_linear_allreduce``): one
    kernel computes this rank's x W^T on the tensor cores and sums the ranks' fp32 partial
    tiles over NVLink peer memory.  Decode-size inputs (at most 128 rows)."""

    name = "FusedLinearAllReduce"

    def __init__(self, group=None):
        self._open(group, int(_lib.load().mvb_linear_allreduce_buffer_bytes()))

    def eligible(self, x: torch.Tensor, w: torch.Tensor) -> bool:
        n, k = w.shape
        if not (x.is_cuda and x.dim() == 2 and x.dtype in (torch.bfloat16, torch.float16) and w.dtype == x.dtype):
            return False
        if x.shape[0] > 128 or x.shape[1] != k or n % 64 or 128 % (n // 64):
            return False
        splits = 128 // (n // 64)
        return (k % (64 * splits) == 0 and x.stride(1) == 1 and w.stride(1) == 1 and x.stride(0) % 8 == 0
                and w.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0)

    def __call__(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
        _lib.call("linear_allreduce", "mvb_linear_allreduce", ctypes.byref(self.peers), _lib.desc(x), _lib.desc(w),
                  _lib.desc(out), _lib.stream_of(x))
        return out


_oneshot: dict = {}


def enable_oneshot(group=None, max_bytes: int = 4 << 20) -> OneShotAllReduce:
    """Collective: routes this group's eligible all-reduces through the one-shot kernel."""
    ar = OneShotAllReduce(group, max_bytes)
    _oneshot[group] = ar
    return ar


def disable_oneshot(group=None) -> None:
    """Collective: back to NCCL for this group; frees the buffers."""
    ar = _oneshot.pop(group, None)
    if ar is not None:
        ar.close()


_fused: dict = {}


def enable_fused_linear(group=None) -> FusedLinearAllReduce:
    """Collective: RowParallelLinear layers of this group run their projection and all-reduce
    as one kernel where the input qualifies (decode batches)."""
    f = FusedLinearAllReduce(group)
    _fused[group] = f
    return f


def disable_fused_linear(group=None) -> None:
    """Collective: back to a GEMM followed by an all-reduce; frees the buffers."""
    f = _fused.pop(group, None)
    if f is not None:
        f.close()


def fused_linear(x: torch.Tensor, w: torch.Tensor, group=None):
    """sum over ranks of x W^T through the fused kernel, or None when it is not enabled for
    ``group`` or the shapes do not qualify."""
    f = _fused.get(group)
    if f is None or not f.eligible(x, w):
        return None
    return f(x, w)


def all_gather_block(t: torch.Tensor, block: int) -> torch.Tensor:
    """``[block, *t.shape]``: ``t`` from each rank of this rank's block of ``block``
    consecutive ranks (NCCL all-gather over the world; the blocks are small statistics)."""
    rank, world = dist.get_rank(), dist.get_world_size()
    out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t.contiguous())
    first = (rank // block) * block
    return out[first:first + block]


def all_reduce(t: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of ``t`` over the ranks of ``group``; returns the result (``t`` itself when NCCL
    reduces it in place)."""
    ar = _oneshot.get(group)
    if ar is not None and ar.eligible(t):
        return ar(t)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t
