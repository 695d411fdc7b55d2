"""Batch x KV-head sharding of the attention path over the GPUs of one node.

Every (batch row, KV head) pair -- with the query heads of its group -- is an
independent attention problem for prefill, backward and decode, so ranks own
contiguous blocks of pairs and never reduce.  The only collective is the
gather of each rank's outputs to the caller's rank: NCCL over NVLink through
``torch.distributed`` (``gather_to_root``), or copy-engine writes into a
buffer of the root rank (``RootWindow``), which take no SMs from the kernels
that run meanwhile.  tensorsmith itself has no such path: its only
multi-process code is a host-staged TCP all-reduce for data parallelism
(src/tensorsmith/distributed.py:22-218).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class ShardPlan:
    """Contiguous block of (batch, kv_head) pairs owned by ``rank``."""

    batch: int
    kv_heads: int
    world_size: int
    rank: int

    def __post_init__(self):
        if self.world_size <= 0 or not 0 <= self.rank < self.world_size:
            raise ValueError("rank must be in [0, world_size)")
        if self.batch <= 0 or self.kv_heads <= 0:
            raise ValueError("batch and kv_heads must be positive")

    @property
    def pairs(self) -> int:
        return self.batch * self.kv_heads

    def bounds(self, rank: int | None = None) -> tuple[int, int]:
        r = self.rank if rank is None else rank
        return r * self.pairs // self.world_size, (r + 1) * self.pairs // self.world_size

    @property
    def start(self) -> int:
        return self.bounds()[0]

    @property
    def stop(self) -> int:
        return self.bounds()[1]

    @property
    def size(self) -> int:
        return self.stop - self.start

    @property
    def even(self) -> bool:
        return self.pairs % self.world_size == 0

    def pair_ids(self) -> list[tuple[int, int]]:
        return [divmod(i, self.kv_heads) for i in range(self.start, self.stop)]


def shard_view(x: torch.Tensor, plan: ShardPlan, group: int = 1) -> torch.Tensor:
    """This rank's pairs of a [B, H, T, C] tensor, as a view (no copy).

    ``group`` is the number of heads per pair (query heads per KV head for
    queries/outputs, 1 for keys/values).  When the shard covers whole batch
    rows the result is ``x[b0:b1]`` (any layout, BTHD-permuted included);
    otherwise the (B, H) dims are flattened into a [1, pairs*group, T, C] view,
    which needs them to be flattenable without a copy.
    """
    b, h, t, c = x.shape
    if b != plan.batch or h != plan.kv_heads * group:
        raise ValueError("tensor does not match the shard plan")
    if plan.start % plan.kv_heads == 0 and plan.stop % plan.kv_heads == 0:
        return x[plan.start // plan.kv_heads : plan.stop // plan.kv_heads]
    if x.stride(0) != h * x.stride(1):
        raise ValueError("shard splits a batch row of a layout whose (B, H) dims do not flatten")
    flat = x.as_strided((1, b * h, t, c), (b * h * x.stride(1), x.stride(1), x.stride(2), x.stride(3)))
    return flat[:, plan.start * group : plan.stop * group]


def gather_to_root(local: torch.Tensor, plan: ShardPlan, out=None, root: int = 0, group=None,
                   async_op: bool = False):
    """Gather every rank's shard into ``out`` on ``root``.

    ``out`` is the full tensor (the ranks' shards stacked along dim 0 in rank
    order, contiguous) or a list of one contiguous tensor per rank shaped like
    ``local``, which lets a caller gather one block of its pairs at a time into
    strided places of a larger buffer.  One NCCL gather (grouped send/recv) per
    call; other ranks return None.  Shards must be equal-sized (the plan is even).

    With ``async_op=True`` the call returns the collective's work handle (None
    on a single rank) instead of ``out``.  The gather runs on the process
    group's stream after the work already queued on the current stream; the
    current stream goes on without it (the next block's kernels overlap the
    transfer) until ``work.wait()`` orders it after the gather.  Because only
    the handle comes back, an asynchronous call on ``root`` must be given
    ``out`` (a ValueError otherwise): a buffer allocated here could not reach
    the caller."""
    if async_op and out is None and (plan.world_size == 1 or dist.get_rank(group) == root):
        raise ValueError("an asynchronous gather needs `out` on the root rank (only the work handle is returned)")
    if plan.world_size == 1:
        target = out[0] if isinstance(out, (list, tuple)) else out
        if target is not None:
            target.copy_(local)
        if async_op:
            return None
        return target if target is not None else local
    if not plan.even:
        raise ValueError("gather needs an even shard plan (pairs divisible by world size)")
    rank = dist.get_rank(group)
    if rank != root:
        work = dist.gather(local.contiguous(), None, dst=root, group=group, async_op=async_op)
        return work if async_op else None
    if isinstance(out, (list, tuple)):
        if len(out) != plan.world_size or any(t.shape != local.shape or not t.is_contiguous() for t in out):
            raise ValueError("gather targets must be one contiguous tensor per rank shaped like the shard")
        work = dist.gather(local.contiguous(), list(out), dst=root, group=group, async_op=async_op)
        return work if async_op else out
    if out is None:
        shape = list(local.shape)
        shape[0] *= plan.world_size
        out = torch.empty(shape, dtype=local.dtype, device=local.device)
    if not out.is_contiguous():
        raise ValueError("gather target must be contiguous")
    chunks = [c.view(local.shape) for c in out.reshape((plan.world_size, -1) + tuple(local.shape[2:])).unbind(0)]
    contiguous = all(c.is_contiguous() for c in chunks)
    if async_op and not contiguous:
        raise ValueError("an asynchronous gather needs targets that are contiguous per rank")
    targets = chunks if contiguous else [torch.empty_like(local) for _ in chunks]
    work = dist.gather(local.contiguous(), targets, dst=root, group=group, async_op=async_op)
    if async_op:
        return work
    if not contiguous:
        for c, t in zip(chunks, targets):
            c.copy_(t)
    return out


class RootWindow:
    """A contiguous buffer on the root rank that every rank writes into with
    copy-engine transfers over NVLink (CUDA IPC), so a gather overlaps the
    compute kernels without taking SMs from them (an NCCL gather runs kernels
    that occupy whole SMs while it moves data).

    Collective: every rank of ``group`` constructs it with the same ``shape``
    and ``dtype``; the root allocates the buffer (``buffer`` on the root,
    None elsewhere) and exports it, the other ranks map it.  ``ok`` is False on
    every rank when any rank could not map it (no peer access between the
    GPUs, or an allocation that cannot be exported); callers then keep their
    NCCL path.  ``put(src, offset)`` queues one ``cudaMemcpyAsync`` of a
    contiguous tensor to byte ``offset`` of the buffer on ``stream``; the
    root's buffer holds the data once the writer's stream passed the copy,
    which a later collective on that stream (``done``) makes known to the
    root.  ``close()`` unmaps it (collective).
    """

    def __init__(self, shape, dtype, device, group=None, root: int = 0):
        self.group, self.root = group, root
        self.rank = dist.get_rank(group)
        self.nbytes = int(torch.Size(shape).numel()) * torch.empty((), dtype=dtype).element_size()
        self.buffer = None
        self._peer_base = None
        self._dst = 0
        payload = [None]
        if self.rank == root:
            self.buffer = torch.empty(shape, dtype=dtype, device=device)
            payload[0] = _export(self.buffer)
            if payload[0] is not None:
                self._dst = self.buffer.data_ptr()
        src = dist.get_global_rank(group, root) if group is not None else root
        dist.broadcast_object_list(payload, src=src, group=group)
        mine = payload[0] is not None
        if mine and self.rank != root:
            handle, offset = payload[0]
            self._peer_base = _open(handle)
            mine = self._peer_base is not None
            if mine:
                self._dst = self._peer_base + offset
        flags = [None] * dist.get_world_size(group)
        dist.all_gather_object(flags, mine, group=group)
        self.ok = all(flags)

    def put(self, src: torch.Tensor, offset: int, stream: torch.cuda.Stream) -> None:
        if not self.ok:
            raise RuntimeError("RootWindow is not mapped on every rank")
        if not src.is_contiguous():
            raise ValueError("put needs a contiguous source")
        nbytes = src.numel() * src.element_size()
        if offset < 0 or offset + nbytes > self.nbytes:
            raise ValueError("put outside the window")
        from cuda.bindings import runtime as rt

        (err,) = rt.cudaMemcpyAsync(self._dst + offset, src.data_ptr(), nbytes,
                                    rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice, stream.cuda_stream)
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"cudaMemcpyAsync into the root window failed: {err}")

    def done(self, device) -> None:
        """On the current stream of every rank: after it, the root's stream sees
        every copy that the ranks' current streams ordered before this call."""
        flag = torch.zeros(1, device=device)
        dist.all_reduce(flag, group=self.group)

    def close(self) -> None:
        if self._peer_base is not None:
            from cuda.bindings import runtime as rt

            torch.cuda.synchronize()
            rt.cudaIpcCloseMemHandle(self._peer_base)
            self._peer_base = None
        dist.barrier(group=self.group)
        self.buffer = None


def _export(t: torch.Tensor):
    """(IPC handle bytes, offset of ``t`` in its allocation), or None when the
    tensor cannot be exported (host memory, no CUDA driver, no cuda-python)."""
    if not t.is_cuda:
        return None
    try:
        from cuda.bindings import driver as drv
        from cuda.bindings import runtime as rt

        err, base, _ = drv.cuMemGetAddressRange(drv.CUdeviceptr(t.data_ptr()))
        if err != drv.CUresult.CUDA_SUCCESS:
            return None
        err, handle = rt.cudaIpcGetMemHandle(int(base))
        if err != rt.cudaError_t.cudaSuccess:
            return None
        return bytes(handle.reserved), t.data_ptr() - int(base)
    except (ImportError, RuntimeError):
        return None


def _open(handle_bytes: bytes):
    """Device address of the root's mapped allocation, or None."""
    try:
        from cuda.bindings import runtime as rt

        handle = rt.cudaIpcMemHandle_t()
        handle.reserved = handle_bytes
        err, ptr = rt.cudaIpcOpenMemHandle(handle, rt.cudaIpcMemLazyEnablePeerAccess)
        if err != rt.cudaError_t.cudaSuccess:
            return None
        return int(ptr)
    except (ImportError, RuntimeError):
        return None
