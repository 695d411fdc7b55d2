"""Minimal mirror of tensorsmith's reverse-mode tape for CUDA arrays.

The engine's attention op records exactly one node per call through
``Tensor._from_op(data, parents, backward, op)``, the interface of
tensorsmith's src/tensorsmith/tensor.py:121-135; ``backward`` runs a reverse
sweep with that tape's contract (tensor.py:247-267, :662-724: contributions
summed per tensor and cast to its dtype, one VJP call per node), implemented
here by consumer counting.  This mirror carries torch CUDA arrays in
``_data`` so the engine can be driven and tested without CuPy; inside
tensorsmith itself ``tensorsmith_b200.interop.attention_node`` hands the same
kind of node to the library's own ``Tensor._from_op``.
"""

from __future__ import annotations

from contextlib import ContextDecorator
from contextvars import ContextVar
from dataclasses import dataclass

import numpy as np
import torch

_grad_enabled: ContextVar[bool] = ContextVar("tensorsmith_b200_grad_enabled", default=True)


class no_grad(ContextDecorator):
    """Disable graph recording in a block (thread/task local), as tensor.py:22-31."""

    def __enter__(self):
        self._token = _grad_enabled.set(False)
        return self

    def __exit__(self, *exc):
        _grad_enabled.reset(self._token)
        return False


class enable_grad(ContextDecorator):
    def __enter__(self):
        self._token = _grad_enabled.set(True)
        return self

    def __exit__(self, *exc):
        _grad_enabled.reset(self._token)
        return False


def is_grad_enabled() -> bool:
    return _grad_enabled.get()


@dataclass(frozen=True)
class Device:
    """``cpu`` or ``cuda:N`` (the subset of device.py:27-48 the engine needs)."""

    type: str = "cpu"
    index: int | None = None

    def __str__(self) -> str:
        return f"cuda:{self.index}" if self.type == "cuda" else self.type


def as_device(value) -> Device:
    if isinstance(value, Device):
        return value
    if value is None:
        return Device("cpu")
    dev = torch.device(value)
    if dev.type == "cuda":
        return Device("cuda", 0 if dev.index is None else dev.index)
    if dev.type == "cpu":
        return Device("cpu")
    raise ValueError(f"unknown device {value!r}; expected cpu or cuda")


def _torch_device(dev: Device) -> torch.device:
    return torch.device("cuda", dev.index) if dev.type == "cuda" else torch.device("cpu")


_NP_TO_TORCH = {
    np.dtype(np.float32): torch.float32,
    np.dtype(np.float64): torch.float64,
    np.dtype(np.float16): torch.float16,
    np.dtype(np.int64): torch.int64,
    np.dtype(np.int32): torch.int32,
    np.dtype(np.bool_): torch.bool,
}


def _as_torch(data, dtype=None) -> torch.Tensor:
    if isinstance(data, torch.Tensor):
        return data
    arr = np.asarray(data)
    if arr.dtype.name == "bfloat16":
        return torch.from_numpy(arr.view(np.uint16).astype(np.int32) << 16).view(torch.float32).to(
            torch.bfloat16
        )
    if arr.dtype.kind == "f" and dtype is None and arr.dtype not in _NP_TO_TORCH:
        arr = arr.astype(np.float32)
    return torch.from_numpy(np.ascontiguousarray(arr))


class Tensor:
    """An array on a device that can take part in a reverse-mode graph."""

    def __init__(self, data, *, requires_grad: bool = False, device=None, dtype=None):
        if isinstance(data, Tensor):
            data = data._data
        raw = _as_torch(data, dtype)
        target = as_device(device) if device is not None else as_device(raw.device)
        raw = raw.to(device=_torch_device(target), dtype=dtype if dtype is not None else raw.dtype)
        if requires_grad and not raw.is_floating_point():
            raise TypeError("only floating-point tensors can require gradients")
        self._data = raw
        self.requires_grad = bool(requires_grad)
        self.device = target
        self._grad = None
        self._parents: tuple = ()
        self._backward = None
        self._op = ""
        self._graph_freed = False

    @classmethod
    def _from_op(cls, data, parents, backward, op: str) -> "Tensor":
        obj = cls.__new__(cls)
        obj._data = data
        obj.device = parents[0].device
        obj.requires_grad = is_grad_enabled() and any(p.requires_grad for p in parents)
        obj._grad = None
        obj._parents = tuple(parents) if obj.requires_grad else ()
        obj._backward = backward if obj.requires_grad else None
        obj._op = op if obj.requires_grad else ""
        obj._graph_freed = False
        return obj

    # -- array protocol ----------------------------------------------------
    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(self._data.shape)

    @property
    def ndim(self) -> int:
        return self._data.dim()

    @property
    def dtype(self):
        return self._data.dtype

    @property
    def size(self) -> int:
        return int(self._data.numel())

    @property
    def grad(self):
        return None if self._grad is None else Tensor(self._grad)

    def numpy(self) -> np.ndarray:
        data = self._data.detach()
        if data.dtype == torch.bfloat16:
            data = data.float()
        return data.cpu().numpy().copy()

    def detach(self) -> "Tensor":
        return Tensor(self._data)

    def zero_grad(self) -> None:
        self._grad = None

    def permute(self, *dims) -> "Tensor":
        inverse = [0] * len(dims)
        for i, d in enumerate(dims):
            inverse[d] = i
        return Tensor._from_op(self._data.permute(*dims), (self,),
                               lambda g: (g.permute(*inverse),), "permute")

    def __repr__(self) -> str:
        suffix = ", requires_grad=True" if self.requires_grad else ""
        return f"Tensor(shape={self.shape}, dtype={self.dtype}, device='{self.device}'{suffix})"

    # -- autograd ----------------------------------------------------------
    def backward(self, gradient=None, *, retain_graph: bool = False) -> None:
        if not self.requires_grad:
            raise RuntimeError("cannot call backward() on a tensor that does not require gradients")
        if self._graph_freed:
            raise RuntimeError("this autograd tape has already been freed")
        if gradient is None:
            if self.size != 1:
                raise RuntimeError("gradient must be supplied for non-scalar outputs")
            seed = torch.ones_like(self._data)
        else:
            seed = gradient._data if isinstance(gradient, Tensor) else _as_torch(gradient)
            seed = seed.to(self._data.device)
            if tuple(seed.shape) != self.shape:
                raise ValueError(f"gradient shape {tuple(seed.shape)} does not match {self.shape}")
        _run_backward(self, seed, retain_graph=retain_graph)


def _run_backward(root: Tensor, seed, *, retain_graph: bool = False) -> None:
    """Reverse sweep from ``root`` under the tape contract of ``_from_op``.

    Contract (tensorsmith's tape): every recorded use of a tensor sends it one
    gradient contribution; the contributions of all its uses are summed and
    cast to the tensor's dtype before they are stored in ``_grad`` and handed
    to the tensor's own VJP, which returns one contribution (or None) per
    parent.  Here a tensor is processed once every consumer edge into it has
    delivered (consumer counting), so each VJP runs exactly once with its
    complete gradient.  Without ``retain_graph`` the recorded graph is released.
    """
    # Consumer edges per tensor reachable from the root.
    pending_uses: dict[int, int] = {}
    reachable: list[Tensor] = [root]
    seen = {id(root)}
    for node in reachable:  # grows while iterating: a breadth-first walk
        if node._graph_freed:
            raise RuntimeError("this autograd tape has already been freed")
        for parent in node._parents:
            pending_uses[id(parent)] = pending_uses.get(id(parent), 0) + 1
            if id(parent) not in seen:
                seen.add(id(parent))
                reachable.append(parent)
    summed = {id(root): seed}
    ready = [root]
    while ready:
        node = ready.pop()
        grad = summed.pop(id(node), None)
        if grad is not None and node.requires_grad:
            if grad.dtype != node.dtype:
                grad = grad.to(node.dtype)
            node._grad = grad if node._grad is None else node._grad + grad
        parent_grads = None
        if grad is not None and node._backward is not None:
            parent_grads = tuple(node._backward(grad))
            if len(parent_grads) != len(node._parents):
                raise RuntimeError(
                    f"{node._op}: backward gave {len(parent_grads)} gradients for {len(node._parents)} inputs")
        for index, parent in enumerate(node._parents):
            contribution = None if parent_grads is None else parent_grads[index]
            if contribution is not None and parent.requires_grad:
                key = id(parent)
                summed[key] = contribution if key not in summed else summed[key] + contribution
            pending_uses[id(parent)] -= 1
            if pending_uses[id(parent)] == 0:
                ready.append(parent)
    if not retain_graph:
        for node in reachable:
            if node._backward is not None:
                node._parents, node._backward, node._graph_freed = (), None, True


def tensor(data, **kwargs) -> Tensor:
    return Tensor(data, **kwargs)
