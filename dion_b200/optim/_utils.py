"""Shared optimizer plumbing: DTensor helpers, same-shape batching, the
cooperative async task runtime, and the scalar (AdamW / Lion) updates.

Behavioural parity notes (reference files):
  * ``to_local`` / ``dtensor_from_local``: ada_dion/optim/dion_utils.py:8-45
  * batching key (shape, placements, dtype) and padding: dion_utils.py:48-76
  * ``AsyncTask`` / ``AsyncRuntime``: dion_utils.py:79-145
"""
from __future__ import annotations

import contextlib

import math
from collections import OrderedDict
from typing import Any, Callable, Dict, Generator, Iterable, Iterator, List, Optional, Sequence, Tuple, Union

import torch
from torch import Tensor
from torch.distributed.tensor import DTensor

from .. import ops

__all__ = [
    "to_local",
    "dtensor_from_local",
    "create_param_batches",
    "group_by_signature",
    "pad_batch",
    "AsyncTask",
    "AsyncRuntime",
    "scalar_update",
]


def to_local(t: Union[Tensor, Sequence[Tensor]]):
    """Local shard of a DTensor (or list of them); plain tensors pass through."""
    if isinstance(t, (list, tuple)):
        return [x.to_local() if isinstance(x, DTensor) else x for x in t]
    return t.to_local() if isinstance(t, DTensor) else t


def dtensor_from_local(local: Union[Tensor, List[Tensor]], ref: Union[Tensor, List[Tensor]]):
    """Wrap local tensors with the mesh and placements of ``ref`` (no-op for plain tensors)."""
    if isinstance(local, (list, tuple)):
        refs = ref if isinstance(ref, (list, tuple)) else [ref] * len(local)
        return [dtensor_from_local(x, r) for x, r in zip(local, refs)]
    if not isinstance(ref, DTensor):
        return local
    return DTensor.from_local(local, device_mesh=ref.device_mesh, placements=ref.placements, run_check=False,
                              shape=ref.shape, stride=ref.stride())


def _signature(p: Tensor) -> Tuple:
    placements = tuple(p.placements) if isinstance(p, DTensor) else None
    return (tuple(p.shape), placements, p.dtype)


def group_by_signature(params: Iterable[Tensor]) -> "OrderedDict[Tuple, List[Tensor]]":
    """Group tensors with identical (global shape, placements, dtype), keeping first-seen order."""
    groups: "OrderedDict[Tuple, List[Tensor]]" = OrderedDict()
    for p in params:
        groups.setdefault(_signature(p), []).append(p)
    return groups


def create_param_batches(params: Sequence[Tensor], batch_size: int) -> Iterator[List[Tensor]]:
    """Yield lists of up to ``batch_size`` same-signature tensors."""
    for group in group_by_signature(params).values():
        for i in range(0, len(group), batch_size):
            yield group[i : i + batch_size]


def pad_batch(batch: List[Tensor], batch_size: int) -> List[Tensor]:
    """Pad a short batch with zero tensors shaped like its first element."""
    assert 0 < len(batch) <= batch_size
    return list(batch) + [torch.zeros_like(batch[0]) for _ in range(batch_size - len(batch))]


class AsyncTask:
    """A generator-backed unit of optimizer work; each ``yield`` marks a point
    where the task waits on an asynchronous collective."""

    def __init__(self, gen: Generator[None, None, None], stream: Optional["torch.cuda.Stream"] = None):
        self._gen = gen
        self._stream = stream
        self.done = False
        self.step()

    def step(self) -> bool:
        """Run the task to its next ``yield`` (on its own CUDA stream, if it has one)."""
        if self.done:
            return False
        try:
            if self._stream is None:
                next(self._gen)
            else:
                with torch.cuda.stream(self._stream):
                    next(self._gen)
            return True
        except StopIteration:
            self.done = True
            return False


class AsyncRuntime:
    """Round-robin scheduler keeping up to ``max_concurrent_tasks`` tasks in
    flight, so the collective of one batch overlaps the math of the next."""

    def __init__(self, tasks: Iterable[AsyncTask], max_concurrent_tasks: int = 3):
        if max_concurrent_tasks <= 0:
            raise ValueError("max_concurrent_tasks must be positive")
        self._tasks = iter(tasks)
        self._max = max_concurrent_tasks

    def run(self) -> None:
        active: List[AsyncTask] = []
        exhausted = False
        while True:
            while not exhausted and len(active) < self._max:
                try:
                    t = next(self._tasks)
                except StopIteration:
                    exhausted = True
                    break
                if not t.done:
                    active.append(t)
            if not active:
                return
            still = []
            for t in active:
                if t.step():
                    still.append(t)
            active = still


def scalar_update(
    algo: str,
    params: List[Tensor],
    grads: List[Tensor],
    states: List[Dict[str, Any]],
    group: Dict[str, Any],
    cautious_wd: bool = False,
) -> None:
    """AdamW / Lion on local shards through the fused multi-tensor kernels."""
    X = to_local(params)
    G = to_local(grads)
    if algo == "adamw":
        ops.adamw_(
            X,
            G,
            to_local([s["momentum"] for s in states]),
            to_local([s["variance"] for s in states]),
            lr=float(group["lr"]),
            beta1=float(group["beta1"]),
            beta2=float(group["beta2"]),
            weight_decay=float(group["weight_decay"]),
            epsilon=float(group["epsilon"]),
            step=int(group["step"]),
            cautious_wd=cautious_wd,
        )
    elif algo == "lion":
        ops.lion_(
            X,
            G,
            to_local([s["momentum"] for s in states]),
            lr=float(group["lr"]),
            beta1=float(group["beta1"]),
            beta2=float(group["beta2"]),
            weight_decay=float(group["weight_decay"]),
            cautious_wd=cautious_wd,
        )
    else:
        raise ValueError(f"Unknown scalar algorithm: {algo}")


class StreamPool:
    """A few CUDA side streams on which independent units of optimizer work
    (same-shape groups) run concurrently, so that one group's kernels fill
    the SMs another group's tail leaves idle. ``session(device, n)`` returns
    a context for one step: ``use(i)`` enters unit i's stream (which first
    waits for the work already queued on the current stream), ``join()``
    makes the current stream wait for every stream used. Inactive (one
    unit, CPU tensors, or disabled): ``use`` is a no-op."""

    def __init__(self, size: int, enabled: bool = True):
        self.size = size
        self.enabled = enabled
        self._pools: Dict[Any, List[Any]] = {}

    def session(self, device, units: int) -> "_StreamSession":
        if not (self.enabled and units > 1 and getattr(device, "type", None) == "cuda"):
            return _StreamSession(None, None)
        pool = self._pools.get(device)
        if pool is None:
            pool = [torch.cuda.Stream(device=device) for _ in range(self.size)]
            self._pools[device] = pool
        return _StreamSession(pool, torch.cuda.current_stream(device))


class _StreamSession:
    def __init__(self, pool, main):
        self.pool, self.main = pool, main
        self.active = pool is not None
        self._used: List[Any] = []

    def use(self, i: int):
        if not self.active:
            return contextlib.nullcontext()
        st = self.pool[i % len(self.pool)]
        if st not in self._used:
            st.wait_stream(self.main)
            self._used.append(st)
        return torch.cuda.stream(st)

    def join(self) -> None:
        for st in self._used:
            self.main.wait_stream(st)
        self._used = []


_DEV_LISTS: Dict[Any, Tensor] = {}


def device_list(values: Sequence, dtype: torch.dtype, device) -> Tensor:
    """A small Python list as a device tensor, cached by value and copied
    from pinned memory: a pageable host-to-device copy blocks the host until
    the current stream drains, which keeps work queued on other streams from
    overlapping it."""
    key = (str(device), dtype, tuple(values))
    t = _DEV_LISTS.get(key)
    if t is None:
        if len(_DEV_LISTS) > 1024:
            # a cached tensor may last have been read by a kernel still queued on
            # another stream than the one that allocated it: let the device
            # drain before its memory can be handed out again (rare: once per
            # 1024 distinct lists)
            if torch.cuda.is_available() and torch.cuda.is_initialized():
                torch.cuda.synchronize()
            _DEV_LISTS.clear()
        t = torch.tensor(list(values), dtype=dtype)
        if getattr(device, "type", str(device)) == "cuda" or str(device).startswith("cuda"):
            t = t.pin_memory().to(device, non_blocking=True)  # asynchronous: pinned source
        else:
            t = t.to(device)
        _DEV_LISTS[key] = t
    return t
