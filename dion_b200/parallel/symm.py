"""Symmetric peer memory for in-kernel collectives over NVLink / NVSwitch.

``SymmetricHeap(group, nbytes)`` gives every rank of a single-node process
group one device region of the same size and maps every peer's region into
this process (CUDA IPC, see csrc/symm.cu). Kernels then address any rank's
copy of an offset directly:

  * ``heap.view(offset, shape, dtype)``  local tensor view
  * ``heap.addr(rank, offset)``          device address on ``rank``'s GPU
  * ``heap.barrier()``                   device-side epoch barrier (bounded
                                         wait; a timeout sets the status word)

The reduce-scatter / all-gather of Dion's power iteration and the all-to-all
of Muon are built from these: a producing GEMM's epilogue stores its tiles
into the owner rank's region, a barrier orders those stores, and the consumer
reads its own region locally. The collectives these replace are the
``reduce_scatter_tensor`` / ``all_gather_into_tensor`` / ``all_to_all`` calls
of ada_dion/optim/adadion_v2.py:927-949,1053-1071 and DION/muon.py:464-491.

The path is used only when every rank of the job is on one node (the IPC
mapping needs that) and can be switched off with ``DION_B200_P2P=0``.
"""
from __future__ import annotations

import itertools
import os
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
from torch import Tensor

from .. import ops

__all__ = ["SymmetricHeap", "p2p_enabled", "heap_for", "cached_for_heap"]

_ALIGN = 256
_UID = itertools.count()
_GUARD = 256  # canary bytes after the data region
_CANARY = 0x5A5AA5A5  # int32 pattern
_SCALAR_TYPE = {torch.float32: 6, torch.bfloat16: 15, torch.int64: 4, torch.uint8: 0}


def p2p_enabled(group, device: torch.device) -> bool:
    """Same answer on every rank: CUDA, extension built, >1 ranks, one node."""
    if os.environ.get("DION_B200_P2P", "1") == "0":
        return False
    if device.type != "cuda" or not ops.has_ext() or not dist.is_initialized():
        return False
    if dist.get_backend(group) != "nccl":
        return False
    W = dist.get_world_size(group)
    if W <= 1:
        return False
    local = int(os.environ.get("LOCAL_WORLD_SIZE", "0") or 0)
    return local >= dist.get_world_size() and torch.cuda.device_count() >= W


def _round(n: int, a: int = _ALIGN) -> int:
    return (n + a - 1) // a * a


class SymmetricHeap:
    def __init__(self, group, nbytes: int, device: Optional[torch.device] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        E = ops.ext()
        self._flag_off = 0
        self.data_off = _round(E.symm_flag_bytes())
        self.nbytes = _round(nbytes)
        try:
            ptr, handle = E.symm_create(self.data_off + self.nbytes + _GUARD)
        except RuntimeError as e:
            # the region is allocated outside PyTorch's caching allocator: give back
            # the allocator's cached, unused blocks (activations of the step that just
            # ran) and try once more
            if "out of memory" not in str(e).lower():
                raise
            torch.cuda.empty_cache()
            ptr, handle = E.symm_create(self.data_off + self.nbytes + _GUARD)
        hd = handle.to(self.device)
        allh = torch.empty(self.world * hd.numel(), dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(allh, hd, group=group)
        allh = allh.cpu().view(self.world, -1)
        self.bases: List[int] = []
        for j in range(self.world):
            self.bases.append(ptr if j == self.rank else E.symm_open(allh[j].contiguous()))
        self._own = ptr
        self._flags = torch.tensor(self.bases, dtype=torch.int64).to(self.device)
        self._closed = False
        self.uid = next(_UID)  # never reused, unlike id()
        self._close_hooks: List[Callable[[], None]] = []
        # canaries: the gap between the flag words and the data, and a guard after the data
        flag_end = E.symm_flag_bytes()
        self._canary_regions = [(flag_end, self.data_off - flag_end), (self.data_off + self.nbytes, _GUARD)]
        for off, size in self._canary_regions:
            E.symm_view(self._own + off, size // 4, 3).fill_(_CANARY)  # 3 = int32
        torch.cuda.synchronize(self.device)

    def check_canaries(self) -> bool:
        """True if no kernel wrote outside the data region of this rank's copy
        (the words before and after it still hold the canary pattern)."""
        E = ops.ext()
        for off, size in self._canary_regions:
            if size <= 0:
                continue
            v = E.symm_view(self._own + off, size // 4, 3)
            if not bool((v == _CANARY).all()):
                return False
        return True

    # ------------------------------------------------------------ addressing
    def addr(self, rank: int, offset: int) -> int:
        return self.bases[rank] + self.data_off + int(offset)

    def view(self, offset: int, shape: Sequence[int], dtype: torch.dtype) -> Tensor:
        n = 1
        for s in shape:
            n *= int(s)
        esz = torch.empty((), dtype=dtype).element_size()
        assert offset % 16 == 0 and offset + n * esz <= self.nbytes, "symmetric heap view out of range"
        return ops.ext().symm_view(self.addr(self.rank, offset), n, _SCALAR_TYPE[dtype]).view(*shape)

    def ptr_tensor(self, addrs: Sequence[int]) -> Tensor:
        return torch.tensor(list(addrs), dtype=torch.int64).to(self.device, non_blocking=True)

    # ------------------------------------------------------------ collectives
    def barrier(self) -> None:
        ops.ext().symm_barrier(self._flags, self.bases[self.rank] + self._flag_off, self.rank, self.world)

    def reduce_slots(self, src: Tensor, dst: Tensor, nslots: int) -> None:
        ops.ext().symm_reduce_slots(src, dst, nslots)

    def push(self, src: Tensor, dst_addrs: Tensor) -> None:
        ops.ext().symm_push(src, dst_addrs)

    def on_close(self, fn: Callable[[], None]) -> None:
        """Run ``fn`` when the heap is closed (before its memory is unmapped)."""
        self._close_hooks.append(fn)

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        hooks, self._close_hooks = self._close_hooks, []
        for fn in hooks:
            fn()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        E = ops.ext()
        for j, b in enumerate(self.bases):
            if j != self.rank:
                E.symm_close(b)
        E.symm_free(self._own)


_HEAPS: Dict[Tuple[int, str], SymmetricHeap] = {}


def heap_for(group, nbytes: int, tag: str, device: torch.device) -> SymmetricHeap:
    """A cached heap of at least ``nbytes`` for (group, tag); regrown (collectively) when too small."""
    key = (id(group), tag)
    h = _HEAPS.get(key)
    if h is None or h.nbytes < nbytes:
        if h is not None:
            h.close()
        h = SymmetricHeap(group, nbytes, device)
        _HEAPS[key] = h
    return h


def cached_for_heap(cache: dict, heap: "SymmetricHeap", key, build: Callable[[], Any]) -> Any:
    """``cache[key]``, built by ``build()`` on first use. Entries hold peer
    addresses and views into ``heap``; each is dropped when the heap closes
    (for example when a larger heap replaces it), so no cached pointer can
    outlive the mapping it points into."""
    v = cache.get(key)
    if v is None:
        v = build()
        cache[key] = v
        heap.on_close(lambda: cache.pop(key, None))
    return v


def release_all() -> None:
    """Unmap and free every cached heap (collective over each heap's group)."""
    for h in list(_HEAPS.values()):
        h.close()
    _HEAPS.clear()
