"""Dion: distributed low-rank orthonormalised updates with error feedback.

Public surface and state layout follow the dion package / the reference's
copy of it (ada_dion/optim/adadion_v2.py:82-249 constructor and validation,
:661-748 state, :857-1112 DDP and FSDP updates, :1298-1448 FSDP x TP update,
:1645-1947 helpers): param-group ``algorithm`` in {"dion", "adamw", "lion"};
per-matrix state ``momentum`` (error feedback folded in) and ``Q`` (DTensor
``Shard(0)`` on the outer shard mesh, ``Shard(1)`` on the inner mesh);
``r = ceil(rank_fraction * min(m, n) / multiple) * multiple``.

One step for a matrix X with momentum M and right factor Q:
    M += G
    P = M Q                       (transposed orientation when m < n)
    P = orthogonalize(P)          (randomised Cholesky QR)
    R = M^T P
    guard all-zero / NaN
    M -= (1 - mu) P R^T           (error feedback)
    Q = R / ||R_col||
    X = (1 - lr*wd) X - sqrt(fan_out/fan_in) * lr * P Q^T

B200 design:
  * momentum and Q of every same-shape group live in one arena tensor
    ([n, rows, cols]); the per-parameter state entries are views of it, so
    every product above is ONE batched tcgen05 GEMM over the group (tf32
    for fp32 state, bf16 for bf16 state) instead of a stack-and-copy;
  * the error-feedback and weight updates run as in-place GEMM epilogues
    (the weight update writes each parameter through a device pointer
    array), so M and X are read and written exactly once;
  * FSDP: arenas are laid out rank-major, so the batched P leaves the GEMM
    already in reduce-scatter order and the gathered P lands in GEMM order.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Any, Dict, Iterator, List, Optional, Tuple, Union

import torch
import torch.distributed as dist
import torch.distributed._functional_collectives as funcol
from torch import Tensor
from torch.distributed import ProcessGroup
from torch.distributed.device_mesh import DeviceMesh
from torch.distributed.tensor import DTensor, Partial, Placement, Replicate, Shard
from torch.optim.optimizer import Optimizer, ParamsT

from .. import ops
from ._utils import AsyncRuntime, AsyncTask, device_list, group_by_signature, scalar_update, to_local
from ..utils.trace import phase
from .linalg import orthogonalize

try:
    from torch.distributed.tensor.placement_types import _StridedShard
except ImportError:  # pragma: no cover
    _StridedShard = None

__all__ = ["Dion", "DionMixedPrecisionConfig", "DionParamConfig"]


def _sync_task(name: str, fn, *args):
    """A task that does all its work on its first step (no collective to overlap)."""
    with phase(name):
        fn(*args)
    return
    yield  # noqa: unreachable -- makes this a generator


@dataclass
class DionMixedPrecisionConfig:
    """dtype overrides for optimizer state; ``None`` = the parameter's dtype."""

    momentum_dtype: Optional[torch.dtype] = None
    Q_dtype: Optional[torch.dtype] = None
    variance_dtype: Optional[torch.dtype] = None


@dataclass
class DionParamConfig:
    outer_shard_tensor_dim: Optional[int] = None
    inner_shard_tensor_dim: Optional[int] = None
    outer_shard_mesh_dim: Optional[int] = None
    inner_shard_mesh_dim: Optional[int] = None
    is_transposed: bool = False
    compressed_all_reduce: bool = False
    Q_sharded_placements: Optional[Tuple[Placement, ...]] = None
    Q_inner_unsharded_placements: Optional[Tuple[Placement, ...]] = None


def _group_of(mesh: Union[DeviceMesh, ProcessGroup, None]) -> Optional[ProcessGroup]:
    if mesh is None:
        return None
    if isinstance(mesh, DeviceMesh):
        return mesh.get_group()
    return mesh


class Dion(Optimizer):
    """Dion optimizer (DDP, FSDP2, HSDP and FSDP x TP layouts)."""

    def __init__(
        self,
        params: ParamsT,
        replicate_mesh: Optional[Union[DeviceMesh, ProcessGroup]] = None,
        outer_shard_mesh: Optional[DeviceMesh] = None,
        inner_shard_mesh: Optional[DeviceMesh] = None,
        replicate_mesh_grad_sync: bool = True,
        rank_fraction: float = 1.0,
        rank_multiple_of: int = 1,
        lr: float = 0.01,
        mu: float = 0.95,
        betas: Tuple[float, float] = (0.9, 0.95),
        weight_decay: float = 0.01,
        epsilon: float = 1e-8,
        power_iters: int = 1,
        qr_method: str = "rcqr",
        cqr_warmup_steps: int = 150,
        rcqr_oversample: float = 1.25,
        mixed_precision_config: Optional[DionMixedPrecisionConfig] = None,
    ):
        if lr < 0.0:
            raise ValueError(f"lr must be non-negative, got {lr}")
        if mu < 0.0:
            raise ValueError(f"mu must be non-negative, got {mu}")
        if len(betas) != 2 or betas[0] < 0.0 or betas[1] < 0.0:
            raise ValueError(f"betas must be two non-negative numbers, got {betas}")
        if weight_decay < 0.0:
            raise ValueError(f"weight_decay must be non-negative, got {weight_decay}")
        if rank_fraction <= 0 or rank_fraction > 1:
            raise ValueError(f"rank_fraction must lie in (0, 1], got {rank_fraction}")
        if rank_multiple_of <= 0:
            raise ValueError(f"rank_multiple_of must be a positive integer, got {rank_multiple_of}")
        if power_iters != 1:
            raise ValueError(f"this Dion runs one power iteration per step (power_iters=1), got {power_iters}")
        if qr_method != "rcqr":
            raise ValueError(f"this Dion orthogonalises with randomised Cholesky QR only (qr_method='rcqr'), got {qr_method!r}")
        if replicate_mesh is not None and not isinstance(replicate_mesh, (DeviceMesh, ProcessGroup)):
            raise TypeError(f"replicate_mesh: expected a DeviceMesh or a ProcessGroup, not {type(replicate_mesh).__name__}")
        for name, mesh in (("Outer", outer_shard_mesh), ("Inner", inner_shard_mesh)):
            if mesh is not None:
                if not isinstance(mesh, DeviceMesh):
                    raise TypeError(f"{name.lower()}_shard_mesh: expected a DeviceMesh, not {type(mesh).__name__}")
                if mesh.ndim != 1:
                    raise ValueError(f"{name.lower()}_shard_mesh has {mesh.ndim} dimensions; pass the 1-D sub-mesh of the sharding dimension")
                if mesh == replicate_mesh:
                    raise ValueError(f"{name.lower()}_shard_mesh and replicate_mesh are the same mesh; they must differ")
        if inner_shard_mesh is not None and inner_shard_mesh == outer_shard_mesh:
            raise ValueError("outer_shard_mesh and inner_shard_mesh are the same mesh; they must differ")

        defaults = dict(
            rank_fraction=rank_fraction,
            rank_multiple_of=rank_multiple_of,
            lr=lr,
            mu=mu,
            beta1=betas[0],
            beta2=betas[1],
            weight_decay=weight_decay,
            epsilon=epsilon,
            oversample=rcqr_oversample,
            algorithm="dion",
            step=0,
        )
        super().__init__(params, defaults)
        self._param_config: Dict[Tensor, DionParamConfig] = {}
        self._replicate_mesh = replicate_mesh
        self._outer_shard_mesh = outer_shard_mesh
        self._inner_shard_mesh = inner_shard_mesh
        self._replicate_mesh_grad_sync = replicate_mesh_grad_sync
        if isinstance(replicate_mesh, DeviceMesh):
            self._replicate_world_size = replicate_mesh.size()
        elif isinstance(replicate_mesh, ProcessGroup):
            self._replicate_world_size = dist.get_world_size(replicate_mesh)
        else:
            self._replicate_world_size = 1
        self._outer_shard_ranks = (
            dist.get_process_group_ranks(outer_shard_mesh.get_group()) if outer_shard_mesh is not None else None
        )
        self._inner_shard_ranks = (
            dist.get_process_group_ranks(inner_shard_mesh.get_group()) if inner_shard_mesh is not None else None
        )
        self._mixed_precision_config = mixed_precision_config or DionMixedPrecisionConfig()
        self._arenas: Dict[Tuple, Dict[str, Any]] = {}
        self._p2p_ptrs: Dict[Tuple, Any] = {}
        # signature sets in flight at once (the reference keeps three, adadion_v2.py:286)
        self._max_concurrent_tasks = 3
        self._side_streams: Dict[Any, List[Any]] = {}
        self._next_stream = 0
        self._use_side_streams = os.environ.get("DION_B200_SIDE_STREAMS", "1") != "0"
        self._q_init_calls = 0

    # ------------------------------------------------------------------ step
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            group["step"] += 1
        # Dion shape groups run as tasks, up to three in flight: a task yields
        # after issuing an asynchronous collective, so that collective overlaps
        # the next task's GEMMs (ada_dion/optim/adadion_v2.py:284-287,
        # ada_dion/optim/dion_utils.py:121-145)
        dion_groups = [(g, [p for p in g["params"] if p.grad is not None]) for g in self.param_groups
                       if g["algorithm"] == "dion"]
        used_streams: List[Any] = []
        AsyncRuntime((t for g, ps in dion_groups if ps for t in self._dion_tasks(g, ps, used_streams)),
                     max_concurrent_tasks=self._max_concurrent_tasks).run()
        if used_streams:  # the rest of the step (and of training) sees every set's update
            main = torch.cuda.current_stream()
            for st in used_streams:
                main.wait_stream(st)
        for group in self.param_groups:
            algo = group["algorithm"]
            params = [p for p in group["params"] if p.grad is not None]
            if not params or algo == "dion":
                continue
            if algo in ("adamw", "lion"):
                states = [self._get_or_initialize_state(p, group) for p in params]
                grads = [p.grad for p in params]
                if self._replicate_mesh is not None and self._replicate_mesh_grad_sync:
                    grads = self._all_reduce_replicate([to_local(g) for g in grads])
                scalar_update(algo, params, grads, states, group)
            else:
                raise ValueError(f"Unknown algorithm: {algo}")
        ops.check_status()
        return loss

    @torch.no_grad()
    def synchronize_for_checkpoint(self):
        """Average every state tensor over the replicate mesh (compressed sync
        lets the momenta of DP replicas drift; a checkpoint needs one copy)."""
        if self._replicate_mesh is None or not self._replicate_mesh_grad_sync:
            return
        tensors = [v for st in self.state.values() for v in st.values() if isinstance(v, Tensor)]
        if tensors:
            local = [to_local(t) for t in tensors]
            reduced = self._all_reduce_replicate(local)
            for t, r in zip(local, reduced):
                t.copy_(r)

    # ------------------------------------------------------------------ config / state
    def _get_dion_param_config(self, x: Tensor) -> DionParamConfig:
        if x in self._param_config:
            return self._param_config[x]
        if x.ndim > 2:
            raise NotImplementedError(f"Dion handles matrices (at most 2 dimensions); this parameter has {x.ndim}")
        using_mesh = any(isinstance(m, DeviceMesh) for m in (self._replicate_mesh, self._outer_shard_mesh,
                                                               self._inner_shard_mesh))
        if using_mesh and not isinstance(x, DTensor):
            raise TypeError("with a DeviceMesh configured, every Dion parameter has to be a DTensor")
        if isinstance(self._replicate_mesh, ProcessGroup) and isinstance(x, DTensor):
            raise TypeError(
                "DTensor parameters need the replicate group as a DeviceMesh; a ProcessGroup was given"
            )
        cfg = DionParamConfig()
        if x.ndim == 2:
            m, n = x.shape
            cfg.is_transposed = m < n
        if isinstance(x, DTensor) and x.ndim == 2:
            mesh = x.device_mesh
            used = [None] * x.ndim
            for mdim, pl in enumerate(x.placements):
                if _StridedShard is not None and isinstance(pl, _StridedShard):
                    raise NotImplementedError(
                        "a strided-sharded matrix (_StridedShard) cannot be orthogonalised per shard: let FSDP and TP "
                        "shard different dimensions of each matrix"
                    )
                if not pl.is_shard():
                    continue
                tdim = pl.dim
                if used[tdim] is not None:
                    raise RuntimeError(f"tensor dimension {tdim} is sharded over two mesh dimensions")
                used[tdim] = mdim
                ranks = dist.get_process_group_ranks(mesh.get_group(mdim))
                outer = ranks == self._outer_shard_ranks
                inner = ranks == self._inner_shard_ranks
                if outer:
                    cfg.outer_shard_tensor_dim, cfg.outer_shard_mesh_dim = tdim, mdim
                if inner:
                    cfg.inner_shard_tensor_dim, cfg.inner_shard_mesh_dim = tdim, mdim
                if outer and inner:
                    raise RuntimeError("the outer and inner shardings resolve to one process group")
                if mesh.size(mdim) > 1 and not outer and not inner:
                    raise RuntimeError(
                        f"mesh dimension {mdim} shards this parameter but is neither the outer nor the inner shard mesh"
                    )
            if cfg.inner_shard_tensor_dim == 0 or cfg.outer_shard_tensor_dim == 1:
                cfg.is_transposed = False
            if cfg.outer_shard_tensor_dim == 0 or cfg.inner_shard_tensor_dim == 1:
                cfg.is_transposed = True
        self._param_config[x] = cfg
        return cfg

    def _rank_of(self, shape, group) -> int:
        m, n = shape
        r = group["rank_fraction"] * min(m, n)
        mult = group["rank_multiple_of"]
        r = mult * math.ceil(r / mult)
        return int(min(r, m, n))

    def _get_or_initialize_state(self, p: Tensor, group: dict) -> dict:
        st = self.state[p]
        if not st:
            algo = group["algorithm"]
            mp = self._mixed_precision_config
            if algo == "dion":
                self._init_dion_states([p], group)
            elif algo == "adamw":
                st["momentum"] = torch.zeros_like(p, dtype=mp.momentum_dtype)
                st["variance"] = torch.zeros_like(p, dtype=mp.variance_dtype)
            elif algo in ("lion", "clion"):
                st["momentum"] = torch.zeros_like(p, dtype=mp.momentum_dtype)
            else:
                raise ValueError(f"Unknown algorithm: {algo}")
        return st

    def _q_placements(self, p: DTensor, cfg: DionParamConfig) -> None:
        pl = [Replicate() for _ in range(p.device_mesh.ndim)]
        if cfg.outer_shard_mesh_dim is not None:
            pl[cfg.outer_shard_mesh_dim] = Shard(0)
        if cfg.inner_shard_mesh_dim is not None:
            pl[cfg.inner_shard_mesh_dim] = Shard(1)
        cfg.Q_sharded_placements = tuple(pl)
        if cfg.inner_shard_mesh_dim is not None:
            pl[cfg.inner_shard_mesh_dim] = Replicate()
            cfg.Q_inner_unsharded_placements = tuple(pl)

    def _init_dion_states(self, params: List[Tensor], group: dict, order: Optional[List[int]] = None,
                          slots: Optional[int] = None) -> None:
        """Allocate momentum and Q for same-signature params as views of two
        arenas; ``order[i]`` is the arena slot of ``params[i]`` (extra slots
        are zero padding used by the rank-major FSDP layout)."""
        mp = self._mixed_precision_config
        p0 = params[0]
        if p0.ndim != 2:
            raise ValueError(
                f"the Dion algorithm updates matrices; this group holds a {p0.ndim}-D parameter (put vectors and "
                "scalars in a group with algorithm='adamw' or 'lion')"
            )
        cfg = self._get_dion_param_config(p0)
        m, n = p0.shape
        r = self._rank_of((m, n), group)
        q_shape = (m, r) if cfg.is_transposed else (n, r)
        if group["rank_fraction"] < 1 and (m + n) * r < m * n:
            cfg.compressed_all_reduce = True
        q_dtype = mp.Q_dtype or p0.dtype
        m_dtype = mp.momentum_dtype or p0.dtype
        order = list(range(len(params))) if order is None else order
        slots = slots or (max(order) + 1)
        local0 = to_local(p0)
        dev = local0.device
        # Q draws come from a generator seeded by the process seed and the
        # order of state creation: identical on every rank and independent of
        # how much randomness earlier steps consumed (sketches, etc.)
        gen = torch.Generator(device=dev)
        gen.manual_seed((torch.initial_seed() * 7919 + 104729 * self._q_init_calls) % (2**63 - 1))
        self._q_init_calls += 1
        mom_arena = torch.zeros((slots,) + tuple(local0.shape), device=dev, dtype=m_dtype)
        if isinstance(p0, DTensor):
            self._q_placements(p0, cfg)
            locals_ = []
            for _ in params:
                # the global Q is drawn identically on every rank (same RNG
                # state), then each rank keeps its shard
                f = torch.randn(q_shape, device=dev, dtype=torch.float32, generator=gen).to(q_dtype)
                qd = DTensor.from_local(f, p0.device_mesh, [Replicate()] * p0.device_mesh.ndim, run_check=False)
                locals_.append(qd.redistribute(placements=cfg.Q_sharded_placements).to_local())
            q_arena = torch.zeros((slots,) + tuple(locals_[0].shape), device=dev, dtype=q_dtype)
            for i, ql in zip(order, locals_):
                q_arena[i].copy_(ql)
        else:
            q_arena = torch.zeros((slots,) + q_shape, device=dev, dtype=q_dtype)
            for i in order:
                q_arena[i].copy_(torch.randn(q_shape, device=dev, dtype=torch.float32, generator=gen))
                self._replicate_broadcast(q_arena[i])
        self._bind_arena(params, order, mom_arena, q_arena, cfg, q_shape)

    def _bind_arena(self, params, order, mom_arena, q_arena, cfg, q_shape) -> None:
        key = tuple(id(p) for p in params)
        self._arenas[key] = {"M": mom_arena, "Q": q_arena, "order": list(order)}
        for p, slot in zip(params, order):
            self._param_config[p] = cfg
            st = self.state[p]
            mom, q = mom_arena[slot], q_arena[slot]
            if isinstance(p, DTensor):
                st["momentum"] = DTensor.from_local(mom, p.device_mesh, p.placements, run_check=False, shape=p.shape,
                                                    stride=p.stride())
                st["Q"] = DTensor.from_local(q, p.device_mesh, cfg.Q_sharded_placements, run_check=False,
                                             shape=torch.Size(q_shape), stride=(q_shape[1], 1))
            else:
                st["momentum"] = mom
                st["Q"] = q

    def _arena(self, params: List[Tensor], group: dict, order: List[int], slots: int) -> Tuple[Tensor, Tensor]:
        """Arena views ([slots, ...]) backing momentum and Q of ``params``.
        State created elsewhere (e.g. loaded from a checkpoint) is packed into
        a fresh arena and re-pointed."""
        if any(not self.state[p] for p in params):
            if all(not self.state[p] for p in params):
                self._init_dion_states(params, group, order, slots)
            else:
                for p in params:
                    if not self.state[p]:
                        self._init_dion_states([p], group)
        key = tuple(id(p) for p in params)
        a = self._arenas.get(key)
        ok = a is not None and a["order"] == list(order) and a["M"].size(0) == slots
        if ok:
            for p, slot in zip(params, order):
                st = self.state[p]
                if (to_local(st["momentum"]).data_ptr() != a["M"][slot].data_ptr()
                        or to_local(st["Q"]).data_ptr() != a["Q"][slot].data_ptr()):
                    ok = False
                    break
        if not ok:
            M0 = to_local(self.state[params[0]]["momentum"])
            Q0 = to_local(self.state[params[0]]["Q"])
            mom_arena = torch.zeros((slots,) + tuple(M0.shape), device=M0.device, dtype=M0.dtype)
            q_arena = torch.zeros((slots,) + tuple(Q0.shape), device=Q0.device, dtype=Q0.dtype)
            for p, slot in zip(params, order):
                mom_arena[slot].copy_(to_local(self.state[p]["momentum"]))
                q_arena[slot].copy_(to_local(self.state[p]["Q"]))
            cfg = self._get_dion_param_config(params[0])
            Qs = self.state[params[0]]["Q"]
            q_shape = tuple(Qs.shape)
            if isinstance(params[0], DTensor) and cfg.Q_sharded_placements is None:
                self._q_placements(params[0], cfg)
            self._bind_arena(params, order, mom_arena, q_arena, cfg, q_shape)
            a = self._arenas[key]
        return a["M"], a["Q"]

    def _replicate_broadcast(self, t: Tensor) -> None:
        rm = self._replicate_mesh
        if rm is None:
            return
        if isinstance(rm, DeviceMesh):
            for g in rm.get_all_groups():
                dist.broadcast(t, group=g, group_src=0)
        else:
            dist.broadcast(t, group=rm, group_src=0)

    def _all_reduce_replicate_async(self, ts: List[Tensor]):
        """Generator form of the replicate-mesh average (in place): issues one
        coalesced asynchronous all-reduce, yields, then waits for it."""
        rm = self._replicate_mesh
        if rm is None:
            return ts
        pg = _group_of(rm)
        ts = [t if t.is_contiguous() else t.contiguous() for t in ts]
        with dist._coalescing_manager(group=pg, async_ops=True) as cm:
            for t in ts:
                dist.all_reduce(t, op=dist.ReduceOp.AVG, group=pg)
        yield
        cm.wait()
        return ts

    def _all_reduce_replicate(self, ts: List[Tensor], op: str = "avg") -> List[Tensor]:
        rm = self._replicate_mesh
        if rm is None:
            return ts
        pg = _group_of(rm)
        if len(ts) == 1:
            return [funcol.all_reduce(ts[0], reduceOp=op, group=pg).wait()]
        return [x.wait() if hasattr(x, "wait") else x for x in funcol.all_reduce_coalesced(ts, reduceOp=op, group=pg)]

    # ------------------------------------------------------------------ dion
    def _task_stream(self, device: torch.device, used: List[Any]):
        """CUDA stream for the next signature set: a pool of
        ``max_concurrent_tasks`` side streams, so the sets in flight also run
        concurrently on the GPU (the factorisations of one set are latency-
        bound and leave most SMs to the next set's GEMMs). Each stream first
        waits for the work already queued on the current stream (the
        gradients)."""
        if device.type != "cuda" or not self._use_side_streams:
            return None
        pool = self._side_streams.get(device)
        if pool is None:
            pool = [torch.cuda.Stream(device=device) for _ in range(self._max_concurrent_tasks)]
            self._side_streams[device] = pool
        st = pool[self._next_stream % len(pool)]
        self._next_stream += 1
        st.wait_stream(torch.cuda.current_stream(device))
        if st not in used:
            used.append(st)
        return st

    def _dion_tasks(self, group: dict, params: List[Tensor], used_streams: Optional[List[Any]] = None
                    ) -> Iterator[AsyncTask]:
        """One task per same-signature set of this group (created lazily, so
        the runtime holds at most ``max_concurrent_tasks`` sets' buffers)."""
        used = used_streams if used_streams is not None else []
        self._next_stream = 0
        for same in group_by_signature(params).values():
            cfg = self._get_dion_param_config(same[0])
            shape = "x".join(str(d) for d in same[0].shape)
            st = self._task_stream(to_local(same[0]).device, used)
            if cfg.inner_shard_mesh_dim is not None:
                yield AsyncTask(_sync_task(f"dion/fsdp_tp/{shape}", self._dion_fsdp_tp, group, same, cfg), st)
            elif cfg.outer_shard_mesh_dim is not None and self._outer_shard_mesh.size() > 1:
                yield AsyncTask(self._dion_sharded_gen(group, same, cfg, f"dion/sharded/{shape}"), st)
            else:
                yield AsyncTask(self._dion_replicated_gen(group, same, cfg, f"dion/replicated/{shape}"), st)

    def _dion_group(self, group: dict, params: List[Tensor]) -> None:
        """All of one group's sets, one after the other (no overlap)."""
        used: List[Any] = []
        for t in self._dion_tasks(group, params, used):
            while t.step():
                pass
        for st in used:
            torch.cuda.current_stream().wait_stream(st)

    # hooks overridden by the adaptive-rank subclass
    def _active_q(self, params, order, Qb):
        """Q view used this step and per-slot active ranks (None: all columns)."""
        return Qb, None

    def _orth(self, P: Tensor, group: dict, ranks) -> Tensor:
        return orthogonalize(P, float(group["oversample"]))

    def _after_update(self, group, params, order, sumsq, ranks) -> None:
        return None

    def _scaled_lr(self, shape, lr: float) -> float:
        fan_out, fan_in = shape
        return math.sqrt(fan_out / fan_in) * lr

    @staticmethod
    def _op_dtype(dt: torch.dtype) -> torch.dtype:
        # bf16 state runs on the bf16 tensor cores, anything else on tf32
        return torch.bfloat16 if dt == torch.bfloat16 else torch.float32

    def _power_p(self, Mb: Tensor, Qb: Tensor, transposed: bool) -> Tensor:
        """P = M Q (or M^T Q), fp32 result."""
        dt = self._op_dtype(Mb.dtype)
        A = Mb.transpose(1, 2) if transposed else Mb
        P = torch.empty((Mb.size(0), A.size(1), Qb.size(-1)), device=Mb.device, dtype=torch.float32)
        ops.matmul(A.to(dt), Qb.to(dt), out=P)
        return P

    def _power_r(self, Mb: Tensor, P: Tensor, transposed: bool) -> Tensor:
        """R = M^T P (or M P), fp32 result."""
        dt = self._op_dtype(Mb.dtype)
        A = Mb if transposed else Mb.transpose(1, 2)
        R = torch.empty((Mb.size(0), A.size(1), P.size(-1)), device=Mb.device, dtype=torch.float32)
        ops.matmul(A.to(dt), P.to(dt), out=R)
        return R

    def _update(self, group, params, order, Mb, Qb, P, R, nz, transposed, sumsq) -> None:
        """Error feedback, Q <- colnorm(R), weight update (all batched); the
        all-zero / NaN guard has already been applied to P and R."""
        lr, mu = float(group["lr"]), float(group["mu"])
        wd, eps = float(group["weight_decay"]), float(group["epsilon"])
        dt = self._op_dtype(Mb.dtype)
        Pm, Rm = P.to(dt), R.to(dt)
        slots = list(Mb.unbind(0))
        # M -= (1 - mu) * P R^T   (R P^T when transposed)
        if transposed:
            ops.matmul_update_(slots, Rm, Pm.transpose(1, 2), gamma=1.0, delta=-(1.0 - mu))
        else:
            ops.matmul_update_(slots, Pm, Rm.transpose(1, 2), gamma=1.0, delta=-(1.0 - mu))
        if sumsq is None:
            sumsq = ops.col_sumsq(R)
        ops.col_normalize(R, sumsq, eps, Qb)
        # X = (1 - lr*wd) X - sqrt(fan_out/fan_in) lr * P Q^T   (Q P^T when transposed)
        X = to_local(params)
        xdt = self._op_dtype(X[0].dtype)
        idx = device_list(order, torch.int64, Mb.device)
        Qn = Qb.index_select(0, idx).to(xdt)
        Px = P.index_select(0, idx).to(xdt)
        s_lr = self._scaled_lr(params[0].shape, lr)
        if transposed:
            ops.matmul_update_(X, Qn, Px.transpose(1, 2), gamma=1.0 - lr * wd, delta=-s_lr)
        else:
            ops.matmul_update_(X, Px, Qn.transpose(1, 2), gamma=1.0 - lr * wd, delta=-s_lr)

    # ---- single device / DDP (replicated parameters)
    def _dion_replicated(self, group: dict, params: List[Tensor], cfg: DionParamConfig) -> None:
        for _ in self._dion_replicated_gen(group, params, cfg, "dion/replicated"):
            pass

    def _dion_replicated_gen(self, group: dict, params: List[Tensor], cfg: DionParamConfig, name: str):
        """Single device / DDP / HSDP-replicated update of one signature set;
        yields after each asynchronous collective."""
        n = len(params)
        order = list(range(n))
        Mb, Qb = self._arena(params, group, order, n)
        Qb, ranks = self._active_q(params, order, Qb)
        G = [to_local(p.grad) for p in params]
        world = self._replicate_world_size
        rm = self._replicate_mesh
        multi = rm is not None and world > 1
        compressed = self._replicate_mesh_grad_sync and cfg.compressed_all_reduce and multi
        if self._replicate_mesh_grad_sync and not cfg.compressed_all_reduce and multi:
            G = yield from self._all_reduce_replicate_async(G)
        with phase(name):
            nz = ops.dion_momentum_add_(list(Mb.unbind(0)), G)
            t = cfg.is_transposed
            P = self._power_p(Mb, Qb, t)
            pd, r = P.shape[1:]
        if multi:
            # each replica orthogonalises every world-th matrix, then all-gather
            pg = _group_of(rm)
            rank = dist.get_rank(pg)
            sets = (n + world - 1) // world
            Pp = torch.zeros((sets * world, pd, r), device=P.device, dtype=P.dtype)
            Pp[:n] = P
            Pv = Pp.view(sets, world, pd, r).transpose(0, 1).contiguous()  # [world, sets, pd, r]
            if compressed:
                mine = torch.empty((sets, pd, r), device=P.device, dtype=P.dtype)
                work = dist.reduce_scatter_tensor(mine, Pv.view(world * sets, pd, r), op=dist.ReduceOp.AVG,
                                                  group=pg, async_op=True)
                yield
                work.wait()
            else:
                mine = Pv[rank].contiguous()
            with phase(name):
                mine = self._orth(mine, group, None if ranks is None else
                                  [ranks[s * world + rank] if s * world + rank < n else 0 for s in range(sets)])
            allp = torch.empty((world, sets, pd, r), device=P.device, dtype=P.dtype)
            work = dist.all_gather_into_tensor(allp.view(world * sets, pd, r), mine.contiguous(), group=pg,
                                               async_op=True)
            yield
            work.wait()
            P = allp.transpose(0, 1).reshape(sets * world, pd, r)[:n].contiguous()
        else:
            with phase(name):
                P = self._orth(P, group, ranks)
        with phase(name):
            R = self._power_r(Mb, P, t)
        if compressed:
            R = (yield from self._all_reduce_replicate_async([R]))[0]
        with phase(name):
            ops.dion_fixup_(P, R, Qb, nz)
            sumsq = ops.col_sumsq(R)
            self._update(group, params, order, Mb, Qb, P, R, nz, t, sumsq)
            self._after_update(group, params, order, sumsq, ranks)

    # ---- FSDP (outer-sharded) parameters
    def _dion_sharded(self, group: dict, params: List[Tensor], cfg: DionParamConfig) -> None:
        for _ in self._dion_sharded_gen(group, params, cfg, "dion/sharded"):
            pass

    def _dion_sharded_gen(self, group: dict, params: List[Tensor], cfg: DionParamConfig, name: str):
        """FSDP (outer-sharded) update of one signature set; on the NCCL path
        it yields after each asynchronous collective (reduce-scatter of P,
        all-gather of the orthogonalised P, all-reduce of the column norms)."""
        mesh = self._outer_shard_mesh
        pg = mesh.get_group()
        W = mesh.size()
        n = len(params)
        sets = (n + W - 1) // W
        # rank-major slots: slot (j, s) holds matrix s*W + j, which rank j orthogonalises
        order = [(i % W) * sets + (i // W) for i in range(n)]
        Mb, Qb = self._arena(params, group, order, sets * W)
        Qb, ranks = self._active_q(params, order, Qb)
        G = [to_local(p.grad) for p in params]
        rm = self._replicate_mesh
        compressed = self._replicate_mesh_grad_sync and cfg.compressed_all_reduce and rm is not None
        if self._replicate_mesh_grad_sync and not cfg.compressed_all_reduce and rm is not None:
            G = yield from self._all_reduce_replicate_async(G)
        with phase(name):
            nz_p = ops.dion_momentum_add_([Mb[o] for o in order], G)
            nz = torch.zeros(sets * W, device=Mb.device, dtype=torch.float32)
            nz[device_list(order, torch.int64, Mb.device)] = nz_p
        t = cfg.is_transposed
        me = mesh.get_local_rank()
        my_ranks = None if ranks is None else ranks[me * sets:(me + 1) * sets]
        heap = self._p2p_heap(pg, Mb, Qb, t, sets, W)
        if heap is not None:
            # fused path: the transfers ride in the GEMM epilogues (no NCCL to overlap)
            with phase(name):
                P_all = self._p2p_power_orth(heap, group, Mb, Qb, t, sets, W, me, my_ranks, compressed)
        else:
            with phase(name):
                P_part = self._power_p(Mb, Qb, t)  # partial sums over this rank's shard
            pd, r = P_part.shape[1:]
            mine = torch.empty((sets, pd, r), device=Mb.device, dtype=torch.float32)
            work = dist.reduce_scatter_tensor(mine, P_part, op=dist.ReduceOp.SUM, group=pg, async_op=True)
            yield
            work.wait()
            del P_part
            if compressed:
                mine = (yield from self._all_reduce_replicate_async([mine]))[0]
            with phase(name):
                mine = self._orth(mine, group, my_ranks)
            P_all = torch.empty((sets * W, pd, r), device=Mb.device, dtype=torch.float32)
            work = dist.all_gather_into_tensor(P_all, mine.contiguous(), group=pg, async_op=True)
            yield
            work.wait()
        with phase(name):
            R = self._power_r(Mb, P_all, t)
        if compressed:
            if heap is not None:
                # P_all lives in the shared heap until the update below: no other set may run here
                R = self._all_reduce_replicate([R])[0]
            else:
                R = (yield from self._all_reduce_replicate_async([R]))[0]
        with phase(name):
            ops.dion_fixup_(P_all, R, Qb, nz)
            sumsq = ops.col_sumsq(R)
        if heap is not None:
            with phase(name):
                sumsq = self._p2p_sum(heap, sumsq, sets, W, me, P_all.size(1))
        else:
            work = dist.all_reduce(sumsq, op=dist.ReduceOp.SUM, group=pg, async_op=True)
            yield
            work.wait()
        with phase(name):
            self._update(group, params, order, Mb, Qb, P_all, R, nz, t, sumsq)
            self._after_update(group, params, order, sumsq, ranks)

    # ---- in-kernel collectives over symmetric peer memory
    def _p2p_heap(self, pg, Mb: Tensor, Qb: Tensor, transposed: bool, sets: int, W: int):
        """The group's symmetric heap when the fused NVLink path applies (the
        decision depends only on shapes and the job layout, so every rank of
        ``pg`` takes the same branch)."""
        from ..parallel.symm import heap_for, p2p_enabled

        if not p2p_enabled(pg, Mb.device):
            return None
        pd = Mb.size(2) if transposed else Mb.size(1)
        r = Qb.size(-1)
        if r % 4:
            return None
        slot = pd * r * 4
        # one heap per signature: sets on different streams never share peer buffers
        return heap_for(pg, 2 * W * sets * slot + W * sets * W * r * 4, f"dion:{pd}x{r}:{sets}", Mb.device)

    def _p2p_sum(self, heap, sumsq: Tensor, sets: int, W: int, me: int, pd: int) -> Tensor:
        """All-reduce (sum) of the column sums of squares [sets*W, r] without
        NCCL: every rank stores its copy into slot ``me`` of every rank's
        sum region (after recv and P_all, so the next group's P stores cannot
        overwrite slots still being summed), one device barrier, a fixed-order
        sum of the W slots. Replaces ada_dion/optim/adadion_v2.py:1091-1096."""
        from ..parallel.symm import cached_for_heap

        r = sumsq.size(1)
        nb = sets * W * r * 4
        base = 2 * W * sets * pd * r * 4
        key = ("p2p_sum", heap.uid, sets, W, pd, r)
        ptrs = cached_for_heap(self._p2p_ptrs, heap, key, lambda: heap.ptr_tensor(
            [heap.addr((me + 1 + i) % W, base + me * nb) for i in range(W)]))
        heap.push(sumsq.contiguous(), ptrs)
        heap.barrier()
        out = torch.empty_like(sumsq)
        heap.reduce_slots(heap.view(base, (W, sets * W, r), torch.float32), out, W)
        return out

    def _p2p_power_orth(self, heap, group: dict, Mb: Tensor, Qb: Tensor, transposed: bool, sets: int, W: int,
                        me: int, my_ranks, compressed: bool) -> Tensor:
        """P = M Q reduce-scattered, orthogonalised and all-gathered without NCCL.

        Heap layout (fp32): recv [W (source), sets, pd, r] then P_all [W*sets, pd, r].
          1. the P GEMM's epilogue stores batch k = j*sets + s straight into rank
             j's recv[me, s] (NVLink stores overlapping the next tiles' MMAs);
          2. device barrier; 3. this rank sums its W recv slots (fixed order);
          4. the orthogonaliser's last GEMM stores each result into P_all[me*sets + s]
             of every rank (nrep = W); 5. device barrier.
        Replaces ada_dion/optim/adadion_v2.py:1051-1071 (reduce-scatter, orthogonalize, all-gather).
        """
        from ..parallel.symm import cached_for_heap

        dt = self._op_dtype(Mb.dtype)
        A = Mb.transpose(1, 2) if transposed else Mb
        pd, r = A.size(1), Qb.size(-1)
        slot = pd * r * 4
        recv_off, pall_off = 0, W * sets * slot
        key = ("p2p", heap.uid, sets, W, pd, r)

        def build():
            rs = [heap.addr(k // sets, recv_off + (me * sets + k % sets) * slot) for k in range(W * sets)]
            order = [(me + 1 + i) % W for i in range(W)]  # replicas to the next ranks first
            ag = [heap.addr(j, pall_off + (me * sets + s) * slot) for s in range(sets) for j in order]
            return heap.ptr_tensor(rs), heap.ptr_tensor(ag)

        rs_ptrs, ag_ptrs = cached_for_heap(self._p2p_ptrs, heap, key, build)
        # start with the matrices owned by the next rank: concurrent ranks store to different GPUs
        ops.matmul_to_ptrs(A.to(dt), Qb.to(dt), rs_ptrs, r, torch.float32, rot_b=((me + 1) % W) * sets)
        heap.barrier()
        recv = heap.view(recv_off, (W, sets, pd, r), torch.float32)
        mine = torch.empty((sets, pd, r), device=Mb.device, dtype=torch.float32)
        heap.reduce_slots(recv, mine, W)
        if compressed:
            mine = self._all_reduce_replicate([mine])[0]
        if my_ranks is None and type(self)._orth is Dion._orth:
            orthogonalize(mine, float(group["oversample"]), out_ptrs=ag_ptrs, nrep=W)
        else:
            out = self._orth(mine, group, my_ranks).float().contiguous()
            for s in range(sets):
                heap.push(out[s], ag_ptrs[s * W:(s + 1) * W])
        heap.barrier()
        return heap.view(pall_off, (W * sets, pd, r), torch.float32)

    # ---- FSDP x TP (inner-sharded) parameters
    def _dion_fsdp_tp(self, group: dict, params: List[Tensor], cfg: DionParamConfig) -> None:
        """Inner-sharded update of one same-signature set, batched: P = M Q
        reduced over the mesh dims that shard the contracted dimension (one
        collective for the whole set), orthogonalised across the inner mesh
        with a distributed randomised Cholesky QR, R = M^T P likewise; the
        all-zero guard, error feedback, column norms and weight update run as
        batched kernels on the local shards (adadion_v2.py:1298-1448 does the
        same per matrix)."""
        from .linalg import distributed_orthogonalize

        for p in params:
            if not self.state[p]:
                self._init_dion_states([p], group)
        lr, mu = float(group["lr"]), float(group["mu"])
        wd, eps = float(group["weight_decay"]), float(group["epsilon"])
        rm = self._replicate_mesh
        states = [self.state[p] for p in params]
        Ms = [st["momentum"] for st in states]
        G_loc = [to_local(p.grad) for p in params]
        if self._replicate_mesh_grad_sync and not cfg.compressed_all_reduce and rm is not None:
            G_loc = self._all_reduce_replicate(G_loc)
        M_loc = [to_local(M) for M in Ms]
        nz = ops.dion_momentum_add_(M_loc, G_loc)  # also: 1 per matrix whose momentum is not all zero
        Qds = [st["Q"] for st in states]
        if cfg.Q_inner_unsharded_placements is not None:
            Qds = [Qd.redistribute(placements=cfg.Q_inner_unsharded_placements) for Qd in Qds]
        Mb = torch.stack([M.mT if cfg.is_transposed else M for M in Ms])  # [n, d, k] DTensor
        Qb = torch.stack(Qds).to(Mb.dtype)
        P = Mb @ Qb
        P = P.redistribute(placements=[Replicate() if pl.is_partial() else pl for pl in P.placements])
        P = distributed_orthogonalize(P, float(group["oversample"]), cfg.inner_shard_mesh_dim)
        R = Mb.mT @ P
        R = R.redistribute(placements=[Replicate() if pl.is_partial() else pl for pl in R.placements])
        Pl = to_local(P).float().contiguous()
        Rl = to_local(R).float().contiguous()
        Q0 = to_local(torch.stack(Qds)).float().contiguous()
        ops.dion_fixup_(Pl, Rl, Q0, nz.to(Pl.device))
        dt = self._op_dtype(M_loc[0].dtype)
        # M -= (1 - mu) P R^T (R P^T when transposed), in place on the tcgen05 GEMM, one launch
        if cfg.is_transposed:
            ops.matmul_update_(M_loc, Rl.to(dt), Pl.to(dt).transpose(1, 2), gamma=1.0, delta=-(1.0 - mu))
        else:
            ops.matmul_update_(M_loc, Pl.to(dt), Rl.to(dt).transpose(1, 2), gamma=1.0, delta=-(1.0 - mu))
        sumsq = ops.col_sumsq(Rl)
        if cfg.outer_shard_mesh_dim is not None:
            dist.all_reduce(sumsq, group=R.device_mesh.get_group(cfg.outer_shard_mesh_dim))
        Qn = torch.empty_like(Rl)
        ops.col_normalize(Rl, sumsq, eps, Qn)
        s_lr = self._scaled_lr(params[0].shape, lr)
        X_loc = [to_local(p) for p in params]
        xdt = self._op_dtype(X_loc[0].dtype)
        # X = (1 - lr wd) X - s_lr P Q^T (Q P^T when transposed), in place
        if cfg.is_transposed:
            ops.matmul_update_(X_loc, Qn.to(xdt), Pl.to(xdt).transpose(1, 2), gamma=1.0 - lr * wd, delta=-s_lr)
        else:
            ops.matmul_update_(X_loc, Pl.to(xdt), Qn.to(xdt).transpose(1, 2), gamma=1.0 - lr * wd, delta=-s_lr)
        Qs = Qds[0]
        stacked = [Shard(pl.dim + 1) if pl.is_shard() else pl for pl in Qs.placements]
        target = [Shard(pl.dim + 1) if pl.is_shard() else pl for pl in cfg.Q_sharded_placements]
        Qfull = DTensor.from_local(Qn.to(to_local(Qs).dtype), Qs.device_mesh, stacked, run_check=False,
                                   shape=(len(params),) + tuple(Qs.shape),
                                   stride=(Qs.numel(),) + tuple(Qs.stride()))
        Qnew = to_local(Qfull.redistribute(placements=target))
        for st, q in zip(states, Qnew.unbind(0)):
            to_local(st["Q"]).copy_(q)
