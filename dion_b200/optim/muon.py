"""Muon: momentum + Newton-Schulz orthogonalised updates, FSDP2/DDP aware.

Same public surface as the ``dion`` package's Muon used by the reference
(DION/muon.py:25-178; called from ada_dion/integration/hybrid_optimizer.py:
201-210): torch.optim constructor, param-group ``algorithm`` in
{"muon", "adamw", "lion"}, ``adjust_lr`` in {"spectral_norm", "rms_norm",
"keller_muon", None}, state keys ``momentum`` (+ ``variance`` for AdamW).

B200 design:
  * every same-shape set of matrices is processed as ONE batch: the momentum
    kernel writes the bf16 Newton-Schulz input straight into a stacked
    buffer (and the per-matrix Frobenius sums of squares), one batched
    Newton-Schulz call runs all 5 iterations on tcgen05 tensor cores with the
    normalisation folded into the first GEMM epilogues, and one multi-tensor
    kernel applies the weight update;
  * FSDP (Shard on a 1-D mesh of W ranks): matrices are dealt round-robin to
    ranks in sets of W; shards travel with a single all-to-all per shape
    group each way (the reference issues one per batch of W,
    DION/muon.py:448-491); DDP replicas orthogonalise their own matrices and
    all-gather the results.
"""
from __future__ import annotations

import contextlib
import math
import os
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple, Union

import torch
import torch.distributed as dist
from torch import Tensor
from torch.distributed import ProcessGroup
from torch.distributed.device_mesh import DeviceMesh
from torch.distributed.tensor import DTensor
from torch.optim.optimizer import Optimizer, ParamsT

from .. import ops
from ..utils.trace import phase
from ._utils import StreamPool, group_by_signature, scalar_update, to_local

__all__ = ["Muon", "adjust_lr_spectral_norm", "adjust_lr_rms_norm", "adjust_lr_keller_muon"]


def adjust_lr_spectral_norm(lr: float, shape: Sequence[int]) -> float:
    """Scale for unit RMS-to-RMS operator norm: sqrt(fan_out / fan_in)."""
    fan_out, fan_in = shape[-2:]
    return lr * math.sqrt(fan_out / fan_in)


def adjust_lr_rms_norm(lr: float, shape: Sequence[int]) -> float:
    """Scale matching AdamW's element-wise RMS: 0.2 * sqrt(max(A, B))."""
    a, b = shape[-2:]
    return lr * 0.2 * math.sqrt(max(a, b))


def adjust_lr_keller_muon(lr: float, shape: Sequence[int]) -> float:
    """Keller Jordan's rule: sqrt(max(1, fan_out / fan_in))."""
    fan_out, fan_in = shape[-2:]
    return lr * math.sqrt(max(1.0, fan_out / fan_in))


_NUM_SMS = 148  # B200

_ADJUST = {
    "spectral_norm": adjust_lr_spectral_norm,
    "rms_norm": adjust_lr_rms_norm,
    "keller_muon": adjust_lr_keller_muon,
    None: lambda lr, shape: lr,
}


def _resolve_coeffs(ns_coeffs) -> Tuple[Tuple[float, float, float], ...]:
    if ns_coeffs is None or ns_coeffs == "dion":
        return ops.DION_NS_COEFFS
    if ns_coeffs == "keller":
        return ops.KELLER_NS_COEFFS
    return tuple(tuple(float(x) for x in t) for t in ns_coeffs)


class Muon(Optimizer):
    """Distributed Muon for FSDP2 (DTensor params) and DDP (ProcessGroup).

    Args:
        params: parameters or param groups (groups may set ``algorithm``).
        distributed_mesh: 1-D DeviceMesh (FSDP shard mesh) or ProcessGroup (DDP).
        lr, mu, betas, weight_decay, epsilon, nesterov, adjust_lr, flatten:
            as in the dion package's Muon.
        newton_schulz_func: optional ``f(X, epsilon) -> Tensor`` replacing the
            built-in batched tensor-core Newton-Schulz.
        ns_coeffs: "dion" (per-iteration 5-tuple schedule, default), "keller"
            (3.4445, -4.7750, 2.0315) x 5, or an explicit list of (a, b, c).
        fsdp_mesh_dim, world_mesh: accepted for signature compatibility with
            the expert-parallel fork of Muon; unused for 1-D meshes.
    """

    def __init__(
        self,
        params: ParamsT,
        distributed_mesh: Optional[Union[DeviceMesh, ProcessGroup]] = None,
        lr: float = 0.01,
        mu: float = 0.95,
        betas: Tuple[float, float] = (0.9, 0.95),
        weight_decay: float = 0.01,
        epsilon: float = 1e-8,
        nesterov: bool = False,
        adjust_lr: Optional[str] = "spectral_norm",
        flatten: bool = False,
        use_triton: bool = False,
        newton_schulz_func: Optional[Callable] = None,
        ns_coeffs=None,
        fsdp_mesh_dim: Optional[int] = None,
        world_mesh: Optional[DeviceMesh] = None,
        tp_mesh: Optional[DeviceMesh] = None,
    ):
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}")
        if mu < 0.0:
            raise ValueError(f"Invalid momentum factor (mu): {mu}")
        if len(betas) != 2 or betas[0] < 0.0 or betas[1] < 0.0:
            raise ValueError(f"Invalid betas: {betas}")
        if adjust_lr not in _ADJUST:
            raise ValueError(
                f"Invalid adjust_lr value: {adjust_lr}. Must be 'spectral_norm', 'rms_norm', 'keller_muon', or None."
            )
        if newton_schulz_func is not None and not callable(newton_schulz_func):
            raise TypeError(f"newton_schulz_func must be callable, got {type(newton_schulz_func)}")
        defaults = dict(
            lr=lr,
            mu=mu,
            beta1=betas[0],
            beta2=betas[1],
            weight_decay=weight_decay,
            algorithm="muon",
            step=0,
            epsilon=epsilon,
            nesterov=nesterov,
            flatten=flatten,
            adjust_lr=adjust_lr,
        )
        super().__init__(params, defaults)
        if isinstance(distributed_mesh, DeviceMesh):
            if distributed_mesh.ndim != 1:
                raise ValueError(
                    f"Only 1D DeviceMesh is supported, but got {distributed_mesh.ndim}D. "
                    "For HSDP, provide the 1D sharded sub-mesh."
                )
            self._rank = distributed_mesh.get_local_rank()
            self._world = distributed_mesh.size()
            self._pg = distributed_mesh.get_group()
        elif isinstance(distributed_mesh, ProcessGroup):
            self._rank = dist.get_rank(distributed_mesh)
            self._world = dist.get_world_size(distributed_mesh)
            self._pg = distributed_mesh
        elif distributed_mesh is None:
            self._rank, self._world, self._pg = 0, 1, None
        else:
            raise TypeError(f"Invalid distributed_mesh type: {type(distributed_mesh)}")
        self._distributed_mesh = distributed_mesh
        self._ns_func = newton_schulz_func
        self._p2p_cache: Dict[Tuple, Any] = {}
        self._ddp_parity: Dict[int, int] = {}  # heap uid -> buffer half of its last replicated Newton-Schulz call
        # shape groups run concurrently on a pool of side streams (their GEMMs fill each other's tail SMs);
        # each group then has its own peer-memory heap
        self._streams = StreamPool(3, os.environ.get("DION_B200_SIDE_STREAMS", "1") != "0")
        self._heap_tag = ""
        self._coeffs = _resolve_coeffs(ns_coeffs)
        self.fsdp_mesh_dim = fsdp_mesh_dim
        self._world_mesh = world_mesh
        # tensor-parallel sub-mesh: TP blocks are gathered at the matrix owner so
        # Newton-Schulz sees the whole matrix (not its TP-local block)
        self._tp_pg = tp_mesh.get_group() if isinstance(tp_mesh, DeviceMesh) and tp_mesh.size() > 1 else None
        self._tp = tp_mesh.size() if self._tp_pg is not None else 1

    # ------------------------------------------------------------------ state
    def _state(self, p: Tensor, algo: str) -> Dict[str, Any]:
        st = self.state[p]
        if not st:
            st["momentum"] = torch.zeros_like(p)
            if algo == "adamw":
                st["variance"] = torch.zeros_like(p)
        return st

    # ------------------------------------------------------------------ step
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            group["step"] += 1
        for group in self.param_groups:
            algo = group["algorithm"]
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            if algo == "muon":
                self._muon_group(group, params)
            elif algo in ("adamw", "lion"):
                states = [self._state(p, algo) for p in params]
                scalar_update(algo, params, [p.grad for p in params], states, group)
            else:
                raise ValueError(f"Unknown algorithm: {algo}")
        ops.check_status()
        return loss

    # ------------------------------------------------------------------ muon
    def _ns(self, U: Tensor, scale: Optional[Tensor], eps: float) -> Tensor:
        """Orthogonalise a stacked [n, m, k] batch."""
        if self._ns_func is not None:
            return torch.stack([self._ns_func(u, epsilon=eps) for u in U.unbind(0)]).to(torch.bfloat16)
        return ops.newton_schulz(U, self._coeffs, eps, scale=scale, clobber_input=True)

    def _muon_group(self, group: Dict[str, Any], params: List[Tensor]) -> None:
        for p in params:
            if p.ndim < 2:
                raise ValueError("Muon optimizer only supports matrix parameters.")
        lr = float(group["lr"])
        decay = 1.0 - lr * float(group["weight_decay"])
        mu = float(group["mu"])
        eps = float(group["epsilon"])
        nesterov = bool(group["nesterov"])
        adjust = _ADJUST[group["adjust_lr"]]
        sigs = list(group_by_signature(params).values())
        # Only groups whose Newton-Schulz GEMMs leave most SMs idle go to side streams: the GEMM is a
        # persistent kernel with a static tile schedule, and two full-size ones sharing the SMs
        # stretch each other's tails (measured: 48 x 4096^2 + 48 x 4096 x 14336 ran 19 % slower).
        small = [self._ns_tiles(same) < 2 * _NUM_SMS for same in sigs]
        streams = self._streams.session(to_local(sigs[0][0]).device, sum(small) + (1 if not all(small) else 0))
        side = 0
        for gi, same in enumerate(sigs):
            p0 = same[0]
            adj_lr = adjust(lr, p0.shape)
            states = [self._state(p, "muon") for p in same]
            shard_dim = self._shard_dim(p0)
            shape = "x".join(str(d) for d in p0.shape)
            self._heap_tag = f":{shape}" if streams.active else ""
            if small[gi]:
                side += 1
            with streams.use(side) if small[gi] else contextlib.nullcontext():
                if shard_dim is not None and self._world > 1:
                    with phase(f"muon/fsdp/{shape}"):
                        self._muon_fsdp(same, states, shard_dim, mu, nesterov, eps, decay, adj_lr, group)
                elif self._world > 1 and self._pg is not None:
                    with phase(f"muon/ddp/{shape}"):
                        self._muon_ddp(same, states, mu, nesterov, eps, decay, adj_lr, group)
                else:
                    with phase(f"muon/local/{shape}"):
                        self._muon_local(same, states, mu, nesterov, eps, decay, adj_lr, group)
        streams.join()

    def _ns_tiles(self, same: List[Tensor]) -> int:
        """256 x 256 output tiles of one Newton-Schulz GEMM over the matrices
        this rank orthogonalises for a same-shape group."""
        shape = to_local(same[0]).shape
        m, k = shape[0], int(math.prod(shape[1:]))
        mats = len(same) if self._world <= 1 else -(-len(same) // self._world)
        s_, l_ = min(m, k), max(m, k)
        if isinstance(same[0], DTensor) and self._world > 1:
            s_, l_ = min(same[0].shape[0], k), max(same[0].shape[0], k)
        return mats * (-(-s_ // 256)) * (-(-l_ // 256))

    def _shard_dim(self, p: Tensor) -> Optional[int]:
        if not isinstance(p, DTensor):
            return None
        shards = [(i, pl) for i, pl in enumerate(p.placements) if pl.is_shard() and p.device_mesh.size(i) > 1]
        names = p.device_mesh.mesh_dim_names or ()
        if not isinstance(self._distributed_mesh, DeviceMesh):
            # tensor parallelism alone (no FSDP mesh): the TP blocks are gathered per matrix
            if self._tp_pg is not None and all(names and names[i] == "tp" for i, _ in shards):
                return None
            raise RuntimeError("Must create optimizer with DeviceMesh if using DTensor parameters.")
        if "tp" in names:
            shards = [(i, pl) for i, pl in shards if names[i] != "tp"]
        if not shards:
            return None
        if len(shards) > 1:
            mesh_dim = self.fsdp_mesh_dim if self.fsdp_mesh_dim is not None else (
                names.index("dp_shard") if "dp_shard" in names else 0)
            match = [s for s in shards if s[0] == mesh_dim]
            if not match:
                raise RuntimeError(f"Expected mesh dim {mesh_dim} to be the FSDP shard dim, got {shards}")
            return match[0][1].dim
        return shards[0][1].dim

    @staticmethod
    def _as_matrix(t: Tensor, flatten: bool) -> Tensor:
        if t.ndim == 2:
            return t
        if flatten:
            return t.reshape(t.shape[0], -1)
        return t  # 3-D+ treated as a batch of matrices by the caller

    def _muon_local(self, params, states, mu, nesterov, eps, decay, adj_lr, group) -> None:
        X = to_local(params)
        G = to_local([p.grad for p in params])
        M = to_local([s["momentum"] for s in states])
        shape = X[0].shape
        if X[0].ndim > 2 and not group["flatten"]:
            mats = int(math.prod(shape[:-2]))
            m, k = shape[-2:]
        else:
            mats = 1
            m, k = (shape[0], int(math.prod(shape[1:])))
        n = len(X)
        U = torch.empty((n * mats, m, k), device=X[0].device, dtype=torch.bfloat16)
        Uv = list(U.view(n, mats * m * k).unbind(0))
        _, scale = ops.muon_momentum_(
            [t.view(-1) for t in M], [g.reshape(-1) for g in G], Uv, mu, nesterov, eps
        )
        if mats > 1:
            # per-matrix norms for stacked 3-D params
            scale = None
        tp_dim = self._tp_dim(params[0]) if mats == 1 and X[0].ndim == 2 else None
        if tp_dim is not None:
            # TP without FSDP: every rank of the TP group orthogonalises the whole matrices
            O = self._ns_tp_gathered(U, tp_dim, eps)
        else:
            O = self._ns(U, scale, eps)
        ops.scaled_update_(X, [o.view(shape) for o in O.view(n, *shape).unbind(0)], decay, [adj_lr] * n)

    def _muon_ddp(self, params, states, mu, nesterov, eps, decay, adj_lr, group) -> None:
        W, r = self._world, self._rank
        X = to_local(params)
        G = to_local([p.grad for p in params])
        M = to_local([s["momentum"] for s in states])
        shape = X[0].shape
        m, k = shape[0], int(math.prod(shape[1:]))
        n = len(X)
        sets = (n + W - 1) // W
        dev = X[0].device
        U = torch.zeros((sets * W, m, k), device=dev, dtype=torch.bfloat16)
        _, scale = ops.muon_momentum_(
            [t.view(-1) for t in M], [g.reshape(-1) for g in G], [u.view(-1) for u in U[:n].unbind(0)], mu, nesterov, eps
        )
        full_scale = torch.zeros(sets * W, device=dev, dtype=torch.float32)
        full_scale[:n] = scale
        # matrices s*W + r belong to this rank
        mine = U.view(sets, W, m, k)[:, r].contiguous()
        if self._ns_func is None and self._p2p_ok((m, k), 1, dev):
            O = self._ns_allgather_p2p(mine, full_scale.view(sets, W)[:, r].contiguous(), sets, m, k, eps)[:n]
            ops.scaled_update_(X, [o.view(shape) for o in O.unbind(0)], decay, [adj_lr] * n)
            return
        O_mine = self._ns(mine, full_scale.view(sets, W)[:, r].contiguous(), eps)
        gathered = torch.empty((W, sets, m, k), device=dev, dtype=torch.bfloat16)
        dist.all_gather_into_tensor(gathered.view(W * sets, m, k), O_mine.contiguous(), group=self._pg)
        O = gathered.transpose(0, 1).reshape(sets * W, m, k)[:n]
        ops.scaled_update_(X, [o.view(shape) for o in O.unbind(0)], decay, [adj_lr] * n)

    def _muon_fsdp(self, params, states, shard_dim, mu, nesterov, eps, decay, adj_lr, group) -> None:
        W, r = self._world, self._rank
        X = to_local(params)
        G = to_local([p.grad for p in params])
        M = to_local([s["momentum"] for s in states])
        if params[0].ndim != 2:
            raise NotImplementedError("FSDP Muon supports 2-D matrices")
        if params[0].shape[shard_dim] % W:
            raise ValueError(
                f"Shard dimension {shard_dim} size {params[0].shape[shard_dim]} is not divisible by world size {W}."
            )
        local_shape = tuple(X[0].shape)
        # the matrix assembled over the FSDP mesh (TP-local when TP also shards it)
        full_shape = tuple(s * W if d == shard_dim else s for d, s in enumerate(local_shape))
        tp_dim = self._tp_dim(params[0])
        n = len(X)
        sets = (n + W - 1) // W
        dev = X[0].device
        if tp_dim is None and shard_dim == 0 and self._ns_func is None and self._p2p_ok(full_shape, W, dev):
            self._muon_fsdp_p2p(X, G, M, full_shape, local_shape, n, sets, mu, nesterov, eps, decay, adj_lr)
            return
        # send[j, s] = my shard of matrix s*W + j (goes to rank j)
        send = torch.zeros((W, sets) + local_shape, device=dev, dtype=torch.bfloat16)
        Uv = [send[i % W, i // W].view(-1) for i in range(n)]
        ops.muon_momentum_([t.view(-1) for t in M], [g.reshape(-1) for g in G], Uv, mu, nesterov, eps)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv.view(W, -1), send.view(W, -1), group=self._pg)
        # recv[j, s] = shard j of matrix s*W + r  -> full matrices [sets, m, k]
        full = recv.movedim(0, 1 + shard_dim).reshape((sets,) + full_shape).contiguous()
        if tp_dim is not None:
            O = self._ns_tp_gathered(full, tp_dim, eps)
        else:
            O = self._ns(full, None, eps)
        # split along shard_dim into W shards -> [W, sets, *local_shape]
        chunks = O.view(
            (sets,) + full_shape[:shard_dim] + (W, full_shape[shard_dim] // W) + full_shape[shard_dim + 1 :]
        ).movedim(1 + shard_dim, 0).contiguous()
        ret = torch.empty_like(chunks)
        dist.all_to_all_single(ret.view(W, -1), chunks.view(W, -1), group=self._pg)
        # ret[j, s] = my shard of matrix s*W + j
        upd = [ret[i % W, i // W] for i in range(n)]
        ops.scaled_update_(X, upd, decay, [adj_lr] * n)

    def _tp_dim(self, p: Tensor) -> Optional[int]:
        """Tensor dim sharded over the TP mesh, if any."""
        if self._tp_pg is None or not isinstance(p, DTensor):
            return None
        names = p.device_mesh.mesh_dim_names or ()
        if "tp" not in names:
            return None
        pl = p.placements[names.index("tp")]
        return pl.dim if pl.is_shard() else None

    def _ns_tp_gathered(self, full: Tensor, tp_dim: int, eps: float) -> Tensor:
        """All-gather the TP blocks of each owned matrix, orthogonalise the whole
        matrix (every TP rank of the owner computes the same result), keep this
        rank's block."""
        T = self._tp
        parts = torch.empty((T,) + tuple(full.shape), device=full.device, dtype=full.dtype)
        dist.all_gather_into_tensor(parts.view(T, -1), full.reshape(1, -1), group=self._tp_pg)
        whole = torch.cat(list(parts.unbind(0)), dim=1 + tp_dim).contiguous()
        O = self._ns(whole, None, eps)
        me = dist.get_rank(self._tp_pg)
        return O.narrow(1 + tp_dim, me * full.shape[1 + tp_dim], full.shape[1 + tp_dim]).contiguous()

    # ---- in-kernel all-to-all over symmetric peer memory
    def _p2p_ok(self, full_shape, W: int, dev: torch.device) -> bool:
        from ..parallel.symm import p2p_enabled

        m, k = full_shape
        return p2p_enabled(self._pg, dev) and m % 8 == 0 and k % 8 == 0 and (m // W) % 8 == 0

    def _ns_allgather_p2p(self, mine: Tensor, scale: Tensor, sets: int, m: int, k: int, eps: float) -> Tensor:
        """DDP Muon without NCCL (DION/muon.py:493-520 all-gathers the
        orthogonalised matrices): the last Newton-Schulz GEMM stores each
        result into every rank's [sets, W, m, k] buffer (replicated epilogue
        stores, next ranks first); one device barrier. Successive calls
        alternate between two halves of the buffer: a rank that is still
        reading call t's results cannot be overwritten by call t+1, and call
        t+2 waits behind call t+1's barrier, which that rank reaches only
        after its reads."""
        from ..parallel.symm import cached_for_heap, heap_for

        W, me = self._world, self._rank
        half = sets * W * m * k * 2
        heap = heap_for(self._pg, 2 * half, "muon_ddp" + self._heap_tag, mine.device)
        par = self._ddp_parity[heap.uid] = 1 - self._ddp_parity.get(heap.uid, 1)
        base = par * half
        key = ("ddp", heap.uid, par, sets, m, k)
        order = [(me + 1 + i) % W for i in range(W)]
        ptrs = cached_for_heap(self._p2p_cache, heap, key, lambda: heap.ptr_tensor(
            [heap.addr(j, base + (s_ * W + me) * m * k * 2) for s_ in range(sets) for j in order]))
        ops.newton_schulz(mine, self._coeffs, eps, scale=scale, clobber_input=True, out_ptrs=ptrs, nrep=W)
        heap.barrier()
        return heap.view(base, (sets * W, m, k), torch.bfloat16)

    def _muon_fsdp_p2p(self, X, G, M, full_shape, local_shape, n, sets, mu, nesterov, eps, decay, adj_lr) -> None:
        """Row-sharded FSDP Muon without NCCL (DION/muon.py:448-491 does two all_to_all calls).

        Heap layout (bf16): gather [sets, m, k] (matrices this rank owns) then
        ret [W (owner), sets, m/W, k] (this rank's row shards coming back).
          1. the momentum kernel writes U for matrix i = s*W + j straight into
             rows [me*m/W, (me+1)*m/W) of rank j's gather[s] (P2P stores);
          2. device barrier;
          3. Newton-Schulz on the full matrices; the last GEMM's epilogue
             stores row shard j of matrix s into rank j's ret[me, s];
          4. device barrier; 5. scaled weight update from ret.
        """
        from ..parallel.symm import cached_for_heap, heap_for

        W, me = self._world, self._rank
        m, k = full_shape
        ms = m // W
        mat = m * k * 2
        gather_off, ret_off = 0, sets * mat
        heap = heap_for(self._pg, 2 * sets * mat, "muon" + self._heap_tag, X[0].device)
        key = (heap.uid, sets, m, k)

        def build():
            # peer rows written only by this extension's kernels (the momentum kernel)
            dst_views = [ops.ext().symm_view(heap.addr(i % W, gather_off + (i // W) * mat + me * ms * k * 2),
                                             ms * k, 15) for i in range(n)]
            ptrs = heap.ptr_tensor([heap.addr(j, ret_off + ((me * sets + s_) * ms * k) * 2)
                                    for s_ in range(sets) for j in range(W)])
            return dst_views, ptrs

        dst_views, ptrs = cached_for_heap(self._p2p_cache, heap, key, build)
        full = heap.view(gather_off, (sets, m, k), torch.bfloat16)
        for i in range(n + (-n) % W):
            if i >= n and i % W == me:  # this rank owns an absent matrix of the last set
                full[i // W].zero_()
        ops.muon_momentum_([t.view(-1) for t in M], [g.reshape(-1) for g in G], dst_views, mu, nesterov, eps)
        heap.barrier()
        # row tiles of the next rank's shard first: concurrent ranks scatter to different GPUs
        ops.newton_schulz(full, self._coeffs, eps, clobber_input=False, out_ptrs=ptrs, rows_per_ptr=ms,
                          rot_rows=((me + 1) % W) * ms)
        heap.barrier()
        ret = heap.view(ret_off, (W, sets, ms, k), torch.bfloat16)
        upd = [ret[i % W, i // W] for i in range(n)]
        ops.scaled_update_(X, upd, decay, [adj_lr] * n)
