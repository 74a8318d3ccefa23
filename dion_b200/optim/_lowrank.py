"""Shared engine of the per-matrix Dion-family research optimizers (AdaDion,
SDion, GSDion, AGDion, QCDion).

All five run the same core per matrix (ada_dion/optim/adadion.py:179-366
is the canonical form; sdion.py:152-218, gsdion.py:179-408, agdion.py:
140-316 and qcdion.py:144-318 repeat it with different control policies):

    M <- mu M + G ;  B = M + G                    (AdaDion: B = M + G only)
    non-transposed (rows <= cols sharded):  P = B Q ; gram = P^T P (+1e-6 I)
        P_o = P chol(gram)^-T (QR fallback) ;  R = B^T P_o
        approx = P_o R^T ; Q' = colnorm(R) ; D = P_o Q'^T
    transposed (rows > cols):  P = qr(B^T Q) ;  R = B P ; approx = R P^T ;
        Q' = colnorm(R) (column norms all-reduced) ; D = Q' P^T
    M <- B - (1 - mu) approx ;  X <- (1 - lr wd) X - lr sqrt(dmin/dmax) D

Here that core lives once, in :class:`LowRankEngine`; each optimizer is a
policy class that decides when to refresh, skip, blend or re-rank. The
products run on the package's tcgen05 GEMM for CUDA bf16/fp32 tensors.
Collectives are plain all-reduces over the optimizer's process group, as
in the reference (this family is single-matrix and Python-level by
design).
"""
from __future__ import annotations

import math
from typing import Any, Dict, Iterable, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import Tensor
from torch.distributed.device_mesh import DeviceMesh
from torch.distributed.tensor import DTensor
from torch.optim import Optimizer

from .. import ops

__all__ = ["LowRankEngine", "LowRankOptimizer", "quantize_int", "col_norm"]


def quantize_int(x: float, q: int) -> int:
    """Round to the nearest multiple of q (q <= 1: nearest integer)."""
    return int(round(x / q) * q) if q > 1 else int(round(x))


def _col_kernels(V: Tensor) -> bool:
    return V.is_cuda and V.dim() == 2 and ops.has_ext()


def col_norm(V: Tensor, eps: float = 1e-12) -> Tensor:
    """Unit-norm columns (the column sum-of-squares / normalise kernels on CUDA)."""
    if _col_kernels(V):
        return ops.col_normalize_2d(V, eps)
    return V / torch.linalg.vector_norm(V.float(), dim=0).clamp(min=eps).to(V.dtype)


def _mm(a: Tensor, b: Tensor) -> Tensor:
    """Matrix product on the tcgen05 GEMM for CUDA bf16/fp32 operands."""
    if a.is_cuda and a.dtype == b.dtype and a.dtype in (torch.bfloat16, torch.float32) and ops.has_ext():
        out_dtype = torch.float32 if a.dtype == torch.float32 else torch.bfloat16
        try:
            return ops.matmul(a, b, out_dtype=out_dtype)
        except (ValueError, RuntimeError):
            pass
    return a @ b


class LowRankEngine:
    """Per-matrix low-rank power step and measurements, with an optional
    process group for sharded (FSDP row-sharded) matrices."""

    def __init__(self, pg, mesh_given: bool):
        self.pg = pg
        self.mesh_given = mesh_given

    # ---- collectives (reference: `_ar`, adadion.py:132-136)
    def all_reduce(self, t: Tensor) -> Tensor:
        if self.pg is not None:
            dist.all_reduce(t, group=self.pg)
        elif not self.mesh_given and dist.is_initialized():
            dist.all_reduce(t)
        return t

    def world_size(self) -> int:
        if self.pg is not None:
            return dist.get_world_size(self.pg)
        return dist.get_world_size() if dist.is_initialized() else 1

    def col_norm_dist(self, V: Tensor, eps: float = 1e-12) -> Tensor:
        """Columns normalised by their norms over all row shards (sums of
        squares all-reduced)."""
        if _col_kernels(V):
            sq = ops.col_sumsq(V.float().contiguous().unsqueeze(0)).view(-1)
        else:
            sq = torch.linalg.vector_norm(V.float(), dim=0).pow(2)
        self.all_reduce(sq) if (self.pg is not None or dist.is_initialized()) else None
        if _col_kernels(V):
            return ops.col_normalize_2d(V, eps, sumsq=sq)
        return V / sq.sqrt().clamp(min=eps).to(V.dtype)

    # ---- orthonormal basis of P
    def _orthonormal_rows_sharded(self, Pf: Tensor) -> Tensor:
        """Orthonormal basis of span(P) for a P whose rows may be split over
        the process group: Gram + 1e-6 I, Cholesky, P L^-T, with a QR of P
        when the factor is not finite (adadion.py:258-270). The shift keeps a
        rank-deficient P factorable, as in the reference.

        CUDA: the Gram and P L^-T on the tcgen05 GEMM in 3xTF32 (fp32-level
        accuracy), the blocked Cholesky kernel and the triangular-inverse
        kernel; one host read decides the QR fallback (the reference's own
        check of the factor)."""
        if Pf.is_cuda and ops.has_ext():
            from .linalg import cholesky_lower, tri_inv_lower

            gram = ops.matmul_precise(Pf.T, Pf)  # fp32-accurate: the Cholesky squares its error
            self.all_reduce(gram)
            gram.diagonal().add_(1e-6)
            L = cholesky_lower(gram.unsqueeze(0))
            if bool(torch.isfinite(L).all()):
                Z = tri_inv_lower(L)[0]
                return ops.matmul_precise(Pf, Z.T)
            Po, _ = torch.linalg.qr(Pf)
            return Po
        gram = Pf.T @ Pf
        self.all_reduce(gram)
        gram.diagonal().add_(1e-6)
        L, info = torch.linalg.cholesky_ex(gram)
        if int(info.max().item()) == 0:
            return torch.linalg.solve_triangular(L, Pf.T, upper=False).T
        Po, _ = torch.linalg.qr(Pf)
        return Po

    # ---- power step
    def power_step(self, B: Tensor, Qbuf: Tensor, r: int, tr: bool, ml: int, n: int,
                   anchor: Optional[Tensor] = None, anchor_alpha: float = 0.0):
        """Returns (D, approx, Q_new, R)."""
        dt = B.dtype
        if not tr:
            Qp = Qbuf[:n, :r]
            Pf = _mm(B, Qp.to(dt)).float()
            Po = self._orthonormal_rows_sharded(Pf)
            Pd = Po.to(dt)
            R = _mm(B.float().T.contiguous(), Po).to(dt)
            self.all_reduce(R)
            approx = _mm(Pd, R.T.contiguous())
            Qn = col_norm(R)
            if anchor is not None and anchor_alpha > 0:
                ar = min(r, anchor.shape[1])
                Qn[:, :ar] = (1 - anchor_alpha) * Qn[:, :ar] + anchor_alpha * anchor[:n, :ar]
                Qn = col_norm(Qn)
            D = _mm(Pd, Qn.T.contiguous())
            return D, approx, Qn, R
        Qp = Qbuf[:ml, :r]
        Phf = _mm(B.float().T.contiguous(), Qp.float())
        self.all_reduce(Phf)
        Po, _ = torch.linalg.qr(Phf, mode="reduced")  # Householder: defined for rank-deficient P too
        Pd = Po.to(dt)
        R = _mm(B, Pd)
        approx = _mm(R, Pd.T.contiguous())
        Qn = self.col_norm_dist(R)
        if anchor is not None and anchor_alpha > 0:
            ar = min(r, anchor.shape[1])
            Qn[:, :ar] = (1 - anchor_alpha) * Qn[:, :ar] + anchor_alpha * anchor[:ml, :ar]
            Qn = self.col_norm_dist(Qn)
        D = _mm(Qn, Pd.T.contiguous())
        return D, approx, Qn, R

    def cheap_step(self, B: Tensor, Qbuf: Tensor, r: int, tr: bool, ml: int, n: int):
        """Projection on the cached basis (no power iteration). Returns (D, approx)."""
        if not tr:
            Q = Qbuf[:n, :r]
            D = _mm(_mm(B, Q), Q.T.contiguous())
        else:
            Q = Qbuf[:ml, :r]
            D = _mm(Q, _mm(B.T.contiguous(), Q).T.contiguous())
        return D, D

    # ---- measurements
    def sq_sum(self, X: Tensor) -> Tensor:
        return self.all_reduce(X.float().pow(2).sum())

    def sq_sums(self, *xs: Tensor, reduce: Optional[List[bool]] = None) -> List[float]:
        """Sums of squares of several tensors with ONE all-reduce and ONE
        host read: the per-matrix measurements of a step are packed into a
        vector instead of a blocking collective per quantity. ``reduce[i]``
        False keeps entry i local (a quantity that is already replicated)."""
        v = torch.stack([x.float().pow(2).sum() for x in xs])
        if reduce is None or all(reduce):
            self.all_reduce(v)
        elif any(reduce):
            mask = torch.tensor(reduce, device=v.device)
            part = torch.where(mask, v, torch.zeros_like(v))
            self.all_reduce(part)
            v = torch.where(mask, part, v)
        return v.tolist()

    def rel_residual(self, A: Tensor, B: Tensor) -> float:
        """||A - B||_F / ||A||_F over all shards."""
        num, den = self.sq_sums(A - B, A)
        return math.sqrt(num) / (math.sqrt(den) + 1e-12)

    def tail(self, M: Tensor, Q: Tensor, tr: bool) -> float:
        """||(I - Q Q^T) M||_F / ||M||_F on the basis side of the orientation."""
        proj = _mm(Q, _mm(Q.T.contiguous(), M)) if tr else _mm(_mm(M, Q), Q.T.contiguous())
        t, m = self.sq_sums(M - proj, M)
        return math.sqrt(t) / (math.sqrt(m) + 1e-12)

    def drift(self, Qn: Tensor, anchor: Optional[Tensor], r: int, tr: bool) -> float:
        if anchor is None:
            return 0.0
        d0 = Qn.shape[0]
        ar = min(r, anchor.shape[1])
        d = (Qn[:, :ar] - anchor[:d0, :ar]).float().pow(2).sum()
        if tr:
            self.all_reduce(d)
        return d.sqrt().item()


class LowRankOptimizer(Optimizer):
    """Base class: step dispatch, AdamW groups, per-matrix state init,
    checkpoint world-size stamp and rank/diagnostic getters."""

    WS_KEY = "_lowrank_ws"  # state_dict world-size stamp
    SEED_TAG = 0x4469_6F6E  # Q buffer seed tag (per optimizer)
    DIAG_KEYS: Tuple[str, ...] = ("r",)

    def __init__(self, params, defaults: Dict[str, Any], device_mesh: Optional[DeviceMesh] = None):
        super().__init__(params, defaults)
        self._device_mesh = device_mesh
        self._pg = device_mesh.get_group() if device_mesh is not None else None
        self.engine = LowRankEngine(self._pg, device_mesh is not None)

    # ---- small helpers
    @staticmethod
    def _local(t: Tensor) -> Tensor:
        return t._local_tensor if isinstance(t, DTensor) else t

    def _ws(self) -> int:
        return self.engine.world_size()

    def _is_matrix(self, p: Tensor) -> bool:
        return p.ndim == 2 and p.shape[0] >= 2 and p.shape[1] >= 2

    def _matrix_params(self) -> Iterable[Tuple[int, Tensor]]:
        i = 0
        for g in self.param_groups:
            if g.get("algorithm") == "adamw":
                continue
            for p in g["params"]:
                yield i, p
                i += 1

    # ---- step
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            if g.get("algorithm") == "adamw":
                self._adamw(g)
            else:
                self._matrix_group(g)
        return loss

    def _adamw(self, g: Dict[str, Any]) -> None:
        """AdamW for scalar groups; state keys ``step``, ``m1``, ``m2`` (adadion.py:155-175)."""
        betas = g.get("betas", g.get("adamw_betas", (0.9, 0.95)))
        eps = g.get("eps", g.get("adamw_eps", 1e-8))
        lr, wd = g.get("lr", self.defaults["lr"]), g.get("weight_decay", 0.0)
        by_step: Dict[int, List[Tensor]] = {}
        for p in g["params"]:
            if p.grad is None:
                continue
            s = self.state[p]
            if len(s) == 0:
                s["step"] = 0
                s["m1"] = torch.zeros_like(p)
                s["m2"] = torch.zeros_like(p)
            s["step"] += 1
            by_step.setdefault(s["step"], []).append(p)
        for t, ps in by_step.items():
            X = [self._local(p) for p in ps]
            G = [self._local(p.grad) for p in ps]
            M1 = [self._local(self.state[p]["m1"]) for p in ps]
            M2 = [self._local(self.state[p]["m2"]) for p in ps]
            # m1 <- b1 m1 + (1-b1) g is the lerp form used by the fused kernel
            ops.adamw_(X, G, M1, M2, lr, betas[0], betas[1], wd, eps, t)

    def _matrix_group(self, g: Dict[str, Any]) -> None:
        for p in g["params"]:
            if p.grad is None:
                continue
            if not self._is_matrix(p):
                pl, grad = self._local(p), self._local(p.grad)
                wd, lr = g["weight_decay"], g["lr"]
                if wd:
                    pl.mul_(1 - lr * wd)
                pl.add_(grad, alpha=-lr)
                continue
            self._matrix_step(p, g, self.state[p])

    def _matrix_step(self, p: Tensor, g: Dict[str, Any], st: Dict[str, Any]) -> None:  # pragma: no cover
        raise NotImplementedError

    # ---- state helpers
    def _geometry(self, p: Tensor, g: Dict[str, Any]):
        pl = self._local(p)
        mf, n = tuple(p.shape)
        ml = pl.shape[0]
        dmin, dmax = min(mf, n), max(mf, n)
        ss = math.sqrt(dmin / dmax)
        rc = min(dmin, g["rank_max"])
        return pl, mf, n, ml, ss, rc

    def _init_common(self, p: Tensor, g: Dict[str, Any], st: Dict[str, Any], bc_cap: int) -> None:
        """M, Qbuf (column-normalised seeded Gaussian), r, tr."""
        pl, mf, n, ml, ss, rc = self._geometry(p, g)
        tr = mf > n
        bc = min(rc, bc_cap)
        ir = min(g["init_rank"], rc, bc)
        ws = self._ws()
        if ws > 1 and isinstance(p, DTensor):
            assert mf % ws == 0 and ml == mf // ws
        gen = torch.Generator(device=pl.device)
        gen.manual_seed(self.SEED_TAG + n * 1000 + bc)
        d0 = ml if tr else n
        Qbuf = F.normalize(torch.randn(d0, bc, device=pl.device, dtype=pl.dtype, generator=gen), dim=0)
        re = min(g["rank_min"], rc, bc)
        st["M"] = torch.zeros_like(pl)
        st["Qbuf"] = Qbuf
        st["r"] = int(max(1, min(max(re, ir), rc, bc)))
        st["tr"] = tr
        st["step"] = 0

    def _refill(self, Qbuf: Tensor, lo: int, hi: int, step: int, gen: Optional[torch.Generator] = None) -> None:
        """Fresh unit-norm Gaussian columns [lo, hi) of Qbuf. Without an
        explicit generator the draws are a pure function of (process seed,
        optimizer tag, Qbuf's shape, step, lo, hi), like the initial Qbuf
        (keyed by shape), so every rank and a run resumed from a checkpoint
        draw the same columns (CUDA: the Philox + column-normalise kernels)."""
        if hi <= lo:
            return
        if gen is None:
            ops.keyed_unit_columns_(Qbuf[:, lo:hi], self.SEED_TAG, Qbuf.shape[0], Qbuf.shape[1], step, lo, hi)
            return
        Qbuf[:, lo:hi].copy_(F.normalize(
            torch.randn(Qbuf.shape[0], hi - lo, device=Qbuf.device, dtype=Qbuf.dtype, generator=gen), dim=0))

    @staticmethod
    def _write_q(st: Dict[str, Any], Qn: Tensor, r: int) -> None:
        st["Qbuf"][: Qn.shape[0], :r].copy_(Qn)

    @staticmethod
    def _nan_guard(D: Tensor) -> Tuple[Tensor, bool]:
        if torch.isnan(D).any() or torch.isinf(D).any():
            return torch.zeros_like(D), True
        return D, False

    # ---- checkpoint
    # Per-matrix state entries that hold None until first set (EMAs, anchors).
    # A flattened DCP checkpoint (the container's format) stores only tensors
    # and numbers, so state_dict() leaves out entries that are None (put back
    # by load_state_dict()) and text diagnostics such as SDion's last mode.
    NULLABLE_STATE: Tuple[str, ...] = ()
    # Under FSDP the state is kept as plain local tensors. Entries whose rows
    # follow the parameter's row shard ("always", or "tr" when the matrix is
    # handled transposed so the basis lives on its rows) are checkpointed as
    # DTensors with the parameter's placements, so DCP stores every rank's
    # rows (a plain tensor would be saved once, as if replicated).
    ROW_SHARDED_STATE: Dict[str, str] = {"M": "always", "Dr_ema": "always", "Qbuf": "tr", "Q_anchor": "tr",
                                         "Q_prev_proj": "tr"}

    def _checkpoint_entry(self, p: Tensor, st: Dict[str, Any], k: str, v: Any) -> Any:
        mode = self.ROW_SHARDED_STATE.get(k)
        if not (isinstance(v, Tensor) and isinstance(p, DTensor)) or mode is None or (mode == "tr" and not st.get("tr")):
            return v
        shape = torch.Size((p.shape[0],) + tuple(v.shape[1:]))
        stride = tuple(int(math.prod(shape[i + 1:])) for i in range(len(shape)))
        return DTensor.from_local(v.contiguous(), p.device_mesh, p.placements, run_check=False, shape=shape,
                                  stride=stride)

    def state_dict(self):
        sd = super().state_dict()
        params = [p for g in self.param_groups for p in g["params"]]
        sd["state"] = {k: {n: (self._checkpoint_entry(params[k], st, n, v) if isinstance(k, int) and k < len(params)
                               else v)
                           for n, v in st.items() if v is not None and not isinstance(v, str)}
                       for k, st in sd["state"].items()}
        ws = self._ws()
        if ws > 1:
            sd[self.WS_KEY] = ws
        return sd

    def load_state_dict(self, state_dict):
        sd = dict(state_dict)
        saved = sd.pop(self.WS_KEY, None)
        if saved is not None and saved != self._ws():
            raise RuntimeError(f"Checkpoint world_size={saved} != current {self._ws()}")
        super().load_state_dict(sd)
        for st in self.state.values():
            for k, v in list(st.items()):
                if isinstance(v, DTensor):  # back to this rank's rows
                    st[k] = v.to_local()
            if "M" in st:
                for k in self.NULLABLE_STATE:
                    st.setdefault(k, None)

    # ---- diagnostics
    def get_rank(self) -> Dict[str, int]:
        out = {}
        for i, p in self._matrix_params():
            if self._is_matrix(p) and "r" in self.state[p]:
                out[self._diag_name(i)] = self.state[p]["r"]
        return out

    def _diag_name(self, i: int) -> str:
        return f"p{i}"

    def get_diagnostics(self) -> Dict[str, Any]:
        out = {}
        for i, p in self._matrix_params():
            if not self._is_matrix(p):
                continue
            st = self.state[p]
            for k in self.DIAG_KEYS:
                if k in st:
                    out[f"p{i}/{k.lstrip('_')}"] = st[k]
        return out

    def get_anchor_drift(self) -> Dict[str, float]:
        """||Qbuf - Q_anchor||_F per matrix (0 right after a refresh)."""
        out = {}
        for i, p in self._matrix_params():
            if not self._is_matrix(p):
                continue
            st = self.state[p]
            Qa = st.get("Q_anchor")
            if Qa is not None and "Qbuf" in st:
                r = st.get("r", 0)
                d0 = min(st["Qbuf"].shape[0], Qa.shape[0])
                rc = min(r, Qa.shape[1])
                d = (st["Qbuf"][:d0, :rc] - Qa[:d0, :rc]).norm().item()
                out[self._diag_name(i)] = d if math.isfinite(d) else 0.0
        return out
