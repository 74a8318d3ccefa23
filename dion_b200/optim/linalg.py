"""Orthogonalisation for Dion's power iteration.

``orthogonalize(P)`` for a batch of fp32 matrices P (b, d, r):
  * d <  r : QR of P (reduced Q), torch.linalg;
  * d >= r : randomised Cholesky QR (the reference's "rcqr",
    ada_dion/optim/adadion_v2.py:1645-1685):
        S ~ N(0, 1/k), k = ceil(oversample*r/128)*128
        R1 = qr(S P).R ;  P = P R1^-1
        R2 = chol(P^T P) ;  P = P R2^-1
The big products (S P, P R^-1, P^T P) run on the tcgen05 tensor cores
(tf32, fp32 accumulate); the r x r / k x r factorisations are the package's
blocked sm_100a kernels (fp32 panels, tcgen05 3xTF32 trailing updates).
Square P (d == r, the reference's QR branch at adadion_v2.py:1660-1662) also
takes the randomised path on the GPU: both give the orthonormal factor of P
up to column signs, and Dion's update P Q^T and error feedback P R^T are
unchanged by a sign flip of a column of P (R = M^T P flips with it).

``distributed_orthogonalize`` is the inner-sharded (TP) variant
(adadion_v2.py:1690-1790): rows of P are split across the inner mesh, the
sketch S P and the Gram P^T P are reduce-scattered so each rank factors one
matrix of the batch, and the triangular factors are all-gathered.
"""
from __future__ import annotations

import itertools
import math
from typing import Optional

import torch
from torch import Tensor
from torch.distributed.tensor import DTensor, Replicate, Shard

from .. import ops

__all__ = ["orthogonalize", "distributed_orthogonalize", "sketch_size", "tri_inv_lower", "tri_inv_upper",
           "cholesky_lower", "cholesky_upper", "qr_r"]


def sketch_size(r: int, oversample: float) -> int:
    return int(math.ceil(oversample * r / 128.0) * 128)


_MAX_KERNEL_DIM = 1600  # the unblocked cluster kernels keep a panel of this many rows in shared memory
_QR_MAX_ROWS = 11200     # blocked QR: panel rows split over at most 8 CTAs of 1400 rows


def _use_kernels(t: Tensor, rows: int) -> bool:
    return t.is_cuda and ops.has_ext() and rows <= _MAX_KERNEL_DIM


def _cuda_ext(t: Tensor) -> bool:
    return t.is_cuda and ops.has_ext()


def tri_inv_lower(S: Tensor, upper: bool = False) -> Tensor:
    """Z = L^-1 (lower) for L = lower(S), or L = upper(S)^T when ``upper``."""
    if _cuda_ext(S):
        Z = torch.empty(S.shape, device=S.device, dtype=S.dtype)
        ops.ext().tri_inv_lower(S.contiguous(), Z, bool(upper))
        return Z
    L = S.mT if upper else S
    eye = torch.eye(S.size(-1), device=S.device, dtype=S.dtype).expand_as(S)
    return torch.linalg.solve_triangular(torch.tril(L), eye, upper=False)


def tri_inv_upper(R: Tensor) -> Tensor:
    """Inverse of a batch of upper-triangular matrices."""
    return tri_inv_lower(R, upper=True).mT


def cholesky_lower(A: Tensor) -> Tensor:
    """Lower Cholesky factor of a batch of SPD matrices; non-SPD matrices give
    NaN entries that the Dion guard later discards (as cholesky_ex does).

    CUDA: blocked right-looking Cholesky whose trailing update (SYRK) runs
    on the tcgen05 GEMM in 3xTF32 (any r with 16-byte rows), else the
    unblocked cluster kernel (r <= 1600)."""
    r = A.size(-1)
    if _cuda_ext(A) and r % 4 == 0:
        L = A.contiguous().clone()
        info = torch.empty(A.size(0), dtype=torch.int32, device=A.device)
        ops.ext().cholesky_blocked(L, info)
        return torch.tril(L)
    if _use_kernels(A, r):
        L = A.contiguous().clone()
        info = torch.empty(A.size(0), dtype=torch.int32, device=A.device)
        ops.ext().cholesky_lower(L, info)
        return torch.tril(L)
    L, _ = torch.linalg.cholesky_ex(A)
    return L


def cholesky_upper(A: Tensor) -> Tensor:
    return cholesky_lower(A).mT


def qr_r(A: Tensor) -> Tensor:
    """R factor (upper) of the Householder QR of a batch of tall matrices.

    CUDA: blocked Householder with the compact-WY trailing update on the
    tcgen05 GEMM in 3xTF32 (n % 4 == 0, m <= 11200), else the unblocked
    cluster kernel (m <= 1600)."""
    m, n = A.size(-2), A.size(-1)
    if _cuda_ext(A) and n % 4 == 0 and m <= _QR_MAX_ROWS:
        W = A.contiguous().clone()
        R = torch.empty(A.size(0), n, n, device=A.device, dtype=A.dtype)
        ops.ext().qr_r_blocked(W, R)
        return R
    if _use_kernels(A, m):
        W = A.contiguous().clone()
        R = torch.empty(A.size(0), n, n, device=A.device, dtype=A.dtype)
        ops.ext().qr_r(W, R)
        return R
    return torch.linalg.qr(A, mode="r")[1]


def _apply_inv_lower_t(P: Tensor, Z: Tensor) -> Tensor:
    """P Z^T (Z lower): the tensor-core GEMM reads Z's rows as a K-major operand."""
    if P.is_cuda:
        return ops.matmul(P, Z.transpose(1, 2))
    return P @ Z.mT


_SKETCH_CALLS = itertools.count()


def _sketch(b: int, k: int, d: int, device, generator: Optional[torch.Generator]) -> Tensor:
    """S ~ N(0, 1/k) of shape [b, k, d]. On the GPU (no explicit generator):
    the package's Philox kernel keyed by the process seed and a call counter,
    so a run is reproducible whatever else consumes torch's RNG."""
    if generator is None and torch.device(device).type == "cuda" and ops.has_ext():
        return ops.philox_normal((b, k, d), torch.initial_seed(), next(_SKETCH_CALLS), math.sqrt(1.0 / k), device)
    S = torch.randn((b, k, d), device=device, dtype=torch.float32, generator=generator)
    return S.mul_(math.sqrt(1.0 / k))


def orthogonalize(P: Tensor, oversample: float = 1.25, generator: Optional[torch.Generator] = None,
                  out_ptrs: Optional[Tensor] = None, nrep: int = 1) -> Optional[Tensor]:
    """Orthonormal-column basis of every P[i] (see module doc).

    With ``out_ptrs`` (CUDA, fp32, int64 device array of ``b * nrep``
    addresses, entry ``i*nrep + j``) the result is not returned: the last
    GEMM's epilogue stores matrix i to all ``nrep`` addresses, which may be
    peer GPUs' memory (the all-gather of the orthonormal P fused into the
    GEMM that produces it).
    """
    assert P.ndim == 3, "Expected a batch of matrices"
    dtype = P.dtype
    Pf = P.float().contiguous()
    b, d, r = Pf.shape
    assert out_ptrs is None or P.is_cuda, "out_ptrs needs CUDA tensors"
    if d < r or (d == r and not (P.is_cuda and ops.has_ext())):
        # wide P (d < r: Q is d x d) is not produced by Dion's rank rule (r <= min(m, n))
        Q, _ = torch.linalg.qr(Pf)
        if out_ptrs is not None:
            Qc = Q.float().contiguous()
            for i in range(b):
                ops.ext().symm_push(Qc[i], out_ptrs[i * nrep:(i + 1) * nrep])
            return None
        return Q.to(dtype)
    k = sketch_size(r, oversample)
    S = _sketch(b, k, d, P.device, generator)
    SP = ops.matmul(S, Pf) if P.is_cuda else S @ Pf
    if P.is_cuda:
        # P <- P R1^-1 with R1 = qr(SP).R ; then CholeskyQR: P <- P chol(P^T P)^-T
        R1 = qr_r(SP)
        Pf = _apply_inv_lower_t(Pf, tri_inv_lower(R1, upper=True))
        PP = ops.matmul(Pf.transpose(1, 2), Pf, symmetric=True)
        L2 = cholesky_lower(PP)
        Z2 = tri_inv_lower(L2)
        if out_ptrs is not None:
            ops.matmul_to_ptrs(Pf, Z2.transpose(1, 2), out_ptrs, r, torch.float32, nrep=nrep)
            return None
        Pf = _apply_inv_lower_t(Pf, Z2)
        return Pf.to(dtype)
    R1 = qr_r(SP)
    Pf = torch.linalg.solve_triangular(R1, Pf, upper=True, left=False)
    PP = Pf.mT @ Pf
    R2 = cholesky_upper(PP)
    Pf = torch.linalg.solve_triangular(R2, Pf, upper=True, left=False)
    return Pf.to(dtype)


def _right_solve(P: Tensor, R: Tensor) -> Tensor:
    """P R^-1 for upper-triangular R."""
    if P.is_cuda:
        return _apply_inv_lower_t(P.contiguous(), tri_inv_lower(R.contiguous(), upper=True))
    return torch.linalg.solve_triangular(R, P, upper=True, left=False)


def distributed_orthogonalize(P: DTensor, oversample: float = 1.25, shard_mesh_dim: Optional[int] = None) -> DTensor:
    """Orthogonalise a batch of row-sharded DTensor matrices (see module doc)."""
    assert isinstance(P, DTensor)
    assert P.ndim >= 3
    dtype = P.dtype
    orig = P.placements
    full_rep = [Replicate() for _ in orig]
    batch_sharded = list(full_rep)
    if shard_mesh_dim is not None:
        batch_sharded[shard_mesh_dim] = Shard(0)
    mesh = P.device_mesh
    d, r = P.shape[-2:]
    if d <= r:
        single = P.redistribute(placements=batch_sharded)
        loc = single.to_local().float()
        if d == r and loc.is_cuda and ops.has_ext() and loc.size(0) > 0:
            Q = orthogonalize(loc.contiguous(), oversample)  # square: the kernels' randomised path
        else:
            Q, _ = torch.linalg.qr(loc, mode="reduced")
        out = DTensor.from_local(Q.to(dtype).contiguous(), mesh, single.placements, run_check=False,
                                 shape=single.shape, stride=single.stride())
        return out.redistribute(placements=orig)
    k = sketch_size(r, oversample)
    P_local = P.to_local().float().contiguous()
    S_local = _sketch(P_local.size(0), k, P_local.size(1), P_local.device, None)
    SP_local = ops.matmul(S_local, P_local) if P_local.is_cuda else S_local @ P_local
    sp_pl = [pl if not (pl.is_shard() and pl.dim == P.ndim - 2) else None for pl in orig]
    from torch.distributed.tensor import Partial

    sp_pl = [Partial() if x is None else x for x in sp_pl]
    SP = DTensor.from_local(SP_local, mesh, sp_pl, run_check=False)
    SP_single = SP.redistribute(placements=batch_sharded)
    R_local = qr_r(SP_single.to_local().float().contiguous())
    bsz = P.shape[0]
    rr_shape, rr_stride = torch.Size((bsz, r, r)), (r * r, r, 1)
    # explicit global shape: with fewer matrices than ranks some local batches are empty
    R = DTensor.from_local(R_local, mesh, SP_single.placements, run_check=False, shape=rr_shape,
                           stride=rr_stride).redistribute(placements=full_rep)
    P_local = _right_solve(P_local, R.to_local().contiguous())
    PP_local = ops.matmul(P_local.transpose(1, 2), P_local, symmetric=True) if P_local.is_cuda else P_local.mT @ P_local
    PP = DTensor.from_local(PP_local, mesh, sp_pl, run_check=False)
    PP_single = PP.redistribute(placements=batch_sharded)
    R2_local = cholesky_upper(PP_single.to_local().contiguous()).contiguous()
    R2 = DTensor.from_local(R2_local, mesh, PP_single.placements, run_check=False, shape=rr_shape,
                            stride=rr_stride).redistribute(placements=full_rep)
    P_local = _right_solve(P_local, R2.to_local().contiguous())
    return DTensor.from_local(P_local.to(dtype).contiguous(), mesh, orig, run_check=False, shape=P.shape,
                              stride=P.stride())
