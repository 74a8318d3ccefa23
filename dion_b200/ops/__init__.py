"""Device ops of dion_b200.

CUDA tensors run the hand-written sm_100a kernels of the ``dion_b200._C``
extension; CPU tensors run the plain PyTorch definition of the same op (the
oracle used by the tests). A CUDA tensor never falls back silently: if the
extension is missing the op raises.
"""
from __future__ import annotations

import itertools
import math
from typing import List, Optional, Sequence, Tuple

import torch
from torch import Tensor

from ._ext import ext, has_ext, check_status, clear_status, StatusError  # noqa: F401

__all__ = [
    "matmul",
    "matmul_update_",
    "matmul_to_ptrs",
    "matmul_precise",
    "philox_normal",
    "random_unit_columns_",
    "keyed_unit_columns_",
    "keyed_stream",
    "newton_schulz",
    "muon_momentum_",
    "scaled_update_",
    "adamw_",
    "lion_",
    "multi_sumsq",
    "dion2_select_rows",
    "dion2_gather_decay_",
    "dion2_update_",
    "check_status",
    "clear_status",
    "StatusError",
    "has_ext",
    "KELLER_NS_COEFFS",
    "DION_NS_COEFFS",
]

# Keller Jordan's fixed quintic coefficients (used 5x).
KELLER_NS_COEFFS: Tuple[Tuple[float, float, float], ...] = ((3.4445, -4.7750, 2.0315),) * 5
# Per-iteration schedule used by the dion package's Muon
# (DION/muon.py:676-703 zeropower_via_newtonschulz5).
DION_NS_COEFFS: Tuple[Tuple[float, float, float], ...] = (
    (4.0848, -6.8946, 2.9270),
    (3.9505, -6.3029, 2.6377),
    (3.7418, -5.5913, 2.3037),
    (2.8769, -3.1427, 1.2046),
    (2.8366, -3.0525, 1.2012),
)


def _as3d(t: Tensor) -> Tensor:
    return t if t.dim() == 3 else t.unsqueeze(0)


def _tma_ok(t: Tensor) -> bool:
    """True if a 3-D view has one unit stride and 16-byte aligned other strides."""
    if t.data_ptr() % 16:
        return False
    q = 16 // t.element_size()
    s = t.stride()
    if s[2] == 1:
        inner_ok = s[1] % q == 0 or t.size(1) == 1
    elif s[1] == 1:
        inner_ok = s[2] % q == 0 or t.size(2) == 1
    else:
        return False
    return inner_ok and (t.size(0) == 1 or s[0] % q == 0)


def _tma_operands(A3: Tensor, B3: Tensor) -> Tuple[Tensor, Tensor]:
    """Return views the TMA path accepts, copying into K-major buffers with K
    padded to a 16-byte multiple when a stride is unaligned."""
    if _tma_ok(A3) and _tma_ok(B3):
        return A3, B3
    K = A3.size(-1)
    pad = (-K) % (16 // A3.element_size())
    A3 = torch.nn.functional.pad(A3.contiguous(), (0, pad)) if pad or not _tma_ok(A3) else A3
    if not _tma_ok(A3):
        A3 = torch.nn.functional.pad(A3.contiguous(), (0, pad))
    if pad or not _tma_ok(B3):
        B3 = torch.nn.functional.pad(B3.transpose(1, 2).contiguous(), (0, pad)).transpose(1, 2)
    if not (_tma_ok(A3) and _tma_ok(B3)):
        raise ValueError("dion_b200.ops.matmul: operand layout not supported by TMA")
    return A3, B3


def matmul(
    A: Tensor,
    B: Tensor,
    out: Optional[Tensor] = None,
    *,
    C: Optional[Tensor] = None,
    alpha: float = 1.0,
    beta: float = 0.0,
    symmetric: bool = False,
    out_dtype: torch.dtype = torch.bfloat16,
) -> Tensor:
    """``out = alpha * A @ B + beta * C`` for (batched) ``A`` and ``B``.

    bf16 operands run on the bf16 tensor cores; fp32 operands run on the
    tf32 tensor cores (fp32 accumulate, fp32 output).

    ``A`` is ``[..., M, K]`` and ``B`` is ``[..., K, N]``; either may be a
    transposed view (K- or MN-major storage). With ``symmetric=True`` the
    product is known to be symmetric and only its upper triangle is computed
    on the tensor cores (then mirrored).
    """
    squeeze = A.dim() == 2
    A3, B3 = _as3d(A), _as3d(B)
    batch, M, K = A3.shape
    N = B3.size(-1)
    if A.dtype == torch.float32:
        out_dtype = torch.float32
    if out is None:
        out = torch.empty((batch, M, N), device=A.device, dtype=out_dtype)
    out3 = _as3d(out)
    C3 = _as3d(C) if C is not None else None
    if not A.is_cuda:
        res = alpha * torch.matmul(A3.float(), B3.float())
        if C3 is not None and beta != 0.0:
            res = res + beta * C3.float()
        out3.copy_(res.to(out3.dtype))
        return out3.squeeze(0) if squeeze else out3
    A3, B3 = _tma_operands(A3, B3)
    q_out = 16 // out3.element_size()
    if out3.stride(-1) != 1 or (out3.stride(-2) % q_out and M > 1) or out3.data_ptr() % 16 or \
            (C3 is not None and (C3.stride(-1) != 1 or C3.stride(-2) % q_out or C3.data_ptr() % 16)):
        # output rows not 16-byte aligned: compute into a padded buffer, copy out
        Np = -(-N // q_out) * q_out
        tmp = torch.empty((batch, M, Np), device=A.device, dtype=out3.dtype)[:, :, :N]
        Ct = None
        if C3 is not None and beta != 0.0:
            Ct = torch.empty((batch, M, Np), device=A.device, dtype=out3.dtype)[:, :, :N]
            Ct.copy_(C3)
        ext().gemm(A3, B3, tmp, Ct, float(alpha), float(beta), None, 0, 0, bool(symmetric), False, 1.0, 1.0, 0)
        out3.copy_(tmp)
        return out3.squeeze(0) if squeeze else out3
    ext().gemm(A3, B3, out3, C3, float(alpha), float(beta), None, 0, 0, bool(symmetric), False, 1.0, 1.0, 0)
    return out3.squeeze(0) if squeeze else out3


def _tf32_split(x: Tensor) -> Tuple[Tensor, Tensor]:
    """x = hi + lo with hi exactly representable in tf32 (the low 13 mantissa
    bits cleared) and lo = x - hi exact in fp32."""
    x = x.contiguous()
    hi = (x.view(torch.int32) & -8192).view(torch.float32)
    return hi, x - hi


_PRECISE_KC = 256


def matmul_precise(A: Tensor, B: Tensor) -> Tensor:
    """fp32 ``A @ B`` with about fp32 accuracy on the tf32 tensor cores.

    A B ~ Ahi Bhi + Ahi Blo + Alo Bhi (the dropped Alo Blo term and the tf32
    reading of the lo parts are ~2^-21 relative; Markidis et al. 2018),
    evaluated per K chunk of 256 as ONE GEMM on operands concatenated along
    K ([Ahi | Ahi | Alo] times [Bhi ; Blo ; Bhi]). The tensor cores' fp32
    accumulator drops low bits at every k step, an error that grows with the
    number of steps, so the chunks run as a batch with short accumulators and
    are summed in fp32 afterwards. CPU: plain fp32 matmul."""
    if not A.is_cuda:
        return A.float() @ B.float()
    squeeze = A.dim() == 2
    A3, B3 = _as3d(A.float()), _as3d(B.float())
    b, m, K = A3.shape
    n = B3.size(-1)
    kc = min(_PRECISE_KC, K)
    c = -(-K // kc)
    Ah, Al = _tf32_split(A3)
    Bh, Bl = _tf32_split(B3)
    if c * kc != K:
        pad = c * kc - K
        Ah, Al = (torch.nn.functional.pad(t, (0, pad)) for t in (Ah, Al))
        Bh, Bl = (torch.nn.functional.pad(t, (0, 0, 0, pad)) for t in (Bh, Bl))
    Ah, Al = (t.view(b, m, c, kc).transpose(1, 2) for t in (Ah, Al))
    Bh, Bl = (t.view(b, c, kc, n) for t in (Bh, Bl))
    Acat = torch.cat([Ah, Ah, Al], dim=-1).reshape(b * c, m, 3 * kc)
    Bcat = torch.cat([Bh, Bl, Bh], dim=-2).reshape(b * c, 3 * kc, n)
    out = matmul(Acat, Bcat).view(b, c, m, n)
    out = out[:, 0] if c == 1 else out.sum(dim=1)
    return out[0] if squeeze else out


_SCALAR_TYPE = {torch.float32: 6, torch.bfloat16: 15}
_PTR_CACHE: dict = {}


def _ptr_tensor(ts: Sequence[Tensor]) -> Tensor:
    key = (ts[0].device, tuple(t.data_ptr() for t in ts))
    p = _PTR_CACHE.get(key)
    if p is None:
        if len(_PTR_CACHE) > 4096:
            _PTR_CACHE.clear()
        p = torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64).to(ts[0].device, non_blocking=True)
        _PTR_CACHE[key] = p
    return p


def matmul_update_(
    outs: Sequence[Tensor],
    A: Tensor,
    B: Tensor,
    *,
    gamma: float = 1.0,
    delta: float = 1.0,
    alpha: float = 1.0,
) -> None:
    """In place, for every b: ``outs[b] = gamma * outs[b] + delta * alpha * A[b] @ B[b]``.

    ``outs`` are separate tensors (e.g. parameters) of identical shape and
    row stride; ``A``/``B`` are batched operands. One launch: the kernel
    reads the output addresses from a device pointer array.
    """
    A3, B3 = _as3d(A), _as3d(B)
    assert len(outs) == A3.size(0)
    if not A.is_cuda:
        for o, a, b in zip(outs, A3.unbind(0), B3.unbind(0)):
            o.copy_((gamma * o.float() + delta * alpha * (a.float() @ b.float())).to(o.dtype))
        return
    o0 = outs[0]
    assert all(o.shape == o0.shape and o.stride() == o0.stride() and o.dtype == o0.dtype for o in outs)
    assert o0.dim() == 2 and o0.stride(1) == 1
    q = 16 // o0.element_size()
    if o0.stride(0) % q or any(o.data_ptr() % 16 for o in outs):
        # unaligned parameter rows: product first, then the axpby in place
        prod = matmul(A3, B3, out_dtype=torch.float32)
        for o, pr in zip(outs, prod.unbind(0)):
            o.copy_((gamma * o.float() + delta * alpha * pr).to(o.dtype))
        return
    A3, B3 = _tma_operands(A3, B3)
    ptrs = _ptr_tensor(outs)
    ext().gemm(A3, B3, o0.unsqueeze(0), None, float(alpha), 0.0, None, 0, 0, False, True, float(gamma), float(delta),
               0, ptrs, o0.stride(0), _SCALAR_TYPE[o0.dtype])


def matmul_to_ptrs(
    A: Tensor,
    B: Tensor,
    ptrs: Tensor,
    ldd: int,
    out_dtype: torch.dtype,
    *,
    nrep: int = 1,
    rows_per_ptr: int = 0,
    alpha: float = 1.0,
    rot_b: int = 0,
    rot_rows: int = 0,
) -> None:
    """``alpha * A[b] @ B[b]`` stored through a device pointer array.

    Row ``i`` of batch ``b`` goes to ``ptrs[(b*splits + i//rows_per_ptr)*nrep + rep]``
    (local row ``i % rows_per_ptr``, row stride ``ldd`` elements) for every
    ``rep < nrep``; ``splits = ceil(M / rows_per_ptr)`` (1 when 0). The
    addresses may be peer-GPU memory: the GEMM epilogue then writes each tile
    over NVLink as soon as it leaves the tensor cores. ``rot_b`` /
    ``rot_rows`` rotate the tile order (batch, row tile) so that ranks writing
    to peers concurrently start on different destinations.
    """
    A3, B3 = _as3d(A), _as3d(B)
    assert A.is_cuda and ptrs.is_cuda and ptrs.dtype == torch.int64
    A3, B3 = _tma_operands(A3, B3)
    dummy = torch.empty((1, 1, 1), device=A.device, dtype=out_dtype)
    ext().gemm_ex(A3, B3, dummy, None, float(alpha), 0.0, None, 0, 0, False, False, 1.0, 1.0, 0, ptrs, int(ldd),
                  _SCALAR_TYPE[out_dtype], int(nrep), int(rows_per_ptr), int(rot_b), int(rot_rows))


def _ns_reference(U: Tensor, coeffs: Sequence[Tuple[float, float, float]], eps: float) -> Tensor:
    """Plain PyTorch quintic Newton-Schulz in fp32 (oracle / CPU path)."""
    X = U.float()
    tall = X.size(-2) > X.size(-1)
    if tall:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + eps)
    for a, b, c in coeffs:
        A = X @ X.mT
        Bm = b * A + c * (A @ A)
        X = a * X + Bm @ X
    if tall:
        X = X.mT
    return X


def newton_schulz(
    U: Tensor,
    coeffs: Sequence[Tuple[float, float, float]] = KELLER_NS_COEFFS,
    eps: float = 1e-7,
    *,
    scale: Optional[Tensor] = None,
    out: Optional[Tensor] = None,
    clobber_input: bool = False,
    out_ptrs: Optional[Tensor] = None,
    rows_per_ptr: int = 0,
    rot_rows: int = 0,
    nrep: int = 1,
) -> Tensor:
    """Orthogonalise each matrix of ``U`` (``[batch, m, n]`` or ``[m, n]``).

    ``scale`` (fp32, one value per matrix) is ``1/(||U_b||_F + eps)``; it is
    computed here when not given (the Muon momentum kernel produces it for
    free). Returns bf16.

    With ``out_ptrs`` (int64 device array, ``batch * m/rows_per_ptr``
    addresses) the result is not written to ``out``: the last GEMM stores rows
    ``[j*rows_per_ptr, (j+1)*rows_per_ptr)`` of matrix b at ``out_ptrs[b*splits + j]``
    (row stride n), and with ``nrep`` > 1 to ``out_ptrs[(b*splits + j)*nrep + rep]``
    for every rep. Used to scatter row shards straight to their owner GPUs,
    or to broadcast each result to every GPU.
    """
    squeeze = U.dim() == 2
    U3 = _as3d(U)
    if not U.is_cuda:
        res = _ns_reference(U3, coeffs, eps).to(torch.bfloat16)
        if out is not None:
            _as3d(out).copy_(res)
            return out
        return res.squeeze(0) if squeeze else res
    if U3.dtype != torch.bfloat16 or not U3.is_contiguous():
        U3 = U3.to(torch.bfloat16).contiguous()
        clobber_input = True
    m, n = U3.shape[-2:]
    if out_ptrs is not None:
        assert m % 8 == 0 and n % 8 == 0 and rows_per_ptr >= 0, "pointer-output Newton-Schulz needs 8-aligned shapes"
        if scale is None:
            ss = multi_sumsq(list(U3.unbind(0)))
            scale = 1.0 / (ss.sqrt() + eps)
        out3 = _as3d(out) if out is not None else torch.empty_like(U3)
        flat = [float(x) for abc in coeffs for x in abc]
        ext().newton_schulz_ex(U3, scale.float().contiguous(), flat, out3, bool(clobber_input), out_ptrs,
                               int(rows_per_ptr), int(rot_rows), int(nrep))
        return out3
    if (m % 8) or (n % 8):
        # pad both dims with zeros: orthogonalisation of [[X, 0], [0, 0]] keeps X's block
        pm, pn = (-m) % 8, (-n) % 8
        Up = torch.nn.functional.pad(U3, (0, pn, 0, pm)).contiguous()
        res = newton_schulz(Up, coeffs, eps, scale=scale, clobber_input=True)[..., :m, :n]
        res = res.contiguous()
        if out is not None:
            _as3d(out).copy_(res)
            return out
        return res.squeeze(0) if squeeze else res
    if scale is None:
        ss = multi_sumsq(list(U3.unbind(0)))
        scale = 1.0 / (ss.sqrt() + eps)
    out3 = _as3d(out) if out is not None else torch.empty_like(U3)
    flat = [float(x) for abc in coeffs for x in abc]
    ext().newton_schulz(U3, scale.float().contiguous(), flat, out3, bool(clobber_input))
    return out3.squeeze(0) if (squeeze and out is None) else out3


def multi_sumsq(X: List[Tensor]) -> Tensor:
    """fp32 sum of squares of each tensor (deterministic order)."""
    if not X:
        return torch.empty(0)
    if not X[0].is_cuda:
        return torch.stack([x.float().square().sum() for x in X])
    out = torch.empty(len(X), device=X[0].device, dtype=torch.float32)
    ext().multi_sumsq([x.contiguous() for x in X], out)
    return out


def muon_momentum_(
    M: List[Tensor], G: List[Tensor], U: List[Tensor], mu: float, nesterov: bool, eps: float = 1e-7
) -> Tuple[Tensor, Tensor]:
    """``M = mu*M + G``; ``U = bf16(nesterov ? mu*M + G : M)``.

    Returns ``(sumsq, scale)`` per tensor with ``scale = 1/(||U||_F + eps)``.
    """
    n = len(M)
    if n == 0:
        return torch.empty(0), torch.empty(0)
    if not M[0].is_cuda:
        sumsq = []
        for m, g, u in zip(M, G, U):
            m.mul_(mu).add_(g.to(m.dtype))
            src = m * mu + g.to(m.dtype) if nesterov else m
            u.copy_(src.to(torch.bfloat16))
            sumsq.append(u.float().square().sum())
        ss = torch.stack(sumsq)
        return ss, 1.0 / (ss.sqrt() + eps)
    dev = M[0].device
    sumsq = torch.empty(n, device=dev, dtype=torch.float32)
    scale = torch.empty(n, device=dev, dtype=torch.float32)
    ext().muon_momentum(M, [g.contiguous() for g in G], U, float(mu), bool(nesterov), sumsq, scale, float(eps))
    return sumsq, scale


def scaled_update_(X: List[Tensor], U: List[Tensor], decay: float, lrs: Sequence[float] | Tensor) -> None:
    """``X[i] = decay * X[i] - lrs[i] * U[i]`` in place."""
    if not X:
        return
    if not X[0].is_cuda:
        for i, (x, u) in enumerate(zip(X, U)):
            lr = float(lrs[i])
            x.copy_((decay * x.float() - lr * u.float()).to(x.dtype))
        return
    if not isinstance(lrs, Tensor):
        # staged through pinned memory: an asynchronous copy (a pageable one
        # would make the host wait for the stream's queued work)
        lrs = torch.tensor([float(v) for v in lrs], dtype=torch.float32).pin_memory().to(X[0].device,
                                                                                         non_blocking=True)
    ext().scaled_update(X, [u.contiguous() for u in U], float(decay), lrs.float())


def adamw_(
    X: List[Tensor],
    G: List[Tensor],
    M: List[Tensor],
    V: List[Tensor],
    lr: float,
    beta1: float,
    beta2: float,
    weight_decay: float,
    epsilon: float,
    step: int,
    cautious_wd: bool = False,
) -> None:
    """Fused multi-tensor AdamW (decoupled weight decay, bias-corrected)."""
    if not X:
        return
    if not X[0].is_cuda:
        bc1 = 1 - beta1**step
        bc2s = math.sqrt(1 - beta2**step)
        for x, g, m, v in zip(X, G, M, V):
            gf = g.to(m.dtype)
            m.lerp_(gf, 1 - beta1)
            v.lerp_((gf * gf).to(v.dtype), 1 - beta2)
            upd = m / (v.sqrt() / bc2s + epsilon)
            if cautious_wd:
                mask = (upd * x >= 0).to(x.dtype)
                x.sub_(x * mask * (lr * weight_decay))
            else:
                x.mul_(1 - lr * weight_decay)
            x.sub_((upd * (lr / bc1)).to(x.dtype))
        return
    ext().adamw(X, [g.contiguous() for g in G], M, V, float(lr), float(beta1), float(beta2), float(weight_decay),
                float(epsilon), int(step), bool(cautious_wd))


def lion_(
    X: List[Tensor],
    G: List[Tensor],
    M: List[Tensor],
    lr: float,
    beta1: float,
    beta2: float,
    weight_decay: float,
    cautious_wd: bool = False,
) -> None:
    """Fused multi-tensor Lion."""
    if not X:
        return
    if not X[0].is_cuda:
        for x, g, m in zip(X, G, M):
            gf = g.to(m.dtype)
            u = m.lerp(gf, 1 - beta1).sign_()
            m.lerp_(gf, 1 - beta2)
            if cautious_wd:
                mask = (u * x >= 0).to(x.dtype)
                x.sub_(x * mask * (lr * weight_decay))
            else:
                x.mul_(1 - lr * weight_decay)
            x.sub_((u * lr).to(x.dtype))
        return
    ext().lion(X, [g.contiguous() for g in G], M, float(lr), float(beta1), float(beta2), float(weight_decay),
               bool(cautious_wd))


# ---------------------------------------------------------------- Dion helpers
def dion_momentum_add_(M: List[Tensor], G: List[Tensor]) -> Tensor:
    """``M += G`` for each pair; returns fp32 flags (1 if M is not all zero)."""
    if not M:
        return torch.empty(0)
    if not M[0].is_cuda:
        out = []
        for m, g in zip(M, G):
            m.add_(g.to(m.dtype))
            out.append(float(bool((m != 0).any())))
        return torch.tensor(out, dtype=torch.float32)
    nz = torch.empty(len(M), device=M[0].device, dtype=torch.float32)
    ext().dion_momentum_add([m for m in M], [g.contiguous() for g in G], nz)
    return nz


def dion_fixup_(P: Tensor, R: Tensor, Q0: Tensor, nz: Tensor) -> None:
    """All-zero / NaN guard: ``P = nan_to_num(P)*nz``, ``R = nan_to_num(R)*nz + Q0*(1-nz)`` per matrix."""
    if not P.is_cuda:
        keep = nz.view(-1, 1, 1).to(P.dtype)
        P.copy_(P.nan_to_num() * keep)
        R.copy_(R.nan_to_num() * keep + Q0.to(R.dtype) * (1 - keep))
        return
    ext().dion_fixup(P, R, Q0.contiguous(), nz)


def col_sumsq(R: Tensor) -> Tensor:
    """Per-column sum of squares of each matrix of ``R`` ([b, rows, r] fp32) -> [b, r]."""
    if not R.is_cuda:
        return R.float().square().sum(dim=-2)
    out = torch.empty(R.size(0), R.size(2), device=R.device, dtype=torch.float32)
    ext().col_sumsq(R.contiguous(), out)
    return out


_PHILOX_M = (0xD2511F53, 0xCD9E8D57)
_PHILOX_W = (0x9E3779B9, 0xBB67AE85)
_MASK32 = 0xFFFFFFFF


def _philox_cpu(nblk: int, key: int, stream: int) -> Tensor:
    """Philox-4x32-10 blocks [nblk, 4] (uint32 values in int64), counter
    (j_lo, j_hi, stream_lo, stream_hi), key (key_lo, key_hi)."""
    j = torch.arange(nblk, dtype=torch.int64)
    c = [j & _MASK32, (j >> 32) & _MASK32, torch.full_like(j, stream & _MASK32),
         torch.full_like(j, (stream >> 32) & _MASK32)]
    k0, k1 = key & _MASK32, (key >> 32) & _MASK32
    for _ in range(10):
        p0 = _PHILOX_M[0] * c[0]  # < 2^64: the int64 bit pattern is the unsigned product
        p1 = _PHILOX_M[1] * c[2]
        hi0, lo0 = (p0 >> 32) & _MASK32, p0 & _MASK32
        hi1, lo1 = (p1 >> 32) & _MASK32, p1 & _MASK32
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
        k0 = (k0 + _PHILOX_W[0]) & _MASK32
        k1 = (k1 + _PHILOX_W[1]) & _MASK32
    return torch.stack(c, dim=1)


def philox_normal(shape: Sequence[int], key: int, stream: int, scale: float = 1.0,
                  device: torch.device | str = "cuda") -> Tensor:
    """N(0, scale^2) fp32 values that are a pure function of (key, stream,
    index): Philox-4x32-10 counters (Salmon et al., SC'11) + Box-Muller.
    The same call gives the same values on every rank and launch; the CPU
    version (plain torch integer arithmetic) is the oracle for the kernel."""
    n = 1
    for d in shape:
        n *= int(d)
    key &= (1 << 64) - 1
    stream &= (1 << 64) - 1
    dev = torch.device(device)
    if dev.type == "cuda":
        out = torch.empty(n, device=dev, dtype=torch.float32)
        ext().philox_normal(out, key - (1 << 64) if key >= (1 << 63) else key,
                            stream - (1 << 64) if stream >= (1 << 63) else stream, float(scale))
        return out.view(*shape)
    blocks = _philox_cpu((n + 3) // 4, key, stream)
    u = (blocks.to(torch.float32) + 1.0) * 2.3283064365386963e-10
    ra = torch.sqrt(-2.0 * torch.log(u[:, 0]))
    rb = torch.sqrt(-2.0 * torch.log(u[:, 2]))
    ta, tb = 6.283185307179586 * u[:, 1], 6.283185307179586 * u[:, 3]
    z = torch.stack([ra * torch.cos(ta), ra * torch.sin(ta), rb * torch.cos(tb), rb * torch.sin(tb)], dim=1)
    return (z.reshape(-1)[:n] * scale).view(*shape).to(dev)


def effective_rank(sumsq: Tensor, slots: Tensor, ranks: Tensor) -> Tensor:
    """Entropy effective rank of each selected row of ``sumsq`` ([b, width]
    column sums of squares) over its first ``ranks[i]`` columns -> [n] fp32."""
    if not sumsq.is_cuda:
        rows = sumsq.index_select(0, slots.long()).clamp_min(0).sqrt()
        width = rows.size(1)
        active = torch.arange(width, device=rows.device).unsqueeze(0) < ranks.long().unsqueeze(1)
        sig = torch.where(active, rows + 1e-12, torch.zeros_like(rows))
        prob = sig / (sig.sum(dim=1, keepdim=True) + 1e-12)
        ent = -(torch.where(active, prob * torch.log(prob + 1e-12), torch.zeros_like(prob))).sum(dim=1)
        return torch.exp(ent)
    out = torch.empty(slots.numel(), device=sumsq.device, dtype=torch.float32)
    ext().effective_rank(sumsq.float().contiguous(), slots.long().contiguous(), ranks.int().contiguous(), out)
    return out


def col_normalize(R: Tensor, sumsq: Tensor, eps: float, out: Tensor) -> Tensor:
    """``out = R / (sqrt(sumsq) + eps)`` column-wise, written in ``out``'s dtype."""
    if not R.is_cuda:
        out.copy_((R.float() / (sumsq.unsqueeze(-2).sqrt() + eps)).to(out.dtype))
        return out
    ext().col_normalize(R.contiguous(), sumsq.contiguous(), float(eps), out)
    return out


_REFILL_CALLS = itertools.count()
_REFILL_STREAM_TAG = 0x5146 << 48  # keeps refill streams apart from the sketch's call counter


def random_unit_columns_(Q: Tensor, key: Optional[int] = None, stream: Optional[int] = None) -> Tensor:
    """Fill the 2-D (column-strided allowed) view ``Q`` with unit-norm Gaussian
    columns: Philox normals, column sums of squares, column normalise (three
    kernels, written straight into ``Q``). Keyed by the process seed and a
    call counter unless given, so every rank that makes the same calls gets
    the same columns. CPU tensors use torch's generator."""
    rows, cols = Q.shape
    if rows == 0 or cols == 0:
        return Q
    if not Q.is_cuda:
        z = torch.randn(rows, cols, dtype=torch.float32)
        Q.copy_((z / z.norm(dim=0, keepdim=True).clamp_min(1e-12)).to(Q.dtype))
        return Q
    key = torch.initial_seed() if key is None else key
    stream = _REFILL_STREAM_TAG | next(_REFILL_CALLS) if stream is None else stream
    z = philox_normal((1, rows, cols), key, stream, 1.0, Q.device)
    if Q.stride(1) == 1 and Q.dtype in (torch.float32, torch.bfloat16):
        return col_normalize(z, col_sumsq(z), 1e-12, Q.unsqueeze(0))[0]
    Q.copy_(col_normalize(z, col_sumsq(z), 1e-12, torch.empty_like(z))[0])
    return Q


_KEYED_STREAM_TAG = 0x4B59 << 48  # keyed refills: apart from the counter-keyed streams


def _mix64(x: int) -> int:
    """splitmix64 finaliser (Steele, Lea and Flood, OOPSLA 2014)."""
    m = (1 << 64) - 1
    x = (x + 0x9E3779B97F4A7C15) & m
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & m
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & m
    return x ^ (x >> 31)


def keyed_stream(*parts: int) -> int:
    """A 48-bit stream id that is a pure function of ``parts`` (tagged so it
    never meets the call-counter streams)."""
    h = 0
    for v in parts:
        h = _mix64(h ^ (int(v) & ((1 << 64) - 1)))
    return _KEYED_STREAM_TAG | (h & ((1 << 48) - 1))


def keyed_unit_columns_(Q: Tensor, *parts: int) -> Tensor:
    """Unit-norm Gaussian columns in the 2-D view ``Q`` that are a pure
    function of the process seed and ``parts`` (e.g. a step counter and the
    column range): a run resumed from a checkpoint, and every rank, draws the
    same columns as an uninterrupted run. CUDA: the Philox and column
    kernels; CPU: torch's generator seeded from the same key."""
    rows, cols = Q.shape
    if rows == 0 or cols == 0:
        return Q
    stream = keyed_stream(*parts)
    if Q.is_cuda and has_ext():
        return random_unit_columns_(Q, stream=stream)
    gen = torch.Generator(device=Q.device)
    gen.manual_seed(_mix64(torch.initial_seed() ^ stream) & ((1 << 63) - 1))
    z = torch.randn(rows, cols, device=Q.device, dtype=torch.float32, generator=gen)
    Q.copy_((z / z.norm(dim=0, keepdim=True).clamp_min(1e-12)).to(Q.dtype))
    return Q


def col_normalize_2d(V: Tensor, eps: float = 1e-12, sumsq: Optional[Tensor] = None) -> Tensor:
    """``V`` with unit-norm columns (norms from ``sumsq`` [cols] when given,
    e.g. after an all-reduce), as a new tensor of V's dtype; column kernels
    on CUDA."""
    if not V.is_cuda:
        sq = V.float().square().sum(dim=0) if sumsq is None else sumsq.float()
        return V / sq.sqrt().clamp(min=eps).to(V.dtype)
    Vf = V.float().contiguous().unsqueeze(0)
    sq = col_sumsq(Vf) if sumsq is None else sumsq.float().contiguous().view(1, -1)
    out = torch.empty(V.shape, device=V.device, dtype=V.dtype)
    col_normalize(Vf, sq, eps, out.unsqueeze(0))
    return out


def as_batch(ts: Sequence[Tensor]) -> Optional[Tensor]:
    """If the tensors are equally spaced views of one storage (an arena),
    return the [n, ...] strided view covering them; else None."""
    t0 = ts[0]
    if len(ts) == 1:
        return t0.unsqueeze(0)
    if any(t.shape != t0.shape or t.stride() != t0.stride() or t.dtype != t0.dtype for t in ts):
        return None
    try:
        if any(t.untyped_storage().data_ptr() != t0.untyped_storage().data_ptr() for t in ts):
            return None
    except RuntimeError:
        return None
    es = t0.element_size()
    d = (ts[1].data_ptr() - t0.data_ptr())
    if d <= 0 or d % es:
        return None
    step = d // es
    for i, t in enumerate(ts):
        if t.data_ptr() != t0.data_ptr() + i * d:
            return None
    return t0.as_strided((len(ts),) + tuple(t0.shape), (step,) + tuple(t0.stride()))


# ---------------------------------------------------------------- Dion2 row selection
def _uniform_matrices(ts: Sequence[Tensor]) -> bool:
    t0 = ts[0]
    return (t0.dim() == 2 and t0.stride(1) == 1 and t0.dtype in (torch.float32, torch.bfloat16)
            and all(t.shape == t0.shape and t.stride() == t0.stride() and t.dtype == t0.dtype for t in ts))


def dion2_select_rows(M: Sequence[Tensor], k: int, scores: Optional[Tensor] = None,
                      reduce_scores=None) -> Tuple[Tensor, Tensor]:
    """Top-``k`` rows of each matrix by L1 row norm (or by the given
    ``scores`` [n, rows]); returns ``idx`` [n, k] (int64, ascending rows) and
    ``pos`` [n, rows] (int32 slot of each row in ``idx``, -1 if unselected).
    ``reduce_scores(scores)`` may sum the scores over ranks that hold other
    columns, so that all of them pick the same rows."""
    n = len(M)
    rows, cols = M[0].shape
    dev = M[0].device
    if scores is None:
        scores = torch.empty((n, rows), device=dev, dtype=torch.float32)
        ext().dion2_row_scores(_ptr_tensor(M), rows, cols, M[0].stride(0), _SCALAR_TYPE[M[0].dtype], scores)
    if reduce_scores is not None:
        reduce_scores(scores)
    idx = torch.empty((n, k), device=dev, dtype=torch.int64)
    pos = torch.empty((n, rows), device=dev, dtype=torch.int32)
    ext().dion2_topk_rows(scores.contiguous(), k, idx, pos)
    return idx, pos


def dion2_gather_decay_(M: Sequence[Tensor], idx: Tensor, decay: float) -> Tensor:
    """``sel[b] = bf16(M[b][idx[b]])`` and, in the same pass, ``M[b][idx[b]] *= decay``."""
    n, k = idx.shape
    cols = M[0].shape[1]
    sel = torch.empty((n, k, cols), device=M[0].device, dtype=torch.bfloat16)
    ext().dion2_gather_decay(_ptr_tensor(M), cols, M[0].stride(0), _SCALAR_TYPE[M[0].dtype], idx.contiguous(),
                             float(decay), sel)
    return sel


def dion2_update_(X: Sequence[Tensor], pos: Tensor, U: Tensor, keep: float, alpha: float) -> None:
    """``X[b] = keep * X[b] - alpha * U[b][pos[b][i]]`` on the selected rows,
    ``keep * X[b]`` on the others (one launch over every matrix)."""
    rows, cols = X[0].shape
    ext().dion2_update(_ptr_tensor(X), rows, cols, X[0].stride(0), _SCALAR_TYPE[X[0].dtype], pos.contiguous(),
                       U.contiguous(), float(keep), float(alpha))

