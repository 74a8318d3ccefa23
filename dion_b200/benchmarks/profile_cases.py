"""Small, self-contained launches of each hand-written kernel for profiling
(one case per process; inputs above the 126 MB L2 where the op allows, a
few hundred MB on the device at most). Every case runs its op ``--reps``
times after one warm-up and prints the CUDA-event time of the last launch.

    python -m dion_b200.benchmarks.profile_cases gemm_bf16
    ncu --set full --clock-control none -k regex:gemm_tc -s 1 -c 1 -o prof \\
        python -m dion_b200.benchmarks.profile_cases gemm_bf16
"""
from __future__ import annotations

import argparse
import json
from typing import Callable, Dict

import torch

from .. import ops
from ..ops import fused
from ..optim import linalg as LA

CASES: Dict[str, Callable[[], Callable[[], None]]] = {}


def case(fn):
    CASES[fn.__name__] = fn
    return fn


@case
def gemm_bf16():
    A = torch.randn(8192, 4096, device="cuda", dtype=torch.bfloat16)
    B = torch.randn(4096, 8192, device="cuda", dtype=torch.bfloat16)
    D = torch.empty(8192, 8192, device="cuda", dtype=torch.bfloat16)
    return lambda: ops.matmul(A, B, out=D)


@case
def gemm_tf32():
    A = torch.randn(4096, 4096, device="cuda")
    B = torch.randn(4096, 4096, device="cuda")
    D = torch.empty(4096, 4096, device="cuda")
    return lambda: ops.matmul(A, B, out=D)


@case
def syrk_bf16():
    X = torch.randn(4096, 14336, device="cuda", dtype=torch.bfloat16)
    S = torch.empty(4096, 4096, device="cuda", dtype=torch.bfloat16)
    return lambda: ops.matmul(X, X.t(), out=S, symmetric=True)


@case
def dion_error_feedback():
    """M -= (1 - mu) P R^T in place through the pointer-array PARAM epilogue (8 x 4096 x 4096, r = 1024)."""
    M = [torch.randn(4096, 4096, device="cuda", dtype=torch.bfloat16) for _ in range(8)]
    P = torch.randn(8, 4096, 1024, device="cuda", dtype=torch.bfloat16)
    R = torch.randn(8, 4096, 1024, device="cuda", dtype=torch.bfloat16)
    return lambda: ops.matmul_update_(M, P, R.transpose(1, 2), gamma=1.0, delta=-0.05)


@case
def newton_schulz():
    U = torch.randn(4, 4096, 4096, device="cuda", dtype=torch.bfloat16)
    return lambda: ops.newton_schulz(U, ops.KELLER_NS_COEFFS)


@case
def newton_schulz_2048():
    """The 1B model's 2048 x 2048 group: 32 matrices (short K: the shape that runs furthest below peak)."""
    U = torch.randn(32, 2048, 2048, device="cuda", dtype=torch.bfloat16)
    return lambda: ops.newton_schulz(U, ops.KELLER_NS_COEFFS)


@case
def qr_r():
    A = torch.randn(8, 1280, 1024, device="cuda")
    return lambda: LA.qr_r(A)


@case
def cholesky():
    A = torch.randn(8, 2048, 1024, device="cuda")
    G = A.mT @ A / 2048 + torch.eye(1024, device="cuda")
    return lambda: LA.cholesky_lower(G)


@case
def tri_inv():
    A = torch.randn(8, 2048, 1024, device="cuda")
    L = torch.linalg.cholesky(A.mT @ A / 2048 + torch.eye(1024, device="cuda"))
    return lambda: LA.tri_inv_lower(L)


@case
def col_norms():
    R = torch.randn(8, 4096, 1024, device="cuda")
    Q = torch.empty_like(R)

    def run():
        s = ops.col_sumsq(R)
        ops.col_normalize(R, s, 1e-8, Q)
    return run


@case
def dion_fixup():
    P = torch.randn(8, 4096, 1024, device="cuda")
    R = torch.randn(8, 4096, 1024, device="cuda")
    Q0 = torch.randn(8, 4096, 1024, device="cuda")
    nz = torch.ones(8, device="cuda")
    return lambda: ops.dion_fixup_(P, R, Q0, nz)


@case
def effective_rank():
    s = torch.rand(96, 1024, device="cuda")
    slots = torch.arange(96, device="cuda")
    ranks = torch.full((96,), 1024, device="cuda", dtype=torch.int32)
    return lambda: ops.effective_rank(s, slots, ranks)


@case
def scaled_update():
    X = [torch.randn(4096, 4096, device="cuda", dtype=torch.bfloat16) for _ in range(8)]
    U = [torch.randn(4096, 4096, device="cuda", dtype=torch.bfloat16) for _ in range(8)]
    return lambda: ops.scaled_update_(X, U, 0.999, [0.02] * 8)


@case
def muon_momentum():
    M = [torch.zeros(4096, 4096, device="cuda") for _ in range(8)]
    G = [torch.randn(4096, 4096, device="cuda", dtype=torch.bfloat16) for _ in range(8)]
    U = [torch.empty(4096, 4096, device="cuda", dtype=torch.bfloat16) for _ in range(8)]
    return lambda: ops.muon_momentum_([m.view(-1) for m in M], [g.view(-1) for g in G], [u.view(-1) for u in U],
                                      0.95, False)


@case
def adamw():
    n = 1 << 24
    X = [torch.randn(n, device="cuda") for _ in range(4)]
    G = [torch.randn(n, device="cuda") for _ in range(4)]
    M = [torch.zeros(n, device="cuda") for _ in range(4)]
    V = [torch.zeros(n, device="cuda") for _ in range(4)]
    return lambda: ops.adamw_(X, G, M, V, 1e-3, 0.9, 0.95, 0.1, 1e-8, 3)


@case
def lion():
    n = 1 << 24
    X = [torch.randn(n, device="cuda") for _ in range(4)]
    G = [torch.randn(n, device="cuda") for _ in range(4)]
    M = [torch.zeros(n, device="cuda") for _ in range(4)]
    return lambda: ops.lion_(X, G, M, 1e-4, 0.9, 0.99, 0.1)


@case
def dion_momentum_add():
    """M += G with the per-matrix all-zero flags (8 x 4096^2 fp32 state, bf16 gradients)."""
    M = [torch.zeros(4096, 4096, device="cuda") for _ in range(8)]
    G = [torch.randn(4096, 4096, device="cuda", dtype=torch.bfloat16) for _ in range(8)]
    return lambda: ops.dion_momentum_add_(M, G)


@case
def dion2_select():
    """Dion2 row scores + top-k + gather/decay + sparse update (16 x 4096 x 4096 fp32, fraction 1/4)."""
    M = [torch.randn(4096, 4096, device="cuda") for _ in range(16)]
    X = [torch.randn(4096, 4096, device="cuda") for _ in range(16)]

    def run():
        idx, pos = ops.dion2_select_rows(M, 1024)
        sel = ops.dion2_gather_decay_(M, idx, 0.999)
        ops.dion2_update_(X, pos, sel, 0.999, 0.01)
    return run


@case
def orthogonalize():
    """Dion's randomised Cholesky QR for 6 matrices 4096 x 1024 (one rank of 8, one shape group)."""
    P = torch.randn(6, 4096, 1024, device="cuda")
    return lambda: LA.orthogonalize(P)


@case
def rms_norm():
    x = torch.randn(32768, 2048, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(2048, device="cuda")
    return lambda: fused.rms_norm(x, w, 1e-5)


@case
def swiglu():
    a = torch.randn(32768, 8192, device="cuda", dtype=torch.bfloat16)
    b = torch.randn_like(a)
    return lambda: fused.swiglu(a, b)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("case", choices=sorted(CASES))
    p.add_argument("--reps", type=int, default=2)
    a = p.parse_args(argv)
    torch.manual_seed(0)
    fn = CASES[a.case]()
    fn()  # warm-up (tensor maps, attributes, first-launch costs)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(a.reps):
        e0.record()
        fn()
        e1.record()
    torch.cuda.synchronize()
    ops.check_status()
    print(json.dumps({"case": a.case, "ms_last": e0.elapsed_time(e1)}))


if __name__ == "__main__":
    main()
