"""Kernel microbenchmarks: the tcgen05 GEMM (bf16 / tf32, general and
symmetric), batched Newton-Schulz and the fused elementwise kernels, each
against the equivalent PyTorch/cuBLAS call on the same device. CUDA-event
timing after warm-up; inputs larger than L2 where the op allows.

    python -m dion_b200.benchmarks.kernel_bench [--only gemm,ns,...] [--small]

Prints one JSON line per case: ``{"case", "ms", "ref_ms", "tflops" | "gbs", ...}``.
"""
from __future__ import annotations

import argparse
import json

import torch

from .. import ops


def _time(fn, warmup=3, iters=10):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def bench_gemm(small: bool):
    n = 4096 if small else 8192
    out = []
    for dt in (torch.bfloat16, torch.float32):
        A = torch.randn(n, n, device="cuda", dtype=dt)
        B = torch.randn(n, n, device="cuda", dtype=dt)
        C = torch.empty(n, n, device="cuda", dtype=torch.bfloat16 if dt == torch.bfloat16 else torch.float32)
        E = ops.ext()
        mode = E.gemm_pair_mode()
        E.set_gemm_pair_mode(0)
        ms_single = _time(lambda: ops.matmul(A, B, out=C))
        E.set_gemm_pair_mode(1)
        ms_pair = _time(lambda: ops.matmul(A, B, out=C))
        E.set_gemm_pair_mode(mode)
        ms = min(ms_single, ms_pair)
        torch.backends.cuda.matmul.allow_tf32 = True
        ref = _time(lambda: torch.matmul(A, B, out=C))
        torch.backends.cuda.matmul.allow_tf32 = False
        fl = 2 * n**3
        out.append({"case": f"gemm_{'bf16' if dt == torch.bfloat16 else 'tf32'}_{n}^3", "ms": ms, "ref_ms": ref,
                    "tflops": fl / ms / 1e9, "ref_tflops": fl / ref / 1e9,
                    "tflops_1cta": fl / ms_single / 1e9, "tflops_cta_pair": fl / ms_pair / 1e9})
    X = torch.randn(4096, 14336 if not small else 8192, device="cuda", dtype=torch.bfloat16)
    S = torch.empty(4096, 4096, device="cuda", dtype=torch.bfloat16)
    ms = _time(lambda: ops.matmul(X, X.t(), out=S, symmetric=True))
    ref = _time(lambda: torch.matmul(X, X.t(), out=S))
    fl = 2 * 4096 * 4096 * X.shape[1]
    out.append({"case": f"syrk_bf16_4096x{X.shape[1]}", "ms": ms, "ref_ms": ref, "tflops_equiv": fl / ms / 1e9,
                "ref_tflops": fl / ref / 1e9})
    return out


def _ns_torch(U, coeffs, eps=1e-7):
    X = U
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + eps)
    for a, b, c in coeffs:
        A = X @ X.mT
        Bm = b * A + c * (A @ A)
        X = a * X + Bm @ X
    return X


def bench_ns(small: bool):
    out = []
    cases = [(8, 4096, 4096), (4, 4096, 14336)] if not small else [(4, 2048, 2048), (2, 2048, 8192)]
    for b, m, n in cases:
        U = torch.randn(b, m, n, device="cuda", dtype=torch.bfloat16)
        co = ops.KELLER_NS_COEFFS
        E = ops.ext()
        mode = E.gemm_pair_mode()
        times = {}
        for pm in (0, 1):
            E.set_gemm_pair_mode(pm)
            times[pm] = _time(lambda: ops.newton_schulz(U, co), warmup=2, iters=5)
        E.set_gemm_pair_mode(mode)
        ms = min(times.values())
        ref = _time(lambda: _ns_torch(U, co), warmup=2, iters=5)
        fl = 5 * b * (4 * m * m * n + 2 * m**3)  # dense-equivalent FLOPs of the iteration
        out.append({"case": f"newton_schulz_{b}x{m}x{n}", "ms": ms, "ref_ms": ref, "tflops_equiv": fl / ms / 1e9,
                    "ref_tflops": fl / ref / 1e9, "ms_1cta": times[0], "ms_cta_pair": times[1]})
    return out


def bench_elementwise(small: bool):
    out = []
    R, D = (32768, 2048) if not small else (8192, 2048)
    x = torch.randn(R, D, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(D, device="cuda")
    from ..ops import fused

    ms = _time(lambda: fused.rms_norm(x, w, 1e-5))
    ref = _time(lambda: torch.nn.functional.rms_norm(x, (D,), w.bfloat16(), 1e-5))
    out.append({"case": f"rmsnorm_fwd_{R}x{D}", "ms": ms, "ref_ms": ref, "gbs": 2 * x.numel() * 2 / ms / 1e6})
    a = torch.randn(R, 4 * D, device="cuda", dtype=torch.bfloat16)
    bb = torch.randn_like(a)
    ms = _time(lambda: fused.swiglu(a, bb))
    ref = _time(lambda: torch.nn.functional.silu(a) * bb)
    out.append({"case": f"swiglu_fwd_{R}x{4 * D}", "ms": ms, "ref_ms": ref, "gbs": 3 * a.numel() * 2 / ms / 1e6})
    n = 48
    Xs = [torch.randn(1 << 20, device="cuda") for _ in range(n)]
    Gs = [torch.randn(1 << 20, device="cuda") for _ in range(n)]
    Ms = [torch.zeros(1 << 20, device="cuda") for _ in range(n)]
    Vs = [torch.zeros(1 << 20, device="cuda") for _ in range(n)]
    ms = _time(lambda: ops.adamw_(Xs, Gs, Ms, Vs, 1e-3, 0.9, 0.95, 0.1, 1e-8, 3))
    ref_opt = torch.optim.AdamW([torch.nn.Parameter(x.clone()) for x in Xs], lr=1e-3, fused=True)
    for p, g in zip(ref_opt.param_groups[0]["params"], Gs):
        p.grad = g
    ref = _time(lambda: ref_opt.step())
    out.append({"case": f"adamw_{n}x1M_fp32", "ms": ms, "ref_ms": ref, "gbs": n * (1 << 20) * 4 * 7 / ms / 1e6})
    return out


def bench_linalg(small: bool):
    from ..optim import linalg as LA

    out = []
    b, m, r = (8, 1280, 1024) if not small else (4, 640, 512)
    A = torch.randn(b, m, r, device="cuda")
    ms = _time(lambda: LA.qr_r(A), warmup=1, iters=3)
    ref = _time(lambda: torch.linalg.qr(A, mode="r"), warmup=1, iters=3)

    def unblocked_qr():
        W, R = A.clone(), torch.empty(b, r, r, device="cuda")
        ops.ext().qr_r(W, R)

    old = _time(unblocked_qr, warmup=1, iters=3)
    out.append({"case": f"qr_r_{b}x{m}x{r}", "ms": ms, "ref_ms": ref, "unblocked_ms": old})
    if not small:
        A6 = A[:6].contiguous()  # the matrices one rank of 8 factors per shape group (48 matrices)
        out.append({"case": f"qr_r_6x{m}x{r}", "ms": _time(lambda: LA.qr_r(A6), warmup=1, iters=3)})
    G = A.mT @ A / m + torch.eye(r, device="cuda")
    ms = _time(lambda: LA.cholesky_lower(G), warmup=1, iters=3)
    ref = _time(lambda: torch.linalg.cholesky_ex(G), warmup=1, iters=3)

    def unblocked_chol():
        L, info = G.clone(), torch.empty(b, dtype=torch.int32, device="cuda")
        ops.ext().cholesky_lower(L, info)

    old = _time(unblocked_chol, warmup=1, iters=3)
    out.append({"case": f"cholesky_{b}x{r}", "ms": ms, "ref_ms": ref, "unblocked_ms": old})
    L = torch.linalg.cholesky(G)
    ms = _time(lambda: LA.tri_inv_lower(L), warmup=1, iters=3)
    eye = torch.eye(r, device="cuda").expand(b, r, r)
    ref = _time(lambda: torch.linalg.solve_triangular(L, eye, upper=False), warmup=1, iters=3)
    out.append({"case": f"tri_inv_{b}x{r}", "ms": ms, "ref_ms": ref})
    P = torch.randn(b, 4 * r, r, device="cuda")
    ms = _time(lambda: LA.orthogonalize(P), warmup=1, iters=3)
    out.append({"case": f"orthogonalize_rcqr_{b}x{4 * r}x{r}", "ms": ms})
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--only", default="gemm,ns,elementwise")
    p.add_argument("--small", action="store_true")
    a = p.parse_args(argv)
    torch.manual_seed(0)
    fns = {"gemm": bench_gemm, "ns": bench_ns, "elementwise": bench_elementwise, "linalg": bench_linalg}
    for name in a.only.split(","):
        try:
            for rec in fns[name](a.small):
                print(json.dumps(rec), flush=True)
        except Exception as e:  # keep going: one failing case must not hide the others
            print(json.dumps({"case": name, "error": repr(e)[:300]}), flush=True)


if __name__ == "__main__":
    main()
