"""Loader for the in-tree CUDA extension ``dion_b200._C``."""
from __future__ import annotations

import importlib
from typing import Optional

_EXT = None
_ERR: Optional[BaseException] = None


class StatusError(RuntimeError):
    """A kernel gave up on a bounded device-side wait (see common.cuh codes)."""


_CODES = {
    0x101: "GEMM TMA producer wait timed out",
    0x102: "GEMM MMA issuer wait timed out",
    0x103: "GEMM epilogue wait timed out",
    0x201: "peer wait timed out in a communication kernel",
    0x301: "Cholesky factor not positive definite",
}


def _load():
    global _EXT, _ERR
    if _EXT is None and _ERR is None:
        try:
            _EXT = importlib.import_module("dion_b200._C")
        except ImportError as e:  # pragma: no cover - depends on the build
            _ERR = e
    return _EXT


def has_ext() -> bool:
    return _load() is not None


def ext():
    """Return the extension module; raise loudly if it was not built."""
    mod = _load()
    if mod is None:
        raise RuntimeError(
            "dion_b200 CUDA extension is not built (run `python setup.py build_ext --inplace`): " f"{_ERR}"
        )
    return mod


def check_status(clear: bool = True) -> None:
    """Raise :class:`StatusError` if any kernel reported a timeout.

    Reads the host-mapped status word; does not synchronise the device, so
    an error surfaces at the first check after the failing kernel finished.
    """
    mod = _load()
    if mod is None or not _cuda_ok():
        return
    code = mod.status_read()
    if code:
        if clear:
            mod.status_clear()
        raise StatusError(f"dion_b200 device status 0x{code:x}: {_CODES.get(code, 'unknown')}")


def _cuda_ok() -> bool:
    import torch

    return torch.cuda.is_available()


def clear_status() -> None:
    mod = _load()
    if mod is not None and _cuda_ok():
        mod.status_clear()
