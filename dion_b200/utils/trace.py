"""Named phases for profiles: NVTX ranges (Nsight) and ``record_function``
events (PyTorch profiler / Chrome traces).

    with phase("dion/power_p"):
        ...

Free when neither a PyTorch profiler is recording nor ``DION_B200_TRACE=1``
is set, so the optimizers keep their phases on the hot path permanently.
"""
from __future__ import annotations

import contextlib
import os

import torch

__all__ = ["phase", "tracing_enabled"]

_FORCE = os.environ.get("DION_B200_TRACE", "0") == "1"


def tracing_enabled() -> bool:
    return _FORCE or torch.autograd.profiler._is_profiler_enabled


@contextlib.contextmanager
def phase(name: str):
    if not tracing_enabled():
        yield
        return
    nv = torch.cuda.is_available()
    if nv:
        torch.cuda.nvtx.range_push(name)
    try:
        with torch.profiler.record_function(name):
            yield
    finally:
        if nv:
            torch.cuda.nvtx.range_pop()
