"""Optimizers: Muon, Dion, Dion2, AdaDion, AdaDionV2 and the research
variants SDion, GSDion, AGDion, QCDion, plus the scalar AdamW/Lion rules."""
from __future__ import annotations

import importlib

from .muon import Muon

_LAZY = {
    "oracle": None,
    "Dion": ".dion",
    "DionMixedPrecisionConfig": ".dion",
    "Dion2": ".dion2",
    "AdaDionV2": ".adadion_v2",
    "AdaDion": ".adadion",
    "SDion": ".sdion",
    "GSDion": ".gsdion",
    "AGDion": ".agdion",
    "QCDion": ".qcdion",
}

__all__ = ["Muon"] + [k for k in _LAZY if k != "oracle"]


def __getattr__(name):
    if name == "oracle":
        return importlib.import_module(".oracle", __name__)
    if name in _LAZY:
        mod = importlib.import_module(_LAZY[name], __name__)
        return getattr(mod, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
