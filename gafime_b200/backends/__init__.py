"""Backend resolution (gafime/backends/__init__.py:14-56) -- GPU only.

The reference falls back CUDA -> Metal -> C++ core -> numpy.  This package has exactly
one backend, the B200 engine; asking for a CPU backend, or a machine without a usable
GPU, raises instead of silently computing somewhere else.
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np

from ..config import EngineConfig
from .base import Backend, BackendInfo
from .native_cuda_backend import NativeCudaBackend

__all__ = ["Backend", "BackendInfo", "NativeCudaBackend", "resolve_backend"]

GPU_NAMES = ("auto", "cuda", "gpu")


def resolve_backend(config: EngineConfig, X: np.ndarray, y: np.ndarray) -> Tuple[Backend, List[str]]:
    requested = (config.backend or "auto").lower()
    if requested not in GPU_NAMES:
        raise ValueError(f"backend {config.backend!r} is not available: gafime_b200 runs on the GPU "
                         f"only (use one of {GPU_NAMES})")
    backend = NativeCudaBackend.from_config(config)
    ok, warnings = backend.check_budget(X, y, config.budget)
    if not ok:
        raise RuntimeError("; ".join(warnings) + " (raise ComputeBudget.vram_budget_mb; there is no CPU fallback)")
    return backend, warnings
