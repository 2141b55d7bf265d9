"""Input checks (gafime/utils/arrays.py:8-39, gafime/utils/safety.py:15-27)."""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np

from .config import ComputeBudget


def coerce_inputs(X, y, feature_names: Optional[Sequence[str]] = None, keep_float32: bool = False
                  ) -> Tuple[np.ndarray, np.ndarray, List[str]]:
    """The reference's checks and float64 arrays.  keep_float32: float32 input stays float32
    (the engine's GPU path scores fp32 columns, and fp32 -> fp64 -> fp32 is the identity, so
    the double-size copy would change nothing but the time)."""
    Xa, ya = np.asarray(X), np.asarray(y)
    if Xa.ndim != 2:
        raise ValueError("X must be a 2D array-like of shape (n_samples, n_features).")
    if ya.ndim != 1:
        raise ValueError("y must be a 1D array-like of shape (n_samples,).")
    if Xa.shape[0] != ya.shape[0]:
        raise ValueError("X and y must have the same number of samples.")
    if not (np.issubdtype(Xa.dtype, np.number) and np.issubdtype(ya.dtype, np.number)):
        raise ValueError("X and y must be numeric.")
    if not (np.isfinite(Xa).all() and np.isfinite(ya).all()):
        raise ValueError("X and y must be finite (no NaN or inf).")
    Xa = np.ascontiguousarray(Xa, dtype=np.float32 if keep_float32 and Xa.dtype == np.float32 else np.float64)
    ya = np.ascontiguousarray(ya, dtype=np.float32 if keep_float32 and ya.dtype == np.float32 else np.float64)
    if feature_names is None:
        names = [f"f{i}" for i in range(Xa.shape[1])]
    else:
        names = [str(n) for n in feature_names]
        if len(names) != Xa.shape[1]:
            raise ValueError("feature_names length must match X's feature count.")
    return Xa, ya, names


def estimate_combinations(n_features: int, k: int) -> int:
    return math.comb(n_features, k) if 1 <= k <= n_features else 0


def validate_budget(n_features: int, budget: ComputeBudget) -> List[str]:
    if budget.max_comb_size < 1:
        raise ValueError("max_comb_size must be >= 1.")
    if budget.max_combinations_per_k < 1:
        raise ValueError("max_combinations_per_k must be >= 1.")
    out: List[str] = []
    if budget.top_features_for_higher_k < 1 and budget.max_comb_size > 1:
        out.append("top_features_for_higher_k < 1; higher-order combos will be empty.")
    if budget.max_comb_size > n_features:
        out.append("max_comb_size exceeds feature count; will cap to n_features.")
    return out
