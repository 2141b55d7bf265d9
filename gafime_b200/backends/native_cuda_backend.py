"""GPU backend: every score comes from libgafime_cuda.so.

Mirrors NativeCudaBackend (gafime/backends/native_cuda_backend.py:24-468) but replaces its
per-pair loop (one launch + sync per pair, :368-379) with one all-pairs call over the
features the combo list touches, and scores unaries on the GPU too (the reference used
numpy for them, :383-404).  There is no CPU fallback: a failure raises.
"""
from __future__ import annotations

from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from .. import _native
from ..config import ComputeBudget, EngineConfig
from ..metrics import GPU_METRICS, MetricSuite
from .base import Backend, BackendInfo


class NativeCudaBackend(Backend):
    name = "cuda-b200"
    device_label = "cuda"
    is_gpu = True

    def __init__(self, device_id: int = 0, operator: str = "multiply", center: bool = True,
                 div_eps: float = 1e-8) -> None:
        _native.load()
        if operator not in ("multiply", "add", "subtract", "divide"):
            raise ValueError(f"unsupported operator {operator!r}")
        self.device_id = int(device_id)
        self.operator = operator
        self.center = bool(center)
        self.div_eps = float(div_eps)
        info = _native.device_info(self.device_id)
        self._device_name = info["name"]
        self._memory_mb = info["memory_mb"]
        self._cc = info["compute_capability"]
        self.device_label = f"cuda:{self.device_id}"
        # one resident bucket, reused while the same arrays and columns are scored
        self._cache: Optional[Tuple[object, object, Tuple[int, ...], _native.Bucket]] = None

    @classmethod
    def from_config(cls, config: EngineConfig) -> "NativeCudaBackend":
        return cls(config.device_id, config.operator, config.center, config.div_eps)

    def info(self) -> BackendInfo:
        return BackendInfo(self.name, f"{self._device_name} (SM{self._cc[0]}.{self._cc[1]})", True,
                           self._memory_mb, None)

    def check_budget(self, X, y, budget: ComputeBudget):
        if not budget.keep_in_vram:
            return False, ["keep_in_vram is False; the GPU engine needs the matrix resident."]
        n, f = np.shape(X)
        need_mb = ((f + 1) * ((n + 255) // 256 * 256) * 4) / (1024 * 1024)
        if budget.vram_budget_mb > 0 and need_mb > budget.vram_budget_mb:
            return False, [f"VRAM budget exceeded ({need_mb:.1f}MB > {budget.vram_budget_mb}MB)."]
        warnings = []
        if need_mb > 0.8 * self._memory_mb:
            warnings.append(f"Data may exceed GPU memory ({need_mb:.1f}MB / {self._memory_mb}MB).")
        return True, warnings

    # -- buckets ------------------------------------------------------------------
    def _bucket(self, X: np.ndarray, y: np.ndarray, cols: Tuple[int, ...]) -> _native.Bucket:
        c = self._cache
        if c is not None and c[0] is X and c[1] is y and c[2] == cols:
            return c[3]
        self.release()
        sub = X[:, list(cols)] if len(cols) != X.shape[1] or list(cols) != list(range(X.shape[1])) else X
        b = _native.Bucket(X.shape[0], len(cols), device=self.device_id)
        b.upload(np.asarray(sub, dtype=np.float32), np.asarray(y, dtype=np.float32))
        self._cache = (X, y, cols, b)
        return b

    def release(self) -> None:
        if self._cache is not None:
            self._cache[3].free()
            self._cache = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    # -- scoring ------------------------------------------------------------------
    def score_combos(self, X, y, combos: Iterable[Tuple[int, ...]], metric_suite: MetricSuite
                     ) -> Dict[Tuple[int, ...], Dict[str, float]]:
        combos_list = list(combos)
        if not combos_list:
            return {}
        for m in metric_suite.metric_names:
            if m not in GPU_METRICS:
                raise NotImplementedError(f"metric {m!r} is not on the GPU scoring path")
        if any(len(c) > 2 for c in combos_list):
            raise NotImplementedError("combos of more than two features are not on the GPU path")
        X = np.asarray(X)
        y = np.asarray(y)
        out: Dict[Tuple[int, ...], Dict[str, float]] = {c: {} for c in combos_list}
        unaries = [c for c in combos_list if len(c) == 1]
        pairs = [c for c in combos_list if len(c) == 2]
        if unaries:
            cols = tuple(sorted({c[0] for c in unaries}))
            pos = {f: i for i, f in enumerate(cols)}
            b = self._bucket(X, y, cols)
            cache = {}
            for m in metric_suite.metric_names:
                base = "pearson" if m in ("pearson", "r2") else "mutual_info"
                if base not in cache:
                    cache[base] = b.unary_scores(base, metric_suite.mi_bins)
                v = cache[base]
                for c in unaries:
                    s = float(v[pos[c[0]]])
                    out[c][m] = s * s if m == "r2" else s
        if pairs:
            cols = tuple(sorted({i for c in pairs for i in c}))
            pos = {f: i for i, f in enumerate(cols)}
            b = self._bucket(X, y, cols)
            f = len(cols)
            need_reverse = self.operator == "divide" and any(pos[a] > pos[c] for a, c in pairs)
            cache = {}
            for m in metric_suite.metric_names:
                base = "pearson" if m in ("pearson", "r2") else "mutual_info"
                if base not in cache:
                    cache[base] = b.scores(self.operator, metric=base, center=self.center,
                                           div_eps=self.div_eps, mi_bins=metric_suite.mi_bins)
                v = cache[base]
                rev = None
                if need_reverse:
                    rev = self._reverse_divide_scores(X, y, cols, base, metric_suite.mi_bins)
                for a, c in pairs:
                    i, j = pos[a], pos[c]
                    if i < j:
                        s = float(v[_tri(i, j, f)])
                    elif self.operator == "divide":
                        # x_a / x_c with a after c: from the column-reversed bucket
                        s = float(rev[_tri(f - 1 - i, f - 1 - j, f)])
                    else:
                        s = float(v[_tri(j, i, f)])
                        if self.operator == "subtract" and base == "pearson":
                            s = -s  # x_a - x_c = -(x_c - x_a)
                    out[(a, c)][m] = s * s if m == "r2" else s
        return out

    def _reverse_divide_scores(self, X, y, cols, base, bins):
        rcols = tuple(reversed(cols))
        sub = np.asarray(X[:, list(rcols)], dtype=np.float32)
        with _native.Bucket(X.shape[0], len(rcols), device=self.device_id) as b:
            b.upload(sub, np.asarray(y, dtype=np.float32))
            return b.scores("divide", metric=base, center=self.center, div_eps=self.div_eps,
                            mi_bins=bins)

    def top_pairs(self, X, y, k: int, metric: str = "pearson", mi_bins: int = 16,
                  ops: Sequence[str] = ()) -> Dict[str, Tuple[np.ndarray, np.ndarray, np.ndarray]]:
        """The k best pairs i<j of all columns per operator, without materialising every score."""
        cols = tuple(range(np.shape(X)[1]))
        b = self._bucket(np.asarray(X), np.asarray(y), cols)
        return b.topk(list(ops) or [self.operator], k, metric=metric, center=self.center,
                      div_eps=self.div_eps, mi_bins=mi_bins)


def _tri(i: int, j: int, f: int) -> int:
    """Row-major upper-triangle index of pair (i, j), i < j."""
    return i * f - i * (i + 1) // 2 + (j - i - 1)
