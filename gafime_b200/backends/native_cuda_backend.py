"""GPU backend: every score comes from libgafime_cuda.so.

Mirrors NativeCudaBackend (gafime/backends/native_cuda_backend.py:24-468) but replaces its
per-pair loop (one launch + sync per pair, :368-379) with one all-pairs call over the
features the combo list touches, and scores unaries on the GPU too (the reference used
numpy for them, :383-404).  There is no CPU fallback: a failure raises.

The matrix is uploaded once per array (the reference re-uploads matrix and target for
every call, :339-352).  Column subsets and bootstrap resamples are gathered from it on the
device, and a new target (permutation tests) replaces only the target column.
"""
from __future__ import annotations

from typing import Dict, Iterable, Optional, Sequence, Tuple

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
        # the matrix last scored, resident on the device with its column-subset buckets
        self._cache: Optional[_Resident] = None

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
    def _resident(self, X: np.ndarray, y: np.ndarray) -> "_Resident":
        r = self._cache
        if r is not None and r.X is X:
            return r
        self.release()
        self._cache = _Resident(X, y, self.device_id)
        return self._cache

    def release(self) -> None:
        if self._cache is not None:
            self._cache.free()
            self._cache = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    # -- scoring ------------------------------------------------------------------
    def score_combos(self, X, y, combos: Iterable[Tuple[int, ...]], metric_suite: MetricSuite
                     ) -> Dict[Tuple[int, ...], Dict[str, float]]:
        X = np.asarray(X)
        y = np.asarray(y)
        res = self._resident(X, y)
        return self._score(lambda cols: (res.bucket(cols, y), False), combos, metric_suite)

    def score_resampled(self, X, y, rows, combos: Iterable[Tuple[int, ...]], metric_suite: MetricSuite
                        ) -> Dict[Tuple[int, ...], Dict[str, float]]:
        """score_combos(X[rows], y[rows], ...) with the rows gathered on the device from the
        resident matrix (bootstrap stability)."""
        X = np.asarray(X)
        y = np.asarray(y)
        res = self._resident(X, y)
        rows = np.asarray(rows, dtype=np.int64)
        return self._score(lambda cols: (res.gather(cols, y, rows), True), combos, metric_suite)

    def _score(self, bucket_for, combos, metric_suite: MetricSuite):
        combos_list = list(combos)
        if not combos_list:
            return {}
        for m in metric_suite.metric_names:
            if m not in GPU_METRICS:
                raise NotImplementedError(f"metric {m!r} is not on the GPU scoring path")
        if any(len(c) > 2 for c in combos_list):
            raise NotImplementedError("combos of more than two features are not on the GPU path")
        out: Dict[Tuple[int, ...], Dict[str, float]] = {c: {} for c in combos_list}
        unaries = [c for c in combos_list if len(c) == 1]
        pairs = [c for c in combos_list if len(c) == 2]
        if unaries:
            cols = tuple(sorted({c[0] for c in unaries}))
            pos = {f: i for i, f in enumerate(cols)}
            b, temp = bucket_for(cols)
            try:
                cache = {}
                for m in metric_suite.metric_names:
                    base = _BASE[m]
                    if base not in cache:
                        cache[base] = (b.spearman([(i,) for i in range(len(cols))]) if base == "spearman"
                                       else b.unary_scores(base, metric_suite.mi_bins))
                    v = cache[base]
                    for c in unaries:
                        s = float(v[pos[c[0]]])
                        out[c][m] = s * s if m == "r2" else s
            finally:
                if temp:
                    b.free()
        if pairs:
            cols = tuple(sorted({i for c in pairs for i in c}))
            pos = {f: i for i, f in enumerate(cols)}
            f = len(cols)
            need_reverse = self.operator == "divide" and any(pos[a] > pos[c] for a, c in pairs)
            b, temp = bucket_for(cols)
            rb, rtemp = bucket_for(tuple(reversed(cols))) if need_reverse else (None, False)
            try:
                cache = {}
                for m in metric_suite.metric_names:
                    base = _BASE[m]
                    if base == "spearman":
                        # ranks of x_a op x_c in the combo's own orientation
                        if base not in cache:
                            cache[base] = b.spearman([(pos[a], pos[c]) for a, c in pairs], self.operator,
                                                     center=self.center, div_eps=self.div_eps)
                        for p, (a, c) in enumerate(pairs):
                            out[(a, c)][m] = float(cache[base][p])
                        continue
                    if base not in cache:
                        cache[base] = b.scores(self.operator, metric=base, center=self.center,
                                               div_eps=self.div_eps, mi_bins=metric_suite.mi_bins)
                        if need_reverse:
                            # x_a / x_c with a after c: from the column-reversed bucket
                            cache[base + "/rev"] = rb.scores("divide", metric=base, center=self.center,
                                                             div_eps=self.div_eps,
                                                             mi_bins=metric_suite.mi_bins)
                    v = cache[base]
                    rev = cache.get(base + "/rev")
                    for a, c in pairs:
                        i, j = pos[a], pos[c]
                        if i < j:
                            s = float(v[_tri(i, j, f)])
                        elif self.operator == "divide":
                            s = float(rev[_tri(f - 1 - i, f - 1 - j, f)])
                        else:
                            s = float(v[_tri(j, i, f)])
                            if self.operator == "subtract" and base == "pearson":
                                s = -s  # x_a - x_c = -(x_c - x_a)
                        out[(a, c)][m] = s * s if m == "r2" else s
            finally:
                if temp:
                    b.free()
                if rtemp:
                    rb.free()
        return out

    def top_pairs(self, X, y, k: int, metric: str = "pearson", mi_bins: int = 16,
                  ops: Sequence[str] = ()) -> Dict[str, Tuple[np.ndarray, np.ndarray, np.ndarray]]:
        """The k best pairs i<j of all columns per operator, without materialising every score."""
        X = np.asarray(X)
        y = np.asarray(y)
        b = self._resident(X, y).bucket(tuple(range(X.shape[1])), y)
        return b.topk(list(ops) or [self.operator], k, metric=metric, center=self.center,
                      div_eps=self.div_eps, mi_bins=mi_bins)


_BASE = {"pearson": "pearson", "r2": "pearson", "mutual_info": "mutual_info", "spearman": "spearman"}


def _tri(i: int, j: int, f: int) -> int:
    """Row-major upper-triangle index of pair (i, j), i < j."""
    return i * f - i * (i + 1) // 2 + (j - i - 1)


class _Resident:
    """One host matrix uploaded once (all columns + the target it came with), and buckets
    of column subsets gathered from it on the device.  Each bucket remembers which target
    array it holds; a different one replaces only the target column."""

    max_subsets = 4

    def __init__(self, X: np.ndarray, y: np.ndarray, device: int) -> None:
        self.X = X
        n, f = X.shape
        self.all_cols = tuple(range(f))
        self.full = _native.Bucket(n, f, device=device)
        try:
            self.full.upload_rows(X, y)  # transposed to columns on the device
        except Exception:
            self.full.free()
            raise
        self.y_of = {id(self.full): y}
        self.subsets: Dict[Tuple[int, ...], _native.Bucket] = {}

    def _with_target(self, b: _native.Bucket, y: np.ndarray) -> _native.Bucket:
        if self.y_of.get(id(b)) is not y:
            b.set_target(y)
            self.y_of[id(b)] = y
        return b

    def bucket(self, cols: Tuple[int, ...], y: np.ndarray) -> _native.Bucket:
        if cols == self.all_cols:
            return self._with_target(self.full, y)
        b = self.subsets.pop(cols, None)
        if b is None:
            self._with_target(self.full, y)
            b = _native.Bucket.gather(self.full, cols)
            self.y_of[id(b)] = y
            while len(self.subsets) >= self.max_subsets:
                old = self.subsets.pop(next(iter(self.subsets)))
                self.y_of.pop(id(old), None)
                old.free()
        self.subsets[cols] = b  # most recently used last
        return self._with_target(b, y)

    def gather(self, cols: Tuple[int, ...], y: np.ndarray, rows: np.ndarray) -> _native.Bucket:
        """A temporary bucket of rows `rows` of columns `cols` (and of the target y)."""
        self._with_target(self.full, y)
        return _native.Bucket.gather(self.full, cols, rows)

    def free(self) -> None:
        for b in self.subsets.values():
            b.free()
        self.subsets.clear()
        self.full.free()
        self.y_of.clear()
