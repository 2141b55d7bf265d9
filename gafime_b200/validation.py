"""Bootstrap stability and permutation p-values (gafime/validation/stability.py:17-50,
gafime/validation/permutation.py:17-54).  Both re-score through the backend, so every
repeat runs on the GPU: a bootstrap gathers its rows on the device and a permutation
uploads only the permuted target."""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np

from .metrics import MetricSuite
from .reporting import PermutationResult, StabilityResult


class StabilityAnalyzer:
    def __init__(self, metric_suite: MetricSuite, backend) -> None:
        self.metric_suite = metric_suite
        self.backend = backend

    def assess(self, X, y, combos, repeats: int, rng: np.random.Generator) -> List[StabilityResult]:
        if repeats <= 1:
            return []
        combos = list(combos)
        names = self.metric_suite.metric_names
        seen = {c: {m: [] for m in names} for c in combos}
        resampled = getattr(self.backend, "score_resampled", None)
        for _ in range(repeats):
            idx = self.backend.sample_indices(X.shape[0], rng)
            if resampled is not None:
                # the same rows, gathered on the device from the resident matrix
                scores = resampled(X, y, idx, combos, self.metric_suite)
            else:
                scores = self.backend.score_combos(X[idx], y[idx], combos, self.metric_suite)
            for c, ms in scores.items():
                for m, v in ms.items():
                    seen[c][m].append(v)
        return [StabilityResult(c, {m: float(np.mean(v)) for m, v in d.items()},
                                {m: float(np.std(v)) for m, v in d.items()}) for c, d in seen.items()]


def _exceeds_null(null_value: float, actual: float, metric: str) -> bool:
    if metric in ("pearson", "spearman"):
        return abs(null_value) >= abs(actual)
    return null_value >= actual


class PermutationTester:
    def __init__(self, metric_suite: MetricSuite, backend) -> None:
        self.metric_suite = metric_suite
        self.backend = backend

    def test(self, X, y, combos, num_permutations: int, rng: np.random.Generator,
             actual_scores: Optional[Dict[Tuple[int, ...], Dict[str, float]]] = None
             ) -> List[PermutationResult]:
        if num_permutations <= 0:
            return []
        combos = list(combos)
        if actual_scores is None:
            actual_scores = self.backend.score_combos(X, y, combos, self.metric_suite)
        names = self.metric_suite.metric_names
        hits = {c: {m: 0 for m in names} for c in combos}
        for _ in range(num_permutations):
            y_perm = self.backend.permute(y, rng)
            for c, ms in self.backend.score_combos(X, y_perm, combos, self.metric_suite).items():
                for m, v in ms.items():
                    if _exceeds_null(v, actual_scores[c][m], m):
                        hits[c][m] += 1
        return [PermutationResult(c, {m: float((k + 1) / (num_permutations + 1)) for m, k in d.items()})
                for c, d in hits.items()]
