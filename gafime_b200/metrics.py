"""Metric names and the metric suite handed to backends (gafime/metrics/base.py:13-43).

Scores are computed on the GPU by the backend; the suite only carries which metrics
are wanted and the MI bin count.  ``r2`` is derived as Pearson r squared
(gafime_core.cpp:591-594); ``spearman`` sorts each combo's values on the device
(gafime_core.cpp:595-607).
"""
from __future__ import annotations

from typing import Iterable, Tuple

SUPPORTED_METRICS = ("pearson", "spearman", "mutual_info", "r2")
GPU_METRICS = ("pearson", "spearman", "mutual_info", "r2")


class MetricSuite:
    def __init__(self, metric_names: Iterable[str], mi_bins: int = 16) -> None:
        self.metric_names: Tuple[str, ...] = tuple(metric_names)
        self.mi_bins = int(mi_bins)
        bad = [m for m in self.metric_names if m not in SUPPORTED_METRICS]
        if bad:
            raise ValueError(f"Unsupported metrics: {bad}.")


def metric_strength(metrics) -> float:
    """|r| for correlations, the raw value otherwise; the max over metrics
    (gafime/engine.py:130-137)."""
    vals = [abs(v) if name in ("pearson", "spearman") else v for name, v in metrics.items()]
    return max(vals) if vals else 0.0
