"""The backend interface the engine talks to (gafime/backends/base.py:23-89)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np

from ..config import ComputeBudget, EngineConfig
from ..metrics import MetricSuite


@dataclass(frozen=True)
class BackendInfo:
    name: str
    device: str
    is_gpu: bool
    memory_total_mb: Optional[int]
    memory_free_mb: Optional[int]


class Backend:
    """Interface only: every concrete backend of this package runs on the GPU."""

    name = "abstract"
    device_label = "none"
    is_gpu = False

    def metric_suite(self, config: EngineConfig) -> MetricSuite:
        return MetricSuite(config.metric_names, mi_bins=config.mi_bins)

    def info(self) -> BackendInfo:
        return BackendInfo(self.name, self.device_label, self.is_gpu, None, None)

    def check_budget(self, X: np.ndarray, y: np.ndarray, budget: ComputeBudget) -> Tuple[bool, List[str]]:
        return True, []

    def to_device(self, array: np.ndarray) -> np.ndarray:
        return np.asarray(array)

    def to_host(self, array: np.ndarray) -> np.ndarray:
        return np.asarray(array)

    def score_combos(self, X: np.ndarray, y: np.ndarray, combos: Iterable[Tuple[int, ...]],
                     metric_suite: MetricSuite) -> Dict[Tuple[int, ...], Dict[str, float]]:
        raise NotImplementedError

    def sample_indices(self, n_samples: int, rng: np.random.Generator):
        return rng.integers(0, n_samples, size=n_samples)

    def permute(self, y, rng: np.random.Generator):
        return y[rng.permutation(y.shape[0])]
