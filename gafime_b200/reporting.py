"""Result records of an analysis (same fields as gafime/reporting/report.py:10-57)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

from .backends.base import BackendInfo
from .config import EngineConfig


@dataclass(frozen=True)
class InteractionResult:
    combo: Tuple[int, ...]
    feature_names: Tuple[str, ...]
    metrics: Dict[str, float]


@dataclass(frozen=True)
class StabilityResult:
    combo: Tuple[int, ...]
    metrics_mean: Dict[str, float]
    metrics_std: Dict[str, float]


@dataclass(frozen=True)
class PermutationResult:
    combo: Tuple[int, ...]
    p_values: Dict[str, float]


@dataclass(frozen=True)
class Decision:
    signal_detected: bool
    message: str


@dataclass
class DiagnosticReport:
    config: EngineConfig
    feature_names: List[str]
    interactions: List[InteractionResult] = field(default_factory=list)
    stability: List[StabilityResult] = field(default_factory=list)
    permutations: List[PermutationResult] = field(default_factory=list)
    warnings: List[str] = field(default_factory=list)
    decision: Optional[Decision] = None
    backend: Optional[BackendInfo] = None

    def to_dict(self) -> Dict[str, object]:
        return {
            "config": self.config,
            "feature_names": self.feature_names,
            "interactions": [vars(r) for r in self.interactions],
            "stability": [vars(r) for r in self.stability],
            "permutations": [vars(r) for r in self.permutations],
            "warnings": list(self.warnings),
            "decision": None if self.decision is None else vars(self.decision),
            "backend": None if self.backend is None else vars(self.backend),
        }
