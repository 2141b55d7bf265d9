"""GafimeEngine.analyze (gafime/engine.py:16-171) on the GPU backend.

Same stages and random-generator order as the reference: unary scores -> top features ->
pair plan -> pair scores -> bootstrap stability -> permutation p-values -> decision."""
from __future__ import annotations

from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np

from .backends import resolve_backend
from .config import EngineConfig
from .metrics import metric_strength
from .planning import plan_higher_order, plan_unary, select_top_features
from .reporting import Decision, DiagnosticReport, InteractionResult
from .utils import coerce_inputs, validate_budget
from .validation import PermutationTester, StabilityAnalyzer


class GafimeEngine:
    def __init__(self, config: Optional[EngineConfig] = None) -> None:
        self.config = config or EngineConfig()
        self.metric_suite = None
        self.backend = None

    def analyze(self, X, y, feature_names: Optional[Iterable[str]] = None) -> DiagnosticReport:
        cfg = self.config
        X_arr, y_arr, names = coerce_inputs(X, y, feature_names, keep_float32=True)
        warnings = validate_budget(X_arr.shape[1], cfg.budget)
        backend, more = resolve_backend(cfg, X_arr, y_arr)
        warnings.extend(more)
        self.backend = backend
        self.metric_suite = backend.metric_suite(cfg)
        rng = np.random.default_rng(cfg.random_seed)
        X_dev, y_dev = backend.to_device(X_arr), backend.to_device(y_arr)

        unary, w = plan_unary(X_arr.shape[1], cfg.budget.max_combinations_per_k, rng)
        warnings.extend(w)
        unary_results, unary_scores = self._score_combos(X_dev, y_dev, unary, names)
        strength = {c[0]: metric_strength(m) for c, m in unary_scores.items()}
        top = select_top_features(strength, cfg.budget.top_features_for_higher_k)
        higher, w = plan_higher_order(top, cfg.budget.max_comb_size, cfg.budget.max_combinations_per_k, rng)
        warnings.extend(w)
        higher_results, higher_scores = self._score_combos(X_dev, y_dev, higher, names)

        scores = {**unary_scores, **higher_scores}
        all_combos = unary + higher
        stability = StabilityAnalyzer(self.metric_suite, backend).assess(
            X_dev, y_dev, all_combos, cfg.num_repeats, rng)
        permutations = PermutationTester(self.metric_suite, backend).test(
            X_dev, y_dev, all_combos, cfg.permutation_tests, rng, actual_scores=scores)
        decision = _make_decision(scores, permutations, stability, cfg)
        return DiagnosticReport(config=cfg, feature_names=names,
                                interactions=unary_results + higher_results, stability=stability,
                                permutations=permutations, warnings=warnings, decision=decision,
                                backend=backend.info())

    def _score_combos(self, X, y, combos, names: List[str]):
        combos = list(combos)
        scores = self.backend.score_combos(X, y, combos, self.metric_suite)
        results = [InteractionResult(c, tuple(names[i] for i in c), scores[c]) for c in combos]
        return results, scores


def _make_decision(scores: Dict[Tuple[int, ...], Dict[str, float]], permutations, stability,
                   config: EngineConfig) -> Decision:
    p_map = {r.combo: r.p_values for r in permutations}
    s_map = {r.combo: r.metrics_std for r in stability}
    found = False
    for combo, metrics in scores.items():
        pv, sd = p_map.get(combo, {}), s_map.get(combo, {})
        for name, value in metrics.items():
            p_ok = (not pv) or pv.get(name, 1.0) <= config.permutation_p_threshold
            s_ok = (not sd) or sd.get(name, 1.0) <= config.stability_std_threshold
            if p_ok and s_ok and metric_strength({name: value}) > 0:
                found = True
                break
        if found:
            break
    msg = ("Learnable feature-based signal detected." if found
           else "No learnable feature-based signal detected for this target.")
    return Decision(signal_detected=found, message=msg)
