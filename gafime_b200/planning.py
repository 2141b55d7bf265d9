"""Which combos get scored (gafime/planning/combinations.py:11-63).

The random generator is consumed in the same order as the reference (shuffle of the
unary list only when capped, then one shuffle of the selected features before pair
enumeration), so a given seed plans the same pairs."""
from __future__ import annotations

import itertools
from typing import Dict, List, Sequence, Tuple

import numpy as np


def plan_unary(n_features: int, max_count: int, rng: np.random.Generator):
    idx = list(range(n_features))
    if n_features <= max_count:
        return [(i,) for i in idx], []
    rng.shuffle(idx)
    return [(i,) for i in idx[:max_count]], ["Unary combinations capped by max_combinations_per_k."]


def select_top_features(feature_scores: Dict[int, float], top_n: int) -> List[int]:
    if top_n <= 0:
        return []
    ranked = sorted(feature_scores.items(), key=lambda kv: kv[1], reverse=True)
    return [i for i, _ in ranked[:top_n]]


def plan_higher_order(feature_indices: Sequence[int], max_comb_size: int,
                      max_combinations_per_k: int, rng: np.random.Generator):
    warnings: List[str] = []
    if max_comb_size < 2 or not feature_indices:
        return [], warnings
    idx = list(feature_indices)
    rng.shuffle(idx)
    combos: List[Tuple[int, ...]] = []
    for k in range(2, max_comb_size + 1):
        block = list(itertools.islice(itertools.combinations(idx, k), max_combinations_per_k))
        if len(block) >= max_combinations_per_k:
            warnings.append(f"k={k} combinations capped by max_combinations_per_k.")
        combos.extend(block)
        if len(idx) < k + 1:
            break
    return combos, warnings
