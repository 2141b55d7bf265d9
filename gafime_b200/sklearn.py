"""scikit-learn transformer (gafime/sklearn.py:10-110) on the GPU engine.

``fit`` runs the engine and keeps the k pairs with the largest |metric|.  As in the
reference, ``operator`` only shapes ``transform`` unless ``score_operator=True``, which
also scores the pairs with that operator (the reference always scores the centred
product, gafime/sklearn.py:49-57)."""
from __future__ import annotations

import numpy as np
from sklearn.base import BaseEstimator, TransformerMixin
from sklearn.utils.validation import check_array, check_is_fitted, check_X_y

from .config import ComputeBudget, EngineConfig
from .engine import GafimeEngine


class GafimeSelector(BaseEstimator, TransformerMixin):
    def __init__(self, k: int = 10, backend: str = "auto", metric: str = "pearson",
                 operator: str = "multiply", n_jobs: int = -1, verbose: bool = False,
                 score_operator: bool = False, device_id: int = 0):
        self.k = k
        self.backend = backend
        self.metric = metric
        self.operator = operator
        self.n_jobs = n_jobs
        self.verbose = verbose
        self.score_operator = score_operator
        self.device_id = device_id

    def fit(self, X, y):
        X, y = check_X_y(X, y, accept_sparse=False, dtype=[np.float32, np.float64])
        scored_op = self.operator if self.score_operator else "multiply"
        config = EngineConfig(backend=self.backend, metric_names=(self.metric,),
                              budget=ComputeBudget(max_comb_size=2), device_id=self.device_id,
                              operator=scored_op, center=not self.score_operator)
        report = GafimeEngine(config=config).analyze(X, y)
        if self.verbose:
            print(report.decision.message if report.decision else "")
        ranked = sorted(report.interactions, key=lambda r: abs(r.metrics.get(self.metric, 0.0)),
                        reverse=True)
        self.top_interactions_ = [r.combo for r in ranked if len(r.combo) == 2][: self.k]
        self.n_features_in_ = X.shape[1]
        return self

    def transform(self, X):
        check_is_fitted(self, ["top_interactions_", "n_features_in_"])
        X = check_array(X, accept_sparse=False, dtype=[np.float32, np.float64])
        if X.shape[1] != self.n_features_in_:
            raise ValueError(f"Shape of input is different from what was seen in `fit` "
                             f"({X.shape[1]} != {self.n_features_in_})")
        extra = np.empty((X.shape[0], len(self.top_interactions_)), dtype=X.dtype)
        for c, (i, j) in enumerate(self.top_interactions_):
            a, b = X[:, i], X[:, j]
            if self.operator == "multiply":
                extra[:, c] = a * b
            elif self.operator == "add":
                extra[:, c] = a + b
            elif self.operator == "subtract":
                extra[:, c] = a - b
            elif self.operator == "divide":
                extra[:, c] = a / (b + 1e-8)  # the reference's transform rule, gafime/sklearn.py:105
            else:
                raise ValueError(f"Unsupported operator encountered during transform: {self.operator}")
        return np.hstack((X, extra))
