"""The plugin mirror end to end on the GPU against the reference's own results."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_selector_top5_equals_reference_selector(golden):
    from gafime_b200 import GafimeSelector
    g = golden("config1_centred.npz")
    sel = GafimeSelector(k=5).fit(g["X"], g["y"])
    # same combos in the same (shuffled) orientation as the reference's top_interactions_
    assert [tuple(map(int, c)) for c in sel.top_interactions_] == \
        [tuple(map(int, c)) for c in g["selector_top_core"]]
    assert sel.transform(g["X"]).shape == (1000, 55)


def test_engine_report_matches_reference_engine(golden):
    from gafime_b200 import EngineConfig, GafimeEngine
    from gafime_b200.config import ComputeBudget
    g = golden("engine_report.npz")
    cfg = EngineConfig(metric_names=("pearson",),
                       budget=ComputeBudget(max_comb_size=2, top_features_for_higher_k=8),
                       num_repeats=3, permutation_tests=10)
    rep = GafimeEngine(cfg).analyze(g["X"], g["y"])
    combos = [list(r.combo) + [-1] * (2 - len(r.combo)) for r in rep.interactions]
    assert combos == g["combos"].tolist()
    got = np.array([r.metrics["pearson"] for r in rep.interactions])
    np.testing.assert_array_less(np.abs(got - g["pearson"]), 1e-4 * np.abs(g["pearson"]) + 1e-6)
    stab = np.array([(r.metrics_mean["pearson"], r.metrics_std["pearson"]) for r in rep.stability])
    np.testing.assert_allclose(stab, g["stability"], rtol=1e-4, atol=1e-6)
    pv = np.array([r.p_values["pearson"] for r in rep.permutations])
    np.testing.assert_array_equal(pv, g["p_values"])
    assert rep.decision.signal_detected == bool(g["decision"])
    assert rep.backend.is_gpu


def test_selector_in_sklearn_pipeline_and_grid_search():
    from sklearn.linear_model import LogisticRegression
    from sklearn.model_selection import GridSearchCV
    from sklearn.pipeline import Pipeline
    from gafime_b200 import GafimeSelector
    rng = np.random.RandomState(42)
    X = rng.randn(100, 10).astype(np.float32)
    y = rng.randint(0, 2, size=100).astype(np.float32)
    pipe = Pipeline([("miner", GafimeSelector(k=5)), ("clf", LogisticRegression())])
    pipe.fit(X, y)
    assert pipe.predict(X).shape == (100,)
    grid = GridSearchCV(Pipeline([("miner", GafimeSelector()), ("clf", LogisticRegression())]),
                        {"miner__k": [2, 4], "miner__metric": ["pearson"]}, cv=2)
    grid.fit(X, y)
    assert grid.best_params_["miner__k"] in (2, 4)


@pytest.mark.parametrize("op", ["add", "subtract", "divide"])
def test_score_operator_routes_the_operator(oracle, op):
    """With score_operator=True every planned combo (a, b) is scored as x_a op x_b on raw
    columns; each score matches the oracle and the selector keeps the best by |r|."""
    from gafime_b200 import EngineConfig, GafimeEngine, GafimeSelector
    from gafime_b200.config import ComputeBudget
    rng = np.random.default_rng(4)
    X = rng.lognormal(0, 1, (3000, 12)).astype(np.float32)
    y = (X[:, 2] / X[:, 9] + rng.standard_normal(3000) > 1.0).astype(np.float32)
    cfg = EngineConfig(metric_names=("pearson",), budget=ComputeBudget(max_comb_size=2),
                       operator=op, center=False, num_repeats=0, permutation_tests=0)
    rep = GafimeEngine(cfg).analyze(X, y)
    pairs = [r for r in rep.interactions if len(r.combo) == 2]
    a = np.array([r.combo[0] for r in pairs], np.int32)
    b = np.array([r.combo[1] for r in pairs], np.int32)
    want = oracle.raw_pearson(X, y, op, a, b, div_eps=1e-8)
    got = np.array([r.metrics["pearson"] for r in pairs])
    np.testing.assert_array_less(np.abs(got - want), 1e-4 * np.abs(want) + 1e-6)
    sel = GafimeSelector(k=3, operator=op, score_operator=True).fit(X, y)
    best = np.argsort(-np.abs(want), kind="stable")[:3]
    assert [tuple(map(int, c)) for c in sel.top_interactions_] == \
        [(int(a[p]), int(b[p])) for p in best]


def test_mutual_info_metric_through_the_engine(golden):
    from gafime_b200 import EngineConfig, GafimeEngine
    from gafime_b200.config import ComputeBudget
    g = golden("mi_3class.npz")
    cfg = EngineConfig(metric_names=("mutual_info",), mi_bins=32, num_repeats=0, permutation_tests=0,
                       budget=ComputeBudget(max_comb_size=2, top_features_for_higher_k=12))
    rep = GafimeEngine(cfg).analyze(g["X"], g["y"])
    pairs = {tuple(sorted(r.combo)): r.metrics["mutual_info"] for r in rep.interactions if len(r.combo) == 2}
    pi, pj = np.triu_indices(12, k=1)
    for p, (a, b) in enumerate(zip(pi, pj)):
        assert abs(pairs[(int(a), int(b))] - g["core_b32"][p, 1]) <= 1e-5


def test_engine_uploads_the_matrix_once(golden, monkeypatch):
    """Unary and pair scoring, 3 bootstraps and 10 permutations: one host-to-device copy
    of the matrix; bootstraps gather rows on the device, permutations replace the target."""
    from gafime_b200 import EngineConfig, GafimeEngine, _native
    from gafime_b200.config import ComputeBudget
    calls = {"upload": 0, "target": 0, "gather": 0}
    up, rows, tgt = _native.Bucket.upload_packed, _native.Bucket.upload_rows, _native.Bucket.set_target
    gat = _native.Bucket.gather.__func__

    def count(name, fn):
        def wrapped(*a, **k):
            calls[name] += 1
            return fn(*a, **k)
        return wrapped
    monkeypatch.setattr(_native.Bucket, "upload_packed", count("upload", up))
    monkeypatch.setattr(_native.Bucket, "upload_rows", count("upload", rows))
    monkeypatch.setattr(_native.Bucket, "set_target", count("target", tgt))
    monkeypatch.setattr(_native.Bucket, "gather", classmethod(count("gather", gat)))
    g = golden("engine_report.npz")
    cfg = EngineConfig(metric_names=("pearson",),
                       budget=ComputeBudget(max_comb_size=2, top_features_for_higher_k=8),
                       num_repeats=3, permutation_tests=10)
    rep = GafimeEngine(cfg).analyze(g["X"], g["y"])
    assert calls["upload"] == 1
    assert calls["gather"] >= 3 * 2 + 1
    assert calls["target"] >= 10
    assert len(rep.permutations) == len(rep.interactions)


def test_engine_default_metrics_match_reference_engine(golden):
    """EngineConfig's default metrics (pearson, spearman, mutual_info, r2): interactions,
    bootstrap means / stds, permutation p-values and the decision of the reference engine."""
    from gafime_b200 import EngineConfig, GafimeEngine
    from gafime_b200.config import ComputeBudget
    g = golden("engine_default_metrics.npz")
    ref = golden("engine_report.npz")
    cfg = EngineConfig(budget=ComputeBudget(max_comb_size=2, top_features_for_higher_k=8),
                       num_repeats=3, permutation_tests=10)
    assert list(cfg.metric_names) == g["metric_names"].tolist()
    rep = GafimeEngine(cfg).analyze(ref["X"], ref["y"])
    names = list(cfg.metric_names)
    combos = [list(r.combo) + [-1] * (2 - len(r.combo)) for r in rep.interactions]
    assert combos == g["combos"].tolist()
    tol = {"pearson": (1e-4, 1e-6), "spearman": (0, 1e-10), "mutual_info": (0, 1e-5), "r2": (2e-4, 1e-6)}
    got = np.array([[r.metrics[m] for m in names] for r in rep.interactions])
    mean = np.array([[r.metrics_mean[m] for m in names] for r in rep.stability])
    std = np.array([[r.metrics_std[m] for m in names] for r in rep.stability])
    for k, m in enumerate(names):
        rt, at = tol[m]
        np.testing.assert_allclose(got[:, k], g["metrics"][:, k], rtol=rt, atol=at, err_msg=m)
        np.testing.assert_allclose(mean[:, k], g["stab_mean"][:, k], rtol=rt, atol=at, err_msg=m)
        np.testing.assert_allclose(std[:, k], g["stab_std"][:, k], rtol=max(rt, 1e-3), atol=max(at, 1e-6),
                                   err_msg=m)
    pv = np.array([[r.p_values[m] for m in names] for r in rep.permutations])
    np.testing.assert_array_equal(pv, g["p_values"])
    assert rep.decision.signal_detected == bool(g["decision"])


def test_engine_finds_the_planted_pair_among_named_features(oracle):
    """The reference's backend verification run (tests/docker_backend_verification.py:10-42):
    y = 0.8 cat * bird + 0.3 dog - 0.2 mouse + noise, two repeats and two permutations.  The
    strongest interaction is cat * bird (the reference engine: r = 0.8975), every pair's
    Pearson equals the oracle's centred-product score, and two permutations cannot reach
    p < 0.05, so no signal is declared (as the reference reports)."""
    from gafime_b200 import EngineConfig, GafimeEngine
    from gafime_b200.config import ComputeBudget
    rng = np.random.RandomState(42)
    n = 2000
    cat, dog, bird, mouse = (rng.randn(n).astype(np.float32) for _ in range(4))
    y = (0.8 * cat * bird + 0.3 * dog - 0.2 * mouse + 0.1 * rng.randn(n)).astype(np.float32)
    X = np.column_stack([cat, dog, bird, mouse])
    cfg = EngineConfig(budget=ComputeBudget(max_comb_size=2, max_combinations_per_k=50),
                       permutation_tests=2, num_repeats=2)
    rep = GafimeEngine(cfg).analyze(X, y, feature_names=["cat", "dog", "bird", "mouse"])
    top = max(rep.interactions, key=lambda r: abs(r.metrics.get("pearson", 0.0)))
    assert tuple(sorted(top.combo)) == (0, 2) and set(top.feature_names) == {"cat", "bird"}
    pairs = [r for r in rep.interactions if len(r.combo) == 2]
    assert len(pairs) == 6
    a = np.array([min(r.combo) for r in pairs], np.int32)
    b = np.array([max(r.combo) for r in pairs], np.int32)
    want, _ = oracle.centred_scores(X, y, a, b)
    got = np.array([r.metrics["pearson"] for r in pairs])
    np.testing.assert_array_less(np.abs(got - want), 1e-4 * np.abs(want) + 1e-6)
    assert rep.decision is not None and not rep.decision.signal_detected
