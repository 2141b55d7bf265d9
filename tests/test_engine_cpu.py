"""Host logic of the plugin mirror, without a GPU: planning pinned to the reference's
planning outputs, input checks, backend resolution with no CPU fallback."""
import numpy as np
import pytest

from gafime_b200.config import ComputeBudget, EngineConfig
from gafime_b200.metrics import MetricSuite, metric_strength
from gafime_b200.planning import plan_higher_order, plan_unary, select_top_features
from gafime_b200.utils import coerce_inputs, validate_budget


@pytest.mark.parametrize("seed", [0, 7, 11])
def test_planning_matches_reference(golden, seed):
    g = golden("planning.npz")
    rng = np.random.default_rng(seed)
    u, _ = plan_unary(20, 8, rng)
    h, w = plan_higher_order([i[0] for i in u], 2, 9, rng)
    assert np.array(u, dtype=np.int32).reshape(-1).tolist() == g[f"unary_{seed}"].tolist()
    assert np.array(h, dtype=np.int32).tolist() == g[f"pairs_{seed}"].tolist()
    assert w == ["k=2 combinations capped by max_combinations_per_k."]


def test_select_top_features_and_strength():
    assert select_top_features({0: 0.1, 1: 0.5, 2: 0.3}, 2) == [1, 2]
    assert select_top_features({0: 0.1}, 0) == []
    assert metric_strength({"pearson": -0.4, "mutual_info": 0.2}) == 0.4
    assert metric_strength({}) == 0.0


def test_config_defaults_match_reference():
    c = EngineConfig()
    assert c.metric_names == ("pearson", "spearman", "mutual_info", "r2")
    assert (c.num_repeats, c.permutation_tests, c.random_seed, c.mi_bins) == (3, 25, 7, 16)
    b = ComputeBudget()
    assert (b.max_comb_size, b.max_combinations_per_k, b.top_features_for_higher_k) == (2, 5000, 50)
    assert (c.operator, c.center, c.div_eps) == ("multiply", True, 1e-8)


def test_input_checks():
    with pytest.raises(ValueError):
        coerce_inputs(np.array([[1.0, np.nan]]), np.array([1.0]))
    with pytest.raises(ValueError):
        coerce_inputs(np.ones((3, 2)), np.ones(4))
    X, y, names = coerce_inputs(np.ones((3, 2), dtype=np.float32), [1, 2, 3])
    assert X.dtype == np.float64 and names == ["f0", "f1"]
    with pytest.raises(ValueError):
        validate_budget(3, ComputeBudget(max_comb_size=0))
    with pytest.raises(ValueError):
        MetricSuite(["kendall"])


def test_resolve_backend_has_no_cpu_fallback():
    from gafime_b200.backends import resolve_backend
    for name in ("python", "core", "cpu", "numpy", "metal"):
        with pytest.raises(ValueError):
            resolve_backend(EngineConfig(backend=name), np.ones((4, 2)), np.ones(4))


def test_gpu_backend_fails_loudly_without_a_gpu():
    from gafime_b200 import _native
    lib = _native.load(require_gpu=False)
    if lib.gafime_cuda_available() == 1:
        pytest.skip("a GPU is present")
    from gafime_b200 import GafimeSelector
    with pytest.raises(RuntimeError):
        GafimeSelector(k=2).fit(np.random.rand(20, 4), np.random.rand(20))


def test_coerce_keeps_float32_only_when_asked():
    X32 = np.arange(6, dtype=np.float32).reshape(3, 2)
    Xa, ya, _ = coerce_inputs(X32, np.ones(3, dtype=np.float32), keep_float32=True)
    assert Xa.dtype == np.float32 and ya.dtype == np.float32
    np.testing.assert_array_equal(Xa, X32)
    Xb, _, _ = coerce_inputs(X32.astype(np.float64), [1, 2, 3], keep_float32=True)
    assert Xb.dtype == np.float64
