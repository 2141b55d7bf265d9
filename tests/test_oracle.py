"""Pin the CPU oracle against golden vectors made by the reference's own code.

The fixtures come from tests/golden/make_golden.py (gafime_core.score_combos,
GafimeSelector.fit, the reference numpy metrics and cpu_backend.cpp compiled
unmodified).  If the oracle disagrees with them it cannot be trusted as the
oracle of the CUDA path.
"""
import numpy as np
import pytest

OPS = ["multiply", "add", "subtract", "divide"]


def test_config1_centred_pearson_matches_gafime_core(golden, oracle):
    g = golden("config1_centred.npz")
    p, m = oracle.centred_scores(g["X"], g["y"], pearson=True, mi=True, mi_bins=16)
    # Same operation order as gafime_core.cpp -> bit-identical doubles.
    np.testing.assert_array_equal(p, g["core_scores"][:, 0])
    np.testing.assert_array_equal(m, g["core_scores"][:, 1])
    # The reference's numpy twin agrees to rounding.
    np.testing.assert_allclose(p, g["numpy_scores"][:, 0], rtol=0, atol=1e-14)
    np.testing.assert_allclose(m, g["numpy_scores"][:, 1], rtol=0, atol=1e-12)


def test_config1_topk_matches_selector(golden, oracle):
    g = golden("config1_centred.npz")
    pi, pj = oracle.all_pairs(g["X"].shape[1])
    p, _ = oracle.centred_scores(g["X"], g["y"])
    top = oracle.topk(p, pi, pj, 5)
    got = {(int(min(a, b)), int(max(a, b))) for a, b in zip(pi[top], pj[top])}
    for key in ("selector_top_core", "selector_top_python"):
        want = {(int(min(a, b)), int(max(a, b))) for a, b in g[key]}
        assert got == want
    # Known answer from the reference run: (3,15) is the best pair.
    assert (int(pi[top[0]]), int(pj[top[0]])) == (3, 15)


@pytest.mark.parametrize("bins,key", [(32, "core_b32"), (16, "core_b16")])
def test_mi_3class_matches_gafime_core(golden, oracle, bins, key):
    g = golden("mi_3class.npz")
    _, m = oracle.centred_scores(g["X"], g["y"], pearson=False, mi=True, mi_bins=bins)
    col = 1 if key == "core_b32" else 0
    np.testing.assert_array_equal(m, g[key][:, col])


@pytest.mark.parametrize("op_id,op", list(enumerate(OPS)))
def test_raw_op_stats_match_cpu_backend(golden, oracle, op_id, op):
    """The oracle keeps fp64 sums; the reference casts them to float32, so each
    stat must agree to within one float32 rounding of the fp64 value."""
    g = golden("raw_ops.npz")
    r, st = oracle.raw_pearson(g["X"], g["y"], op, div_eps=1e-8, with_stats=True)
    ref = g["ref_stats"][op_id][:, :6].astype(np.float64)
    np.testing.assert_array_equal(st.astype(np.float32), ref.astype(np.float32))
    # The validation half of the reference stats is empty (val_fold_id=255).
    assert np.all(g["ref_stats"][op_id][:, 6:] == 0)


def test_edge_cases_match_reference(golden, oracle):
    g = golden("edge.npz")
    p, m = oracle.centred_scores(g["X"], g["y"], pearson=True, mi=True, mi_bins=4)
    np.testing.assert_array_equal(p, g["core_scores"][:, 0])
    np.testing.assert_array_equal(m, g["core_scores"][:, 1])
    # constant column 1 -> Pearson 0 and MI 0 for every pair touching it
    pi, pj = oracle.all_pairs(4)
    touch = (pi == 1) | (pj == 1)
    assert np.all(p[touch] == 0) and np.all(m[touch] == 0)
    for op_id, op in enumerate(OPS):
        _, st = oracle.raw_pearson(g["X"], g["y"], op, with_stats=True)
        np.testing.assert_array_equal(st.astype(np.float32), g["ref_stats"][op_id][:, :6])
        _, stn = oracle.raw_pearson(g["X_nan"], g["y"], op, with_stats=True)
        np.testing.assert_array_equal(stn.astype(np.float32), g["ref_stats_nan"][op_id][:, :6])


def test_divisors_at_the_clamp_match_reference(golden, oracle):
    """Safe divide at its clamp (cpu_backend.cpp:93-94, eps = 1e-8): -0.0 becomes -eps
    (copysign), values below eps are replaced, eps itself is kept, subnormals are clamped;
    every operator's stats equal the reference library's after its float cast."""
    g = golden("divisors.npz")
    assert np.signbit(g["X"][1, 1]) and g["X"][1, 1] == 0.0
    for op_id, op in enumerate(OPS):
        _, st = oracle.raw_pearson(g["X"], g["y"], op, div_eps=1e-8, with_stats=True)
        np.testing.assert_array_equal(st.astype(np.float32), g["ref_stats"][op_id][:, :6])


def test_topk_tie_order_is_pair_ascending(oracle):
    s = np.array([0.5, -0.5, 0.2, 0.5])
    pi = np.array([3, 0, 1, 0], dtype=np.int32)
    pj = np.array([4, 2, 2, 1], dtype=np.int32)
    assert oracle.topk(s, pi, pj, 3).tolist() == [3, 1, 0]


def test_interaction_materialiser_matches_reference_cpu(golden, oracle):
    """The oracle's restatement of the materialiser equals gafime_feature_interaction_cpu
    (cpu_backend.cpp:316-370) bit for bit on combos of valid features."""
    g = golden("interaction.npz")
    off = g["off"]
    combos = [g["idx"][off[c]:off[c + 1]].tolist() for c in range(len(off) - 1)]
    np.testing.assert_array_equal(oracle.feature_interaction(g["X"], g["means"], combos), g["out"])


def test_interaction_materialiser_degenerate_combos(oracle):
    """Invalid feature ids are skipped and an empty combo gives 1 (kernels.cu:1646-1676)."""
    X = np.arange(12, dtype=np.float32).reshape(4, 3)
    m = X.mean(axis=0).astype(np.float32)
    out = oracle.feature_interaction(X, m, [[0], [1, 2], [], [5], [0, 7, 2]])
    np.testing.assert_array_equal(out[:, 0], X[:, 0])
    np.testing.assert_array_equal(out[:, 1], (X[:, 1] - m[1]) * (X[:, 2] - m[2]))
    assert np.all(out[:, 2] == 1.0) and np.all(out[:, 3] == 1.0)
    np.testing.assert_array_equal(out[:, 4], out[:, 1] * 0 + (X[:, 0] - m[0]) * (X[:, 2] - m[2]))


def _chain_cases(g, prefix):
    feats, ops = g[f"{prefix}_feats"], g[f"{prefix}_ops"]
    for q in range(feats.shape[0]):
        a = int((feats[q] >= 0).sum())
        yield q, feats[q, :a].tolist(), ops[q, :a].tolist()


def test_chain_stats_match_reference_cpu(golden, oracle):
    """Small-bucket chains (unary operators, per-step combiners, folds, arity 2-5) equal
    gafime_fused_interaction_perpair_cpu after the reference's float cast."""
    g = golden("chains.npz")
    X, y, mask, vf = g["X"], g["y"], g["mask"], int(g["val_fold"])
    for q, feats, ops in _chain_cases(g, "chain"):
        inter = g["chain_inter"][q, :len(feats) - 1].tolist()
        st = oracle.chain_stats([X[:, c] for c in feats], y, mask, ops, inter, vf)
        np.testing.assert_array_equal(st.astype(np.float32), g["chain_stats"][q])
    for q, feats, ops in _chain_cases(g, "fused"):
        inter = [int(g["fused_type"][q])] * (len(feats) - 1)
        st = oracle.chain_stats([X[:, c] for c in feats], y, mask, ops, inter, vf)
        np.testing.assert_array_equal(st.astype(np.float32), g["fused_stats"][q])


def test_pair_mi_centred_multiply_equals_gafime_core(golden, oracle):
    g = golden("mi_3class.npz")
    for bins, key, col in ((32, "core_b32", 1), (16, "core_b16", 0)):
        m = oracle.pair_mi(g["X"], g["y"], "multiply", center=True, mi_bins=bins)
        np.testing.assert_array_equal(m, g[key][:, col])


@pytest.mark.parametrize("target", ["y3", "yc"])
@pytest.mark.parametrize("op_id,op", list(enumerate(OPS)))
def test_pair_mi_raw_ops_match_reference_numpy_mi(golden, oracle, target, op_id, op):
    """fp32 interactions binned with gafime_core's rule vs the reference's numpy metric
    (np.histogram2d): the bin rules agree except for values within rounding of an
    interior edge, which this data does not hold."""
    g = golden("raw_mi.npz")
    t = 0 if target == "y3" else 1
    m = oracle.pair_mi(g["X"], g[target], op, center=False, mi_bins=int(g["bins"]), div_eps=1e-8)
    np.testing.assert_allclose(m, g["mi"][t, op_id], rtol=0, atol=1e-12)


@pytest.mark.parametrize("target", ["y3", "yc"])
def test_unary_mi_matches_gafime_core(golden, oracle, target):
    g = golden("raw_mi.npz")
    m = oracle.unary_mi(g["X"], g[target], mi_bins=int(g["bins"]))
    np.testing.assert_array_equal(m, g["unary_mi"][0 if target == "y3" else 1])


@pytest.mark.parametrize("target", ["y3", "yc"])
def test_spearman_matches_gafime_core(golden, oracle, target):
    """Average-tie ranks (discrete and binary columns, a 3-class target) and the Pearson of
    ranks: the same arithmetic in the same order as gafime_core, so equal to rounding."""
    g = golden("spearman.npz")
    combos = [tuple(int(v) for v in c if v >= 0) for c in g["combos"]]
    got = oracle.spearman(g["X"], g[target], combos)
    np.testing.assert_allclose(got, g["spearman"][0 if target == "y3" else 1], rtol=0, atol=1e-13)


def test_gram_oracle_matches_the_element_rounded_oracle(golden, oracle):
    """The fp64 Gram restatement (exact products) equals the per-pair element-rounded
    restatement within the parity tolerance on normal, lognormal and Zipf-code columns, and
    the latter is pinned to the reference's cpu_backend.cpp (raw_ops.npz)."""
    rng = np.random.default_rng(3)
    n = 20000
    codes = np.minimum(np.floor((1.0 - rng.random((n, 8)) * (1.0 - 900.0 ** -0.1)) ** -10.0) - 1.0, 899.0)
    X = np.hstack([rng.standard_normal((n, 8)), rng.lognormal(0.0, 1.0, (n, 8)), codes]).astype(np.float32)
    y = (0.3 * X[:, 1] * X[:, 9] + rng.standard_normal(n)).astype(np.float32)
    got = oracle.gram_raw_pearson(np.ascontiguousarray(X.T), y, chunk_elems=1 << 16)
    want = oracle.raw_pearson(X, y, "multiply")
    assert np.all(np.abs(got - want) <= 1e-4 * np.abs(want) + 1e-6)
    g = golden("raw_ops.npz")
    Xg, yg = g["X"], g["y"]
    got = oracle.gram_raw_pearson(np.ascontiguousarray(Xg.T), yg)
    want = oracle.raw_pearson(Xg, yg, "multiply")
    assert np.all(np.abs(got - want) <= 1e-4 * np.abs(want) + 1e-6)
