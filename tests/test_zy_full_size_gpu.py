"""Parity at the configured sizes of the three large workloads, after every cheaper parity
file (a run that stops at the first failure has already checked everything else):

* 1e7 x 512 banking-style table (Zipf-like integer codes + normals), multiply, k = 1000:
  all 130,816 pair scores against the fp64 Gram oracle, the top-k set modulo ties, the
  Gram oracle pinned to the element-rounded oracle on the returned pairs;
* 2e6 x 2048 wide table, 16 planted pairs, multiply, k = 1000: the k returned scores
  against the element-rounded oracle, every pair among 201 random columns (20,100 pairs)
  against the Gram oracle, no sampled pair outside the top-k above the k-th score, the 16
  planted pairs first;
* 4e6 x 128 three-class table, centred multiply, MI with 32 equal-width bins, k = 50: every
  pair's MI against the oracle, the top-k set modulo ties, (5, 9) then (12, 60) first.

Tolerances as in test_gpu_parity.py: Pearson 1e-4 * |r| + 1e-6 per pair, MI 1e-5 absolute,
top-k sets equal modulo ties.  Inputs are seeded synthetic tables with the configured shapes
and value distributions, generated column by column on host threads (one seeded generator
per column)."""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

from test_gpu_parity import assert_pearson_close, assert_topk_equivalent

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def native():
    from gafime_b200 import _native
    _native.load()
    return _native


def _need_host_memory(gb):
    try:
        import psutil
    except ImportError:
        return
    avail = psutil.virtual_memory().available / 1e9
    if avail < gb:
        pytest.skip(f"needs {gb:.0f} GB of free host memory, {avail:.0f} GB available")


def _fill_columns(packed, fill, first, last, threads=16):
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(fill, range(first, last)))


def _zipf_codes(rng, n, card):
    """Integer codes 0 .. card-1 with P(code = c) ~ (c + 1)^-1.1: the continuous power law
    of exponent 1.1 on [1, card + 1), sampled by inverting its distribution function, then
    floored."""
    u = rng.random(n)
    x = (1.0 - u * (1.0 - (card + 1.0) ** -0.1)) ** -10.0
    return np.minimum(np.floor(x) - 1.0, card - 1.0).astype(np.float32)


def _check_sampled_topk(gi, gs, sample_pairs, sample_scores, topset):
    kth = np.abs(gs[len(gi) - 1])
    for (a, c), w in zip(sample_pairs, sample_scores):
        if (a, c) not in topset:
            assert abs(w) <= kth * (1 + 1e-4) + 1e-6, ((a, c), w, kth)


def test_banking_table_at_full_size(native, oracle):
    _need_host_memory(32)
    n, f, k = 10_000_000, 512, 1000
    packed = np.empty((f + 1, n), dtype=np.float32)

    def fill(c):
        r = np.random.default_rng(40_000 + c)
        if c < 256:
            packed[c] = _zipf_codes(r, n, int(r.integers(2, 1001)))
        else:
            packed[c] = r.standard_normal(n, dtype=np.float32)

    _fill_columns(packed, fill, 0, f)
    r = np.random.default_rng(41_000)
    y = 0.5 * packed[7].astype(np.float64) * packed[300] + 0.3 * packed[301].astype(np.float64) * packed[302] \
        + r.standard_normal(n)
    packed[f] = y.astype(np.float32)
    del y
    with native.Bucket(n, f) as b:
        b.upload_packed(packed)
        gi, gj, gs = b.topk(["multiply"], k)["multiply"]
        allsc = b.scores("multiply")
    pi, pj = oracle.all_pairs(f)
    want = oracle.gram_raw_pearson(packed[:f], packed[f])
    assert_pearson_close(allsc, want)
    assert_topk_equivalent(gi, gj, want, pi, pj, k)
    assert (int(gi[0]), int(gj[0])) == (7, 300)
    # the Gram oracle agrees with the element-rounded oracle on the 200 best pairs
    X, yv = packed[:f].T, packed[f]
    top = slice(0, 200)
    exact = oracle.raw_pearson(X, yv, "multiply", gi[top].astype(np.int32), gj[top].astype(np.int32))
    pos = {(int(a), int(c)): p for p, (a, c) in enumerate(zip(pi, pj))}
    assert_pearson_close(np.array([want[pos[(int(a), int(c))]] for a, c in zip(gi[top], gj[top])]), exact)
    assert_pearson_close(gs[top], exact)


def test_wide_table_at_full_size(native, oracle):
    _need_host_memory(26)
    n, f, k = 2_000_000, 2048, 1000
    packed = np.empty((f + 1, n), dtype=np.float32)

    def fill(c):
        packed[c] = np.random.default_rng(50_000 + c).standard_normal(n, dtype=np.float32)

    _fill_columns(packed, fill, 0, f)
    r = np.random.default_rng(51_000)
    planted = r.permutation(f)[:32].reshape(16, 2)
    beta = np.linspace(0.05, 0.5, 16) * r.choice([-1.0, 1.0], 16)
    logit = np.zeros(n)
    for (a, c), w in zip(planted, beta):
        logit += w * packed[a].astype(np.float64) * packed[c]
    packed[f] = (r.random(n) < 1.0 / (1.0 + np.exp(-logit))).astype(np.float32)
    del logit
    with native.Bucket(n, f) as b:
        b.upload_packed(packed)
        gi, gj, gs = b.topk(["multiply"], k)["multiply"]
        allsc = b.scores("multiply")
    assert len(gi) == k and np.all(np.diff(np.abs(gs)) <= 0)
    X, yv = packed[:f].T, packed[f]
    assert_pearson_close(gs, oracle.raw_pearson(X, yv, "multiply", gi.astype(np.int32), gj.astype(np.int32)))
    # every pair among 201 random columns, from the Gram oracle (pinned below)
    cols = np.sort(np.random.default_rng(52_000).choice(f, 201, replace=False))
    sub = oracle.gram_raw_pearson(packed[cols], packed[f])
    si, sj = np.triu_indices(len(cols), k=1)
    ci, cj = cols[si], cols[sj]
    p_all = ci * f - ci * (ci + 1) // 2 + (cj - ci - 1)
    assert_pearson_close(allsc[p_all], sub)
    pin = np.random.default_rng(53_000).choice(len(si), 300, replace=False)
    assert_pearson_close(sub[pin], oracle.raw_pearson(X, yv, "multiply", ci[pin].astype(np.int32),
                                                      cj[pin].astype(np.int32)))
    topset = {(int(a), int(c)) for a, c in zip(gi, gj)}
    _check_sampled_topk(gi, gs, [(int(a), int(c)) for a, c in zip(ci, cj)], sub, topset)
    want = {(int(min(a, c)), int(max(a, c))) for a, c in planted}
    assert {(int(a), int(c)) for a, c in zip(gi[:16], gj[:16])} == want


def test_three_class_mi_table_at_full_size(native, oracle):
    _need_host_memory(8)
    n, f, k = 4_000_000, 128, 50
    packed = np.empty((f + 1, n), dtype=np.float32)

    def fill(c):
        packed[c] = np.random.default_rng(60_000 + c).standard_normal(n, dtype=np.float32)

    _fill_columns(packed, fill, 0, f)
    r = np.random.default_rng(61_000)
    e = r.standard_normal((4, n))
    s0 = packed[5].astype(np.float64) * packed[9] + 0.5 * e[0]
    s1 = packed[12].astype(np.float64) + packed[60] + 0.5 * e[1]
    packed[f] = np.argmax(np.stack([s0, s1, e[2] + 0.5 * e[3]]), axis=0).astype(np.float32)
    del e, s0, s1
    with native.Bucket(n, f) as b:
        b.upload_packed(packed)
        gi, gj, gs = b.topk(["multiply"], k, metric="mutual_info", center=True, mi_bins=32)["multiply"]
        allmi = b.scores("multiply", metric="mutual_info", center=True, mi_bins=32)
    pi, pj = oracle.all_pairs(f)
    want = oracle.pair_mi(packed[:f].T, packed[f], "multiply", center=True, mi_bins=32)
    np.testing.assert_allclose(allmi, want, rtol=0, atol=1e-5)
    assert_topk_equivalent(gi, gj, want, pi, pj, k, rtol=0, atol=1e-5)
    assert [(int(a), int(c)) for a, c in zip(gi[:2], gj[:2])] == [(5, 9), (12, 60)]
