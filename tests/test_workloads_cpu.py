"""bench.py's synthetic workloads against the shapes and value distributions of the configured
workloads (N(0,1) and lognormal(0,1) columns, Zipf(1.1) integer codes of cardinality 2-1000,
Bernoulli, 3-class and continuous targets, planted pairs), at small row counts on the CPU."""
import numpy as np

import bench


def test_config1_and_config2_columns_and_targets():
    X, y = bench.make_config1()
    assert X.shape == (1000, 50) and X.dtype == np.float32 and set(np.unique(y)) <= {0.0, 1.0}
    X, y = bench.make_config2(n=20000)
    assert X.shape == (20000, 256) and X.dtype == np.float32
    assert np.all(np.abs(X[:, :128].mean(axis=0)) < 0.05)
    assert X[:, 128:].min() > 0 and abs(np.log(X[:, 128:]).std() - 1.0) < 0.02
    assert set(np.unique(y)) == {0.0, 1.0}


def test_config2_scaled_width_keeps_pairs_per_gpu():
    for world in (1, 2, 4, 8):
        f = bench.scaled_width(world)
        assert abs(f * (f - 1) / 2 / world - 32640) / 32640 < 0.01
    f, n = bench.scaled_width(2), 5000
    packed = np.empty((f + 1, n), dtype=np.float32)
    bench.fill_config2_scaled(packed, n)
    assert np.all(np.abs(packed[:f // 2].mean(axis=1)) < 0.1) and packed[f // 2:f].min() > 0
    assert set(np.unique(packed[f])) == {0.0, 1.0}


def test_config3_three_classes():
    X, y = bench.make_config3(n=30000)
    assert X.shape == (30000, 128) and set(np.unique(y)) == {0.0, 1.0, 2.0}


def test_config4_zipf_codes_and_regression_target():
    n = 40000
    packed = np.empty((513, n), dtype=np.float32)
    bench.fill_config4(packed, n)
    codes = packed[:256]
    assert np.all(codes == np.round(codes)) and codes.min() == 0 and codes.max() <= 999
    # Zipf frequencies: code 0 is the most frequent value of every code column
    for c in range(0, 256, 37):
        assert np.bincount(codes[c].astype(np.int64)).argmax() == 0
    assert np.all(np.abs(packed[256:512].mean(axis=1)) < 0.05)
    assert len(np.unique(packed[512])) > n // 2   # continuous target


def test_config5_planted_pairs():
    n = 4000
    packed = np.empty((2049, n), dtype=np.float32)
    idx = bench.fill_config5(packed, n)
    assert idx.shape == (16, 2) and len(np.unique(idx)) == 32   # 16 pairs of distinct columns
    assert set(np.unique(packed[2048])) == {0.0, 1.0}


def test_config5_column_subset_matches_the_full_table():
    """A rank of a sharded run builds only the column blocks its shard reads: those columns
    and the target equal the full build's, and the other columns are left untouched."""
    n = 3000
    full = np.empty((2049, n), dtype=np.float32)
    bench.fill_config5(full, n)
    cols = list(range(128, 384)) + list(range(1920, 2048))
    part = np.zeros((2049, n), dtype=np.float32)
    bench.fill_config5(part, n, cols=cols)
    assert np.array_equal(part[cols], full[cols])
    assert np.array_equal(part[2048], full[2048])
    assert not part[:128].any() and not part[384:1920].any()
