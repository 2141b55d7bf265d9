"""The small-bucket ABI (gafime_bucket_*, gafime_interleaved_compute, gafime_fused_interaction)
against the reference CPU library's outputs (tests/golden/chains.npz) and the oracle.

Tolerance: the 12 stats are fp64 sums cast to float, like the reference; transcendental
unary operators may differ from the CPU's libm by an ulp per element, so the stats are
compared at 1e-5 relative (1e-3 absolute for sums near zero)."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-3


@pytest.fixture(scope="module")
def lib():
    from gafime_b200 import _native
    return _native.load()


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


class Small:
    def __init__(self, lib, X, y, mask):
        self.lib = lib
        self.h = ctypes.c_void_p()
        assert lib.gafime_bucket_alloc(X.shape[0], X.shape[1], ctypes.byref(self.h)) == 0
        self.cols = [np.ascontiguousarray(X[:, c], dtype=np.float32) for c in range(X.shape[1])]
        for c, col in enumerate(self.cols):
            assert lib.gafime_bucket_upload_feature(self.h, c, _p(col)) == 0
        self.y = np.ascontiguousarray(y, dtype=np.float32)
        self.mask = np.ascontiguousarray(mask, dtype=np.uint8)
        assert lib.gafime_bucket_upload_target(self.h, _p(self.y)) == 0
        assert lib.gafime_bucket_upload_mask(self.h, _p(self.mask)) == 0

    def compute(self, feats, ops, inter, vf):
        st = np.zeros(12, np.float32)
        f = np.array(feats, np.int32)
        o = np.array(ops, np.int32)
        t = np.array(list(inter) + [0], np.int32)
        rc = self.lib.gafime_bucket_compute(self.h, _p(f), _p(o), len(feats), _p(t), vf, _p(st))
        return rc, st

    def free(self):
        assert self.lib.gafime_bucket_free(self.h) == 0


def _cases(g, prefix):
    feats, ops = g[f"{prefix}_feats"], g[f"{prefix}_ops"]
    for q in range(feats.shape[0]):
        a = int((feats[q] >= 0).sum())
        yield q, feats[q, :a].tolist(), ops[q, :a].tolist()


def test_bucket_compute_matches_reference_cpu(lib, golden):
    g = golden("chains.npz")
    vf = int(g["val_fold"])
    b = Small(lib, g["X"], g["y"], g["mask"])
    try:
        for q, feats, ops in _cases(g, "chain"):
            rc, st = b.compute(feats, ops, g["chain_inter"][q, :len(feats) - 1].tolist(), vf)
            assert rc == 0
            np.testing.assert_allclose(st, g["chain_stats"][q], rtol=RTOL, atol=ATOL, err_msg=str((feats, ops)))
    finally:
        b.free()


def _train_r(st):
    """Train-fold Pearson from the 12 float stats (n, sx, sy, sxx, syy, sxy first), the
    formula of fused_kernel.py:236-264."""
    n, sx, sy, sxx, syy, sxy = (float(v) for v in st[:6])
    den = np.sqrt((n * sxx - sx * sx) * (n * syy - sy * sy))
    return (n * sxy - sx * sy) / den if den > 0 else 0.0


def test_mixed_interaction_chain(lib, oracle):
    """A * B then + C against A * B * C on a target made of A * B + C, as the reference's
    per-pair interaction test does (tests/test_perpair_interactions.py:21-82): both chains'
    stats equal the oracle's, and the mixed chain's train r beats the all-multiply one's by
    more than 0.1."""
    rng = np.random.default_rng(42)
    n = 10000
    A, B, C = (rng.standard_normal(n).astype(np.float32) for _ in range(3))
    y = (A * B + C + 0.1 * rng.standard_normal(n)).astype(np.float32)
    mask = rng.integers(0, 5, n, dtype=np.uint8)
    b = Small(lib, np.column_stack([A, B, C]), y, mask)
    try:
        got = {inter: b.compute([0, 1, 2], [0, 0, 0], inter, 0) for inter in ((0, 1), (0, 0))}
    finally:
        b.free()
    for inter, (rc, st) in got.items():
        assert rc == 0
        want = oracle.chain_stats([A, B, C], y, mask, [0, 0, 0], list(inter), 0)
        np.testing.assert_allclose(st, want, rtol=RTOL, atol=ATOL, err_msg=str(inter))
    assert _train_r(got[(0, 1)][1]) > _train_r(got[(0, 0)][1]) + 0.1


def test_planted_product_is_detected(lib, oracle):
    """The reference's signal-detection check (tests/scientific_benchmark.py:160-229): with
    y = f0 * f1 + noise, the chain f0 * f1 has |train r| > 0.9 and f0 * noise, f1 * noise
    stay below 0.1; the stats equal the oracle's."""
    rng = np.random.RandomState(42)
    n = 10000
    cols = [rng.randn(n).astype(np.float32) for _ in range(3)]
    y = (cols[0] * cols[1] + rng.randn(n) * 0.1).astype(np.float32)
    mask = np.random.default_rng(42).integers(0, 5, size=n, dtype=np.uint8)
    b = Small(lib, np.column_stack(cols), y, mask)
    try:
        got = {pair: b.compute(list(pair), [0, 0], [0], 0) for pair in ((0, 1), (0, 2), (1, 2))}
    finally:
        b.free()
    for pair, (rc, st) in got.items():
        assert rc == 0
        want = oracle.chain_stats([cols[c] for c in pair], y, mask, [0, 0], [0], 0)
        np.testing.assert_allclose(st, want, rtol=RTOL, atol=ATOL, err_msg=str(pair))
    assert abs(_train_r(got[(0, 1)][1])) > 0.9
    assert abs(_train_r(got[(0, 2)][1])) < 0.1 and abs(_train_r(got[(1, 2)][1])) < 0.1


def test_fused_interaction_matches_reference_cpu(lib, golden):
    g = golden("chains.npz")
    vf = int(g["val_fold"])
    X = g["X"]
    y = np.ascontiguousarray(g["y"], dtype=np.float32)
    mask = np.ascontiguousarray(g["mask"], dtype=np.uint8)
    for q, feats, ops in _cases(g, "fused"):
        cols = [np.ascontiguousarray(X[:, c], dtype=np.float32) for c in feats]
        ptrs = (ctypes.c_void_p * len(cols))(*[c.ctypes.data for c in cols])
        o = np.array(ops, np.int32)
        st = np.zeros(12, np.float32)
        rc = lib.gafime_fused_interaction(ptrs, _p(y), _p(mask), _p(o), len(feats), int(g["fused_type"][q]), vf,
                                          len(y), _p(st))
        assert rc == 0
        np.testing.assert_allclose(st, g["fused_stats"][q], rtol=RTOL, atol=ATOL)


def test_batch_and_interleaved_agree_with_single_calls(lib, oracle):
    rng = np.random.default_rng(4)
    n = 30_000
    X = rng.standard_normal((n, 5)).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    mask = rng.integers(0, 3, n).astype(np.uint8)
    b = Small(lib, X, y, mask)
    try:
        N = 200
        idx = rng.integers(0, 5, (N, 2)).astype(np.int32)
        ops = rng.integers(0, 11, (N, 2)).astype(np.int32)
        inter = rng.integers(0, 6, N).astype(np.int32)
        st = np.zeros((N, 12), np.float32)
        rc = lib.gafime_bucket_compute_batch(b.h, _p(idx), _p(ops), _p(inter), N, 1, _p(st))
        assert rc == 0
        for q in range(0, N, 17):
            rc, one = b.compute(idx[q].tolist(), ops[q].tolist(), [int(inter[q])], 1)
            assert rc == 0
            np.testing.assert_allclose(st[q], one, rtol=1e-6, atol=1e-4)
            ref = oracle.chain_stats([X[:, c] for c in idx[q]], y, mask, ops[q], [inter[q]], 1)
            np.testing.assert_allclose(st[q], ref.astype(np.float32), rtol=RTOL, atol=ATOL)
        # interleaved: two slots over the same rows
        fa, oa = np.array([0, 1], np.int32), np.array([1, 2], np.int32)
        fb, ob = np.array([2, 3], np.int32), np.array([6, 0], np.int32)
        sa, sb = np.zeros(12, np.float32), np.zeros(12, np.float32)
        assert lib.gafime_interleaved_compute(b.h, _p(fa), _p(oa), 2, 1, _p(fb), _p(ob), 2, 0, 0, 1, _p(sa),
                                              _p(sb)) == 0
        np.testing.assert_allclose(sa, b.compute([0, 1], [1, 2], [1], 1)[1], rtol=1e-6, atol=1e-4)
        np.testing.assert_allclose(sb, b.compute([2, 3], [6, 0], [0], 1)[1], rtol=1e-6, atol=1e-4)
        # a rolling operator in slot B makes every row NaN there, and the row counts for neither slot
        ob_roll = np.array([11, 0], np.int32)
        assert lib.gafime_interleaved_compute(b.h, _p(fa), _p(oa), 2, 1, _p(fb), _p(ob_roll), 2, 0, 5, 1, _p(sa),
                                              _p(sb)) == 0
        assert np.all(sa == 0) and np.all(sb == 0)
    finally:
        b.free()


def test_small_bucket_argument_errors(lib):
    h = ctypes.c_void_p()
    assert lib.gafime_bucket_alloc(100, 6, ctypes.byref(h)) == -1     # more than 5 features
    assert lib.gafime_bucket_alloc(0, 3, ctypes.byref(h)) == -1
    assert lib.gafime_bucket_free(None) == 0
    X = np.ones((64, 3), np.float32)
    b = Small(lib, X, np.ones(64, np.float32), np.zeros(64, np.uint8))
    try:
        assert b.compute([0], [0], [], 255)[0] == -1                    # arity 1
        assert b.compute([0, 3], [0, 0], [0], 255)[0] == -1             # feature out of range
        assert b.compute([0, 1], [0, 13], [0], 255)[0] == -1            # unknown unary op
        assert b.compute([0, 1], [0, 0], [6], 255)[0] == -1             # unknown combiner
        col = np.ones(64, np.float32)
        assert lib.gafime_bucket_upload_feature(b.h, 3, _p(col)) == -1
        idx = np.zeros(2, np.int32)
        st = np.zeros(12 * 1025, np.float32)
        assert lib.gafime_bucket_compute_batch(b.h, _p(idx), _p(idx), _p(idx), 1025, 0, _p(st)) == -1
        f3 = np.array([0, 1, 2], np.int32)
        assert lib.gafime_interleaved_compute(b.h, _p(f3), _p(f3), 3, 0, _p(f3), _p(f3), 2, 0, 0, 0, _p(st),
                                              _p(st)) == -1
    finally:
        b.free()


def test_async_pipeline_fifo_backpressure_and_results(lib):
    import time
    rng = np.random.default_rng(12)
    n = 20_000
    X = rng.standard_normal((n, 4)).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    mask = rng.integers(0, 4, n).astype(np.uint8)
    b = Small(lib, X, y, mask)
    pipe = ctypes.c_void_p()
    assert lib.gafime_pipeline_init(b.h, 3, ctypes.byref(pipe)) == 0
    try:
        batches = []
        for s in range(5):
            N = 50 + 30 * s
            idx = rng.integers(0, 4, (N, 2)).astype(np.int32)
            ops = rng.integers(0, 11, (N, 2)).astype(np.int32)
            inter = rng.integers(0, 6, N).astype(np.int32)
            batches.append((idx, ops, inter))
        slot = ctypes.c_int(-2)
        for s in range(4):
            idx, ops, inter = batches[s]
            assert lib.gafime_pipeline_submit(pipe, _p(idx), _p(ops), _p(inter), len(inter), ctypes.byref(slot)) == 0
            assert slot.value == s
        assert lib.gafime_pipeline_pending(pipe) == 4
        idx, ops, inter = batches[4]
        assert lib.gafime_pipeline_submit(pipe, _p(idx), _p(ops), _p(inter), len(inter), ctypes.byref(slot)) == -5
        assert slot.value == -1
        # poll returns the oldest batch first (bounded wait for it to finish)
        out = np.zeros(1024 * 12, np.float32)
        got = ctypes.c_int(0)
        t0 = time.time()
        while True:
            rc = lib.gafime_pipeline_poll(pipe, _p(out), ctypes.byref(got))
            if rc == 0:
                break
            assert rc == -6 and time.time() - t0 < 30
            time.sleep(0.001)
        results = [out[:got.value * 12].reshape(-1, 12).copy()]
        assert got.value == len(batches[0][2])
        assert lib.gafime_pipeline_submit(pipe, _p(idx), _p(ops), _p(inter), len(inter), ctypes.byref(slot)) == 0
        assert lib.gafime_pipeline_wait(pipe, _p(out), ctypes.byref(got)) == 0
        results.append(out[:got.value * 12].reshape(-1, 12).copy())
        allout = np.zeros(5 * 1024 * 12, np.float32)
        total = ctypes.c_int(0)
        assert lib.gafime_pipeline_flush(pipe, _p(allout), ctypes.byref(total)) == 0
        assert lib.gafime_pipeline_pending(pipe) == 0
        assert lib.gafime_pipeline_poll(pipe, _p(out), ctypes.byref(got)) == -6
        rest = allout[:total.value * 12].reshape(-1, 12)
        sizes = [len(bt[2]) for bt in batches[2:]]
        assert total.value == sum(sizes)
        off = 0
        for sz in sizes:
            results.append(rest[off:off + sz])
            off += sz
        for (idx, ops, inter), res in zip(batches, results):
            ref = np.zeros((len(inter), 12), np.float32)
            assert lib.gafime_bucket_compute_batch(b.h, _p(idx), _p(ops), _p(inter), len(inter), 3, _p(ref)) == 0
            np.testing.assert_allclose(res, ref, rtol=1e-6, atol=1e-4)
    finally:
        assert lib.gafime_pipeline_free(pipe) == 0
        b.free()


def test_pearson_cuda_matches_cpu_formula(lib):
    """gafime_pearson_cuda (declared by the reference without a GPU body) follows
    gafime_pearson_cpu's arithmetic: fp64 sums, r cast to float."""
    rng = np.random.default_rng(2)
    for n in (1, 7, 1000, 300_001):
        x = rng.standard_normal(n).astype(np.float32)
        y = (0.3 * x + rng.standard_normal(n)).astype(np.float32)
        r = np.zeros(1, np.float32)
        assert lib.gafime_pearson_cuda(_p(x), _p(y), n, _p(r)) == 0
        xd, yd = x.astype(np.float64), y.astype(np.float64)
        sx, sy = xd.sum(), yd.sum()
        vx, vy = (xd * xd).sum() - sx * (sx / n), (yd * yd).sum() - sy * (sy / n)
        cov = (xd * yd).sum() - sx * (sy / n)
        want = 0.0 if (vx <= 0 or vy <= 0) else cov / np.sqrt(vx * vy)
        np.testing.assert_allclose(r[0], np.float32(want), rtol=1e-6, atol=1e-7)
    const = np.ones(10, np.float32)
    r = np.zeros(1, np.float32)
    assert lib.gafime_pearson_cuda(_p(const), _p(const), 10, _p(r)) == 0 and r[0] == 0.0
    assert lib.gafime_pearson_cuda(_p(const), _p(const), 0, _p(r)) == -1
