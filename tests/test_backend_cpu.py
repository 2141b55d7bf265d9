"""Host logic of the GPU backend's resident matrix, with the device bucket replaced by a
recording fake (no GPU): one upload per matrix, target-only replacement, device gathers for
column subsets, least-recently-used eviction of subset buckets."""
import numpy as np
import pytest


class FakeBucket:
    log = []

    def __init__(self, n, f, device=None):
        self.n, self.f, self.device, self.freed = n, f, device, False
        FakeBucket.log.append(("alloc", n, f))

    def upload_rows(self, X, y):
        FakeBucket.log.append(("upload_rows", X.shape))

    def set_target(self, y):
        FakeBucket.log.append(("set_target", self.f))

    @classmethod
    def gather(cls, src, cols, rows=None):
        b = cls(src.n if rows is None else len(rows), len(cols))
        FakeBucket.log.append(("gather", tuple(cols), rows is not None))
        return b

    def free(self):
        self.freed = True
        FakeBucket.log.append(("free", self.f))


@pytest.fixture
def resident(monkeypatch):
    from gafime_b200 import _native
    from gafime_b200.backends import native_cuda_backend as ncb
    monkeypatch.setattr(_native, "Bucket", FakeBucket)
    FakeBucket.log = []
    return ncb._Resident


def kinds(log, kind):
    return [e for e in log if e[0] == kind]


def test_one_upload_target_only_replacement_and_subset_eviction(resident):
    X = np.zeros((10, 8), dtype=np.float32)
    y1, y2 = np.zeros(10, dtype=np.float32), np.ones(10, dtype=np.float32)
    r = resident(X, y1, device=0)
    assert len(kinds(FakeBucket.log, "upload_rows")) == 1
    full = r.bucket(tuple(range(8)), y1)
    assert kinds(FakeBucket.log, "set_target") == []          # same target: nothing moves
    r.bucket(tuple(range(8)), y2)
    assert len(kinds(FakeBucket.log, "set_target")) == 1      # new target: the target only
    subsets = [(0, 1), (2, 3), (4, 5), (6, 7)]
    made = [r.bucket(c, y2) for c in subsets]
    assert len(kinds(FakeBucket.log, "gather")) == 4
    assert r.bucket((0, 1), y2) is made[0]                    # cached, now most recent
    r.bucket((1, 2), y2)                                      # a fifth subset evicts (2, 3)
    assert made[1].freed and not made[0].freed
    assert len(kinds(FakeBucket.log, "upload_rows")) == 1
    r.bucket((0, 1), y1)                                      # cached subset, other target
    assert kinds(FakeBucket.log, "set_target")[-1] == ("set_target", 2)
    tmp = r.gather((3, 4), y1, np.array([0, 0, 9]))
    assert tmp.n == 3 and ("gather", (3, 4), True) in FakeBucket.log
    r.free()
    assert full.freed and all(b.freed for b in made)


def test_stability_resampled_path_draws_the_same_rows():
    """A backend with score_resampled gets the same bootstrap rows (same generator draws) as
    the reference's X[idx], y[idx] path."""
    from gafime_b200.backends.base import Backend
    from gafime_b200.metrics import MetricSuite
    from gafime_b200.validation import StabilityAnalyzer

    class Plain(Backend):
        def score_combos(self, X, y, combos, suite):
            return {c: {"pearson": float(np.sum(X[:, c[0]] * y))} for c in combos}

    class Resampling(Plain):
        def score_resampled(self, X, y, rows, combos, suite):
            return self.score_combos(X[rows], y[rows], combos, suite)

    rng0 = np.random.default_rng(4)
    X = rng0.standard_normal((50, 3))
    y = rng0.standard_normal(50)
    suite = MetricSuite(["pearson"])
    a = StabilityAnalyzer(suite, Plain()).assess(X, y, [(0,), (2,)], 3, np.random.default_rng(9))
    b = StabilityAnalyzer(suite, Resampling()).assess(X, y, [(0,), (2,)], 3, np.random.default_rng(9))
    assert [(r.combo, r.metrics_mean, r.metrics_std) for r in a] == \
        [(r.combo, r.metrics_mean, r.metrics_std) for r in b]
