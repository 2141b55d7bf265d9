"""The no-allocation entry point against the regular one.

gafime_allpairs_scores_noalloc exists for programs that own the GPU's memory
themselves (an arena or caching allocator holding most of the device, or a host
application handing the library buffers from its own pool): such a caller cannot
let a library call cudaMalloc, which could fail for lack of room, fragment the
pool, or stall other streams.  The entry point takes the caller's device buffers
and keeps its intermediates in a fixed __device__ array.

Here the test itself owns the buffers (allocated with torch) and checks the
no-allocation scores against gafime_allpairs_scores on a bucket and against the
oracle, with the same tolerance as the other parity tests (1e-4 relative + 1e-6
absolute), on calls in a row with different data, shapes (feature counts that are
not multiples of the 64-column tile, row counts below the padded stride) and all four
operators, so that whatever one call left in the shared array cannot leak into the
next.  The entry point computes the pair moments with the CUDA-core kernel and runs
the same accuracy guard as the allocating path.  This file is named to be collected
last.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _data(seed, n, f):
    rng = np.random.default_rng(seed)
    X = np.hstack([rng.standard_normal((n, f - f // 2)),
                   rng.lognormal(0.0, 1.0, (n, f // 2))]).astype(np.float32)
    y = (rng.random(n) < 0.45).astype(np.float32)
    return X, y


def _noalloc_scores(lib, X, y, op_id, eps):
    import torch
    n, f = X.shape
    ld = (n + 255) // 256 * 256
    dx = torch.zeros((f, ld), dtype=torch.float32, device="cuda")
    dx[:, :n] = torch.from_numpy(np.ascontiguousarray(X.T)).cuda()
    dy = torch.from_numpy(y).cuda()
    out = torch.full((f * (f - 1) // 2,), float("nan"), dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.gafime_allpairs_scores_noalloc(dx.data_ptr(), ld, dy.data_ptr(), n, f, op_id,
                                            eps, out.data_ptr(), stream)
    assert rc == 0, rc
    return out.cpu().numpy()


def test_noalloc_scores_match_the_allocating_entry_point(oracle):
    import torch  # noqa: F401  (initialises CUDA for the test-owned buffers)
    from gafime_b200 import _native
    lib = _native.load()
    calls = [  # calls in a row: different data, shapes and operators
        (_data(1, 50_000, 150), "multiply", 1e-8),
        (_data(2, 7_777, 70), "divide", 1e-6),
        (_data(3, 12_345, 97), "add", 1e-8),
        (_data(4, 30_001, 131), "subtract", 1e-8),
    ]
    for (X, y), op, eps in calls:
        got = _noalloc_scores(lib, X, y, _native.INTERACT[op], eps)
        with _native.Bucket(X.shape[0], X.shape[1]) as b:
            b.upload(X, y)
            want = b.scores(op, div_eps=eps)
        assert np.all(np.isfinite(got))
        np.testing.assert_array_less(np.abs(got - want), 1e-4 * np.abs(want) + 1e-6)
        ref = oracle.raw_pearson(X, y, op, div_eps=eps)
        np.testing.assert_array_less(np.abs(got - ref), 1e-4 * np.abs(ref) + 1e-6)


def test_noalloc_columns_far_from_zero_match_the_oracle(oracle):
    """Columns 100 standard deviations from zero: the moment kernel's fp32 runs alone miss
    the bound here, and the accuracy guard's exact re-score (in the shared array) holds it."""
    from gafime_b200 import _native
    lib = _native.load()
    rng = np.random.default_rng(5)
    n, f = 40000, 8
    X = (100.0 + rng.standard_normal((n, f)) * rng.uniform(0.5, 2.0, f)).astype(np.float32)
    y = (rng.random(n) < 1 / (1 + np.exp(-(X[:, 1] - X[:, 1].mean())))).astype(np.float32)
    for op in ("multiply", "divide"):
        got = _noalloc_scores(lib, X, y, _native.INTERACT[op], 1e-6)
        ref = oracle.raw_pearson(X, y, op, div_eps=1e-6)
        np.testing.assert_array_less(np.abs(got - ref), 1e-4 * np.abs(ref) + 1e-6)


def test_noalloc_rejects_nonzero_padding_rows():
    """Rows n .. ld-1 of the caller's columns must be zero (the moment kernel sums them)."""
    import torch
    from gafime_b200 import _native
    lib = _native.load()
    n, f, ld = 1000, 4, 1024
    dx = torch.zeros((f, ld), dtype=torch.float32, device="cuda")
    dx[:, :n] = torch.randn((f, n), device="cuda")
    dx[2, n + 5] = 1.0
    dy = torch.ones(n, dtype=torch.float32, device="cuda")
    out = torch.zeros(f * (f - 1) // 2, dtype=torch.float64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.gafime_allpairs_scores_noalloc(dx.data_ptr(), ld, dy.data_ptr(), n, f, 0, 1e-8,
                                              out.data_ptr(), s) == -1


def test_noalloc_rejects_sizes_beyond_its_limits():
    import torch
    from gafime_b200 import _native
    lib = _native.load()
    dx = torch.zeros((2, 256), dtype=torch.float32, device="cuda")
    dy = torch.zeros(256, dtype=torch.float32, device="cuda")
    out = torch.zeros(1, dtype=torch.float64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    too_many_features = _native.load().gafime_allpairs_scores_noalloc(
        dx.data_ptr(), 256, dy.data_ptr(), 256, 257, 0, 1e-8, out.data_ptr(), s)
    too_many_rows = lib.gafime_allpairs_scores_noalloc(
        dx.data_ptr(), 2097152 + 256, dy.data_ptr(), 256, 2, 0, 1e-8, out.data_ptr(), s)
    ragged_ld = lib.gafime_allpairs_scores_noalloc(
        dx.data_ptr(), 300, dy.data_ptr(), 256, 2, 0, 1e-8, out.data_ptr(), s)
    assert too_many_features == too_many_rows == ragged_ld == -1
