"""The no-allocation entry point against the regular one.

gafime_allpairs_scores_noalloc exists for programs that own the GPU's memory
themselves (an arena or caching allocator holding most of the device, or a host
application handing the library buffers from its own pool): such a caller cannot
let a library call cudaMalloc, which could fail for lack of room, fragment the
pool, or stall other streams.  The entry point takes the caller's device buffers
and keeps its intermediates in a fixed __device__ array.

Here the test itself owns the buffers (allocated with torch) and checks the
no-allocation scores against gafime_allpairs_scores on a bucket, with the same
tolerance as the other parity tests (1e-4 relative + 1e-6 absolute), on two calls
in a row with different data, shapes and operators, so that whatever the first
call left in the shared array cannot leak into the second.  This file is named to
be collected last.
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


def test_noalloc_scores_match_the_allocating_entry_point():
    import torch  # noqa: F401  (initialises CUDA for the test-owned buffers)
    from gafime_b200 import _native
    lib = _native.load()
    calls = [  # two calls in a row: different data, shape and operator
        (_data(1, 50_000, 150), "multiply", 1e-8),
        (_data(2, 7_777, 70), "divide", 1e-6),
    ]
    for (X, y), op, eps in calls:
        got = _noalloc_scores(lib, X, y, _native.INTERACT[op], eps)
        with _native.Bucket(X.shape[0], X.shape[1]) as b:
            b.upload(X, y)
            want = b.scores(op, div_eps=eps)
        assert np.all(np.isfinite(got))
        np.testing.assert_array_less(np.abs(got - want), 1e-4 * np.abs(want) + 1e-6)


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
