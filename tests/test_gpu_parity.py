"""Parity of the CUDA path (through the C ABI) with the oracle and the reference goldens.

Tolerances (stated per test):
  * Pearson: |r_gpu - r_oracle| <= 1e-4 * |r_oracle| + 1e-6 for every pair -- the
    required bound is 1e-4 relative; the 1e-6 absolute floor covers pairs with
    |r| ~ 1e-3 and below, where relative error is meaningless.
  * MI: 1e-5 absolute.
  * top-k: identical pair sets except pairs whose oracle score ties the k-th score
    within the tolerance (tie class).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

OPS = ["multiply", "add", "subtract", "divide"]


@pytest.fixture(scope="module")
def native():
    from gafime_b200 import _native
    _native.load()
    return _native


def bucket_for(native, X, y):
    b = native.Bucket(X.shape[0], X.shape[1])
    b.upload(X, y)
    return b


def assert_pearson_close(got, want, rtol=1e-4, atol=1e-6):
    err = np.abs(got - want)
    bad = err > rtol * np.abs(want) + atol
    assert not bad.any(), (np.flatnonzero(bad)[:10], got[bad][:5], want[bad][:5])


def assert_topk_equivalent(gi, gj, want_scores, pi, pj, k, rtol=1e-4, atol=1e-6):
    """GPU top-k (gi, gj) vs the oracle scores of all pairs: same set modulo ties."""
    mag = np.abs(want_scores)
    order = np.lexsort((pj, pi, -mag))
    kth = mag[order[k - 1]]
    tol = rtol * kth + atol
    must = {(int(pi[p]), int(pj[p])) for p in order if mag[p] > kth + tol}
    may = {(int(pi[p]), int(pj[p])) for p in order if mag[p] >= kth - tol}
    got = {(int(a), int(b)) for a, b in zip(gi, gj)}
    assert len(got) == k
    assert must <= got, sorted(must - got)[:5]
    assert got <= may, sorted(got - may)[:5]


def test_config1_centred_pearson_matches_gafime_core(native, golden, oracle):
    g = golden("config1_centred.npz")
    with bucket_for(native, g["X"], g["y"]) as b:
        s = b.scores("multiply", center=True)
        assert_pearson_close(s, g["core_scores"][:, 0])
        top = b.topk(["multiply"], 5, center=True)["multiply"]
    got = {(int(i), int(j)) for i, j in zip(top[0], top[1])}
    want = {(int(min(a, c)), int(max(a, c))) for a, c in g["selector_top_core"]}
    assert got == want
    assert (int(top[0][0]), int(top[1][0])) == (3, 15)


def test_config1_mutual_info_matches_gafime_core(native, golden):
    g = golden("config1_centred.npz")
    with bucket_for(native, g["X"], g["y"]) as b:
        m = b.scores("multiply", metric="mutual_info", center=True, mi_bins=16)
    np.testing.assert_allclose(m, g["core_scores"][:, 1], rtol=0, atol=1e-5)


@pytest.mark.parametrize("bins,key,col", [(32, "core_b32", 1), (16, "core_b16", 0)])
def test_mi_3class_matches_gafime_core(native, golden, bins, key, col):
    g = golden("mi_3class.npz")
    with bucket_for(native, g["X"], g["y"]) as b:
        m = b.scores("multiply", metric="mutual_info", center=True, mi_bins=bins)
        top = b.topk(["multiply"], 10, metric="mutual_info", center=True, mi_bins=bins)["multiply"]
    want = g[key][:, col]
    np.testing.assert_allclose(m, want, rtol=0, atol=1e-5)
    pi, pj = np.triu_indices(g["X"].shape[1], k=1)
    assert_topk_equivalent(top[0], top[1], want, pi, pj, 10, rtol=0, atol=1e-5)


@pytest.mark.parametrize("target", ["y3", "yc"])
@pytest.mark.parametrize("center", [False, True])
@pytest.mark.parametrize("op", OPS)
def test_mi_all_ops_match_oracle(native, golden, oracle, op, center, target):
    """MI of every operator, raw (fp32 interaction) and centred (fp64), 3-class and
    continuous targets: 1e-5 absolute against the oracle; the raw interactions also
    against the reference's numpy MI of the same fp32 columns."""
    g = golden("raw_mi.npz")
    X, y = g["X"], g[target]
    want = oracle.pair_mi(X, y, op, center=center, mi_bins=16, div_eps=1e-8)
    with bucket_for(native, X, y) as b:
        got = b.scores(op, metric="mutual_info", center=center, div_eps=1e-8, mi_bins=16)
        top = b.topk([op], 10, metric="mutual_info", center=center, div_eps=1e-8, mi_bins=16)[op]
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-5)
    if not center:
        np.testing.assert_allclose(got, g["mi"][0 if target == "y3" else 1, OPS.index(op)], rtol=0, atol=1e-5)
    pi, pj = np.triu_indices(X.shape[1], k=1)
    assert_topk_equivalent(top[0], top[1], want, pi, pj, 10, rtol=0, atol=1e-5)


@pytest.mark.parametrize("bins,n,f", [(64, 4000, 70), (255, 6000, 130)])
def test_mi_many_target_bins(native, oracle, bins, n, f):
    """A continuous target fills most of its bins: joint histograms of bins x U counters
    well past what fits in shared memory (U ~ bins), and at 255 bins more than one batch
    of tiles."""
    rng = np.random.default_rng(bins)
    X = rng.standard_normal((n, f)).astype(np.float32)
    y = (X[:, 2].astype(np.float64) * X[:, 5] + 0.5 * rng.standard_normal(n)).astype(np.float32)
    want = oracle.pair_mi(X, y, "multiply", center=True, mi_bins=bins)
    with bucket_for(native, X, y) as b:
        got = b.scores("multiply", metric="mutual_info", center=True, mi_bins=bins)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-5)


@pytest.mark.parametrize("target", ["y3", "yc"])
def test_unary_mi_matches_gafime_core(native, golden, oracle, target):
    g = golden("raw_mi.npz")
    with bucket_for(native, g["X"], g[target]) as b:
        got = b.unary_scores("mutual_info", mi_bins=16)
    np.testing.assert_allclose(got, g["unary_mi"][0 if target == "y3" else 1], rtol=0, atol=1e-5)


def test_unary_mi_joint_histogram_past_shared_memory(native, oracle):
    """255 x 255 bins of a uniform target: the joint histogram (260 KB) is counted in
    global memory."""
    rng = np.random.default_rng(3)
    X = rng.standard_normal((60000, 5)).astype(np.float32)
    y = rng.random(60000).astype(np.float32)
    with bucket_for(native, X, y) as b:
        got = b.unary_scores("mutual_info", mi_bins=255)
    np.testing.assert_allclose(got, oracle.unary_mi(X, y, mi_bins=255), rtol=0, atol=1e-5)


@pytest.mark.parametrize("n,f", [(33, 5), (257, 64), (1000, 70), (1, 3), (2, 2), (70001, 6)])
def test_mi_ragged_shapes(native, oracle, n, f):
    rng = np.random.default_rng(n + 7 * f)
    X = rng.standard_normal((n, f)).astype(np.float32)
    y = (rng.random(n) < 0.3).astype(np.float32)
    with bucket_for(native, X, y) as b:
        for op, center in (("multiply", True), ("add", False), ("divide", False)):
            want = oracle.pair_mi(X, y, op, center=center, mi_bins=16, div_eps=1e-6)
            got = b.scores(op, metric="mutual_info", center=center, div_eps=1e-6, mi_bins=16)
            np.testing.assert_allclose(got, want, rtol=0, atol=1e-5)


@pytest.mark.parametrize("op", OPS)
def test_raw_ops_match_oracle_and_reference_stats(native, golden, oracle, op):
    g = golden("raw_ops.npz")
    X, y = g["X"], g["y"]
    want = oracle.raw_pearson(X, y, op, div_eps=1e-8)
    with bucket_for(native, X, y) as b:
        s = b.scores(op, div_eps=1e-8)
        assert_pearson_close(s, want)
        # legacy single-pair ABI: 12 float stats equal the reference library's
        pi, pj = np.triu_indices(X.shape[1], k=1)
        ref = g["ref_stats"][OPS.index(op)]
        for p in range(0, len(pi), 7):
            st = b.compute_pair(int(pi[p]), int(pj[p]), 0, 0, OPS.index(op), 255)
            np.testing.assert_allclose(st, ref[p], rtol=2e-7, atol=0)


@pytest.mark.parametrize("n,f", [(1000, 70), (20000, 129), (33, 5), (31, 2), (257, 64), (1, 3)])
@pytest.mark.parametrize("center", [False, True])
def test_all_ops_ragged_shapes(native, oracle, n, f, center):
    rng = np.random.default_rng(n * 131 + f)
    X = np.hstack([rng.standard_normal((n, f - f // 2)),
                   rng.lognormal(0, 1, (n, f // 2))]).astype(np.float32)
    y = (rng.random(n) < 0.4).astype(np.float32)
    Xo = X - X.astype(np.float64).mean(axis=0) if center else X
    with bucket_for(native, X, y) as b:
        for op in OPS:
            want = oracle.raw_pearson(np.asarray(Xo, dtype=np.float32), y, op, div_eps=1e-6)
            got = b.scores(op, center=center, div_eps=1e-6)
            assert_pearson_close(got, want, rtol=1e-4, atol=2e-6)
            k = min(8, len(want))
            top = b.topk([op], k, center=center, div_eps=1e-6)[op]
            pi, pj = np.triu_indices(f, k=1)
            assert_topk_equivalent(top[0], top[1], want, pi, pj, k, atol=2e-6)


def test_multi_op_call_equals_single_op_calls(native):
    rng = np.random.default_rng(5)
    X = rng.standard_normal((5000, 90)).astype(np.float32)
    y = (X[:, 3] * X[:, 40] + rng.standard_normal(5000) > 0).astype(np.float32)
    with bucket_for(native, X, y) as b:
        multi = b.topk(OPS, 25, div_eps=1e-6)
        for op in OPS:
            single = b.topk([op], 25, div_eps=1e-6)[op]
            for a, c in zip(multi[op], single):
                np.testing.assert_array_equal(a, c)
        assert (int(multi["multiply"][0][0]), int(multi["multiply"][1][0])) == (3, 40)


def test_deterministic_bitwise(native):
    rng = np.random.default_rng(9)
    X = rng.lognormal(0, 1, (30000, 100)).astype(np.float32)
    y = rng.random(30000).astype(np.float32)
    with bucket_for(native, X, y) as b:
        a = [b.scores(op, div_eps=1e-6) for op in OPS]
        c = [b.scores(op, div_eps=1e-6) for op in OPS]
    for u, v in zip(a, c):
        np.testing.assert_array_equal(u, v)


def test_shards_merge_to_the_single_process_topk(native):
    rng = np.random.default_rng(11)
    X = rng.standard_normal((4000, 200)).astype(np.float32)
    y = rng.standard_normal(4000).astype(np.float32)
    with bucket_for(native, X, y) as b:
        full = b.topk(["multiply", "divide"], 50, div_eps=1e-6)
        for n_shards in (2, 3, 8):
            parts = [b.topk(["multiply", "divide"], 50, div_eps=1e-6, shard_id=s, n_shards=n_shards)
                     for s in range(n_shards)]
            for op in ("multiply", "divide"):
                ci = np.concatenate([p[op][0] for p in parts])
                cj = np.concatenate([p[op][1] for p in parts])
                cs = np.concatenate([p[op][2] for p in parts])
                mi, mj, ms = native.merge_topk(ci, cj, cs, 50)
                np.testing.assert_array_equal(mi, full[op][0])
                np.testing.assert_array_equal(mj, full[op][1])
                np.testing.assert_array_equal(ms, full[op][2])


def test_device_lists_merge_to_the_single_process_topk(native):
    """The multi-GPU exchange on device buffers: each shard's gafime_allpairs_topk_device
    lists, laid side by side as an all-gather leaves them, merge on the device
    (gafime_topk_merge_device) to the single-process top-k, including shards with no tile
    (9 shards of 200 columns: more shards than 128-column block pairs)."""
    import torch
    rng = np.random.default_rng(12)
    X = rng.standard_normal((4000, 200)).astype(np.float32)
    y = rng.standard_normal(4000).astype(np.float32)
    ops, k = ["multiply", "divide"], 50
    L = native.list_len(k)
    with bucket_for(native, X, y) as b:
        full = b.topk(ops, k, div_eps=1e-6)
        for n_shards in (1, 2, 3, 9):
            gathered = torch.zeros(n_shards * len(ops) * L * 2, dtype=torch.int64, device="cuda")
            for s in range(n_shards):
                part = torch.zeros(len(ops) * L * 2, dtype=torch.int64, device="cuda")
                torch.cuda.synchronize()
                b.topk_device(ops, k, part.data_ptr(), div_eps=1e-6, shard_id=s, n_shards=n_shards)
                torch.cuda.synchronize()
                b.merge_device(part.data_ptr(), 1, ops, k)   # a lone shard's own lists merge too
                gathered[s * len(ops) * L * 2:(s + 1) * len(ops) * L * 2] = part
            torch.cuda.synchronize()
            got = b.merge_device(gathered.data_ptr(), n_shards, ops, k)
            for op in ops:
                for u, v in zip(got[op], full[op]):
                    np.testing.assert_array_equal(u, v)


def test_shards_sum_the_same_row_chunks_as_one_gpu(native):
    """Bit-identity of a sharded top-k on a table whose row chunking would change with the
    number of tiles a shard holds (200,000 rows, 300 columns: 6 tensor-core tiles, chunks
    well under the 8192-row cap).  The chunks follow from the matrix alone, so every shard
    count gives the single-GPU scores bit for bit."""
    import torch
    rng = np.random.default_rng(21)
    X = rng.standard_normal((200_000, 300)).astype(np.float32)
    y = (X[:, 3] * X[:, 200] + rng.standard_normal(200_000)).astype(np.float32)
    ops, k = ["multiply", "add", "divide"], 40
    L = native.list_len(k)
    with bucket_for(native, X, y) as b:
        full = b.topk(ops, k, div_eps=1e-6)
        assert (int(full["multiply"][0][0]), int(full["multiply"][1][0])) == (3, 200)
        for n_shards in (2, 3):
            gathered = torch.zeros(n_shards * len(ops) * L * 2, dtype=torch.int64, device="cuda")
            for s in range(n_shards):
                part = gathered[s * len(ops) * L * 2:(s + 1) * len(ops) * L * 2]
                torch.cuda.synchronize()
                b.topk_device(ops, k, part.data_ptr(), div_eps=1e-6, shard_id=s, n_shards=n_shards)
            torch.cuda.synchronize()
            got = b.merge_device(gathered.data_ptr(), n_shards, ops, k)
            for op in ops:
                for u, v in zip(got[op], full[op]):
                    np.testing.assert_array_equal(u, v)


def test_sharded_ingest_by_column_ranges(native):
    """The sharded-ingest entry points on one GPU: features uploaded range by range
    (gafime_contiguous_bucket_upload_columns, as the ranks of a replicated bucket do before
    their all-gather) score exactly like one upload; gafime_contiguous_bucket_device_columns
    reports feature c at base + c * ld; a value written through that address and declared
    with gafime_contiguous_bucket_mark_updated is checked by the next scoring call."""
    import torch
    rng = np.random.default_rng(31)
    n, f = 5000, 300
    X = rng.standard_normal((n, f)).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    packed = np.ascontiguousarray(np.vstack([X.T, y[None, :]]))
    with bucket_for(native, X, y) as ref:
        want = ref.topk(["multiply", "divide"], 30, div_eps=1e-6)
    with native.Bucket(n, f) as b:
        for c0, c1 in ((0, 100), (100, 128), (128, 300)):
            b.upload_columns(packed[c0:c1], c0, packed[f])
        torch.cuda.synchronize()
        got = b.topk(["multiply", "divide"], 30, div_eps=1e-6)
        for op in ("multiply", "divide"):
            for u, v in zip(got[op], want[op]):
                np.testing.assert_array_equal(u, v)
        p0, ld = b.device_columns(0, f)
        p7, ld7 = b.device_columns(7, 8)
        assert ld == ld7 >= n and p7 == p0 + 7 * ld * 4

        class _Col:   # feature 7 on the device
            __cuda_array_interface__ = {"shape": (ld,), "typestr": "<f4", "data": (p7, False),
                                        "version": 3, "stream": None}

        col = torch.as_tensor(_Col(), device="cuda")
        assert torch.equal(col[:n].cpu(), torch.from_numpy(X[:, 7]))
        assert not col[n:].any()          # padding rows are zero
        col[11] = float("nan")
        torch.cuda.synchronize()
        b.mark_updated()
        with pytest.raises(native.GafimeError) as e:
            b.topk(["multiply"], 3)
        assert e.value.code == -1


def test_non_finite_input_is_rejected(native):
    X = np.ones((100, 4), dtype=np.float32)
    X[5, 2] = np.nan
    y = np.arange(100, dtype=np.float32)
    with bucket_for(native, X, y) as b:
        with pytest.raises(native.GafimeError) as e:
            b.topk(["multiply"], 3)
        assert e.value.code == -1
        # the legacy single-pair path skips NaN rows like cpu_backend.cpp:274
        st = b.compute_pair(2, 3)
        assert st[0] == 99


def test_legacy_fold_split_and_unary_ops(native, golden):
    g = golden("edge.npz")
    X, y = g["X_nan"], g["y"]
    with bucket_for(native, X, y) as b:
        for op in range(4):
            st = b.compute_pair(0, 2, 0, 0, op, 255)
            np.testing.assert_allclose(st, g["ref_stats_nan"][op][1], rtol=2e-7)  # pair (0, 2)
    rng = np.random.default_rng(2)
    X = rng.standard_normal((3000, 3)).astype(np.float32)
    y = rng.standard_normal(3000).astype(np.float32)
    mask = (np.arange(3000) % 5).astype(np.uint8)
    with native.Bucket(3000, 3) as b:
        b.upload(X, y, mask)
        st = b.compute_pair(0, 1, 1, 6, 0, 2)   # log(|a|) * a^2, fold 2 held out
    la = np.log(np.abs(X[:, 0]) + np.float32(1e-8)).astype(np.float32)
    x = (la * (X[:, 1] * X[:, 1])).astype(np.float32).astype(np.float64)
    val = mask == 2
    for h, sel in ((0, ~val), (1, val)):
        yy = y[sel].astype(np.float64)
        xx = x[sel]
        want = [sel.sum(), xx.sum(), yy.sum(), (xx * xx).sum(), (yy * yy).sum(), (xx * yy).sum()]
        np.testing.assert_allclose(st[6 * h:6 * h + 6], want, rtol=1e-5, atol=1e-3)


@pytest.fixture(scope="module")
def config2():
    from bench import make_config2
    return make_config2()


@pytest.mark.parametrize("op", OPS)
def test_config2_full_size_properties(native, oracle, config2, op):
    """Config 2 at full size (1e6 x 256, 128 normal + 128 lognormal): the k best pairs
    and a random sample of others match the oracle pair by pair, and no sampled pair
    outside the top-k beats the k-th score."""
    X, y = config2
    k = 100
    with bucket_for(native, X, y) as b:
        top = b.topk([op], k, div_eps=1e-6)[op]
        allsc = b.scores(op, div_eps=1e-6)
    gi, gj, gs = top
    want = oracle.raw_pearson(X, y, op, gi.astype(np.int32), gj.astype(np.int32), div_eps=1e-6)
    assert_pearson_close(gs, want)
    rng = np.random.default_rng(0)
    pi, pj = np.triu_indices(256, k=1)
    sample = rng.choice(len(pi), 200, replace=False)
    ws = oracle.raw_pearson(X, y, op, pi[sample].astype(np.int32), pj[sample].astype(np.int32),
                            div_eps=1e-6)
    assert_pearson_close(allsc[sample], ws)
    kth = np.abs(gs[-1])
    topset = {(int(a), int(c)) for a, c in zip(gi, gj)}
    for p, w in zip(sample, ws):
        if (int(pi[p]), int(pj[p])) not in topset:
            assert abs(w) <= kth * (1 + 1e-4) + 1e-6
    if op == "multiply":
        assert (int(gi[0]), int(gj[0])) == (3, 17)


_CUDA_CORE_SCRIPT = r"""
import sys, numpy as np
sys.path.insert(0, sys.argv[1])
from gafime_b200 import _native
d = np.load(sys.argv[2])
with _native.Bucket(d["X"].shape[0], d["X"].shape[1]) as b:
    b.upload(d["X"], d["y"])
    out = {op: b.scores(op, div_eps=1e-6) for op in ("multiply", "add", "subtract", "divide")}
np.savez(sys.argv[3], **out)
"""


def test_tensor_core_moments_match_cuda_core_kernel(native, tmp_path):
    """The tcgen05 Gram path (default) and the CUDA-core kernel (GAFIME_PAIR_MOMENTS=cuda-core,
    a separate process) score the same pairs to the parity tolerance."""
    import os
    import subprocess
    import sys
    rng = np.random.default_rng(21)
    n, f = 70_000, 300   # two full 128-blocks + a ragged one, 9 chunks of rows
    X = np.hstack([rng.standard_normal((n, 150)), rng.lognormal(0, 1, (n, 150))]).astype(np.float32)
    y = (X[:, 7] * X[:, 160] + rng.standard_normal(n) > 1.0).astype(np.float32)
    src = tmp_path / "in.npz"
    dst = tmp_path / "out.npz"
    np.savez(src, X=X, y=y)
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, GAFIME_PAIR_MOMENTS="cuda-core")
    subprocess.run([sys.executable, "-c", _CUDA_CORE_SCRIPT, repo, str(src), str(dst)], env=env,
                   check=True, timeout=600)
    ref = np.load(dst)
    with bucket_for(native, X, y) as b:
        for op in OPS:
            assert_pearson_close(b.scores(op, div_eps=1e-6), ref[op])


@pytest.mark.parametrize("kernel", ["planes", "fused"])
def test_each_gram_kernel_matches_cuda_core_kernel(native, tmp_path, kernel):
    """Both tensor-core Gram kernels, each forced with GAFIME_GRAM_KERNEL in a separate process
    (the B-planes kernel is otherwise chosen for wide tables only), score like the CUDA-core
    kernel for all four operators, with a ragged last column block and a ragged last row
    chunk."""
    import os
    import subprocess
    import sys
    rng = np.random.default_rng(23)
    n, f = 50_003, 300
    X = np.hstack([rng.standard_normal((n, 150)), rng.lognormal(0, 1, (n, 150))]).astype(np.float32)
    y = (X[:, 11] * X[:, 200] + rng.standard_normal(n) > 1.0).astype(np.float32)
    X[:, 5] += 40.0   # one column far from zero: the accuracy guard on each kernel
    src = tmp_path / "in.npz"
    np.savez(src, X=X, y=y)
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    outs = {}
    for name, extra in ((kernel, {"GAFIME_GRAM_KERNEL": kernel}), ("cuda_core", {"GAFIME_PAIR_MOMENTS": "cuda-core"})):
        dst = tmp_path / f"{name}.npz"
        subprocess.run([sys.executable, "-c", _CUDA_CORE_SCRIPT, repo, str(src), str(dst)],
                       env=dict(os.environ, **extra), check=True, timeout=600)
        outs[name] = np.load(dst)
    for op in OPS:
        assert_pearson_close(outs[kernel][op], outs["cuda_core"][op])


def test_interaction_materialiser_matches_oracle(native, golden, oracle):
    """gafime_feature_interaction_cuda equals the oracle (and through it the reference CPU
    materialiser) bit for bit, including invalid feature ids and empty combos."""
    g = golden("interaction.npz")
    off = g["off"]
    combos = [g["idx"][off[c]:off[c + 1]].tolist() for c in range(len(off) - 1)]
    np.testing.assert_array_equal(native.feature_interaction(g["X"], g["means"], combos), g["out"])
    rng = np.random.default_rng(8)
    X = rng.standard_normal((5000, 40)).astype(np.float32)
    m = X.mean(axis=0).astype(np.float32)
    combos = [[int(a)] for a in range(40)] + [[int(a), int(b)] for a, b in rng.integers(0, 40, (300, 2))]
    combos += [[1, 2, 3], [4, 50, 6], [], [-1], [7, 7, 7, 7]]
    np.testing.assert_array_equal(native.feature_interaction(X, m, combos), oracle.feature_interaction(X, m, combos))


@pytest.mark.parametrize("n,f,n_combos,size", [(10, 10, 5, 2), (1, 50, 10, 3), (1023, 127, 200, 2),
                                               (4096, 4096, 64, 2)])
def test_interaction_materialiser_smoke_shapes(native, oracle, n, f, n_combos, size):
    """The reference's kernel smoke scenarios (tests/smoke_tests/verify_kernel.py): a 10 x 10
    sanity case, a single row, prime dimensions, a 4096 x 4096 matrix; combos of distinct
    features drawn at random, bit-identical to the oracle."""
    rng = np.random.default_rng(42)
    X = rng.standard_normal((n, f)).astype(np.float32)
    m = X.mean(axis=0).astype(np.float32)
    combos = [rng.choice(f, size=size, replace=False).tolist() for _ in range(n_combos)]
    got = native.feature_interaction(X, m, combos)
    assert got.shape == (n, n_combos)
    np.testing.assert_array_equal(got, oracle.feature_interaction(X, m, combos))


def test_interaction_materialiser_rejects_bad_arguments(native):
    lib = native.load()
    X = np.zeros((4, 3), np.float32)
    m = np.zeros(3, np.float32)
    out = np.zeros((4, 2), np.float32)
    idx = np.array([0, 1], np.int32)
    bad_off = np.array([0, 2, 1], np.int32)   # decreasing
    rc = lib.gafime_feature_interaction_cuda(X.ctypes.data, m.ctypes.data, out.ctypes.data, idx.ctypes.data,
                                             bad_off.ctypes.data, 4, 3, 2)
    assert rc == -1
    assert lib.gafime_feature_interaction_cuda(None, m.ctypes.data, out.ctypes.data, idx.ctypes.data,
                                               bad_off.ctypes.data, 4, 3, 2) == -1


def test_gather_equals_upload_of_the_host_gather(native):
    """A bucket gathered on the device (column subset, bootstrap rows with repeats) scores
    bit-identically to one uploaded from the same rows and columns gathered on the host."""
    rng = np.random.default_rng(21)
    n, f = 5000, 40
    X = np.hstack([rng.standard_normal((n, 30)), rng.lognormal(0, 1, (n, 10))]).astype(np.float32)
    y = (X[:, 3] * X[:, 31] + rng.standard_normal(n) > 0).astype(np.float32)
    cols = [31, 3, 17, 0, 39, 8]
    rows = rng.integers(0, n, size=n + 123)
    with bucket_for(native, X, y) as full:
        for r in (None, rows):
            g = native.Bucket.gather(full, cols, r)
            try:
                Xh = X[:, cols] if r is None else X[r][:, cols]
                yh = y if r is None else y[r]
                with bucket_for(native, np.ascontiguousarray(Xh), yh) as h:
                    for op in OPS:
                        np.testing.assert_array_equal(g.scores(op, center=True, div_eps=1e-6),
                                                      h.scores(op, center=True, div_eps=1e-6))
                    np.testing.assert_array_equal(g.scores("multiply", metric="mutual_info", center=True),
                                                  h.scores("multiply", metric="mutual_info", center=True))
                    np.testing.assert_array_equal(g.unary_scores(), h.unary_scores())
            finally:
                g.free()
        with pytest.raises(native.GafimeError) as e:
            native.Bucket.gather(full, [0, f], None)
        assert e.value.code == -1
        with pytest.raises(native.GafimeError):
            native.Bucket.gather(full, [0, 1], np.array([0, n]))


def test_set_target_equals_fresh_upload(native):
    rng = np.random.default_rng(22)
    X = rng.standard_normal((3000, 20)).astype(np.float32)
    y1 = (rng.random(3000) < 0.5).astype(np.float32)
    y2 = (X[:, 2] * X[:, 9] > 0).astype(np.float32)
    with bucket_for(native, X, y1) as b, bucket_for(native, X, y2) as ref:
        b.scores("multiply", center=True)
        b.set_target(y2)
        np.testing.assert_array_equal(b.scores("multiply", center=True), ref.scores("multiply", center=True))
        np.testing.assert_array_equal(b.topk(OPS, 7)["add"][2], ref.topk(OPS, 7)["add"][2])
        bad = y2.copy()
        bad[7] = np.inf
        b.set_target(bad)
        with pytest.raises(native.GafimeError) as e:
            b.scores("multiply")
        assert e.value.code == -1
        b.set_target(y2)
        np.testing.assert_array_equal(b.scores("multiply"), ref.scores("multiply"))


@pytest.mark.parametrize("target", ["y3", "yc"])
def test_spearman_matches_gafime_core(native, golden, target):
    """Unaries and centred products with tied values (discrete and binary columns, 3-class
    target): ranks are exact, the sums differ from gafime_core's only in summation order."""
    g = golden("spearman.npz")
    combos = [tuple(int(v) for v in c if v >= 0) for c in g["combos"]]
    with bucket_for(native, g["X"], g[target]) as b:
        got = b.spearman(combos)
    np.testing.assert_allclose(got, g["spearman"][0 if target == "y3" else 1], rtol=0, atol=1e-12)


@pytest.mark.parametrize("center", [True, False])
@pytest.mark.parametrize("op", OPS)
def test_spearman_operators_match_oracle(native, golden, oracle, op, center):
    g = golden("spearman.npz")
    X, y = g["X"], g["yc"]
    f = X.shape[1]
    combos = [(a, c) for a in range(f) for c in range(f) if a != c][::3] + [(2,), (5,)]
    want = oracle.spearman(X, y, combos, op, center=center, div_eps=1e-6)
    with bucket_for(native, X, y) as b:
        got = b.spearman(combos, op, center=center, div_eps=1e-6)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-12)


def test_spearman_large_with_long_tie_runs(native, oracle):
    """300k rows: a binary and a 3-valued column make tie runs of ~100k rows."""
    rng = np.random.default_rng(31)
    n = 300_000
    X = np.column_stack([rng.standard_normal(n), rng.integers(0, 2, n), rng.integers(0, 3, n),
                         rng.lognormal(0, 1, n)]).astype(np.float32)
    y = (X[:, 0] * X[:, 2] + rng.standard_normal(n)).astype(np.float32)
    combos = [(0,), (1,), (2,), (0, 1), (1, 2), (0, 3), (2, 3)]
    want = oracle.spearman(X, y, combos)
    with bucket_for(native, X, y) as b:
        got = b.spearman(combos)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-12)


def test_mi_min_max_filter_edge_columns(native, oracle):
    """Pass 1 scans fp32 products and recomputes fp64 ones only near the running min / max:
    sorted columns (a new extreme every row), tiny and huge columns (outside the range the
    fp32 bound covers, so those chunks run exact), a ramp and rounded (tied) values."""
    rng = np.random.default_rng(41)
    n = 20000
    X = np.column_stack([rng.standard_normal(n), np.sort(rng.standard_normal(n)),
                         rng.standard_normal(n) * 1e-20, rng.standard_normal(n) * 1e20,
                         np.linspace(-1, 1, n), -np.sort(rng.lognormal(0, 1, n)),
                         np.round(rng.standard_normal(n), 1)]).astype(np.float32)
    y = rng.integers(0, 3, n).astype(np.float32)
    want = oracle.pair_mi(X, y, "multiply", center=True, mi_bins=16)
    with bucket_for(native, X, y) as b:
        got = b.scores("multiply", metric="mutual_info", center=True, mi_bins=16)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-5)


@pytest.mark.parametrize("n,f", [(5000, 300), (20000, 129), (777, 64), (3000, 2), (40000, 256)])
def test_streamed_upload_topk_equals_upload_then_topk(native, n, f):
    """The copy of each 128-column block overlapped with the tiles it completes: the same
    statistics, row chunks and moments as upload + topk, so bit-identical results."""
    rng = np.random.default_rng(n + f)
    X = np.hstack([rng.standard_normal((n, f - f // 2)), rng.lognormal(0, 1, (n, f // 2))]).astype(np.float32)
    y = (X[:, 0] * X[:, f - 1] + rng.standard_normal(n) > 0).astype(np.float32)
    packed = native.pack_columns(X, y)
    k = min(50, f * (f - 1) // 2)
    for ops in (OPS, ["multiply"], ["divide"]):
        with native.Bucket(n, f) as a, native.Bucket(n, f) as s:
            a.upload_packed(packed)
            want = a.topk(ops, k, div_eps=1e-6)
            got = s.topk_from_host(packed, ops, k, div_eps=1e-6)
            for op in ops:
                for u, v in zip(got[op], want[op]):
                    np.testing.assert_array_equal(u, v)
            # the bucket holds the data afterwards, like an upload
            np.testing.assert_array_equal(s.scores("add"), a.scores("add"))
    with native.Bucket(n, f) as a, native.Bucket(n, f) as s:
        a.upload_packed(packed)
        for shard in range(3):
            want = a.topk(["multiply"], k, shard_id=shard, n_shards=3)
            got = s.topk_from_host(packed, ["multiply"], k, shard_id=shard, n_shards=3)
            for u, v in zip(got["multiply"], want["multiply"]):
                np.testing.assert_array_equal(u, v)


def test_streamed_upload_rejects_non_finite(native):
    rng = np.random.default_rng(9)
    X = rng.standard_normal((1000, 140)).astype(np.float32)
    y = rng.standard_normal(1000).astype(np.float32)
    for where in ((3, 135), (999, 0)):
        Xb = X.copy()
        Xb[where] = np.nan
        with native.Bucket(1000, 140) as s:
            with pytest.raises(native.GafimeError) as e:
                s.topk_from_host(native.pack_columns(Xb, y), ["multiply"], 5)
            assert e.value.code == -1
    yb = y.copy()
    yb[10] = np.inf
    with native.Bucket(1000, 140) as s:
        with pytest.raises(native.GafimeError):
            s.topk_from_host(native.pack_columns(X, yb), ["multiply"], 5)
        s.topk_from_host(native.pack_columns(X, y), ["multiply"], 5)  # a finite upload clears it


@pytest.mark.parametrize("n,f", [(100_000, 256), (33, 5), (70_001, 129), (1, 3)])
def test_upload_rows_equals_column_upload(native, n, f):
    """Row-major upload transposed on the device: the same bucket as the column upload."""
    rng = np.random.default_rng(n + f)
    X = rng.standard_normal((n, f)).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    with native.Bucket(n, f) as a, native.Bucket(n, f) as r:
        a.upload(X, y)
        r.upload_rows(X, y)
        if f > 1 and n > 1:
            np.testing.assert_array_equal(r.scores("multiply"), a.scores("multiply"))
            np.testing.assert_array_equal(r.unary_scores(), a.unary_scores())
        for c in range(0, f, max(1, f // 7)):
            np.testing.assert_array_equal(r.compute_pair(c, (c + 1) % f), a.compute_pair(c, (c + 1) % f))
    Xb = X.copy()
    Xb[n // 2, f - 1] = np.inf
    with native.Bucket(n, f) as r:
        r.upload_rows(Xb, y)
        with pytest.raises(native.GafimeError):
            r.topk(["multiply"], 1)


def test_sharded_streamed_call_copies_and_checks_its_blocks_only(native):
    """With n_shards > 1 a streamed call moves (and checks) only the column blocks its
    tiles read: a NaN in a block it does not read leaves its result unchanged."""
    rng = np.random.default_rng(13)
    n, f, shards = 4000, 724, 8
    X = rng.standard_normal((n, f)).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    for shard in range(shards):
        tiles = native.shard_tiles(f, shard, shards)
        read = {int(v) // 2 for v in np.asarray(tiles).reshape(-1)}
        unread = [B for B in range((f + 127) // 128) if B not in read]
        if not unread:
            continue
        Xb = X.copy()
        Xb[7, 128 * unread[0]] = np.nan
        with native.Bucket(n, f) as a, native.Bucket(n, f) as s:
            a.upload(X, y)
            want = a.topk(["multiply"], 20, shard_id=shard, n_shards=shards)["multiply"]
            got = s.topk_from_host(native.pack_columns(Xb, y), ["multiply"], 20, shard_id=shard,
                                   n_shards=shards)["multiply"]
            for u, v in zip(got, want):
                np.testing.assert_array_equal(u, v)
        return
    pytest.fail("no shard leaves a column block unread")


@pytest.mark.parametrize("op", OPS)
def test_columns_far_from_zero_hold_the_bound(native, oracle, op):
    """Columns 100 standard deviations from zero (pair conditioning S2 / (n var_x) ~1e3 to
    1e4): the fp32 moment accumulations alone miss the 1e-4 bound here, so the accuracy
    guard must flag these pairs and re-score them exactly, in both the every-pair and the
    top-k calls."""
    rng = np.random.default_rng(5)
    n, f = 40000, 8
    X = (100.0 + rng.standard_normal((n, f)) * rng.uniform(0.5, 2.0, f)).astype(np.float32)
    y = (rng.random(n) < 1 / (1 + np.exp(-(X[:, 1] - X[:, 1].mean())))).astype(np.float32)
    want = oracle.raw_pearson(X, y, op, div_eps=1e-6)
    with bucket_for(native, X, y) as b:
        assert_pearson_close(b.scores(op, div_eps=1e-6), want)
        if op in ("multiply", "divide"):
            assert b.rescored() > 0
        i, j, sc = b.topk([op], 10, div_eps=1e-6)[op]
        pi, pj = np.triu_indices(f, k=1)
        pos = {(int(a), int(c)): p for p, (a, c) in enumerate(zip(pi, pj))}
        got = np.array([sc[q] for q in range(len(i))])
        ref = np.array([want[pos[(int(i[q]), int(j[q]))]] for q in range(len(i))])
        assert_pearson_close(got, ref)


@pytest.mark.parametrize("op", OPS)
def test_divisors_at_the_clamp(native, golden, oracle, op):
    """Safe divide at its clamp (eps = 1e-8): signed zeros, divisors below, at and above eps,
    subnormals, a column on the scale of eps.  The single-pair ABI's 12 stats equal the
    reference library's for every pair, and the all-pairs scores match the oracle for every
    pair (multiply (1, 2) through the accuracy guard's exact re-score)."""
    g = golden("divisors.npz")
    X, y = g["X"], g["y"]
    op_id = OPS.index(op)
    pi, pj = np.triu_indices(X.shape[1], k=1)
    with bucket_for(native, X, y) as b:
        for p in range(len(pi)):
            st = b.compute_pair(int(pi[p]), int(pj[p]), 0, 0, op_id, 255)
            np.testing.assert_allclose(st, g["ref_stats"][op_id][p], rtol=1e-6, atol=0, err_msg=str(p))
        got = b.scores(op, div_eps=1e-8)
    want = oracle.raw_pearson(X, y, op, div_eps=1e-8)
    assert_pearson_close(got, want)


def test_products_tiny_against_their_columns(native, golden, oracle):
    """Multiply (1, 2) of the clamp fixture: x is -2e-16 on a third of the rows and 0 elsewhere
    while the columns reach 3.  The Gram path rebuilds sum(a*b) from centred columns, whose
    rounding is on the scale of the columns' spreads, so the guard flags this pair and the
    exact re-score gives the oracle's score."""
    g = golden("divisors.npz")
    X, y = g["X"], g["y"]
    with bucket_for(native, X, y) as b:
        got = b.scores("multiply", div_eps=1e-8)
        assert b.rescored() >= 1
    want = oracle.raw_pearson(X, y, "multiply", div_eps=1e-8)
    pi, pj = np.triu_indices(X.shape[1], k=1)
    p = int(np.flatnonzero((pi == 1) & (pj == 2))[0])
    assert_pearson_close(got[p:p + 1], want[p:p + 1])


def test_guard_flags_nothing_on_well_conditioned_columns(native):
    """Normal and lognormal columns (the 1e6 x 256 workload's distributions, at 1e5 rows): the
    accuracy guard re-scores no pair, so such workloads pay only its check."""
    rng = np.random.default_rng(21)
    n = 100_000
    X = np.hstack([rng.standard_normal((n, 32)), rng.lognormal(0.0, 1.0, (n, 32))]).astype(np.float32)
    y = (rng.random(n) < 1 / (1 + np.exp(-X[:, 3] * X[:, 17]))).astype(np.float32)
    with bucket_for(native, X, y) as b:
        b.topk(["multiply", "add", "subtract", "divide"], 50, div_eps=1e-6)
        assert b.rescored() == 0


def test_guard_rescore_matches_the_oracle_on_a_mixed_table(native, oracle):
    """Half of the columns sit 200 standard deviations from zero (year- or price-like), half
    are N(0,1): pairs among the offset columns are re-scored, the rest are not, and every
    score and the top-k set agree with the oracle for all four operators."""
    rng = np.random.default_rng(22)
    n, f = 30000, 40
    X = rng.standard_normal((n, f))
    X[:, :20] = 2000.0 + 10.0 * X[:, :20]
    X = X.astype(np.float32)
    y = (0.02 * (X[:, 2] - 2000.0) * X[:, 30] + rng.standard_normal(n)).astype(np.float32)
    pi, pj = np.triu_indices(f, k=1)
    with bucket_for(native, X, y) as b:
        for op in OPS:
            want = oracle.raw_pearson(X, y, op, div_eps=1e-6)
            assert_pearson_close(b.scores(op, div_eps=1e-6), want)
            flagged = b.rescored()
            assert 0 < flagged < len(pi), (op, flagged)
            i, j, sc = b.topk([op], 25, div_eps=1e-6)[op]
            assert_topk_equivalent(i, j, want, pi, pj, 25)
            pos = {(int(a), int(c)): p for p, (a, c) in enumerate(zip(pi, pj))}
            assert_pearson_close(sc, np.array([want[pos[(int(a), int(c))]] for a, c in zip(i, j)]))


def test_wide_table_matches_the_oracle_and_streams_identically(native, oracle):
    """1024 columns (8 column blocks): multiply and divide against the oracle on the top-k and
    on sampled pairs, and the streamed call equal to upload + top-k (with the B-planes kernel
    forced, test_each_gram_kernel_matches_cuda_core_kernel covers that kernel)."""
    rng = np.random.default_rng(29)
    n, f = 20_000, 1024
    X = np.hstack([rng.standard_normal((n, 512)), rng.lognormal(0, 1, (n, 512))]).astype(np.float32)
    y = (X[:, 3] * X[:, 700] + rng.standard_normal(n) > 0.5).astype(np.float32)
    pi, pj = np.triu_indices(f, k=1)
    sample = np.random.default_rng(0).choice(len(pi), 3000, replace=False)
    with bucket_for(native, X, y) as b:
        for op in ("multiply", "divide"):
            allsc = b.scores(op, div_eps=1e-6)
            ws = oracle.raw_pearson(X, y, op, pi[sample].astype(np.int32), pj[sample].astype(np.int32),
                                    div_eps=1e-6)
            assert_pearson_close(allsc[sample], ws)
            gi, gj, gs = b.topk([op], 64, div_eps=1e-6)[op]
            assert_pearson_close(gs, oracle.raw_pearson(X, y, op, gi.astype(np.int32), gj.astype(np.int32),
                                                        div_eps=1e-6))
        want = b.topk(["multiply", "divide"], 64, div_eps=1e-6)
    with native.Bucket(n, f) as s:
        got = s.topk_from_host(native.pack_columns(X, y), ["multiply", "divide"], 64, div_eps=1e-6)
    for op in ("multiply", "divide"):
        for u, v in zip(got[op], want[op]):
            np.testing.assert_array_equal(u, v)


@pytest.mark.parametrize("op,center", [("multiply", True), ("add", False), ("divide", False)])
def test_quantile_mi_matches_the_oracle(native, oracle, op, center):
    """Mutual information with quantile bins on the interaction (a mode the reference does not
    have; the oracle's restatement is its definition): every pair's score at 1e-5 absolute
    and the top-k set, on a table with a planted product, tied integer codes (repeated cut
    points), a constant column (a constant interaction for multiply) and a 3-class target."""
    rng = np.random.default_rng(31)
    n, f, k = 20_000, 24, 20
    X = rng.standard_normal((n, f)).astype(np.float32)
    X[:, 6:10] = rng.integers(0, 4, (n, 4)).astype(np.float32)
    X[:, 11] = 0.0
    s0 = X[:, 2].astype(np.float64) * X[:, 5] + 0.5 * rng.standard_normal(n)
    y = np.argmax(np.stack([s0, X[:, 3] + 0.5 * rng.standard_normal(n), rng.standard_normal(n)]), axis=0)
    y = y.astype(np.float32)
    pi, pj = np.triu_indices(f, k=1)
    want = oracle.pair_mi_quantile(X, y, op, center=center, mi_bins=32, div_eps=1e-6)
    with bucket_for(native, X, y) as b:
        got = b.scores(op, metric="mutual_info_quantile", center=center, mi_bins=32, div_eps=1e-6)
        gi, gj, gs = b.topk([op], k, metric="mutual_info_quantile", center=center, mi_bins=32, div_eps=1e-6)[op]
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-5)
    assert_topk_equivalent(gi, gj, want, pi, pj, k, rtol=0, atol=1e-5)
    if op == "multiply":
        assert (int(gi[0]), int(gj[0])) == (2, 5)
