"""Multi-process sharding and merge on CPU: world_size 2 gloo ranks.

Each rank scores the pairs of its shard (gafime_shard_tiles, the assignment
gafime_allpairs_topk uses) with the oracle, keeps its local top-k, all-gathers the
candidates over gloo and merges them with gafime_topk_merge; every rank must end with
the single-process top-k.  The GPU version of the same sequence runs in bench.py."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

K = 25


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, X, y, op, out):
    import torch.distributed as dist
    from gafime_b200 import _native
    from oracle import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pi, pj = _native.shard_pairs(X.shape[1], rank, world)
        s = orc.raw_pearson(X, y, op, pi, pj, div_eps=1e-6)
        top = orc.topk(s, pi, pj, K)
        mine = (pi[top], pj[top], s[top])
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        ci = np.concatenate([g[0] for g in gathered])
        cj = np.concatenate([g[1] for g in gathered])
        cs = np.concatenate([g[2] for g in gathered])
        out[rank] = _native.merge_topk(ci, cj, cs, K)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("op", ["multiply", "divide"])
def test_two_gloo_ranks_merge_to_the_global_topk(oracle, op):
    from gafime_b200 import build
    build.build()
    rng = np.random.default_rng(8)
    X = rng.standard_normal((2000, 150)).astype(np.float32)
    y = rng.standard_normal(2000).astype(np.float32)
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, X, y, op, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    pi, pj = oracle.all_pairs(150)
    s = oracle.raw_pearson(X, y, op, pi, pj, div_eps=1e-6)
    best = oracle.topk(s, pi, pj, K)
    for r in range(2):
        i, j, sc = out[r]
        assert list(zip(i.tolist(), j.tolist())) == list(zip(pi[best].tolist(), pj[best].tolist()))
        np.testing.assert_array_equal(sc, s[best])


def test_shards_partition_the_pair_space():
    from gafime_b200 import _native
    for f, world in ((256, 8), (300, 3), (70, 4), (2, 2), (724, 8)):
        seen = set()
        loads = []
        for r in range(world):
            pi, pj = _native.shard_pairs(f, r, world)
            pairs = set(zip(pi.tolist(), pj.tolist()))
            assert not (pairs & seen)
            seen |= pairs
            loads.append(len(pairs))
        assert len(seen) == f * (f - 1) // 2
        if f >= 724:  # enough tiles for the greedy split to balance within 10 %
            assert max(loads) <= 1.1 * (f * (f - 1) / 2) / world


def test_shards_read_few_column_blocks():
    """Blocks of equal pair count trade shards toward fewer 128-column blocks per shard
    (each shard's statistics pass covers the blocks it reads); the loads are unchanged."""
    from gafime_b200 import _native
    for f, world, most in ((724, 8, 3), (512, 4, 3), (362, 2, 3), (2048, 8, 8), (2048, 4, 12)):
        reads = []
        for r in range(world):
            t = _native.shard_tiles(f, r, world)
            reads.append(len({int(x) // 2 for x in np.asarray(t).reshape(-1)}))
        assert max(reads) <= most, reads


def test_grouped_assignment_balances_the_wide_table():
    """At 2048 columns the pair space goes out in group-pair units: over 8 shards each holds
    one cross-group unit or two in-group units (8 of 16 column blocks), within 0.1 % of the
    mean pair count; over 4 shards 12 blocks each."""
    from gafime_b200 import _native
    f = 2048
    total = f * (f - 1) // 2
    for world, blocks in ((8, 8), (4, 12)):
        loads = []
        for r in range(world):
            pi, pj = _native.shard_pairs(f, r, world)
            loads.append(len(pi))
            t = _native.shard_tiles(f, r, world)
            assert len({int(x) // 2 for x in np.asarray(t).reshape(-1)}) == blocks
        assert sum(loads) == total
        assert max(loads) <= 1.001 * total / world


def test_shard_assignment_is_cheap_for_wide_matrices():
    """The assignment runs on the host before every sharded call: bounded work, kept per
    process (8000 columns over 8 shards: well under a second for all shards)."""
    import time
    from gafime_b200 import _native
    t = time.perf_counter()
    for r in range(8):
        _native.shard_tiles(8000, r, 8)
    assert time.perf_counter() - t < 2.0
    t = time.perf_counter()
    for r in range(8):
        _native.shard_tiles(8000, r, 8)
    assert time.perf_counter() - t < 0.1
