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
        if f >= 724:
            # the plan balances tile work (64 x 64 tiles computed, 3 or 4 per 128-block), not
            # pair counts: the busiest shard is within one block of the mean
            tiles = [len(_native.shard_tiles(f, r, world)) for r in range(world)]
            assert sum(tiles) == ((f + 63) // 64) * ((f + 63) // 64 + 1) // 2
            assert max(tiles) <= sum(tiles) / world + 4, tiles


def test_shards_read_few_column_blocks():
    """A shard prepares every 128-column block its tiles read, so the plan's cost counts
    those blocks beside the tile work and the plans keep them few."""
    from gafime_b200 import _native
    for f, world, most in ((724, 8, 3), (512, 4, 3), (362, 2, 3), (2048, 8, 11), (2048, 4, 12)):
        reads = []
        for r in range(world):
            t = _native.shard_tiles(f, r, world)
            reads.append(len({int(x) // 2 for x in np.asarray(t).reshape(-1)}))
        assert max(reads) <= most, reads


def test_wide_table_plan_balances_work_and_reads():
    """At 2048 columns (136 Gram tiles: 16 diagonal of 3 work units, 120 of 4) the plan
    costs a shard 4 x its 64-tiles + 3 x the 128-column blocks it reads.  Over 4 shards every
    shard gets 132 tiles and reads 12 of 16 blocks; over 8, 65-67 tiles and at most 11
    blocks, the busiest shard within 1 % of the mean cost."""
    from gafime_b200 import _native
    f = 2048
    total = f * (f - 1) // 2
    for world in (4, 8):
        tiles, reads, pairs = [], [], 0
        for r in range(world):
            t = np.asarray(_native.shard_tiles(f, r, world)).reshape(-1)
            tiles.append(len(t) // 2)
            reads.append(len({int(x) // 2 for x in t}))
            pairs += len(_native.shard_pairs(f, r, world)[0])
        assert pairs == total and sum(tiles) == 528
        cost = [4 * a + 3 * b for a, b in zip(tiles, reads)]
        if world == 4:
            assert tiles == [132] * 4 and reads == [12] * 4
        else:
            assert min(tiles) >= 65 and max(tiles) <= 67 and max(reads) <= 11, (tiles, reads)
            assert max(cost) <= 1.01 * sum(cost) / world, cost


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
