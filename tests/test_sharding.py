"""Multi-GPU partitioning logic on CPU (gloo, world size 2): row and vocab
shards, the all-gather of per-row results and the max-merge of vocab-shard
partials, checked against the single-process margin rules
(src/diagnosis.rs:58-80, 490-492)."""
import os
import socket

import numpy as np
import pytest

from laplacesscissors_b200 import diagnosis
from laplacesscissors_b200.sharding import (merge_vocab_partials, gather_rows, pack_key, pack_partials, row_shard,
                                            shard_partials, unpack_key, unpack_partials, vocab_shard)


@pytest.mark.parametrize("total,world", [(4096, 8), (10, 3), (151936, 8), (5, 8), (0, 2)])
def test_row_shards_cover_exactly(total, world):
    spans = [row_shard(total, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == total
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1
    assert vocab_shard(total, world, world - 1) == spans[-1]
    with pytest.raises(ValueError):
        row_shard(total, world, world)


def test_key_packing_orders_like_first_argmax():
    rng = np.random.default_rng(3)
    v = rng.standard_normal(1000).astype(np.float32)
    v[[5, 17, 900]] = 7.5  # ties: the lowest index must win
    v[3] = -0.0
    keys = pack_key(v, np.arange(1000))
    val, idx = unpack_key(keys.max(keepdims=True))
    assert val[0] == 7.5 and idx[0] == 5
    back, ix = unpack_key(keys)
    assert np.array_equal(back.view(np.uint32), v.view(np.uint32)) and np.array_equal(ix, np.arange(1000))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        rows, vocab = 37, 1001
        z = rng.standard_normal((rows, vocab)).astype(np.float32)
        z[4, 100] = z[4, 900] = 9.0  # a tie across shards
        targets = rng.integers(0, vocab, rows).astype(np.uint32)
        targets[4] = 100
        v0, v1 = vocab_shard(vocab, world, rank)
        keys, tl = shard_partials(z[:, v0:v1], targets, v0)
        margin, amax, tlog = merge_vocab_partials(keys, tl, targets)
        # the packed form of the GPU path: one all-reduce MAX over int64 [2 rows]
        import torch
        packed = torch.from_numpy(pack_partials(keys, tl))
        dist.all_reduce(packed, op=dist.ReduceOp.MAX)
        p_margin, p_amax, p_tl = unpack_partials(packed.numpy(), targets)
        assert np.array_equal(p_margin, margin) and np.array_equal(p_amax, amax)
        assert np.array_equal(p_tl.view(np.uint32), tlog.view(np.uint32))
        lo, hi = row_shard(rows, world, rank)
        got = gather_rows({"margin": margin[lo:hi], "argmax": amax[lo:hi], "target": tlog[lo:hi]}, rows)
        q.put((rank, margin, amax, tlog, got["margin"], got["argmax"], got["target"], z, targets))
    finally:
        dist.destroy_process_group()


def test_vocab_shards_merge_and_row_gather_world2():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, margin, amax, tlog, g_margin, g_amax, g_tl, z, targets in results:
        for i in range(z.shape[0]):
            t = int(targets[i])
            assert amax[i] == diagnosis.argmax(z[i])
            assert margin[i] == diagnosis.minimum_margin(z[i], t)
            assert tlog[i] == z[i, t]
        assert np.array_equal(g_margin, margin) and np.array_equal(g_amax, amax) and np.array_equal(g_tl, tlog)
