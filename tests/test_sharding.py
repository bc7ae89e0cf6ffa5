"""Batch x head sharding (host logic): partitions, and a world-size-2 gloo
run in which each rank computes its head shard of the forward with the CPU
oracle and the shards are gathered back; the result must equal the
unsharded forward exactly."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from telescope_cache_b200.sharding import gather_batch, gather_heads, head_shard, local_heads, shard_range


def test_shard_range_covers_units_once():
    for units in (0, 1, 5, 16, 17, 32):
        for world in (1, 2, 3, 4, 8):
            blocks = [shard_range(units, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == units
            for (a, b), (c, d) in zip(blocks, blocks[1:]):
                assert b == c and b - a >= d - c >= b - a - 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_head_shard_keeps_gqa_groups():
    Hq, Hkv = 12, 3
    seen = []
    for r in range(2):
        k0, k1, q0, q1 = head_shard(Hq, Hkv, 2, r)
        assert q0 == k0 * 4 and q1 == k1 * 4
        seen += list(range(q0, q1))
    assert seen == list(range(Hq))
    with pytest.raises(ValueError):
        head_shard(10, 3, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import numerics as O
        r = np.random.Generator(np.random.PCG64(7))
        B, N, Hq, Hkv, D = 2, 48, 6, 3, 8
        fmap, cache = {1: 4, 2: 6}, 10
        q = r.standard_normal((B, N, Hq, D))
        k = r.standard_normal((B, N, Hkv, D))
        v = r.standard_normal((B, N, Hkv, D))
        E = Hq // Hkv
        tq, tk, tv = (torch.from_numpy(a) for a in (q, k, v))
        lq = local_heads(tq, Hq, E=E).numpy()
        lk = local_heads(tk, Hkv).numpy()
        lv = local_heads(tv, Hkv).numpy()
        kl, vl, _ = O.build_tree(lk, lv, O.qk_weights(lq, lk), 2)
        lo, llse = O.forward(lq, kl, vl, fmap, cache, 20.0)
        out = gather_heads(torch.from_numpy(np.ascontiguousarray(lo)), Hq, E=E).numpy()
        lse = gather_heads(torch.from_numpy(np.ascontiguousarray(llse)), Hq, E=E).numpy()
        # batch sharding of the same job
        b0, b1 = shard_range(B, world, rank)
        kb, vb, _ = O.build_tree(k[b0:b1], v[b0:b1], O.qk_weights(q[b0:b1], k[b0:b1]), 2)
        bo, _ = O.forward(q[b0:b1], kb, vb, fmap, cache, 20.0)
        out_b = gather_batch(torch.from_numpy(np.ascontiguousarray(bo)), B).numpy()
        if rank == 0:
            kf, vf, _ = O.build_tree(k, v, O.qk_weights(q, k), 2)
            want, want_lse = O.forward(q, kf, vf, fmap, cache, 20.0)
            np.save(os.environ["TC_SHARD_RESULT"], np.array([np.array_equal(out, want),
                                                             np.array_equal(lse, want_lse),
                                                             np.array_equal(out_b, want)]))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_head_and_batch_shards_match_unsharded(tmp_path):
    res = tmp_path / "res.npy"
    os.environ["TC_SHARD_RESULT"] = str(res)
    mp.start_processes(_worker, args=(2, _free_port(), None), nprocs=2, join=True, start_method="spawn")
    assert np.load(res).all()
