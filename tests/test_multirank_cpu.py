"""Multi-rank host logic on CPU with world_size-2 gloo process groups: the
benchmark's barrier / max-over-ranks timing, per-rank workload seeds, and the
KV-head-sharded decode's sharding and output assembly (oracle attention per
rank, gathered with the same all-gather as the GPU path)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))


def _bench_worker(rank, world, port, results):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench

    _init(rank, world, port)
    try:
        bench.barrier(dist)
        t = bench.reduce_max(dist, float(rank + 1) * 1.5, torch.device("cpu"))
        lens = bench.seeded_lengths(1234 + 7919 * rank, 8, *bench.DECODE_CTX)
        results[rank] = (t, lens.tolist())
    finally:
        dist.destroy_process_group()


def test_bench_timing_is_max_over_ranks_and_workloads_differ():
    world, port = 2, _free_port()
    results = mp.Manager().dict()
    mp.spawn(_bench_worker, args=(world, port, results), nprocs=world, join=True)
    assert results[0][0] == results[1][0] == 3.0
    assert results[0][1] != results[1][1]


def _head_shard_worker(rank, world, port, results):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from oracle import gqa
    from snapmind_b200.head_shard import gather_heads, head_range, shard_query

    _init(rank, world, port)
    try:
        rng = np.random.RandomState(0)  # identical inputs on every rank
        B, Hq, H, D, T = 3, 8, 4, 16, 37
        q = rng.standard_normal((B, Hq, D))
        k = rng.standard_normal((B, H, T, D))
        v = rng.standard_normal((B, H, T, D))
        lo, hi = head_range(H, world, rank)
        q_local = shard_query(torch.from_numpy(q), H, world, rank).numpy()
        # this rank's attention over its kv heads only (the oracle stands in for the kernel)
        local = gqa.gqa_attention(q_local[:, :, None, :], k[:, lo:hi], v[:, lo:hi], D ** -0.5)[:, :, 0, :]
        full = gather_heads(torch.from_numpy(local), world)
        want = gqa.gqa_attention(q[:, :, None, :], k, v, D ** -0.5)[:, :, 0, :]
        results[rank] = float(np.abs(full.numpy() - want).max())
    finally:
        dist.destroy_process_group()


def test_head_sharded_decode_assembles_all_heads():
    world, port = 2, _free_port()
    results = mp.Manager().dict()
    mp.spawn(_head_shard_worker, args=(world, port, results), nprocs=world, join=True)
    assert results[0] < 1e-12 and results[1] < 1e-12


def test_head_range_rejects_uneven_split():
    from snapmind_b200.head_shard import head_range

    assert head_range(8, 4, 3) == (6, 8)
    with pytest.raises(ValueError):
        head_range(8, 3, 0)


class _OraclePool:
    """Stands in for a PagedKVPool holding kv heads [lo, hi) of every layer: decode is
    the oracle attention (the same sharding and assembly code runs around it)."""

    def __init__(self, k, v, lo, hi):
        self.k, self.v, self.lo, self.hi = k, v, lo, hi
        self.n_kv_heads = hi - lo

    def decode(self, layer, q_local, out=None, **kw):
        from oracle import gqa

        d = q_local.shape[-1]
        res = gqa.gqa_attention(q_local.numpy()[:, :, None, :], self.k[layer][:, self.lo:self.hi],
                                self.v[layer][:, self.lo:self.hi], d ** -0.5)[:, :, 0, :]
        t = torch.from_numpy(res).to(q_local.dtype)
        if out is None:
            return t
        out.copy_(t)
        return out


def _decode_step_worker(rank, world, port, results):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import gqa
    from snapmind_b200.head_shard import HeadShardedDecode, head_range

    _init(rank, world, port)
    try:
        rng = np.random.RandomState(1)  # identical inputs on every rank
        L, B, Hq, H, D, T = 3, 2, 8, 4, 16, 29
        q = rng.standard_normal((L, B, Hq, D))
        k = rng.standard_normal((L, B, H, T, D))
        v = rng.standard_normal((L, B, H, T, D))
        lo, hi = head_range(H, world, rank)
        dec = HeadShardedDecode(_OraclePool(k, v, lo, hi), Hq, world, rank)
        step = dec.decode_step(torch.from_numpy(q)).numpy()
        per_layer = np.stack([dec.decode(layer, torch.from_numpy(q[layer])).numpy() for layer in range(L)])
        want = np.stack([gqa.gqa_attention(q[layer][:, :, None, :], k[layer], v[layer], D ** -0.5)[:, :, 0, :]
                         for layer in range(L)])
        results[rank] = (float(np.abs(step - want).max()), bool(np.array_equal(step, per_layer)))
    finally:
        dist.destroy_process_group()


def test_head_sharded_decode_step_assembles_every_layer():
    """decode_step (one all-gather for all layers of a step) equals the per-layer
    decode bit for bit and the full-head oracle, on every rank."""
    world, port = 2, _free_port()
    results = mp.Manager().dict()
    mp.spawn(_decode_step_worker, args=(world, port, results), nprocs=world, join=True)
    for r in range(world):
        assert results[r][0] < 1e-12 and results[r][1], dict(results)
