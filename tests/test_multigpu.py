"""KV-head-sharded paged decode on 2 GPUs (skipped with fewer GPUs): the NCCL
all-gather version, and the version whose decode kernel stores the rows into
every rank's buffer over NVLink (plain stores through CUDA IPC peer mappings),
each per layer and with one exchange per multi-layer step."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import datetime
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    from oracle import bf16, gqa
    from snapmind_b200 import PagedKVPool
    from snapmind_b200.head_shard import HeadShardedDecode, PeerHeadShardedDecode, head_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        rng = np.random.RandomState(0)  # same full problem on every rank
        B, Hq, H, D, bs = 6, 32, 8, 128, 16
        lens = rng.randint(1, 700, size=B)
        k = bf16.round_to_bf16(rng.standard_normal((B, H, int(lens.max()), D)).astype(np.float32))
        v = bf16.round_to_bf16(rng.standard_normal((B, H, int(lens.max()), D)).astype(np.float32))
        q = bf16.round_to_bf16(rng.standard_normal((B, Hq, D)).astype(np.float32))
        lo, hi = head_range(H, world, rank)
        nbs = (lens + bs - 1) // bs
        nb = int(nbs.sum())
        W = int(nbs.max())
        tables = np.zeros((B, W), np.int32)
        pool = PagedKVPool(2, hi - lo, D, nb, B, W, block_size=bs, dtype=torch.bfloat16)
        kp = np.zeros((nb, hi - lo, bs, D), np.float32)
        vp = np.zeros_like(kp)
        off = 0
        for b in range(B):
            for j in range(nbs[b]):
                t0, t1 = j * bs, min(lens[b], (j + 1) * bs)
                tables[b, j] = off
                kp[off, :, : t1 - t0] = k[b, lo:hi, t0:t1]
                vp[off, :, : t1 - t0] = v[b, lo:hi, t0:t1]
                off += 1
        for layer in range(2):  # layer 1 holds the same rows, swapped K/V
            pool.k[layer].copy_(torch.from_numpy(kp if layer == 0 else vp).to(torch.bfloat16))
            pool.v[layer].copy_(torch.from_numpy(vp if layer == 0 else kp).to(torch.bfloat16))
        pool.set_state(tables, lens, np.zeros(0, np.int32))
        dec = HeadShardedDecode(pool, Hq, world, rank)
        out = dec.decode(0, torch.from_numpy(q).cuda().to(torch.bfloat16))
        torch.cuda.synchronize()
        pool.check()
        want = np.stack([gqa.gqa_attention(q[b][None, :, None], k[b][None, :, : lens[b]], v[b][None, :, : lens[b]],
                                           D ** -0.5)[0, :, 0] for b in range(B)])
        err = float(np.abs(out.float().cpu().numpy() - want).max())
        # the fused version: several epochs (both receive buffers), each equal to the NCCL version
        pdec = PeerHeadShardedDecode(pool, Hq, world, rank)
        same = True
        for _ in range(5):
            qe = torch.from_numpy(bf16.round_to_bf16(rng.standard_normal((B, Hq, D)).astype(np.float32)))
            qe = qe.cuda().to(torch.bfloat16)
            ref = dec.decode(0, qe)
            got = pdec.decode(0, qe).clone()
            torch.cuda.synchronize()
            pdec.check()
            same = same and bool(torch.equal(got, ref))
        pdec.close()
        # one exchange per step for both layers: the fused form equals the NCCL form and
        # the per-layer decode, over four steps (both receive regions twice)
        sdec = PeerHeadShardedDecode(pool, Hq, world, rank, n_layers=2)
        for _ in range(4):
            qs = torch.from_numpy(bf16.round_to_bf16(rng.standard_normal((2, B, Hq, D)).astype(np.float32)))
            qs = qs.cuda().to(torch.bfloat16)
            # one split plan for every form, so each (layer, sequence) row is computed the same way
            ref = dec.decode_step(qs, split_tokens=64)
            per = torch.stack([dec.decode(layer, qs[layer], split_tokens=64) for layer in range(2)])
            got = sdec.decode_step(qs, split_tokens=64).clone()
            torch.cuda.synchronize()
            sdec.check()
            same = same and bool(torch.equal(got, ref)) and bool(torch.equal(ref, per))
        sdec.close()
        results[rank] = (err, same)
    finally:
        dist.destroy_process_group()


def test_head_sharded_decode_two_gpus(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    results = mp.Manager().dict()
    mp.spawn(_worker, args=(2, _free_port(), results), nprocs=2, join=True)
    assert results[0][0] < 2e-2 and results[1][0] < 2e-2, dict(results)
    assert results[0][1] and results[1][1], dict(results)
