"""The head-sharded decode with output rows stored into every rank's buffer
(snapmind_paged_gqa_decode_peers + snapmind_peer_sync), on one GPU.

The ranks are emulated in one process: each "rank" has its own pool (its kv
heads), receive buffers and flag array, all on cuda:0; the decodes and
signals of all ranks are launched one after another on one stream and the
waits come after all of them, so no kernel ever waits for one that has not
already finished.
Checked: every rank's buffer equals the concatenated local decodes bit for
bit and the oracle within the bf16/fp32 tolerances, over several epochs and
both buffer parities; a wait on a flag that nothing sets gives up and reports.
"""
import time

import numpy as np
import pytest
import torch

from oracle import bf16, gqa

pytestmark = pytest.mark.gpu


def _problem(rng, lens, H, Hq, D, dtype):
    B = len(lens)
    T = max(1, int(max(lens)))
    k = rng.standard_normal((B, H, T, D)).astype(np.float32)
    v = rng.standard_normal((B, H, T, D)).astype(np.float32)
    if dtype == torch.bfloat16:
        k, v = bf16.round_to_bf16(k), bf16.round_to_bf16(v)
    return k, v


def _shard_pool(k, v, lens, lo, hi, bs, dtype):
    from snapmind_b200 import PagedKVPool

    B, _, _, D = k.shape
    nbs = [max(1, (int(n) + bs - 1) // bs) for n in lens]
    nb, W = int(sum(nbs)), int(max(nbs))
    pool = PagedKVPool(1, hi - lo, D, nb, B, W, block_size=bs, dtype=dtype)
    kp = np.zeros((nb, hi - lo, bs, D), np.float32)
    vp = np.zeros_like(kp)
    tables = np.zeros((B, W), np.int32)
    perm = np.random.RandomState(7).permutation(nb)  # shuffled physical blocks
    off = 0
    for b in range(B):
        for j in range(nbs[b]):
            t0, t1 = j * bs, min(int(lens[b]), (j + 1) * bs)
            tables[b, j] = perm[off]
            if t1 > t0:
                kp[perm[off], :, : t1 - t0] = k[b, lo:hi, t0:t1]
                vp[perm[off], :, : t1 - t0] = v[b, lo:hi, t0:t1]
            off += 1
    pool.k[0].copy_(torch.from_numpy(kp).to(dtype))
    pool.v[0].copy_(torch.from_numpy(vp).to(dtype))
    pool.set_state(tables, np.asarray(lens, np.int32), np.zeros(0, np.int32))
    return pool


@pytest.mark.parametrize("dtype,world", [(torch.bfloat16, 2), (torch.bfloat16, 4), (torch.float32, 2)])
def test_peer_decode_emulated_ranks(cuda_device, dtype, world):
    import snapmind_b200._lib as lib
    from snapmind_b200.head_shard import PeerTargets, head_range

    rng = np.random.RandomState(11)
    H, Hq, D, bs = 8, 32, 128, 16
    lens = [0, 1, 37, 700, 2500, 64]  # empty, single token, direct, split over several CTAs
    B = len(lens)
    k, v = _problem(rng, lens, H, Hq, D, dtype)
    group = Hq // H
    pools = [_shard_pool(k, v, lens, *head_range(H, world, r), bs, dtype) for r in range(world)]
    elem = torch.empty((), dtype=dtype).element_size()
    bufs = [torch.zeros((2, B, Hq, D), dtype=dtype, device=cuda_device) for _ in range(world)]
    flags = [torch.zeros(world, dtype=torch.int32, device=cuda_device) for _ in range(world)]
    errs = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    flag_ptrs = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=cuda_device)
    out_ptrs = [torch.tensor([bf.data_ptr() + par * B * Hq * D * elem for bf in bufs], dtype=torch.int64,
                             device=cuda_device) for par in (0, 1)]
    l = lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    for epoch in range(1, 5):
        q = rng.standard_normal((B, Hq, D)).astype(np.float32)
        if dtype == torch.bfloat16:
            q = bf16.round_to_bf16(q)
        qd = torch.from_numpy(q).to(cuda_device, dtype)
        par = epoch & 1
        local = []
        for r in range(world):
            lo, hi = head_range(H, world, r)
            q_r = qd[:, lo * group: hi * group]
            local.append(pools[r].decode(0, q_r))
            t = PeerTargets(out_ptrs[par], world, lo * group, Hq * D, D)
            assert pools[r].decode(0, q_r, peers=t) is None
            lib.check(l.snapmind_peer_sync(flag_ptrs.data_ptr(), None, world, r, epoch, lib.PEER_SIGNAL,
                                           errs.data_ptr(), stream), "signal")
        for r in range(world):
            lib.check(l.snapmind_peer_sync(None, flags[r].data_ptr(), world, r, epoch, lib.PEER_WAIT,
                                           errs.data_ptr(), stream), "wait")
        torch.cuda.synchronize()
        for p in pools:
            p.check()
        assert int(errs.item()) == 0
        assert all(int(x) == epoch for f in flags for x in f.cpu())
        whole = torch.cat(local, dim=1)
        want = np.zeros((B, Hq, D))
        for b, n in enumerate(lens):
            if n:
                want[b] = gqa.gqa_attention(q[b][None, :, None], k[b][None, :, :n], v[b][None, :, :n],
                                            D ** -0.5)[0, :, 0]
        for r in range(world):
            got = bufs[r][par]
            assert torch.equal(got, whole), (epoch, r)
            np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=tol, atol=tol)
        assert float(whole[0].abs().max()) == 0.0  # the empty sequence attends nothing


def test_peer_wait_gives_up_on_a_flag_nobody_sets(cuda_device):
    import snapmind_b200._lib as lib

    flags = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    flags[0] = 5  # one rank arrived, the other never does
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    lib.check(lib.load().snapmind_peer_sync(None, flags.data_ptr(), 2, 0, 5, lib.PEER_WAIT, err.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream), "wait")
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(err.item()) & lib.DEVERR_TIMEOUT
    assert 1.5 < dt < 10.0, dt
    # the context is still usable
    assert float((torch.ones(4, device=cuda_device) * 2).sum()) == 8.0
    # an arrived epoch (or a later one) passes at once
    err.zero_()
    flags[1] = 6
    lib.check(lib.load().snapmind_peer_sync(None, flags.data_ptr(), 2, 0, 5, lib.PEER_WAIT, err.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream), "wait")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
