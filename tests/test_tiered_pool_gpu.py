"""Batched tiered pool on the B200: device placement decisions bit-exact against the
oracle policy, chunk bytes intact across evict/refetch, attention over the
resident tokens against the oracle."""
import numpy as np
import pytest
import torch

from oracle import bf16, gqa
from oracle.tiered_pool import TieredPoolOracle

pytestmark = pytest.mark.gpu


def _make(B=3, L=2, H=2, D=128, chunk=64, max_tokens=64 * 40, pool_chunks=24, sink=4, window=256, n_req=4):
    from snapmind_b200.tiered_pool import TieredKVPool

    pool = TieredKVPool(L, H, D, B, max_tokens, pool_chunks, chunk=chunk, sink=sink, window=window,
                        n_requests=n_req, dtype=torch.bfloat16)
    orc = TieredPoolOracle(B, pool.max_chunks, pool_chunks, chunk, sink, window, pool.stage_in_base,
                           pool.stage_out_base)
    return pool, orc


def _check_state(pool, orc, where):
    assert np.array_equal(pool.chunk_slot.cpu().numpy(), orc.chunk_slot), where
    assert np.array_equal(pool.slot_owner.cpu().numpy(), orc.slot_owner), where
    assert np.array_equal(pool.table_lens.cpu().numpy(), orc.table_lens), where
    t = pool.tables.cpu().numpy()
    for b in range(orc.batch):
        n = int((orc.chunk_slot[b] >= 0).sum())
        assert np.array_equal(t[b, :n], orc.tables[b, :n]), where


def test_tiered_pool_policy_data_and_attention(cuda_device):
    rng = np.random.RandomState(0)
    pool, orc = _make()
    B, L, H, D, chunk = pool.B, pool.L, pool.H, pool.D, pool.chunk
    lens = np.array([64 * 20 + 10, 64 * 12, 64 * 30 + 63])
    pool.fill_backing(seed=1, lens=lens + 200)
    # start: sink chunk + window chunks resident, a few older ones
    resident = []
    for b in range(B):
        n = (lens[b] + chunk - 1) // chunk
        win = [c for c in range(n) if (c + 1) * chunk > lens[b] - pool.window]
        resident.append(sorted(set([0] + win + [1, 2])))
    pool.install(lens, resident)
    # mirror in the oracle
    s = 0
    for b, cs in enumerate(resident):
        for c in cs:
            orc.slot_owner[s] = (b << 16) | c
            orc.chunk_slot[b, c] = s
            s += 1
    orc.seq_lens[:] = lens
    orc.step(0, 0, [])
    _check_state(pool, orc, "install")
    # shadow copy of every token's K/V (backing + appended) for the attention check
    shadow_k = pool.backing[:, :, 0].float().clone()  # [B][chunks][L][H][chunk][D]
    shadow_v = pool.backing[:, :, 1].float().clone()
    Hq = 4
    recent: list = []
    next_req = pool.pick_requests(rng, pool.n_requests)
    pool.prefetch(next_req)
    for step in range(1, 90):
        req = next_req
        recent = (recent + req)[-2 * pool.n_requests:]
        next_req = pool.pick_requests(rng, pool.n_requests, exclude=set(recent + req))
        q = torch.from_numpy(bf16.round_to_bf16(rng.standard_normal((L, B, Hq, D)).astype(np.float32))).cuda()
        kn = torch.from_numpy(bf16.round_to_bf16(rng.standard_normal((L, B, H, D)).astype(np.float32))).cuda()
        vn = torch.from_numpy(bf16.round_to_bf16(rng.standard_normal((L, B, H, D)).astype(np.float32))).cuda()
        out = torch.empty((L, B, Hq, D), dtype=torch.bfloat16, device="cuda")
        pos = pool.host_lens.copy()
        pool.step(q.to(torch.bfloat16), kn.to(torch.bfloat16), vn.to(torch.bfloat16), out, req, next_req)
        plan, ok = orc.step(step, 1, req)
        assert ok
        assert int(pool.plan_count.item()) == len(plan)
        assert pool.plan[: len(plan)].cpu().numpy().tolist() == [list(p) for p in plan], step
        _check_state(pool, orc, f"step {step}")
        for b in range(B):
            c, r = divmod(int(pos[b]), chunk)
            shadow_k[b, c, :, :, r] = kn[:, b].float().cpu()
            shadow_v[b, c, :, :, r] = vn[:, b].float().cpu()
        if step % 15 == 0:
            torch.cuda.synchronize()
            pool.check()
            # resident slot contents == the chunk's tokens; attention == oracle over resident tokens
            kk = pool.k.float().cpu()
            vv = pool.v.float().cpu()
            for b in range(B):
                length = int(pool.host_lens[b])
                res = [c for c in range(pool.max_chunks) if orc.chunk_slot[b, c] >= 0]
                for c in res:
                    n = min(chunk, length - c * chunk)
                    slot = orc.chunk_slot[b, c]
                    assert torch.equal(kk[:, slot, :, :n], shadow_k[b, c, :, :, :n]), (step, b, c)
                    assert torch.equal(vv[:, slot, :, :n], shadow_v[b, c, :, :, :n]), (step, b, c)
                for layer in range(L):
                    ks = np.concatenate([shadow_k[b, c, layer, :, : min(chunk, length - c * chunk)].numpy()
                                         for c in res], axis=1)
                    vs = np.concatenate([shadow_v[b, c, layer, :, : min(chunk, length - c * chunk)].numpy()
                                         for c in res], axis=1)
                    want = gqa.gqa_attention(q[layer, b].float().cpu().numpy()[None, :, None, :], ks[None],
                                             vs[None], D ** -0.5)[0, :, 0]
                    np.testing.assert_allclose(out[layer, b].float().cpu().numpy(), want, rtol=2e-2, atol=2e-2)
    torch.cuda.synchronize()
    # completed chunks were written back to the backing
    for b in range(B):
        length = int(pool.host_lens[b])
        for c in range(int(lens[b]) // chunk, length // chunk):
            assert torch.equal(pool.backing[b, c, 0].float(), shadow_k[b, c]), (b, c)
    assert pool.h2d_bytes > 0 and pool.d2h_bytes > 0


def test_tiered_pool_install_over_stale_snapshots(cuda_device):
    """Install over a pool whose residency snapshots show fewer resident chunks than
    the installed set: the decode's split plan at step 2 comes from the installed
    map, so no sequence is cut short, and the attention matches the oracle."""
    pool, _ = _make(B=2, L=1, H=2, pool_chunks=40, window=128, n_req=4)
    B, H, D, chunk = pool.B, pool.H, pool.D, pool.chunk
    lens = np.array([64 * 30, 64 * 30])
    pool.fill_backing(seed=3, lens=lens + 64)
    for snap in pool._snap:  # stale snapshots from an earlier use: nothing resident
        snap.fill_(-1)
    resident = [list(range(18)) + [29], list(range(18)) + [29]]
    pool.install(lens, resident)
    rng = np.random.RandomState(5)
    Hq = 4
    for _ in range(3):
        q = torch.from_numpy(bf16.round_to_bf16(rng.standard_normal((1, B, Hq, D)).astype(np.float32))).cuda()
        kn = torch.from_numpy(bf16.round_to_bf16(rng.standard_normal((1, B, H, D)).astype(np.float32))).cuda()
        out = torch.empty((1, B, Hq, D), dtype=torch.bfloat16, device="cuda")
        pool.step(q.to(torch.bfloat16), kn.to(torch.bfloat16), kn.to(torch.bfloat16), out, [], None)
        assert pool._resident_bound() >= int((pool.chunk_slot >= 0).sum(dim=1).max().item())
    torch.cuda.synchronize()
    pool.check()  # a split plan sized below a resident length would have flagged a device error
    kk, vv = pool.k.float().cpu(), pool.v.float().cpu()
    slots = pool.chunk_slot.cpu().numpy()
    for b in range(B):
        length = int(pool.host_lens[b])
        res = [c for c in range(pool.max_chunks) if slots[b, c] >= 0]
        ks = np.concatenate([kk[0, slots[b, c], :, : min(chunk, length - c * chunk)].numpy() for c in res], axis=1)
        vs = np.concatenate([vv[0, slots[b, c], :, : min(chunk, length - c * chunk)].numpy() for c in res], axis=1)
        want = gqa.gqa_attention(q[0, b].float().cpu().numpy()[None, :, None, :], ks[None], vs[None], D ** -0.5)
        np.testing.assert_allclose(out[0, b].float().cpu().numpy(), want[0, :, 0], rtol=2e-2, atol=2e-2)


def test_tiered_pool_rejects_too_many_requests(cuda_device):
    pool, _ = _make(n_req=2)
    with pytest.raises(ValueError, match="staging slots"):
        pool.prefetch([(0, 1), (0, 2), (1, 1)])
