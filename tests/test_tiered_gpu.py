"""B200 TieredPagedKVCache against the reference's recorded behaviour and the oracle."""
import numpy as np
import pytest
import torch

from inputs import randn
from oracle import tiered as otiered
from replay import load_tiered_ops, replay_tiered

pytestmark = pytest.mark.gpu


def _entry_arrays(cache, cid, layer):
    torch.cuda.synchronize()  # cold entries arrive by async D2H on the copy stream
    e = cache._chunks[cid][layer]
    if e["k"] is None:
        return None
    return e["k"].float().cpu().numpy(), e["v"].float().cpu().numpy()


def _to_input(a, tag):
    t = torch.from_numpy(a).cuda()
    return t.to(torch.bfloat16) if tag == "bf16" else t


@pytest.mark.parametrize("scenario", load_tiered_ops(), ids=lambda s: s["name"])
def test_tiered_replays_reference_bit_exact(cuda_device, scenario):
    from snapmind_b200.kv_cache.tiered import TieredPagedKVCache

    cache = TieredPagedKVCache(**scenario["config"], device="cuda")
    replay_tiered(
        scenario,
        cache,
        to_input=_to_input,
        to_numpy=lambda t: t.float().cpu().numpy(),
        make_score=lambda s, as_tensor: torch.tensor(s) if as_tensor else s,
        state_of=lambda c: (c._hot_set, c._chunks.keys(), c.chunk_layout(), c._total_tokens),
        entry_arrays=_entry_arrays,
    )


def test_tiered_registered_and_cold_chunks_in_pinned_memory(cuda_device):
    import snapmind_b200
    from snapmind_b200.kv_cache.tiered import TieredPagedKVCache

    assert snapmind_b200.KV_CACHE.get("tiered") is TieredPagedKVCache
    c = snapmind_b200.KV_CACHE.create("tiered", max_seq_len=1024, n_layers=1, n_heads=2, head_dim=64,
                                      pool_tokens=128, chunk_size=64)
    for t in range(64 * 6):
        k = torch.randn(1, 2, 1, 64, device="cuda")
        c.store(0, k, k, t)
    c.store(0, torch.randn(1, 2, 1, 64, device="cuda"), torch.randn(1, 2, 1, 64, device="cuda"), 64 * 6)
    torch.cuda.synchronize()
    cold = [cid for cid in c._chunks if cid not in c._hot_set]
    assert cold, "expected evicted chunks"
    for cid in cold:
        assert c._chunks[cid][0]["k"].is_pinned()
    for cid in c._hot_set:
        assert c._chunks[cid][0]["k"].is_cuda
    u = c.memory_usage()
    assert u["gpu_bytes"] > 0 and u["cpu_bytes"] > 0


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_tiered_random_ops_match_oracle(cuda_device, seed):
    from snapmind_b200.kv_cache.tiered import TieredPagedKVCache

    rng = np.random.RandomState(seed)
    L, H, D, chunk = 2, 2, 32, 8
    pool = int(rng.choice([8, 16, 24, 40]))
    ours = TieredPagedKVCache(max_seq_len=4096, n_layers=L, n_heads=H, head_dim=D, pool_tokens=pool,
                              chunk_size=chunk, device="cuda")
    ref = otiered.TieredPagedKVCacheOracle(max_seq_len=4096, n_layers=L, n_heads=H, head_dim=D, pool_tokens=pool,
                                           chunk_size=chunk)
    pos = 0
    for step in range(80):
        r = rng.rand()
        if r < 0.7:
            layer = int(rng.randint(L))
            t = int(rng.randint(1, 2 * chunk))
            p = pos if rng.rand() < 0.8 else int(rng.randint(0, pos + 1))
            k = randn(10000 * seed + step, (1, H, t, D))
            v = randn(20000 * seed + step, (1, H, t, D))
            ours.store(layer, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), p)
            ref.store(layer, k, v, p)
            if layer == L - 1:
                pos = max(pos, p + t)
        elif r < 0.85:
            cids = list(ref.chunks)
            scores = {cid: float(rng.rand()) for cid in cids if rng.rand() < 0.7}
            ours.score_and_repage(scores)
            ref.score_and_repage(scores)
        elif r < 0.95:
            ours.layer_dicts()
            ref.layer_dicts()
        else:
            ours.reset()
            ref.reset()
            pos = 0
        assert ours._hot_set == ref.hot_set
        assert ours.chunk_layout() == ref.chunk_layout()
        assert ours.memory_usage() == ref.memory_usage()
        for li in range(L):
            ok, ov = ours.fetch(li)
            rk, rv = ref.fetch(li)
            assert tuple(ok.shape) == tuple(rk.shape)
            np.testing.assert_array_equal(ok.cpu().numpy(), rk)
            np.testing.assert_array_equal(ov.cpu().numpy(), rv)
