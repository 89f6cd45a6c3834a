"""B200 PagedKVCache against the reference's own behaviour (golden scripts), the
reference's test suite (fixture substitution) and random scripts checked by the oracle."""
import numpy as np
import pytest
import torch

from inputs import randn
from oracle import bf16, paged
from replay import load_paged_ops, replay

pytestmark = pytest.mark.gpu


def _cache_factory(dtype):
    from snapmind_b200.kv_cache.paged import PagedKVCache

    return lambda cfg: PagedKVCache(**cfg, dtype=dtype, device="cuda")


def _to_input(a, tag):
    t = torch.from_numpy(a).cuda()
    return t.to(torch.bfloat16) if tag == "bf16" else t


def _f32_np(t):
    return t.float().cpu().numpy()


def _bf16_np(t):
    return t.to(torch.bfloat16).contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("scenario", load_paged_ops(), ids=lambda s: s["name"])
def test_fp32_pool_replays_reference_bit_exact(cuda_device, scenario):
    replay(scenario, _cache_factory(torch.float32), _to_input, _f32_np, "f32")


@pytest.mark.parametrize("scenario", load_paged_ops(), ids=lambda s: s["name"])
def test_bf16_pool_replays_reference_bit_exact(cuda_device, scenario):
    # the reference pool is fp32; fp32 -> bf16 rounding of it equals rounding at append
    replay(scenario, _cache_factory(torch.bfloat16), _to_input, _bf16_np, "bf16")


def test_cpu_inputs_are_accepted(cuda_device):
    from snapmind_b200.kv_cache.paged import PagedKVCache

    c = PagedKVCache(max_seq_len=64, n_layers=1, n_heads=2, head_dim=32)
    k = torch.randn(1, 2, 5, 32)
    c.store(0, k, k * 2, 0)
    kk, vv = c.fetch(0)
    assert kk.is_cuda and torch.equal(kk.cpu(), k) and torch.equal(vv.cpu(), k * 2)
    c.check_device_errors()


# ---- the reference test suite (snapmind/tests/kv_cache/test_paged.py) on the B200 plugin
@pytest.fixture
def paged_cache(cuda_device):
    from snapmind_b200.kv_cache.paged import PagedKVCache

    return PagedKVCache(max_seq_len=128, n_layers=2, n_heads=4, head_dim=64, block_size=16)


def _r(*shape):
    return torch.randn(*shape, device="cuda")


class TestReferenceSuiteOnB200:
    def test_store_fetch_round_trip(self, paged_cache):
        k, v = _r(1, 4, 10, 64), _r(1, 4, 10, 64)
        paged_cache.store(layer_idx=0, key=k, value=v, seq_pos=0)
        k_out, v_out = paged_cache.fetch(layer_idx=0)
        assert torch.allclose(k, k_out, atol=1e-6) and torch.allclose(v, v_out, atol=1e-6)

    def test_append_grows_sequence(self, paged_cache):
        k1, v1 = _r(1, 4, 5, 64), _r(1, 4, 5, 64)
        paged_cache.store(0, k1, v1, 0)
        k2, v2 = _r(1, 4, 3, 64), _r(1, 4, 3, 64)
        paged_cache.store(0, k2, v2, 5)
        k_out, _ = paged_cache.fetch(0)
        assert k_out.shape[-2] == 8
        assert torch.allclose(k_out[:, :, :5], k1, atol=1e-6) and torch.allclose(k_out[:, :, 5:8], k2, atol=1e-6)

    def test_crosses_block_boundary(self, paged_cache):
        k = _r(1, 4, 20, 64)
        paged_cache.store(0, k, k, 0)
        k_out, _ = paged_cache.fetch(0)
        assert k_out.shape[-2] == 20 and torch.allclose(k, k_out, atol=1e-6)

    def test_different_layers_are_independent(self, paged_cache):
        k0, k1 = _r(1, 4, 5, 64), _r(1, 4, 7, 64)
        paged_cache.store(0, k0, k0, 0)
        paged_cache.store(1, k1, k1, 0)
        assert paged_cache.fetch(0)[0].shape[-2] == 5 and paged_cache.fetch(1)[0].shape[-2] == 7

    def test_evict_reduces_length(self, paged_cache):
        k = _r(1, 4, 20, 64)
        paged_cache.store(0, k, k, 0)
        paged_cache.evict(tokens_to_keep=10)
        assert paged_cache.fetch(0)[0].shape[-2] <= 10

    def test_evict_keeps_most_recent(self, paged_cache):
        k = _r(1, 4, 20, 64)
        paged_cache.store(0, k, k, 0)
        paged_cache.evict(tokens_to_keep=5)
        k_out, _ = paged_cache.fetch(0)
        assert torch.allclose(k_out[:, :, -5:], k[:, :, -5:], atol=1e-6)

    def test_evict_all_layers(self, paged_cache):
        for i in range(2):
            k = _r(1, 4, 15, 64)
            paged_cache.store(i, k, k, 0)
        paged_cache.evict(tokens_to_keep=3)
        for i in range(2):
            assert paged_cache.fetch(i)[0].shape[-2] == 3

    def test_reset_clears_all(self, paged_cache):
        paged_cache.store(0, _r(1, 4, 10, 64), _r(1, 4, 10, 64), 0)
        paged_cache.store(1, _r(1, 4, 10, 64), _r(1, 4, 10, 64), 0)
        paged_cache.reset()
        for i in range(2):
            assert paged_cache.fetch(i)[0].numel() == 0

    def test_empty_cache_returns_empty(self, paged_cache):
        assert paged_cache.fetch(0)[0].numel() == 0

    def test_blocks_are_reused_after_eviction(self, paged_cache):
        k = _r(1, 4, 32, 64)
        paged_cache.store(0, k, k, 0)
        before = paged_cache.memory_usage()
        paged_cache.evict(tokens_to_keep=4)
        paged_cache.store(0, _r(1, 4, 10, 64), _r(1, 4, 10, 64), 0)
        assert paged_cache.memory_usage()["used_blocks"] <= before["used_blocks"]

    def test_memory_usage_keys(self, paged_cache):
        paged_cache.store(0, _r(1, 4, 10, 64), _r(1, 4, 10, 64), 0)
        usage = paged_cache.memory_usage()
        assert {"num_tokens", "total_bytes", "used_blocks", "max_blocks"} <= set(usage)

    def test_out_of_blocks_message(self, paged_cache):
        with pytest.raises(RuntimeError, match="PagedKVCache: out of blocks"):
            paged_cache.store(0, _r(1, 4, 200, 64), _r(1, 4, 200, 64), 0)


# ---- random scripts, bit-exact against the oracle ------------------------------
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random_scripts_match_oracle(cuda_device, dtype, seed):
    from snapmind_b200.kv_cache.paged import PagedKVCache

    rng = np.random.RandomState(seed)
    L, H, D, bs, mb = 3, int(rng.choice([1, 2, 8])), int(rng.choice([8, 64, 128])), int(rng.choice([4, 16, 32])), 40
    ours = PagedKVCache(max_seq_len=mb * bs, n_layers=L, n_heads=H, head_dim=D, block_size=bs, max_blocks=mb, dtype=dtype)
    ref = paged.PagedKVCacheOracle(max_seq_len=mb * bs, n_layers=L, n_heads=H, head_dim=D, block_size=bs, max_blocks=mb)
    np_round = {torch.float32: lambda a: a, torch.bfloat16: bf16.round_to_bf16,
                torch.float16: lambda a: a.astype(np.float16).astype(np.float32)}[dtype]
    for step in range(60):
        r = rng.rand()
        layer = int(rng.randint(L))
        if r < 0.6:
            t = int(rng.randint(0, 3 * bs))
            k = randn(1000 * seed + step, (1, H, t, D))
            v = randn(5000 + 1000 * seed + step, (1, H, t, D))
            errs = []
            for obj, kk, vv in ((ref, np_round(k), np_round(v)), (ours, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())):
                try:
                    obj.store(layer, kk, vv, 0)
                    errs.append(None)
                except RuntimeError as e:
                    errs.append(str(e))
            assert errs[0] == errs[1]
        elif r < 0.75:
            keep = int(rng.randint(0, 3 * bs))
            errs = []
            for obj in (ref, ours):
                try:
                    obj.evict(keep)
                    errs.append(None)
                except RuntimeError as e:
                    errs.append(type(e).__name__)
            assert errs[0] == errs[1]
        elif r < 0.78:
            ref.reset()
            ours.reset()
        assert ours.block_tables() == ref.block_tables
        assert ours._slot_counts == ref.slot_counts
        assert ours._free_blocks == ref.free_blocks
        for li in range(L):
            try:
                rk, rv = ref.fetch(li)
            except RuntimeError:
                with pytest.raises(RuntimeError):
                    ours.fetch(li)
                continue
            ok, ov = ours.fetch(li)
            assert tuple(ok.shape) == rk.shape
            np.testing.assert_array_equal(ok.float().cpu().numpy(), rk)
            np.testing.assert_array_equal(ov.float().cpu().numpy(), rv)
    ours.check_device_errors()
