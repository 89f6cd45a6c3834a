"""MLA latent cache on the B200: the reference layer's cache protocol replayed on
PagedLatentDict (bit-exact contents), and the batched latent pool against the oracle."""
import json

import numpy as np
import pytest
import torch

from inputs import digest, randn
from oracle import bf16, paged
from replay import GOLDEN

pytestmark = pytest.mark.gpu


def _mla_cases():
    return json.loads((GOLDEN / "mla.json").read_text())


@pytest.mark.parametrize("case", _mla_cases(), ids=lambda m: m["name"])
def test_paged_latent_dict_replays_reference_cache(cuda_device, case):
    from snapmind_b200.mla import MLALatentPool, PagedLatentDict

    arrays = np.load(GOLDEN / "mla.npz")
    dt = torch.bfloat16 if case["dtype"] == "bf16" else torch.float32
    R, P = case["kv_lora_rank"], case["qk_rope_head_dim"]

    def rows(key):
        a = arrays[f"{case['name']}__{key}"]
        t = torch.from_numpy(bf16.bf16_to_f32(a) if case["dtype"] == "bf16" else a)
        return t.to("cuda", dt)

    pool = MLALatentPool(n_layers=2, num_blocks=8, max_seqs=2, max_blocks_per_seq=4, block_size=16,
                         kv_lora_rank=R, rope_dim=P, dtype=dt)
    d = PagedLatentDict(pool, layer=1, batch=2)
    for si, st in enumerate(case["steps"]):
        lat_new, rope_new = rows(f"s{si}_latent_new"), rows(f"s{si}_rope_new")
        # the cache protocol of MultiHeadLatentAttention.forward (mla.py:208-215)
        cached_lat, cached_rope = d.get("k"), d.get("k_rope")
        if cached_lat is not None:
            lat_new = torch.cat([cached_lat, lat_new], dim=-2)
            rope_new = torch.cat([cached_rope, rope_new], dim=-2)
        d["k"], d["k_rope"] = lat_new, rope_new
        k, kr = d["k"], d["k_rope"]
        assert list(k.shape) == st["k_shape"] and list(kr.shape) == st["k_rope_shape"]
        if dt == torch.bfloat16:
            bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
            assert digest(bits(k)) == st["k_bits"] and digest(bits(kr)) == st["k_rope_bits"]
        else:
            assert digest(k.cpu().numpy()) == st["k_bits"] and digest(kr.cpu().numpy()) == st["k_rope_bits"]
    pool.check()


def test_latent_pool_random_append_gather_matches_oracle(cuda_device):
    from snapmind_b200.mla import MLALatentPool

    rng = np.random.RandomState(4)
    L, B, bs, R, P = 2, 5, 64, 512, 64
    pool = MLALatentPool(n_layers=L, num_blocks=64, max_seqs=B, max_blocks_per_seq=12, block_size=bs,
                         kv_lora_rank=R, rope_dim=P, dtype=torch.bfloat16)
    pool.latent.zero_()
    pool.rope.zero_()
    lat_pool = np.zeros((L, 64, 1, bs, R), np.float32)
    rope_pool = np.zeros((L, 64, 1, bs, P), np.float32)
    tables, lens, top = np.zeros((B, 12), np.int64), np.zeros(B, np.int64), 64
    free = np.arange(63, -1, -1)
    for step, n_new in enumerate([100, 1, 1, 63, 1, 130]):
        pool.reserve(n_new, batch=B)
        tables, lens, top, err = paged.reserve(tables, lens, free, top, n_new, bs)
        assert err is None
        lat = bf16.round_to_bf16(randn(50 + step, (L, B, n_new, R)))
        rope = bf16.round_to_bf16(randn(90 + step, (L, B, n_new, P)))
        pool.append(None, torch.from_numpy(lat).cuda().to(torch.bfloat16), torch.from_numpy(rope).cuda().to(torch.bfloat16))
        paged.append(lat_pool, lat_pool, tables, lens - n_new, lat[:, :, None], lat[:, :, None], bs)
        paged.append(rope_pool, rope_pool, tables, lens - n_new, rope[:, :, None], rope[:, :, None], bs)
    assert np.array_equal(pool.block_tables.cpu().numpy(), tables)
    for layer in range(L):
        lat_g, rope_g = pool.gather(layer, B)
        want_lat, _ = paged.gather(lat_pool[layer:layer + 1], lat_pool[layer:layer + 1], tables, lens, bs)
        want_rope, _ = paged.gather(rope_pool[layer:layer + 1], rope_pool[layer:layer + 1], tables, lens, bs)
        np.testing.assert_array_equal(lat_g.float().cpu().numpy().reshape(-1), want_lat[0])
        np.testing.assert_array_equal(rope_g.float().cpu().numpy().reshape(-1), want_rope[0])
    pool.check()
