"""The ``gqa_paged`` attention plugin and the paged cache's layer views on the GPU.

* the plugin against the reference GQA math (torch fp32 on the same device,
  ``DenseDictGQA``): causal prefill, decode steps, a multi-token step without a
  mask, no cache, a bf16 pool;
* an unmodified reference-style layer writing through ``PagedLayerView``;
* the end-to-end case: the Llama harness generating greedily with the plugin
  over a ``"paged"`` cache must give the reference's ids, logits and final
  cache (tests/golden/e2e_llama.*, made by running the reference), for the
  small shape and for the TinyLlama shape (22 layers, 32/4 heads, head_dim 64,
  256-token prompt, 64 generated tokens).
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from llama_harness import (SMALL, TINYLLAMA, DenseDictGQA, LlamaHarness, generate, init_weights,
                           param_checksums, prompt_ids)
from oracle.paged import PagedKVCacheOracle

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _golden():
    return json.loads((GOLDEN / "e2e_llama.json").read_text()), np.load(GOLDEN / "e2e_llama.npz")


def _pair(device, d_model=256, n_heads=8, n_kv=2, seed=0):
    from snapmind_b200 import ATTENTION
    from llama_harness import Rope

    pe = Rope(d_model // n_heads, 256, 10000.0).to(device)
    torch.manual_seed(seed)
    ref = DenseDictGQA(d_model, n_heads, n_kv, pe=pe).to(device)
    mine = ATTENTION.create("gqa_paged", d_model=d_model, n_heads=n_heads, n_kv_heads=n_kv, pe=pe).to(device)
    mine.load_state_dict(ref.state_dict())
    return ref, mine


def _causal(n, device):
    return torch.triu(torch.full((n, n), float("-inf")), diagonal=1).to(device)


@torch.no_grad()
def test_plugin_matches_reference_math_fp32(cuda_device):
    from snapmind_b200 import KV_CACHE

    dev = cuda_device
    ref, mine = _pair(dev)
    cache = KV_CACHE.create("paged", max_seq_len=256, n_layers=1, n_heads=2, head_dim=32, block_size=16)
    view = cache.layer_dicts()[0]
    d = {"k": None, "v": None}
    g = torch.Generator(device="cpu").manual_seed(1)
    # causal prefill of 37 tokens
    x = torch.randn(1, 37, 256, generator=g).to(dev)
    a, _ = ref(x, kv_cache=d, mask=_causal(37, dev))
    b, w = mine(x, kv_cache=view, mask=_causal(37, dev))
    assert w is None
    torch.testing.assert_close(b, a, rtol=1e-5, atol=1e-5)
    pos = 37
    for _ in range(5):  # decode steps
        x = torch.randn(1, 1, 256, generator=g).to(dev)
        p = torch.tensor([pos], device=dev)
        a, _ = ref(x, kv_cache=d, position_ids=p)
        b, _ = mine(x, kv_cache=view, position_ids=p)
        torch.testing.assert_close(b, a, rtol=1e-5, atol=1e-5)
        pos += 1
    # three tokens at once without a mask: every query sees every token, as in the reference
    x = torch.randn(1, 3, 256, generator=g).to(dev)
    p = torch.arange(pos, pos + 3, device=dev)[None]
    a, _ = ref(x, kv_cache=d, position_ids=p)
    b, _ = mine(x, kv_cache=view, position_ids=p)
    torch.testing.assert_close(b, a, rtol=1e-5, atol=1e-5)
    # the pool holds exactly the K/V the reference layer accumulated
    k, v = cache.fetch(0)
    assert torch.equal(k, d["k"]) and torch.equal(v, d["v"])
    cache.check_device_errors()


@torch.no_grad()
def test_plugin_without_cache_and_bf16_pool(cuda_device):
    from snapmind_b200 import PagedKVCache

    dev = cuda_device
    ref, mine = _pair(dev, seed=3)
    x = torch.randn(1, 50, 256, generator=torch.Generator().manual_seed(2)).to(dev)
    a, _ = ref(x, mask=_causal(50, dev))
    b, _ = mine(x, mask=_causal(50, dev))
    torch.testing.assert_close(b, a, rtol=1e-5, atol=1e-5)

    cache = PagedKVCache(256, 1, 2, 32, dtype=torch.bfloat16)
    b16, _ = mine(x, kv_cache=cache.layer_dicts()[0], mask=_causal(50, dev))
    torch.testing.assert_close(b16, a, rtol=2e-2, atol=2e-2)
    with pytest.raises(ValueError):
        mine(x, kv_cache=PagedKVCache(256, 1, 2, 32).layer_dicts()[0], mask=torch.zeros(50, 50, device=dev))
    with pytest.raises(TypeError):
        mine(x, kv_cache={"k": None, "v": None})


@torch.no_grad()
def test_reference_style_layer_writes_through_views(cuda_device):
    """An unmodified dict-protocol layer (read, cat, assign) over the views
    stores into the pool, with the reference's block allocation."""
    from snapmind_b200 import PagedKVCache

    dev = cuda_device
    ref, _ = _pair(dev, seed=5)
    cache = PagedKVCache(256, 2, 2, 32, block_size=16)
    views = cache.layer_dicts()
    oracle = PagedKVCacheOracle(256, 2, 2, 32, block_size=16)
    dicts = [{"k": None, "v": None} for _ in range(2)]
    g = torch.Generator().manual_seed(4)
    for n_new, layer_order in [(21, (0, 1)), (1, (1, 0)), (1, (0, 1)), (12, (0, 1))]:
        x = torch.randn(1, n_new, 256, generator=g).to(dev)
        for layer in layer_order:
            mask = _causal(n_new, dev) if dicts[layer]["k"] is None else None
            ref(x, kv_cache=dicts[layer], mask=mask)
            before = cache.num_tokens(layer)
            ref(x, kv_cache=views[layer], mask=mask)
            k_new = dicts[layer]["k"][:, :, -n_new:].cpu().numpy()
            v_new = dicts[layer]["v"][:, :, -n_new:].cpu().numpy()
            oracle.store(layer, k_new, v_new, 0)
            assert cache.num_tokens(layer) == before + n_new == views[layer]["k"].shape[-2]
    assert cache.block_tables() == oracle.block_tables
    for layer in range(2):
        k, v = cache.fetch(layer)
        assert torch.equal(k, dicts[layer]["k"]) and torch.equal(v, dicts[layer]["v"])
        assert views[layer]["k"] is views[layer]["k"]  # one gather until the cache changes
    assert len(views[0]) == 2 and list(views[0]) == ["k", "v"]
    cache.reset()
    assert views[0]["k"] is None and views[0].get("v") is None


def _run_e2e(name, shape, device, attn_cls=None, max_blocks=None):
    from snapmind_b200 import PagedGroupedQueryAttention, PagedKVCache

    meta, z = _golden()
    rec = meta[name]
    model = LlamaHarness(shape, attn_cls or PagedGroupedQueryAttention)
    init_weights(model, rec["weight_seed"])
    got = param_checksums(model)
    assert [(n, s) for n, s, _ in got] == [(n, s) for n, s, _ in rec["params"]]
    assert all(a == b for (_, _, a), (_, _, b) in zip(got, rec["params"]))
    model.to(device)
    hd = shape.d_model // shape.n_heads
    cache = PagedKVCache(shape.max_seq_len, shape.n_layers, shape.n_kv_heads, hd, max_blocks=max_blocks)
    ids, tops = generate(model, prompt_ids(shape.vocab_size, rec["prompt_len"], rec["prompt_seed"]),
                         rec["n_generated"], cache.layer_dicts())
    cache.check_device_errors()
    return rec, z, cache, ids, tops


def _check_tops(tops, rec, rtol):
    worst = 0.0
    for (vals, idx), (gv, gi) in zip(tops, rec["top2"]):
        assert idx[0] == gi[0]
        worst = max(worst, float(np.max(np.abs(np.array(vals) - gv) / (np.abs(gv) + 1e-3))))
    assert worst < rtol, worst


@torch.no_grad()
def test_e2e_small_llama_matches_reference(cuda_device):
    rec, z, cache, ids, tops = _run_e2e("small", SMALL, cuda_device)
    assert ids == rec["ids"]
    _check_tops(tops, rec, 1e-4)
    k = torch.stack([cache.fetch(i)[0][0] for i in range(SMALL.n_layers)]).cpu().numpy()
    v = torch.stack([cache.fetch(i)[1][0] for i in range(SMALL.n_layers)]).cpu().numpy()
    np.testing.assert_allclose(k, z["small_k"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(v, z["small_v"], rtol=1e-4, atol=1e-5)
    # block tables: the reference allocator's order for a 24-token prefill then 7 single tokens per layer
    oracle = PagedKVCacheOracle(SMALL.max_seq_len, SMALL.n_layers, SMALL.n_kv_heads, 32, block_size=16)
    for n_new in [rec["prompt_len"]] + [1] * (rec["n_generated"] - 1):
        for layer in range(SMALL.n_layers):
            oracle.store(layer, np.zeros((1, 2, n_new, 32), np.float32), np.zeros((1, 2, n_new, 32), np.float32), 0)
    assert cache.block_tables() == oracle.block_tables


@torch.no_grad()
def test_e2e_small_llama_reference_layer_over_views(cuda_device):
    rec, z, cache, ids, tops = _run_e2e("small", SMALL, cuda_device, attn_cls=DenseDictGQA)
    assert ids == rec["ids"]
    k = torch.stack([cache.fetch(i)[0][0] for i in range(SMALL.n_layers)]).cpu().numpy()
    np.testing.assert_allclose(k, z["small_k"], rtol=1e-4, atol=1e-5)


@torch.no_grad()
def test_e2e_tinyllama_matches_reference(cuda_device):
    # the reference's default pool (max_seq_len / block_size blocks) is shared by all
    # layers' tables, so a pool that every layer writes needs n_layers times as many
    n_blocks = TINYLLAMA.n_layers * TINYLLAMA.max_seq_len // 16
    rec, z, cache, ids, tops = _run_e2e("tinyllama", TINYLLAMA, cuda_device, max_blocks=n_blocks)
    assert ids == rec["ids"]
    _check_tops(tops, rec, 2e-4)
    idx = z["tinyllama_sample_idx"]
    for layer in range(TINYLLAMA.n_layers):
        k, v = cache.fetch(layer)
        assert list(k.shape[1:]) == rec["cache_shape"][1:]
        kf, vf = k[0].reshape(-1).cpu().numpy(), v[0].reshape(-1).cpu().numpy()
        np.testing.assert_allclose(kf[idx], z["tinyllama_k_sample"][layer], rtol=1e-3, atol=1e-4)
        np.testing.assert_allclose(vf[idx], z["tinyllama_v_sample"][layer], rtol=1e-3, atol=1e-4)
        np.testing.assert_allclose(kf.astype(np.float64).sum(), rec["k_sums"][layer], rtol=1e-3, atol=1e-2)
        np.testing.assert_allclose(vf.astype(np.float64).sum(), rec["v_sums"][layer], rtol=1e-3, atol=1e-2)


@torch.no_grad()
@pytest.mark.parametrize("use_graph", [True, False])
def test_graph_decoder_matches_reference_and_eager(cuda_device, use_graph):
    """Greedy generation with the decode step captured in a CUDA graph: the
    reference's ids for the TinyLlama case, the same final cache and block
    tables as the eager run (the small case compares them exactly)."""
    from snapmind_b200 import PagedGroupedQueryAttention, PagedKVCache
    from snapmind_b200.engine import GraphDecoder

    meta, z = _golden()
    for name, shape, n_blocks in (("small", SMALL, None), ("tinyllama", TINYLLAMA, TINYLLAMA.n_layers * 128)):
        rec = meta[name]
        model = LlamaHarness(shape, PagedGroupedQueryAttention)
        init_weights(model, rec["weight_seed"])
        model.to(cuda_device)
        hd = shape.d_model // shape.n_heads
        prompt = prompt_ids(shape.vocab_size, rec["prompt_len"], rec["prompt_seed"])
        cache = PagedKVCache(shape.max_seq_len, shape.n_layers, shape.n_kv_heads, hd, max_blocks=n_blocks)
        ids = GraphDecoder(model, cache, use_graph=use_graph).generate(prompt, rec["n_generated"])
        assert ids == rec["ids"], name
        eager = PagedKVCache(shape.max_seq_len, shape.n_layers, shape.n_kv_heads, hd, max_blocks=n_blocks)
        ids_e, _ = generate(model, prompt, rec["n_generated"], eager.layer_dicts())
        assert ids_e == ids
        assert cache.block_tables() == eager.block_tables()
        assert cache.memory_usage() == eager.memory_usage()
        for layer in range(shape.n_layers):
            k, v = cache.fetch(layer)
            ke, ve = eager.fetch(layer)
            torch.testing.assert_close(k, ke, rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(v, ve, rtol=1e-5, atol=1e-6)


@torch.no_grad()
@pytest.mark.parametrize("use_graph", [True, False])
def test_batched_graph_decoder_matches_single_sequences(cuda_device, use_graph):
    """B prompts decoded together on a PagedKVPool give, per sequence, the ids and
    cached K/V of decoding that prompt alone (small Llama shape, fp32)."""
    from snapmind_b200 import PagedGroupedQueryAttention, PagedKVCache, PagedKVPool
    from snapmind_b200.engine import BatchedGraphDecoder, GraphDecoder

    sh, B, T, n_gen = SMALL, 3, 24, 8
    model = LlamaHarness(sh, PagedGroupedQueryAttention)
    init_weights(model, 7)
    model.to(cuda_device)
    hd = sh.d_model // sh.n_heads
    prompts = torch.stack([prompt_ids(sh.vocab_size, T, 100 + i) for i in range(B)])
    pool = PagedKVPool(sh.n_layers, sh.n_kv_heads, hd, num_blocks=64, max_seqs=B, max_blocks_per_seq=8,
                       block_size=16, dtype=torch.float32)
    ids = BatchedGraphDecoder(model, pool, B, use_graph=use_graph).generate(prompts, n_gen)
    assert list(pool.host_lens[:B]) == [T + n_gen - 1] * B
    k_all, v_all = pool.gather(B)
    off = 0
    for b in range(B):
        cache = PagedKVCache(sh.max_seq_len, sh.n_layers, sh.n_kv_heads, hd)
        want = GraphDecoder(model, cache).generate(prompts[b], n_gen)
        assert ids[b] == want, b
        n = T + n_gen - 1
        for layer in range(sh.n_layers):
            k, v = cache.fetch(layer)
            got_k = k_all[layer, off: off + k.numel()].reshape(k.shape)
            got_v = v_all[layer, off: off + v.numel()].reshape(v.shape)
            torch.testing.assert_close(got_k, k, rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(got_v, v, rtol=1e-5, atol=1e-6)
        off += sh.n_kv_heads * n * hd
