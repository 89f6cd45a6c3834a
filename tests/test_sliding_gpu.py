"""The "sliding_window" cache and window attention on the GPU.

* the cache driven by the reference's script: K bytes equal the reference's
  (tests/golden/sliding_window.json), V equal the oracle's (which stores V where
  the reference builds it from the cached keys), memory_usage and shapes equal;
* snapmind_paged_gqa_decode_window (tensor-core and CUDA-core kernels) against
  dense attention over [start, len) for starts inside the first block, past
  whole blocks, and at or past the length;
* gqa_paged over the cache's layer views against the reference's Mistral flow
  (dense GQA on a dict cache, sliding-window mask in prefill, trim to the
  window after each step).
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from inputs import digest, randn
from make_golden import SLIDING_OPS, sliding_inputs
from oracle import bf16, gqa
from oracle.sliding_window import SlidingWindowOracle

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "sliding_window.json"


def test_sliding_cache_matches_reference_script(cuda_device):
    from snapmind_b200 import KV_CACHE

    d = json.loads(GOLDEN.read_text())
    cfg = d["config"]
    cache = KV_CACHE.create("sliding_window", max_seq_len=64, n_layers=cfg["n_layers"], n_heads=cfg["n_heads"],
                            head_dim=cfg["head_dim"], window_size=cfg["window_size"], block_size=4)
    oracle = SlidingWindowOracle(cfg["n_layers"], cfg["window_size"])
    for op, rec in zip(SLIDING_OPS, d["steps"]):
        kind, layer, n, _ = op
        if kind == "store":
            k, v = sliding_inputs(op, cfg)
            cache.store(layer, torch.from_numpy(k), torch.from_numpy(v), 0)
            oracle.store(layer, k, v)
        elif kind == "evict":
            cache.evict(n)
            oracle.evict(n)
        else:
            cache.reset()
            oracle.reset()
        assert cache.memory_usage() == rec["memory_usage"]
        for i, lr in enumerate(rec["layers"]):
            k, v = cache.fetch(i)
            assert list(k.shape) == lr["shape"]
            assert digest(k.cpu().numpy()) == lr["k"]
            assert np.array_equal(v.cpu().numpy(), oracle.fetch(i)[1])
    cache.check_device_errors()


def _window_pool(lens, H, D, bs, dtype, seed):
    from snapmind_b200 import PagedKVPool

    lens = np.asarray(lens)
    nbs = (lens + bs - 1) // bs
    nb = int(nbs.sum()) + 2
    perm = np.random.RandomState(seed).permutation(nb).astype(np.int32)
    W = int(nbs.max())
    tables = np.zeros((len(lens), W), np.int32)
    off = 0
    for b in range(len(lens)):
        tables[b, : nbs[b]] = perm[off: off + nbs[b]]
        off += nbs[b]
    kp = bf16.round_to_bf16(randn(seed + 1, (nb, H, bs, D)))
    vp = bf16.round_to_bf16(randn(seed + 2, (nb, H, bs, D)))
    pool = PagedKVPool(1, H, D, nb, len(lens), W, block_size=bs, dtype=dtype)
    pool.k[0].copy_(torch.from_numpy(kp).to(dtype))
    pool.v[0].copy_(torch.from_numpy(vp).to(dtype))
    pool.set_state(tables, lens, perm[off:])
    return pool, kp, vp, tables


@pytest.mark.parametrize("dtype,D,bs", [(torch.bfloat16, 128, 16), (torch.float32, 64, 16), (torch.bfloat16, 64, 32)])
def test_window_decode_matches_dense(cuda_device, dtype, D, bs):
    from snapmind_b200 import _lib

    H, Hq = 4, 16
    lens = [700, 33, 130, 1, 64, 900]
    starts = [5, 0, 16 * 3 + 7, 1, 64, 100]  # inside the first block, none, past blocks, == len, == len, deep
    pool, kp, vp, tables = _window_pool(lens, H, D, bs, dtype, seed=len(lens) + D)
    q = bf16.round_to_bf16(randn(77, (len(lens), Hq, D)))
    qt = torch.from_numpy(q).cuda().to(dtype)
    out = torch.empty((len(lens), Hq, D), dtype=dtype, device="cuda")
    st = torch.tensor(starts, dtype=torch.int32, device="cuda")
    lib = _lib.load()
    max_len = max(lens)
    split = lib.snapmind_paged_gqa_decode_split_tokens(len(lens), H, max_len, bs)
    ws = torch.zeros(lib.snapmind_paged_gqa_decode_workspace_bytes(len(lens), Hq, H, D, max_len, split),
                     dtype=torch.uint8, device="cuda")
    for flags in (0, _lib.DECODE_FORCE_GENERIC):
        rc = lib.snapmind_paged_gqa_decode_window(
            qt.data_ptr(), qt.stride(0), qt.stride(1), pool.k[0].data_ptr(), pool.v[0].data_ptr(),
            _lib.dtype_code(dtype), pool.block_tables.data_ptr(), pool.max_blocks_per_seq,
            pool.max_blocks_per_seq, pool.seq_lens.data_ptr(), st.data_ptr(), out.data_ptr(), out.stride(0),
            out.stride(1), D ** -0.5, len(lens), Hq, H, D, bs, pool.num_blocks, max_len, split, flags,
            ws.data_ptr(), ws.numel(), pool.err.data_ptr(), _lib.stream_handle())
        _lib.check(rc, "decode_window")
        pool.check()
        got = out.float().cpu().numpy()
        for b, (n, s0) in enumerate(zip(lens, starts)):
            if s0 >= n:
                assert not got[b].any()
                continue
            rows_k = np.concatenate([kp[p] for p in tables[b][: (n + bs - 1) // bs]], axis=1)[:, :n]
            rows_v = np.concatenate([vp[p] for p in tables[b][: (n + bs - 1) // bs]], axis=1)[:, :n]
            want = gqa.gqa_attention(q[b][None, :, None], rows_k[None, :, s0:], rows_v[None, :, s0:],
                                     D ** -0.5)[0, :, 0]
            tol = 1e-5 if dtype == torch.float32 else 2e-2
            np.testing.assert_allclose(got[b], want, rtol=tol, atol=tol)


@torch.no_grad()
@pytest.mark.parametrize("window,prompt", [(16, 10), (16, 40), (24, 24)])
def test_gqa_paged_sliding_matches_mistral_flow(cuda_device, window, prompt):
    """Prefill with the sliding-window mask, then decode steps past the window;
    the reference layer on a dict trimmed to the window after each step (the
    Mistral block) is the comparison."""
    from snapmind_b200 import ATTENTION, KV_CACHE

    from llama_harness import DenseDictGQA, Rope

    dev = cuda_device
    rope = Rope(32, 256, 10000.0).to(dev)
    torch.manual_seed(0)
    ref = DenseDictGQA(256, 8, 2, pe=rope).to(dev)
    mine = ATTENTION.create("gqa_paged", d_model=256, n_heads=8, n_kv_heads=2, pe=rope).to(dev)
    mine.load_state_dict(ref.state_dict(), strict=False)
    cache = KV_CACHE.create("sliding_window", max_seq_len=256, n_layers=1, n_heads=2, head_dim=32,
                            window_size=window, block_size=8)
    view = cache.layer_dicts()[0]
    d = {"k": None, "v": None}
    g = torch.Generator().manual_seed(window + prompt)
    x = torch.randn(1, prompt, 256, generator=g).to(dev)
    i = torch.arange(prompt)[:, None]
    j = torch.arange(prompt)[None, :]
    mask = torch.where((j <= i) & (j >= i - window + 1), 0.0, float("-inf")).to(dev)
    a, _ = ref(x, kv_cache=d, mask=mask)
    b, _ = mine(x, kv_cache=view, mask=mask)
    torch.testing.assert_close(b, a, rtol=1e-5, atol=1e-5)
    d["k"], d["v"] = d["k"][..., -window:, :], d["v"][..., -window:, :]
    pos = prompt
    for _ in range(window + 5):
        x = torch.randn(1, 1, 256, generator=g).to(dev)
        p = torch.tensor([pos], device=dev)
        a, _ = ref(x, kv_cache=d, position_ids=p)
        b, _ = mine(x, kv_cache=view, position_ids=p)
        torch.testing.assert_close(b, a, rtol=1e-5, atol=1e-5)
        d["k"], d["v"] = d["k"][..., -window:, :], d["v"][..., -window:, :]
        pos += 1
    k, v = cache.fetch(0)
    assert torch.equal(k, d["k"]) and torch.equal(v, d["v"])
    cache.check_device_errors()
