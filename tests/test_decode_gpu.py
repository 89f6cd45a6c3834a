"""Paged GQA decode attention on the B200 against the reference GQA forward
(golden) and the oracle (random shapes, ragged lengths, many splits)."""
import json

import numpy as np
import pytest
import torch

from inputs import randn
from oracle import bf16, gqa
from replay import GOLDEN
from test_oracle_golden import gqa_case_inputs, load_gqa, tolerance

pytestmark = pytest.mark.gpu

TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def build_pool(k_list, v_list, dtype, bs=16, seed=0, slack=1.1):
    """A PagedKVPool holding one sequence per (H, T_b, D) entry, blocks shuffled."""
    from snapmind_b200 import PagedKVPool

    B = len(k_list)
    H, D = k_list[0].shape[0], k_list[0].shape[2]
    lens = np.array([k.shape[1] for k in k_list])
    nbs = (lens + bs - 1) // bs
    nb = max(1, int(nbs.sum() * slack) + 1)
    perm = np.random.RandomState(seed).permutation(nb).astype(np.int32)
    W = max(1, int(nbs.max()))
    tables = np.zeros((B, W), np.int32)
    off = 0
    for b in range(B):
        tables[b, : nbs[b]] = perm[off : off + nbs[b]]
        off += nbs[b]
    kp = np.zeros((nb, H, bs, D), np.float32)
    vp = np.zeros_like(kp)
    for b in range(B):
        for j in range(nbs[b]):
            t0, t1 = j * bs, min(lens[b], (j + 1) * bs)
            kp[tables[b, j], :, : t1 - t0] = k_list[b][:, t0:t1]
            vp[tables[b, j], :, : t1 - t0] = v_list[b][:, t0:t1]
    pool = PagedKVPool(1, H, D, nb, max_seqs=B, max_blocks_per_seq=W, block_size=bs, dtype=dtype)
    pool.k[0].copy_(torch.from_numpy(kp).to(dtype))
    pool.v[0].copy_(torch.from_numpy(vp).to(dtype))
    pool.set_state(tables, lens, perm[off:])
    return pool, kp, vp, tables, lens


@pytest.mark.parametrize("force_generic", [False, True])
@pytest.mark.parametrize("case", json.loads((GOLDEN / "gqa_decode.json").read_text()), ids=lambda m: m["name"])
def test_decode_matches_reference_gqa_forward(cuda_device, case, force_generic):
    meta, arrays = load_gqa()
    q, k, v, out = gqa_case_inputs(case, arrays)
    dt = TORCH_DT[case["dtype"]]
    pool, *_ = build_pool([k], [v], dt)
    qt = torch.from_numpy(q)[None].cuda().to(dt)
    got = pool.decode(0, qt, scale=case["scale"], force_generic=force_generic)
    pool.check()
    rtol, atol = tolerance(case["dtype"])
    np.testing.assert_allclose(got[0].float().cpu().numpy(), out, rtol=rtol, atol=atol)


SHAPES = [(32, 8, 128), (32, 4, 64), (4, 2, 8), (8, 8, 64), (16, 1, 128), (12, 4, 96), (6, 2, 256), (20, 1, 32)]


@pytest.mark.parametrize("force_generic", [False, True])
@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("hq,h,d", SHAPES)
def test_decode_random_matches_oracle(cuda_device, hq, h, d, dt, force_generic):
    rng = np.random.RandomState(hq * 1000 + h * 10 + d)
    lens = list(rng.randint(1, 300, size=5)) + [0, 1, 15, 16, 17, 64, 65]
    rnd = {"f32": lambda a: a, "bf16": bf16.round_to_bf16, "f16": lambda a: a.astype(np.float16).astype(np.float32)}[dt]
    ks = [rnd(randn(11 + i, (h, n, d))) for i, n in enumerate(lens)]
    vs = [rnd(randn(51 + i, (h, n, d))) for i, n in enumerate(lens)]
    pool, kp, vp, tables, lens_a = build_pool(ks, vs, TORCH_DT[dt], seed=3)
    q = rnd(randn(99, (len(lens), hq, d)))
    scale = d ** -0.5
    want = gqa.paged_gqa_decode(q, kp, vp, tables, lens_a, scale, 16)
    for split in (64, 256, 0):  # several splits per sequence, then the automatic plan
        got = pool.decode(0, torch.from_numpy(q).cuda().to(TORCH_DT[dt]), scale=scale, split_tokens=split,
                          force_generic=force_generic)
        pool.check()
        rtol, atol = tolerance(dt if dt == "f32" else "bf16")
        if dt == "f16":
            rtol, atol = 5e-3, 5e-3
        np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=rtol, atol=atol)


@pytest.mark.parametrize("bs", [16, 32, 64, 8])
@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_decode_block_sizes_tensor_core_vs_oracle(cuda_device, bs, dt):
    """Block sizes 16/32/64 take the TMA + tensor-core kernel; 8 falls back to CUDA cores."""
    hq, h, d = 32, 8, 128
    lens = [1, 63, 64, 65, 200, 511, 1000]
    rnd = bf16.round_to_bf16 if dt == "bf16" else (lambda a: a.astype(np.float16).astype(np.float32))
    ks = [rnd(randn(600 + i, (h, n, d))) for i, n in enumerate(lens)]
    vs = [rnd(randn(700 + i, (h, n, d))) for i, n in enumerate(lens)]
    pool, kp, vp, tables, lens_a = build_pool(ks, vs, TORCH_DT[dt], bs=bs, seed=bs)
    q = rnd(randn(8, (len(lens), hq, d)))
    want = gqa.paged_gqa_decode(q, kp, vp, tables, lens_a, d ** -0.5, bs)
    for split in (64, 128, 0):
        got = pool.decode(0, torch.from_numpy(q).cuda().to(TORCH_DT[dt]), split_tokens=max(split, bs) if split else 0)
        pool.check()
        np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=2e-2, atol=2e-2)


def test_decode_tensor_core_matches_cuda_core(cuda_device):
    """The two kernels agree closely on a config-3-like batch (bf16)."""
    rng = np.random.RandomState(11)
    lens = list(rng.randint(1, 3000, size=24))
    h, hq, d = 8, 32, 128
    ks = [bf16.round_to_bf16(randn(800 + i, (h, n, d))) for i, n in enumerate(lens)]
    vs = [bf16.round_to_bf16(randn(900 + i, (h, n, d))) for i, n in enumerate(lens)]
    pool, *_ = build_pool(ks, vs, torch.bfloat16, seed=2)
    q = torch.from_numpy(bf16.round_to_bf16(randn(5, (len(lens), hq, d)))).cuda().to(torch.bfloat16)
    fast = pool.decode(0, q, split_tokens=256)
    slow = pool.decode(0, q, split_tokens=256, force_generic=True)
    pool.check()
    torch.testing.assert_close(fast.float(), slow.float(), rtol=1e-2, atol=1e-2)


def test_decode_long_context_many_splits_and_repeat(cuda_device):
    """Contexts up to 8192 (config-3 range), tickets reset between calls."""
    rng = np.random.RandomState(5)
    lens = list(rng.randint(1024, 8193, size=6))
    h, hq, d = 8, 32, 128
    ks = [bf16.round_to_bf16(randn(300 + i, (h, n, d))) for i, n in enumerate(lens)]
    vs = [bf16.round_to_bf16(randn(400 + i, (h, n, d))) for i, n in enumerate(lens)]
    pool, kp, vp, tables, lens_a = build_pool(ks, vs, torch.bfloat16, seed=9)
    q = bf16.round_to_bf16(randn(7, (len(lens), hq, d)))
    want = gqa.paged_gqa_decode(q, kp, vp, tables, lens_a, d ** -0.5, 16)
    qt = torch.from_numpy(q).cuda().to(torch.bfloat16)
    first = pool.decode(0, qt, split_tokens=512)
    second = pool.decode(0, qt, split_tokens=512)
    pool.check()
    assert torch.equal(first, second)
    np.testing.assert_allclose(first.float().cpu().numpy(), want, rtol=2e-2, atol=2e-2)
    generic = pool.decode(0, qt, split_tokens=512, force_generic=True)
    np.testing.assert_allclose(generic.float().cpu().numpy(), want, rtol=2e-2, atol=2e-2)


def test_decode_flags_a_split_plan_that_is_too_short(cuda_device):
    h, hq, d = 2, 4, 64
    ks = [randn(1, (h, 300, d))]
    pool, *_ = build_pool(ks, ks, torch.float32)
    q = torch.randn(1, hq, d, device="cuda")
    pool.decode(0, q, split_tokens=64, max_seq_len=128)  # plan covers 128 of 300 tokens
    with pytest.raises(RuntimeError, match="split plan"):
        pool.check()
