"""Generate golden vectors by running the reference snapmind code itself.

Usage (in a checkout where the reference is importable):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference /path/to/snapmind

Writes, next to this script:
  * paged_ops.json      — scripted store/fetch/evict/reset/memory_usage/layer_dicts
                          sequences on the reference ``PagedKVCache``: block
                          tables, slot counts, free sets, errors and sha256 of
                          every fetched tensor after each step;
  * paged_batched.json  — many sequences on one shuffled shared pool: each
                          (sequence, layer) is a reference ``PagedKVCache`` with
                          the given block table, prefilled then appended one
                          token; sha256 of the fetched K/V;
  * gqa_decode.npz / gqa_decode.json — the reference ``GroupedQueryAttention``
                          forward for one decode token over a ``PagedKVCache``
                          (q/k/v projections saved, out_proj set to identity so
                          the output is the attention result itself);
  * tiered_ops.json, mla.npz/json, indexer.npz/json — the tiered cache, MLA
                          layer and lookahead indexer driven the same way;
  * engine_indexer.json — the reference engine's indexer cadence
                          (GenerateEngine._run_indexer) over a tiered cache
                          and a lookahead indexer: scores, hot set and live
                          contents after every re-page;
  * e2e_llama.npz / e2e_llama.json — the reference ``LlamaModel`` generating
                          greedily from a seeded prompt with seeded N(0, 0.02)
                          weights (a small shape and the TinyLlama shape).

Inputs are regenerated from seeds with ``inputs.randn`` (frozen RandomState
stream), so the fixtures hold seeds, small tensors and digests only.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from inputs import digest, engine_hidden, engine_key_state, engine_repage_steps, engine_token, randn  # noqa: E402,E501


def _bf16_bits(t):
    import torch

    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def _fetch_record(k, v):
    import torch

    rec = {"shape": list(k.shape), "dtype": str(k.dtype).replace("torch.", "")}
    rec["k_sha_f32"] = digest(k.to(torch.float32).numpy())
    rec["v_sha_f32"] = digest(v.to(torch.float32).numpy())
    rec["k_sha_bf16"] = digest(_bf16_bits(k))
    rec["v_sha_bf16"] = digest(_bf16_bits(v))
    return rec


def run_paged_scenario(cfg, ops):
    import torch
    from snapmind.kv_cache.paged import PagedKVCache

    cache = PagedKVCache(**cfg)
    H, D = cfg["n_heads"], cfg["head_dim"]
    records = []
    for op in ops:
        rec: dict = {}
        try:
            kind = op["op"]
            if kind == "store":
                k = torch.from_numpy(randn(op["seed"], (1, H, op["T"], D)))
                v = torch.from_numpy(randn(op["seed"] + 1000, (1, H, op["T"], D)))
                if op.get("dtype") == "bf16":
                    k, v = k.to(torch.bfloat16), v.to(torch.bfloat16)
                cache.store(op["layer"], k, v, op.get("seq_pos", 0))
            elif kind == "fetch":
                k, v = cache.fetch(op["layer"])
                rec["fetch"] = _fetch_record(k, v)
            elif kind == "evict":
                cache.evict(op["keep"])
            elif kind == "reset":
                cache.reset()
            elif kind == "memory_usage":
                rec["usage"] = cache.memory_usage()
            elif kind == "layer_dicts":
                d = cache.layer_dicts()
                rec["layers"] = {
                    str(i): (None if e["k"] is None else _fetch_record(e["k"], e["v"])) for i, e in d.items()
                }
            else:
                raise ValueError(kind)
            rec["error"] = None
        except Exception as e:  # the reference's own error behaviour is part of the fixture
            rec["error"] = [type(e).__name__, str(e)]
        rec["tables"] = [list(map(int, bt)) for bt in cache._block_tables]
        rec["slot_counts"] = list(map(int, cache._slot_counts))
        rec["free"] = sorted(map(int, cache._free_blocks))
        records.append({"op": op, "expect": rec})
    return records


PAGED_SCENARIOS = [
    {
        # the fixture of snapmind/tests/kv_cache/test_paged.py:5-9, scripted
        "name": "test_paged_fixture",
        "config": {"max_seq_len": 128, "n_layers": 2, "n_heads": 4, "head_dim": 64, "block_size": 16},
        "ops": [
            {"op": "fetch", "layer": 0},
            {"op": "store", "layer": 0, "T": 10, "seed": 1},
            {"op": "store", "layer": 1, "T": 7, "seed": 2},
            {"op": "fetch", "layer": 0},
            {"op": "fetch", "layer": 1},
            {"op": "store", "layer": 0, "T": 20, "seed": 3, "seq_pos": 10},
            {"op": "fetch", "layer": 0},
            {"op": "memory_usage"},
            {"op": "evict", "keep": 5},
            {"op": "fetch", "layer": 0},
            {"op": "fetch", "layer": 1},
            {"op": "store", "layer": 1, "T": 40, "seed": 4},
            {"op": "fetch", "layer": 1},
            {"op": "memory_usage"},
            # multi-block non-aligned compaction: the reference raises mid-way
            {"op": "evict", "keep": 20},
            {"op": "fetch", "layer": 1},
            # reuses a block that evict returned while layer 1 still lists it
            {"op": "store", "layer": 0, "T": 60, "seed": 5},
            {"op": "fetch", "layer": 0},
            {"op": "fetch", "layer": 1},
            {"op": "store", "layer": 0, "T": 100, "seed": 6},  # out of blocks
            {"op": "fetch", "layer": 0},
            {"op": "layer_dicts"},
            {"op": "evict", "keep": 16},  # block-aligned start
            {"op": "layer_dicts"},
            {"op": "evict", "keep": 0},
            {"op": "layer_dicts"},
            {"op": "memory_usage"},
            {"op": "reset"},
            {"op": "fetch", "layer": 1},
            {"op": "store", "layer": 1, "T": 33, "seed": 7},
            {"op": "fetch", "layer": 1},
            {"op": "evict", "keep": 3},
            {"op": "fetch", "layer": 1},
        ],
    },
    {
        # Llama-3-8B KV head shape, bf16 inputs into the fp32 reference pool
        "name": "llama3_kv_bf16_inputs",
        "config": {"max_seq_len": 512, "n_layers": 3, "n_heads": 8, "head_dim": 128, "block_size": 16},
        "ops": [
            {"op": "store", "layer": 0, "T": 37, "seed": 11, "dtype": "bf16"},
            {"op": "store", "layer": 1, "T": 16, "seed": 12, "dtype": "bf16"},
            {"op": "store", "layer": 2, "T": 1, "seed": 13, "dtype": "bf16"},
            {"op": "store", "layer": 0, "T": 1, "seed": 14, "dtype": "bf16"},
            {"op": "store", "layer": 1, "T": 1, "seed": 15, "dtype": "bf16"},
            {"op": "layer_dicts"},
            {"op": "store", "layer": 2, "T": 200, "seed": 16, "dtype": "bf16"},
            {"op": "evict", "keep": 9},
            {"op": "layer_dicts"},
            {"op": "memory_usage"},
        ],
    },
    {
        # block_size 8, odd head_dim, many small stores
        "name": "small_blocks",
        "config": {"max_seq_len": 64, "n_layers": 2, "n_heads": 2, "head_dim": 24, "block_size": 8,
                   "max_blocks": 6},
        "ops": [
            {"op": "store", "layer": 0, "T": 3, "seed": 21},
            {"op": "store", "layer": 0, "T": 3, "seed": 22},
            {"op": "store", "layer": 1, "T": 9, "seed": 23},
            {"op": "store", "layer": 0, "T": 3, "seed": 24},
            {"op": "layer_dicts"},
            {"op": "evict", "keep": 4},
            {"op": "layer_dicts"},
            {"op": "store", "layer": 1, "T": 30, "seed": 25},
            {"op": "layer_dicts"},
            {"op": "memory_usage"},
        ],
    },
]


def make_paged_ops(out: Path):
    data = []
    for sc in PAGED_SCENARIOS:
        data.append({"name": sc["name"], "config": sc["config"], "steps": run_paged_scenario(sc["config"], sc["ops"])})
    out.write_text(json.dumps(data, indent=1))


def make_paged_batched(out: Path):
    import torch
    from snapmind.kv_cache.paged import PagedKVCache

    L, H, D, bs = 2, 8, 128, 16
    lens = [0, 1, 16, 17, 33, 100, 32, 48]
    need_after = [(n + 1 + bs - 1) // bs for n in lens]
    pool = int(np.ceil(1.1 * sum(need_after)))
    perm = np.random.RandomState(99).permutation(pool).astype(np.int64)
    width = max(need_after) + 2
    tables = np.zeros((len(lens), width), dtype=np.int64)
    off = 0
    for b, n in enumerate(lens):
        nb = (n + bs - 1) // bs
        tables[b, :nb] = perm[off:off + nb]
        off += nb
    free_stack = perm[off:].copy()
    top = len(free_stack)
    # expected growth: ascending sequence order, from the top of the stack
    tables_after = tables.copy()
    taken = 0
    for b, n in enumerate(lens):
        have = (n + bs - 1) // bs
        for k in range(need_after[b] - have):
            tables_after[b, have + k] = free_stack[top - 1 - taken]
            taken += 1
    records = []
    for b, n in enumerate(lens):
        for layer in range(L):
            ref = PagedKVCache(max_seq_len=pool * bs, n_layers=1, n_heads=H, head_dim=D, block_size=bs,
                               max_blocks=pool)
            ref._block_tables[0] = [int(x) for x in tables_after[b, :need_after[b]]]
            ref._free_blocks = set()
            seed = 1000 + 10 * b + layer
            if n:
                kp = torch.from_numpy(randn(seed, (1, H, n, D))).to(torch.bfloat16)
                vp = torch.from_numpy(randn(seed + 500, (1, H, n, D))).to(torch.bfloat16)
                ref.store(0, kp, vp, 0)
            ka = torch.from_numpy(randn(seed + 2000, (1, H, 1, D))).to(torch.bfloat16)
            va = torch.from_numpy(randn(seed + 2500, (1, H, 1, D))).to(torch.bfloat16)
            ref.store(0, ka, va, n)
            k, v = ref.fetch(0)
            records.append({"seq": b, "layer": layer, "seed": seed, **_fetch_record(k, v)})
    data = {
        "config": {"n_layers": L, "n_heads": H, "head_dim": D, "block_size": bs, "num_blocks": pool},
        "lens": lens,
        "tables": tables.tolist(),
        "free_stack": free_stack.tolist(),
        "tables_after": tables_after.tolist(),
        "free_top_after": top - taken,
        "seeds": "prefill k=randn(seed,(1,H,n,D)) v=randn(seed+500); append k=randn(seed+2000,(1,H,1,D)) v=randn(seed+2500); all rounded to bf16",
        "fetch": records,
    }
    out.write_text(json.dumps(data, indent=1))


GQA_CASES = [
    # name, Hq, H, D, T_cached, dtype, seed
    ("tiny_test_shape", 4, 2, 8, 20, "f32", 31),
    ("tinyllama_kv", 32, 4, 64, 100, "f32", 32),
    ("llama3_kv_f32", 32, 8, 128, 300, "f32", 33),
    ("llama3_kv_bf16", 32, 8, 128, 300, "bf16", 34),
    ("mha_block_edge", 4, 4, 32, 16, "f32", 35),
]


def make_gqa(out_npz: Path, out_json: Path):
    import torch
    from snapmind.kv_cache.paged import PagedKVCache
    from snapmind.layers.attention.gqa import GroupedQueryAttention

    arrays = {}
    meta = []
    for name, hq, h, d, t, dt, seed in GQA_CASES:
        torch.manual_seed(seed)
        gqa = GroupedQueryAttention(d_model=hq * d, n_heads=hq, n_kv_heads=h, pe=None)
        with torch.no_grad():
            gqa.out_proj.weight.copy_(torch.eye(hq * d))
        cache = PagedKVCache(max_seq_len=t + 1, n_layers=1, n_heads=h, head_dim=d, block_size=16)
        kc = torch.from_numpy(randn(seed + 1, (1, h, t, d)))
        vc = torch.from_numpy(randn(seed + 2, (1, h, t, d)))
        x = torch.from_numpy(randn(seed + 3, (1, 1, hq * d)))
        if dt == "bf16":
            kc, vc, x = kc.to(torch.bfloat16), vc.to(torch.bfloat16), x.to(torch.bfloat16)
            gqa = gqa.to(torch.bfloat16)
        cache.store(0, kc, vc, 0)
        kv = cache.layer_dicts()[0]
        if dt == "bf16":
            kv = {"k": kv["k"].to(torch.bfloat16), "v": kv["v"].to(torch.bfloat16)}
        with torch.no_grad():
            q = gqa.q_proj(x).view(hq, d)
            k_new = gqa.k_proj(x).view(h, d)
            v_new = gqa.v_proj(x).view(h, d)
            out, _ = gqa(x, kv_cache=kv)
        out = out.view(hq, d)
        assert kv["k"].shape[-2] == t + 1
        enc = (lambda a: _bf16_bits(a)) if dt == "bf16" else (lambda a: a.float().numpy())
        for key, val in (("q", q), ("k_new", k_new), ("v_new", v_new), ("out", out)):
            arrays[f"{name}__{key}"] = enc(val)
        meta.append({"name": name, "n_q_heads": hq, "n_kv_heads": h, "head_dim": d, "cached_tokens": t,
                     "dtype": dt, "seed": seed, "scale": d ** -0.5,
                     "cached_k": "randn(seed+1,(1,H,T,D))", "cached_v": "randn(seed+2,(1,H,T,D))"})
    np.savez_compressed(out_npz, **arrays)
    out_json.write_text(json.dumps(meta, indent=1))


TIERED_SCENARIOS = [
    {
        "name": "decode_token_major_evicting",
        "config": {"max_seq_len": 512, "n_layers": 2, "n_heads": 2, "head_dim": 16, "pool_tokens": 24,
                   "chunk_size": 8},
        "ops": [
            {"op": "decode", "start": 0, "count": 45, "seed": 1},
            {"op": "layer_dicts"},
            {"op": "memory_usage"},
            {"op": "score_and_repage", "scores": {"0": 0.9, "1": 0.2, "2": 0.7, "3": 0.5, "4": 0.49}},
            {"op": "fetch", "layer": 0},
            {"op": "fetch", "layer": 1},
            {"op": "decode", "start": 45, "count": 20, "seed": 2},
            {"op": "fetch", "layer": 0},
            {"op": "layer_dicts"},
            {"op": "score_and_repage", "scores": {"1": 0.8, "5": 0.9, "6": 0.1}, "tensor": True, "threshold": 0.6},
            {"op": "memory_usage"},
            {"op": "evict", "keep": 10},
            {"op": "score_and_repage", "scores": {}},
            {"op": "reset"},
            {"op": "fetch", "layer": 0},
            {"op": "layer_dicts"},
            {"op": "decode", "start": 0, "count": 9, "seed": 3},
            {"op": "layer_dicts"},
        ],
    },
    {
        # layer-major prefill: one active chunk is shared by all layers (loses data)
        "name": "layer_major_prefill",
        "config": {"max_seq_len": 512, "n_layers": 3, "n_heads": 2, "head_dim": 8, "pool_tokens": 16,
                   "chunk_size": 8},
        "ops": [
            {"op": "store", "layer": 0, "T": 30, "pos": 0, "seed": 11},
            {"op": "store", "layer": 1, "T": 30, "pos": 0, "seed": 12},
            {"op": "store", "layer": 2, "T": 10, "pos": 0, "seed": 13},
            {"op": "layer_dicts"},
            {"op": "memory_usage"},
            {"op": "decode", "start": 30, "count": 5, "seed": 14},
            {"op": "layer_dicts"},
            {"op": "score_and_repage", "scores": {"1": 0.7, "2": 0.7}},
            {"op": "memory_usage"},
        ],
    },
    {
        # chunk-crossing multi-token stores, repeated positions, position jumps
        "name": "multi_token_duplicates_jumps",
        "config": {"max_seq_len": 512, "n_layers": 2, "n_heads": 2, "head_dim": 16, "pool_tokens": 32,
                   "chunk_size": 8},
        "ops": [
            {"op": "store", "layer": 0, "T": 13, "pos": 5, "seed": 21},
            {"op": "store", "layer": 1, "T": 13, "pos": 5, "seed": 22},
            {"op": "store", "layer": 0, "T": 1, "pos": 17, "seed": 23},
            {"op": "store", "layer": 1, "T": 3, "pos": 16, "seed": 24},
            {"op": "layer_dicts"},
            {"op": "store", "layer": 0, "T": 20, "pos": 100, "seed": 25},
            {"op": "layer_dicts"},
            {"op": "store", "layer": 0, "T": 8, "pos": 200, "seed": 26},
            {"op": "store", "layer": 0, "T": 8, "pos": 200, "seed": 27},
            {"op": "store", "layer": 1, "T": 1, "pos": 300, "seed": 28},
            {"op": "layer_dicts"},
            {"op": "memory_usage"},
            {"op": "score_and_repage", "scores": {"2": 0.6, "12": 0.9}},
            {"op": "fetch", "layer": 1},
        ],
    },
    {
        "name": "batch2_bf16",
        "config": {"max_seq_len": 512, "n_layers": 2, "n_heads": 2, "head_dim": 32, "pool_tokens": 48,
                   "chunk_size": 16},
        "ops": [
            {"op": "decode", "start": 0, "count": 70, "seed": 31, "batch": 2, "dtype": "bf16"},
            {"op": "layer_dicts"},
            {"op": "score_and_repage", "scores": {"0": 0.1, "1": 0.9, "2": 0.4}},
            {"op": "memory_usage"},
            {"op": "fetch", "layer": 1},
        ],
    },
    {
        "name": "reference_defaults",
        "config": {"max_seq_len": 4096, "n_layers": 2, "n_heads": 8, "head_dim": 64},
        "ops": [
            {"op": "decode", "start": 0, "count": 150, "seed": 41},
            {"op": "layer_dicts"},
            {"op": "score_and_repage", "scores": {"0": 0.1, "1": 0.1}},
            {"op": "memory_usage"},
        ],
    },
]


def tiered_inputs(op, n_layers, n_heads, head_dim):
    """The (layer, key, value, seq_pos) stores an op performs, as float32 numpy."""
    b = op.get("batch", 1)
    if op["op"] == "store":
        k = randn(op["seed"], (b, n_heads, op["T"], head_dim))
        v = randn(op["seed"] + 1000, (b, n_heads, op["T"], head_dim))
        return [(op["layer"], k, v, op["pos"])]
    out = []
    for t in range(op["count"]):
        for layer in range(n_layers):
            s = op["seed"] * 100000 + t * n_layers + layer
            out.append((layer, randn(s, (b, n_heads, 1, head_dim)), randn(s + 50000, (b, n_heads, 1, head_dim)),
                        op["start"] + t))
    return out


def _tiered_state(cache):
    import torch

    layout, chunk_bytes, data = {}, {}, {}
    for cid, layers in cache._chunks.items():
        layout[str(cid)] = [None if e["k"] is None else int(e["k"].shape[-2]) for e in layers]
        chunk_bytes[str(cid)] = sum(2 * e["k"].numel() * e["k"].element_size() for e in layers if e["k"] is not None)
        data[str(cid)] = [None if e["k"] is None else [digest(e["k"].to(torch.float32).numpy()),
                                                        digest(e["v"].to(torch.float32).numpy())] for e in layers]
    return {"hot": sorted(cache._hot_set), "chunks": sorted(cache._chunks), "layout": layout,
            "chunk_bytes": chunk_bytes, "chunk_data": data, "total_tokens": cache._total_tokens}


def _live_record(k, v):
    import torch

    if k is None:
        return None
    return {"shape": list(k.shape), "k": digest(k.to(torch.float32).numpy()), "v": digest(v.to(torch.float32).numpy())}


def make_tiered(out: Path):
    import torch
    from snapmind.kv_cache.tiered import TieredPagedKVCache

    data = []
    for sc in TIERED_SCENARIOS:
        cfg = sc["config"]
        cache = TieredPagedKVCache(**cfg, device="cpu")
        steps = []
        for op in sc["ops"]:
            rec: dict = {}
            kind = op["op"]
            if kind in ("store", "decode"):
                for layer, k, v, pos in tiered_inputs(op, cfg["n_layers"], cfg["n_heads"], cfg["head_dim"]):
                    kt, vt = torch.from_numpy(k), torch.from_numpy(v)
                    if op.get("dtype") == "bf16":
                        kt, vt = kt.to(torch.bfloat16), vt.to(torch.bfloat16)
                    cache.store(layer, kt, vt, pos)
            elif kind == "layer_dicts":
                d = cache.layer_dicts()
                rec["live"] = {str(i): _live_record(e["k"], e["v"]) for i, e in d.items()}
            elif kind == "fetch":
                k, v = cache.fetch(op["layer"])
                rec["fetch"] = None if k.numel() == 0 else _live_record(k, v)
            elif kind == "score_and_repage":
                scores = {int(c): (torch.tensor(s) if op.get("tensor") else s) for c, s in op["scores"].items()}
                cache.score_and_repage(scores, threshold=op.get("threshold", 0.5))
                if cache._live_dicts is not None:
                    rec["live"] = {str(i): _live_record(e["k"], e["v"]) for i, e in cache._live_dicts.items()}
            elif kind == "memory_usage":
                rec["usage_reported_cpu_device"] = cache.memory_usage()
            elif kind == "evict":
                cache.evict(op["keep"])
            elif kind == "reset":
                cache.reset()
            rec["state"] = _tiered_state(cache)
            steps.append({"op": op, "expect": rec})
        data.append({"name": sc["name"], "config": cfg, "steps": steps})
    out.write_text(json.dumps(data, indent=1))


MLA_CASES = [
    # name, d_model, heads, kv_lora_rank, nope, rope, v_head, dtype, seed, store_weights
    ("mla_tiny_f32", 16, 4, 8, 4, 4, 4, "f32", 51, True),
    ("mla_small_f32", 64, 4, 32, 16, 8, 16, "f32", 52, True),
    ("mla_deepseek_rank_bf16", 1024, 8, 512, 128, 64, 128, "bf16", 53, False),
]
MLA_STEPS = [(20, None), (1, 20), (1, 21), (3, None)]  # (new tokens, decode position or None)


def make_mla(out_npz: Path, out_json: Path):
    """Reference MLA forward with a dict kv_cache: per step the kv_proj rows it
    appended, the cache contents after the step, and (small shapes) the weights
    and outputs that pin the oracle's MLA attention math."""
    import torch
    from snapmind.layers.attention.mla import MultiHeadLatentAttention

    arrays, meta = {}, []
    for name, d_model, heads, rank, nope, rope, vdim, dt, seed, store_w in MLA_CASES:
        torch.manual_seed(seed)
        mla = MultiHeadLatentAttention(d_model=d_model, n_heads=heads, kv_lora_rank=rank, qk_nope_head_dim=nope,
                                       qk_rope_head_dim=rope, v_head_dim=vdim, max_seq_len=256)
        assert heads * vdim == d_model
        with torch.no_grad():
            mla.out_proj.weight.copy_(torch.eye(d_model))
        if dt == "bf16":
            mla = mla.to(torch.bfloat16)
        enc = (lambda a: _bf16_bits(a)) if dt == "bf16" else (lambda a: a.detach().float().numpy())
        if store_w:
            for wname in ("kv_proj", "k_up_proj", "v_up_proj", "q_proj"):
                arrays[f"{name}__w_{wname}"] = enc(getattr(mla, wname).weight)
        cache: dict = {}
        steps = []
        for si, (n_new, pos) in enumerate(MLA_STEPS):
            x = torch.from_numpy(randn(seed * 10 + si, (2, n_new, d_model)))
            if dt == "bf16":
                x = x.to(torch.bfloat16)
            with torch.no_grad():
                kv = mla.kv_proj(x)
                pid = None if pos is None else torch.tensor([pos])
                out, _ = mla(x, kv_cache=cache, position_ids=pid)
            arrays[f"{name}__s{si}_x"] = enc(x)
            arrays[f"{name}__s{si}_latent_new"] = enc(kv[..., :rank])
            arrays[f"{name}__s{si}_rope_new"] = enc(kv[..., rank:])
            arrays[f"{name}__s{si}_out"] = enc(out)
            steps.append({"n_new": n_new, "position": pos,
                          "k_shape": list(cache["k"].shape), "k_rope_shape": list(cache["k_rope"].shape),
                          "k_bits": digest(_bf16_bits(cache["k"])) if dt == "bf16" else digest(cache["k"].numpy()),
                          "k_rope_bits": digest(_bf16_bits(cache["k_rope"])) if dt == "bf16"
                          else digest(cache["k_rope"].numpy())})
        meta.append({"name": name, "d_model": d_model, "n_heads": heads, "kv_lora_rank": rank,
                     "qk_nope_head_dim": nope, "qk_rope_head_dim": rope, "v_head_dim": vdim, "dtype": dt,
                     "seed": seed, "rope_theta": 10000.0, "max_seq_len": 256, "weights_stored": store_w,
                     "steps": steps})
    np.savez_compressed(out_npz, **arrays)
    out_json.write_text(json.dumps(meta, indent=1))


INDEXER_CASES = [
    # name, d_model, kv_lora_rank, n_heads, n_chunks, chunk, dtype, seed, store_weights
    ("indexer_small_f32", 64, 32, 4, 12, 16, "f32", 61, True),
    ("indexer_default_f32", 2048, 512, 4, 40, 64, "f32", 62, False),
    ("indexer_default_bf16", 2048, 512, 4, 24, 64, "bf16", 63, False),
]


def make_indexer(out_npz: Path, out_json: Path):
    """Reference LookaheadSparseIndexer: frozen keys and scores.  Weights come from
    torch.manual_seed(seed) then the module constructor (stored for small cases)."""
    import torch
    from snapmind.layers.indexer.lookahead import LookaheadSparseIndexer

    arrays, meta = {}, []
    for name, d_model, rank, heads, n_chunks, chunk, dt, seed, store_w in INDEXER_CASES:
        torch.manual_seed(seed)
        idx = LookaheadSparseIndexer(d_model=d_model, n_layers=24, kv_lora_rank=rank, n_indexer_heads=heads)
        tdt = torch.bfloat16 if dt == "bf16" else torch.float32
        idx = idx.to(tdt)
        enc = (lambda a: _bf16_bits(a)) if dt == "bf16" else (lambda a: a.detach().float().numpy())
        if store_w:
            for wname in ("q_down_proj", "q_up_proj", "w_proj"):
                arrays[f"{name}__w_{wname}"] = enc(getattr(idx, wname).weight)
        # chunk keys: (chunk tokens, rank + 64) like MLA latent+rope rows; chunk 3 absent
        key_states = {}
        for c in range(n_chunks):
            if c == 3:
                continue
            t = chunk if c < n_chunks - 1 else chunk // 2 + 1  # a partial last chunk
            key_states[c] = torch.from_numpy(randn(seed * 1000 + c, (t, rank + 64))).to(tdt)
        hidden = {lid: torch.from_numpy(randn(seed * 1000 + 500 + lid, (1, d_model))).to(tdt) for lid in (10, 12, 20, 5)}
        with torch.no_grad():
            uninit = idx.score(hidden, [0, 1])
            idx.build_frozen_keys(key_states, list(range(n_chunks)))
            ids = list(range(n_chunks)) + [n_chunks + 5]
            scores = idx.score(hidden, ids)
            fallback = idx.score({5: hidden[5]}, ids)  # no indexer layer present: min layer used
        for c in sorted(idx._frozen_keys):
            arrays[f"{name}__frozen_{c}"] = enc(idx._frozen_keys[c])
        meta.append({
            "name": name, "d_model": d_model, "kv_lora_rank": rank, "n_indexer_heads": heads, "n_chunks": n_chunks,
            "chunk": chunk, "dtype": dt, "seed": seed, "weights_stored": store_w,
            "key_states": {str(c): list(v.shape) for c, v in key_states.items()},
            "uninitialized": {str(c): float(v) for c, v in uninit.items()},
            "scores": {str(c): float(v.float()) for c, v in scores.items()},
            "fallback_scores": {str(c): float(v.float()) for c, v in fallback.items()},
        })
    np.savez_compressed(out_npz, **arrays)
    out_json.write_text(json.dumps(meta, indent=1))


ENGINE_CASES = [
    # The reference engine's indexer cadence (snapmind/engine/generate.py:76-86, 112-114) over a
    # tiered cache: the prompt is stored token-major, _run_indexer runs once after the prompt and
    # then every `interval` decode steps.  "frozen": keys are frozen for every completed chunk
    # before each re-page (the reference engine itself never builds them, so its indexer stays
    # uninitialised and scores every chunk 0.5 -- the case without frozen keys).
    {"name": "engine_uninitialised", "seed": 81, "prompt": 300, "end": 900, "interval": 64, "frozen": False,
     "threshold": 0.5, "cache": {"max_seq_len": 2048, "n_layers": 2, "n_heads": 2, "head_dim": 16,
                                 "pool_tokens": 256, "chunk_size": 64},
     "indexer": {"d_model": 64, "kv_lora_rank": 32}},
    {"name": "engine_frozen_keys", "seed": 82, "prompt": 333, "end": 1300, "interval": 64, "frozen": True,
     "threshold": 0.5, "cache": {"max_seq_len": 2048, "n_layers": 2, "n_heads": 2, "head_dim": 16,
                                 "pool_tokens": 256, "chunk_size": 64},
     "indexer": {"d_model": 64, "kv_lora_rank": 32}},
    {"name": "engine_frozen_keys_wide_pool", "seed": 83, "prompt": 200, "end": 1100, "interval": 64,
     "frozen": True, "threshold": 0.6, "cache": {"max_seq_len": 2048, "n_layers": 3, "n_heads": 2,
                                                  "head_dim": 16, "pool_tokens": 512, "chunk_size": 64},
     "indexer": {"d_model": 96, "kv_lora_rank": 32}},
]


def make_engine_indexer(out: Path):
    """Drive the reference TieredPagedKVCache and LookaheadSparseIndexer through the
    reference engine's own _run_indexer (called on a stand-in holding the attributes
    it reads) and record the scores, hot set and live contents after every re-page."""
    from types import SimpleNamespace

    import torch
    from snapmind.core.config import IndexerConfig
    from snapmind.engine.generate import GenerateEngine
    from snapmind.kv_cache.tiered import TieredPagedKVCache
    from snapmind.layers.indexer.lookahead import LookaheadSparseIndexer

    data = []
    for case in ENGINE_CASES:
        cache = TieredPagedKVCache(**case["cache"], device="cpu")
        torch.manual_seed(case["seed"])
        idx = LookaheadSparseIndexer(d_model=case["indexer"]["d_model"], n_layers=24,
                                     kv_lora_rank=case["indexer"]["kv_lora_rank"])
        cfg = IndexerConfig(indexer_type="lookahead_sparse", indexer_interval=case["interval"],
                            score_threshold=case["threshold"], kv_lora_rank=case["indexer"]["kv_lora_rank"])
        engine = SimpleNamespace(_indexer=idx, _hook_states={}, _kvcache=cache, _indexer_config=cfg)
        cache.reset()  # GenerateEngine._make_kv_cache (snapmind/engine/generate.py:88-90)
        cache.layer_dicts()
        chunk = case["cache"]["chunk_size"]
        repage = set(engine_repage_steps(case))
        frozen_done = 0
        records, margin = [], float("inf")
        with torch.no_grad():
            for t in range(case["end"]):
                for layer in range(case["cache"]["n_layers"]):
                    k, v = engine_token(case, t, layer)
                    cache.store(layer, torch.from_numpy(k), torch.from_numpy(v), t)
                step = t + 1
                if step not in repage:
                    continue
                if case["frozen"]:
                    done = step // chunk
                    ks = {c: torch.from_numpy(engine_key_state(case, c)) for c in range(frozen_done, done)}
                    idx.build_frozen_keys(ks, list(range(frozen_done, done)))
                    frozen_done = done
                engine._hook_states = {lid: torch.from_numpy(h) for lid, h in engine_hidden(case, step).items()}
                # the reference engine's own indexer step (snapmind/engine/generate.py:76-86)
                n_ids = max(1, step // chunk)
                scores = idx.score(engine._hook_states, list(range(n_ids)))
                GenerateEngine._run_indexer(engine, step)
                margin = min([margin] + [abs(float(sc) - case["threshold"]) for sc in scores.values()
                                         if float(sc) != case["threshold"]])
                live = cache._live_dicts
                records.append({
                    "step": step,
                    "scores": {str(c): float(sc) for c, sc in scores.items()},
                    "hot": sorted(cache._hot_set),
                    "chunks": sorted(cache._chunks),
                    "total_tokens": cache._total_tokens,
                    "live": None if live is None else {str(i): _live_record(e["k"], e["v"]) for i, e in live.items()},
                })
        if case["frozen"]:
            assert margin > 1e-3, f"{case['name']}: a score within {margin} of the threshold; pick another seed"
        data.append({**case, "threshold_margin": margin, "records": records})
        print(f"engine {case['name']}: {len(records)} re-pages, hot after last {records[-1]['hot']}")
    out.write_text(json.dumps(data, indent=1))


SLIDING_OPS = [  # (op, layer, tokens or keep, seed)
    ("store", 0, 5, 401), ("store", 1, 3, 402), ("store", 0, 1, 403), ("store", 0, 9, 404),
    ("store", 1, 20, 405), ("store", 0, 1, 406), ("evict", None, 0, None), ("store", 1, 1, 407),
    ("evict", None, 6, None), ("store", 0, 2, 408), ("store", 0, 30, 409), ("store", 1, 12, 410),
    ("reset", None, None, None), ("store", 0, 4, 411),
]
SLIDING_CFG = {"n_layers": 2, "n_heads": 2, "head_dim": 8, "window_size": 12}


def sliding_inputs(op, cfg):
    _, layer, n, seed = op
    shape = (1, cfg["n_heads"], n, cfg["head_dim"])
    return randn(seed, shape), randn(seed + 1000, shape)


def make_sliding(out: Path):
    """The reference SlidingWindowKVCache driven by SLIDING_OPS: after each op,
    the shape and digest of every layer's fetched K and V and memory_usage()."""
    import torch
    from snapmind.kv_cache.sliding_window import SlidingWindowKVCache

    cfg = SLIDING_CFG
    cache = SlidingWindowKVCache(max_seq_len=64, n_layers=cfg["n_layers"], n_heads=cfg["n_heads"],
                                 head_dim=cfg["head_dim"], window_size=cfg["window_size"])
    steps = []
    for op in SLIDING_OPS:
        kind, layer, n, _ = op
        if kind == "store":
            k, v = sliding_inputs(op, cfg)
            cache.store(layer, torch.from_numpy(k), torch.from_numpy(v), 0)
        elif kind == "evict":
            cache.evict(n)
        else:
            cache.reset()
        rec = {"memory_usage": cache.memory_usage(), "layers": []}
        for i in range(cfg["n_layers"]):
            k, v = cache.fetch(i)
            rec["layers"].append({"shape": list(k.shape), "k": digest(k.numpy()), "v": digest(v.numpy())})
        steps.append(rec)
    out.write_text(json.dumps({"config": cfg, "steps": steps}, indent=1))


E2E_CASES = [
    # (name, shape name, weight seed, prompt seed, prompt length, generated ids, cache sample per layer)
    ("small", "SMALL", 7, 11, 24, 8, None),
    ("tinyllama", "TINYLLAMA", 0, 1, 256, 64, 512),
]


def make_e2e(out_npz: Path, out_json: Path, names=None):
    """The reference ``LlamaModel`` (snapmind/models/llama.py) generating greedily
    from a seeded prompt, with its cache dicts taken from ``PagedKVCache.layer_dicts()``
    as ``GenerateEngine._make_kv_cache`` does (snapmind/engine/generate.py:88-90):
    generated ids, each step's top-2 logits, per-parameter checksums of the
    seeded weights and the final cache (whole for the small case; per-layer sums
    and a seeded sample of entries for the TinyLlama case)."""
    import torch
    from llama_harness import SMALL, TINYLLAMA, init_weights, param_checksums, prompt_ids
    from snapmind.core.config import ModelConfig
    from snapmind.engine.prefill import prefill
    from snapmind.kv_cache.paged import PagedKVCache
    from snapmind.models.llama import LlamaModel
    from snapmind.sampling.greedy import GreedySampler

    shapes = {"SMALL": SMALL, "TINYLLAMA": TINYLLAMA}
    arrays, meta = {}, {}
    if out_json.exists():
        meta = json.loads(out_json.read_text())
        with np.load(out_npz) as z:
            arrays = dict(z)
    for name, shape_name, wseed, pseed, plen, n_gen, n_sample in E2E_CASES:
        if names and name not in names:
            continue
        sh = shapes[shape_name]
        cfg = ModelConfig(model_type="llama", d_model=sh.d_model, n_heads=sh.n_heads, n_kv_heads=sh.n_kv_heads,
                          n_layers=sh.n_layers, d_ff=sh.d_ff, vocab_size=sh.vocab_size,
                          max_seq_len=sh.max_seq_len, norm_eps=sh.norm_eps, rope_theta=sh.rope_theta)
        model = LlamaModel(cfg)
        init_weights(model, wseed)
        model.eval()
        hd = sh.d_model // sh.n_heads
        cache = PagedKVCache(max_seq_len=sh.max_seq_len, n_layers=sh.n_layers, n_heads=sh.n_kv_heads, head_dim=hd)
        cache.reset()
        kv = cache.layer_dicts()
        prompt = prompt_ids(sh.vocab_size, plen, pseed)
        sampler = GreedySampler()
        logits, _ = prefill(model, prompt[None], kv)
        logits = logits[0]
        ids, tops = [], []
        step = plen
        for i in range(n_gen):
            top = torch.topk(logits, 2)
            tops.append((top.values.tolist(), top.indices.tolist()))
            ids.append(int(sampler.sample(logits).item()))
            if i == n_gen - 1:
                break
            with torch.no_grad():  # the body of snapmind/engine/decode.py decode_step, keeping the logits
                logits = model(torch.tensor([[ids[-1]]]), kv_cache=kv, position_ids=torch.tensor([step]))[0, -1]
            step += 1
        ks = torch.stack([kv[i]["k"][0] for i in range(sh.n_layers)]).numpy()  # (L, H, T, D)
        vs = torch.stack([kv[i]["v"][0] for i in range(sh.n_layers)]).numpy()
        rec = {"shape": shape_name, "weight_seed": wseed, "prompt_seed": pseed, "prompt_len": plen,
               "n_generated": n_gen, "ids": ids, "top2": tops, "cache_shape": list(ks.shape),
               "params": param_checksums(model),
               "k_sums": ks.astype(np.float64).sum(axis=(1, 2, 3)).tolist(),
               "v_sums": vs.astype(np.float64).sum(axis=(1, 2, 3)).tolist()}
        if n_sample is None:
            arrays[f"{name}_k"], arrays[f"{name}_v"] = ks, vs
        else:
            rng = np.random.RandomState(wseed + 100)
            flat = rng.choice(ks[0].size, size=n_sample, replace=False)
            arrays[f"{name}_sample_idx"] = flat.astype(np.int64)
            arrays[f"{name}_k_sample"] = ks.reshape(sh.n_layers, -1)[:, flat]
            arrays[f"{name}_v_sample"] = vs.reshape(sh.n_layers, -1)[:, flat]
        meta[name] = rec
        print(f"e2e {name}: ids {ids[:8]}...")
    np.savez_compressed(out_npz, **arrays)
    out_json.write_text(json.dumps(meta, indent=1))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SNAPMIND_REFERENCE", "/root/reference"))
    ap.add_argument("--only", nargs="*", default=None,
                    help="fixtures to regenerate: paged, gqa, tiered, mla, indexer, engine, e2e, sliding "
                         "(default: all)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, str(HERE.parent))
    import torch

    torch.set_num_threads(4)
    want = set(args.only) if args.only else {"paged", "gqa", "tiered", "mla", "indexer", "engine", "e2e", "sliding"}
    if "paged" in want:
        make_paged_ops(HERE / "paged_ops.json")
        make_paged_batched(HERE / "paged_batched.json")
    if "gqa" in want:
        make_gqa(HERE / "gqa_decode.npz", HERE / "gqa_decode.json")
    if "tiered" in want:
        make_tiered(HERE / "tiered_ops.json")
    if "mla" in want:
        make_mla(HERE / "mla.npz", HERE / "mla.json")
    if "indexer" in want:
        make_indexer(HERE / "indexer.npz", HERE / "indexer.json")
    if "engine" in want:
        make_engine_indexer(HERE / "engine_indexer.json")
    if "e2e" in want:
        make_e2e(HERE / "e2e_llama.npz", HERE / "e2e_llama.json")
    if "sliding" in want:
        make_sliding(HERE / "sliding_window.json")
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
