"""Replay the reference-generated paged-cache scripts (tests/golden/paged_ops.json)
against any object with the PagedKVCache API, and check every recorded fact."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from inputs import digest, randn

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_paged_ops():
    return json.loads((GOLDEN / "paged_ops.json").read_text())


def load_paged_batched():
    return json.loads((GOLDEN / "paged_batched.json").read_text())


def replay(scenario, make_cache, to_input, to_numpy, digest_key, check_free=True):
    """Run every step; ``to_input`` turns a float32 numpy array (+ dtype tag) into
    the cache's input type, ``to_numpy`` turns a fetched tensor into the array
    whose digest is compared under ``digest_key`` ("f32" or "bf16")."""
    cfg = scenario["config"]
    cache = make_cache(cfg)
    H, D = cfg["n_heads"], cfg["head_dim"]
    for i, step in enumerate(scenario["steps"]):
        op, exp = step["op"], step["expect"]
        where = f"{scenario['name']} step {i} {op}"
        err = None
        got = {}
        try:
            kind = op["op"]
            if kind == "store":
                k = to_input(randn(op["seed"], (1, H, op["T"], D)), op.get("dtype"))
                v = to_input(randn(op["seed"] + 1000, (1, H, op["T"], D)), op.get("dtype"))
                cache.store(op["layer"], k, v, op.get("seq_pos", 0))
            elif kind == "fetch":
                got["fetch"] = cache.fetch(op["layer"])
            elif kind == "evict":
                cache.evict(op["keep"])
            elif kind == "reset":
                cache.reset()
            elif kind == "memory_usage":
                got["usage"] = cache.memory_usage()
            elif kind == "layer_dicts":
                got["layers"] = cache.layer_dicts()
        except Exception as e:  # compared with the reference's recorded error
            err = [type(e).__name__, str(e)]
        if exp["error"] is None:
            assert err is None, f"{where}: unexpected error {err}"
        else:
            assert err is not None, f"{where}: expected {exp['error']}"
            assert err[0] == exp["error"][0], f"{where}: {err} vs {exp['error']}"
            if exp["error"][1].startswith("PagedKVCache"):
                assert err[1] == exp["error"][1]
        tables = cache.block_tables() if hasattr(cache, "block_tables") and callable(cache.block_tables) else cache.block_tables
        assert [list(t) for t in tables] == exp["tables"], where
        counts = cache._slot_counts if hasattr(cache, "_slot_counts") else cache.slot_counts
        assert list(counts) == exp["slot_counts"], where
        if check_free:
            free = cache._free_blocks if hasattr(cache, "_free_blocks") else cache.free_blocks
            assert sorted(free) == exp["free"], where
        if "fetch" in exp:
            _check_fetch(got["fetch"], exp["fetch"], to_numpy, digest_key, where)
        if "usage" in exp:
            usage = got["usage"]
            for key, val in exp["usage"].items():
                if key == "total_bytes" and digest_key == "bf16":
                    continue  # pool bytes depend on the pool dtype
                assert usage[key] == val, f"{where}: {key}"
        if "layers" in exp:
            for li, rec in exp["layers"].items():
                d = got["layers"][int(li)]
                if rec is None:
                    assert d["k"] is None and d["v"] is None, where
                else:
                    _check_fetch((d["k"], d["v"]), rec, to_numpy, digest_key, f"{where} layer {li}")


def _check_fetch(kv, rec, to_numpy, digest_key, where):
    k, v = kv
    assert list(k.shape) == rec["shape"], f"{where}: shape {tuple(k.shape)} vs {rec['shape']}"
    ka, va = to_numpy(k), to_numpy(v)
    assert digest(ka) == rec[f"k_sha_{digest_key}"], f"{where}: K bytes differ"
    assert digest(va) == rec[f"v_sha_{digest_key}"], f"{where}: V bytes differ"
