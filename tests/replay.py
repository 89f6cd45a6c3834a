"""Replay the reference-generated paged-cache scripts (tests/golden/paged_ops.json)
against any object with the PagedKVCache API, and check every recorded fact."""
from __future__ import annotations

import json
from pathlib import Path

from inputs import digest, engine_hidden, engine_key_state, engine_token, randn

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


# ---------------------------------------------------------------------------
# tiered cache (tests/golden/tiered_ops.json)
# ---------------------------------------------------------------------------
def load_tiered_ops():
    return json.loads((GOLDEN / "tiered_ops.json").read_text())


def tiered_inputs(op, n_layers, n_heads, head_dim):
    """Same stores as tests/golden/make_golden.py::tiered_inputs."""
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


def replay_tiered(scenario, cache, to_input, to_numpy, make_score, state_of, entry_arrays):
    """Drive ``cache`` through the recorded ops and compare every recorded fact.

    to_input(array, dtype_tag) -> cache input; to_numpy(tensor) -> float32 array;
    make_score(float, as_tensor) -> score value; state_of(cache) -> (hot, chunks,
    layout, total_tokens); entry_arrays(cache, cid, layer) -> (k, v) float32 or None.
    """
    cfg = scenario["config"]
    for i, step in enumerate(scenario["steps"]):
        op, exp = step["op"], step["expect"]
        where = f"{scenario['name']} step {i} {op['op']}"
        kind = op["op"]
        got = {}
        if kind in ("store", "decode"):
            for layer, k, v, pos in tiered_inputs(op, cfg["n_layers"], cfg["n_heads"], cfg["head_dim"]):
                cache.store(layer, to_input(k, op.get("dtype")), to_input(v, op.get("dtype")), pos)
        elif kind == "layer_dicts":
            got["live"] = cache.layer_dicts()
        elif kind == "fetch":
            got["fetch"] = cache.fetch(op["layer"])
        elif kind == "score_and_repage":
            scores = {int(c): make_score(s, op.get("tensor", False)) for c, s in op["scores"].items()}
            cache.score_and_repage(scores, threshold=op.get("threshold", 0.5))
            got["live"] = getattr(cache, "_live_dicts", None) or getattr(cache, "live_dicts", None)
        elif kind == "memory_usage":
            got["usage"] = cache.memory_usage()
        elif kind == "evict":
            cache.evict(op["keep"])
        elif kind == "reset":
            cache.reset()
        st = exp["state"]
        hot, chunks, layout, total = state_of(cache)
        assert sorted(hot) == st["hot"], where
        assert sorted(chunks) == st["chunks"], where
        assert {str(c): n for c, n in layout.items()} == st["layout"], where
        assert total == st["total_tokens"], where
        for cid, per_layer in st["chunk_data"].items():
            for layer, rec in enumerate(per_layer):
                arr = entry_arrays(cache, int(cid), layer)
                if rec is None:
                    assert arr is None, f"{where}: chunk {cid} layer {layer}"
                else:
                    assert digest(arr[0]) == rec[0] and digest(arr[1]) == rec[1], f"{where}: chunk {cid} layer {layer}"
        if "live" in exp:
            for li, rec in exp["live"].items():
                d = got["live"][int(li)]
                _check_live(d["k"], d["v"], rec, to_numpy, f"{where} live {li}")
        if "fetch" in exp:
            k, v = got["fetch"]
            if exp["fetch"] is None:
                assert k.numel() == 0 if hasattr(k, "numel") else k.size == 0
            else:
                _check_live(k, v, exp["fetch"], to_numpy, f"{where} fetch")
        if "usage_reported_cpu_device" in exp:
            ref = exp["usage_reported_cpu_device"]
            gpu = sum(b for c, b in st["chunk_bytes"].items() if int(c) in st["hot"])
            cpu = sum(b for c, b in st["chunk_bytes"].items() if int(c) not in st["hot"])
            assert gpu + cpu == ref["cpu_bytes"] + ref["gpu_bytes"], where
            u = got["usage"]
            assert (u["gpu_bytes"], u["cpu_bytes"]) == (gpu, cpu), f"{where}: {u}"
            for key in ("hot_chunks", "cold_chunks", "total_tokens", "pool_slots"):
                assert u[key] == ref[key], f"{where}: {key}"


def _check_live(k, v, rec, to_numpy, where):
    if rec is None:
        assert k is None and v is None, where
        return
    assert k is not None, where
    assert list(k.shape) == rec["shape"], f"{where}: {tuple(k.shape)} vs {rec['shape']}"
    assert digest(to_numpy(k)) == rec["k"], f"{where}: K differs"
    assert digest(to_numpy(v)) == rec["v"], f"{where}: V differs"


# ---- the engine's indexer cadence over a tiered cache (engine_indexer.json)
def load_engine_indexer():
    return json.loads((GOLDEN / "engine_indexer.json").read_text())


def engine_run_indexer(score, hook_states, kvcache, step, threshold, chunk_size=64):
    """GenerateEngine._run_indexer (snapmind/engine/generate.py:76-86), restated:
    score chunks 0 .. max(1, step // chunk_size) - 1 from the hooked hidden states,
    then re-page the cache at the configured threshold."""
    if score is None or not hook_states:
        return None
    chunk_ids = list(range(max(1, step // chunk_size)))
    scores = score(hook_states, chunk_ids)
    if hasattr(kvcache, "score_and_repage"):
        kvcache.score_and_repage(scores, threshold=threshold)
    return scores


def replay_engine_indexer(case, cache, indexer, to_input, to_numpy, state_of, live_of, score_tol):
    """Drive ``cache`` and ``indexer`` the way the reference engine does (stores of every
    layer per token, frozen keys of completed chunks, the indexer step at the recorded
    steps) and check the scores, hot set, chunk ids, token count and live contents
    after every re-page against the reference's record."""
    chunk = case["cache"]["chunk_size"]
    recs = {r["step"]: r for r in case["records"]}
    cache.reset()
    cache.layer_dicts()
    frozen_done = 0
    for t in range(case["end"]):
        for layer in range(case["cache"]["n_layers"]):
            k, v = engine_token(case, t, layer)
            cache.store(layer, to_input(k), to_input(v), t)
        step = t + 1
        if step not in recs:
            continue
        rec = recs[step]
        where = f"{case['name']} step {step}"
        if case["frozen"]:
            done = step // chunk
            ids = list(range(frozen_done, done))
            indexer.build_frozen_keys({c: to_input(engine_key_state(case, c)) for c in ids}, ids)
            frozen_done = done
        hidden = {lid: to_input(h) for lid, h in engine_hidden(case, step).items()}
        scores = engine_run_indexer(indexer.score, hidden, cache, step, case["threshold"], chunk)
        assert sorted(scores) == sorted(int(c) for c in rec["scores"]), where
        for c, want in rec["scores"].items():
            got = float(scores[int(c)])
            assert abs(got - want) <= score_tol, f"{where}: chunk {c} score {got} vs {want}"
        hot, chunks, total = state_of(cache)
        assert sorted(hot) == rec["hot"], f"{where}: hot {sorted(hot)} vs {rec['hot']}"
        assert sorted(chunks) == rec["chunks"], where
        assert total == rec["total_tokens"], where
        live = live_of(cache)
        for i in range(case["cache"]["n_layers"]):
            e = live[i]
            _check_live(e["k"], e["v"], rec["live"][str(i)], to_numpy, f"{where} layer {i}")
    assert frozen_done > 0 or not case["frozen"]
