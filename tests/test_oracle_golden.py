"""The oracle against golden vectors produced by running the reference itself."""
import json

import numpy as np
import pytest

from inputs import digest, randn
from oracle import bf16, gqa, paged
from replay import GOLDEN, load_paged_batched, load_paged_ops, replay


def _np_input(a, dtype):
    return bf16.round_to_bf16(a) if dtype == "bf16" else a


@pytest.mark.parametrize("scenario", load_paged_ops(), ids=lambda s: s["name"])
def test_oracle_replays_reference_paged_ops(scenario):
    replay(
        scenario,
        make_cache=lambda cfg: paged.PagedKVCacheOracle(**cfg),
        to_input=_np_input,
        to_numpy=lambda a: np.ascontiguousarray(a, dtype=np.float32),
        digest_key="f32",
    )


@pytest.mark.parametrize("scenario", load_paged_ops(), ids=lambda s: s["name"])
def test_oracle_replays_reference_paged_ops_bf16_digest(scenario):
    replay(
        scenario,
        make_cache=lambda cfg: paged.PagedKVCacheOracle(**cfg),
        to_input=_np_input,
        to_numpy=lambda a: bf16.f32_to_bf16(np.asarray(a, dtype=np.float32)),
        digest_key="bf16",
    )


def batched_oracle_run(g):
    cfg = g["config"]
    L, H, D, bs, nb = cfg["n_layers"], cfg["n_heads"], cfg["head_dim"], cfg["block_size"], cfg["num_blocks"]
    lens = np.array(g["lens"])
    tables = np.array(g["tables"])
    k_pool = np.zeros((L, nb, H, bs, D), np.float32)
    v_pool = np.zeros_like(k_pool)
    recs = {(r["seq"], r["layer"]): r for r in g["fetch"]}
    # prefill each sequence with its own tokens
    for b, n in enumerate(lens):
        if n == 0:
            continue
        kn = np.stack([bf16.round_to_bf16(randn(recs[(b, l)]["seed"], (1, H, n, D)))[0] for l in range(L)])
        vn = np.stack([bf16.round_to_bf16(randn(recs[(b, l)]["seed"] + 500, (1, H, n, D)))[0] for l in range(L)])
        paged.append(k_pool, v_pool, tables[b:b + 1], [0], kn[:, None], vn[:, None], bs)
    free = np.array(g["free_stack"])
    tables2, lens2, top2, err = paged.reserve(tables, lens, free, len(free), 1, bs)
    assert err is None
    ka = np.stack([np.stack([bf16.round_to_bf16(randn(recs[(b, l)]["seed"] + 2000, (H, 1, D))) for b in range(len(lens))]) for l in range(L)])
    va = np.stack([np.stack([bf16.round_to_bf16(randn(recs[(b, l)]["seed"] + 2500, (H, 1, D))) for b in range(len(lens))]) for l in range(L)])
    paged.append(k_pool, v_pool, tables2, lens2 - 1, ka, va, bs)
    kg, vg = paged.gather(k_pool, v_pool, tables2, lens2, bs)
    return tables2, lens2, top2, kg, vg


def test_oracle_batched_matches_reference_fetch():
    g = load_paged_batched()
    H, D = g["config"]["n_heads"], g["config"]["head_dim"]
    tables2, lens2, top2, kg, vg = batched_oracle_run(g)
    assert tables2.tolist() == g["tables_after"]
    assert top2 == g["free_top_after"]
    offs = np.concatenate([[0], np.cumsum(lens2)]) * H * D
    for r in g["fetch"]:
        b, l = r["seq"], r["layer"]
        k = kg[l, offs[b]:offs[b + 1]].reshape(1, H, lens2[b], D)
        v = vg[l, offs[b]:offs[b + 1]].reshape(1, H, lens2[b], D)
        assert digest(k) == r["k_sha_f32"]
        assert digest(v) == r["v_sha_f32"]
        assert digest(bf16.f32_to_bf16(k)) == r["k_sha_bf16"]


def load_gqa():
    meta = json.loads((GOLDEN / "gqa_decode.json").read_text())
    arrays = np.load(GOLDEN / "gqa_decode.npz")
    return meta, arrays


def gqa_case_inputs(m, arrays):
    """(q (Hq,D), K (H,T+1,D), V, expected out (Hq,D)) as float32, bf16 values exact."""
    name, h, d, t = m["name"], m["n_kv_heads"], m["head_dim"], m["cached_tokens"]
    dec = (lambda a: bf16.bf16_to_f32(a)) if m["dtype"] == "bf16" else (lambda a: a.astype(np.float32))
    q, kn, vn, out = (dec(arrays[f"{name}__{k}"]) for k in ("q", "k_new", "v_new", "out"))
    kc = randn(m["seed"] + 1, (1, h, t, d))[0]
    vc = randn(m["seed"] + 2, (1, h, t, d))[0]
    if m["dtype"] == "bf16":
        kc, vc = bf16.round_to_bf16(kc), bf16.round_to_bf16(vc)
    k = np.concatenate([kc, kn[:, None, :]], axis=1)
    v = np.concatenate([vc, vn[:, None, :]], axis=1)
    return q, k, v, out


def tolerance(dtype):
    return (1e-5, 1e-5) if dtype == "f32" else (2e-2, 2e-2)


@pytest.mark.parametrize("case", json.loads((GOLDEN / "gqa_decode.json").read_text()), ids=lambda m: m["name"])
def test_oracle_gqa_matches_reference_forward(case):
    meta, arrays = load_gqa()
    q, k, v, out = gqa_case_inputs(case, arrays)
    got = gqa.gqa_attention(q[None, :, None, :], k[None], v[None], case["scale"])[0, :, 0, :]
    rtol, atol = tolerance(case["dtype"])
    np.testing.assert_allclose(got, out, rtol=rtol, atol=atol)


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf, 1e-40], np.float32)
    import torch

    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert (bf16.f32_to_bf16(x) == want).all()


# ---------------------------------------------------------------------------
# tiered cache oracle against the reference's recorded behaviour
# ---------------------------------------------------------------------------
from oracle import tiered as otiered  # noqa: E402
from replay import load_tiered_ops, replay_tiered  # noqa: E402


@pytest.mark.parametrize("scenario", load_tiered_ops(), ids=lambda s: s["name"])
def test_tiered_oracle_replays_reference(scenario):
    cfg = scenario["config"]
    cache = otiered.TieredPagedKVCacheOracle(**cfg)
    bf16_ops = any(st["op"].get("dtype") == "bf16" for st in scenario["steps"])
    elem = 2 if bf16_ops else 4
    cache_usage = cache.memory_usage
    cache.memory_usage = lambda: cache_usage(elem_size=elem)

    def entry_arrays(c, cid, layer):
        e = c.chunks[cid][layer]
        return None if e["k"] is None else (np.asarray(e["k"], np.float32), np.asarray(e["v"], np.float32))

    replay_tiered(
        scenario,
        cache,
        to_input=lambda a, tag: bf16.round_to_bf16(a) if tag == "bf16" else a,
        to_numpy=lambda a: np.asarray(a, np.float32),
        make_score=lambda s, as_tensor: s,
        state_of=lambda c: (c.hot_set, c.chunks.keys(), c.chunk_layout(), c.total_tokens),
        entry_arrays=entry_arrays,
    )


# ---------------------------------------------------------------------------
# MLA: oracle attention math and latent cache semantics against the reference
# ---------------------------------------------------------------------------
from oracle import mla as omla  # noqa: E402


def load_mla():
    return json.loads((GOLDEN / "mla.json").read_text()), np.load(GOLDEN / "mla.npz")


def mla_array(arrays, m, key):
    a = arrays[f"{m['name']}__{key}"]
    return bf16.bf16_to_f32(a) if m["dtype"] == "bf16" else a.astype(np.float32)


@pytest.mark.parametrize("case", json.loads((GOLDEN / "mla.json").read_text()), ids=lambda m: m["name"])
def test_mla_cache_is_concatenation_of_appended_rows(case):
    meta, arrays = load_mla()
    lat, rope = [], []
    for si, st in enumerate(case["steps"]):
        lat.append(mla_array(arrays, case, f"s{si}_latent_new"))
        rope.append(mla_array(arrays, case, f"s{si}_rope_new"))
        k = np.concatenate(lat, axis=1)
        kr = np.concatenate(rope, axis=1)
        assert list(k.shape) == st["k_shape"] and list(kr.shape) == st["k_rope_shape"]
        if case["dtype"] == "bf16":
            assert digest(bf16.f32_to_bf16(k)) == st["k_bits"]
            assert digest(bf16.f32_to_bf16(kr)) == st["k_rope_bits"]
        else:
            assert digest(k) == st["k_bits"] and digest(kr) == st["k_rope_bits"]


@pytest.mark.parametrize("case", [m for m in json.loads((GOLDEN / "mla.json").read_text()) if m["weights_stored"]],
                         ids=lambda m: m["name"])
def test_oracle_mla_forward_matches_reference(case):
    meta, arrays = load_mla()
    w = {k: mla_array(arrays, case, f"w_{k}") for k in ("kv_proj", "k_up_proj", "v_up_proj", "q_proj")}
    w["out_proj"] = np.eye(case["d_model"])
    cache: dict = {}
    for si, st in enumerate(case["steps"]):
        x = mla_array(arrays, case, f"s{si}_x")
        pid = None if st["position"] is None else [st["position"]]
        out = omla.mla_forward(x, w, case, cache, pid)
        np.testing.assert_allclose(out, mla_array(arrays, case, f"s{si}_out"), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", [m for m in json.loads((GOLDEN / "mla.json").read_text()) if m["weights_stored"]],
                         ids=lambda m: m["name"])
def test_absorbed_unrotated_decode_equals_reference_decode_math(case):
    """The B200 decode form (absorbed q, raw rope) equals the reference decode math."""
    meta, arrays = load_mla()
    H, R, dn, dr, dv = (case[k] for k in ("n_heads", "kv_lora_rank", "qk_nope_head_dim", "qk_rope_head_dim", "v_head_dim"))
    w = {k: mla_array(arrays, case, f"w_{k}").astype(np.float64) for k in ("kv_proj", "k_up_proj", "v_up_proj", "q_proj")}
    w["out_proj"] = np.eye(case["d_model"])
    cache: dict = {}
    for si, st in enumerate(case["steps"]):
        x = mla_array(arrays, case, f"s{si}_x").astype(np.float64)
        pid = None if st["position"] is None else [st["position"]]
        ref = omla.mla_forward(x, w, case, cache, pid)
        if pid is None:
            continue
        q = x @ w["q_proj"].T  # (B, 1, H*(dn+dr))
        qn = q[:, 0, : H * dn].reshape(-1, H, dn)
        qp = q[:, 0, H * dn:].reshape(-1, H, dr)
        q_lat = omla.absorb_query(qn, w["k_up_proj"], H, dn)
        T = cache["k"].shape[1]
        for b in range(x.shape[0]):
            o_lat = omla.sparse_mla_decode(q_lat[b], qp[b], cache["k"][b], cache["k_rope"][b], np.arange(T),
                                           (dn + dr) ** -0.5)
            out = np.einsum("hr,hvr->hv", o_lat, w["v_up_proj"].reshape(H, dv, R)).reshape(-1)
            # equal up to the float32 rounding of the rotation tables
            np.testing.assert_allclose(out, ref[b, 0], rtol=1e-6, atol=1e-9)


# ---------------------------------------------------------------------------
# indexer oracle against the reference LookaheadSparseIndexer
# ---------------------------------------------------------------------------
from oracle import indexer as oidx  # noqa: E402


def load_indexer():
    return json.loads((GOLDEN / "indexer.json").read_text()), np.load(GOLDEN / "indexer.npz")


def indexer_key_states(m):
    """The chunk key states of tests/golden/make_golden.py::make_indexer (float32, bf16-rounded if bf16)."""
    ks = {}
    for c, shape in m["key_states"].items():
        a = randn(m["seed"] * 1000 + int(c), tuple(shape))
        ks[int(c)] = bf16.round_to_bf16(a) if m["dtype"] == "bf16" else a
    hidden = {lid: randn(m["seed"] * 1000 + 500 + lid, (1, m["d_model"])) for lid in (10, 12, 20, 5)}
    if m["dtype"] == "bf16":
        hidden = {k: bf16.round_to_bf16(v) for k, v in hidden.items()}
    return ks, hidden


@pytest.mark.parametrize("case", json.loads((GOLDEN / "indexer.json").read_text()), ids=lambda m: m["name"])
def test_oracle_frozen_keys_match_reference(case):
    meta, arrays = load_indexer()
    ks, _ = indexer_key_states(case)
    tol = 1e-6 if case["dtype"] == "f32" else 8e-3
    for c, k in ks.items():
        ref = arrays[f"{case['name']}__frozen_{c}"]
        ref = bf16.bf16_to_f32(ref) if case["dtype"] == "bf16" else ref
        np.testing.assert_allclose(oidx.frozen_key(k, case["kv_lora_rank"]), ref, rtol=tol, atol=tol)


@pytest.mark.parametrize("case", [m for m in json.loads((GOLDEN / "indexer.json").read_text()) if m["weights_stored"]],
                         ids=lambda m: m["name"])
def test_oracle_scores_match_reference(case):
    meta, arrays = load_indexer()
    ks, hidden = indexer_key_states(case)
    w = {k: arrays[f"{case['name']}__w_{k}"].astype(np.float64) for k in ("q_down_proj", "q_up_proj", "w_proj")}
    frozen = {c: oidx.frozen_key(k, case["kv_lora_rank"]) for c, k in ks.items()}
    ids = [int(c) for c in case["scores"]]
    assert oidx.score(hidden, [0, 1], frozen, w, initialized=False) == {0: 0.5, 1: 0.5}
    got = oidx.score(hidden, ids, frozen, w)
    for c in ids:
        assert got[c] == pytest.approx(case["scores"][str(c)], abs=1e-6)
    fb = oidx.score({5: hidden[5]}, ids, frozen, w)
    for c in ids:
        assert fb[c] == pytest.approx(case["fallback_scores"][str(c)], abs=1e-6)


def test_stable_topk_breaks_ties_by_lower_chunk_id():
    s = np.array([0.5, 0.7, 0.7, 0.1, 0.7, 0.5])
    assert oidx.stable_topk(s, 4).tolist() == [1, 2, 4, 0]
    assert oidx.stable_topk(s[:2], 4).tolist() == [1, 0, -1, -1]
