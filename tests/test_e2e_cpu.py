"""The end-to-end harness pinned to the reference on the CPU: the small Llama
shape with the reference attention math must reproduce the reference run
(weights, generated ids, logits, final cache) recorded in tests/golden/e2e_llama.*."""
import json
from pathlib import Path

import numpy as np
import torch

from llama_harness import SMALL, LlamaHarness, generate, init_weights, param_checksums, prompt_ids

GOLDEN = Path(__file__).resolve().parent / "golden"


def _golden():
    meta = json.loads((GOLDEN / "e2e_llama.json").read_text())
    return meta, np.load(GOLDEN / "e2e_llama.npz")


def test_harness_weights_match_reference_recipe():
    meta, _ = _golden()
    rec = meta["small"]
    model = LlamaHarness(SMALL)
    init_weights(model, rec["weight_seed"])
    got = param_checksums(model)
    assert [(n, s) for n, s, _ in got] == [(n, s) for n, s, _ in rec["params"]]
    for (n, _, a), (_, _, b) in zip(got, rec["params"]):
        assert a == b, n


def test_harness_reproduces_reference_generation_on_cpu():
    meta, z = _golden()
    rec = meta["small"]
    torch.manual_seed(0)
    model = LlamaHarness(SMALL)
    init_weights(model, rec["weight_seed"])
    kv = {i: {"k": None, "v": None} for i in range(SMALL.n_layers)}
    ids, tops = generate(model, prompt_ids(SMALL.vocab_size, rec["prompt_len"], rec["prompt_seed"]),
                         rec["n_generated"], kv)
    assert ids == rec["ids"]
    for (vals, idx), (gv, gi) in zip(tops, rec["top2"]):
        assert idx == gi
        np.testing.assert_allclose(vals, gv, rtol=1e-5, atol=1e-6)
    k = torch.stack([kv[i]["k"][0] for i in range(SMALL.n_layers)]).numpy()
    v = torch.stack([kv[i]["v"][0] for i in range(SMALL.n_layers)]).numpy()
    np.testing.assert_allclose(k, z["small_k"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(v, z["small_v"], rtol=1e-5, atol=1e-6)
