"""Seeded inputs shared by the golden generator and the tests.

``randn`` uses numpy's legacy ``RandomState`` stream, whose output is frozen
across numpy versions, so fixtures can store seeds instead of tensors.
"""
from __future__ import annotations

import hashlib

import numpy as np


def randn(seed: int, shape) -> np.ndarray:
    return np.random.RandomState(seed).standard_normal(shape).astype(np.float32)


def digest(a: np.ndarray) -> str:
    """sha256 of the array's bytes in C order (dtype and shape are checked separately)."""
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---- the engine indexer cadence (engine_indexer.json)
def engine_token(case, t, layer):
    """K and V of token t of one layer, [1, H, 1, D] float32."""
    c = case["cache"]
    s = case["seed"] * 100000 + t * c["n_layers"] + layer
    shape = (1, c["n_heads"], 1, c["head_dim"])
    return randn(s, shape), randn(s + 5000000, shape)


def engine_key_state(case, cid):
    """Latent rows of chunk cid as an MLA layer would freeze them: [chunk, rank + 64]."""
    shape = (case["cache"]["chunk_size"], case["indexer"]["kv_lora_rank"] + 64)
    return randn(case["seed"] * 7919 + cid, shape) * np.float32(4.0)


def engine_hidden(case, step):
    """The engine's hooked hidden states (output[0, -1, :]) at a re-page step, scaled so
    that the scores spread well away from the threshold (a random-init indexer fed unit
    inputs scores every chunk within a few 1e-3 of 0.5)."""
    d = case["indexer"]["d_model"]
    return {lid: randn(case["seed"] * 31337 + step * 7 + lid, (d,)) * np.float32(16.0) for lid in (10, 12, 20)}


def engine_repage_steps(case):
    """The steps at which the engine runs its indexer: once after the prompt, then
    every `interval` decode steps (snapmind/engine/generate.py:107-114)."""
    steps = [case["prompt"]]
    steps += [t for t in range(case["prompt"] + 1, case["end"] + 1) if t % case["interval"] == 0]
    return steps
