"""Oracle: lookahead sparse indexer (snapmind/layers/indexer/lookahead.py) on numpy,
plus the sigmoid-gated score and stable top-k of the B200 chunk selector.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
"""
from __future__ import annotations

import numpy as np


def frozen_key(k, rank):
    """build_frozen_keys for one chunk (lookahead.py:40-50): mean over tokens of the
    first ``rank`` columns, keepdim."""
    return np.asarray(k, np.float64)[..., :rank].mean(axis=-2, keepdims=True)


def score_single(h, frozen, w):
    """_score_single (lookahead.py:82-106) with weights q_down (R x d), q_up (nR x R), w_proj (n x d)."""
    h = np.asarray(h, np.float64)
    batch_h = h[None] if h.ndim == 1 else h
    q_up = (batch_h @ w["q_down_proj"].T) @ w["q_up_proj"].T
    n_heads = w["w_proj"].shape[0]
    q_heads = q_up.reshape(-1, n_heads, frozen.shape[-1])
    wts = (batch_h @ w["w_proj"].T).reshape(-1, n_heads)
    fused = np.zeros((q_heads.shape[0], 1))
    for hi in range(n_heads):
        raw = q_heads[:, hi, :] @ frozen.reshape(-1, frozen.shape[-1]).T
        fused = fused + np.maximum(raw, 0.0) * wts[:, hi:hi + 1]
    return float((1.0 / (1.0 + np.exp(-fused))).mean())


def score(hidden_states, chunk_ids, frozen_keys, w, indexer_layers=(10, 12, 20), initialized=True):
    """LookaheadSparseIndexer.score (lookahead.py:52-80)."""
    if not initialized or not chunk_ids:
        return {cid: 0.5 for cid in chunk_ids}
    avail = [lid for lid in indexer_layers if lid in hidden_states]
    if not avail:
        h = np.asarray(hidden_states[min(hidden_states)], np.float64)
        h = h[0] if h.shape[0] == 1 else h
    else:
        hs = [np.asarray(hidden_states[lid], np.float64) for lid in avail]
        hs = [x[0] if x.shape[0] == 1 else x for x in hs]
        h = np.stack(hs).mean(axis=0)
    return {cid: (score_single(h, frozen_keys[cid], w) if cid in frozen_keys else 0.0) for cid in chunk_ids}


def sigmoid_scores(q, keys, scale, bias):
    """sigmoid(q . k * scale + bias) for keys (C, D)."""
    return 1.0 / (1.0 + np.exp(-(np.asarray(keys, np.float64) @ np.asarray(q, np.float64) * scale + bias)))


def stable_topk(scores, k):
    """Indices of the k largest scores, ties broken by the lower index (stable descending sort)."""
    order = np.argsort(-np.asarray(scores, np.float64), kind="stable")
    out = np.full(k, -1, np.int64)
    out[: min(k, len(order))] = order[:k]
    return out
