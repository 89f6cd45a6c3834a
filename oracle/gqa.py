"""Oracle: GQA attention math (snapmind/layers/attention/gqa.py:69-82) on numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Computed in float64 from the given (already rounded) inputs, so the oracle is
at least as accurate as the reference's own fp32/bf16 evaluation; parity
tolerances are the ones stated for the path (fp32: rtol 1e-5 with atol 1e-5 for
near-zero outputs of cancelling sums; bf16: rtol 2e-2, atol 2e-2).
"""
from __future__ import annotations

import numpy as np


def gqa_attention(q, k, v, scale, mask=None, dtype=np.float64):
    """softmax(q k^T * scale [+ mask]) v with k/v repeated per query group.

    q: (B, Hq, Tq, D); k, v: (B, H, T, D) -> (B, Hq, Tq, D) in ``dtype``
    (float64 for parity checks; float32 when timing the reference's fp32 path).
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    n_rep = q.shape[1] // k.shape[1]
    if n_rep > 1:  # repeat_interleave(n_rep, dim=1), gqa.py:69-71
        k = np.repeat(k, n_rep, axis=1)
        v = np.repeat(v, n_rep, axis=1)
    attn = np.matmul(q, np.swapaxes(k, -2, -1)) * scale  # gqa.py:73-74
    if mask is not None:
        attn = attn + mask
    if attn.shape[-1] == 0:
        return np.zeros(q.shape[:-1] + (v.shape[-1],))
    attn = attn - attn.max(axis=-1, keepdims=True)  # softmax, gqa.py:79
    w = np.exp(attn)
    w = w / w.sum(axis=-1, keepdims=True)
    return np.matmul(w, v)  # gqa.py:82


def paged_gqa_decode(q, k_pool, v_pool, tables, lens, scale, block_size):
    """Decode attention of q (B, Hq, D) over each sequence's lens[b] paged tokens.

    k_pool, v_pool: one layer, [num_blocks][H][bs][D].  Returns (B, Hq, D) float64:
    the GQA math applied to what PagedKVCache.fetch returns for each sequence.
    """
    batch, n_q, d = q.shape
    out = np.zeros((batch, n_q, d))
    for b in range(batch):
        n = int(lens[b])
        nb = (n + block_size - 1) // block_size
        blocks = [int(x) for x in tables[b][:nb]]
        if n == 0:
            continue
        kc = np.concatenate([k_pool[p] for p in blocks], axis=1)[:, :n]  # (H, n, D)
        vc = np.concatenate([v_pool[p] for p in blocks], axis=1)[:, :n]
        out[b] = gqa_attention(q[b][None, :, None, :], kc[None], vc[None], scale)[0, :, 0, :]
    return out
