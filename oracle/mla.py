"""Oracle: MLA attention (snapmind/layers/attention/mla.py) and its latent-absorbed
sparse decode form, on numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

``mla_forward`` restates MultiHeadLatentAttention.forward (mla.py:186-245,
without dropout and with out_proj applied as given): projections, the dict
cache concatenation, per-head up-projection of every cached latent, RoPE on q
and on the cached raw rope keys (mla.py:151-176), softmax attention.

``sparse_mla_decode`` is the form the B200 kernel computes for one decode
token over a set of cached positions: with the query's no-rope part absorbed
through the key up-projection (q_lat[h] = W_uk[h]^T q_nope[h]), the score of
position t is scale * (q_lat[h] . c_t + q_pe[h] . k_pe_t) and the output is the
latent average sum_t p_t c_t (the value up-projection is applied afterwards).
In the reference decode path every cached rope key is rotated by the query's
own position (mla.py:170-176 with a length-1 position_ids), and a common
rotation leaves the dot product unchanged, so q_pe is the raw q_rope there.
"""
from __future__ import annotations

import numpy as np


def rope_tables(dim, max_seq_len, theta):
    """cos/sin tables of mla.py:151-161, computed in float32 like the reference."""
    freqs = (1.0 / (np.float32(theta) ** (np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim)))).astype(np.float32)
    positions = np.arange(max_seq_len, dtype=np.float32)
    angles = np.outer(positions, freqs).astype(np.float32)
    cos, sin = np.cos(angles), np.sin(angles)
    return np.concatenate([cos, cos], -1), np.concatenate([sin, sin], -1)


def rotate_half(x):
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], -1)


def apply_rope(t, cos_tab, sin_tab, position_ids=None):  # mla.py:163-176
    if position_ids is None:
        cos, sin = cos_tab[: t.shape[-2]], sin_tab[: t.shape[-2]]
        while cos.ndim < t.ndim:
            cos, sin = cos[None], sin[None]
    else:
        cos, sin = cos_tab[np.asarray(position_ids)], sin_tab[np.asarray(position_ids)]
        if cos.ndim == 3 and t.ndim == 4:
            cos, sin = cos[:, :, None], sin[:, :, None]
    return t * cos + rotate_half(t) * sin


def softmax(a):
    a = a - a.max(-1, keepdims=True)
    e = np.exp(a)
    return e / e.sum(-1, keepdims=True)


def mla_forward(x, w, cfg, cache, position_ids=None):
    """One MLA forward (q_lora_rank None).  ``w`` holds kv_proj/k_up_proj/v_up_proj/
    q_proj/out_proj weights (out_features x in_features); ``cache`` is a dict that
    is grown like the reference's.  Returns (B, Tq, d_model) in float64."""
    x = np.asarray(x, np.float64)
    H, R, dn, dr, dv = cfg["n_heads"], cfg["kv_lora_rank"], cfg["qk_nope_head_dim"], cfg["qk_rope_head_dim"], cfg["v_head_dim"]
    B, Tq, _ = x.shape
    q = x @ w["q_proj"].T
    q_nope, q_rope_raw = q[..., : H * dn], q[..., H * dn:]
    kv = x @ w["kv_proj"].T
    k_latent, k_rope_raw = kv[..., :R], kv[..., R:]
    if cache.get("k") is not None:  # mla.py:208-215
        k_latent = np.concatenate([cache["k"], k_latent], -2)
        k_rope_raw = np.concatenate([cache["k_rope"], k_rope_raw], -2)
    cache["k"], cache["k_rope"] = k_latent, k_rope_raw
    T = k_latent.shape[-2]
    k_nope = (k_latent @ w["k_up_proj"].T).reshape(B, T, H, dn).transpose(0, 2, 1, 3)
    v = (k_latent @ w["v_up_proj"].T).reshape(B, T, H, dv).transpose(0, 2, 1, 3)
    qn = q_nope.reshape(B, Tq, H, dn).transpose(0, 2, 1, 3)
    qr = q_rope_raw.reshape(B, Tq, H, dr).transpose(0, 2, 1, 3)
    cos, sin = rope_tables(dr, cfg["max_seq_len"], cfg["rope_theta"])
    qr = apply_rope(qr, cos, sin, position_ids)
    kr = apply_rope(k_rope_raw, cos, sin, position_ids)[:, None].repeat(H, axis=1)
    qf = np.concatenate([qn, qr], -1)
    kf = np.concatenate([k_nope, kr], -1)
    attn = softmax(qf @ kf.transpose(0, 1, 3, 2) * (dn + dr) ** -0.5)
    out = (attn @ v).transpose(0, 2, 1, 3).reshape(B, Tq, H * dv)
    return out @ w["out_proj"].T


def absorb_query(q_nope, w_kup, n_heads, nope_dim):
    """q_lat[b, h] = W_uk[h]^T q_nope[b, h]; q_nope (B, H, dn), W_uk (H*dn, R)."""
    wk = np.asarray(w_kup, np.float64).reshape(n_heads, nope_dim, -1)
    return np.einsum("bhd,hdr->bhr", np.asarray(q_nope, np.float64), wk)


def sparse_positions(length, selected_chunks, chunk, sink, window):
    """Sorted positions attended by one query: sink prefix, recent window and the
    selected chunks (dedup'd, clipped to the sequence)."""
    pos = set(range(min(sink, length)))
    pos.update(range(max(0, length - window), length))
    for c in selected_chunks:
        pos.update(range(c * chunk, min(length, (c + 1) * chunk)))
    return np.array(sorted(pos), dtype=np.int64)


def sparse_mla_decode(q_lat, q_pe, latent, rope, positions, scale):
    """q_lat (H, R), q_pe (H, P), latent (T, R), rope (T, P) -> (H, R) latent output."""
    c = np.asarray(latent, np.float64)[positions]
    kp = np.asarray(rope, np.float64)[positions]
    s = (np.asarray(q_lat, np.float64) @ c.T + np.asarray(q_pe, np.float64) @ kp.T) * scale
    return softmax(s) @ c
