"""Grouped-query attention that attends straight from the paged KV pool.

``PagedGroupedQueryAttention`` is a drop-in for snapmind's
``GroupedQueryAttention`` (snapmind/layers/attention/gqa.py:11-85), registered
as ``"gqa_paged"`` in this package's ``ATTENTION``: the same constructor, the
same submodules (``q_proj``, ``k_proj``, ``v_proj``, ``out_proj``, created in
the same order, so state dicts load either way and a seeded construction gives
the same weights), the same forward signature and output.

The reference layer grows the layer's cache dict with ``torch.cat`` and runs
dense attention over ``repeat_interleave``-d K/V (gqa.py:62-85), re-reading and
re-copying the whole history every step.  This layer, given the layer view of a
``"paged"`` cache of this package (``PagedKVCache.layer_dicts()[i]``):

* appends the new K/V rows into the cache's pool with the append kernel
  (``PagedKVCache.store``: the reference's block allocation order);
* runs the paged GQA decode kernel over the layer's block table
  (``PagedKVCache.attend``): one query is a decode step; ``T`` queries are a
  causal prefill, one kernel row per query sharing the table row.

RoPE runs as one kernel over q and k in place (``snapmind_rope_qk``,
bit-identical to ``apply_to_qk`` on the same device) when ``pe`` exposes the
reference's rotate-half tables — ``cos_cached`` / ``sin_cached`` of shape
``[n_pos, head_dim]`` and ``_rotate_half``, as
snapmind/layers/positional/rope.py:11-61 does; any other ``pe`` is applied
with its own ``apply_to_qk``.  The projections and the output projection stay
torch, as in the reference.  Without a cache (``kv_cache=None``) the layer
attends causally over its own ``T`` tokens through a transient one-layer pool.

Differences a caller can see: the attention weights are not materialised (the
second output is ``None``); ``mask`` must be ``None`` or the causal mask of
snapmind/layers/attention/sdpa.py ``create_causal_mask`` (what the reference
models pass), anything else raises ``ValueError``; dropout is not applied
(inference only); the batch is 1, as in the reference cache.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from snapmind_b200 import _lib
from snapmind_b200.kv_cache.paged import PagedKVCache, PagedLayerView
from snapmind_b200.kv_cache.sliding_window import SlidingLayerView
from snapmind_b200.paged_pool import PoolLayerView
from snapmind_b200.registry import ATTENTION

try:  # the reference's attention contract (snapmind/layers/attention/base.py:9-22) when importable
    from snapmind.layers.attention.base import AttentionABC as _AttentionBase
except ImportError:
    _AttentionBase = nn.Module

_ROPE_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


def _is_causal_mask(mask: torch.Tensor, n_q: int, n_k: int) -> bool:
    """True if ``mask`` is ``triu(full(-inf), diagonal=1)`` of shape (n_q, n_k), n_q == n_k."""
    if mask.shape[-2:] != (n_q, n_k) or n_q != n_k:
        return False
    m = mask.reshape(n_q, n_k)
    upper = torch.ones((n_q, n_k), dtype=torch.bool, device=m.device).triu(1)
    ok = torch.where(upper, torch.isneginf(m), m == 0)
    return bool(ok.all())


def _is_window_mask(mask: torch.Tensor, n: int, window: int) -> bool:
    """True if ``mask`` is snapmind/models/mistral.py ``create_sliding_window_mask(n, window)``:
    row i open on ``[max(0, i - window + 1), i]``, ``-inf`` elsewhere."""
    if mask.shape[-2:] != (n, n):
        return False
    m = mask.reshape(n, n)
    i = torch.arange(n, device=m.device)[:, None]
    j = torch.arange(n, device=m.device)[None, :]
    allowed = (j <= i) & (j >= i - window + 1)
    return bool(torch.where(allowed, m == 0, torch.isneginf(m)).all())


@ATTENTION.register("gqa_paged")
class PagedGroupedQueryAttention(_AttentionBase):
    def __init__(
        self,
        d_model: int,
        n_heads: int,
        n_kv_heads: int | None = None,
        dropout: float = 0.0,
        bias: bool = False,
        pe: nn.Module | None = None,
        head_dim: int | None = None,
    ):
        super().__init__()
        if head_dim is None:
            assert d_model % n_heads == 0
        self.d_model = d_model
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads if n_kv_heads is not None else n_heads
        self.n_rep = self.n_heads // self.n_kv_heads
        self.head_dim = head_dim if head_dim is not None else d_model // n_heads
        self.dropout = dropout
        self.pe = pe

        self.q_proj = nn.Linear(d_model, n_heads * self.head_dim, bias=bias)
        self.k_proj = nn.Linear(d_model, self.n_kv_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(d_model, self.n_kv_heads * self.head_dim, bias=bias)
        self.out_proj = nn.Linear(n_heads * self.head_dim, d_model, bias=bias)

    def _split_heads(self, x: torch.Tensor, n_heads: int) -> torch.Tensor:
        batch, seq_len, _ = x.shape
        return x.view(batch, seq_len, n_heads, self.head_dim).transpose(1, 2)

    def _rope_tables(self, q: torch.Tensor):
        """(cos, sin) for the fused kernel, or None to use ``pe.apply_to_qk``."""
        pe = self.pe
        cos, sin = getattr(pe, "cos_cached", None), getattr(pe, "sin_cached", None)
        if not (isinstance(cos, torch.Tensor) and isinstance(sin, torch.Tensor) and hasattr(pe, "_rotate_half")):
            return None
        if cos.dim() != 2 or cos.shape != sin.shape or cos.shape[1] != self.head_dim or self.head_dim % 2:
            return None
        if q.dtype not in _ROPE_DTYPES or cos.device != q.device or torch.is_grad_enabled():
            return None
        if cos.dtype != torch.float32 or not cos.is_contiguous():
            cos = cos.float().contiguous()
        if sin.dtype != torch.float32 or not sin.is_contiguous():
            sin = sin.float().contiguous()
        return cos, sin

    def _rope(self, q, k, position_ids, tables, err: torch.Tensor) -> None:
        cos, sin = tables
        batch, n_tok = q.shape[0], q.shape[2]
        pos, pos_stride = None, 0
        if position_ids is not None:
            pos = position_ids.reshape(-1)
            if pos.numel() == batch * n_tok and batch > 1:
                pos_stride = n_tok  # one position list per sequence
            elif pos.numel() != n_tok:
                raise ValueError(f"gqa_paged: {pos.numel()} positions for {batch} x {n_tok} tokens")
            pos = pos.to(device=q.device, dtype=torch.int64).contiguous()
        status = _lib.load().snapmind_rope_qk(
            q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), q.shape[1],
            k.data_ptr(), k.stride(0), k.stride(1), k.stride(2), k.shape[1],
            _lib.dtype_code(q.dtype), q.shape[0], n_tok, self.head_dim, cos.data_ptr(), sin.data_ptr(),
            cos.shape[0], None if pos is None else pos.data_ptr(), pos_stride, err.data_ptr(),
            _lib.stream_handle(q.device),
        )  # fmt: skip
        _lib.check(status, "gqa_paged rope")

    def forward(
        self,
        x: torch.Tensor,
        kv_cache: PagedLayerView | None = None,
        position_ids: torch.Tensor | None = None,
        mask: torch.Tensor | None = None,
    ) -> tuple[torch.Tensor, None]:
        if isinstance(kv_cache, PoolLayerView):
            return self._forward_pool(x, kv_cache, position_ids, mask)
        if isinstance(kv_cache, SlidingLayerView):
            return self._forward_window(x, kv_cache, position_ids, mask)
        if x.shape[0] != 1:
            raise ValueError("gqa_paged: the paged cache holds one sequence (batch 1); use a pool view for more")
        q = self._split_heads(self.q_proj(x), self.n_heads)
        k = self._split_heads(self.k_proj(x), self.n_kv_heads)
        v = self._split_heads(self.v_proj(x), self.n_kv_heads)

        n_new = x.shape[1]
        if kv_cache is None:
            cache = PagedKVCache(n_new, 1, self.n_kv_heads, self.head_dim, dtype=k.dtype, device=x.device)
            layer = 0
        elif isinstance(kv_cache, PagedLayerView):
            cache, layer = kv_cache.cache, kv_cache.layer_idx
        else:
            raise TypeError(
                "gqa_paged attends from a snapmind_b200 paged cache: pass PagedKVCache.layer_dicts()[i], "
                f"got {type(kv_cache).__name__}"
            )
        if cache.n_heads != self.n_kv_heads or cache.head_dim != self.head_dim:
            raise ValueError(
                f"gqa_paged: cache holds {cache.n_heads} heads x {cache.head_dim}, "
                f"layer needs {self.n_kv_heads} x {self.head_dim}"
            )
        if self.pe is not None:
            tables = self._rope_tables(q)
            if tables is not None:
                self._rope(q, k, position_ids, tables, cache._err)  # in place on the fresh projections
            else:
                q, k = self.pe.apply_to_qk(q, k, position_ids)
        if cache.device_steps_active:  # one token at the device counters (a captured decode step)
            if n_new != 1 or mask is not None:
                raise ValueError("gqa_paged: device steps take one token and no mask")
            cache.store_device(layer, k, v)
            qd = q if q.dtype == cache.dtype else q.to(cache.dtype)
            out = cache.attend_device(layer, qd, scale=self.head_dim ** -0.5)
            out = out.to(x.dtype).transpose(1, 2).reshape(1, 1, self.n_heads * self.head_dim)
            return self.out_proj(out), None
        cached = cache.num_tokens(layer)
        causal = True
        if mask is not None:
            if not _is_causal_mask(mask, n_new, cached + n_new):
                raise ValueError("gqa_paged supports no mask or the causal mask only")
        elif n_new > 1 and cached > 0:
            causal = False  # the reference attends every new query to every token here

        cache.store(layer, k, v, cached)
        qd = q if q.dtype == cache.dtype else q.to(cache.dtype)
        out = cache.attend(layer, qd, scale=self.head_dim ** -0.5, causal=causal)
        out = out.to(x.dtype).transpose(1, 2).reshape(1, n_new, self.n_heads * self.head_dim)
        return self.out_proj(out), None

    def _forward_pool(self, x, view: PoolLayerView, position_ids, mask):
        """B sequences of a ``PagedKVPool`` (grown by the caller's ``reserve`` for this
        forward): one token each is a batched decode step; ``T`` tokens each (the
        same ``T`` for all) is a causal prefill, attended per sequence."""
        pool, layer = view.pool, view.layer
        batch, n_new = x.shape[0], x.shape[1]
        if batch != view.batch:
            raise ValueError(f"gqa_paged: view holds {view.batch} sequences, input has {batch}")
        if pool.n_kv_heads != self.n_kv_heads or pool.head_dim != self.head_dim:
            raise ValueError("gqa_paged: pool heads / head_dim do not match the layer")
        q = self._split_heads(self.q_proj(x), self.n_heads)
        k = self._split_heads(self.k_proj(x), self.n_kv_heads)
        v = self._split_heads(self.v_proj(x), self.n_kv_heads)
        if self.pe is not None:
            tables = self._rope_tables(q)
            if tables is not None:
                self._rope(q, k, position_ids, tables, pool.err)
            else:
                q, k = self.pe.apply_to_qk(q, k, position_ids)
        qd = q if q.dtype == pool.dtype else q.to(pool.dtype)
        if n_new == 1:
            if mask is not None:
                raise ValueError("gqa_paged: a decode step takes no mask")
            pool.append(layer, k[:, :, 0], v[:, :, 0])
            out = pool.decode(layer, qd[:, :, 0], max_seq_len=view.capacity)
            out = out.to(x.dtype).reshape(batch, 1, self.n_heads * self.head_dim)
        else:
            if view.stored and mask is None:
                raise ValueError("gqa_paged: pool views take multi-token steps as causal prefill only")
            if mask is not None and not _is_causal_mask(mask, n_new, n_new):
                raise ValueError("gqa_paged supports no mask or the causal mask only")
            pool.append(layer, k, v)
            out = torch.empty((batch, self.n_heads, n_new, self.head_dim), dtype=pool.dtype, device=x.device)
            lens = pool.host_lens
            for b in range(batch):
                pool.attend_causal(layer, b, qd[b], out[b], int(lens[b]))
            out = out.to(x.dtype).transpose(1, 2).reshape(batch, n_new, self.n_heads * self.head_dim)
        view.stored += n_new
        return self.out_proj(out), None

    def _forward_window(self, x, view: SlidingLayerView, position_ids, mask):
        """One sequence over a ``"sliding_window"`` cache, with the reference's window
        semantics (snapmind/models/mistral.py:14-21 and 48-60): a prefill on an
        empty window takes the sliding-window (or causal) mask, query i seeing
        rows ``[i - window + 1, i]`` — run in chunks of at most ``window``
        queries; without a mask every query sees every held token plus the new
        ones.  The window is trimmed to ``window_size`` afterwards, as the
        reference's Mistral block does."""
        cache, layer = view.cache, view.layer_idx
        if x.shape[0] != 1:
            raise ValueError("gqa_paged: the sliding-window cache holds one sequence (batch 1)")
        q = self._split_heads(self.q_proj(x), self.n_heads)
        k = self._split_heads(self.k_proj(x), self.n_kv_heads)
        v = self._split_heads(self.v_proj(x), self.n_kv_heads)
        if cache.n_heads != self.n_kv_heads or cache.head_dim != self.head_dim:
            raise ValueError("gqa_paged: cache heads / head_dim do not match the layer")
        if self.pe is not None:
            tables = self._rope_tables(q)
            if tables is not None:
                self._rope(q, k, position_ids, tables, cache._err)
            else:
                q, k = self.pe.apply_to_qk(q, k, position_ids)
        w, n_new, n_old = cache.window_size, x.shape[1], cache.num_tokens(layer)
        if mask is not None:
            if n_old:
                raise ValueError("gqa_paged: a masked prefill needs an empty window")
            if not (_is_window_mask(mask, n_new, w) or (n_new <= w and _is_causal_mask(mask, n_new, n_new))):
                raise ValueError("gqa_paged: the mask must be the sliding-window mask of the cache's window")
            chunk = w
        else:
            if n_old + n_new > 2 * w:
                raise ValueError("gqa_paged: an unmasked step of more than window_size tokens on a full window")
            chunk = n_new
        outs = []
        dev = x.device
        for c0 in range(0, n_new, chunk):
            kc, vc = k[:, :, c0:c0 + chunk], v[:, :, c0:c0 + chunk]
            qc = q[:, :, c0:c0 + chunk]
            tc = kc.shape[2]
            cache._append(layer, kc, vc)
            skip = cache._skip[layer]
            total = skip + cache.num_tokens(layer)
            if mask is not None:
                rows = torch.arange(total - tc, total, dtype=torch.int32, device=dev)
                lens = rows + 1
                starts = torch.clamp(rows - w + 1, min=skip)
            else:
                lens = torch.full((tc,), total, dtype=torch.int32, device=dev)
                starts = torch.full((tc,), skip, dtype=torch.int32, device=dev)
            qd = qc if qc.dtype == cache.dtype else qc.to(cache.dtype)
            outs.append(cache.attend(layer, qd, lens, starts, scale=self.head_dim ** -0.5))
            if mask is not None:
                cache._trim(layer, w)
        cache._trim(layer, w)
        out = torch.cat(outs, dim=2) if len(outs) > 1 else outs[0]
        out = out.to(x.dtype).transpose(1, 2).reshape(1, n_new, self.n_heads * self.head_dim)
        return self.out_proj(out), None
