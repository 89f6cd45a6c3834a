"""Many sequences on one paged KV pool — the batched form of PagedKVCache.

The reference cache holds one sequence per instance (snapmind/kv_cache/paged.py:51-52
reads ``key[0]`` only).  Serving many sequences needs the same slot arithmetic
over one shared pool; this class is that extension, with all state on the GPU:

* ``k``, ``v``: ``[layer][block][head][slot][dim]``; a block id is valid in every
  layer, so one block table row per sequence serves all layers;
* ``block_tables`` int32 ``[max_seqs][max_blocks_per_seq]``, ``seq_lens`` int32;
* a device free stack (``free_stack``, ``free_top``) from which
  ``snapmind_kv_reserve`` grows tables deterministically (ascending sequence
  order, blocks from the top of the stack).

Block bookkeeping (tables, lengths, free stack, reserve/release) is in
:class:`snapmind_b200.block_pool.BlockPool`.
"""
from __future__ import annotations

from collections.abc import MutableMapping

import torch

from snapmind_b200 import _lib
from snapmind_b200.block_pool import BlockPool


class PagedKVPool(BlockPool):
    def __init__(
        self,
        n_layers: int,
        n_kv_heads: int,
        head_dim: int,
        num_blocks: int,
        max_seqs: int,
        max_blocks_per_seq: int,
        block_size: int = 16,
        dtype: torch.dtype = torch.bfloat16,
        device: torch.device | str | None = None,
    ):
        super().__init__(num_blocks, max_seqs, max_blocks_per_seq, block_size, device)
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        self.dtype = dtype
        self._dcode = _lib.dtype_code(dtype)
        shape = (n_layers, num_blocks, n_kv_heads, block_size, head_dim)
        self.k = torch.empty(shape, dtype=dtype, device=self.device)
        self.v = torch.empty(shape, dtype=dtype, device=self.device)
        self.layer_stride = num_blocks * n_kv_heads * block_size * head_dim
        self._workspace = _lib.DecodeWorkspace(self.device)

    def append(self, layer: int | None, k_new: torch.Tensor, v_new: torch.Tensor, slot_starts=None,
               slot_start0: int | None = None) -> None:
        """Write new tokens' K/V rows.

        ``k_new``: ``[B, H, D]`` (one token, layer ``layer``), ``[B, H, T, D]``,
        or ``[L, B, H, T, D]`` with ``layer=None`` (all layers at once).  By
        default token t of sequence b goes to slot ``seq_lens[b] - T + t`` — the
        slots that the last ``reserve(T)`` added.
        """
        if k_new.dim() == 3:
            k_new, v_new = k_new.unsqueeze(2), v_new.unsqueeze(2)
        if k_new.dim() == 4:
            if layer is None:
                raise ValueError("layer is required for [B, H, T, D] inputs")
            k_new, v_new = k_new.unsqueeze(0), v_new.unsqueeze(0)
            n_layers, base = 1, layer
        else:
            n_layers, base = k_new.shape[0], (0 if layer is None else layer)
        if k_new.stride() != v_new.stride():
            k_new, v_new = k_new.contiguous(), v_new.contiguous()
        _, batch, n_heads, n_tokens, head_dim = k_new.shape
        if n_heads != self.n_kv_heads or head_dim != self.head_dim:
            raise ValueError(f"expected {self.n_kv_heads} heads of {self.head_dim}, got {tuple(k_new.shape)}")
        starts_ptr, start0 = self._slot_args(n_tokens, slot_starts, slot_start0)
        st = k_new.stride()
        status = _lib.load().snapmind_kv_append(
            self.k[base].data_ptr(), self.v[base].data_ptr(), self._dcode, self.layer_stride,
            k_new.data_ptr(), v_new.data_ptr(), _lib.dtype_code(k_new.dtype),
            st[0], st[1], st[2], st[3],
            self.block_tables.data_ptr(), self.max_blocks_per_seq, 0, self.max_blocks_per_seq,
            starts_ptr, start0,
            n_layers, batch, n_tokens, n_heads, head_dim, self.block_size, self.num_blocks,
            self.err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, "PagedKVPool.append")

    # ----------------------------------------------------------------- reads
    def gather(self, batch: int | None = None, layers: range | None = None, out=None):
        """Packed K/V of the first ``batch`` sequences.

        Returns ``(k, v)`` of shape ``[n_layers, total_tokens * H * D]`` where the
        row of each layer is the concatenation over b of ``(H, len_b, D)`` — for
        one sequence the tensor ``PagedKVCache.fetch`` returns.
        """
        batch = self.max_seqs if batch is None else batch
        layers = range(self.n_layers) if layers is None else layers
        total = int(self._host_lens[:batch].sum())
        per_layer = total * self.n_kv_heads * self.head_dim
        if out is None:
            k_out = torch.empty((len(layers), per_layer), dtype=self.dtype, device=self.device)
            v_out = torch.empty_like(k_out)
        else:
            k_out, v_out = out
            for t in (k_out, v_out):
                if t.dtype != self.dtype or t.shape[0] < len(layers) or t[0].numel() < per_layer or not t.is_contiguous():
                    raise ValueError("gather output too small or not contiguous")
        if per_layer == 0 or len(layers) == 0:
            return k_out, v_out
        status = _lib.load().snapmind_kv_gather(
            self.k[layers.start].data_ptr(), self.v[layers.start].data_ptr(), self._dcode, self.layer_stride,
            k_out.data_ptr(), v_out.data_ptr(), per_layer, per_layer,
            self.block_tables.data_ptr(), self.max_blocks_per_seq, 0, self.max_blocks_per_seq,
            self.seq_lens.data_ptr(), 0,
            len(layers), batch, self.n_kv_heads, self.head_dim, self.block_size, self.num_blocks,
            self.err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, "PagedKVPool.gather")
        return k_out, v_out

    def _decode_workspace(self, batch, n_q_heads, max_len, split):
        lib = _lib.load()
        need = lib.snapmind_paged_gqa_decode_workspace_bytes(
            batch, n_q_heads, self.n_kv_heads, self.head_dim, max_len, split
        )
        return self._workspace.get(batch, self.n_kv_heads, need)

    def decode_layers(self, q: torch.Tensor, out: torch.Tensor | None = None, scale: float | None = None,
                      split_tokens: int = 0, max_seq_len: int | None = None, peers=None) -> torch.Tensor | None:
        """Paged GQA decode of layers 0 .. L-1 in one launch: ``q`` ``[L, B, Hq, D]`` ->
        ``[L, B, Hq, D]``.

        The pool is layer-contiguous, so block ``p`` of layer ``l`` is block
        ``l * num_blocks + p`` of one pool spanning every layer; launch row
        ``l * B + b`` is sequence ``b`` of layer ``l``, its table row shifted by
        ``l * num_blocks`` (entries outside ``[0, num_blocks)`` stay invalid, so the
        kernel still flags them).  ``q`` (and ``out``) must step uniformly over
        (layer, sequence) rows: ``stride(0) == B * stride(1)``.  ``peers`` as in
        ``decode``, with ``out_stride_seq`` the row stride of every rank's
        ``[L, B, Hq, D]`` receive region."""
        n_l, batch, n_q, d = q.shape
        if n_l > self.k.shape[0]:
            raise ValueError(f"{n_l} layers > the pool's {self.k.shape[0]}")
        if q.dtype != self.dtype or q.stride(-1) != 1 or q.stride(0) != batch * q.stride(1):
            raise ValueError("q must be [L, B, Hq, D] in the pool's dtype with uniformly strided rows")
        if out is None and peers is None:
            out = torch.empty((n_l, batch, n_q, d), dtype=self.dtype, device=self.device)
        if out is not None and (out.stride(-1) != 1 or out.stride(0) != batch * out.stride(1)):
            raise ValueError("out must be [L, B, Hq, D] with uniformly strided rows")
        scale = self.head_dim ** -0.5 if scale is None else scale
        if max_seq_len is None:
            max_seq_len = max(1, int(self._host_lens[:batch].max())) if batch else 1
        rows = n_l * batch
        lib = _lib.load()
        split = split_tokens or lib.snapmind_paged_gqa_decode_split_tokens(rows, self.n_kv_heads, max_seq_len,
                                                                           self.block_size)
        ws = self._decode_workspace(rows, n_q, max_seq_len, split)
        t = self.block_tables[:batch]
        offs = torch.arange(n_l, dtype=torch.int32, device=self.device).view(n_l, 1, 1) * self.num_blocks
        tables = torch.where((t >= 0) & (t < self.num_blocks), t.unsqueeze(0) + offs, torch.full_like(t, -1))
        lens = self.seq_lens[:batch].unsqueeze(0).expand(n_l, batch).contiguous()
        span = n_l * self.num_blocks
        if peers is not None:
            status = lib.snapmind_paged_gqa_decode_peers(
                q.data_ptr(), q.stride(1), q.stride(2), self.k.data_ptr(), self.v.data_ptr(), self._dcode,
                tables.data_ptr(), self.max_blocks_per_seq, self.max_blocks_per_seq, lens.data_ptr(), None,
                peers.out_ptrs.data_ptr(), peers.n, peers.head_offset, peers.out_stride_seq, peers.out_stride_head,
                float(scale), rows, n_q, self.n_kv_heads, self.head_dim, self.block_size, span,
                max_seq_len, split, 0, ws.data_ptr(), ws.numel(), self.err.data_ptr(), self._stream(),
            )  # fmt: skip
            _lib.check(status, "PagedKVPool.decode_layers (peers)")
            return None
        status = lib.snapmind_paged_gqa_decode(
            q.data_ptr(), q.stride(1), q.stride(2), self.k.data_ptr(), self.v.data_ptr(), self._dcode,
            tables.data_ptr(), self.max_blocks_per_seq, self.max_blocks_per_seq, lens.data_ptr(),
            out.data_ptr(), out.stride(1), out.stride(2), float(scale), rows, n_q, self.n_kv_heads, self.head_dim,
            self.block_size, span, max_seq_len, split, 0, ws.data_ptr(), ws.numel(), self.err.data_ptr(),
            self._stream(),
        )  # fmt: skip
        _lib.check(status, "PagedKVPool.decode_layers")
        return out

    def decode(self, layer: int, q: torch.Tensor, out: torch.Tensor | None = None, scale: float | None = None,
               batch: int | None = None, split_tokens: int = 0, force_generic: bool = False,
               max_seq_len: int | None = None, peers=None, append=None) -> torch.Tensor | None:
        """Paged GQA decode attention of ``q`` ``[B, Hq, D]`` against layer ``layer``.

        ``peers`` (a ``head_shard.PeerTargets``) sends the output rows to the
        output buffers of every rank of a head-sharded decode instead of ``out``
        and returns None.  ``append=(k_new, v_new)`` (``[B, H, D]``, the pool's
        dtype) stores this step's token of every sequence (the last slot the
        latest ``reserve(1)`` gave it) in the same launch, in place of an
        ``append`` call before the decode."""
        batch = q.shape[0] if batch is None else batch
        n_q = q.shape[1]
        if peers is not None and append is not None:
            raise ValueError("decode with peers does not store the step's token: append it first")
        if q.dtype != self.dtype:
            raise TypeError(f"q dtype {q.dtype} != pool dtype {self.dtype}")
        if q.stride(-1) != 1:
            q = q.contiguous()
        if out is None and peers is None:
            out = torch.empty((batch, n_q, self.head_dim), dtype=self.dtype, device=self.device)
        scale = self.head_dim ** -0.5 if scale is None else scale
        if max_seq_len is None:
            max_seq_len = max(1, int(self._host_lens[:batch].max())) if batch else 1
        max_len = max_seq_len
        lib = _lib.load()
        split = split_tokens or lib.snapmind_paged_gqa_decode_split_tokens(
            batch, self.n_kv_heads, max_len, self.block_size
        )
        ws = self._decode_workspace(batch, n_q, max_len, split)
        if peers is not None:
            status = lib.snapmind_paged_gqa_decode_peers(
                q.data_ptr(), q.stride(0), q.stride(1),
                self.k[layer].data_ptr(), self.v[layer].data_ptr(), self._dcode,
                self.block_tables.data_ptr(), self.max_blocks_per_seq, self.max_blocks_per_seq,
                self.seq_lens.data_ptr(), None,
                peers.out_ptrs.data_ptr(), peers.n, peers.head_offset, peers.out_stride_seq, peers.out_stride_head,
                float(scale), batch, n_q, self.n_kv_heads, self.head_dim, self.block_size, self.num_blocks,
                max_len, split, _lib.DECODE_FORCE_GENERIC if force_generic else 0,
                ws.data_ptr(), ws.numel(), self.err.data_ptr(), self._stream(),
            )  # fmt: skip
            _lib.check(status, "PagedKVPool.decode (peers)")
            return None
        if append is not None:
            k_new, v_new = append
            if k_new.dtype != self.dtype or v_new.dtype != self.dtype or k_new.stride() != v_new.stride():
                raise TypeError("append rows must have the pool's dtype and matching strides")
            if k_new.shape != (batch, self.n_kv_heads, self.head_dim) or k_new.stride(-1) != 1:
                raise ValueError(f"append rows must be [{batch}, {self.n_kv_heads}, {self.head_dim}], "
                                 f"head dim contiguous, got {tuple(k_new.shape)}")
            status = lib.snapmind_paged_gqa_decode_append(
                q.data_ptr(), q.stride(0), q.stride(1),
                self.k[layer].data_ptr(), self.v[layer].data_ptr(), self._dcode,
                self.block_tables.data_ptr(), self.max_blocks_per_seq, self.max_blocks_per_seq,
                self.seq_lens.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), k_new.stride(1),
                out.data_ptr(), out.stride(0), out.stride(1),
                float(scale), batch, n_q, self.n_kv_heads, self.head_dim, self.block_size, self.num_blocks,
                max_len, split, _lib.DECODE_FORCE_GENERIC if force_generic else 0,
                ws.data_ptr(), ws.numel(), self.err.data_ptr(), self._stream(),
            )  # fmt: skip
            _lib.check(status, "PagedKVPool.decode (append)")
            return out
        status = lib.snapmind_paged_gqa_decode(
            q.data_ptr(), q.stride(0), q.stride(1),
            self.k[layer].data_ptr(), self.v[layer].data_ptr(), self._dcode,
            self.block_tables.data_ptr(), self.max_blocks_per_seq, self.max_blocks_per_seq,
            self.seq_lens.data_ptr(),
            out.data_ptr(), out.stride(0), out.stride(1),
            float(scale), batch, n_q, self.n_kv_heads, self.head_dim, self.block_size, self.num_blocks,
            max_len, split, _lib.DECODE_FORCE_GENERIC if force_generic else 0,
            ws.data_ptr(), ws.numel(), self.err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, "PagedKVPool.decode")
        return out

    def _lens_ladder(self, n: int) -> torch.Tensor:
        lad = getattr(self, "_ladder", None)
        if lad is None or lad.numel() < n:
            lad = torch.arange(1, max(n, 1) + 1, dtype=torch.int32, device=self.device)
            self._ladder = lad
        return lad

    def attend_causal(self, layer: int, b: int, q: torch.Tensor, out: torch.Tensor, n_b: int,
                      scale: float | None = None) -> torch.Tensor:
        """Causal attention of the newest ``T`` tokens of sequence ``b``
        (``q``/``out`` ``[Hq, T, D]``, sequence length ``n_b``): query t sees the
        first ``n_b - T + t + 1`` tokens; one decode-kernel row per query, all
        on the sequence's table row."""
        n_q, n_t = q.shape[0], q.shape[1]
        if n_t == 0:
            return out
        scale = self.head_dim ** -0.5 if scale is None else scale
        lad = self._lens_ladder(n_b)
        lib = _lib.load()
        split = lib.snapmind_paged_gqa_decode_split_tokens(n_t, self.n_kv_heads, n_b, self.block_size)
        ws = self._decode_workspace(n_t, n_q, n_b, split)
        status = lib.snapmind_paged_gqa_decode(
            q.data_ptr(), q.stride(1), q.stride(0),
            self.k[layer].data_ptr(), self.v[layer].data_ptr(), self._dcode,
            self.block_tables[b].data_ptr(), 0, self.max_blocks_per_seq, lad.data_ptr() + 4 * (n_b - n_t),
            out.data_ptr(), out.stride(1), out.stride(0),
            float(scale), n_t, n_q, self.n_kv_heads, self.head_dim, self.block_size, self.num_blocks,
            n_b, split, 0, ws.data_ptr(), ws.numel(), self.err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, "PagedKVPool.attend_causal")
        return out

    def layer_views(self, batch: int) -> dict[int, "PoolLayerView"]:
        """One ``kv_cache`` view per layer for sequences ``0 .. batch - 1``."""
        return {i: PoolLayerView(self, i, batch) for i in range(self.n_layers)}


class PoolLayerView(MutableMapping):
    """The ``kv_cache`` of one layer for a batch of sequences of a
    :class:`PagedKVPool`, read and written by the ``gqa_paged`` attention plugin.

    The sequences are ragged, so the view holds no dense K/V tensor: ``"k"`` /
    ``"v"`` read as ``None`` until the layer has stored tokens (a model's prefill
    test, e.g. ``kv_cache.get("k") is None``) and as an empty placeholder after.
    The caller grows the sequences (``reserve``) before each forward; the
    plugin appends the new rows and attends from the pool.  ``capacity``, when
    set, is the length bound the decode split plan is made for (fixed plans
    for CUDA-graph replay).
    """

    KEYS = ("k", "v")

    def __init__(self, pool: PagedKVPool, layer: int, batch: int):
        self.pool, self.layer, self.batch = pool, layer, batch
        self.stored = 0
        self.capacity: int | None = None
        self._placeholder = torch.empty(0, dtype=pool.dtype, device=pool.device)

    def __getitem__(self, key):
        if key not in self.KEYS:
            raise KeyError(key)
        return None if self.stored == 0 else self._placeholder

    def __setitem__(self, key, value):
        raise TypeError("PoolLayerView is written by the gqa_paged attention plugin only")

    def __delitem__(self, key):
        raise TypeError("PoolLayerView entries cannot be deleted")

    def __iter__(self):
        return iter(self.KEYS)

    def __len__(self):
        return len(self.KEYS)
