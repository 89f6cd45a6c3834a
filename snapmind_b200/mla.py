"""MLA latent cache on the B200: paged compressed-latent rows.

The reference MLA layer keeps, per layer, the compressed latent ``k`` (width
``kv_lora_rank``) and the raw, un-rotated rope key ``k_rope`` (width
``qk_rope_head_dim``) and grows both with ``torch.cat``
(snapmind/layers/attention/mla.py:115-126).  Here both live in paged pools that
share one block table per sequence:

* ``latent``: ``[layer][block][1][slot][kv_lora_rank]``,
* ``rope``:   ``[layer][block][1][slot][rope_dim]``,

written by the ``snapmind_kv_append`` kernel and read back by
``snapmind_kv_gather`` (both in single-pool mode).  With ``block_size`` equal to
the indexer's chunk size (64), one block is one indexer chunk.

:class:`PagedLatentDict` is the per-layer ``kv_cache`` mapping the reference
``MultiHeadLatentAttention.forward`` reads and assigns: ``get("k")`` returns
the gathered latent ``(B, T, R)``, and the assignment of the concatenated
tensors stores only the rows past what the cache already holds.
"""
from __future__ import annotations

from collections.abc import MutableMapping

import torch

from snapmind_b200 import _lib
from snapmind_b200.block_pool import BlockPool


class MLALatentPool(BlockPool):
    def __init__(
        self,
        n_layers: int,
        num_blocks: int,
        max_seqs: int,
        max_blocks_per_seq: int,
        block_size: int = 64,
        kv_lora_rank: int = 512,
        rope_dim: int = 64,
        dtype: torch.dtype = torch.bfloat16,
        device: torch.device | str | None = None,
    ):
        super().__init__(num_blocks, max_seqs, max_blocks_per_seq, block_size, device)
        self.n_layers, self.kv_lora_rank, self.rope_dim = n_layers, kv_lora_rank, rope_dim
        self.dtype = dtype
        self._dcode = _lib.dtype_code(dtype)
        self.latent = torch.empty((n_layers, num_blocks, 1, block_size, kv_lora_rank), dtype=dtype, device=self.device)
        self.rope = torch.empty((n_layers, num_blocks, 1, block_size, rope_dim), dtype=dtype, device=self.device)

    def _append_one(self, pool: torch.Tensor, rows: torch.Tensor, base: int, n_layers: int, starts_ptr, start0):
        # rows: [L, B, T, W]
        if rows.stride(-1) != 1:
            rows = rows.contiguous()
        st = rows.stride()
        _, batch, n_tokens, width = rows.shape
        status = _lib.load().snapmind_kv_append(
            pool[base].data_ptr(), None, self._dcode, pool[0].numel(),
            rows.data_ptr(), None, _lib.dtype_code(rows.dtype),
            st[0], st[1], 0, st[2],
            self.block_tables.data_ptr(), self.max_blocks_per_seq, 0, self.max_blocks_per_seq,
            starts_ptr, start0,
            n_layers, batch, n_tokens, 1, width, self.block_size, self.num_blocks,
            self.err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, "MLALatentPool.append")

    def append(self, layer: int | None, latent_new: torch.Tensor, rope_new: torch.Tensor, slot_starts=None,
               slot_start0: int | None = None) -> None:
        """Write new tokens' latent/rope rows.

        ``latent_new``: ``[B, T, R]`` for layer ``layer`` or ``[L, B, T, R]`` with
        ``layer=None``; ``rope_new`` likewise with width ``rope_dim``.  Token t of
        sequence b goes to slot ``seq_lens[b] - T + t`` unless slots are given.
        """
        if latent_new.dim() == 3:
            if layer is None:
                raise ValueError("layer is required for [B, T, R] inputs")
            latent_new, rope_new = latent_new.unsqueeze(0), rope_new.unsqueeze(0)
            n_layers, base = 1, layer
        else:
            n_layers, base = latent_new.shape[0], (0 if layer is None else layer)
        if latent_new.shape[-1] != self.kv_lora_rank or rope_new.shape[-1] != self.rope_dim:
            raise ValueError("latent/rope widths do not match the pool")
        starts_ptr, start0 = self._slot_args(latent_new.shape[2], slot_starts, slot_start0)
        self._append_one(self.latent, latent_new, base, n_layers, starts_ptr, start0)
        self._append_one(self.rope, rope_new, base, n_layers, starts_ptr, start0)

    def gather(self, layer: int, batch: int, seq_len: int | None = None, out=None):
        """Latent ``(B, T, R)`` and rope ``(B, T, P)`` of the first ``batch`` sequences
        of one layer; ``seq_len`` (all sequences) defaults to the pool lengths,
        which must then be equal.  ``out`` may pass preallocated (latent, rope)."""
        if seq_len is None:
            lens = self._host_lens[:batch]
            if batch and (lens != lens[0]).any():
                raise ValueError("gather of a dense (B, T, R) view needs equal lengths")
            seq_len = int(lens[0]) if batch else 0
        outs = []
        for i, (pool, width) in enumerate(((self.latent, self.kv_lora_rank), (self.rope, self.rope_dim))):
            if out is None:
                o = torch.empty((batch, seq_len, width), dtype=self.dtype, device=self.device)
            else:
                o = out[i]
                if o.shape != (batch, seq_len, width) or o.dtype != self.dtype or not o.is_contiguous():
                    raise ValueError("gather output has the wrong shape, dtype or layout")
            if batch and seq_len:
                status = _lib.load().snapmind_kv_gather(
                    pool[layer].data_ptr(), None, self._dcode, 0,
                    o.data_ptr(), None, 0, o.numel(),
                    self.block_tables.data_ptr(), self.max_blocks_per_seq, 0, self.max_blocks_per_seq,
                    None, seq_len,
                    1, batch, 1, width, self.block_size, self.num_blocks,
                    self.err.data_ptr(), self._stream(),
                )  # fmt: skip
                _lib.check(status, "MLALatentPool.gather")
            outs.append(o)
        return outs[0], outs[1]


    def sparse_decode(self, layer: int, q_lat: torch.Tensor, q_pe: torch.Tensor, selected: torch.Tensor | None,
                      sink: int = 4, window: int = 1024, scale: float | None = None, n_splits: int | None = None,
                      out: torch.Tensor | None = None, batch: int | None = None) -> torch.Tensor:
        """Sparse MLA decode attention of one query token per sequence.

        ``q_lat`` ``[B, H, kv_lora_rank]`` (the no-rope query absorbed through the
        key up-projection), ``q_pe`` ``[B, H, rope_dim]``, ``selected`` int32
        ``[B, k]`` chunk ids (block ids of the sequence, -1 unused).  Attends over
        positions < sink, >= len - window and the selected chunks; returns the
        latent output ``[B, H, kv_lora_rank]``.  ``n_splits`` (CTAs per
        sequence and head group) defaults to the kernel's choice for the batch.
        """
        batch = q_lat.shape[0] if batch is None else batch
        H = q_lat.shape[1]
        if scale is None:
            raise ValueError("scale is required (MLA uses (qk_nope_head_dim + qk_rope_head_dim) ** -0.5)")
        q_lat = q_lat.contiguous()
        q_pe = q_pe.contiguous()
        if out is None:
            out = torch.empty((batch, H, self.kv_lora_rank), dtype=self.dtype, device=self.device)
        k = 0 if selected is None else selected.shape[1]
        lib = _lib.load()
        if n_splits is None:
            n_splits = lib.snapmind_sparse_mla_default_splits(batch, H, self.kv_lora_rank, self.rope_dim,
                                                              self.block_size, self._dcode)
        need = lib.snapmind_sparse_mla_workspace_bytes(batch, H, self.kv_lora_rank, n_splits)
        if getattr(self, "_sparse_ws", None) is None:
            self._sparse_ws = _lib.DecodeWorkspace(self.device)
        # tickets: one per (sequence, group of 16 heads) of the split-combining kernel
        ws = self._sparse_ws.get(batch, (H + 15) // 16, need)
        status = lib.snapmind_sparse_mla_decode(
            q_lat.data_ptr(), q_pe.data_ptr(), self._dcode, self.latent[layer].data_ptr(),
            self.rope[layer].data_ptr(), self.block_tables.data_ptr(), self.max_blocks_per_seq,
            self.max_blocks_per_seq, self.seq_lens.data_ptr(), None if selected is None else selected.data_ptr(),
            k, sink, window, float(scale), batch, H, self.kv_lora_rank, self.rope_dim, self.block_size,
            self.num_blocks, n_splits, out.data_ptr(), ws.data_ptr(), ws.numel(), self.err.data_ptr(),
            self._stream(),
        )  # fmt: skip
        _lib.check(status, "MLALatentPool.sparse_decode")
        return out


class PagedLatentDict(MutableMapping):
    """The ``kv_cache`` dict of one MLA layer for a dense batch of ``batch``
    sequences (pool sequences ``0..batch-1``), backed by an :class:`MLALatentPool`.

    Protocol of the reference layer (mla.py:115-126): ``get("k")`` /
    ``get("k_rope")`` return the cached tensors or None; the layer concatenates
    new rows and assigns ``kv_cache["k"], kv_cache["k_rope"] = ...``.  The
    assignment keeps only the rows beyond the cached length (the prefix is the
    tensor this mapping returned) and appends them on the GPU; blocks are
    reserved in the pool the first time any layer reaches a new length.
    """

    KEYS = ("k", "k_rope")

    def __init__(self, pool: MLALatentPool, layer: int, batch: int):
        self.pool, self.layer, self.batch = pool, layer, batch
        self.length = 0
        self._pending: torch.Tensor | None = None

    def __getitem__(self, key):
        if key not in self.KEYS:
            raise KeyError(key)
        if self.length == 0:
            raise KeyError(key)
        lat, rope = self.pool.gather(self.layer, self.batch, self.length)
        return lat if key == "k" else rope

    def get(self, key, default=None):
        try:
            return self[key]
        except KeyError:
            return default

    def __setitem__(self, key, value):
        if key == "k":
            self._pending = value
            return
        if key != "k_rope" or self._pending is None:
            raise KeyError(f"PagedLatentDict expects 'k' then 'k_rope' assignments, got {key!r}")
        latent, rope = self._pending, value
        self._pending = None
        total = latent.shape[-2]
        if latent.shape[0] != self.batch or rope.shape[-2] != total:
            raise ValueError("latent/rope batch or length mismatch")
        n_new = total - self.length
        if n_new < 0:
            raise ValueError("the MLA cache cannot shrink")
        if n_new == 0:
            return
        grow = total - int(self.pool.host_lens[: self.batch].max())
        if grow > 0:
            self.pool.reserve(grow, batch=self.batch)
        dev = self.pool.device
        lat_new = latent[:, self.length :, :].to(dev, self.pool.dtype)
        rope_new = rope[:, self.length :, :].to(dev, self.pool.dtype)
        self.pool.append(self.layer, lat_new, rope_new, slot_starts=self.length)
        self.length = total

    def __delitem__(self, key):
        raise TypeError("PagedLatentDict entries cannot be deleted")

    def __iter__(self):
        return iter(self.KEYS if self.length else ())

    def __len__(self):
        return len(self.KEYS) if self.length else 0
