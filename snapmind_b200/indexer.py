"""Lookahead sparse indexer on the B200.

``LookaheadSparseIndexer`` is a drop-in for snapmind's module of the same name
(snapmind/layers/indexer/lookahead.py:11-106), registered as
``"lookahead_sparse"`` in this package's ``INDEXER``: the same constructor,
the same projection layers (created in the same order, so a seeded
construction gives the same weights), the same control flow in ``score``
(uninitialised -> 0.5, missing chunk -> 0.0, hooked layers averaged, fallback
to the lowest layer).  The chunk work runs in CUDA kernels: frozen keys are
chunk means computed by ``snapmind_indexer_pool_chunks``, and every requested
chunk is scored in one ``snapmind_indexer_score_ref`` launch instead of a
Python loop that recomputes the query projection per chunk.  The query
projections themselves are dense GEMVs on hidden states and stay torch.

``ChunkSelector`` is the batched selector of the sparse-attention path: chunk
keys projected to ``index_dim`` straight from the paged latent pool (mean-pool
and projection fused in one kernel, incremental per new chunk), and
``sigmoid(q . k / sqrt(index_dim) + b)`` with a stable top-k per sequence.
"""
from __future__ import annotations

import abc

import torch
import torch.nn as nn

from snapmind_b200 import _lib
from snapmind_b200.registry import INDEXER


try:  # the reference's indexer contract itself (snapmind/layers/indexer/base.py:6-18) when importable
    from snapmind.layers.indexer.base import IndexerABC
except ImportError:

    class IndexerABC(abc.ABC):  # type: ignore[no-redef]
        """Stand-in for the reference's indexer contract: one abstract ``score``."""

        @abc.abstractmethod
        def score(self, hidden_states: dict[int, torch.Tensor], chunk_ids: list[int]) -> dict[int, torch.Tensor]: ...


def chunk_means(k: torch.Tensor, width: int) -> torch.Tensor:
    """Mean over the token dim of the first ``width`` columns: (..., T, W) -> (..., 1, width) fp32."""
    if k.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        k = k.float()
    lead, t, w = k.shape[:-2], k.shape[-2], k.shape[-1]
    k3 = k.reshape(-1, t, w)
    if k3.stride(-1) != 1 or k3.stride(-2) != w:
        k3 = k3.contiguous()
    out = torch.empty((k3.shape[0], width), dtype=torch.float32, device=k.device)
    table = torch.zeros(1, dtype=torch.int32, device=k.device)
    lib = _lib.load()
    for i in range(k3.shape[0]):
        status = lib.snapmind_indexer_pool_chunks(
            k3[i].data_ptr(), _lib.dtype_code(k3.dtype), w, width,
            table.data_ptr(), 1, 1, None, 1, t, 1, 0, 1, 1,
            None, 0, 0, out[i].data_ptr(), None, 0, None, _lib.stream_handle(k.device),
        )  # fmt: skip
        _lib.check(status, "indexer chunk mean")
    return out.reshape(*lead, 1, width)


@INDEXER.register("lookahead_sparse")
class LookaheadSparseIndexer(nn.Module, IndexerABC):
    def __init__(
        self,
        d_model: int,
        n_layers: int,
        kv_lora_rank: int = 512,
        qk_rope_head_dim: int = 64,
        q_lora_rank: int = 2048,
        indexer_layers: list[int] | None = None,
        n_indexer_heads: int = 4,
    ):
        nn.Module.__init__(self)
        self.d_model = d_model
        self.n_layers = n_layers
        self.kv_lora_rank = kv_lora_rank
        self.qk_rope_head_dim = qk_rope_head_dim
        self.q_lora_rank = q_lora_rank
        self.indexer_layers = indexer_layers or [10, 12, 20]
        self.n_indexer_heads = n_indexer_heads
        # same layers, same order as lookahead.py:35-39
        self.q_down_proj = nn.Linear(d_model, kv_lora_rank, bias=False)
        self.q_up_proj = nn.Linear(kv_lora_rank, n_indexer_heads * kv_lora_rank, bias=False)
        self.w_proj = nn.Linear(d_model, n_indexer_heads, bias=False)
        self._frozen_keys: dict[int, torch.Tensor] = {}
        self._initialized = False

    def _device(self) -> torch.device:
        dev = self.q_down_proj.weight.device
        if dev.type != "cuda":
            raise RuntimeError("snapmind_b200 LookaheadSparseIndexer runs on a CUDA device; call .cuda() first")
        return dev

    def build_frozen_keys(self, key_states: dict[int, torch.Tensor], chunk_ids: list[int]) -> None:
        dev = self._device()
        for cid in chunk_ids:
            k = key_states.get(cid)
            if k is not None:
                self._frozen_keys[cid] = chunk_means(k.to(dev), self.kv_lora_rank)
        self._initialized = True

    def score(self, hidden_states: dict[int, torch.Tensor], chunk_ids: list[int]) -> dict[int, torch.Tensor]:
        if not self._initialized or not chunk_ids:
            return {cid: torch.tensor(0.5) for cid in chunk_ids}
        dev = self._device()
        available = [lid for lid in self.indexer_layers if lid in hidden_states]
        if not available:
            h = hidden_states[min(hidden_states.keys())].squeeze(0)
        else:
            h = torch.stack([hidden_states[lid].squeeze(0) for lid in available], dim=0).mean(dim=0)
        h = h.to(dev, self.q_down_proj.weight.dtype)
        batch_h = h.unsqueeze(0) if h.dim() == 1 else h
        with torch.no_grad():
            q = self.q_up_proj(self.q_down_proj(batch_h)).float().contiguous()
            w = self.w_proj(batch_h).float().contiguous()
        present = [cid for cid in chunk_ids if cid in self._frozen_keys]
        out: dict[int, torch.Tensor] = {}
        if present:
            keys = torch.cat([self._frozen_keys[cid].reshape(-1, self.kv_lora_rank) for cid in present]).contiguous()
            if keys.shape[0] != len(present):
                raise RuntimeError("frozen keys must be one row per chunk (2-D key states)")
            scores = torch.empty(len(present), dtype=torch.float32, device=dev)
            status = _lib.load().snapmind_indexer_score_ref(
                q.data_ptr(), w.data_ptr(), q.shape[0], self.n_indexer_heads, keys.data_ptr(), len(present),
                self.kv_lora_rank, scores.data_ptr(), _lib.stream_handle(dev))
            _lib.check(status, "LookaheadSparseIndexer.score")
            for i, cid in enumerate(present):
                out[cid] = scores[i]
        zero = torch.tensor(0.0, device=dev)
        return {cid: out.get(cid, zero) for cid in chunk_ids}


class ChunkSelector:
    """Top-k chunk selection over a paged MLA latent pool (block = chunk).

    keys[b, c] = W_k . mean(latent rows of chunk c)   (fp32, ``index_dim``)
    score[b, c] = sigmoid(q_b . keys[b, c] / sqrt(index_dim) + bias),  q_b = W_q . h_b
    """

    def __init__(self, pool, d_model: int, index_dim: int = 128, seed: int = 0, dtype=torch.bfloat16):
        self.pool = pool
        self.index_dim = index_dim
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.w_q = (torch.randn(index_dim, d_model, generator=g) * d_model ** -0.5).to(pool.device, dtype)
        self.w_k = (torch.randn(index_dim, pool.kv_lora_rank, generator=g) * pool.kv_lora_rank ** -0.5).to(
            pool.device, dtype)
        self.bias = float(torch.randn(1, generator=g).item() * 0.02)
        self.max_chunks = pool.max_blocks_per_seq
        self.keys = torch.zeros((pool.max_seqs, self.max_chunks, index_dim), dtype=torch.float32, device=pool.device)
        self._topk_ws: torch.Tensor | None = None
        self._pool_ws: torch.Tensor | None = None

    def update_keys(self, layer: int, chunk_begin: int, chunk_count: int, batch: int | None = None) -> None:
        """Pool + project chunks [chunk_begin, chunk_begin + chunk_count) of each sequence."""
        pool = self.pool
        batch = pool.max_seqs if batch is None else batch
        lib = _lib.load()
        need = lib.snapmind_indexer_pool_workspace_bytes(batch, chunk_count, pool.kv_lora_rank)
        if chunk_count * batch >= 1024:  # a bulk (re)build: room for the fp32 means
            if self._pool_ws is None or self._pool_ws.numel() < need:
                # room for a few more chunks per sequence, so growing sequences do not reallocate
                grow = lib.snapmind_indexer_pool_workspace_bytes(batch, chunk_count + 64, pool.kv_lora_rank)
                self._pool_ws = torch.empty(grow, dtype=torch.uint8, device=pool.device)
            ws, ws_bytes = self._pool_ws.data_ptr(), self._pool_ws.numel()
        else:
            ws, ws_bytes = None, 0
        status = lib.snapmind_indexer_pool_chunks(
            pool.latent[layer].data_ptr(), pool._dcode, pool.kv_lora_rank, pool.kv_lora_rank,
            pool.block_tables.data_ptr(), pool.max_blocks_per_seq, pool.max_blocks_per_seq,
            pool.seq_lens.data_ptr(), batch, pool.block_size, pool.num_blocks,
            chunk_begin, chunk_count, self.max_chunks,
            self.w_k.data_ptr(), _lib.dtype_code(self.w_k.dtype), self.index_dim,
            self.keys.data_ptr(), ws, ws_bytes, pool.err.data_ptr(), pool._stream(),
        )  # fmt: skip
        _lib.check(status, "ChunkSelector.update_keys")

    def query(self, hidden: torch.Tensor) -> torch.Tensor:
        """q [B, index_dim] fp32 = W_q . h for hidden [B, d_model] (one kernel, W_q read once)."""
        h = hidden.to(self.w_q.dtype).contiguous()
        out = torch.empty((h.shape[0], self.index_dim), dtype=torch.float32, device=h.device)
        status = _lib.load().snapmind_indexer_query(
            h.data_ptr(), self.w_q.data_ptr(), _lib.dtype_code(self.w_q.dtype), out.data_ptr(), h.shape[0],
            h.shape[1], self.index_dim, _lib.stream_handle(h.device))
        _lib.check(status, "ChunkSelector.query")
        return out

    def select(self, q: torch.Tensor, n_chunks: torch.Tensor | int, k: int = 32, all_scores: bool = False):
        """Top-k chunk ids (int32 [B, k], -1 past the valid chunks) and their scores."""
        batch = q.shape[0]
        idx = torch.empty((batch, k), dtype=torch.int32, device=q.device)
        sc = torch.empty((batch, k), dtype=torch.float32, device=q.device)
        full = torch.empty((batch, self.max_chunks), dtype=torch.float32, device=q.device) if all_scores else None
        nc_ptr, nc0 = (None, int(n_chunks)) if isinstance(n_chunks, int) else (n_chunks.data_ptr(), 0)
        lib = _lib.load()
        need = lib.snapmind_indexer_topk_workspace_bytes(batch, self.max_chunks, k)
        if self._topk_ws is None or self._topk_ws.numel() < need:
            self._topk_ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=q.device)  # left zeroed
        status = lib.snapmind_indexer_topk(
            q.data_ptr(), self.keys.data_ptr(), _lib.dtype_code(torch.float32), nc_ptr, nc0, batch,
            self.max_chunks, self.index_dim, self.index_dim ** -0.5, self.bias, k,
            idx.data_ptr(), sc.data_ptr(), None if full is None else full.data_ptr(),
            self._topk_ws.data_ptr(), self._topk_ws.numel(), _lib.stream_handle(q.device))
        _lib.check(status, "ChunkSelector.select")
        return (idx, sc, full) if all_scores else (idx, sc)
