"""Device block bookkeeping shared by the batched paged pools.

Block tables (int32 ``[max_seqs][max_blocks_per_seq]``), sequence lengths and a
free-block stack all live on the GPU; ``snapmind_kv_reserve`` grows tables
deterministically (ascending sequence order, blocks from the top of the stack)
and ``snapmind_kv_release`` returns them.  Host mirrors of the lengths and the
free count let callers raise ``RuntimeError("PagedKVCache: out of blocks")``
before launching — the reference's error (snapmind/kv_cache/paged.py:92-93) —
and size outputs without a device sync.
"""
from __future__ import annotations

import numpy as np
import torch

from snapmind_b200 import _lib


class BlockPool:
    def __init__(self, num_blocks: int, max_seqs: int, max_blocks_per_seq: int, block_size: int,
                 device: torch.device | str | None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        _lib.require_cuda(self.device)
        _lib.load()
        self.num_blocks, self.max_seqs, self.block_size = num_blocks, max_seqs, block_size
        self.max_blocks_per_seq = max_blocks_per_seq
        self.block_tables = torch.zeros((max_seqs, max_blocks_per_seq), dtype=torch.int32, device=self.device)
        self.seq_lens = torch.zeros(max_seqs, dtype=torch.int32, device=self.device)
        # free_stack[top-1] is popped first; initially block 0, then 1, ...
        self.free_stack = torch.arange(num_blocks - 1, -1, -1, dtype=torch.int32, device=self.device)
        self.free_top = torch.tensor([num_blocks], dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._host_lens = np.zeros(max_seqs, dtype=np.int64)
        self._host_free = num_blocks

    def _stream(self) -> int:
        return _lib.stream_handle(self.device)

    @property
    def host_lens(self) -> np.ndarray:
        return self._host_lens

    def set_state(self, tables: np.ndarray, lens: np.ndarray, free_stack: np.ndarray) -> None:
        """Install block tables, lengths and the free stack (e.g. a shuffled pool)."""
        tables = np.asarray(tables)
        b, w = tables.shape
        if b > self.max_seqs or w > self.max_blocks_per_seq:
            raise ValueError("tables larger than the pool's table capacity")
        if tables.size and (tables.min() < 0 or tables.max() >= self.num_blocks):
            raise ValueError("block id outside the pool")
        full = np.zeros((self.max_seqs, self.max_blocks_per_seq), dtype=np.int32)
        full[:b, :w] = tables
        self.block_tables.copy_(torch.from_numpy(full))
        lens_full = np.zeros(self.max_seqs, dtype=np.int32)
        lens_full[: len(lens)] = lens
        self.seq_lens.copy_(torch.from_numpy(lens_full))
        self._host_lens = lens_full.astype(np.int64)
        fs = np.zeros(self.num_blocks, dtype=np.int32)
        fs[: len(free_stack)] = free_stack
        self.free_stack.copy_(torch.from_numpy(fs))
        self.free_top.fill_(len(free_stack))
        self._host_free = len(free_stack)

    def check(self) -> None:
        """Synchronise and raise if a kernel flagged an error on this pool."""
        word = int(self.err.item())
        if word:
            self.err.zero_()
            _lib.raise_device_error(word, type(self).__name__)

    def reserve(self, n_new: int = 1, batch: int | None = None) -> None:
        """Grow the first ``batch`` sequences by ``n_new`` tokens (tables + lengths)."""
        batch = self.max_seqs if batch is None else batch
        bs = self.block_size
        lens = self._host_lens[:batch]
        need = int(((lens + n_new + bs - 1) // bs - (lens + bs - 1) // bs).sum())
        if need > self._host_free:
            raise RuntimeError(_lib.OUT_OF_BLOCKS_MSG)
        if batch and int(((lens + n_new + bs - 1) // bs).max()) > self.max_blocks_per_seq:
            raise ValueError("sequence would outgrow its block table row")
        status = _lib.load().snapmind_kv_reserve(
            self.block_tables.data_ptr(), self.max_blocks_per_seq, self.max_blocks_per_seq,
            self.seq_lens.data_ptr(), batch, n_new, bs,
            self.free_stack.data_ptr(), self.free_top.data_ptr(), self.num_blocks,
            self.err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, f"{type(self).__name__}.reserve")
        self._host_lens[:batch] += n_new
        self._host_free -= need

    def blocks_needed(self, n_new: int, batch: int) -> int:
        """Blocks the first ``batch`` sequences take to grow by ``n_new`` tokens."""
        bs = self.block_size
        lens = self._host_lens[:batch]
        return int(((lens + n_new + bs - 1) // bs - (lens + bs - 1) // bs).sum())

    def reserve_device(self, n_new: int, batch: int) -> None:
        """The device part of ``reserve`` only (no host mirrors, no checks): a
        launch that a CUDA graph can replay.  The caller checks the capacity
        for all replays up front and accounts them with ``account_host``."""
        status = _lib.load().snapmind_kv_reserve(
            self.block_tables.data_ptr(), self.max_blocks_per_seq, self.max_blocks_per_seq,
            self.seq_lens.data_ptr(), batch, n_new, self.block_size,
            self.free_stack.data_ptr(), self.free_top.data_ptr(), self.num_blocks,
            self.err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, f"{type(self).__name__}.reserve_device")

    def account_host(self, n_new: int, batch: int) -> None:
        """Advance the host mirrors as ``reserve(n_new, batch)`` would."""
        need = self.blocks_needed(n_new, batch)
        self._host_lens[:batch] += n_new
        self._host_free -= need

    def release(self, seq_ids: list[int]) -> None:
        """Return the blocks of finished sequences to the free stack."""
        if not seq_ids:
            return
        if min(seq_ids) < 0 or max(seq_ids) >= self.max_seqs or len(set(seq_ids)) != len(seq_ids):
            raise ValueError("release: sequence ids must be distinct and inside the pool")
        ids = torch.tensor(seq_ids, dtype=torch.int32, device=self.device)
        freed = int(sum((self._host_lens[s] + self.block_size - 1) // self.block_size for s in seq_ids))
        status = _lib.load().snapmind_kv_release(
            self.block_tables.data_ptr(), self.max_blocks_per_seq, self.max_blocks_per_seq,
            self.seq_lens.data_ptr(), ids.data_ptr(), len(seq_ids), self.block_size,
            self.free_stack.data_ptr(), self.free_top.data_ptr(), self.num_blocks,
            self.err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, f"{type(self).__name__}.release")
        for s in seq_ids:
            self._host_lens[s] = 0
        self._host_free += freed

    def _slot_args(self, n_tokens: int, slot_starts, slot_start0):
        """(device starts pointer or None, scalar start) for an append of n_tokens."""
        if slot_starts is None:
            starts_ptr, start0 = self.seq_lens.data_ptr(), -n_tokens
        else:
            starts_ptr = None if isinstance(slot_starts, int) else slot_starts.data_ptr()
            start0 = slot_starts if isinstance(slot_starts, int) else 0
        if slot_start0 is not None:
            start0 = slot_start0
        return starts_ptr, start0
