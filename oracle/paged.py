"""Oracle: paged KV cache (snapmind/kv_cache/paged.py) restated on numpy arrays.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

``PagedKVCacheOracle`` is the single-sequence reference class, operation for
operation: the same free ``set`` with the same ``pop``/``add`` sequence, per-layer
block tables over that one set, the per-token store loop, the per-block fetch
concatenation and the evict compaction including its failure when the kept
tokens do not fit in the first kept block.  Its pool keeps the reference layout
``(max_blocks, block_size, n_heads, head_dim)``.

The batched functions restate the same slot arithmetic for many sequences over
the B200 pool layout ``pool[layer][block][head][slot][dim]``, plus the
deterministic device block reservation policy of ``snapmind_kv_reserve``.
"""
from __future__ import annotations

import numpy as np

OUT_OF_BLOCKS = "PagedKVCache: out of blocks"


class PagedKVCacheOracle:
    """snapmind/kv_cache/paged.py:9-145 on numpy (fp32 pool by default)."""

    def __init__(self, max_seq_len, n_layers, n_heads, head_dim, block_size=16, max_blocks=None,
                 dtype=np.float32):
        self.n_layers = n_layers
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.block_size = block_size
        max_blocks = max_blocks or (max_seq_len + block_size - 1) // block_size  # :24
        self.max_blocks = max_blocks
        shape = (max_blocks, block_size, n_heads, head_dim)  # :27
        self.k = np.zeros(shape, dtype=dtype)
        self.v = np.zeros(shape, dtype=dtype)
        self.free_blocks = set(range(max_blocks))  # :30
        self.block_tables: list[list[int]] = [[] for _ in range(n_layers)]
        self.slot_counts: list[int] = [0] * n_layers

    def store(self, layer_idx, key, value, seq_pos):  # :34-54
        num_tokens = key.shape[-2]
        slot_start = self.slot_counts[layer_idx]
        for offset in range(num_tokens):
            slot = slot_start + offset
            block_idx = slot // self.block_size
            within = slot % self.block_size
            bt = self.block_tables[layer_idx]
            while len(bt) <= block_idx:
                if not self.free_blocks:
                    raise RuntimeError(OUT_OF_BLOCKS)
                bt.append(self.free_blocks.pop())
            phys = bt[block_idx]
            self.k[phys, within] = key[0, :, offset, :]
            self.v[phys, within] = value[0, :, offset, :]
        self.slot_counts[layer_idx] = slot_start + num_tokens

    def fetch(self, layer_idx):  # :56-78
        bt = self.block_tables[layer_idx]
        if not bt:
            empty = np.empty((0, self.n_heads, self.head_dim), dtype=self.k.dtype)
            return empty, empty.copy()
        num_slots = self.slot_counts[layer_idx]
        blocks_needed = (num_slots + self.block_size - 1) // self.block_size
        k_parts, v_parts = [], []
        remaining = num_slots
        for b in bt[:blocks_needed]:
            take = min(remaining, self.block_size)
            k_parts.append(self.k[b, :take])
            v_parts.append(self.v[b, :take])
            remaining -= take
        if not k_parts:
            raise RuntimeError("torch.cat(): expected a non-empty list of Tensors")
        k = np.concatenate(k_parts, axis=0).transpose(1, 0, 2)[None]
        v = np.concatenate(v_parts, axis=0).transpose(1, 0, 2)[None]
        return np.ascontiguousarray(k), np.ascontiguousarray(v)

    def evict(self, tokens_to_keep):  # :80-116
        bs = self.block_size
        for layer_idx in range(self.n_layers):
            total = self.slot_counts[layer_idx]
            if total <= tokens_to_keep:
                continue
            start_slot = total - tokens_to_keep
            start_block = start_slot // bs
            offset_in_block = start_slot % bs
            bt = self.block_tables[layer_idx]
            blocks_needed = (offset_in_block + tokens_to_keep + bs - 1) // bs
            kept = bt[start_block:start_block + blocks_needed]
            freed = bt[:start_block] + bt[start_block + blocks_needed:]
            for b in freed:
                self.free_blocks.add(b)
            if offset_in_block > 0 and kept:
                first = kept[0]
                remaining = tokens_to_keep
                src_off, dst_off = offset_in_block, 0
                for b in kept:
                    take = min(bs - src_off, remaining)
                    # a slice of the block dimension is clipped at block_size; the
                    # reference's tensor assignment fails when it is shorter than src
                    dst_len = max(0, min(bs, dst_off + take) - min(bs, dst_off))
                    if dst_len != take:
                        raise RuntimeError(
                            f"The expanded size of the tensor ({dst_len}) must match the "
                            f"existing size ({take}) at non-singleton dimension 0."
                        )
                    src = self.k[b, src_off:src_off + take].copy()
                    self.k[first, dst_off:dst_off + take] = src
                    src = self.v[b, src_off:src_off + take].copy()
                    self.v[first, dst_off:dst_off + take] = src
                    dst_off += take
                    remaining -= take
                    src_off = 0
                needed = (dst_off + bs - 1) // bs
                for b in kept[needed:]:
                    self.free_blocks.add(b)
                kept = kept[:needed]
            self.block_tables[layer_idx] = kept
            self.slot_counts[layer_idx] = tokens_to_keep

    def reset(self):  # :118-123
        self.k[...] = 0
        self.v[...] = 0
        self.free_blocks = set(range(self.max_blocks))
        self.block_tables = [[] for _ in range(self.n_layers)]
        self.slot_counts = [0] * self.n_layers

    def memory_usage(self):  # :125-135
        total_bytes = self.k.size * self.k.itemsize + self.v.size * self.v.itemsize
        return {
            "num_tokens": sum(self.slot_counts),
            "total_bytes": total_bytes,
            "used_blocks": sum(len(bt) for bt in self.block_tables),
            "max_blocks": self.max_blocks,
        }

    def layer_dicts(self):  # :137-145
        out = {}
        for i in range(self.n_layers):
            k, v = self.fetch(i)
            out[i] = {"k": None, "v": None} if k.size == 0 else {"k": k, "v": v}
        return out


# ---------------------------------------------------------------------------
# batched forms over pool[layer][block][head][slot][dim]
# ---------------------------------------------------------------------------
def slot_location(tables_row, slot, block_size):
    """(physical block, row) of a logical slot — snapmind/kv_cache/paged.py:86-90,97."""
    return int(tables_row[slot // block_size]), slot % block_size


def append(k_pool, v_pool, tables, slot_starts, k_new, v_new, block_size):
    """Write k_new[l, b, h, t, :] to slot slot_starts[b] + t of sequence b, layer l.

    k_pool, v_pool: [L][num_blocks][H][bs][D] (modified in place);
    tables: [B][W] int; k_new, v_new: [L][B][H][T][D].
    """
    n_layers, batch, n_heads, n_tokens, _ = k_new.shape
    for b in range(batch):
        for t in range(n_tokens):
            phys, row = slot_location(tables[b], int(slot_starts[b]) + t, block_size)
            k_pool[:n_layers, phys, :, row, :] = k_new[:, b, :, t, :]
            v_pool[:n_layers, phys, :, row, :] = v_new[:, b, :, t, :]


def gather(k_pool, v_pool, tables, lens, block_size):
    """Per layer, the concatenation over b of (H, lens[b], D) — paged.py:103-125 per sequence."""
    outs_k, outs_v = [], []
    for layer in range(k_pool.shape[0]):
        ks, vs = [], []
        for b, n in enumerate(lens):
            n = int(n)
            nb = (n + block_size - 1) // block_size
            blocks = [int(x) for x in tables[b][:nb]]
            if n == 0:
                continue
            kc = np.concatenate([k_pool[layer, p] for p in blocks], axis=1)[:, :n]  # (H, n, D)
            vc = np.concatenate([v_pool[layer, p] for p in blocks], axis=1)[:, :n]
            ks.append(kc.reshape(-1))
            vs.append(vc.reshape(-1))
        outs_k.append(np.concatenate(ks) if ks else np.zeros(0, k_pool.dtype))
        outs_v.append(np.concatenate(vs) if vs else np.zeros(0, v_pool.dtype))
    return np.stack(outs_k), np.stack(outs_v)


def reserve(tables, lens, free_stack, free_top, n_new, block_size):
    """Deterministic batched block growth (policy of ``snapmind_kv_reserve``).

    Each sequence that needs new blocks for ``n_new`` more tokens takes them
    from the top of the free stack, sequences in ascending order, table entries
    in ascending order.  Returns (tables, lens, free_top, error) with copies;
    on error ("out_of_blocks" / "table") nothing changes.
    """
    tables = np.array(tables, copy=True)
    lens = np.array(lens, copy=True)
    need = []
    for b in range(len(lens)):
        have = (int(lens[b]) + block_size - 1) // block_size
        want = (int(lens[b]) + n_new + block_size - 1) // block_size
        if want > tables.shape[1]:
            return tables, np.array(lens), free_top, "table"
        need.append((have, want - have))
    total = sum(n for _, n in need)
    if total > free_top:
        return tables, lens, free_top, "out_of_blocks"
    taken = 0
    for b, (have, n) in enumerate(need):
        for k in range(n):
            tables[b, have + k] = free_stack[free_top - 1 - taken]
            taken += 1
        lens[b] += n_new
    return tables, lens, free_top - total, None
