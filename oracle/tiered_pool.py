"""Oracle: placement policy of the batched tiered pool (``snapmind_tiered_plan``).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The policy extends the reference tiered cache (snapmind/kv_cache/tiered.py:95-154:
fixed hot capacity, pinned sink chunk 0 and recent chunks, eviction of unpinned
chunks) to many sequences with least-recently-used eviction, as the benchmark
configuration asks; the reference has no LRU, so this restatement is the
specification the device kernel is checked against.
"""
from __future__ import annotations

import numpy as np


def chunk_pinned(c, length, chunk, sink, window):
    if sink > 0 and c == 0:
        return True
    if (c + 1) * chunk > length - window:
        return True
    return (c + 1) * chunk >= length


class TieredPoolOracle:
    def __init__(self, batch, max_chunks, n_slots, chunk, sink, window, stage_in_base, stage_out_base):
        self.batch, self.max_chunks, self.n_slots = batch, max_chunks, n_slots
        self.chunk, self.sink, self.window = chunk, sink, window
        self.stage_in_base, self.stage_out_base = stage_in_base, stage_out_base
        self.slot_owner = np.full(n_slots, -1, np.int64)
        self.slot_last = np.zeros(n_slots, np.int64)
        self.chunk_slot = np.full((batch, max_chunks), -1, np.int64)
        self.seq_lens = np.zeros(batch, np.int64)
        self.tables = np.zeros((batch, max_chunks), np.int64)
        self.table_lens = np.zeros(batch, np.int64)

    def step(self, step, n_new, requests):
        """One placement step; returns the copy plan [(src slot, dst slot)]."""
        cands = []
        for s in range(self.n_slots):
            owner = self.slot_owner[s]
            if owner < 0:
                cands.append((0, s))
            else:
                seq, c = owner >> 16, owner & 0xFFFF
                if not chunk_pinned(c, self.seq_lens[seq] + n_new, self.chunk, self.sink, self.window):
                    cands.append((1 + self.slot_last[s], s))
        cands.sort()
        order = [s for _, s in cands]
        nxt = [0]
        plan = []

        def take(seq, c):
            while nxt[0] < len(order):
                s = order[nxt[0]]
                nxt[0] += 1
                owner = self.slot_owner[s]
                if owner >= 0:
                    if self.slot_last[s] == step:
                        continue
                    self.chunk_slot[owner >> 16, owner & 0xFFFF] = -1
                self.slot_owner[s] = (seq << 16) | c
                self.slot_last[s] = step
                self.chunk_slot[seq, c] = s
                return s
            return -1

        ok = True
        for b in range(self.batch):
            old = int(self.seq_lens[b])
            new = old + n_new
            if old > 0 and old % self.chunk == 0 and n_new > 0:
                src = self.chunk_slot[b, old // self.chunk - 1]
                if src >= 0:
                    plan.append((int(src), self.stage_out_base + b))
            for c in range((old + self.chunk - 1) // self.chunk, (new + self.chunk - 1) // self.chunk):
                if take(b, c) < 0:
                    ok = False
            self.seq_lens[b] = new
        for i, (b, c) in enumerate(requests):
            if not (0 <= b < self.batch) or c < 0 or c >= self.max_chunks or c * self.chunk >= self.seq_lens[b]:
                continue
            cur = self.chunk_slot[b, c]
            if cur >= 0:
                self.slot_last[cur] = step
                continue
            s = take(b, c)
            if s < 0:
                ok = False
                continue
            plan.append((self.stage_in_base + i, s))
        for b in range(self.batch):
            length = self.seq_lens[b]
            nch = min(self.max_chunks, (length + self.chunk - 1) // self.chunk)
            res = [c for c in range(nch) if self.chunk_slot[b, c] >= 0]
            self.tables[b, : len(res)] = [self.chunk_slot[b, c] for c in res]
            self.table_lens[b] = sum(min(self.chunk, length - c * self.chunk) for c in res)
        return plan, ok
