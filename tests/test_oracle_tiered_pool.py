"""Properties of the tiered-pool placement policy (oracle), checked on CPU."""
import numpy as np

from oracle.tiered_pool import TieredPoolOracle, chunk_pinned


def test_policy_invariants_random_run():
    rng = np.random.RandomState(1)
    B, chunk, n_slots, sink, window = 4, 8, 30, 4, 24
    o = TieredPoolOracle(B, 200, n_slots, chunk, sink, window, stage_in_base=n_slots, stage_out_base=n_slots + 4)
    # sequences start empty; growth admits every new chunk
    for step in range(1, 300):
        reqs = []
        for _ in range(4):
            b = int(rng.randint(B))
            done = int(o.seq_lens[b]) // chunk
            if done > 1:
                reqs.append((b, int(rng.randint(0, done))))
        last_before = o.slot_last.copy()
        owner_before = o.slot_owner.copy()
        plan, ok = o.step(step, 1, reqs)
        assert ok
        # capacity and consistency
        res = np.argwhere(o.chunk_slot >= 0)
        assert len(res) <= n_slots
        for b, c in res:
            s = o.chunk_slot[b, c]
            assert o.slot_owner[s] == (b << 16) | c
        # pinned chunks of every sequence are resident
        for b in range(B):
            length = int(o.seq_lens[b])
            for c in range((length + chunk - 1) // chunk):
                if chunk_pinned(c, length, chunk, sink, window):
                    assert o.chunk_slot[b, c] >= 0, (step, b, c)
        # every evicted chunk was least recently used among the evictable ones
        evicted = [s for s in range(n_slots) if owner_before[s] >= 0 and o.slot_owner[s] != owner_before[s]]
        survivors = [t for t in range(n_slots) if owner_before[t] >= 0 and o.slot_owner[t] == owner_before[t]
                     and o.slot_last[t] != step
                     and not chunk_pinned(owner_before[t] & 0xFFFF, o.seq_lens[owner_before[t] >> 16], chunk,
                                          sink, window)]
        for s in evicted:
            for t in survivors:
                assert (last_before[s], s) < (last_before[t], t), (step, s, t)
        # table lengths count the resident tokens
        for b in range(B):
            length = int(o.seq_lens[b])
            want = sum(min(chunk, length - c * chunk) for c in range(o.max_chunks) if o.chunk_slot[b, c] >= 0)
            assert o.table_lens[b] == want


def test_requests_touch_resident_chunks_and_admit_cold_ones():
    o = TieredPoolOracle(1, 50, 6, 8, 4, 8, stage_in_base=6, stage_out_base=10)
    o.seq_lens[:] = [80]  # 10 chunks; pinned: 0 and 9 (window of 8 tokens)
    for c, s in ((0, 0), (9, 1), (3, 2), (4, 3)):
        o.slot_owner[s] = c
        o.chunk_slot[0, c] = s
    o.slot_last[:4] = [0, 0, 5, 7]
    plan, ok = o.step(10, 0, [(0, 4), (0, 6), (0, 7), (0, 8)])
    assert ok
    # chunk 4 touched; 6 and 7 take the free slots 4, 5; 8 evicts the LRU chunk 3 (slot 2)
    assert plan == [(6 + 1, 4), (6 + 2, 5), (6 + 3, 2)]
    assert o.chunk_slot[0, 3] == -1 and o.chunk_slot[0, 8] == 2 and o.slot_last[3] == 10
