"""The tiered placement kernel (``snapmind_tiered_plan``) at large batches against
the oracle policy: more admissions in one launch than its shared-memory
admission log holds (lookups then read the chunk -> slot map back), requests for
chunks evicted, admitted or touched earlier in the same launch, and a batch
above the limit for staging the sequence lengths in shared memory."""
import ctypes

import numpy as np
import pytest
import torch

from oracle.tiered_pool import TieredPoolOracle

pytestmark = pytest.mark.gpu

CHUNK, SINK, WINDOW, N_SLOTS, N_REQ, MAX_CHUNKS = 64, 4, 64, 8192, 64, 8


def _oracle(batch, lens, resident, step, seed):
    """The pool state before the step: resident chunks in slots 0, 1, ... with seeded last uses."""
    rng = np.random.RandomState(seed)
    orc = TieredPoolOracle(batch, MAX_CHUNKS, N_SLOTS, CHUNK, SINK, WINDOW, N_SLOTS, N_SLOTS + N_REQ)
    s = 0
    for b in range(batch):
        for c in resident[b]:
            orc.slot_owner[s] = (b << 16) | c
            orc.slot_last[s] = rng.randint(0, step)
            orc.chunk_slot[b, c] = s
            s += 1
    orc.seq_lens[:] = lens
    assert s <= N_SLOTS
    return orc


def _run(batch, lens, resident, requests, step, seed):
    from snapmind_b200 import _lib

    orc = _oracle(batch, lens, resident, step, seed)

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).cuda()

    owner, last, cslot, slens = dev(orc.slot_owner), dev(orc.slot_last), dev(orc.chunk_slot), dev(orc.seq_lens)
    max_plan = batch + N_REQ
    tables = torch.zeros((batch, MAX_CHUNKS), dtype=torch.int32, device="cuda")
    tlens = torch.zeros(batch, dtype=torch.int32, device="cuda")
    plan = torch.zeros((max_plan, 2), dtype=torch.int32, device="cuda")
    count = torch.zeros(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    arr = ctypes.c_int32 * N_REQ
    rs, rc = arr(*[r[0] for r in requests]), arr(*[r[1] for r in requests])
    lib = _lib.load()
    status = lib.snapmind_tiered_plan(
        owner.data_ptr(), last.data_ptr(), cslot.data_ptr(), slens.data_ptr(), tables.data_ptr(), tlens.data_ptr(),
        plan.data_ptr(), count.data_ptr(), batch, MAX_CHUNKS, N_SLOTS, CHUNK, SINK, WINDOW, step, 1, N_SLOTS,
        N_SLOTS + N_REQ, max_plan, rs, rc, len(requests), err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(status, "tiered_plan")
    want_plan, ok = orc.step(step, 1, requests)
    torch.cuda.synchronize()
    assert ok and int(err.item()) == 0
    assert int(count.item()) == len(want_plan)
    assert plan[: len(want_plan)].cpu().numpy().tolist() == [list(p) for p in want_plan]
    assert np.array_equal(owner.cpu().numpy(), orc.slot_owner)
    assert np.array_equal(last.cpu().numpy(), orc.slot_last)
    assert np.array_equal(cslot.cpu().numpy(), orc.chunk_slot)
    assert np.array_equal(slens.cpu().numpy(), orc.seq_lens)
    assert np.array_equal(tlens.cpu().numpy(), orc.table_lens)
    t = tables.cpu().numpy()
    for b in range(batch):
        n = int((orc.chunk_slot[b] >= 0).sum())
        assert np.array_equal(t[b, :n], orc.tables[b, :n]), b
    return want_plan


def test_plan_admission_log_overflow(cuda_device):
    """2100 sequences cross into a new chunk at once: 2100 admissions (more than the
    2048 the log holds), 208 of them by LRU eviction of unpinned chunks, and 64
    requests for cold, just-evicted, just-admitted and resident chunks."""
    rng = np.random.RandomState(3)
    batch = 2100
    lens = np.full(batch, 5 * CHUNK)
    resident = [[0, 3, 4] for _ in range(batch)]  # chunk 3 is evictable after this step's growth
    kinds = [(1,), (2,), (3,), (4,), (5,), (0,), (6,)]  # cold, cold, maybe evicted, resident, admitted, sink, past the end
    requests = []
    seen = set()
    while len(requests) < N_REQ:
        b = int(rng.randint(0, batch))
        c = kinds[rng.randint(0, len(kinds))][0]
        if (b, c) not in seen:
            seen.add((b, c))
            requests.append((b, c))
    # chunks this step's growth evicts (a dry run of the policy without requests)
    dry = _oracle(batch, lens, resident, 100, 4)
    dry.step(100, 1, [])
    evicted = [b for b in range(batch) if dry.chunk_slot[b, 3] < 0]
    assert len(evicted) == 208
    requests[:8] = [(b, 3) for b in evicted[:8]]  # re-admitted in the same launch
    requests[-1] = (batch + 5, 1)  # out of range: skipped
    plan = _run(batch, lens, resident, requests, step=100, seed=4)
    assert len(plan) > batch  # every sequence's completed chunk written back, plus admitted requests


def test_plan_unstaged_batch(cuda_device):
    """4200 sequences (above the 4096 whose lengths are staged in shared memory): a
    third cross into a new chunk, 208 of them by evicting LRU unpinned chunks."""
    rng = np.random.RandomState(5)
    batch = 4200
    lens = np.where(np.arange(batch) % 3 == 0, 3 * CHUNK, 10)
    resident = [[0, 1, 2] if lens[b] == 3 * CHUNK else [0] for b in range(batch)]
    requests = [(int(b), int(c)) for b, c in zip(rng.choice(batch, N_REQ, replace=False), rng.randint(0, 4, N_REQ))]
    _run(batch, lens, resident, requests, step=60, seed=6)
