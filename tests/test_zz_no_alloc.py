"""The allocation-free decode entry point, through the C ABI.

snapmind_paged_gqa_decode_noalloc serves callers that cannot allocate device
memory on the decode path (a foreign host bound through the C ABI without a
CUDA allocator of its own, or a serving loop that must not call cudaMalloc
between steps).  It keeps its scratch in a static device array shared by every
call, so these tests check that two calls in a row — the second one reusing
the scratch the first left behind — give exactly the output of the allocating
entry point (the same kernel and split plan, so bit for bit), that a smaller
call after a larger one is not disturbed by the larger call's leftovers, and
that an oversized call is refused.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _pool(seed=3, batch=24, dtype=torch.bfloat16):
    from snapmind_b200 import PagedKVPool

    rng = np.random.RandomState(seed)
    H, D, bs = 8, 128, 16
    lens = rng.randint(1, 2000, size=batch)
    nbs = (lens + bs - 1) // bs
    nb = int(nbs.sum() * 1.1) + 1
    perm = rng.permutation(nb).astype(np.int32)
    W = int(nbs.max())
    tables = np.zeros((batch, W), np.int32)
    off = 0
    for b in range(batch):
        tables[b, : nbs[b]] = perm[off : off + nbs[b]]
        off += nbs[b]
    pool = PagedKVPool(1, H, D, nb, max_seqs=batch, max_blocks_per_seq=W, block_size=bs, dtype=dtype)
    g = torch.Generator(device="cuda").manual_seed(seed)
    pool.k.normal_(generator=g)
    pool.v.normal_(generator=g)
    pool.set_state(tables, lens, perm[off:])
    return pool


def _noalloc(pool, q, out, split_tokens, max_seq_len):
    from snapmind_b200 import _lib

    lib = _lib.load()
    return lib.snapmind_paged_gqa_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1),
        pool.k[0].data_ptr(), pool.v[0].data_ptr(), _lib.dtype_code(pool.dtype),
        pool.block_tables.data_ptr(), pool.max_blocks_per_seq, pool.max_blocks_per_seq,
        pool.seq_lens.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        pool.head_dim ** -0.5, q.shape[0], q.shape[1], pool.n_kv_heads, pool.head_dim,
        pool.block_size, pool.num_blocks, max_seq_len, split_tokens, 0,
        pool.err.data_ptr(), _lib.stream_handle(),
    )  # fmt: skip


@pytest.mark.parametrize("split_tokens", [256, 0])
def test_noalloc_decode_matches_allocating_decode_twice(cuda_device, split_tokens):
    from snapmind_b200 import _lib

    pool = _pool()
    B, Hq, D = 24, 32, 128
    max_len = int(pool.host_lens[:B].max())
    for call in range(2):
        q = torch.randn(B, Hq, D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(call))
        q = q.to(torch.bfloat16)
        want = pool.decode(0, q, split_tokens=split_tokens, max_seq_len=max_len)
        got = torch.full_like(want, float("nan"))
        rc = _noalloc(pool, q, got, split_tokens, max_len)
        _lib.check(rc, "snapmind_paged_gqa_decode_noalloc")
        torch.cuda.synchronize()
        pool.check()
        assert torch.equal(got, want), f"call {call}: allocation-free output differs from the allocating decode"


def test_noalloc_decode_smaller_call_after_larger_call(cuda_device):
    """A larger call (more sequences, longer contexts, more splits) leaves tickets and
    partials in the shared scratch; the smaller call after it, and the larger one
    again after that, still equal the allocating decode bit for bit."""
    from snapmind_b200 import _lib

    big, small = _pool(seed=5, batch=24), _pool(seed=6, batch=5)
    for i, (pool, B, split) in enumerate(((big, 24, 64), (small, 5, 128), (big, 24, 64), (small, 5, 0))):
        max_len = int(pool.host_lens[:B].max())
        gen = torch.Generator(device="cuda").manual_seed(100 + i)
        q = torch.randn(B, 32, 128, device="cuda", generator=gen).to(torch.bfloat16)
        want = pool.decode(0, q, split_tokens=split, max_seq_len=max_len)
        got = torch.full_like(want, float("nan"))
        _lib.check(_noalloc(pool, q, got, split, max_len), "snapmind_paged_gqa_decode_noalloc")
        torch.cuda.synchronize()
        pool.check()
        assert torch.equal(got, want), f"call {i} (batch {B}): allocation-free output differs"


def test_noalloc_decode_rejects_oversized_scratch(cuda_device):
    from snapmind_b200 import _lib

    pool = _pool(batch=4)
    q = torch.zeros(4, 32, 128, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(q)
    # 4 x 32 heads x 8192 splits of 64 tokens x 520 B is far beyond the static scratch
    rc = _noalloc(pool, q, out, 64, 64 * 8192)
    assert rc == _lib.ERR_BAD_ARGUMENT
    msg = _lib.last_error()
    assert "static scratch" in msg and str(_lib.NOALLOC_DECODE_SCRATCH_BYTES) in msg
