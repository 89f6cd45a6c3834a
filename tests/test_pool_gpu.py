"""Batched paged pool (many sequences, one shuffled pool): reserve / append /
gather / release on the B200, bit-exact against the reference-generated fixture
and against the oracle."""
import numpy as np
import pytest
import torch

from inputs import digest, randn
from oracle import bf16, paged
from replay import load_paged_batched

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_batched_fixture_bit_exact(cuda_device):
    from snapmind_b200 import PagedKVPool

    g = load_paged_batched()
    c = g["config"]
    L, H, D, bs, nb = c["n_layers"], c["n_heads"], c["head_dim"], c["block_size"], c["num_blocks"]
    lens = np.array(g["lens"])
    tables = np.array(g["tables"])
    B = len(lens)
    pool = PagedKVPool(L, H, D, nb, max_seqs=B, max_blocks_per_seq=tables.shape[1], block_size=bs,
                       dtype=torch.bfloat16)
    pool.set_state(tables, lens, np.array(g["free_stack"]))
    recs = {(r["seq"], r["layer"]): r for r in g["fetch"]}
    for b, n in enumerate(lens):
        if n == 0:
            continue
        for l in range(L):
            k = torch.from_numpy(randn(recs[(b, l)]["seed"], (1, H, n, D))).cuda().to(torch.bfloat16)
            v = torch.from_numpy(randn(recs[(b, l)]["seed"] + 500, (1, H, n, D))).cuda().to(torch.bfloat16)
            _append_one(pool, l, b, k, v)
    pool.reserve(1, batch=B)
    ka = torch.stack([torch.stack([torch.from_numpy(randn(recs[(b, l)]["seed"] + 2000, (H, 1, D))) for b in range(B)]) for l in range(L)])
    va = torch.stack([torch.stack([torch.from_numpy(randn(recs[(b, l)]["seed"] + 2500, (H, 1, D))) for b in range(B)]) for l in range(L)])
    pool.append(None, ka.cuda().to(torch.bfloat16), va.cuda().to(torch.bfloat16))
    assert pool.block_tables[:B, : tables.shape[1]].cpu().numpy().tolist() == g["tables_after"]
    assert int(pool.free_top.item()) == g["free_top_after"]
    kg, vg = pool.gather(batch=B)
    pool.check()
    lens2 = lens + 1
    offs = np.concatenate([[0], np.cumsum(lens2)]) * H * D
    for r in g["fetch"]:
        b, l = r["seq"], r["layer"]
        k = kg[l, offs[b]:offs[b + 1]]
        v = vg[l, offs[b]:offs[b + 1]]
        assert digest(_bits(k)) == r["k_sha_bf16"], (b, l)
        assert digest(_bits(v)) == r["v_sha_bf16"], (b, l)
        assert digest(k.float().cpu().numpy()) == r["k_sha_f32"], (b, l)


def _append_one(pool, layer, b, k, v):
    """Prefill one sequence: write (1, H, n, D) rows at slots 0.. of sequence b."""
    from snapmind_b200 import _lib

    n = k.shape[2]
    st = k.stride()
    lib = _lib.load()
    rc = lib.snapmind_kv_append(
        pool.k[layer].data_ptr(), pool.v[layer].data_ptr(), pool._dcode, pool.layer_stride,
        k.data_ptr(), v.data_ptr(), _lib.dtype_code(k.dtype), 0, st[0], st[1], st[2],
        pool.block_tables[b].data_ptr(), pool.max_blocks_per_seq, 0, pool.max_blocks_per_seq,
        None, 0, 1, 1, n, pool.n_kv_heads, pool.head_dim, pool.block_size, pool.num_blocks,
        pool.err.data_ptr(), _lib.stream_handle(),
    )  # fmt: skip
    _lib.check(rc, "append")


@pytest.mark.parametrize(
    "dtype,H,D,bs",
    [(torch.bfloat16, 8, 128, 16), (torch.float32, 4, 64, 16), (torch.float16, 2, 24, 8), (torch.bfloat16, 3, 20, 32)],
)
def test_random_batched_matches_oracle(cuda_device, dtype, H, D, bs):
    from snapmind_b200 import PagedKVPool

    rng = np.random.RandomState(7)
    L, B = 3, 37
    lens = rng.randint(0, 9 * bs, size=B)
    lens[:3] = [0, bs, bs - 1]
    steps, T = 3, 2
    need = (lens + steps * T + bs - 1) // bs
    nb = int(need.sum() * 1.1) + 4
    perm = rng.permutation(nb).astype(np.int32)
    W = int(need.max()) + 1
    tables = np.zeros((B, W), np.int32)
    off = 0
    for b in range(B):
        k = (lens[b] + bs - 1) // bs
        tables[b, :k] = perm[off:off + k]
        off += k
    free = perm[off:]
    pool = PagedKVPool(L, H, D, nb, max_seqs=B, max_blocks_per_seq=W, block_size=bs, dtype=dtype)
    pool.k.zero_()
    pool.v.zero_()
    pool.set_state(tables, lens, free)
    kp = np.zeros((L, nb, H, bs, D), np.float32)
    vp = np.zeros_like(kp)
    rnd = {torch.float32: lambda a: a, torch.bfloat16: bf16.round_to_bf16,
           torch.float16: lambda a: a.astype(np.float16).astype(np.float32)}[dtype]
    o_tables, o_lens, o_top = tables.copy(), lens.copy(), len(free)
    for s in range(steps):
        pool.reserve(T, batch=B)
        o_tables, o_lens, o_top, err = paged.reserve(o_tables, o_lens, free, o_top, T, bs)
        assert err is None
        kn = randn(100 + s, (L, B, H, T, D))
        vn = randn(200 + s, (L, B, H, T, D))
        pool.append(None, torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda())
        paged.append(kp, vp, o_tables, o_lens - T, rnd(kn), rnd(vn), bs)
        assert np.array_equal(pool.block_tables.cpu().numpy(), o_tables)
        assert np.array_equal(pool.seq_lens.cpu().numpy(), o_lens)
        assert int(pool.free_top.item()) == o_top
    # the prefill rows were never written: compare only appended slots via a full gather of both
    # (the oracle pool starts at zero like the device pool)
    kg, vg = pool.gather(batch=B)
    ok, ov = paged.gather(kp, vp, o_tables, o_lens, bs)
    np.testing.assert_array_equal(kg.float().cpu().numpy(), ok)
    np.testing.assert_array_equal(vg.float().cpu().numpy(), ov)
    pool.check()


def test_reserve_out_of_blocks_and_release(cuda_device):
    from snapmind_b200 import PagedKVPool

    pool = PagedKVPool(1, 2, 64, num_blocks=5, max_seqs=3, max_blocks_per_seq=4, block_size=16,
                       dtype=torch.bfloat16)
    pool.reserve(16, batch=3)  # 3 blocks
    assert pool.block_tables[:, 0].cpu().tolist() == [0, 1, 2]
    with pytest.raises(RuntimeError, match="PagedKVCache: out of blocks"):
        pool.reserve(16, batch=3)  # needs 3, has 2
    assert int(pool.free_top.item()) == 2
    pool.release([1])
    assert int(pool.free_top.item()) == 3
    assert pool.seq_lens.cpu().tolist() == [16, 0, 16]
    pool.reserve(16, batch=3)
    # stack is [4, 3, 1] (1 just released): seq0 takes 1, seq1 takes 3, seq2 takes 4
    assert pool.block_tables[:, :2].cpu().tolist() == [[0, 1], [3, 0], [2, 4]]
    pool.check()


def test_device_error_word_flags_bad_block_ids(cuda_device):
    from snapmind_b200 import PagedKVPool

    pool = PagedKVPool(1, 1, 32, num_blocks=4, max_seqs=1, max_blocks_per_seq=2, block_size=16,
                       dtype=torch.float32)
    pool.block_tables.fill_(7)  # outside the pool: the kernels must skip and flag, not fault
    pool.seq_lens.fill_(20)
    pool._host_lens[:] = 20
    pool.gather(batch=1)
    with pytest.raises(RuntimeError, match="block id outside the pool"):
        pool.check()


@pytest.mark.parametrize("dtype,bs,split,force_generic", [
    (torch.bfloat16, 16, 0, False), (torch.bfloat16, 16, 64, False), (torch.bfloat16, 64, 128, False),
    (torch.float16, 32, 0, False), (torch.bfloat16, 16, 0, True), (torch.float32, 16, 0, False)])
def test_decode_with_append_equals_append_then_decode(cuda_device, dtype, bs, split, force_generic):
    """The fused store of this step's token (snapmind_paged_gqa_decode_append) leaves
    the pool with exactly the bytes the append kernel writes and gives exactly the
    output of append-then-decode, over steps that cross block and split boundaries;
    the reference store these replace is snapmind/kv_cache/paged.py:34-54."""
    from snapmind_b200 import PagedKVPool

    rng = np.random.RandomState(11)
    B, H, Hq, D = 7, 8, 32, 128
    lens = rng.randint(1, 300, size=B)
    lens[0] = 1  # a sequence whose first token arrives through the fused store
    lens[1] = bs * 4 - 1  # its next token starts a new block
    steps = 5
    nbs = (lens + steps + bs - 1) // bs
    nb = int(nbs.sum()) + 4
    perm = rng.permutation(nb).astype(np.int32)
    W = int(nbs.max())
    tables = np.zeros((B, W), np.int32)
    off = 0
    need = (lens + bs - 1) // bs
    for b in range(B):
        tables[b, : need[b]] = perm[off: off + need[b]]
        off += need[b]
    pools = []
    for _ in range(2):
        pool = PagedKVPool(1, H, D, nb, max_seqs=B, max_blocks_per_seq=W, block_size=bs, dtype=dtype)
        g = torch.Generator(device="cuda").manual_seed(5)
        pool.k.normal_(generator=g)
        pool.v.normal_(generator=g)
        pool.set_state(tables, lens, perm[off:])
        pools.append(pool)
    fused, ref = pools
    for step in range(steps):
        gen = torch.Generator(device="cuda").manual_seed(100 + step)
        q = torch.randn(B, Hq, D, device="cuda", generator=gen).to(dtype)
        kn = torch.randn(B, H, D, device="cuda", generator=gen).to(dtype)
        vn = torch.randn(B, H, D, device="cuda", generator=gen).to(dtype)
        max_len = int(lens.max()) + steps
        for pool in pools:
            pool.reserve(1, batch=B)
        want_out = None
        ref.append(0, kn, vn)
        want_out = ref.decode(0, q, split_tokens=split, force_generic=force_generic, max_seq_len=max_len)
        got_out = fused.decode(0, q, split_tokens=split, force_generic=force_generic, max_seq_len=max_len,
                               out=torch.empty_like(want_out), append=(kn, vn))
        torch.cuda.synchronize()
        fused.check()
        ref.check()
        assert torch.equal(fused.k, ref.k) and torch.equal(fused.v, ref.v), f"step {step}: pool bytes differ"
        assert torch.equal(got_out, want_out), f"step {step}: outputs differ"
    assert torch.equal(fused.block_tables, ref.block_tables)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_decode_layers_one_launch_equals_per_layer(cuda_device, dtype):
    """decode_layers (every layer in one launch over the layer-contiguous pool, row
    l * B + b = sequence b of layer l) equals the per-layer decode bit for bit under
    the same split plan, for contiguous queries and for a head slice of them."""
    from snapmind_b200 import PagedKVPool

    rng = np.random.RandomState(21)
    L, B, H, Hq, D, bs = 3, 5, 8, 32, 128, 16
    lens = rng.randint(1, 500, size=B)
    nbs = (lens + bs - 1) // bs
    nb = int(nbs.sum()) + 2
    perm = rng.permutation(nb).astype(np.int32)
    W = int(nbs.max())
    tables = np.zeros((B, W), np.int32)
    off = 0
    for b in range(B):
        tables[b, : nbs[b]] = perm[off: off + nbs[b]]
        off += nbs[b]
    pool = PagedKVPool(L, H, D, nb, max_seqs=B, max_blocks_per_seq=W, block_size=bs, dtype=dtype)
    g = torch.Generator(device="cuda").manual_seed(9)
    pool.k.normal_(generator=g)
    pool.v.normal_(generator=g)
    pool.set_state(tables, lens, perm[off:])
    q = torch.randn(L, B, Hq, D, device="cuda", generator=g).to(dtype)
    got = pool.decode_layers(q, split_tokens=64)
    want = torch.stack([pool.decode(layer, q[layer], split_tokens=64) for layer in range(L)])
    torch.cuda.synchronize()
    pool.check()
    assert torch.equal(got, want)
    # a strided view (rows of a wider tensor, as a head-sharded rank's query slice is)
    wide = torch.randn(L, B, 2 * Hq, D, device="cuda", generator=g).to(dtype)
    qv = wide[:, :, :Hq]
    got_v = pool.decode_layers(qv, split_tokens=64)
    want_v = torch.stack([pool.decode(layer, qv[layer], split_tokens=64) for layer in range(L)])
    torch.cuda.synchronize()
    assert torch.equal(got_v, want_v)


def test_decode_after_a_smaller_batch_keeps_tickets_zero(cuda_device):
    """The decode workspace holds split tickets for every (row, kv head) first and
    partials after them: a multi-split call over few rows writes partials where a
    later call over more rows keeps tickets.  The pool clears that stretch before
    the larger call, which must equal the same call on a fresh pool."""
    from snapmind_b200 import PagedKVPool

    rng = np.random.RandomState(31)
    B, H, Hq, D, bs = 15, 8, 32, 128, 16
    lens = rng.randint(200, 900, size=B)
    nbs = (lens + bs - 1) // bs
    nb = int(nbs.sum())
    perm = rng.permutation(nb).astype(np.int32)
    W = int(nbs.max())
    tables = np.zeros((B, W), np.int32)
    off = 0
    for b in range(B):
        tables[b, : nbs[b]] = perm[off: off + nbs[b]]
        off += nbs[b]
    pools = []
    for _ in range(2):
        pool = PagedKVPool(1, H, D, nb, max_seqs=B, max_blocks_per_seq=W, block_size=bs, dtype=torch.bfloat16)
        g = torch.Generator(device="cuda").manual_seed(3)
        pool.k.normal_(generator=g)
        pool.v.normal_(generator=g)
        pool.set_state(tables, lens, np.zeros(0, np.int32))
        pools.append(pool)
    used, fresh = pools
    q = torch.randn(B, Hq, D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(4)).to(torch.bfloat16)
    used.decode(0, q[:2], split_tokens=64)  # 2 rows, many splits: partials right after 16 ticket slots
    got = used.decode(0, q, split_tokens=64)
    want = fresh.decode(0, q, split_tokens=64)
    torch.cuda.synchronize()
    used.check()
    assert torch.equal(got, want)
