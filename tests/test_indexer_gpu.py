"""Indexer, chunk selection and sparse MLA decode on the B200 against the
reference indexer (golden) and the oracle."""
import json

import numpy as np
import pytest
import torch

from inputs import randn
from oracle import bf16
from oracle import indexer as oidx
from oracle import mla as omla
from replay import GOLDEN
from test_oracle_golden import indexer_key_states

pytestmark = pytest.mark.gpu


def _cases():
    return json.loads((GOLDEN / "indexer.json").read_text())


@pytest.mark.parametrize("case", _cases(), ids=lambda m: m["name"])
def test_lookahead_indexer_matches_reference(cuda_device, case):
    from snapmind_b200.indexer import LookaheadSparseIndexer

    arrays = np.load(GOLDEN / "indexer.npz")
    dt = torch.bfloat16 if case["dtype"] == "bf16" else torch.float32
    torch.manual_seed(case["seed"])  # same construction as the reference -> same weights
    idx = LookaheadSparseIndexer(d_model=case["d_model"], n_layers=24, kv_lora_rank=case["kv_lora_rank"],
                                 n_indexer_heads=case["n_indexer_heads"]).to("cuda", dt)
    if case["weights_stored"]:
        for wname in ("q_down_proj", "q_up_proj", "w_proj"):
            np.testing.assert_array_equal(getattr(idx, wname).weight.detach().float().cpu().numpy(),
                                          arrays[f"{case['name']}__w_{wname}"])
    ks, hidden = indexer_key_states(case)
    ks_t = {c: torch.from_numpy(k).cuda().to(dt) for c, k in ks.items()}
    hid_t = {lid: torch.from_numpy(h).cuda().to(dt) for lid, h in hidden.items()}
    assert {c: float(v) for c, v in idx.score(hid_t, [0, 1]).items()} == {0: 0.5, 1: 0.5}
    idx.build_frozen_keys(ks_t, list(range(case["n_chunks"])))
    tol = 1e-6 if case["dtype"] == "f32" else 8e-3
    for c in ks:
        ref = arrays[f"{case['name']}__frozen_{c}"]
        ref = bf16.bf16_to_f32(ref) if case["dtype"] == "bf16" else ref
        np.testing.assert_allclose(idx._frozen_keys[c].cpu().numpy(), ref, rtol=tol, atol=tol)
    ids = [int(c) for c in case["scores"]]
    stol = 1e-5 if case["dtype"] == "f32" else 2e-2
    got = idx.score(hid_t, ids)
    for c in ids:
        assert float(got[c]) == pytest.approx(case["scores"][str(c)], abs=stol), c
    fb = idx.score({5: hid_t[5]}, ids)
    for c in ids:
        assert float(fb[c]) == pytest.approx(case["fallback_scores"][str(c)], abs=stol), c


def _latent_pool(B, lens, bs=64, R=512, P=64, seed=0, dtype=torch.bfloat16):
    """An MLALatentPool with seeded rows on shuffled blocks, plus the oracle copy."""
    from snapmind_b200.mla import MLALatentPool

    lens = np.asarray(lens)
    nbs = (lens + bs - 1) // bs
    nb = int(nbs.sum()) + 3
    perm = np.random.RandomState(seed).permutation(nb).astype(np.int32)
    W = int(nbs.max())
    tables = np.zeros((B, W), np.int32)
    off = 0
    for b in range(B):
        tables[b, : nbs[b]] = perm[off : off + nbs[b]]
        off += nbs[b]
    lat = bf16.round_to_bf16(randn(seed + 1, (nb, bs, R)))
    rope = bf16.round_to_bf16(randn(seed + 2, (nb, bs, P)))
    pool = MLALatentPool(1, nb, B, W, block_size=bs, kv_lora_rank=R, rope_dim=P, dtype=dtype)
    pool.latent[0, :, 0].copy_(torch.from_numpy(lat).to(dtype))
    pool.rope[0, :, 0].copy_(torch.from_numpy(rope).to(dtype))
    pool.set_state(tables, lens, perm[off:])
    return pool, lat, rope, tables


def _seq_rows(arr, tables, b, n, bs):
    blocks = [int(x) for x in tables[b][: (n + bs - 1) // bs]]
    return np.concatenate([arr[p] for p in blocks], axis=0)[:n] if n else arr[:0].reshape(0, arr.shape[-1])


def test_chunk_selector_keys_and_stable_topk(cuda_device):
    from snapmind_b200.indexer import ChunkSelector

    B, bs = 3, 64
    lens = [64 * 40 + 17, 64 * 3, 64 * 50]
    pool, lat, rope, tables = _latent_pool(B, lens, bs=bs, seed=5)
    sel = ChunkSelector(pool, d_model=256, index_dim=128, seed=1)
    n_chunks = [(n + bs - 1) // bs for n in lens]
    sel.update_keys(0, 0, max(n_chunks), batch=B)
    wk = sel.w_k.float().cpu().numpy().astype(np.float64)
    for b in range(B):
        rows = _seq_rows(lat, tables, b, lens[b], bs)
        for c in range(n_chunks[b]):
            want = wk @ rows[c * bs:(c + 1) * bs].astype(np.float64).mean(axis=0)
            np.testing.assert_allclose(sel.keys[b, c].cpu().numpy(), want, rtol=1e-4, atol=1e-4)
    hidden = torch.from_numpy(randn(9, (B, 256))).cuda()
    q = sel.query(hidden)
    nct = torch.tensor(n_chunks, dtype=torch.int32, device="cuda")
    idx, sc, full = sel.select(q, nct, k=32, all_scores=True)
    torch.cuda.synchronize()
    for b in range(B):
        s_all = full[b, : n_chunks[b]].cpu().numpy()
        # bit-exact: the stable descending order of the scores the kernel reports
        assert idx[b].cpu().numpy().tolist() == oidx.stable_topk(s_all, 32).tolist()
        want = oidx.sigmoid_scores(q[b].cpu().numpy(), sel.keys[b, : n_chunks[b]].cpu().numpy(),
                                   128 ** -0.5, sel.bias)
        np.testing.assert_allclose(s_all, want, rtol=1e-5, atol=1e-6)
        valid = idx[b][idx[b] >= 0].cpu().numpy()
        np.testing.assert_allclose(sc[b, : len(valid)].cpu().numpy(), s_all[valid], rtol=0, atol=0)


def test_chunk_keys_bulk_two_kernel_path(cuda_device):
    """A bulk key rebuild (>= 1024 chunks) goes through the mean + projection
    kernels with a workspace; ragged last chunks and chunks past a sequence's
    length (zeros) included.  Checked against the float64 mean and projection,
    and against the fused kernel (no workspace) on the same chunks."""
    from snapmind_b200 import _lib
    from snapmind_b200.indexer import ChunkSelector

    B, bs = 4, 64
    lens = [64 * 300, 64 * 299 + 5, 64 * 120 + 63, 64 * 250]
    pool, lat, rope, tables = _latent_pool(B, lens, bs=bs, seed=21)
    sel = ChunkSelector(pool, d_model=256, index_dim=128, seed=2)
    max_c = int(pool.max_blocks_per_seq)
    sel.update_keys(0, 0, max_c, batch=B)  # 4 x 301 chunks: two-kernel path
    assert sel._pool_ws is not None
    two = sel.keys.clone()
    # the fused kernel over the same chunks, through the ABI without a workspace
    fused = torch.zeros_like(sel.keys)
    rc = _lib.load().snapmind_indexer_pool_chunks(
        pool.latent[0].data_ptr(), pool._dcode, 512, 512, pool.block_tables.data_ptr(), max_c, max_c,
        pool.seq_lens.data_ptr(), B, bs, pool.num_blocks, 0, max_c, max_c, sel.w_k.data_ptr(),
        _lib.dtype_code(sel.w_k.dtype), 128, fused.data_ptr(), None, 0, pool.err.data_ptr(), _lib.stream_handle())
    _lib.check(rc, "pool fused")
    pool.check()
    wk = sel.w_k.float().cpu().numpy().astype(np.float64)
    two_np, fused_np = two.cpu().numpy(), fused.cpu().numpy()
    for b in range(B):
        n_chunks = (lens[b] + bs - 1) // bs
        rows = _seq_rows(lat, tables, b, lens[b], bs)
        for c in range(n_chunks):
            want = wk @ rows[c * bs:(c + 1) * bs].astype(np.float64).mean(axis=0)
            np.testing.assert_allclose(two_np[b, c], want, rtol=1e-4, atol=1e-4)
        assert not two_np[b, n_chunks:].any()
    # the bulk path projects on tensor cores with the means split into two bf16 terms
    np.testing.assert_allclose(two_np, fused_np, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("sliced", [False, True])
def test_topk_tie_break_on_equal_scores(cuda_device, sliced):
    from snapmind_b200 import _lib

    B, C, D, k = 2, 300, 8, 10
    keys = torch.zeros((B, C, D), device="cuda")
    keys[:, ::7, 0] = 1.0  # chunks 0, 7, 14, ... tie at the top score, the rest tie below
    q = torch.ones((B, D), device="cuda")
    idx = torch.empty((B, k), dtype=torch.int32, device="cuda")
    lib = _lib.load()
    ws = torch.zeros(lib.snapmind_indexer_topk_workspace_bytes(B, C, k), dtype=torch.uint8, device="cuda")
    rc = lib.snapmind_indexer_topk(q.data_ptr(), keys.data_ptr(), 0, None, C, B, C, D, 1.0, 0.0, k,
                                   idx.data_ptr(), None, None, ws.data_ptr() if sliced else None, ws.numel(),
                                   _lib.stream_handle())
    _lib.check(rc, "topk")
    want = [0, 7, 14, 21, 28, 35, 42, 49, 56, 63]
    assert idx.cpu().tolist() == [want, want]
    assert int(ws[: 4 * B].count_nonzero()) == 0  # tickets reset; candidates are scratch
    # only the chunks past 128 tie at the top: the winners come from later slices
    keys.zero_()
    keys[:, 130::9, 0] = 1.0
    rc = lib.snapmind_indexer_topk(q.data_ptr(), keys.data_ptr(), 0, None, C, B, C, D, 1.0, 0.0, k,
                                   idx.data_ptr(), None, None, ws.data_ptr() if sliced else None, ws.numel(),
                                   _lib.stream_handle())
    _lib.check(rc, "topk")
    want = list(range(130, 300, 9))[:k]
    assert idx.cpu().tolist() == [want, want]


@pytest.mark.parametrize("k,n_chunks", [(32, [2048, 1500, 7]), (200, [600, 129, 1000]), (5, [1, 0, 257]),
                                         (64, [5000, 4500, 10])])  # 40 slices: lanes merge two lists each
def test_topk_sliced_equals_single_cta(cuda_device, k, n_chunks):
    """Both kernels against the oracle's stable top-k of the scores, at sizes
    where slices, ragged lengths and k > 128 (all candidates kept) occur."""
    from snapmind_b200 import _lib

    B, C, D = len(n_chunks), 2050, 128
    g = torch.Generator(device="cpu").manual_seed(k)
    keys = torch.randn((B, C, D), generator=g).cuda()
    keys[0, 1000:1010] = keys[0, 999]  # exact ties across a slice boundary
    q = torch.randn((B, D), generator=g).cuda()
    nct = torch.tensor(n_chunks, dtype=torch.int32, device="cuda")
    lib = _lib.load()
    ws = torch.zeros(lib.snapmind_indexer_topk_workspace_bytes(B, C, k), dtype=torch.uint8, device="cuda")
    got = []
    for sliced in (False, True):
        idx = torch.empty((B, k), dtype=torch.int32, device="cuda")
        sc = torch.empty((B, k), dtype=torch.float32, device="cuda")
        full = torch.empty((B, C), dtype=torch.float32, device="cuda")
        rc = lib.snapmind_indexer_topk(q.data_ptr(), keys.data_ptr(), 0, nct.data_ptr(), 0, B, C, D, D ** -0.5, 0.1,
                                       k, idx.data_ptr(), sc.data_ptr(), full.data_ptr(),
                                       ws.data_ptr() if sliced else None, ws.numel(), _lib.stream_handle())
        _lib.check(rc, "topk")
        got.append((idx.cpu().numpy(), sc.cpu().numpy(), full.cpu().numpy()))
        for b in range(B):
            s_all = full[b, : n_chunks[b]].cpu().numpy()
            want = oidx.stable_topk(s_all, k).tolist()
            assert idx[b].cpu().numpy().tolist() == want
    assert (got[0][0] == got[1][0]).all()
    for b in range(B):
        np.testing.assert_array_equal(got[0][2][b, : n_chunks[b]], got[1][2][b, : n_chunks[b]])
    assert int(ws[: 4 * B].count_nonzero()) == 0  # tickets reset


@pytest.mark.parametrize("H", [32, 128])  # mma.sync kernel (32 heads), tcgen05 kernel (128 heads)
@pytest.mark.parametrize("sink,window,n_splits", [(4, 1024, 4), (0, 0, 1), (4, 200, 3), (70, 5000, 2),
                                                   (150, 100, 3), (130, 0, 2), (64, 64, 1)])  # sinks past chunk 0
def test_sparse_mla_decode_matches_oracle(cuda_device, sink, window, n_splits, H):
    B, R, P, bs, k = 4, 512, 64, 64, 8
    lens = [64 * 30 + 5, 700, 64 * 20, 1]
    pool, lat, rope, tables = _latent_pool(B, lens, bs=bs, seed=11)
    rng = np.random.RandomState(3)
    selected = np.full((B, k), -1, np.int32)
    for b in range(B):
        nc = (lens[b] + bs - 1) // bs
        picks = rng.randint(0, nc + 2, size=k - 2)  # some past the end, some repeated
        selected[b, : k - 2] = picks
    q_lat = bf16.round_to_bf16(randn(21, (B, H, R)) * 0.05)
    q_pe = bf16.round_to_bf16(randn(22, (B, H, P)) * 0.05)
    scale = (128 + 64) ** -0.5
    out = pool.sparse_decode(0, torch.from_numpy(q_lat).cuda().to(torch.bfloat16),
                             torch.from_numpy(q_pe).cuda().to(torch.bfloat16),
                             torch.from_numpy(selected).cuda(), sink=sink, window=window, scale=scale,
                             n_splits=n_splits)
    pool.check()
    got = out.float().cpu().numpy()
    for b in range(B):
        rows_c = _seq_rows(lat, tables, b, lens[b], bs)
        rows_p = _seq_rows(rope, tables, b, lens[b], bs)
        sel_b = [int(c) for c in selected[b] if 0 <= c < (lens[b] + bs - 1) // bs]
        pos = omla.sparse_positions(lens[b], sel_b, bs, sink, window)
        if len(pos) == 0:
            np.testing.assert_array_equal(got[b], 0)
            continue
        want = omla.sparse_mla_decode(q_lat[b], q_pe[b], rows_c, rows_p, pos, scale)
        np.testing.assert_allclose(got[b], want, rtol=2e-2, atol=2e-2)
    # the same call again reuses the workspace tickets
    out2 = pool.sparse_decode(0, torch.from_numpy(q_lat).cuda().to(torch.bfloat16),
                              torch.from_numpy(q_pe).cuda().to(torch.bfloat16),
                              torch.from_numpy(selected).cuda(), sink=sink, window=window, scale=scale,
                              n_splits=n_splits)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("R,P,dt", [(512, 64, torch.float32), (256, 32, torch.bfloat16)])
def test_sparse_mla_decode_cuda_core_path(cuda_device, R, P, dt):
    """Shapes the tensor-core kernel does not take (fp32, other widths) run the CUDA-core kernel."""
    B, H, bs, k = 3, 16, 64, 6
    lens = [64 * 12 + 9, 300, 64 * 5]
    pool, lat, rope, tables = _latent_pool(B, lens, bs=bs, R=R, P=P, seed=13, dtype=dt)
    rng = np.random.RandomState(4)
    selected = rng.randint(-1, 14, size=(B, k)).astype(np.int32)
    q_lat = bf16.round_to_bf16(randn(31, (B, H, R)) * 0.05)
    q_pe = bf16.round_to_bf16(randn(32, (B, H, P)) * 0.05)
    scale = (128 + 64) ** -0.5
    out = pool.sparse_decode(0, torch.from_numpy(q_lat).cuda().to(dt), torch.from_numpy(q_pe).cuda().to(dt),
                             torch.from_numpy(selected).cuda(), sink=4, window=128, scale=scale, n_splits=2)
    pool.check()
    got = out.float().cpu().numpy()
    tol = 1e-4 if dt == torch.float32 else 2e-2
    for b in range(B):
        sel_b = [int(c) for c in selected[b] if 0 <= c < (lens[b] + bs - 1) // bs]
        pos = omla.sparse_positions(lens[b], sel_b, bs, 4, 128)
        want = omla.sparse_mla_decode(q_lat[b], q_pe[b], _seq_rows(lat, tables, b, lens[b], bs),
                                      _seq_rows(rope, tables, b, lens[b], bs), pos, scale)
        np.testing.assert_allclose(got[b], want, rtol=tol, atol=tol)


@pytest.mark.parametrize("n_splits", [1, 3, None])
def test_sparse_mla_tcgen05_rising_scores_and_poisoned_slots(cuda_device, n_splits):
    """128 heads (tcgen05 kernel): scores that rise by ~40 in log2 units along the
    sequence for half of the heads (the reference maximum is raised and the
    output rescaled in TMEM several times) and fall for the other half (no
    rescale after the first tile), with NaN in every pool slot that holds no
    token (rows past each sequence's end and the spare blocks)."""
    B, H, R, P, bs = 2, 128, 512, 64, 64
    lens = [64 * 31 + 17, 64 * 12]
    pool, lat, rope, tables = _latent_pool(B, lens, bs=bs, seed=41)
    u = np.random.RandomState(5).standard_normal(R)
    u /= np.linalg.norm(u)
    nb = lat.shape[0]
    scale = (128 + 64) ** -0.5
    slope = 0.02 / (scale * 1.4426950408889634)  # q . k grows by 0.02 log2 units per position
    for b in range(B):
        for j, blk in enumerate(tables[b][: (lens[b] + bs - 1) // bs]):
            t = j * bs + np.arange(bs)
            lat[blk] = bf16.round_to_bf16(0.1 * lat[blk] + np.outer(slope * t, u).astype(np.float32))
    poison = np.zeros((nb, bs), bool)
    used = set()
    for b in range(B):
        nbk = (lens[b] + bs - 1) // bs
        used.update(int(x) for x in tables[b][:nbk])
        if lens[b] % bs:
            poison[tables[b][nbk - 1], lens[b] % bs:] = True
    for blk in range(nb):
        if blk not in used:
            poison[blk] = True
    lat_dev = lat.copy()
    rope_dev = rope.copy()
    lat_dev[poison] = np.nan
    rope_dev[poison] = np.nan
    pool.latent[0, :, 0].copy_(torch.from_numpy(lat_dev).to(torch.bfloat16))
    pool.rope[0, :, 0].copy_(torch.from_numpy(rope_dev).to(torch.bfloat16))
    sign = np.where(np.arange(H) % 2 == 0, 1.0, -1.0)[:, None]
    q_lat = bf16.round_to_bf16((sign * u[None, :] + 0.01 * randn(51, (B, H, R))).astype(np.float32))
    q_pe = bf16.round_to_bf16(randn(52, (B, H, P)) * 0.05)
    selected = np.array([[3, 9, 20, -1], [0, 5, 7, 11]], np.int32)
    kw = {} if n_splits is None else {"n_splits": n_splits}
    out = pool.sparse_decode(0, torch.from_numpy(q_lat).cuda().to(torch.bfloat16),
                             torch.from_numpy(q_pe).cuda().to(torch.bfloat16), torch.from_numpy(selected).cuda(),
                             sink=4, window=300, scale=scale, **kw)
    pool.check()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    for b in range(B):
        sel_b = [int(c) for c in selected[b] if 0 <= c < (lens[b] + bs - 1) // bs]
        pos = omla.sparse_positions(lens[b], sel_b, bs, 4, 300)
        want = omla.sparse_mla_decode(q_lat[b], q_pe[b], _seq_rows(lat, tables, b, lens[b], bs),
                                      _seq_rows(rope, tables, b, lens[b], bs), pos, scale)
        np.testing.assert_allclose(got[b], want, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("dt,batch,d_model,out_dim", [(torch.bfloat16, 8, 7168, 128), (torch.bfloat16, 37, 1000, 96),
                                                      (torch.float32, 5, 300, 128), (torch.float16, 17, 4100, 64)])
def test_indexer_query_matches_fp64_product(cuda_device, dt, batch, d_model, out_dim):
    """snapmind_indexer_query (the selector's W_q . h): 16-byte and scalar paths,
    more than 16 sequences (a second grid row), against the fp64 product of the
    same rounded inputs."""
    from snapmind_b200 import _lib

    g = torch.Generator(device="cpu").manual_seed(d_model + batch)
    h = torch.randn((batch, d_model), generator=g).to(dt)
    w = (torch.randn((out_dim, d_model), generator=g) * d_model ** -0.5).to(dt)
    out = torch.empty((batch, out_dim), dtype=torch.float32, device="cuda")
    hd, wd = h.cuda(), w.cuda()
    rc = _lib.load().snapmind_indexer_query(hd.data_ptr(), wd.data_ptr(), _lib.dtype_code(dt), out.data_ptr(), batch,
                                            d_model, out_dim, _lib.stream_handle())
    _lib.check(rc, "indexer_query")
    want = h.double() @ w.double().T
    np.testing.assert_allclose(out.cpu().double().numpy(), want.numpy(), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("n_splits", [1, 2, 5])
def test_sparse_mla_tcgen05_dtypes_and_splits(cuda_device, dt, n_splits):
    """128 heads on the tcgen05 kernel in both 16-bit types: every chunk scored by
    the two CTAs of a cluster (each over half of the 576 columns) and combined,
    at split counts that leave some splits with one chunk and some with none."""
    B, H, R, P, bs, k = 3, 128, 512, 64, 64, 6
    lens = [64 * 9 + 33, 64 * 2, 64 * 14]
    pool, lat, rope, tables = _latent_pool(B, lens, bs=bs, seed=61, dtype=dt)
    selected = np.array([[0, 3, 5, 8, -1, 2], [1, 1, 0, -1, -1, -1], [13, 2, 7, 9, 4, 11]], np.int32)
    q_lat = bf16.round_to_bf16(randn(62, (B, H, R)) * 0.05)
    q_pe = bf16.round_to_bf16(randn(63, (B, H, P)) * 0.05)
    scale = (128 + 64) ** -0.5
    out = pool.sparse_decode(0, torch.from_numpy(q_lat).cuda().to(dt), torch.from_numpy(q_pe).cuda().to(dt),
                             torch.from_numpy(selected).cuda(), sink=4, window=100, scale=scale, n_splits=n_splits)
    pool.check()
    got = out.float().cpu().numpy()
    for b in range(B):
        sel_b = [int(c) for c in selected[b] if 0 <= c < (lens[b] + bs - 1) // bs]
        pos = omla.sparse_positions(lens[b], sel_b, bs, 4, 100)
        want = omla.sparse_mla_decode(q_lat[b], q_pe[b], _seq_rows(lat, tables, b, lens[b], bs),
                                      _seq_rows(rope, tables, b, lens[b], bs), pos, scale)
        np.testing.assert_allclose(got[b], want, rtol=2e-2, atol=2e-2)


def test_sparse_mla_tcgen05_flags_block_outside_pool(cuda_device):
    """A table entry past the pool is skipped by the kernel (no load is issued for
    it) and reported through the device error word; the other sequence is
    unaffected."""
    B, H, R, P, bs = 2, 128, 512, 64, 64
    lens = [64 * 6, 64 * 5 + 3]
    pool, lat, rope, tables = _latent_pool(B, lens, bs=bs, seed=71)
    bad = pool.block_tables.clone()
    bad[0, 2] = pool.num_blocks + 5
    pool.block_tables.copy_(bad)
    q_lat = torch.from_numpy(bf16.round_to_bf16(randn(72, (B, H, R)) * 0.05)).cuda().to(torch.bfloat16)
    q_pe = torch.from_numpy(bf16.round_to_bf16(randn(73, (B, H, P)) * 0.05)).cuda().to(torch.bfloat16)
    selected = torch.tensor([[1, 2, 3], [0, 1, 2]], dtype=torch.int32, device="cuda")
    scale = (128 + 64) ** -0.5
    out = pool.sparse_decode(0, q_lat, q_pe, selected, sink=4, window=64, scale=scale, n_splits=2)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="block id outside the pool"):
        pool.check()
    pos = omla.sparse_positions(lens[1], [0, 1, 2], bs, 4, 64)
    want = omla.sparse_mla_decode(q_lat[1].float().cpu().numpy(), q_pe[1].float().cpu().numpy(),
                                  _seq_rows(lat, tables, 1, lens[1], bs), _seq_rows(rope, tables, 1, lens[1], bs),
                                  pos, scale)
    np.testing.assert_allclose(out[1].float().cpu().numpy(), want, rtol=2e-2, atol=2e-2)
