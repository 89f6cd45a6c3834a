"""Properties at the benchmark's full sizes, where the oracle cannot run the
whole workload in seconds.

* Paged GQA decode over the decode workload (128 sequences, contexts
  U[1024, 8192], 8 kv / 32 q heads, head_dim 128, block 16, bf16, shuffled
  blocks; one layer): the TMA / tensor-core kernel and the CUDA-core kernel
  agree on every sequence, and sampled sequences match the oracle.
* KV append / gather over the gather workload (64 sequences, contexts
  U[512, 4096]; two of its 32 layers): a gather returns exactly the stored
  rows, and one appended token lands last with everything before unchanged.
* MLA latent cache + indexer + sparse attention over the MLA workload (8
  sequences x 131072 tokens, 128 heads, rank 512, rope 64, chunk 64): the
  top-32 is the oracle's stable order of the kernel's own scores for every
  sequence, and the tcgen05 attention matches the oracle on sampled sequences.
"""
import numpy as np
import pytest
import torch

from oracle import gqa, indexer as oidx, mla as omla

pytestmark = pytest.mark.gpu


def _shuffled_tables(rng, lens, bs, slack_blocks=0):
    nbs = (np.asarray(lens) + bs - 1) // bs
    nb = int(nbs.sum()) + slack_blocks
    perm = rng.permutation(nb).astype(np.int32)
    tables = np.zeros((len(lens), int(nbs.max())), np.int32)
    off = 0
    for b, n in enumerate(nbs):
        tables[b, :n] = perm[off:off + n]
        off += n
    return nb, tables, perm[off:]


def _seq_rows(pool_layer, table_row, n):
    """[H, n, D] rows of one sequence from a pool layer [blocks, H, bs, D]."""
    blocks = pool_layer[torch.as_tensor(table_row, device=pool_layer.device, dtype=torch.long)]
    h, d = blocks.shape[1], blocks.shape[3]
    return blocks.permute(1, 0, 2, 3).reshape(h, -1, d)[:, :n]


def test_decode_full_workload(cuda_device):
    from snapmind_b200 import PagedKVPool

    rng = np.random.RandomState(2024)
    B, H, HQ, D, bs = 128, 8, 32, 128, 16
    lens = rng.randint(1024, 8193, size=B)
    nb, tables, free = _shuffled_tables(rng, lens, bs)
    pool = PagedKVPool(1, H, D, nb, B, tables.shape[1], block_size=bs, dtype=torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(7)
    pool.k.normal_(generator=g)
    pool.v.normal_(generator=g)
    pool.set_state(tables, lens, free)
    q = torch.randn((B, HQ, D), device="cuda", generator=g).to(torch.bfloat16)
    fast = pool.decode(0, q)
    generic = pool.decode(0, q, force_generic=True)
    torch.cuda.synchronize()
    pool.check()
    assert torch.isfinite(fast.float()).all()
    np.testing.assert_allclose(fast.float().cpu().numpy(), generic.float().cpu().numpy(), rtol=2e-2, atol=2e-2)
    for b in (int(np.argmin(lens)), int(np.argmax(lens)), 77):
        k = _seq_rows(pool.k[0], tables[b], int(lens[b])).float().cpu().numpy()
        v = _seq_rows(pool.v[0], tables[b], int(lens[b])).float().cpu().numpy()
        want = gqa.gqa_attention(q[b].float().cpu().numpy()[None, :, None], k[None], v[None], D ** -0.5)[0, :, 0]
        np.testing.assert_allclose(fast[b].float().cpu().numpy(), want, rtol=2e-2, atol=2e-2)


def test_append_gather_full_workload(cuda_device):
    from snapmind_b200 import PagedKVPool

    rng = np.random.RandomState(99)
    B, L, H, D, bs = 64, 2, 8, 128, 16
    lens = rng.randint(512, 4097, size=B)
    nb, tables, free = _shuffled_tables(rng, lens + 1, bs, slack_blocks=B)
    tables_now = np.where(np.arange(tables.shape[1])[None, :] < ((lens + bs - 1) // bs)[:, None], tables, 0)
    # blocks the next token needs come from the free stack: hand back the reserved ones
    extra = [tables[b, (lens[b] + bs - 1) // bs] for b in range(B) if lens[b] % bs == 0]
    free = np.concatenate([free, np.asarray(extra, np.int32)]).astype(np.int32)
    pool = PagedKVPool(L, H, D, nb, B, tables.shape[1], block_size=bs, dtype=torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(11)
    pool.k.normal_(generator=g)
    pool.v.normal_(generator=g)
    pool.set_state(tables_now, lens, free)

    def expected(pool_t, n_of):
        return torch.stack([
            torch.cat([_seq_rows(pool_t[layer], pool.block_tables[b].cpu().numpy(), int(n_of[b])).reshape(-1)
                       for b in range(B)])
            for layer in range(L)])

    k_out, v_out = pool.gather(B)
    torch.cuda.synchronize()
    pool.check()
    assert torch.equal(k_out, expected(pool.k, lens)) and torch.equal(v_out, expected(pool.v, lens))
    # one more token per sequence: reserve, append every layer, gather again
    before_k = [_seq_rows(pool.k[layer], tables_now[b], int(lens[b])).clone() for layer in range(L) for b in (0, B - 1)]
    pool.reserve(1, batch=B)
    k_new = torch.randn((L, B, H, D), device="cuda", generator=g).to(torch.bfloat16)
    v_new = torch.randn((L, B, H, D), device="cuda", generator=g).to(torch.bfloat16)
    for layer in range(L):
        pool.append(layer, k_new[layer], v_new[layer])
    k2, v2 = pool.gather(B)
    torch.cuda.synchronize()
    pool.check()
    lens2 = lens + 1
    assert torch.equal(k2, expected(pool.k, lens2)) and torch.equal(v2, expected(pool.v, lens2))
    table_rows = pool.block_tables.cpu().numpy()
    for layer in range(L):
        for b in range(B):
            rows_k = _seq_rows(pool.k[layer], table_rows[b], int(lens2[b]))
            rows_v = _seq_rows(pool.v[layer], table_rows[b], int(lens2[b]))
            assert torch.equal(rows_k[:, -1], k_new[layer, b]) and torch.equal(rows_v[:, -1], v_new[layer, b])
    i = 0
    for layer in range(L):
        for b in (0, B - 1):
            assert torch.equal(_seq_rows(pool.k[layer], table_rows[b], int(lens[b])), before_k[i])
            i += 1


def test_mla_indexer_sparse_attention_full_workload(cuda_device):
    from snapmind_b200.indexer import ChunkSelector
    from snapmind_b200.mla import MLALatentPool

    B, CTX, CH, R, P, HEADS, K = 8, 131072, 64, 512, 64, 128, 32
    n_ck = CTX // CH
    width = n_ck + 2
    nb = B * width
    pool = MLALatentPool(1, nb, B, width, block_size=CH, kv_lora_rank=R, rope_dim=P, dtype=torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(5)
    pool.latent.normal_(generator=g)
    pool.rope.normal_(generator=g)
    rng = np.random.RandomState(6)
    perm = rng.permutation(nb).astype(np.int32)
    tables = perm[: B * n_ck].reshape(B, n_ck)
    pool.set_state(tables, np.full(B, CTX), perm[B * n_ck:])
    sel = ChunkSelector(pool, d_model=7168, index_dim=128, seed=8)
    sel.update_keys(0, 0, n_ck, batch=B)
    hidden = torch.randn((B, 7168), device="cuda", generator=g).to(torch.bfloat16)
    n_chunks = torch.full((B,), n_ck, dtype=torch.int32, device="cuda")
    q = sel.query(hidden)
    idx, sc, full = sel.select(q, n_chunks, k=K, all_scores=True)
    q_lat = (torch.randn((B, HEADS, R), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    q_pe = (torch.randn((B, HEADS, P), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    scale = (128 + 64) ** -0.5
    out = pool.sparse_decode(0, q_lat, q_pe, idx, sink=4, window=1024, scale=scale)
    torch.cuda.synchronize()
    pool.check()
    idx_h = idx.cpu().numpy()
    for b in range(B):
        assert idx_h[b].tolist() == oidx.stable_topk(full[b, :n_ck].cpu().numpy(), K).tolist()
    lat0 = pool.latent[0, :, 0]  # [blocks, CH, R]
    rope0 = pool.rope[0, :, 0]
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    for b in (0, B - 1):
        pos = omla.sparse_positions(CTX, [int(c) for c in idx_h[b] if c >= 0], CH, 4, 1024)
        pos_t = torch.as_tensor(pos, device="cuda", dtype=torch.long)
        blk = torch.as_tensor(tables[b], device="cuda", dtype=torch.long)[pos_t // CH]
        rows_c = lat0[blk, pos_t % CH].float().cpu().numpy()
        rows_p = rope0[blk, pos_t % CH].float().cpu().numpy()
        want = omla.sparse_mla_decode(q_lat[b].float().cpu().numpy(), q_pe[b].float().cpu().numpy(), rows_c, rows_p,
                                      np.arange(len(pos)), scale)
        np.testing.assert_allclose(got[b], want, rtol=2e-2, atol=2e-2)
