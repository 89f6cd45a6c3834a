"""The reference engine's indexer -> re-page cadence on the B200 plugins.

snapmind/engine/generate.py creates the indexer by registry key (:51) and, once
after the prompt and then every `indexer_interval` decode steps, scores the
completed chunks and re-pages the KV cache (:76-86, :107-114).  Here the
B200 "lookahead_sparse" indexer and the B200 "tiered" cache, created by key,
go through that cadence on the seeded token stream of engine_indexer.json;
after every re-page the scores, the hot set, the chunk ids and the bytes of
the live K/V dicts must equal the reference's record."""
import pytest
import torch

from replay import load_engine_indexer, replay_engine_indexer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", load_engine_indexer(), ids=lambda c: c["name"])
def test_engine_indexer_cadence_matches_reference(cuda_device, case):
    import snapmind_b200

    cache = snapmind_b200.KV_CACHE.create("tiered", **case["cache"], device="cuda")
    torch.manual_seed(case["seed"])  # same construction as the reference -> same weights
    indexer = snapmind_b200.INDEXER.create("lookahead_sparse", d_model=case["indexer"]["d_model"], n_layers=24,
                                           kv_lora_rank=case["indexer"]["kv_lora_rank"]).to("cuda")
    replay_engine_indexer(case, cache, indexer, to_input=lambda a: torch.from_numpy(a).cuda(),
                          to_numpy=lambda t: t.float().cpu().numpy(),
                          state_of=lambda c: (c._hot_set, c._chunks.keys(), c._total_tokens),
                          live_of=lambda c: c._live_dicts, score_tol=1e-5)
