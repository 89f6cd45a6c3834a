"""The oracle against the reference engine's indexer cadence (engine_indexer.json):
the tiered-cache oracle and the indexer oracle, driven through the engine's
_run_indexer step, reproduce every recorded re-page (scores, hot set, live contents)."""
import numpy as np
import pytest

from oracle import indexer as oidx
from oracle.tiered import TieredPagedKVCacheOracle
from replay import load_engine_indexer, replay_engine_indexer


class OracleIndexer:
    """oracle.indexer with the weights a seeded construction of the module gives
    (the B200 module creates the reference's layers in the reference's order)."""

    def __init__(self, case):
        import torch

        from snapmind_b200.indexer import LookaheadSparseIndexer

        torch.manual_seed(case["seed"])
        m = LookaheadSparseIndexer(d_model=case["indexer"]["d_model"], n_layers=24,
                                   kv_lora_rank=case["indexer"]["kv_lora_rank"])
        self.w = {n: getattr(m, n).weight.detach().double().numpy() for n in ("q_down_proj", "q_up_proj", "w_proj")}
        self.rank = case["indexer"]["kv_lora_rank"]
        self.frozen: dict[int, np.ndarray] = {}
        self.initialized = False

    def build_frozen_keys(self, key_states, chunk_ids):
        for c in chunk_ids:
            if c in key_states:
                self.frozen[c] = oidx.frozen_key(key_states[c], self.rank)
        self.initialized = True

    def score(self, hidden_states, chunk_ids):
        return oidx.score(hidden_states, chunk_ids, self.frozen, self.w, initialized=self.initialized)


@pytest.mark.parametrize("case", load_engine_indexer(), ids=lambda c: c["name"])
def test_oracle_replays_engine_indexer_cadence(case):
    cache = TieredPagedKVCacheOracle(**case["cache"])
    replay_engine_indexer(case, cache, OracleIndexer(case), to_input=lambda a: a, to_numpy=lambda a: a,
                          state_of=lambda c: (c.hot_set, c.chunks.keys(), c.total_tokens),
                          live_of=lambda c: c.live_dicts, score_tol=1e-5)


def test_engine_golden_exercises_the_policy():
    """The recorded cadence evicts and re-fetches chunks (not every re-page keeps
    everything hot), and the frozen-key cases score chunks on both sides of the threshold."""
    cases = {c["name"]: c for c in load_engine_indexer()}
    for name in ("engine_frozen_keys", "engine_frozen_keys_wide_pool"):
        c = cases[name]
        hot_sets = [tuple(r["hot"]) for r in c["records"]]
        assert len(set(hot_sets)) > 3
        below = sum(v < c["threshold"] for r in c["records"] for v in r["scores"].values())
        above = sum(v >= c["threshold"] for r in c["records"] for v in r["scores"].values())
        assert below > 10 and above > 10
        assert c["threshold_margin"] > 1e-3
