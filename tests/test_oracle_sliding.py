"""The sliding-window oracle against the reference's own run (tests/golden/sliding_window.json):
with the reference's store (V built from the cached keys) it reproduces every
fetched tensor and memory_usage exactly."""
import json
from pathlib import Path

from inputs import digest
from make_golden import SLIDING_OPS, sliding_inputs
from oracle.sliding_window import SlidingWindowOracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "sliding_window.json"


def test_sliding_oracle_reproduces_reference():
    d = json.loads(GOLDEN.read_text())
    cfg = d["config"]
    o = SlidingWindowOracle(cfg["n_layers"], cfg["window_size"], v_from_cached_k=True)
    for op, rec in zip(SLIDING_OPS, d["steps"]):
        kind, layer, n, _ = op
        if kind == "store":
            k, v = sliding_inputs(op, cfg)
            o.store(layer, k, v)
        elif kind == "evict":
            o.evict(n)
        else:
            o.reset()
        assert o.memory_usage() == rec["memory_usage"]
        for i, lr in enumerate(rec["layers"]):
            k, v = o.fetch(i)
            assert list(k.shape) == lr["shape"]
            assert digest(k) == lr["k"] and digest(v) == lr["v"]
