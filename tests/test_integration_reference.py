"""The B200 plugins as members of snapmind's own class hierarchy and registries.

Runs where the reference tree is present (it is read as a library, not run on
a GPU): every plugin must be a subclass of the reference contract it replaces
(snapmind/kv_cache/base.py:9, snapmind/layers/attention/base.py:9-22,
snapmind/layers/indexer/base.py:6-18), register into the reference's
``KV_CACHE`` / ``ATTENTION`` / ``INDEXER`` (snapmind/core/registry.py:92-111)
under the keys a snapmind config names, and accept every constructor argument
of the reference class it stands in for, with the same kind and default.
"""
import importlib
import inspect
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
REF = Path("/root/reference")

pytestmark = pytest.mark.skipif(not (REF / "snapmind").is_dir(), reason="the snapmind reference tree is not here")

# reference class each plugin stands in for
REFERENCE_CLASS = {
    "paged": "snapmind.kv_cache.paged:PagedKVCache",
    "tiered": "snapmind.kv_cache.tiered:TieredPagedKVCache",
    "sliding_window": "snapmind.kv_cache.sliding_window:SlidingWindowKVCache",
    "gqa_paged": "snapmind.layers.attention.gqa:GroupedQueryAttention",
    "lookahead_sparse": "snapmind.layers.indexer.lookahead:LookaheadSparseIndexer",
}
# defaults that differ on purpose: the tiered cache's home device is the GPU, not "cpu"
DEFAULT_DIFFERS = {("tiered", "device")}


def _load(path):
    module, name = path.split(":")
    return getattr(importlib.import_module(module), name)


def test_plugins_subclass_reference_contracts_when_imported_with_snapmind():
    """A fresh interpreter with snapmind importable: the plugins are real subclasses."""
    script = (
        "import json\n"
        "from snapmind_b200.integration import plugin_table, _contract\n"
        "from snapmind_b200.kv_cache.base import FROM_REFERENCE\n"
        "rows = {key: _contract(c) in cls.__mro__ for _, key, cls, c in plugin_table()}\n"
        "print(json.dumps({'from_reference': FROM_REFERENCE, 'rows': rows}))\n"
    )
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(REF), str(ROOT)]), PYTHONDONTWRITEBYTECODE="1")
    res = subprocess.run([sys.executable, "-c", script], env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    got = json.loads(res.stdout.strip().splitlines()[-1])
    assert got["from_reference"] is True
    assert got["rows"] == {key: True for key in REFERENCE_CLASS}, got


def test_register_with_snapmind(monkeypatch):
    monkeypatch.syspath_prepend(str(REF))
    monkeypatch.setenv("PYTHONDONTWRITEBYTECODE", "1")
    from snapmind_b200.integration import _contract, plugin_table, register_with_snapmind

    done = register_with_snapmind()
    registry = importlib.import_module("snapmind.core.registry")
    assert done == {"KV_CACHE": ["paged", "tiered", "sliding_window"], "ATTENTION": ["gqa_paged"],
                    "INDEXER": ["lookahead_sparse"]}
    for reg_name, key, cls, contract in plugin_table():
        reg = getattr(registry, reg_name)
        assert key in reg and reg.get(key) is cls, (reg_name, key)
        assert issubclass(cls, _contract(contract)), key
    # a reference module imported again registers nothing new, and the reference's
    # duplicate-key rule still holds for a caller that does not override
    importlib.import_module("snapmind.kv_cache.paged")
    assert registry.KV_CACHE.get("paged").__module__ == "snapmind_b200.kv_cache.paged"
    with pytest.raises(registry.RegistryError):
        register_with_snapmind(override=False)


@pytest.mark.parametrize("key", sorted(REFERENCE_CLASS))
def test_constructor_accepts_reference_arguments(monkeypatch, key):
    monkeypatch.syspath_prepend(str(REF))
    from snapmind_b200.integration import plugin_table

    ours = {k: cls for _, k, cls, _ in plugin_table()}[key]
    ref = _load(REFERENCE_CLASS[key])
    mine = inspect.signature(ours.__init__).parameters
    for name, p in inspect.signature(ref.__init__).parameters.items():
        assert name in mine, f"{key}: reference argument '{name}' missing"
        q = mine[name]
        assert q.kind == p.kind, f"{key}: '{name}' is {q.kind}, reference {p.kind}"
        if (key, name) not in DEFAULT_DIFFERS:
            assert q.default == p.default, f"{key}: '{name}' default {q.default!r}, reference {p.default!r}"
    # anything extra is keyword-only or defaulted, so reference call sites still bind
    extra = [n for n in mine if n not in inspect.signature(ref.__init__).parameters]
    for n in extra:
        q = mine[n]
        assert q.kind in (q.KEYWORD_ONLY, q.VAR_KEYWORD) or q.default is not q.empty, f"{key}: extra '{n}'"
