"""Registry semantics restated from snapmind/core/registry.py (mirrors snapmind/tests/test_registry.py)."""
import pytest

from snapmind_b200.registry import KV_CACHE, Registry, RegistryError


def test_register_create_get_list():
    r = Registry("thing", expected_type=object)

    @r.register("a")
    class A:
        def __init__(self, x=1):
            self.x = x

    assert "a" in r and r.list() == ["a"]
    assert r.create("a", x=3).x == 3
    assert r.get("a") is A


def test_duplicate_and_unknown_keys():
    r = Registry("thing", expected_type=object)
    r.register("a", int)
    with pytest.raises(RegistryError):
        r.register("a", float)
    r.register("a", float, override=True)
    assert r.get("a") is float
    with pytest.raises(RegistryError):
        r.create("zzz")
    with pytest.raises(RegistryError):
        r.get("zzz")


def test_type_check():
    class Base:
        pass

    r = Registry("typed", expected_type=Base)
    with pytest.raises(TypeError):
        r.register("x", int)


def test_b200_plugins_registered_under_reference_keys():
    import snapmind_b200  # noqa: F401

    assert "paged" in KV_CACHE
    from snapmind_b200.kv_cache.paged import PagedKVCache

    assert KV_CACHE.get("paged") is PagedKVCache
