"""The C-ABI library loads (no GPU needed) and exports exactly the declared entry points."""
import ctypes
import re
import subprocess

import pytest

import snapmind_b200._lib as lib

HEADER_SYMBOLS_RE = re.compile(r"SNAPMIND_API\s+[\w\s\*]+?\b(snapmind_\w+)\s*\(")


def header_symbols():
    syms = []
    for h in sorted(lib.HEADER_PATH.parent.glob("*.h")):
        syms += HEADER_SYMBOLS_RE.findall(h.read_text())
    return syms


def test_header_declares_symbols():
    syms = header_symbols()
    assert len(syms) == len(set(syms)) and len(syms) >= 8


def test_binding_matches_header():
    assert set(header_symbols()) == set(lib.SIGNATURES)


def test_library_loads_and_exports_every_symbol():
    l = lib.load()
    for name in header_symbols():
        assert hasattr(l, name), name
    assert l.snapmind_abi_version() >= 1


def test_exported_dynamic_symbols_are_exactly_the_header():
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib.LIB_PATH)], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("nm unavailable")
    exported = {ln.split()[-1] for ln in out.stdout.splitlines() if " T " in ln and "snapmind_" in ln}
    assert exported == set(header_symbols())


def test_host_side_argument_errors_need_no_gpu():
    l = lib.load()
    # null pointers / bad sizes are rejected before any CUDA call
    rc = l.snapmind_kv_gather(None, None, 7, 0, None, None, 0, 0, None, 0, 0, 0, None, 0, 1, 1, 1, 1, 16, 1, None, None)
    assert rc == lib.ERR_BAD_ARGUMENT
    assert "dtype" in lib.last_error()
    with pytest.raises(ValueError):
        lib.check(rc, "gather")
    rc = l.snapmind_paged_gqa_decode(None, 0, 0, None, None, 1, None, 0, 0, None, None, 0, 0, 1.0,
                                     1, 6, 4, 128, 16, 1, 0, 0, 0, None, 0, None, None)
    assert rc == lib.ERR_BAD_ARGUMENT and "multiple" in lib.last_error()
    # the peer decode: whole 16-byte vectors per peer store, at least one peer
    peers_args = lambda n_peers, stride_head: l.snapmind_paged_gqa_decode_peers(
        None, 0, 0, None, None, 1, None, 0, 0, None, None, 8, n_peers, 0, 8 * 128, stride_head, 1.0,
        1, 8, 8, 128, 16, 1, 0, 0, 0, None, 0, None, None)
    assert peers_args(0, 128) == lib.ERR_BAD_ARGUMENT and "peer" in lib.last_error()
    assert peers_args(2, 100) == lib.ERR_BAD_ARGUMENT and "16 bytes" in lib.last_error()
    # the flag sync: rank inside the peers, a positive epoch, the arrays the mode needs
    assert l.snapmind_peer_sync(None, None, 2, 2, 1, lib.PEER_WAIT, None, None) == lib.ERR_BAD_ARGUMENT
    assert l.snapmind_peer_sync(None, None, 2, 0, 0, lib.PEER_WAIT, None, None) == lib.ERR_BAD_ARGUMENT
    assert l.snapmind_peer_sync(None, None, 2, 0, 1, lib.PEER_SIGNAL, None, None) == lib.ERR_BAD_ARGUMENT
    assert l.snapmind_peer_sync(None, None, 2, 0, 1, lib.PEER_WAIT, None, None) == lib.ERR_BAD_ARGUMENT
    off = ctypes.c_int64(0)
    assert l.snapmind_ipc_export(None, None, ctypes.byref(off)) == lib.ERR_BAD_ARGUMENT


def test_workspace_size_formula():
    l = lib.load()
    n = l.snapmind_paged_gqa_decode_workspace_bytes(128, 32, 8, 128, 8192, 512)
    counters = (128 * 8 * 4 + 255) // 256 * 256
    assert n == counters + 128 * 32 * 16 * 130 * 4
    assert l.snapmind_paged_gqa_decode_split_tokens(128, 8, 8192, 16) % 64 == 0
