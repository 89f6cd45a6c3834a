"""ctypes binding of ``libsnapmind_b200.so`` (the C ABI in ``include/snapmind_b200.h``).

The library is loaded lazily on first use.  There is no fallback: when the
library is missing, or CUDA is unavailable, every entry point raises.
Status codes map onto the exceptions the reference raises for the same
conditions (``RuntimeError("PagedKVCache: out of blocks")`` for pool exhaustion,
snapmind/kv_cache/paged.py:92-93).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libsnapmind_b200.so")
HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "snapmind_b200.h"

OK = 0
ERR_OUT_OF_BLOCKS = 1
ERR_BAD_ARGUMENT = 2
ERR_CUDA = 3
ERR_TIMEOUT = 4
ERR_UNSUPPORTED = 5

DEVERR_BLOCK_ID = 1
DEVERR_TABLE = 2
DEVERR_SPLIT = 4
DEVERR_OUT_OF_BLOCKS = 8
DEVERR_TIMEOUT = 16
DEVERR_POSITION = 32

DECODE_FORCE_GENERIC = 1

OUT_OF_BLOCKS_MSG = "PagedKVCache: out of blocks"

_DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_int = ctypes.c_int

# name -> (restype, argtypes); kept in the order of the header.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "snapmind_abi_version": (_int, []),
    "snapmind_last_error": (ctypes.c_char_p, []),
    "snapmind_kv_append": (
        _int,
        [_p, _p, _int, _i64, _p, _p, _int, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i32, _p, _i32,
         _i32, _i32, _i32, _i32, _i32, _i32, _i32, _p, _p],
    ),
    "snapmind_kv_gather": (
        _int,
        [_p, _p, _int, _i64, _p, _p, _i64, _i64, _p, _i64, _i64, _i32, _p, _i32, _i32, _i32, _i32, _i32,
         _i32, _i32, _p, _p],
    ),
    "snapmind_kv_copy_slots": (
        _int,
        [_p, _p, _int, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _p, _p],
    ),
    "snapmind_kv_reserve": (
        _int,
        [_p, _i64, _i32, _p, _i32, _i32, _i32, _p, _p, _i32, _p, _p],
    ),
    "snapmind_kv_release": (
        _int,
        [_p, _i64, _i32, _p, _p, _i32, _i32, _p, _p, _i32, _p, _p],
    ),
    "snapmind_kv_concat": (_int, [_p, _i32, _i32, _i32, _int, _p, _p, _i64, _p]),
    "snapmind_tiered_plan": (
        _int,
        [_p, _p, _p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _p, _p, _i32, _p, _p],
    ),
    "snapmind_tiered_move": (_int, [_p, _p, _i64, _i64, _i32, _p, _p, _i32, _p]),
    "snapmind_copy_2d": (_int, [_p, _i64, _p, _i64, _i64, _i64, _p]),
    "snapmind_indexer_pool_chunks": (
        _int,
        [_p, _int, _i64, _i32, _p, _i64, _i32, _p, _i32, _i32, _i32, _i32, _i32, _i32, _p, _int, _i32,
         _p, _p, _i64, _p, _p],
    ),
    "snapmind_indexer_pool_workspace_bytes": (_i64, [_i32, _i32, _i32]),
    "snapmind_rope_qk": (
        _int,
        [_p, _i64, _i64, _i64, _i32, _p, _i64, _i64, _i64, _i32, _int, _i32, _i32, _i32, _p, _p, _i64, _p, _i64,
         _p, _p],
    ),
    "snapmind_indexer_score_ref": (_int, [_p, _p, _i32, _i32, _p, _i32, _i32, _p, _p]),
    "snapmind_indexer_query": (_int, [_p, _p, _int, _p, _i32, _i32, _i32, _p]),
    "snapmind_indexer_topk": (
        _int,
        [_p, _p, _int, _p, _i32, _i32, _i32, _i32, _f32, _f32, _i32, _p, _p, _p, _p, _i64, _p],
    ),
    "snapmind_indexer_topk_workspace_bytes": (_i64, [_i32, _i32, _i32]),
    "snapmind_sparse_mla_default_splits": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "snapmind_sparse_mla_workspace_bytes": (_i64, [_i32, _i32, _i32, _i32]),
    "snapmind_sparse_mla_decode": (
        _int,
        [_p, _p, _int, _p, _p, _p, _i64, _i32, _p, _p, _i32, _i32, _i32, _f32, _i32, _i32, _i32, _i32,
         _i32, _i32, _i32, _p, _p, _i64, _p, _p],
    ),
    "snapmind_paged_gqa_decode_split_tokens": (_i32, [_i32, _i32, _i32, _i32]),
    "snapmind_paged_gqa_decode_workspace_bytes": (_i64, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "snapmind_paged_gqa_decode": (
        _int,
        [_p, _i64, _i64, _p, _p, _int, _p, _i64, _i32, _p, _p, _i64, _i64, _f32, _i32, _i32, _i32,
         _i32, _i32, _i32, _i32, _i32, _i32, _p, _i64, _p, _p],
    ),
    "snapmind_paged_gqa_decode_append": (
        _int,
        [_p, _i64, _i64, _p, _p, _int, _p, _i64, _i32, _p, _p, _p, _i64, _i64, _p, _i64, _i64, _f32, _i32,
         _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _p, _i64, _p, _p],
    ),
    "snapmind_paged_gqa_decode_window": (
        _int,
        [_p, _i64, _i64, _p, _p, _int, _p, _i64, _i32, _p, _p, _p, _i64, _i64, _f32, _i32, _i32, _i32,
         _i32, _i32, _i32, _i32, _i32, _i32, _p, _i64, _p, _p],
    ),
    "snapmind_paged_gqa_decode_peers": (
        _int,
        [_p, _i64, _i64, _p, _p, _int, _p, _i64, _i32, _p, _p, _p, _i32, _i32, _i64, _i64,
         _f32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _p, _i64, _p, _p],
    ),
    "snapmind_peer_sync": (_int, [_p, _p, _i32, _i32, _i32, _i32, _p, _p]),
    "snapmind_ipc_export": (_int, [_p, _p, ctypes.POINTER(_i64)]),
    "snapmind_ipc_open": (_int, [_p, _i64, ctypes.POINTER(_p)]),
    "snapmind_ipc_close": (_int, [_p, _i64]),
    "snapmind_paged_gqa_decode_noalloc": (
        _int,
        [_p, _i64, _i64, _p, _p, _int, _p, _i64, _i32, _p, _p, _i64, _i64, _f32, _i32, _i32, _i32,
         _i32, _i32, _i32, _i32, _i32, _i32, _p, _p],
    ),
}

NOALLOC_DECODE_SCRATCH_BYTES = 16 << 20
IPC_HANDLE_BYTES = 64
PEER_SIGNAL = 1
PEER_WAIT = 2

_lib: ctypes.CDLL | None = None


class SnapmindCudaError(RuntimeError):
    """A CUDA call inside the library failed."""


def load() -> ctypes.CDLL:
    """Load the shared library (once) and declare every entry point."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"snapmind_b200 CUDA library not built ({LIB_PATH}); run `python -m snapmind_b200.build`"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().snapmind_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    """Raise the exception matching a non-zero status."""
    if status == OK:
        return
    msg = last_error()
    if status == ERR_OUT_OF_BLOCKS:
        raise RuntimeError(OUT_OF_BLOCKS_MSG)
    if status == ERR_BAD_ARGUMENT:
        raise ValueError(f"{what}: {msg}")
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    if status == ERR_TIMEOUT:
        raise TimeoutError(f"{what}: {msg}")
    raise SnapmindCudaError(f"{what}: {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise TypeError(f"snapmind_b200: unsupported dtype {dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(device: torch.device) -> None:
    if device.type != "cuda":
        raise RuntimeError(f"snapmind_b200 runs on CUDA devices only (got {device})")
    if not torch.cuda.is_available():
        raise RuntimeError("snapmind_b200: CUDA is not available")


def raise_device_error(word: int, what: str) -> None:
    """Translate a non-zero device error word into an exception."""
    if word == 0:
        return
    if word & DEVERR_OUT_OF_BLOCKS:
        raise RuntimeError(OUT_OF_BLOCKS_MSG)
    parts = []
    if word & DEVERR_BLOCK_ID:
        parts.append("block id outside the pool")
    if word & DEVERR_TABLE:
        parts.append("logical block beyond the block table")
    if word & DEVERR_SPLIT:
        parts.append("sequence longer than the split plan")
    if word & DEVERR_TIMEOUT:
        parts.append("bounded device wait timed out")
    if word & DEVERR_POSITION:
        parts.append("rotary position outside the cos/sin tables")
    raise RuntimeError(f"{what}: device error 0x{word:x} ({', '.join(parts)})")


class DecodeWorkspace:
    """A reusable workspace for the paged GQA decode entry points.

    Its layout (set by the library) is the split tickets first -- one int32 per
    (row, kv head), which every call needs at zero and leaves at zero -- padded
    to 256 bytes, then the partial softmax states.  A call over fewer rows puts
    its partials where a later call over more rows keeps tickets, so the buffer
    tracks how long a prefix is known to be zero, and before a call whose
    tickets reach past it, clears that stretch on the current stream.
    """

    def __init__(self, device):
        self.device = device
        self.buf: torch.Tensor | None = None
        self.clean = 0  # leading bytes known to be zero

    def get(self, rows: int, n_kv_heads: int, need: int) -> torch.Tensor:
        import torch

        tickets = rows * n_kv_heads * 4
        if self.buf is None or self.buf.numel() < need:
            self.buf = torch.zeros(max(need, 256), dtype=torch.uint8, device=self.device)
            self.clean = self.buf.numel()
        if tickets > self.clean:
            self.buf[self.clean:tickets].zero_()
        # after this call: its tickets are zero again, its partials start past the padding
        self.clean = min(max(self.clean, tickets), (tickets + 255) // 256 * 256)
        return self.buf
