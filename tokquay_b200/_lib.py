"""ctypes binding of ``libtokquay_b200.so`` (the C ABI in include/tokquay_b200.h).

The library is loaded once per process.  There is no fallback: if the shared
library is missing or fails to load, every paged operation raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_float, c_int, c_int32, c_int64, c_void_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtokquay_b200.so"

TQ_OK = 0
TQ_ERR_INVALID = 1
TQ_ERR_UNSUPPORTED = 2
TQ_ERR_CUDA = 3
TQ_ERR_CAPACITY = 4
TQ_ERR_DEVICE = 5

# tq_plan_layout indices
PLAN_NUM_TOKENS = 0
PLAN_NUM_SEQS = 1
PLAN_NUM_ITEMS = 2
PLAN_NUM_COMBINE = 3
PLAN_NUM_PARTIALS = 4
PLAN_TABLE_STRIDE = 5
PLAN_MAX_CTX = 6
PLAN_SPLIT_CHUNKS = 7
PLAN_TOTAL_INTS = 8
PLAN_OFF_COUNTS = 9
PLAN_OFF_SEQ_INFO = 10
PLAN_OFF_TABLES = 11
PLAN_OFF_SLOTS = 12
PLAN_OFF_POSITIONS = 13
PLAN_OFF_TOKEN_IDS = 14
PLAN_OFF_LAST_ROWS = 15
PLAN_OFF_ITEMS = 16
PLAN_OFF_COMBINE = 17
PLAN_NUM_CTAS = 18
PLAN_USED_INTS = 19
PLAN_NUM_TILE_CTAS = 20
PLAN_NUM_TILE_MERGES = 21
PLAN_LAYOUT_LEN = 22

# tq_paged_attention's with_tiles bits (enum tq_attn_tiles).
ATTN_TILES = 1
ATTN_TILE_MERGE = 2

# Symbols the header declares, with (restype, argtypes).
_P = c_void_p
SIGNATURES: dict[str, tuple] = {
    "tq_abi_version": (c_int, []),
    "tq_attention_chunk_keys": (c_int, []),
    "tq_attention_warps": (c_int, []),
    "tq_last_error": (ctypes.c_char_p, []),
    "tq_device_status": (c_int, [c_int, POINTER(c_int32)]),
    "tq_plan_step": (c_int, [c_int32, _P, _P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32,
                             c_int32, c_int32, _P, _P, c_int64, _P]),
    "tq_kv_write": (c_int, [_P, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32, _P, c_int64,
                            c_int64, c_int64, _P, _P, c_int32, _P]),
    "tq_qkv_bias_kv_write": (c_int, [_P, c_int64, _P, c_int32, c_int64, _P, _P, c_int64, c_int32, c_int32,
                                     c_int32, c_int32, c_int32, _P, _P, c_int32, _P]),
    "tq_plan_prompt_tiles": (c_int, [c_int32, c_int32, c_int32, c_int32]),
    "tq_paged_attention": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, c_int32, c_int32, c_int32,
                                   c_int32, c_int32, _P, c_int32, _P, c_int32, c_int32, _P, _P, _P, c_int32,
                                   c_float, _P]),
    "tq_paged_attention_noalloc": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, c_int32, c_int32, c_int32,
                                           c_int32, c_int32, _P, c_int32, _P, c_int32, c_int32, c_float,
                                           _P]),
    "tq_embed_layernorm": (c_int, [_P, _P, _P, _P, _P, _P, c_int32, c_int32, _P, _P, c_float,
                                   c_int32, _P, c_int32, _P]),
    "tq_bias_residual_layernorm": (c_int, [_P, _P, _P, c_int32, c_int64, _P, _P, _P, c_float, c_int32, _P,
                                           c_int32, _P]),
    "tq_argmax_rows": (c_int, [_P, c_int64, c_int32, _P, _P, c_int32, _P]),
    "tq_layernorm_rows": (c_int, [_P, _P, _P, _P, _P, c_float, c_int32, _P, c_int32, _P]),
    "tq_bias_gelu": (c_int, [_P, _P, c_int32, c_int64, _P, c_int32, c_int32, _P, c_int32, _P]),
    "tq_lm_head_argmax": (c_int, [_P, _P, _P, c_int64, _P, _P, _P, c_float, c_int32, _P, c_int64, c_int32,
                                  _P, _P, c_int32, _P]),
}

EXPECTED_ABI = 8

# tq_lm_head_argmax limits (TQ_LM_HEAD_* in include/tokquay_b200.h).
LM_HEAD_MAX_ROWS = 64
LM_HEAD_SLICE = 352
LM_HEAD_SCRATCH_BYTES = 520

# Split-K partials the no-allocation attention entry point can hold
# (TQ_NOALLOC_MAX_PARTIALS in include/tokquay_b200.h).
NOALLOC_MAX_PARTIALS = 32768

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


class NativeLibraryMissing(RuntimeError):
    """libtokquay_b200.so is not built or cannot be loaded; there is no fallback path."""


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with every signature declared."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path or os.environ.get("TOKQUAY_B200_LIB") or LIB_PATH)
        if not p.exists():
            raise NativeLibraryMissing(
                f"{p} is missing: build it with `python -m tokquay_b200.build` (needs nvcc); "
                "the paged forward has no CPU or PyTorch fallback"
            )
        try:
            lib = ctypes.CDLL(str(p))
        except OSError as e:
            raise NativeLibraryMissing(f"cannot load {p}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        abi = lib.tq_abi_version()
        if abi != EXPECTED_ABI:
            raise NativeLibraryMissing(f"{p} has ABI {abi}, this package needs {EXPECTED_ABI}")
        _lib = lib
        return lib


def function_address(name: str) -> int:
    """Address of an exported entry point (for native callers such as _hostpack)."""
    return ctypes.cast(getattr(load(), name), c_void_p).value


def last_error() -> str:
    msg = load().tq_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(status: int, what: str) -> None:
    """Raise for a nonzero status: ValueError for a rejected batch or argument
    (as the reference raises), RuntimeError for everything else."""
    if status == TQ_OK:
        return
    msg = last_error()
    if status == TQ_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(f"{what} failed (status {status}): {msg}")


def prompt_tiles(min_rows: int = -1, chunk_cost_pct: int = -1, item_cost_pct: int = -1,
                 max_pieces: int = -1) -> int:
    """Set the planner's prompt-tile knobs (tq_plan_prompt_tiles: sequences
    feeding at least ``min_rows`` tokens go to tensor-core tiles, 0 = never;
    a tile is cut into at most ``max_pieces`` pieces; negative arguments keep
    the current value); returns the previous min_rows."""
    return int(load().tq_plan_prompt_tiles(int(min_rows), int(chunk_cost_pct), int(item_cost_pct),
                                           int(max_pieces)))


def device_status(clear: bool = True) -> int:
    """Synchronise and return (optionally clearing) the device error word."""
    bits = c_int32(0)
    check(load().tq_device_status(int(clear), ctypes.byref(bits)), "tq_device_status")
    return bits.value
