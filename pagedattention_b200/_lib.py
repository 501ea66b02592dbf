"""ctypes binding of libpab200.so (the C ABI in include/pab200.h).

The library is loaded from this package directory (built in-tree by
``python -m pagedattention_b200.build``).  There is no fallback: if the
library is missing or fails to load, every decode call raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpab200.so"

ABI_VERSION = 1

# pab200_status
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_WORKSPACE = -3
ERR_ALIGNMENT = -4
ERR_CUDA = -5

# pab200_dtype
DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_F32 = 2

# pab200_layout
LAYOUT_PAGES = 0
LAYOUT_NHD = 1

# size of the fixed scratch of pab200_decode_noalloc
NOALLOC_SCRATCH_BYTES = 16 << 20

# device status bits
STATUS_BAD_PAGE_ID = 0x1
STATUS_SEQLEN_CLAMP = 0x2
STATUS_NEG_SEQLEN = 0x4
STATUS_WAIT_TIMEOUT = 0x8
STATUS_APPEND_FULL = 0x10

EXPORTED_SYMBOLS = (
    "pab200_decode_workspace_size",
    "pab200_decode_launch_count",
    "pab200_decode",
    "pab200_decode_noalloc",
    "pab200_paged_attention",
    "pab200_paged_attention_workspace_size",
    "pab200_merge_states",
    "pab200_kv_append",
    "pab200_decode_append",
    "pab200_exchange_buffer_bytes",
    "pab200_exchange_buffer_create",
    "pab200_exchange_buffer_open",
    "pab200_exchange_buffer_reset",
    "pab200_exchange_buffer_close",
    "pab200_exchange_buffer_destroy",
    "pab200_exchange_merge",
    "pab200_decode_exchange",
    "pab200_read_status",
    "pab200_strerror",
    "pab200_last_error",
    "pab200_abi_version",
)


class KvAppendArgs(ctypes.Structure):
    """Mirror of ``pab200_kv_append_args`` (field order and types must match)."""

    _fields_ = [
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("k_new", ctypes.c_void_p),
        ("v_new", ctypes.c_void_p),
        ("seqlens", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("layout", ctypes.c_int32),
        ("num_seqs", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_size", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("max_blocks", ctypes.c_int32),
        ("num_pages", ctypes.c_int64),
        ("new_stride_b", ctypes.c_int64),
        ("new_stride_h", ctypes.c_int64),
        ("seqlens_stride_b", ctypes.c_int64),
        ("seqlens_stride_h", ctypes.c_int64),
        ("bt_stride_b", ctypes.c_int64),
        ("bt_stride_h", ctypes.c_int64),
        ("bt_stride_i", ctypes.c_int64),
        ("bt_page_mul", ctypes.c_int32),
        ("bt_page_add", ctypes.c_int32),
        ("increment", ctypes.c_int32),
    ]


class DecodeArgs(ctypes.Structure):
    """Mirror of ``pab200_decode_args`` (field order and types must match)."""

    _fields_ = [
        ("out", ctypes.c_void_p),
        ("q", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("seqlens", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("layout", ctypes.c_int32),
        ("num_seqs", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_size", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("max_blocks", ctypes.c_int32),
        ("num_pages", ctypes.c_int64),
        ("q_stride_b", ctypes.c_int64),
        ("q_stride_h", ctypes.c_int64),
        ("out_stride_b", ctypes.c_int64),
        ("out_stride_h", ctypes.c_int64),
        ("seqlens_stride_b", ctypes.c_int64),
        ("seqlens_stride_h", ctypes.c_int64),
        ("bt_stride_b", ctypes.c_int64),
        ("bt_stride_h", ctypes.c_int64),
        ("bt_stride_i", ctypes.c_int64),
        ("bt_page_mul", ctypes.c_int32),
        ("bt_page_add", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float),
        ("num_splits", ctypes.c_int32),
        ("state_o", ctypes.c_void_p),
        ("state_lse", ctypes.c_void_p),
        ("event_before", ctypes.c_void_p),
        ("event_after", ctypes.c_void_p),
    ]


class LibraryNotBuilt(RuntimeError):
    pass


_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library, with argument types declared."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise LibraryNotBuilt(
            f"{LIB_PATH} is missing; build it with `python -m pagedattention_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    P = ctypes.POINTER(DecodeArgs)
    lib.pab200_decode_workspace_size.argtypes = [P]
    lib.pab200_decode_workspace_size.restype = ctypes.c_size_t
    lib.pab200_decode_launch_count.argtypes = [P]
    lib.pab200_decode_launch_count.restype = ctypes.c_int
    lib.pab200_decode.argtypes = [P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    # plain Python ints are accepted for the pointer and size arguments
    lib.pab200_decode.restype = ctypes.c_int
    lib.pab200_decode_noalloc.argtypes = [P, ctypes.c_void_p]
    lib.pab200_decode_noalloc.restype = ctypes.c_int
    lib.pab200_paged_attention.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.pab200_paged_attention.restype = ctypes.c_int
    lib.pab200_paged_attention_workspace_size.argtypes = [
        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_int64]
    lib.pab200_paged_attention_workspace_size.restype = ctypes.c_size_t
    lib.pab200_kv_append.argtypes = [ctypes.POINTER(KvAppendArgs), ctypes.c_void_p]
    lib.pab200_kv_append.restype = ctypes.c_int
    lib.pab200_decode_append.argtypes = [ctypes.POINTER(DecodeArgs), ctypes.POINTER(KvAppendArgs),
                                         ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.pab200_decode_append.restype = ctypes.c_int
    lib.pab200_merge_states.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
        ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
        ctypes.c_void_p]
    lib.pab200_merge_states.restype = ctypes.c_int
    lib.pab200_exchange_buffer_bytes.argtypes = [ctypes.c_int32, ctypes.c_int64, ctypes.c_int32]
    lib.pab200_exchange_buffer_bytes.restype = ctypes.c_size_t
    lib.pab200_exchange_buffer_create.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p),
                                                  ctypes.c_void_p]
    lib.pab200_exchange_buffer_open.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
    lib.pab200_exchange_buffer_reset.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.pab200_exchange_buffer_close.argtypes = [ctypes.c_void_p]
    lib.pab200_exchange_buffer_destroy.argtypes = [ctypes.c_void_p]
    for f in ("create", "open", "reset", "close", "destroy"):
        getattr(lib, "pab200_exchange_buffer_" + f).restype = ctypes.c_int
    lib.pab200_exchange_merge.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
        ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int64,
        ctypes.c_void_p, ctypes.c_void_p]
    lib.pab200_exchange_merge.restype = ctypes.c_int
    lib.pab200_decode_exchange.argtypes = [
        P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_void_p]
    lib.pab200_decode_exchange.restype = ctypes.c_int
    lib.pab200_read_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32),
                                       ctypes.c_void_p]
    lib.pab200_read_status.restype = ctypes.c_int
    lib.pab200_strerror.argtypes = [ctypes.c_int]
    lib.pab200_strerror.restype = ctypes.c_char_p
    lib.pab200_last_error.argtypes = []
    lib.pab200_last_error.restype = ctypes.c_char_p
    lib.pab200_abi_version.argtypes = []
    lib.pab200_abi_version.restype = ctypes.c_int
    ver = lib.pab200_abi_version()
    if ver != ABI_VERSION:
        raise RuntimeError(f"libpab200.so ABI {ver} != expected {ABI_VERSION}; rebuild it")
    _lib = lib
    return lib


def error_text(lib, rc: int) -> str:
    return f"{lib.pab200_strerror(rc).decode()}: {lib.pab200_last_error().decode()}"


def check(lib, rc: int, what: str) -> None:
    if rc != OK:
        raise RuntimeError(f"{what} failed ({rc}): {error_text(lib, rc)}")
