"""ctypes binding of the C ABI in include/flash_lab_b200.h (libflash_lab_b200.so, built in-tree
by flash-attention-lab_b200/build.py).

The structures below mirror flb_attn_params and flb_decode_params field for field; the library
allocates nothing, so every buffer passed here comes from the caller (PyTorch's allocator in
flash_lab.ops).
"""

from __future__ import annotations

import ctypes
import os
import pathlib

LIB_NAME = "libflash_lab_b200.so"
LIB_PATH = pathlib.Path(__file__).resolve().parent / LIB_NAME

FLB_OK = 0
FLB_ERR_INVALID_ARGUMENT = 1
FLB_ERR_UNSUPPORTED = 2
FLB_ERR_MISALIGNED = 3
FLB_ERR_CUDA = 4
FLB_ERR_WORKSPACE = 5
FLB_ERR_NO_DEVICE = 6

FLB_BF16 = 0
FLB_FP16 = 1
FLB_FP32 = 2

FLB_MAX_PEERS = 8

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32


class AttnParams(ctypes.Structure):
    _fields_ = [
        ("q", _p), ("k", _p), ("v", _p), ("o", _p), ("lse", _p),
        ("q_batch_stride", _i64), ("q_seq_stride", _i64), ("q_head_stride", _i64),
        ("k_batch_stride", _i64), ("k_seq_stride", _i64), ("k_head_stride", _i64),
        ("v_batch_stride", _i64), ("v_seq_stride", _i64), ("v_head_stride", _i64),
        ("o_batch_stride", _i64), ("o_seq_stride", _i64), ("o_head_stride", _i64),
        ("batch", _i32), ("seqlen_q", _i32), ("seqlen_k", _i32), ("heads", _i32),
        ("heads_kv", _i32), ("head_dim", _i32),
        ("causal", _i32), ("dtype", _i32), ("softmax_scale", ctypes.c_float),
        ("status", _p),
    ]


class DecodeParams(ctypes.Structure):
    _fields_ = [
        ("q", _p), ("k_cache", _p), ("v_cache", _p), ("o", _p), ("lse", _p), ("seq_lens", _p),
        ("q_batch_stride", _i64), ("q_head_stride", _i64),
        ("k_batch_stride", _i64), ("k_seq_stride", _i64), ("k_head_stride", _i64),
        ("v_batch_stride", _i64), ("v_seq_stride", _i64), ("v_head_stride", _i64),
        ("o_batch_stride", _i64), ("o_head_stride", _i64),
        ("batch", _i32), ("heads", _i32), ("heads_kv", _i32), ("head_dim", _i32),
        ("max_seqlen", _i32), ("num_splits", _i32), ("dtype", _i32),
        ("softmax_scale", ctypes.c_float),
        ("workspace", _p), ("workspace_bytes", ctypes.c_size_t),
        ("status", _p),
        ("block_tables", _p), ("block_table_stride", _i64),
        ("page_size", _i32), ("num_blocks", _i32),
    ]


class PeerExchange(ctypes.Structure):
    _fields_ = [
        ("world", _i32), ("rank", _i32),
        ("buffers", _p * FLB_MAX_PEERS),
        ("timeout_ns", _i64),
    ]


# Every symbol include/flash_lab_b200.h declares, with its ctypes signature.
SIGNATURES = {
    "flb_version": ([], ctypes.c_int),
    "flb_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "flb_last_error": ([], ctypes.c_char_p),
    "flb_prefill_fwd": ([ctypes.POINTER(AttnParams), _p], ctypes.c_int),
    "flb_decode_num_splits": ([_i32, _i32, _i32, _i32, _i32, _i32], ctypes.c_int),
    "flb_decode_workspace_bytes": ([_i32, _i32, _i32, _i32], ctypes.c_size_t),
    "flb_decode_fwd": ([ctypes.POINTER(DecodeParams), _p], ctypes.c_int),
    "flb_decode_partials": ([ctypes.POINTER(DecodeParams), _i32, _i32, _i32, _p, _p, _p],
                            ctypes.c_int),
    "flb_decode_merge": ([_p, _p, _i32, _i32, _i32, _i32, _i32, _p, _i64, _i64, _p, _p],
                         ctypes.c_int),
    "flb_selftest_umma": ([_p, _p, _p, _p, _p, _p, _p, _p], ctypes.c_int),
    "flb_decode_fwd_static": ([ctypes.POINTER(DecodeParams), _p], ctypes.c_int),
    "flb_decode_static_scratch_bytes": ([], ctypes.c_size_t),
    "flb_peer_handle_bytes": ([], ctypes.c_size_t),
    "flb_peer_alloc": ([ctypes.c_size_t, ctypes.POINTER(_p), _p], ctypes.c_int),
    "flb_peer_open": ([_p, ctypes.POINTER(_p)], ctypes.c_int),
    "flb_peer_close": ([_p], ctypes.c_int),
    "flb_peer_free": ([_p], ctypes.c_int),
    "flb_peer_exchange_bytes": ([_i32, _i32, _i32, _i32, _i32], ctypes.c_size_t),
    "flb_decode_partials_push": ([ctypes.POINTER(DecodeParams), _i32, _i32, _i32,
                                  ctypes.POINTER(PeerExchange), _p], ctypes.c_int),
    "flb_decode_merge_peers": ([ctypes.POINTER(PeerExchange), _i32, _i32, _i32, _i32, _i32, _p,
                                _i64, _i64, _p, _p, _p], ctypes.c_int),
    "flb_peer_exchange_reset": ([ctypes.POINTER(PeerExchange), _p], ctypes.c_int),
}

_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads the library once (raises OSError if it is missing or incomplete)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = os.environ.get("FLASH_LAB_LIBRARY", str(LIB_PATH))
    if not os.path.exists(path):
        raise OSError(f"{path} is not built (run flash-attention-lab_b200/build.py)")
    lib = ctypes.CDLL(path)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the build lacks a declared entry point
        fn.argtypes = args
        fn.restype = res
    _LIB = lib
    return lib


def error_message(lib: ctypes.CDLL, status: int) -> str:
    detail = lib.flb_last_error().decode(errors="replace")
    kind = lib.flb_status_string(status).decode(errors="replace")
    return f"{kind}: {detail}" if detail else kind
