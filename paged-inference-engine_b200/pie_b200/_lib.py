"""ctypes binding of libpaged_attn_b200.so (the C ABI in include/paged_attn_b200.h).

The shared library is built in-tree by ``paged-inference-engine_b200/build.py``
and loaded from this directory.  There is no fallback: if the library is
missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpaged_attn_b200.so")

PA_DTYPE_F16 = 0
PA_DTYPE_BF16 = 1
PA_DTYPE_I8 = 2
PA_DTYPE_F32 = 3

PA_OK = 0
PA_ERR_INVALID = -1
PA_ERR_UNSUPPORTED = -2
PA_ERR_WORKSPACE = -3
PA_ERR_CUDA = -4

PA_STATUS_BAD_BLOCK_ID = 1
PA_STATUS_BAD_POSITION = 2
PA_STATUS_BAD_NUM_BLOCKS = 4
PA_STATUS_BAD_SEQ_INDEX = 8
PA_STATUS_PEER_TIMEOUT = 32

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64


class PaKvCache(ctypes.Structure):
    """Mirror of pa_kv_cache_t."""

    _fields_ = [
        ("k", _vp), ("v", _vp),
        ("dtype", _i32), ("num_blocks", _i32), ("block_size", _i32), ("num_kv_heads", _i32),
        ("head_dim", _i32), ("scale_dtype", _i32),
        ("k_stride_block", _i64), ("k_stride_slot", _i64), ("k_stride_head", _i64),
        ("v_stride_block", _i64), ("v_stride_slot", _i64), ("v_stride_head", _i64),
        ("k_scale", _vp), ("v_scale", _vp),
        ("ks_stride_block", _i64), ("ks_stride_slot", _i64), ("ks_stride_head", _i64),
        ("vs_stride_block", _i64), ("vs_stride_slot", _i64), ("vs_stride_head", _i64),
    ]


class PaPaging(ctypes.Structure):
    """Mirror of pa_paging_t."""

    _fields_ = [
        ("block_table", _vp), ("bt_stride_seq", _i64), ("bt_stride_col", _i64),
        ("bt_cols", _i32), ("num_seqs", _i32),
        ("num_blocks_per_seq", _vp), ("q_len_per_seq", _vp), ("kv_len_per_seq", _vp),
    ]


class PaAttnIO(ctypes.Structure):
    """Mirror of pa_attn_io_t."""

    _fields_ = [
        ("q", _vp), ("q_dtype", _i32), ("num_q_heads", _i32), ("max_q_len", _i32), ("causal_top_left", _i32),
        ("q_stride_seq", _i64), ("q_stride_head", _i64), ("q_stride_row", _i64),
        ("o", _vp), ("o_stride_seq", _i64), ("o_stride_head", _i64), ("o_stride_row", _i64),
        ("lse", _vp), ("l_stride_seq", _i64), ("l_stride_head", _i64), ("l_stride_row", _i64),
        ("softmax_scale", ctypes.c_float), ("_reserved", _i32),
    ]


class PaKvNew(ctypes.Structure):
    """Mirror of pa_kv_new_t."""

    _fields_ = [
        ("k_new", _vp), ("v_new", _vp), ("dtype", _i32), ("num_tokens", _i32),
        ("k_stride_token", _i64), ("k_stride_head", _i64), ("v_stride_token", _i64), ("v_stride_head", _i64),
        ("seq_index", _vp), ("positions", _vp),
    ]


class PaKvProj(ctypes.Structure):
    """Mirror of pa_kv_proj_t."""

    _fields_ = [
        ("x", _vp), ("w", _vp), ("bias", _vp), ("x_stride", _i64), ("w_stride", _i64), ("dtype", _i32),
        ("num_tokens", _i32), ("d_model", _i32), ("_reserved", _i32), ("seq_index", _vp), ("positions", _vp),
    ]


# name -> (restype, argtypes); every symbol include/paged_attn_b200.h declares.
SIGNATURES = {
    "paged_attn_workspace_size": (ctypes.c_int, [ctypes.POINTER(PaAttnIO), ctypes.POINTER(PaKvCache),
                                                 ctypes.POINTER(PaPaging), ctypes.POINTER(ctypes.c_size_t)]),
    "paged_attn_forward": (ctypes.c_int, [ctypes.POINTER(PaAttnIO), ctypes.POINTER(PaKvCache),
                                          ctypes.POINTER(PaPaging), _vp, ctypes.c_size_t, _vp, _vp]),
    "paged_attn_decode": (ctypes.c_int, [ctypes.POINTER(PaAttnIO), ctypes.POINTER(PaKvCache),
                                         ctypes.POINTER(PaPaging), _vp, ctypes.c_size_t, _vp, _vp]),
    "paged_attn_decode_split": (ctypes.c_int, [ctypes.POINTER(PaAttnIO), ctypes.POINTER(PaKvCache),
                                               ctypes.POINTER(PaPaging), _vp, ctypes.c_size_t, _vp, _vp]),
    "paged_attn_reduce": (ctypes.c_int, [ctypes.POINTER(PaAttnIO), ctypes.POINTER(PaKvCache),
                                         ctypes.POINTER(PaPaging), _vp, ctypes.c_size_t, _vp, _vp]),
    "paged_attn_varlen": (ctypes.c_int, [ctypes.POINTER(PaAttnIO), ctypes.POINTER(PaKvCache),
                                         ctypes.POINTER(PaPaging), _vp, ctypes.c_int32, _vp, ctypes.c_size_t,
                                         _vp, _vp]),
    "paged_attn_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _vp]),
    "paged_attn_peer_free": (ctypes.c_int, [_vp]),
    "paged_attn_peer_open": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "paged_attn_peer_close": (ctypes.c_int, [_vp]),
    "paged_attn_decode_peers": (ctypes.c_int, [ctypes.POINTER(PaAttnIO), ctypes.POINTER(PaKvCache),
                                               ctypes.POINTER(PaPaging), _vp, ctypes.c_size_t,
                                               ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, _vp, _vp]),
    "paged_attn_peer_barrier": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, ctypes.c_int32,
                                               ctypes.c_int32, _vp, _vp]),
    "paged_attn_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(PaAttnIO), ctypes.POINTER(PaKvCache),
                                                 ctypes.POINTER(PaPaging), _vp, _vp]),
    "paged_attn_prefill": (ctypes.c_int, [ctypes.POINTER(PaAttnIO), ctypes.POINTER(PaKvCache),
                                          ctypes.POINTER(PaPaging), _vp, _vp]),
    "kv_write_quant": (ctypes.c_int, [ctypes.POINTER(PaKvNew), ctypes.POINTER(PaKvCache), ctypes.POINTER(PaPaging),
                                      _vp, _vp]),
    "kv_write_copy": (ctypes.c_int, [ctypes.POINTER(PaKvNew), ctypes.POINTER(PaKvCache), ctypes.POINTER(PaPaging),
                                     _vp, _vp]),
    "kv_project_write": (ctypes.c_int, [ctypes.POINTER(PaKvProj), ctypes.POINTER(PaKvCache),
                                        ctypes.POINTER(PaPaging), _vp, _vp]),
    "block_pool_init": (ctypes.c_int, [_vp, _vp]),
    "block_pool_apply": (ctypes.c_int, [_vp, _vp, ctypes.c_int32, _vp, _vp]),
    "block_pool_step": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, ctypes.c_int32, _vp, ctypes.c_int64, ctypes.c_int32,
                                       _vp, _vp, _vp, ctypes.c_int32, _vp, _vp]),
    "paged_attn_error_string": (ctypes.c_char_p, []),
    "paged_attn_version": (ctypes.c_char_p, []),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library with typed entry points."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python paged-inference-engine_b200/build.py` "
                "(the paged-attention path has no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class PagedAttnError(RuntimeError):
    """A C-ABI call returned a non-zero PA_ERR_* code."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed (code {code}): {msg}")
        self.code = code


def check(fn: str, code: int) -> None:
    if code != PA_OK:
        msg = load().paged_attn_error_string().decode(errors="replace")
        if code in (PA_ERR_INVALID,):
            raise ValueError(f"{fn}: {msg}")
        raise PagedAttnError(fn, code, msg)
