"""Loader of _pie_b200_torch.so: the torch.library ops over the C ABI (csrc/torch_ops.cpp).

Registers ``torch.ops.pie_b200.{paged_attention, paged_attention_out,
paged_attention_varlen, paged_attention_varlen_out, write_kv}``.  Built in-tree
by ``paged-inference-engine_b200/build.py``; a missing build raises (there is no
fallback).
"""
from __future__ import annotations

import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
EXT_PATH = os.path.join(_HERE, "_pie_b200_torch.so")
_lock = threading.Lock()
_loaded = False


def ops():
    """``torch.ops.pie_b200``, loading the extension on first use."""
    global _loaded
    if not _loaded:
        with _lock:
            if not _loaded:
                if not os.path.exists(EXT_PATH):
                    raise RuntimeError(f"{EXT_PATH} is missing: build it with "
                                       "`python paged-inference-engine_b200/build.py`")
                from . import _lib

                _lib.load()  # the C-ABI library the extension links against
                torch.ops.load_library(EXT_PATH)
                _loaded = True
    return torch.ops.pie_b200
