"""Torch-tensor front end of the C ABI: argument checks, then the registered torch ops.

All tensors live on one CUDA device; every launch goes to torch's current
stream on that device, so calls compose with torch ops and CUDA graphs.
Nothing here computes on the host and there is no fallback path: a missing
library or a non-CUDA tensor raises.

The calls go through the torch.library ops of the extension
(``torch.ops.pie_b200.*``, csrc/torch_ops.cpp), which fill the C structs and
call libpaged_attn_b200.so in C++.  ``PIE_B200_BACKEND=ctypes`` routes the
same calls through the ctypes binding of the C ABI instead (``_lib``): the
two paths launch the same kernels with the same arguments.
"""
from __future__ import annotations

import ctypes
import math
import os
from typing import Optional

import torch

from . import _lib
from ._lib import PaAttnIO, PaKvCache, PaKvNew, PaPaging

_TORCH2PA = {
    torch.float16: _lib.PA_DTYPE_F16,
    torch.bfloat16: _lib.PA_DTYPE_BF16,
    torch.int8: _lib.PA_DTYPE_I8,
    torch.float32: _lib.PA_DTYPE_F32,
}

_CHECK = os.environ.get("PIE_B200_CHECK", "0") not in ("", "0")
BACKEND = os.environ.get("PIE_B200_BACKEND", "torch")
if BACKEND not in ("torch", "ctypes"):
    raise ValueError(f"PIE_B200_BACKEND must be 'torch' or 'ctypes', not {BACKEND!r}")
_MODES = {"auto": 0, "decode": 1, "prefill": 2}


def _torch_ops():
    from . import _torch_ext

    return _torch_ext.ops()


_OPS: dict = {}


def _op(name: str):
    """The registered op's default overload, looked up once (a direct call skips the packet dispatch)."""
    op = _OPS.get(name)
    if op is None:
        op = getattr(_torch_ops(), name).default
        _OPS[name] = op
    return op


def _out_and_lse(shape: tuple, device) -> tuple[torch.Tensor, torch.Tensor]:
    """O (shape) and LSE (shape without head_dim), float16, from one allocation (O first, 256-byte aligned)."""
    n_o = math.prod(shape)
    buf = torch.empty(n_o + math.prod(shape[:-1]), dtype=torch.float16, device=device)
    return buf[:n_o].view(shape), buf[n_o:].view(shape[:-1])


def _i32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.int32 and t.is_contiguous():
        return t
    return t.to(torch.int32).contiguous()


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def kv_cache_desc(k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: Optional[torch.Tensor] = None,
                  v_scale: Optional[torch.Tensor] = None) -> PaKvCache:
    """Descriptor of a pool whose dims are read as [block, slot, head, d].

    Scales: [num_blocks, num_kv_heads] (one per block and head, the reference
    layout) or [num_blocks, block_size, num_kv_heads] (one per token and head).
    """
    check_cache(k_cache, v_cache, k_scale, v_scale)
    nb, bs, h, d = k_cache.shape
    kc = PaKvCache()
    kc.k = k_cache.data_ptr()
    kc.v = v_cache.data_ptr()
    kc.dtype = _TORCH2PA[k_cache.dtype]
    kc.num_blocks, kc.block_size, kc.num_kv_heads, kc.head_dim = nb, bs, h, d
    kc.k_stride_block, kc.k_stride_slot, kc.k_stride_head = k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)
    kc.v_stride_block, kc.v_stride_slot, kc.v_stride_head = v_cache.stride(0), v_cache.stride(1), v_cache.stride(2)
    kc.scale_dtype = _lib.PA_DTYPE_F16
    if k_cache.dtype == torch.int8:
        kc.scale_dtype = _TORCH2PA[k_scale.dtype]
        kc.k_scale = k_scale.data_ptr()
        kc.v_scale = v_scale.data_ptr()
        kc.ks_stride_block, kc.ks_stride_slot, kc.ks_stride_head = _scale_strides(k_scale, nb, bs, h)
        kc.vs_stride_block, kc.vs_stride_slot, kc.vs_stride_head = _scale_strides(v_scale, nb, bs, h)
    return kc


def check_cache(k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: Optional[torch.Tensor] = None,
                v_scale: Optional[torch.Tensor] = None) -> None:
    """Raise ValueError unless the pools (and an INT8 pool's scales) are well formed."""
    if k_cache.dim() != 4 or v_cache.dim() != 4:
        raise ValueError("K/V pools must be 4-D [num_blocks, block_size, num_kv_heads, head_dim]")
    if k_cache.shape != v_cache.shape or k_cache.dtype != v_cache.dtype:
        raise ValueError(f"K and V pools differ: {tuple(k_cache.shape)}/{k_cache.dtype} vs "
                         f"{tuple(v_cache.shape)}/{v_cache.dtype}")
    if k_cache.dtype not in (torch.float16, torch.bfloat16, torch.int8, torch.float32):
        raise ValueError(f"KV pool dtype {k_cache.dtype} unsupported (float16, bfloat16, int8 or float32)")
    if k_cache.stride(3) != 1 or v_cache.stride(3) != 1:
        raise ValueError("KV pools need a contiguous head_dim")
    nb, bs, h, d = k_cache.shape
    if k_cache.dtype == torch.int8:
        if k_scale is None or v_scale is None:
            raise ValueError("an int8 KV pool needs k_scale and v_scale")
        for name, s in (("k_scale", k_scale), ("v_scale", v_scale)):
            if s.dtype not in (torch.float16, torch.float32):
                raise ValueError(f"{name} must be float16 or float32, got {s.dtype}")
            if s.device != k_cache.device:
                raise ValueError(f"{name} is on {s.device}, the pool on {k_cache.device}")
        if k_scale.dtype != v_scale.dtype:
            raise ValueError("k_scale and v_scale dtypes differ")
        _scale_strides(k_scale, nb, bs, h)
        _scale_strides(v_scale, nb, bs, h)


def _scale_strides(s: torch.Tensor, nb: int, bs: int, h: int) -> tuple[int, int, int]:
    if s.dim() == 2:
        if tuple(s.shape) != (nb, h):
            raise ValueError(f"per-block scales must be [{nb}, {h}], got {tuple(s.shape)}")
        return s.stride(0), 0, s.stride(1)
    if s.dim() == 3:
        if tuple(s.shape) != (nb, bs, h):
            raise ValueError(f"per-token scales must be [{nb}, {bs}, {h}], got {tuple(s.shape)}")
        return s.stride(0), s.stride(1), s.stride(2)
    raise ValueError("scales must be 2-D [NB, H] or 3-D [NB, BS, H]")


def pool_layout(K: torch.Tensor, V: torch.Tensor, block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The pools as [block, slot, head, d] views.

    The reference launcher reads dims 1 and 2 as (slot, head)
    (kernels/flash_attention.py:158-159) while the reference model allocates
    its caches as [num_blocks, heads, block_size, d_k]
    (transformer/model.py:64-65) and passes them unchanged
    (transformer/model.py:156-160).  A pool whose dim 1 is not ``block_size``
    but whose dim 2 is can only be the model's layout, so it is read through
    the transposed view; a pool that fits the launcher's layout is read as is.
    """
    if K.dim() == 4 and K.shape[1] != block_size and K.shape[2] == block_size:
        return K.transpose(1, 2), V.transpose(1, 2)
    return K, V


def _paging_tensors(block_table: torch.Tensor, num_blocks: torch.Tensor, q_len: torch.Tensor,
                    kv_len: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """int32 block table (any strides) and contiguous int32 metadata with one entry per sequence."""
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    if bt.dim() != 2:
        raise ValueError("block_table must be 2-D [num_seqs, max_blocks]")
    nbk, ql, kl = _i32(num_blocks), _i32(q_len), _i32(kv_len)
    for name, t in (("num_blocks_per_seq", nbk), ("q_len_per_seq", ql), ("kv_len_per_seq", kl)):
        if t.numel() != bt.shape[0]:
            raise ValueError(f"{name} has {t.numel()} entries for {bt.shape[0]} sequences")
    return bt, nbk, ql, kl


def paging_desc(block_table: torch.Tensor, num_blocks: torch.Tensor, q_len: torch.Tensor,
                kv_len: torch.Tensor, keep: list) -> PaPaging:
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    if bt.dim() != 2:
        raise ValueError("block_table must be 2-D [num_seqs, max_blocks]")
    nbk, ql, kl = _i32(num_blocks), _i32(q_len), _i32(kv_len)
    keep.extend((bt, nbk, ql, kl))
    pg = PaPaging()
    pg.block_table = bt.data_ptr()
    pg.bt_stride_seq, pg.bt_stride_col = bt.stride(0), bt.stride(1)
    pg.bt_cols = bt.shape[1]
    pg.num_seqs = bt.shape[0]
    pg.num_blocks_per_seq, pg.q_len_per_seq, pg.kv_len_per_seq = nbk.data_ptr(), ql.data_ptr(), kl.data_ptr()
    for name, t in (("num_blocks_per_seq", nbk), ("q_len_per_seq", ql), ("kv_len_per_seq", kl)):
        if t.numel() != pg.num_seqs:
            raise ValueError(f"{name} has {t.numel()} entries for {pg.num_seqs} sequences")
    return pg


_workspaces: dict[int, torch.Tensor] = {}
_status: dict[int, torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device split-K workspace, grown on demand (256-byte aligned)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[idx] = ws
    return ws


def status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _status.get(idx)
    if st is None:
        st = torch.zeros(1, dtype=torch.int32, device=device)
        _status[idx] = st
    return st


def _raise_status(fn: str, st: torch.Tensor) -> None:
    v = int(st.item())
    if v:
        st.zero_()
        _raise_status_value(fn, v)


def _raise_status_value(fn: str, v: int) -> None:
    """Raise IndexError naming the bits of a nonzero device status word."""
    if v:
        bits = []
        if v & _lib.PA_STATUS_BAD_BLOCK_ID:
            bits.append("block id outside the pool")
        if v & _lib.PA_STATUS_BAD_POSITION:
            bits.append("position beyond the block table")
        if v & _lib.PA_STATUS_BAD_NUM_BLOCKS:
            bits.append("num_blocks_per_seq wider than the block table")
        if v & _lib.PA_STATUS_BAD_SEQ_INDEX:
            bits.append("sequence index outside the block table")
        if v & _lib.PA_STATUS_PEER_TIMEOUT:
            bits.append("a peer GPU never reached the output-exchange barrier")
        raise IndexError(f"{fn}: device status {v:#x}: " + "; ".join(bits))


def paged_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, q_len_per_seq: torch.Tensor,
                    block_table: torch.Tensor, num_blocks_per_seq: torch.Tensor, block_size: int,
                    kv_len_per_seq: torch.Tensor, k_scale: Optional[torch.Tensor] = None,
                    v_scale: Optional[torch.Tensor] = None, *, out: Optional[torch.Tensor] = None,
                    lse: Optional[torch.Tensor] = None, causal_top_left: bool = False,
                    softmax_scale: Optional[float] = None, mode: str = "auto",
                    status: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Paged causal attention through the C ABI; returns (O fp16, L fp16)."""
    if Q.dim() != 4:
        raise ValueError("Q must be [num_seqs, num_q_heads, max_q_len, head_dim]")
    B, Hq, maxq, D = Q.shape
    K, V = pool_layout(K, V, block_size)
    if K.shape[1] != block_size:
        raise ValueError(f"block_size {block_size} does not match the pool's slot dimension {K.shape[1]}")
    if K.shape[3] != D:
        raise ValueError(f"head_dim of Q ({D}) and of the pool ({K.shape[3]}) differ")
    if block_table.shape[0] != B:
        raise ValueError(f"block_table has {block_table.shape[0]} rows for {B} sequences")
    dev = Q.device
    if Q.dtype not in (torch.float16, torch.bfloat16):
        Q = Q.to(K.dtype if K.dtype in (torch.float16, torch.bfloat16) else torch.float16)
    if Q.stride(3) != 1:
        Q = Q.contiguous()
    if mode not in _MODES:
        raise ValueError(f"mode must be one of {sorted(_MODES)}, not {mode!r}")
    if out is None and lse is None:
        out, lse = _out_and_lse((B, Hq, maxq, D), dev)
    if out is None:
        out = torch.empty((B, Hq, maxq, D), dtype=torch.float16, device=dev)
    elif out.dtype != torch.float16 or tuple(out.shape) != (B, Hq, maxq, D):
        raise ValueError("out must be float16 with Q's shape")
    if lse is None:
        lse = torch.empty((B, Hq, maxq), dtype=torch.float16, device=dev)
    if status is None and _CHECK:
        status = status_word(dev)
    if BACKEND == "torch":
        # pools, scales, devices and metadata lengths are checked by the op (ValueError)
        bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
        _op("paged_attention_out")(Q, K, V, _i32(q_len_per_seq), bt, _i32(num_blocks_per_seq),
                                   _i32(kv_len_per_seq), k_scale, v_scale, bool(causal_top_left),
                                   float(softmax_scale) if softmax_scale else 0.0, _MODES[mode], status, out, lse)
        if _CHECK and status is not None:
            _raise_status("paged_attention", status)
        return out, lse
    for name, t in (("K", K), ("V", V), ("block_table", block_table), ("q_len_per_seq", q_len_per_seq),
                    ("kv_len_per_seq", kv_len_per_seq), ("num_blocks_per_seq", num_blocks_per_seq)):
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, Q on {dev}")
    keep: list = []
    kc = kv_cache_desc(K, V, k_scale, v_scale)
    pg = paging_desc(block_table, num_blocks_per_seq, q_len_per_seq, kv_len_per_seq, keep)
    io = PaAttnIO()
    io.q = Q.data_ptr()
    io.q_dtype = _TORCH2PA[Q.dtype]
    io.num_q_heads, io.max_q_len = Hq, maxq
    io.causal_top_left = 1 if causal_top_left else 0
    io.q_stride_seq, io.q_stride_head, io.q_stride_row = Q.stride(0), Q.stride(1), Q.stride(2)
    io.o = out.data_ptr()
    io.o_stride_seq, io.o_stride_head, io.o_stride_row = out.stride(0), out.stride(1), out.stride(2)
    io.lse = lse.data_ptr()
    io.l_stride_seq, io.l_stride_head, io.l_stride_row = lse.stride(0), lse.stride(1), lse.stride(2)
    io.softmax_scale = float(softmax_scale) if softmax_scale else 0.0

    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    st_ptr = _ptr(status)
    with torch.cuda.device(dev):
        if mode == "prefill":
            _lib.check("paged_attn_prefill", lib.paged_attn_prefill(io, kc, pg, st_ptr, stream))
        else:
            nbytes = ctypes.c_size_t(0)
            _lib.check("paged_attn_workspace_size", lib.paged_attn_workspace_size(io, kc, pg, ctypes.byref(nbytes)))
            ws = workspace(dev, nbytes.value) if nbytes.value else None
            fn = lib.paged_attn_decode if mode == "decode" else lib.paged_attn_forward
            _lib.check(fn.__name__, fn(io, kc, pg, _ptr(ws), 0 if ws is None else ws.numel(), st_ptr, stream))
    if _CHECK and status is not None:
        _raise_status("paged_attention", status)
    return out, lse


def paged_attention_varlen(Q: torch.Tensor, cu_seqlens_q: torch.Tensor, K: torch.Tensor, V: torch.Tensor,
                           block_table: torch.Tensor, num_blocks_per_seq: torch.Tensor, block_size: int,
                           kv_len_per_seq: torch.Tensor, k_scale: Optional[torch.Tensor] = None,
                           v_scale: Optional[torch.Tensor] = None, *, max_q_len: Optional[int] = None,
                           out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
                           causal_top_left: bool = False, softmax_scale: Optional[float] = None,
                           status: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Paged causal attention over ragged query rows through paged_attn_varlen.

    Q is ``[T, Hq, D]`` with the rows of sequence b at
    ``cu_seqlens_q[b] : cu_seqlens_q[b + 1]``; returns O ``[T, Hq, D]`` and L
    ``[T, Hq]`` (fp16).  ``max_q_len`` (the longest sequence's row count) sizes
    the grid; without it one host read of ``cu_seqlens_q`` finds it.
    """
    if Q.dim() != 3:
        raise ValueError("Q must be [total_q_rows, num_q_heads, head_dim]")
    T, Hq, D = Q.shape
    B = block_table.shape[0]
    if cu_seqlens_q.dim() != 1 or cu_seqlens_q.shape[0] != B + 1:
        raise ValueError(f"cu_seqlens_q must hold {B + 1} offsets for {B} sequences")
    K, V = pool_layout(K, V, block_size)
    if K.shape[1] != block_size:
        raise ValueError(f"block_size {block_size} does not match the pool's slot dimension {K.shape[1]}")
    if K.shape[3] != D:
        raise ValueError(f"head_dim of Q ({D}) and of the pool ({K.shape[3]}) differ")
    dev = Q.device
    for name, t in (("K", K), ("V", V), ("block_table", block_table), ("cu_seqlens_q", cu_seqlens_q),
                    ("kv_len_per_seq", kv_len_per_seq), ("num_blocks_per_seq", num_blocks_per_seq)):
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, Q on {dev}")
    cu = _i32(cu_seqlens_q)
    q_start = cu[:-1]
    q_len = (cu[1:] - cu[:-1]).contiguous()
    if max_q_len is None:
        max_q_len = int(q_len.max().item()) if B else 0
    mma_dtype = K.dtype if K.dtype in (torch.float16, torch.bfloat16) else torch.float16
    if Q.dtype not in (torch.float16, torch.bfloat16):
        Q = Q.to(mma_dtype)
    if Q.stride(2) != 1:
        Q = Q.contiguous()
    if out is None:
        out = torch.empty((T, Hq, D), dtype=torch.float16, device=dev)
    elif out.dtype != torch.float16 or tuple(out.shape) != (T, Hq, D):
        raise ValueError("out must be float16 with Q's shape")
    if lse is None:
        lse = torch.empty((T, Hq), dtype=torch.float16, device=dev)
    if status is None and _CHECK:
        status = status_word(dev)
    if BACKEND == "torch":
        check_cache(K, V, k_scale, v_scale)
        bt, nbk, ql, kl = _paging_tensors(block_table, num_blocks_per_seq, q_len, kv_len_per_seq)
        if T:
            _op("paged_attention_varlen_out")(Q, q_start, ql, int(max_q_len), K, V, bt, nbk, kl, k_scale,
                                                    v_scale, bool(causal_top_left),
                                                    float(softmax_scale) if softmax_scale else 0.0, status, out, lse)
        if _CHECK and status is not None:
            _raise_status("paged_attention_varlen", status)
        return out, lse
    keep: list = [cu, q_len]
    kc = kv_cache_desc(K, V, k_scale, v_scale)
    pg = paging_desc(block_table, num_blocks_per_seq, q_len, kv_len_per_seq, keep)
    io = PaAttnIO()
    io.q = Q.data_ptr()
    io.q_dtype = _TORCH2PA[Q.dtype]
    io.num_q_heads, io.max_q_len = Hq, int(max_q_len)
    io.causal_top_left = 1 if causal_top_left else 0
    io.q_stride_seq, io.q_stride_head, io.q_stride_row = 0, Q.stride(1), Q.stride(0)
    io.o = out.data_ptr()
    io.o_stride_seq, io.o_stride_head, io.o_stride_row = 0, out.stride(1), out.stride(0)
    io.lse = lse.data_ptr()
    io.l_stride_seq, io.l_stride_head, io.l_stride_row = 0, lse.stride(1), lse.stride(0)
    io.softmax_scale = float(softmax_scale) if softmax_scale else 0.0

    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    st_ptr = _ptr(status)
    with torch.cuda.device(dev):
        nbytes = ctypes.c_size_t(0)
        _lib.check("paged_attn_workspace_size", lib.paged_attn_workspace_size(io, kc, pg, ctypes.byref(nbytes)))
        ws = workspace(dev, nbytes.value) if nbytes.value else None
        _lib.check("paged_attn_varlen", lib.paged_attn_varlen(io, kc, pg, q_start.data_ptr(), T, _ptr(ws),
                                                              0 if ws is None else ws.numel(), st_ptr, stream))
    if _CHECK and status is not None:
        _raise_status("paged_attention_varlen", status)
    return out, lse


def paged_attention_peers(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, q_len_per_seq: torch.Tensor,
                          block_table: torch.Tensor, num_blocks_per_seq: torch.Tensor, block_size: int,
                          kv_len_per_seq: torch.Tensor, k_scale: Optional[torch.Tensor], v_scale: Optional[torch.Tensor],
                          out: torch.Tensor, out_peer_ptrs: list[int], *,
                          status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode whose O rows go to every GPU of a peer exchange (paged_attn_decode_peers).

    ``out`` is this GPU's view of the destination (it fixes the layout);
    ``out_peer_ptrs[r]`` is the address of the same element 0 in GPU r's
    mapped buffer.  Returns the local LSE [B, Hq, q] (fp16).
    """
    B, Hq, maxq, D = Q.shape
    dev = Q.device
    if Q.stride(3) != 1:
        Q = Q.contiguous()
    keep: list = []
    kc = kv_cache_desc(K, V, k_scale, v_scale)
    pg = paging_desc(block_table, num_blocks_per_seq, q_len_per_seq, kv_len_per_seq, keep)
    if out.dtype != torch.float16 or tuple(out.shape) != (B, Hq, maxq, D):
        raise ValueError("out must be float16 with Q's shape")
    lse = torch.empty((B, Hq, maxq), dtype=torch.float16, device=dev)
    io = PaAttnIO()
    io.q = Q.data_ptr()
    io.q_dtype = _TORCH2PA[Q.dtype]
    io.num_q_heads, io.max_q_len = Hq, maxq
    io.q_stride_seq, io.q_stride_head, io.q_stride_row = Q.stride(0), Q.stride(1), Q.stride(2)
    io.o = out.data_ptr()
    io.o_stride_seq, io.o_stride_head, io.o_stride_row = out.stride(0), out.stride(1), out.stride(2)
    io.lse = lse.data_ptr()
    io.l_stride_seq, io.l_stride_head, io.l_stride_row = lse.stride(0), lse.stride(1), lse.stride(2)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    if status is None and _CHECK:
        status = status_word(dev)
    peers = (ctypes.c_void_p * len(out_peer_ptrs))(*out_peer_ptrs)
    with torch.cuda.device(dev):
        nbytes = ctypes.c_size_t(0)
        _lib.check("paged_attn_workspace_size", lib.paged_attn_workspace_size(io, kc, pg, ctypes.byref(nbytes)))
        ws = workspace(dev, nbytes.value) if nbytes.value else None
        _lib.check("paged_attn_decode_peers",
                   lib.paged_attn_decode_peers(io, kc, pg, _ptr(ws), 0 if ws is None else ws.numel(), peers,
                                               len(out_peer_ptrs), _ptr(status), stream))
    if _CHECK and status is not None:
        _raise_status("paged_attention_peers", status)
    return lse


def write_kv(k_new: torch.Tensor, v_new: torch.Tensor, block_table: torch.Tensor, seq_index: torch.Tensor,
             positions: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
             k_scale: Optional[torch.Tensor] = None, v_scale: Optional[torch.Tensor] = None, *,
             status: Optional[torch.Tensor] = None) -> None:
    """Append new rows [T, Hkv, D] at (seq_index[t], positions[t]) of the pool."""
    if k_new.dim() != 3 or v_new.shape != k_new.shape:
        raise ValueError("k_new / v_new must be [num_tokens, num_kv_heads, head_dim] of equal shape")
    T, H, D = k_new.shape
    if (H, D) != (k_cache.shape[2], k_cache.shape[3]):
        raise ValueError(f"new rows [*, {H}, {D}] do not match the pool [*, *, {k_cache.shape[2]}, {k_cache.shape[3]}]")
    if k_new.dtype not in (torch.float16, torch.bfloat16, torch.float32) or v_new.dtype != k_new.dtype:
        raise ValueError("k_new / v_new must share a float16, bfloat16 or float32 dtype")
    dev = k_cache.device
    if k_new.stride(2) != 1:
        k_new = k_new.contiguous()
    if v_new.stride(2) != 1:
        v_new = v_new.contiguous()
    if k_cache.dtype == torch.int8 and (k_scale is None or k_scale.dim() != 3):
        raise ValueError("quantise-on-write stores one scale per (token, head): scales must be [NB, BS, H]")
    if BACKEND != "torch":
        check_cache(k_cache, v_cache, k_scale, v_scale)  # the op checks them itself
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    si, ps = _i32(seq_index), _i32(positions)
    if si.numel() != T or ps.numel() != T:
        raise ValueError("seq_index / positions need one entry per token")
    if status is None and _CHECK:
        status = status_word(dev)
    if BACKEND == "torch":
        if bt.dim() != 2:
            raise ValueError("block_table must be 2-D [num_seqs, max_blocks]")
        _op("write_kv")(k_new, v_new, bt, si, ps, k_cache, v_cache, k_scale if k_cache.dtype == torch.int8 else None,
                        v_scale if k_cache.dtype == torch.int8 else None, status)
        if _CHECK and status is not None:
            _raise_status("write_kv_cache", status)
        return
    keep: list = []
    kc = kv_cache_desc(k_cache, v_cache, k_scale, v_scale)
    keep.extend((bt, si, ps))
    pg = _lib.PaPaging()
    pg.block_table = bt.data_ptr()
    pg.bt_stride_seq, pg.bt_stride_col = bt.stride(0), bt.stride(1)
    pg.bt_cols, pg.num_seqs = bt.shape[1], bt.shape[0]
    nw = PaKvNew()
    nw.k_new, nw.v_new = k_new.data_ptr(), v_new.data_ptr()
    nw.dtype = _TORCH2PA[k_new.dtype]
    nw.num_tokens = T
    nw.k_stride_token, nw.k_stride_head = k_new.stride(0), k_new.stride(1)
    nw.v_stride_token, nw.v_stride_head = v_new.stride(0), v_new.stride(1)
    nw.seq_index, nw.positions = si.data_ptr(), ps.data_ptr()
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        if k_cache.dtype == torch.int8:
            _lib.check("kv_write_quant", lib.kv_write_quant(nw, kc, pg, _ptr(status), stream))
        else:
            _lib.check("kv_write_copy", lib.kv_write_copy(nw, kc, pg, _ptr(status), stream))
    if _CHECK and status is not None:
        _raise_status("write_kv_cache", status)


def project_write_kv(x: torch.Tensor, w_kv: torch.Tensor, bias: Optional[torch.Tensor], block_table: torch.Tensor,
                     seq_index: torch.Tensor, positions: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     k_scale: Optional[torch.Tensor] = None, v_scale: Optional[torch.Tensor] = None, *,
                     status: Optional[torch.Tensor] = None) -> None:
    """K/V projection of x [T, d_model] with the cache write in its epilogue (kv_project_write).

    ``w_kv`` is [W_k; W_v] ([2 * Hkv * D, d_model], nn.Linear's weight layout)
    and ``bias`` the matching float32 [2 * Hkv * D] (or None): token t's K
    row of head h is ``x[t] @ W_k[h*D:(h+1)*D].T + b_k[h*D:(h+1)*D]``, written
    at (seq_index[t], positions[t]) of the pool like ``write_kv`` writes it.
    """
    if x.dim() != 2 or w_kv.dim() != 2 or x.shape[1] != w_kv.shape[1]:
        raise ValueError("x must be [T, d_model] and w_kv [2 * Hkv * D, d_model]")
    if x.dtype not in (torch.float16, torch.bfloat16) or w_kv.dtype != x.dtype:
        raise ValueError("x and w_kv must share a float16 or bfloat16 dtype")
    if k_cache.dtype == torch.int8 and (k_scale is None or k_scale.dim() != 3):
        raise ValueError("an int8 pool written per token needs per-token scales [NB, BS, H]")
    if w_kv.shape[0] != 2 * k_cache.shape[2] * k_cache.shape[3]:
        raise ValueError(f"w_kv has {w_kv.shape[0]} rows; the pool needs 2 * {k_cache.shape[2]} * {k_cache.shape[3]}")
    if seq_index.numel() != x.shape[0] or positions.numel() != x.shape[0]:
        raise ValueError("seq_index / positions need one entry per token")
    if x.stride(1) != 1:
        x = x.contiguous()
    if w_kv.stride(1) != 1:
        w_kv = w_kv.contiguous()
    dev = k_cache.device
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous()):
        bias = bias.to(torch.float32).contiguous()
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    si, ps = _i32(seq_index), _i32(positions)
    if status is None and _CHECK:
        status = status_word(dev)
    int8 = k_cache.dtype == torch.int8
    if BACKEND == "torch":
        _op("project_write_kv")(x, w_kv, bias, bt, si, ps, k_cache, v_cache, k_scale if int8 else None,
                                v_scale if int8 else None, status)
    else:
        kc = kv_cache_desc(k_cache, v_cache, k_scale, v_scale)
        pg = _lib.PaPaging()
        pg.block_table = bt.data_ptr()
        pg.bt_stride_seq, pg.bt_stride_col = bt.stride(0), bt.stride(1)
        pg.bt_cols, pg.num_seqs = bt.shape[1], bt.shape[0]
        pj = _lib.PaKvProj()
        pj.x, pj.w = x.data_ptr(), w_kv.data_ptr()
        pj.bias = None if bias is None else bias.data_ptr()
        pj.x_stride, pj.w_stride = x.stride(0), w_kv.stride(0)
        pj.dtype = _TORCH2PA[x.dtype]
        pj.num_tokens, pj.d_model = x.shape[0], x.shape[1]
        pj.seq_index, pj.positions = si.data_ptr(), ps.data_ptr()
        lib = _lib.load()
        with torch.cuda.device(dev):
            _lib.check("kv_project_write", lib.kv_project_write(pj, kc, pg, _ptr(status),
                                                                torch.cuda.current_stream(dev).cuda_stream))
    if _CHECK and status is not None:
        _raise_status("project_write_kv", status)
