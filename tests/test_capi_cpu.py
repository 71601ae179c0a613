"""CPU checks of the C ABI: the library loads, exports every function the
header declares, its struct layouts match the ctypes mirrors, and argument
validation answers without touching a GPU.  Also the Python front end's
host-side checks (reference error behaviour)."""
import ctypes
import os
import re
import subprocess

import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "paged_attn_b200.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\**\s*(\w+)\s*\([^;]*\)\s*;", text, flags=re.M)))


def test_library_exports_every_header_function():
    from pie_b200 import _lib

    lib = _lib.load()
    funcs = header_functions()
    assert len(funcs) >= 8, funcs
    for f in funcs:
        assert hasattr(lib, f), f"{f} declared in the header but not exported"
        assert f in _lib.SIGNATURES, f"{f} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(funcs) <= exported
    assert lib.paged_attn_version() == b"0.1.0"


def test_struct_layouts_match_header(tmp_path):
    from pie_b200 import _lib
    from pie_b200.block_pool import PaBlockPool

    structs = {"pa_kv_cache_t": _lib.PaKvCache, "pa_paging_t": _lib.PaPaging, "pa_attn_io_t": _lib.PaAttnIO,
               "pa_kv_new_t": _lib.PaKvNew, "pa_block_pool_t": PaBlockPool, "pa_kv_proj_t": _lib.PaKvProj}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "paged_attn_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    for ln in filter(None, got):
        cname, field, val = ln.split()
        py = structs[cname]
        want = ctypes.sizeof(py) if field == "sizeof" else getattr(py, field).offset
        assert int(val) == want, f"{cname}.{field}: C {val} vs ctypes {want}"


def _descs(head_dim=128, dtype=None, q_heads=8, kv_heads=2):
    from pie_b200 import _lib

    kv = _lib.PaKvCache()
    kv.k = kv.v = 1 << 20
    kv.dtype = _lib.PA_DTYPE_F16 if dtype is None else dtype
    kv.num_blocks, kv.block_size, kv.num_kv_heads, kv.head_dim = 8, 16, kv_heads, head_dim
    kv.k_stride_block = kv.v_stride_block = 16 * kv_heads * head_dim
    kv.k_stride_slot = kv.v_stride_slot = kv_heads * head_dim
    kv.k_stride_head = kv.v_stride_head = head_dim
    pg = _lib.PaPaging()
    pg.block_table = pg.num_blocks_per_seq = pg.q_len_per_seq = pg.kv_len_per_seq = 1 << 21
    pg.bt_stride_seq, pg.bt_stride_col, pg.bt_cols, pg.num_seqs = 4, 1, 4, 2
    io = _lib.PaAttnIO()
    io.q = io.o = 1 << 22
    io.q_dtype, io.num_q_heads, io.max_q_len = _lib.PA_DTYPE_F16, q_heads, 64
    io.q_stride_seq, io.q_stride_head, io.q_stride_row = q_heads * 64 * head_dim, 64 * head_dim, head_dim
    io.o_stride_seq, io.o_stride_head, io.o_stride_row = io.q_stride_seq, io.q_stride_head, io.q_stride_row
    return io, kv, pg


@pytest.mark.parametrize("mutate,code,msg", [
    (lambda io, kv, pg: setattr(kv, "head_dim", 96), -2, b"head_dim"),
    (lambda io, kv, pg: setattr(kv, "dtype", 7), -1, b"dtype"),
    (lambda io, kv, pg: setattr(kv, "block_size", 12), -1, b"power of two"),
    (lambda io, kv, pg: setattr(io, "num_q_heads", 3), -1, b"multiple"),
    (lambda io, kv, pg: setattr(kv, "k_stride_head", 3), -1, b"aligned"),
    (lambda io, kv, pg: setattr(io, "q_stride_row", 5), -1, b"Q rows"),
    (lambda io, kv, pg: setattr(kv, "dtype", 2), -1, b"k_scale"),
    (lambda io, kv, pg: setattr(io, "q_dtype", 3), -1, b"Q dtype"),
])
def test_argument_validation_without_gpu(mutate, code, msg):
    from pie_b200 import _lib

    lib = _lib.load()
    io, kv, pg = _descs()
    mutate(io, kv, pg)
    rc = lib.paged_attn_prefill(io, kv, pg, None, None)
    assert rc == code
    assert msg in lib.paged_attn_error_string()


def test_null_descriptors_rejected():
    from pie_b200 import _lib

    lib = _lib.load()
    io, kv, pg = _descs()
    assert lib.paged_attn_prefill(None, kv, pg, None, None) == _lib.PA_ERR_INVALID
    assert lib.paged_attn_prefill(io, None, pg, None, None) == _lib.PA_ERR_INVALID
    assert lib.paged_attn_prefill(io, kv, None, None, None) == _lib.PA_ERR_INVALID
    nw = _lib.PaKvNew()
    assert lib.kv_write_quant(nw, kv, pg, None, None) == _lib.PA_ERR_INVALID  # fp16 pool / bad dtype


def test_prefill_shape_needs_no_workspace():
    from pie_b200 import _lib

    lib = _lib.load()
    io, kv, pg = _descs()  # max_q_len 64 x group 4 > 16 -> prefill kernel, no workspace, no CUDA call
    n = ctypes.c_size_t(123)
    assert lib.paged_attn_workspace_size(io, kv, pg, ctypes.byref(n)) == 0
    assert n.value == 0


def test_front_end_rejects_cpu_tensors_like_the_reference():
    from kernels.flash_attention import flash_attention_forward

    Q = torch.zeros(1, 2, 1, 64, dtype=torch.float16)
    K = torch.zeros(2, 16, 2, 64, dtype=torch.float16)
    i = torch.ones(1, dtype=torch.int32)
    with pytest.raises(AssertionError, match="Not CUDA Tensors"):
        flash_attention_forward(Q, K, K, i, torch.zeros(1, 1, dtype=torch.int32), i, 16, i, None, None)


def test_scale_layouts_become_strides():
    from pie_b200 import ops

    K = torch.zeros(5, 16, 4, 64, dtype=torch.int8)
    per_block = torch.ones(5, 4)
    per_token = torch.ones(5, 16, 4, dtype=torch.float16)
    d = ops.kv_cache_desc(K, K, per_block, per_block)
    assert (d.ks_stride_block, d.ks_stride_slot, d.ks_stride_head) == (4, 0, 1)
    assert d.scale_dtype == 3
    d = ops.kv_cache_desc(K, K, per_token, per_token)
    assert (d.ks_stride_block, d.ks_stride_slot, d.ks_stride_head) == (64, 4, 1)
    with pytest.raises(ValueError):
        ops.kv_cache_desc(K, K, torch.ones(5, 3), torch.ones(5, 3))
    with pytest.raises(ValueError):
        ops.kv_cache_desc(K, K)  # int8 pool without scales
    # reference model layout [NB, H, BS, D] read through the launcher's stride convention
    M = torch.zeros(5, 4, 16, 64, dtype=torch.float16)
    d = ops.kv_cache_desc(M, M)
    assert (d.k_stride_block, d.k_stride_slot, d.k_stride_head) == (4096, 1024, 64)


def test_varlen_and_peer_entry_points_validate_without_gpu():
    """The ragged-row and peer-exchange entry points reject bad arguments before any CUDA call."""
    import ctypes

    from pie_b200 import _lib

    lib = _lib.load()
    io, kv, pg = _descs()
    # ragged rows: q_start is required, the row count must not be negative, T = 0 is a no-op
    assert lib.paged_attn_varlen(io, kv, pg, None, 10, None, 0, None, None) == _lib.PA_ERR_INVALID
    assert b"q_start" in lib.paged_attn_error_string()
    assert lib.paged_attn_varlen(io, kv, pg, 1 << 23, -1, None, 0, None, None) == _lib.PA_ERR_INVALID
    assert lib.paged_attn_varlen(io, kv, pg, 1 << 23, 0, None, 0, None, None) == _lib.PA_OK
    # peer decode: 1..8 output pointers, decode shapes only
    none = (ctypes.c_void_p * 1)()
    assert lib.paged_attn_decode_peers(io, kv, pg, None, 0, none, 0, None, None) == _lib.PA_ERR_INVALID
    nine = (ctypes.c_void_p * 9)(*([1 << 24] * 9))
    assert lib.paged_attn_decode_peers(io, kv, pg, None, 0, nine, 9, None, None) == _lib.PA_ERR_INVALID
    two = (ctypes.c_void_p * 2)(1 << 24, 1 << 25)
    assert lib.paged_attn_decode_peers(io, kv, pg, None, 0, two, 2, None, None) == _lib.PA_ERR_UNSUPPORTED
    assert b"max_q_len" in lib.paged_attn_error_string()  # max_q_len 64 x group 4 is a prefill shape
    # barrier: rank inside [0, n), every flag pointer present
    flags = (ctypes.c_void_p * 2)(1 << 24, None)
    assert lib.paged_attn_peer_barrier(1 << 24, flags, 2, 2, 1, None, None) == _lib.PA_ERR_INVALID
    assert lib.paged_attn_peer_barrier(1 << 24, flags, 2, 0, 1, None, None) == _lib.PA_ERR_INVALID
    assert b"flag pointer 1" in lib.paged_attn_error_string()
    # set-up helpers reject NULL outputs
    assert lib.paged_attn_peer_alloc(64, None, None) == _lib.PA_ERR_INVALID
    assert lib.paged_attn_peer_open(None, None) == _lib.PA_ERR_INVALID
    assert lib.paged_attn_peer_free(None) == _lib.PA_OK and lib.paged_attn_peer_close(None) == _lib.PA_OK


def test_varlen_front_end_checks_shapes():
    from pie_b200 import ops

    K = torch.zeros(2, 16, 2, 64, dtype=torch.float16)
    i = torch.ones(2, dtype=torch.int32)
    bt = torch.zeros(2, 1, dtype=torch.int32)
    with pytest.raises(ValueError, match="total_q_rows"):
        ops.paged_attention_varlen(torch.zeros(1, 4, 2, 64), torch.zeros(3, dtype=torch.int32), K, K, bt, i, 16, i)
    with pytest.raises(ValueError, match="3 offsets"):
        ops.paged_attention_varlen(torch.zeros(4, 2, 64), torch.zeros(2, dtype=torch.int32), K, K, bt, i, 16, i)
    with pytest.raises(ValueError, match="block_size"):
        ops.paged_attention_varlen(torch.zeros(4, 2, 64), torch.zeros(3, dtype=torch.int32), K, K, bt, i, 8, i)


def test_sharded_decoder_exchange_option():
    from pie_b200.sharded import KVHeadShardedDecoder

    with pytest.raises(ValueError, match="exchange"):
        KVHeadShardedDecoder(8, 2, 64, attention_fn=lambda *a: None, exchange="ring")
    dec = KVHeadShardedDecoder(8, 2, 64, attention_fn=lambda *a: (torch.ones(1, 8, 1, 64), None), exchange="peer")
    # a single process takes the local path: no exchange, no GPU
    out = dec.forward(torch.zeros(1, 8, 1, 64), None, None, None, None, None, 16, None)
    assert out.shape == (1, 8, 1, 64)


def test_block_pool_argument_validation():
    """block_pool_* reject bad descriptors on the host (no launch, no GPU needed)."""
    from pie_b200 import _lib
    from pie_b200.block_pool import PaBlockPool

    lib = _lib.load()
    assert lib.block_pool_init(None, None) == _lib.PA_ERR_INVALID
    d = PaBlockPool(1 << 20, 1 << 20, 1 << 20, 1 << 20, 4, 16, 8, 8, 0)  # table_stride 4 < 8 columns
    assert lib.block_pool_init(ctypes.byref(d), None) == _lib.PA_ERR_INVALID
    assert b"table_stride" in lib.paged_attn_error_string()
    d = PaBlockPool(None, 1 << 20, 1 << 20, 1 << 20, 8, 16, 8, 8, 0)
    assert lib.block_pool_apply(ctypes.byref(d), 1 << 20, 1, None, None) == _lib.PA_ERR_INVALID
    d = PaBlockPool(1 << 20, 1 << 20, 1 << 20, 1 << 20, 8, 16, 8, 8, 0)
    assert lib.block_pool_apply(ctypes.byref(d), None, 3, None, None) == _lib.PA_ERR_INVALID
    assert lib.block_pool_apply(ctypes.byref(d), None, -1, None, None) == _lib.PA_ERR_INVALID
    assert lib.block_pool_apply(ctypes.byref(d), None, 0, None, None) == _lib.PA_OK  # nothing to do
    assert lib.block_pool_step(ctypes.byref(d), None, None, None, None, 2, None, 4, 4, None, None, None, 2, None,
                               None) == _lib.PA_ERR_INVALID
    assert lib.block_pool_step(ctypes.byref(d), None, None, None, None, 0, None, 0, 0, None, None, None, 0, None,
                               None) == _lib.PA_OK


def test_torch_extension_registers_the_ops():
    """The torch.library extension loads without a GPU and its meta kernels give the output shapes."""
    from pie_b200 import _torch_ext

    ops = _torch_ext.ops()
    for name in ("paged_attention", "paged_attention_out", "paged_attention_varlen", "paged_attention_varlen_out",
                 "write_kv"):
        assert hasattr(ops, name), name
    meta = dict(device="meta")
    Q = torch.empty(3, 8, 5, 128, dtype=torch.float16, **meta)
    K = torch.empty(10, 16, 2, 128, dtype=torch.int8, **meta)
    s = torch.empty(10, 16, 2, dtype=torch.float16, **meta)
    i = torch.empty(3, dtype=torch.int32, **meta)
    bt = torch.empty(3, 4, dtype=torch.int32, **meta)
    O, L = ops.paged_attention(Q, K, K, i, bt, i, i, s, s, False, 0.0, 0, None)
    assert O.shape == Q.shape and L.shape == (3, 8, 5) and O.dtype == torch.float16
    q = torch.empty(11, 8, 128, dtype=torch.bfloat16, **meta)
    O, L = ops.paged_attention_varlen(q, i, i, 5, K, K, bt, i, i, s, s, False, 0.0, None)
    assert O.shape == q.shape and L.shape == (11, 8) and O.dtype == torch.float16
