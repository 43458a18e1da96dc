"""CPU checks of the C ABI: the library loads, exports every entry point include/wanb200.h
declares, the ctypes parameter structs have the C layout, and argument validation rejects bad
calls on the host (before any CUDA call, so these run without a GPU)."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT
from wanb200 import _lib as L

HEADER = os.path.join(ROOT, "include", "wanb200.h")


def header_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int64_t|int|const char\*)\s+(wanb200_\w+)\s*\(", src, re.M)))


def test_library_exports_every_declared_function():
    lib = L.load()
    names = header_functions()
    assert len(names) >= 8
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(L.EXPORTS)
    assert lib.wanb200_version() == 201


STRUCTS = {
    "wanb200_gemm_params": L.GemmParams,
    "wanb200_attn_params": L.AttnParams,
    "wanb200_ln_params": L.LnParams,
    "wanb200_qknorm_params": L.QkNormParams,
    "wanb200_residual_params": L.ResidualParams,
    "wanb200_shard_gather_params": L.ShardGatherParams,
    "wanb200_attn_fp8_params": L.AttnFp8Params,
    "wanb200_block_params": L.BlockParams,
    "wanb200_block_weights": L.BlockWeightsC,
    "wanb200_patchify_params": L.PatchifyParams,
    "wanb200_unpatchify_params": L.UnpatchifyParams,
    "wanb200_sumsq_reduce_params": L.SumsqReduceParams,
}


def test_ctypes_structs_match_c_layout(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, cls in STRUCTS.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("  return 0;\n}")
    c = tmp_path / "layout.c"
    c.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.check_call(["gcc", "-o", str(exe), str(c)])
    out = subprocess.check_output([str(exe)]).decode().split("\n")
    got = {}
    for ln in out:
        if ln:
            s, f, v = ln.split()
            got[(s, f)] = int(v)
    for cname, cls in STRUCTS.items():
        assert got[(cname, "size")] == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert got[(cname, fname)] == getattr(cls, fname).offset, (cname, fname)


def _rc_msg(fn, p):
    rc = fn(ctypes.byref(p), None)
    return rc, L.load().wanb200_last_error().decode()


def test_gemm_rejects_bad_shapes_on_host():
    lib = L.load()
    p = L.GemmParams()
    p.a = p.w = p.d = 16
    p.lda = p.ldw = p.ldd = 96
    p.M, p.N, p.K, p.epilogue = 8, 64, 96, L.EPI_NONE
    rc, msg = _rc_msg(lib.wanb200_gemm_bf16, p)
    assert rc == -1 and "multiple of 64" in msg
    p.K, p.lda, p.ldw = 128, 128, 128
    p.N = 40
    rc, msg = _rc_msg(lib.wanb200_gemm_bf16, p)
    assert rc == -1 and "multiple of 32" in msg
    p.N, p.ldd = 64, 64
    p.a = 24  # not 16-byte aligned
    rc, msg = _rc_msg(lib.wanb200_gemm_bf16, p)
    assert rc == -1 and "aligned" in msg
    p.a = 32
    p.epilogue = L.EPI_BIAS  # bias missing
    rc, msg = _rc_msg(lib.wanb200_gemm_bf16, p)
    assert rc == -1 and "bias" in msg
    p.epilogue = 9
    rc, msg = _rc_msg(lib.wanb200_gemm_bf16, p)
    assert rc == -1 and "epilogue" in msg
    p.epilogue, p.bias, p.residual_f32 = L.EPI_BIAS, 48, 1  # an fp32 residual is for the residual epilogues
    rc, msg = _rc_msg(lib.wanb200_gemm_bf16, p)
    assert rc == -1 and "residual_f32" in msg
    p.epilogue, p.residual_f32, p.out_f32 = L.EPI_BIAS_SUMSQ, 0, 1
    rc, msg = _rc_msg(lib.wanb200_gemm_bf16, p)
    assert rc == -1 and "out_f32" in msg


def test_attn_rejects_bad_args_on_host():
    lib = L.load()
    p = L.AttnParams()
    p.q = p.k = p.v = p.o = 256
    for f in ("q_tok_stride", "k_tok_stride", "v_tok_stride", "o_tok_stride"):
        setattr(p, f, 384)
    for f in ("q_batch_stride", "k_batch_stride", "v_batch_stride", "o_batch_stride"):
        setattr(p, f, 384 * 100)
    p.batch, p.heads, p.q_len, p.kv_len, p.head_dim, p.softmax_scale = 2, 3, 100, 100, 64, 0.1
    rc, msg = _rc_msg(lib.wanb200_attn_fwd, p)
    assert rc == -1 and "head_dim" in msg
    p.head_dim = 128
    p.kv_len = 0
    rc, msg = _rc_msg(lib.wanb200_attn_fwd, p)
    assert rc == -1 and "positive" in msg
    p.kv_len = 100
    p.k_tok_stride = 100  # not a multiple of 8
    rc, msg = _rc_msg(lib.wanb200_attn_fwd, p)
    assert rc == -1 and "strides" in msg
    p.k_tok_stride = 256  # smaller than heads * 128
    rc, msg = _rc_msg(lib.wanb200_attn_fwd, p)
    assert rc == -1 and "token stride" in msg


def test_layernorm_and_qknorm_reject_bad_args_on_host():
    lib = L.load()
    p = L.LnParams()
    p.x = p.out = 64
    p.rows, p.dim, p.mode = 4, 300, L.LN_MODULATE
    rc, msg = _rc_msg(lib.wanb200_layernorm, p)
    assert rc == -1 and "multiple of 256" in msg
    p.dim = 512
    rc, msg = _rc_msg(lib.wanb200_layernorm, p)
    assert rc == -1 and "modulate" in msg
    q = L.QkNormParams()
    q.x, q.ld, q.rows, q.width, q.nsections = 64, 384, 4, 100, 1
    rc, msg = _rc_msg(lib.wanb200_qk_norm_rope, q)
    assert rc == -1 and "width" in msg
    # more partial sums per row than the row has threads to add them
    q.width, q.ld = 256, 256
    q.ss[0], q.gamma[0] = 64, 64
    q.ss_parts, q.ss_row_stride = 64, 64
    rc, msg = _rc_msg(lib.wanb200_qk_norm_rope, q)
    assert rc == -1 and "ss_parts" in msg
    q.ss_parts, q.ss_row_stride = 8, 4  # a row's partials would overlap the next row's
    rc, msg = _rc_msg(lib.wanb200_qk_norm_rope, q)
    assert rc == -1 and "ss_row_stride" in msg
    s = L.SumsqReduceParams()
    s.part, s.out, s.rows, s.row_stride, s.nsections, s.parts, s.out_stride = 64, 64, 4, 4, 3, 2, 4
    rc, msg = _rc_msg(lib.wanb200_sumsq_reduce, s)
    assert rc == -1 and "nsections" in msg
    s.nsections, s.out_stride = 2, 3
    rc, msg = _rc_msg(lib.wanb200_sumsq_reduce, s)
    assert rc == -1 and "out_stride" in msg
    s.out_stride, s.part0[1] = 4, 3  # 3 + 2 partials > row stride 4
    rc, msg = _rc_msg(lib.wanb200_sumsq_reduce, s)
    assert rc == -1 and "row_stride" in msg
    r = L.ResidualParams()
    r.out = r.residual = r.y = r.bias = 64
    r.rows, r.dim = 4, 12
    rc, msg = _rc_msg(lib.wanb200_bias_gate_residual, r)
    assert rc == -1 and "dim % 8" in msg


def test_frame_index_and_shard_gather_reject_bad_args_on_host():
    lib = L.load()
    r = L.ResidualParams()
    r.out = r.residual = r.y = r.bias = r.gate_mod = r.gate_e0 = 64
    r.rows, r.dim, r.seq_len, r.tokens_per_frame = 4, 16, 8, 2
    r.rows_per_seq = -1
    rc, msg = _rc_msg(lib.wanb200_bias_gate_residual, r)
    assert rc == -1 and "rows_per_seq" in msg
    g = L.ShardGatherParams()
    g.src, g.src_ld, g.batch, g.shard_rows, g.valid_rows, g.width = 64, 256, 2, 10, 10, 256
    g.dst[0], g.ndst, g.dst_ld, g.dst_batch_stride = 128, 1, 256, 256 * 40
    g.valid_rows = 11  # more valid rows than the shard holds
    rc, msg = _rc_msg(lib.wanb200_shard_gather, g)
    assert rc == -1 and "valid_rows" in msg
    g.valid_rows, g.width = 10, 250
    rc, msg = _rc_msg(lib.wanb200_shard_gather, g)
    assert rc == -1 and "width % 8" in msg
    g.width, g.ndst = 256, 9
    rc, msg = _rc_msg(lib.wanb200_shard_gather, g)
    assert rc == -1 and "ndst" in msg
    g.ndst, g.dst_batch_stride = 1, 256 * 5  # batch 1 would overwrite batch 0's rows
    rc, msg = _rc_msg(lib.wanb200_shard_gather, g)
    assert rc == -1 and "dst_batch_stride" in msg
    g.dst_batch_stride, g.dst[0] = 256 * 40, 72  # destination not 16-byte aligned
    rc, msg = _rc_msg(lib.wanb200_shard_gather, g)
    assert rc == -1 and "aligned" in msg


def test_ops_refuse_cpu_tensors():
    import torch
    from wanb200 import ops
    a = torch.zeros(128, 128, dtype=torch.bfloat16)
    with pytest.raises(L.WanB200Error):
        ops.linear(a, a, None, epilogue=L.EPI_NONE)


def test_block_forward_rejects_bad_args_on_host():
    lib = L.load()
    p = L.BlockParams()
    rc, msg = _rc_msg(lib.wanb200_block_forward, p)
    assert rc == -1 and "dim % 512" in msg
    p.batch, p.seq_len, p.dim, p.local_heads, p.ffn_local, p.num_frames = 2, 1080, 3072, 24, 14336, 6
    p.ctx_len, p.ckv_tok_stride, p.ckv_batch_stride, p.tp_size = 512, 3072, 512 * 3072, 1
    rc, msg = _rc_msg(lib.wanb200_block_forward, p)
    assert rc == -1 and "distinct" in msg
    p.x, p.x_out = 256, 256
    rc, msg = _rc_msg(lib.wanb200_block_forward, p)
    assert rc == -1 and "distinct" in msg
    p.x_out, p.e0, p.cos, p.sin, p.ck, p.cv = 512, 1024, 1024, 1024, 1024, 1024
    rc, msg = _rc_msg(lib.wanb200_block_forward, p)
    assert rc == -1 and "weight pointer" in msg
    for f, _ in L.BlockWeightsC._fields_:
        setattr(p.w, f, 4096)
    rc, msg = _rc_msg(lib.wanb200_block_forward, p)
    assert rc == -1 and "workspace" in msg
    p.local_heads, p.tp_size = 12, 2  # TP without the all-reduce callback
    rc, msg = _rc_msg(lib.wanb200_block_forward, p)
    assert rc == -1 and "all_reduce callback" in msg
    p.local_heads = 10  # heads * 128 * tp != dim
    rc, msg = _rc_msg(lib.wanb200_block_forward, p)
    assert rc == -1 and "local_heads" in msg
    assert lib.wanb200_block_workspace_bytes(2, 1080, 3072, 24, 14336, 512, 1) > 2 * 1080 * 3072 * 4
    assert lib.wanb200_block_workspace_bytes(0, 1080, 3072, 24, 14336, 512, 1) == 0
