"""The allocation-free attention entry point (wanb200_attn_fwd_noalloc), called through the C ABI.

It exists for callers that cannot let a library allocate device memory (an application that has
given all GPU memory to its own pool, or a latency-critical loop that must not pay for cudaMalloc
/ cudaFree).  Its split-KV partials live in a fixed 16 MiB array inside the library that every
call on a device shares, so the tests make two calls in a row with different inputs and check
each against fp32 SDPA (the attention tolerance of the other kernel tests) and, bit for bit,
against the regular entry point (wanb200_attn_fwd with a torch-allocated workspace and the same
split count: the same kernels in the same order, so stale partials in the shared array would
show).  A fresh process that calls only this entry point checks that, once the first call has
loaded the library's kernels, later calls leave the device's free memory unchanged.  A shape
whose partials exceed the fixed array is refused.

This file sorts last so that a run stopping at the first failure has run everything else first;
it passes alone in a fresh process as well.
"""
import ctypes
import math

import pytest
import torch

from wanb200 import _lib as L
from wanb200 import ops

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = 1e-2  # relative RMS, as for the other attention tests


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def randn(*shape, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(*shape, generator=g, device=DEV).to(torch.bfloat16)


def params(q, k, v, o, splits):
    p = L.AttnParams()
    p.q, p.q_tok_stride, p.q_batch_stride = q.data_ptr(), q.stride(1), q.stride(0)
    p.k, p.k_tok_stride, p.k_batch_stride = k.data_ptr(), k.stride(1), k.stride(0)
    p.v, p.v_tok_stride, p.v_batch_stride = v.data_ptr(), v.stride(1), v.stride(0)
    p.o, p.o_tok_stride, p.o_batch_stride = o.data_ptr(), o.stride(1), o.stride(0)
    p.batch, p.heads, p.q_len, p.kv_len, p.head_dim = q.shape[0], q.shape[2], q.shape[1], k.shape[1], 128
    p.softmax_scale = 1.0 / math.sqrt(128)
    p.kv_splits = splits
    return p


def call_noalloc(q, k, v, splits):
    lib = L.load()
    o = torch.empty_like(q)
    p = params(q, k, v, o, splits)
    rc = lib.wanb200_attn_fwd_noalloc(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    L.check(rc, "wanb200_attn_fwd_noalloc")
    return o


def sdpa(q, k, v):
    return torch.nn.functional.scaled_dot_product_attention(
        q.float().transpose(1, 2), k.float().transpose(1, 2), v.float().transpose(1, 2)).transpose(1, 2)


def test_noalloc_attention_matches_sdpa_and_regular_entry_point_twice():
    B, H, Lq, Lk, splits = 1, 6, 1000, 7854, 3  # partials 9.4 MB: inside the 16 MiB array
    for call, seed in enumerate((100, 200)):  # second call: new inputs, the shared array is stale
        q, k, v = randn(B, Lq, H, 128, seed=seed), randn(B, Lk, H, 128, seed=seed + 1), randn(B, Lk, H, 128,
                                                                                              seed=seed + 2)
        o_free = call_noalloc(q, k, v, splits)
        o_ref = ops.attention(q, k, v, kv_splits=splits)
        torch.cuda.synchronize()
        err = rel(o_free, sdpa(q, k, v))
        assert err < TOL, (call, err)
        assert torch.equal(o_free, o_ref), call
    assert L.device_error(reset=True) == 0


def test_noalloc_attention_without_split_and_cross_shape():
    q, kv = randn(2, 300, 4, 128, seed=7), randn(2, 512, 4, 128, seed=8)
    o_free = call_noalloc(q, kv, kv, 1)
    o_ref = ops.attention(q, kv, kv, kv_splits=1)
    torch.cuda.synchronize()
    assert rel(o_free, sdpa(q, kv, kv)) < TOL
    assert torch.equal(o_free, o_ref)


_CHILD = r"""
import ctypes, math, sys
import torch
sys.path[:0] = sys.argv[1:3]
from wanb200 import _lib as L
lib = L.load()
dev = "cuda"
g = torch.Generator(device=dev).manual_seed(5)
q, k, v = (torch.randn(1, n, 6, 128, generator=g, device=dev).to(torch.bfloat16) for n in (1000, 7854, 7854))
outs = [torch.empty_like(q) for _ in range(4)]
ref = torch.nn.functional.scaled_dot_product_attention(
    q.float().transpose(1, 2), k.float().transpose(1, 2), v.float().transpose(1, 2)).transpose(1, 2)
torch.cuda.synchronize()
def call(o):
    p = L.AttnParams()
    p.q, p.q_tok_stride, p.q_batch_stride = q.data_ptr(), q.stride(1), q.stride(0)
    p.k, p.k_tok_stride, p.k_batch_stride = k.data_ptr(), k.stride(1), k.stride(0)
    p.v, p.v_tok_stride, p.v_batch_stride = v.data_ptr(), v.stride(1), v.stride(0)
    p.o, p.o_tok_stride, p.o_batch_stride = o.data_ptr(), o.stride(1), o.stride(0)
    p.batch, p.heads, p.q_len, p.kv_len, p.head_dim = 1, 6, 1000, 7854, 128
    p.softmax_scale, p.kv_splits = 1.0 / math.sqrt(128), 3
    L.check(lib.wanb200_attn_fwd_noalloc(ctypes.byref(p), torch.cuda.current_stream().cuda_stream), "noalloc")
call(outs[0])  # the first call loads the library's kernels and resolves the static array
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for o in outs[1:]:
    call(o)
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
assert lib.wanb200_device_error(0) == 0
for o in outs:
    err = float((o.double() - ref.double()).norm() / ref.double().norm())
    assert err < 1e-2, err
    assert torch.equal(o, outs[0])
print("free", free0, free1)
assert free1 == free0, (free0, free1)
print("OK")
"""


def test_noalloc_alone_in_a_fresh_process_allocates_nothing_after_its_first_call():
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    r = subprocess.run([sys.executable, "-c", _CHILD, root, os.path.join(root, "wan2-ti2v-5b_b200")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr


def test_noalloc_attention_rejects_partials_beyond_the_fixed_array():
    lib = L.load()
    q, kv = randn(1, 7854, 24, 128, seed=9), randn(1, 1024, 24, 128, seed=10)  # 2 splits: 196 MB of partials
    o = torch.empty_like(q)
    p = params(q, kv, kv, o, 2)
    rc = lib.wanb200_attn_fwd_noalloc(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    assert rc == L_EINVAL
    assert "16 MiB" in lib.wanb200_last_error().decode()


L_EINVAL = -1
