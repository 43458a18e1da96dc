"""ctypes binding of libwanb200.so (the C ABI declared in include/wanb200.h).

The library is loaded from this directory only; there is no fallback implementation.  If it
is missing or a CUDA device is absent, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libwanb200.so")

c_void_p, c_int64, c_int, c_float = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
c_float_p = ctypes.POINTER(ctypes.c_float)

EPI_NONE, EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_GATE_RES, EPI_BIAS_RES, EPI_BIAS_SUMSQ, EPI_SCATTER, EPI_BIAS_SILU = range(8)
MAX_PEERS = 8
LN_MODULATE, LN_AFFINE = 0, 1


class GemmParams(ctypes.Structure):
    _fields_ = [("a", c_void_p), ("lda", c_int64), ("w", c_void_p), ("ldw", c_int64), ("d", c_void_p),
                ("ldd", c_int64), ("M", c_int64), ("N", c_int64), ("K", c_int64), ("epilogue", c_int),
                ("bias", c_void_p), ("residual", c_void_p), ("ldr", c_int64), ("gate_mod", c_void_p),
                ("gate_e0", c_void_p), ("gate_frame_stride", c_int64), ("seq_len", c_int64),
                ("tokens_per_frame", c_int64), ("row_offset", c_int64), ("rows_per_seq", c_int64), ("rowss", c_void_p),
                ("ss_cols", c_int64), ("peer_out", c_void_p * 8), ("npeers", c_int), ("src_rank", c_int),
                ("shard_rows", c_int64), ("tile_n", c_int), ("residual_f32", c_int), ("out_f32", c_int)]


class AttnParams(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("q_tok_stride", c_int64), ("q_batch_stride", c_int64),
                ("k", c_void_p), ("k_tok_stride", c_int64), ("k_batch_stride", c_int64),
                ("v", c_void_p), ("v_tok_stride", c_int64), ("v_batch_stride", c_int64),
                ("o", c_void_p), ("o_tok_stride", c_int64), ("o_batch_stride", c_int64),
                ("batch", c_int64), ("heads", c_int64), ("q_len", c_int64), ("kv_len", c_int64),
                ("head_dim", c_int64), ("softmax_scale", c_float), ("kv_splits", c_int), ("workspace", c_void_p),
                ("workspace_bytes", c_int64), ("part_slot0", c_int), ("part_nslots", c_int), ("defer_combine", c_int)]


class LnParams(ctypes.Structure):
    _fields_ = [("x", c_void_p), ("out", c_void_p), ("rows", c_int64), ("dim", c_int64), ("eps", c_float),
                ("mode", c_int), ("modulation", c_void_p), ("e0", c_void_p), ("e0_frame_stride", c_int64),
                ("shift_idx", c_int), ("scale_idx", c_int), ("seq_len", c_int64), ("tokens_per_frame", c_int64),
                ("row_offset", c_int64), ("rows_per_seq", c_int64),
                ("weight", c_void_p), ("bias", c_void_p),
                ("push_out", c_void_p * 8), ("npush", c_int), ("push_row0", c_int64), ("x_f32", c_int),
                ("e0_one_row", c_int)]


class QkNormParams(ctypes.Structure):
    _fields_ = [("x", c_void_p), ("ld", c_int64), ("rows", c_int64), ("nsections", c_int),
                ("col0", c_int64 * 2), ("width", c_int64), ("ss", c_void_p * 2), ("gamma", c_void_p * 2),
                ("ss_parts", c_int), ("ss_row_stride", c_int64), ("inv_dim", c_float), ("eps", c_float), ("rope", c_int), ("cos", c_void_p), ("sin", c_void_p),
                ("seq_len", c_int64)]


class SumsqReduceParams(ctypes.Structure):
    _fields_ = [("part", c_void_p), ("rows", c_int64), ("row_stride", c_int64), ("nsections", c_int),
                ("part0", c_int64 * 2), ("parts", c_int), ("out", c_void_p), ("out_stride", c_int64)]


class ResidualParams(ctypes.Structure):
    _fields_ = [("out", c_void_p), ("residual", c_void_p), ("y", c_void_p), ("rows", c_int64), ("dim", c_int64),
                ("bias", c_void_p), ("gate_mod", c_void_p), ("gate_e0", c_void_p), ("gate_frame_stride", c_int64),
                ("seq_len", c_int64), ("tokens_per_frame", c_int64), ("row_offset", c_int64), ("rows_per_seq", c_int64),
                ("nsum", c_int),
                ("y_slice_stride", c_int64), ("residual_f32", c_int), ("out_f32", c_int)]


class ShardGatherParams(ctypes.Structure):
    _fields_ = [("src", c_void_p), ("src_ld", c_int64), ("batch", c_int64), ("shard_rows", c_int64),
                ("valid_rows", c_int64), ("width", c_int64), ("dst", c_void_p * 8), ("ndst", c_int),
                ("dst_ld", c_int64), ("dst_batch_stride", c_int64), ("dst_row0", c_int64 * 8)]


class AttnFp8Params(ctypes.Structure):
    _fields_ = [("attn", AttnParams), ("fp8_workspace", c_void_p), ("fp8_workspace_bytes", c_int64)]


class PatchifyParams(ctypes.Structure):
    _fields_ = [("latent", c_void_p), ("latent_f32", c_int), ("channels", c_int64), ("frames", c_int64),
                ("height", c_int64), ("width", c_int64), ("pf", c_int), ("ph", c_int), ("pw", c_int),
                ("batch", c_int64), ("out", c_void_p)]


CFG_COMBINE, CFG_SCALE = 0, 1


class UnpatchifyParams(ctypes.Structure):
    _fields_ = [("y", c_void_p), ("batch", c_int64), ("frames", c_int64), ("height", c_int64), ("width", c_int64),
                ("pf", c_int), ("ph", c_int), ("pw", c_int), ("channels", c_int64), ("mode", c_int),
                ("guide", c_float), ("out", c_void_p), ("out_f32", c_int)]


class BlockWeightsC(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("modulation", "w_qkv", "b_qkv", "g_q", "g_k", "w_o", "b_o", "ln3_w",
                                        "ln3_b", "w_cq", "b_cq", "g_cq", "w_co", "b_co", "w1", "b1", "w2", "b2")]


ALLREDUCE_FN = ctypes.CFUNCTYPE(c_int, c_void_p, c_int64, c_int, c_void_p, c_void_p)


class BlockParams(ctypes.Structure):
    _fields_ = [("x", c_void_p), ("x_f32", c_int), ("x_out", c_void_p), ("out_f32", c_int), ("batch", c_int64),
                ("seq_len", c_int64), ("dim", c_int64), ("local_heads", c_int64), ("ffn_local", c_int64),
                ("num_frames", c_int64), ("eps", c_float), ("e0", c_void_p), ("cos", c_void_p), ("sin", c_void_p),
                ("ck", c_void_p), ("cv", c_void_p), ("ctx_len", c_int64), ("ckv_tok_stride", c_int64),
                ("ckv_batch_stride", c_int64), ("w", BlockWeightsC), ("workspace", c_void_p),
                ("workspace_bytes", c_int64), ("tp_size", c_int), ("all_reduce", ALLREDUCE_FN),
                ("all_reduce_ctx", c_void_p)]


EXPORTS = ("wanb200_gemm_bf16", "wanb200_attn_fwd", "wanb200_layernorm", "wanb200_qk_norm_rope",
           "wanb200_bias_gate_residual", "wanb200_last_error", "wanb200_device_error", "wanb200_version",
           "wanb200_struct_sizes", "wanb200_peer_barrier", "wanb200_attn_workspace_bytes",
           "wanb200_attn_kv_splits", "wanb200_attn_fwd_noalloc", "wanb200_shard_gather", "wanb200_attn_fwd_fp8",
           "wanb200_attn_fp8_workspace_bytes", "wanb200_device_error_async", "wanb200_block_forward",
           "wanb200_block_workspace_bytes", "wanb200_patchify", "wanb200_unpatchify_cfg", "wanb200_sumsq_reduce")

_lock = threading.Lock()
_lib = None


class WanB200Error(RuntimeError):
    pass


def load():
    """Load (once) and return the ctypes handle; raises if the library was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise WanB200Error(f"{LIB_PATH} is missing: build it with `python wan2-ti2v-5b_b200/build.py` "
                                   "(there is no fallback implementation)")
            lib = ctypes.CDLL(LIB_PATH)
            lib.wanb200_gemm_bf16.argtypes = [ctypes.POINTER(GemmParams), c_void_p]
            lib.wanb200_attn_fwd.argtypes = [ctypes.POINTER(AttnParams), c_void_p]
            lib.wanb200_layernorm.argtypes = [ctypes.POINTER(LnParams), c_void_p]
            lib.wanb200_qk_norm_rope.argtypes = [ctypes.POINTER(QkNormParams), c_void_p]
            lib.wanb200_bias_gate_residual.argtypes = [ctypes.POINTER(ResidualParams), c_void_p]
            lib.wanb200_shard_gather.argtypes = [ctypes.POINTER(ShardGatherParams), c_void_p]
            for fn in ("wanb200_gemm_bf16", "wanb200_attn_fwd", "wanb200_layernorm", "wanb200_qk_norm_rope",
                       "wanb200_bias_gate_residual", "wanb200_shard_gather"):
                getattr(lib, fn).restype = c_int
            lib.wanb200_last_error.restype = ctypes.c_char_p
            lib.wanb200_last_error.argtypes = []
            lib.wanb200_device_error.argtypes = [c_int]
            lib.wanb200_device_error.restype = c_int
            lib.wanb200_device_error_async.argtypes = [c_void_p, c_void_p]
            lib.wanb200_device_error_async.restype = c_int
            lib.wanb200_version.restype = c_int
            lib.wanb200_struct_sizes.argtypes = [ctypes.POINTER(c_int64), c_int]
            lib.wanb200_struct_sizes.restype = c_int
            lib.wanb200_peer_barrier.argtypes = [ctypes.POINTER(c_void_p), c_int, c_int, c_int, c_void_p]
            lib.wanb200_peer_barrier.restype = c_int
            lib.wanb200_attn_workspace_bytes.argtypes = [c_int64, c_int64, c_int64, c_int]
            lib.wanb200_attn_workspace_bytes.restype = c_int64
            lib.wanb200_attn_kv_splits.argtypes = [c_int64, c_int64, c_int64, c_int64]
            lib.wanb200_attn_kv_splits.restype = c_int
            lib.wanb200_attn_fwd_noalloc.argtypes = [ctypes.POINTER(AttnParams), c_void_p]
            lib.wanb200_attn_fwd_noalloc.restype = c_int
            lib.wanb200_attn_fwd_fp8.argtypes = [ctypes.POINTER(AttnFp8Params), c_void_p]
            lib.wanb200_attn_fwd_fp8.restype = c_int
            lib.wanb200_attn_fp8_workspace_bytes.argtypes = [c_int64, c_int64, c_int64, c_int64]
            lib.wanb200_attn_fp8_workspace_bytes.restype = c_int64
            lib.wanb200_block_forward.argtypes = [ctypes.POINTER(BlockParams), c_void_p]
            lib.wanb200_block_forward.restype = c_int
            lib.wanb200_block_workspace_bytes.argtypes = [c_int64] * 6 + [c_int]
            lib.wanb200_block_workspace_bytes.restype = c_int64
            lib.wanb200_patchify.argtypes = [ctypes.POINTER(PatchifyParams), c_void_p]
            lib.wanb200_patchify.restype = c_int
            lib.wanb200_unpatchify_cfg.argtypes = [ctypes.POINTER(UnpatchifyParams), c_void_p]
            lib.wanb200_unpatchify_cfg.restype = c_int
            lib.wanb200_sumsq_reduce.argtypes = [ctypes.POINTER(SumsqReduceParams), c_void_p]
            lib.wanb200_sumsq_reduce.restype = c_int
            structs = (GemmParams, AttnParams, LnParams, QkNormParams, ResidualParams, ShardGatherParams,
                       AttnFp8Params, BlockParams, PatchifyParams, UnpatchifyParams, SumsqReduceParams)
            sizes = (c_int64 * len(structs))()
            n = lib.wanb200_struct_sizes(sizes, len(structs))
            want = [ctypes.sizeof(c) for c in structs]
            if n != len(structs) or list(sizes) != want:
                raise WanB200Error(f"{LIB_PATH} was built from a different include/wanb200.h (struct sizes "
                                   f"{list(sizes)} vs {want}); rebuild it with `python wan2-ti2v-5b_b200/build.py`")
            _lib = lib
    return _lib


def check(rc: int, what: str):
    if rc != 0:
        msg = load().wanb200_last_error().decode(errors="replace")
        raise WanB200Error(f"{what} failed ({rc}): {msg}")


def device_error(reset: bool = False) -> int:
    """Device-side error word of the current device (synchronizes)."""
    v = load().wanb200_device_error(1 if reset else 0)
    if v < 0:
        check(v, "wanb200_device_error")
    return v


class DeviceErrorProbe:
    """Reads a device's error word behind the work queued on a stream, without synchronizing.

    `post(stream)` queues a copy of the word into page-locked host memory
    (wanb200_device_error_async) and records an event after it; `poll()` returns the value of
    the last copy that has landed (0 while none has); `wait(stream)` queues a fresh copy and
    blocks for it.  The word is sticky (the first expiry stays until reset), so a copy taken at
    any later point reports an earlier expiry: a step driver that posts once per step and polls
    at the start of the next one sees every expiry at most a step or two late, at no cost to the
    pipeline.  While a copy is still in flight, `post` leaves it be and queues nothing.
    """

    def __init__(self, device):
        import torch
        self._torch = torch
        self.device = torch.device(device)
        self._buf = None  # page-locked int32, made on the first post (construction needs no GPU)
        self._event = None
        self._seen = 0

    def post(self, stream=None):
        t = self._torch
        if self._event is not None and not self._event.query():
            return
        if self._event is not None:
            self._seen = int(self._buf[0])
        if self._buf is None:
            self._buf = t.zeros(1, dtype=t.int32).pin_memory()
        st = stream if stream is not None else t.cuda.current_stream(self.device)
        check(load().wanb200_device_error_async(self._buf.data_ptr(), st.cuda_stream), "wanb200_device_error_async")
        self._event = t.cuda.Event()
        self._event.record(st)

    def poll(self) -> int:
        if self._event is not None and self._event.query():
            self._seen = int(self._buf[0])
        return self._seen

    def wait(self, stream=None) -> int:
        if self._event is not None:
            self._event.synchronize()
        self._event = None
        self.post(stream)
        self._event.synchronize()
        self._seen = int(self._buf[0])
        return self._seen


def raise_on_device_error(code: int, where: str):
    """Raise WanB200Error for a non-zero device error word (a bounded wait inside a kernel gave up,
    so the outputs of that launch are incomplete)."""
    if code:
        raise WanB200Error(f"{where}: device error word {code} (a bounded wait expired inside a kernel; the "
                           "results since the last check are not valid; wanb200.device_error(reset=True) clears it)")
