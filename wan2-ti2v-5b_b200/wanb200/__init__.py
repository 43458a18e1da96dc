"""wanb200: the Wan2.2-TI2V-5B DiT block forward on B200 (sm_100a) kernels.

Host side of libwanb200.so (C ABI: include/wanb200.h).  Public surface mirrors the
reference's `models/fast_dit.py`: `FastBlock` (= `_FastBlock`, with `sp=` the Q-local
sequence-parallel block of `WanSelfAttentionSP`), `FastBlockSP` (= `_FastBlockSP`),
`FastCrossKV` (= `_FastCrossKV`), `FastWanDiT`; the device-side sampler and denoise loop
(`FlowUniPC`, `denoise`); the checkpoint reader (`load_wan_checkpoint`,
`FastWanDiT.from_checkpoint`); process-group layouts in `wanb200.parallel`; kernel ops in
`wanb200.ops`.
"""
from ._lib import LIB_PATH, WanB200Error, device_error, load  # noqa: F401
from .block import FastBlock, FastBlockSP, FastCrossKV  # noqa: F401
from .checkpoint import load_wan_checkpoint, save_wan_checkpoint  # noqa: F401
from .dit import CapturedStep, FastWanDiT, block_flops, rope_tables  # noqa: F401
from .unipc import FlowUniPC, denoise  # noqa: F401
from .weights import TI2V_5B, BlockWeights, WanSpec, random_block_state, random_model_state  # noqa: F401

__version__ = "0.1.0"
