"""Hot ops of the serving path: sm_100a kernels for CUDA tensors, PyTorch restatements (the test oracles) on CPU."""
from .attention import (DecodeWorkspace, decode_attention, prefill_attention, prefill_tile_rows, prefill_tiles,
                        varlen_attention)
from .embedding import embed, vq_embed
from .gemm import grouped_linear, linear
from .moe import MoEWorkspace, fused_moe, route, tp_moe
from .norm import layer_norm, rms_norm
from .rope import qkv_rope_store, rope_half_inplace, rope_tables
from .sampling import SamplingTensors, sample

__all__ = [
    "DecodeWorkspace", "decode_attention", "prefill_attention", "prefill_tile_rows", "prefill_tiles", "varlen_attention", "embed", "vq_embed",
    "grouped_linear", "linear", "MoEWorkspace", "fused_moe", "route", "tp_moe", "layer_norm", "rms_norm", "qkv_rope_store", "rope_half_inplace",
    "rope_tables", "SamplingTensors", "sample",
]
