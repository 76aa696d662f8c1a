"""b200kern — B200-native (sm_100a) hot-path kernels behind the operator
surface of bledden/triton-metal's INT4/INT8 matmul, FlashAttention and GQA
templates, plus a KDA chunked forward.

Ops take and return CUDA torch tensors; all compute is in libb2.so.
"""
from .errors import (B2Error, B2ShapeError, B2DtypeError, B2AlignmentError,
                     B2UnsupportedError, B2LaunchError, B2TimeoutError)
from .quant import (int4_matmul, int8_matmul, int4_dequant, gemm_bf16, pack_int4_gptq,
                    unpack_int4_gptq, pack_int4_ref)
from .attention import (flash_attention, flash_attention_template, gqa_attention, decode_attention,
                        kv_cache_attention, batched_kv_decode, paged_attention, sliding_window_attention,
                        rope_attention, repeat_kv)
from .kda import kda_chunk_fwd
from . import _lib

__all__ = [
    "int4_matmul", "int8_matmul", "gemm_bf16", "flash_attention", "flash_attention_template",
    "gqa_attention", "decode_attention", "kv_cache_attention", "batched_kv_decode",
    "paged_attention", "sliding_window_attention", "rope_attention", "repeat_kv", "kda_chunk_fwd", "int4_dequant", "pack_int4_gptq", "unpack_int4_gptq",
    "pack_int4_ref", "B2Error", "B2ShapeError", "B2DtypeError", "B2AlignmentError",
    "B2UnsupportedError", "B2LaunchError", "B2TimeoutError", "load_library",
]


def load_library():
    """Load libb2.so (raises B2Error if it is not built)."""
    return _lib.load()
