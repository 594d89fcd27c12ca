from .conv import causal_conv1d, conv_qkv, kda_forward_decode, kda_forward_extend
from .kda import (
    kda_varlen_chunk,
    kda_varlen_chunk_g,
    kda_varlen_chunk_v2,
    kda_varlen_recurrent,
    kda_varlen_recurrent_g,
    kda_varlen_recurrent_v2,
    move_intermediate_cache_kda,
    prepared_recurrent,
)

__all__ = [
    "causal_conv1d",
    "conv_qkv",
    "kda_forward_decode",
    "kda_forward_extend",
    "kda_varlen_chunk",
    "kda_varlen_chunk_g",
    "kda_varlen_chunk_v2",
    "kda_varlen_recurrent",
    "kda_varlen_recurrent_g",
    "kda_varlen_recurrent_v2",
    "move_intermediate_cache_kda",
    "prepared_recurrent",
]
