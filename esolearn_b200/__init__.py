"""esolearn_b200: B200-native int8 Llama decode for scry-llm (Slush97/esolearn).

The numeric path lives in libscryb200.so (hand-written sm_100a CUDA behind the
C ABI in include/sb_api.h); this package is the host-side mirror of the
reference's model / generation API.
"""
from . import _native
from .llama import (B200Backend, I8Storage, LlamaConfig, LlamaKvCacheHandle, QuantLinear, QuantLlamaB200, QWeight, RopeScaling, Rng,
                    SamplingConfig, argmax_last, generate, generate_batch, matmul_i8_f32, quantize_symmetric, sample_rows, sample_token,
                    tp_shard_qweight, tp_shard_shape, tp_unique_id)

__all__ = [
    "B200Backend", "I8Storage", "LlamaConfig", "RopeScaling", "QuantLlamaB200", "QuantLinear", "LlamaKvCacheHandle", "QWeight", "SamplingConfig", "Rng",
    "generate", "generate_batch", "sample_token", "sample_rows", "argmax_last", "matmul_i8_f32", "quantize_symmetric", "tp_unique_id",
    "tp_shard_qweight", "tp_shard_shape", "_native",
]
