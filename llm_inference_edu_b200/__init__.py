"""B200 (sm_100a) implementation of the reference crate's Qwen2 token loop.

The compute path is the CUDA library ``libqwen_b200.so`` built from
``csrc/`` (see ``build.py``) behind the C ABI in ``include/qwen_b200.h``;
this package is the Python mirror of the crate's API over that ABI.
"""
from .presets import ModelConfig, qwen_0_5b, qwen_7b, tiny_b, tiny_r, tiny_r_weights  # noqa: F401
from .api import (  # noqa: F401
    BatchSession, CacheError, CachedSession, CancelFlag, Decoder, GenerationSession, GroupwiseInt8, LoadError,
    TpComm, inspect_safetensors, qwen_tensor_count,
    LinearError, ModelError, OpError, QbError, QuantError, RopeError, Sampler, Sampling, SamplingError,
    StateError, Temperature, Role, TextStream, Tokenizer, TokenizerError, render_chat,
    embedding, linear, linear_int8, linear_int8_lanes4, linear_lanes4, masked_softmax,
    residual_add, rmsnorm, rope, silu, softmax, tp_shard_of)
from . import synthetic  # noqa: F401
