"""ctypes binding of libqwen_b200.so (the C ABI in include/qwen_b200.h).

The library is built in-tree (``python -m llm_inference_edu_b200.build``).
There is no fallback: if the shared object is missing or fails to load,
importing the package's compute entry points raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwen_b200.so")

# Every symbol declared in include/qwen_b200.h with its ctypes signature.
P, S, U32, U64, I32, F = C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint64, C.c_int32, C.c_float
SIGNATURES = {
    "qb_abi_version": ([], U32),
    "qb_status_name": ([U32], C.c_char_p),
    "qb_last_detail": ([P], None),
    "qb_last_cuda_error": ([], C.c_int),
    "qb_linear_f32": ([P, S, P, S, P, S, S, S, S, P], U32),
    "qb_linear_lanes4_f32": ([P, S, P, S, P, S, S, S, S, P], U32),
    "qb_linear_bf16": ([P, S, P, S, P, S, S, S, S, P], U32),
    "qb_quantize_int8": ([P, S, S, S, S, P, P, P], U32),
    "qb_dequantize_int8": ([P, P, S, S, S, P, S, P], U32),
    "qb_linear_int8": ([P, S, P, P, S, S, S, P, S, S, P], U32),
    "qb_linear_int8_lanes4": ([P, S, P, P, S, S, S, P, S, S, P], U32),
    "qb_embedding": ([P, S, P, S, P, S, S, S, P], U32),
    "qb_residual_add": ([P, S, P, S, P, S, P], U32),
    "qb_rmsnorm": ([P, S, P, S, P, S, S, S, F, P], U32),
    "qb_silu": ([P, S, P, S, P], U32),
    "qb_softmax": ([P, S, P, S, P, S, S, S, P], U32),
    "qb_rope": ([P, S, P, S, S, S, S, S, F, P], U32),
    "qb_rope_static": ([P, S, P, S, S, S, S, S, F, P], U32),
    "qb_model_create": ([P, U32, U32, C.c_int, P], U32),
    "qb_model_set_tensor": ([U64, C.c_int64, U32, U32, P, S], U32),
    "qb_model_finalize": ([U64], U32),
    "qb_model_logical_weight_bytes": ([U64, P], U32),
    "qb_model_read_int8": ([U64, C.c_int64, U32, P, S, P, S], U32),
    "qb_model_free": ([U64], U32),
    "qb_session_create": ([U64, S, U32, S, P], U32),
    "qb_session_step": ([U64, U32, P, S, P], U32),
    "qb_session_append": ([U64, P, S, P, S, P, I32], U32),
    "qb_session_step_profiled": ([U64, U32, P, S, P, P, S, P], U32),
    "qb_session_step_withheld": ([U64, U32, U64], U32),
    "qb_session_reset": ([U64], U32),
    "qb_session_info_get": ([U64, P], U32),
    "qb_session_decode_greedy": ([U64, U32, S, P], U32),
    "qb_session_stream": ([U64, P], U32),
    "qb_session_free": ([U64], U32),
    "qb_generation_create": ([U64, S, P, S, S, U32, S, P], U32),
    "qb_generation_create_sampled": ([U64, S, P, P, S, S, U32, S, P], U32),
    "qb_tokenizer_from_json": ([P, S, P], U32),
    "qb_tokenizer_load_chat": ([P, S, P, S, P, S, P], U32),
    "qb_tokenizer_encode": ([U64, P, S, P, S, P], U32),
    "qb_tokenizer_decode": ([U64, P, S, I32, P, S, P], U32),
    "qb_tokenizer_stop_tokens": ([U64, P, S, P], U32),
    "qb_tokenizer_free": ([U64], U32),
    "qb_tokenizer_stream_create": ([U64, P], U32),
    "qb_tokenizer_stream_push": ([U64, U32, P, S, P, P], U32),
    "qb_tokenizer_stream_pending": ([U64, P], U32),
    "qb_tokenizer_stream_free": ([U64], U32),
    "qb_render_chat": ([P, P, P, S, I32, P, S, P], U32),
    "qb_sampler_create": ([P, I32, P], U32),
    "qb_sampler_validate_vocab": ([U64, S], U32),
    "qb_sampler_reset": ([U64], U32),
    "qb_sampler_sample": ([U64, P, S, P], U32),
    "qb_sampler_sample_device": ([U64, P, S, P], U32),
    "qb_sampler_free": ([U64], U32),
    "qb_generation_start": ([U64, P, S, P], U32),
    "qb_generation_next_token": ([U64, P, P, P], U32),
    "qb_generation_append_context": ([U64, P, S, S, P], U32),
    "qb_generation_replay_history": ([U64, P, S, S, P], U32),
    "qb_generation_reset": ([U64], U32),
    "qb_generation_info_get": ([U64, P], U32),
    "qb_generation_history": ([U64, P, S, P], U32),
    "qb_generation_prefix_logits": ([U64, P, S], U32),
    "qb_generation_free": ([U64], U32),
    "qb_batch_create": ([U64, S, S, U32, P], U32),
    "qb_batch_prefill": ([U64, P, S, P], U32),
    "qb_batch_decode_greedy": ([U64, P, S, P], U32),
    "qb_batch_logits": ([U64, P, S], U32),
    "qb_batch_info_get": ([U64, P], U32),
    "qb_batch_reset": ([U64], U32),
    "qb_batch_stream": ([U64, P], U32),
    "qb_batch_free": ([U64], U32),
    "qb_model_create_tp": ([P, U32, U32, C.c_int, C.c_int, C.c_int, P], U32),
    "qb_model_tp_info": ([U64, P], U32),
    "qb_tp_shard_of": ([P, C.c_int, C.c_int, P], U32),
    "qb_tp_comm_create": ([C.c_int, S, S, P], U32),
    "qb_tp_comm_handle": ([U64, P, S], U32),
    "qb_tp_comm_connect": ([U64, C.c_int, C.c_int, P, S], U32),
    "qb_tp_comm_free": ([U64], U32),
    "qb_batch_create_tp": ([U64, U64, S, S, U32, P], U32),
    "qb_qwen_tensor_count": ([P, P], U32),
    "qb_safetensors_inspect": ([P, S, P, P], U32),
    "qb_model_load_safetensors": ([P, S, P, U32, U32, C.c_int, P], U32),
    "qb_synthetic_normal": ([U64, U64, S, C.c_double, U32, P], U32),
    "qb_synthetic_tokens": ([U64, U64, S, U32, P], U32),
}

_lib = None


def lib():
    """Loads the library (building it first when this checkout has none)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            from . import build
            build.build()
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in list(SIGNATURES.items()) + list(BRIDGE_SIGNATURES.items()):
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


class Detail(C.Structure):
    _fields_ = [("buffer", S), ("expected", S), ("actual", S), ("index", S)]


class ModelConfigC(C.Structure):
    _fields_ = [(n, S) for n in ("vocab_size", "layers", "hidden_dim", "query_heads", "kv_heads",
                                 "head_dim", "ff_dim", "max_tokens")] + \
               [("rope_base", F), ("norm_epsilon", F)]


class SessionInfo(C.Structure):
    _fields_ = [("processed", S), ("capacity", S), ("logical_bytes", S), ("workspace_bytes", S),
                ("valid", I32)]


class GenerationInfo(C.Structure):
    _fields_ = [("processed", S), ("history_len", S), ("generated", S), ("max_new", S),
                ("stop_reason", I32), ("valid", I32), ("logits_ready", I32)]


class BatchInfo(C.Structure):
    _fields_ = [("sequences", S), ("capacity", S), ("processed", S), ("valid", I32)]


class QwenConfigC(C.Structure):
    _fields_ = [("model_type", C.c_char_p), ("hidden_act", C.c_char_p), ("torch_dtype", C.c_char_p),
                ("architectures", C.POINTER(C.c_char_p)), ("architectures_count", S)] + \
               [(n, S) for n in ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                                 "num_attention_heads", "num_key_value_heads", "max_position_embeddings")] + \
               [("rms_norm_eps", F), ("rope_theta", F), ("tie_word_embeddings", I32),
                ("use_sliding_window", I32), ("has_rope_scaling", I32)]


# The poll bridge (include/qwen_b200_bridge.h), the reference Apple host's
# aie_* names.
BRIDGE_SIGNATURES = {
    "aie_abi_version": ([], U32),
    "aie_open": ([U32, P, S, P], U32),
    "aie_begin_ids": ([U64, P, S, U32], U32),
    "aie_begin_text": ([U64, P, S, U32], U32),
    "aie_next": ([U64], U32),
    "aie_reset": ([U64], U32),
    "aie_set_cancel": ([U64, U32], U32),
    "aie_poll": ([U64, P], U32),
    "aie_poll_text": ([U64, P, P, S, P], U32),
    "aie_close": ([U64], U32),
}


class AieEvent(C.Structure):
    _fields_ = [(n, U32) for n in ("kind", "code", "token", "processed", "history")]


class SamplingC(C.Structure):
    _fields_ = [("kind", U32), ("temperature", C.c_float), ("top_k", C.c_uint64), ("seed", C.c_uint64)]


class TpShard(C.Structure):
    _fields_ = [("rank", I32), ("size", I32)] + [(n, S) for n in ("head0", "heads", "kv_head0", "kv_heads",
                                                                    "ff0", "ff", "vocab0", "vocab")]
