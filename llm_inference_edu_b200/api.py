"""Python mirror of the reference crate's token-loop API over the C ABI.

Names, argument meaning and error behaviour follow the Rust crate
(pshevskiy/llm_inference_edu):

  linear / linear_lanes4        src/lib.rs:51, src/kernels.rs:10
  GroupwiseInt8, linear_int8    src/quantization.rs:27-281
  embedding, residual_add, rmsnorm, silu, softmax, masked_softmax
                                src/ops.rs:67-257
  rope                          src/rope.rs:38
  Decoder                       src/model.rs:59-340
  CachedSession                 src/kv_cache.rs:156-475
  GenerationSession, Sampling   src/generation.rs:98-338, src/sampling.rs

Operator entry points take CUDA tensors (device buffers) and write into a
caller-owned output, with the reference's validate-before-write rule.
Errors raise ``QbError`` subclasses named after the Rust error enums; the
``kind`` attribute carries the variant name (``"InvalidLength"``, ...).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import lib
from .presets import ModelConfig

# ----------------------------------------------------------------- errors --

STATUS_NAMES = [
    "Ok", "ZeroDimension", "DimensionOverflow", "InvalidLength", "InvalidGroupSize",
    "InvalidShape", "NonFiniteWeight", "UnrepresentableScale", "Allocation", "InvalidToken",
    "InvalidEpsilon", "NonFinite", "AllMasked", "OddHeadDimension", "PositionOverflow",
    "PositionOutOfRange", "InvalidBase", "InvalidAngle", "InvalidCapacity", "ResourceBudget",
    "InvalidOutputLength", "EmptyInput", "NotEmpty", "Full", "InvalidState", "InvalidConfig",
    "InvalidHandle", "InvalidParameters", "NotStarted", "AlreadyStarted", "Cancelled",
    "EmptyLogits", "CudaError", "DeviceTimeout", "ContextLimit", "TraceLimit", "EmptyPrompt",
    "OutputLimit", "InvalidLayerCount", "Unsupported", "Format", "UnsupportedConfig", "MissingTensor",
    "UnexpectedTensor", "InvalidDtype", "Json", "Encoding", "UnsupportedAssets", "EmptyMessages",
    "InvalidToken", "InvalidStream"]


class QbError(Exception):
    """A non-zero status from the library."""

    def __init__(self, status: int, detail: Optional[_lib.Detail] = None):
        self.status = int(status)
        self.kind = STATUS_NAMES[status] if status < len(STATUS_NAMES) else f"Status{status}"
        self.buffer = detail.buffer if detail else None
        self.expected = detail.expected if detail else None
        self.actual = detail.actual if detail else None
        self.index = detail.index if detail else None
        extra = ""
        if self.kind == "CudaError":
            extra = f" (cuda error {lib().qb_last_cuda_error()})"
        super().__init__(f"{type(self).__name__}::{self.kind}{extra}")


class LinearError(QbError):
    pass


class QuantError(QbError):
    pass


class OpError(QbError):
    pass


class RopeError(QbError):
    pass


class ModelError(QbError):
    pass


class CacheError(QbError):
    pass


class StateError(QbError):
    pass


def _check(status: int, cls=QbError):
    if status:
        d = _lib.Detail()
        lib().qb_last_detail(C.byref(d))
        raise cls(status, d)


def _ptr(t):
    """Device pointer of a CUDA tensor (None passes NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("operator buffers must be CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("operator buffers must be contiguous")
    return C.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        import torch
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return C.c_void_p(int(stream))


# ------------------------------------------------------------ operators --

def linear(x, w, y, tokens: int, input_dim: int, output_dim: int, stream=None):
    """Y = X W^T with FP32 accumulation (src/lib.rs:51-73); BF16 weights
    (torch.bfloat16 / int16 bit patterns) select the BF16 kernel."""
    import torch
    if w.dtype in (torch.bfloat16, torch.int16, torch.uint16):
        f = lib().qb_linear_bf16
    else:
        f = lib().qb_linear_f32
    _check(f(_ptr(x), x.numel(), _ptr(w), w.numel(), _ptr(y), y.numel(), tokens, input_dim,
             output_dim, _stream(stream)), LinearError)


def linear_lanes4(x, w, y, tokens: int, input_dim: int, output_dim: int, stream=None):
    """Same contract as `linear` (src/kernels.rs:10-28)."""
    _check(lib().qb_linear_lanes4_f32(_ptr(x), x.numel(), _ptr(w), w.numel(), _ptr(y), y.numel(),
                                      tokens, input_dim, output_dim, _stream(stream)), LinearError)


class GroupwiseInt8:
    """Device INT8 weights + FP32 scales (src/quantization.rs:27-166).

    group_size is 1..=256 as in the reference, or equal to input_dim for one
    absmax scale per output row."""

    def __init__(self, values, scales, output_dim, input_dim, group_size):
        self.values, self.scales = values, scales
        self._out, self._in, self._group = output_dim, input_dim, group_size

    @classmethod
    def quantize(cls, weights, output_dim: int, input_dim: int, group_size: int, stream=None):
        import torch
        gpr = -(-input_dim // group_size) if group_size else 0
        n = output_dim * input_dim if output_dim and input_dim else 0
        dev = weights.device if weights.is_cuda else torch.device("cuda")
        values = torch.empty(max(n, 1), dtype=torch.int8, device=dev)
        scales = torch.empty(max(output_dim * gpr, 1), dtype=torch.float32, device=dev)
        _check(lib().qb_quantize_int8(_ptr(weights), weights.numel(), output_dim, input_dim,
                                      group_size, _ptr(values), _ptr(scales), _stream(stream)),
               QuantError)
        return cls(values, scales, output_dim, input_dim, group_size)

    def output_dim(self):
        return self._out

    def input_dim(self):
        return self._in

    def group_size(self):
        return self._group

    def groups_per_row(self):
        return -(-self._in // self._group)

    def logical_bytes(self):
        return self._out * self._in + 4 * self._out * self.groups_per_row()

    def dequantize(self, output, stream=None):
        _check(lib().qb_dequantize_int8(_ptr(self.values), _ptr(self.scales), self._out, self._in,
                                        self._group, _ptr(output), output.numel(), _stream(stream)),
               QuantError)


def linear_int8(x, weights: GroupwiseInt8, y, tokens: int, stream=None):
    """Fused dequantizing linear (src/quantization.rs:168-215)."""
    _check(lib().qb_linear_int8(_ptr(x), x.numel(), _ptr(weights.values), _ptr(weights.scales),
                                weights._out, weights._in, weights._group, _ptr(y), y.numel(),
                                tokens, _stream(stream)), QuantError)


def linear_int8_lanes4(x, weights: GroupwiseInt8, y, tokens: int, stream=None):
    """Fused dequantizing linear in the four-lane order (src/quantization.rs:218-281)."""
    _check(lib().qb_linear_int8_lanes4(_ptr(x), x.numel(), _ptr(weights.values), _ptr(weights.scales),
                                       weights._out, weights._in, weights._group, _ptr(y), y.numel(),
                                       tokens, _stream(stream)), QuantError)


def embedding(token_ids: Sequence[int], table, y, vocab_size: int, width: int, stream=None):
    ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.uint64))
    if ids.size and int(ids.max()) >= 2**32:
        ids32 = np.full(ids.size, 0xFFFFFFFF, dtype=np.uint32)
    else:
        ids32 = ids.astype(np.uint32)
    _check(lib().qb_embedding(ids32.ctypes.data_as(C.c_void_p), ids32.size, _ptr(table),
                              table.numel(), _ptr(y), y.numel(), vocab_size, width,
                              _stream(stream)), OpError)


def residual_add(x, residual, y, stream=None):
    _check(lib().qb_residual_add(_ptr(x), x.numel(), _ptr(residual), residual.numel(), _ptr(y),
                                 y.numel(), _stream(stream)), OpError)


def rmsnorm(x, weight, y, rows: int, width: int, epsilon: float, stream=None):
    _check(lib().qb_rmsnorm(_ptr(x), x.numel(), _ptr(weight), weight.numel(), _ptr(y), y.numel(),
                            rows, width, epsilon, _stream(stream)), OpError)


def silu(x, y, stream=None):
    _check(lib().qb_silu(_ptr(x), x.numel(), _ptr(y), y.numel(), _stream(stream)), OpError)


def softmax(logits, y, rows: int, width: int, stream=None):
    _check(lib().qb_softmax(_ptr(logits), logits.numel(), None, 0, _ptr(y), y.numel(), rows, width,
                            _stream(stream)), OpError)


def masked_softmax(logits, mask, y, rows: int, width: int, stream=None):
    _check(lib().qb_softmax(_ptr(logits), logits.numel(), _ptr(mask), mask.numel(), _ptr(y),
                            y.numel(), rows, width, _stream(stream)), OpError)


def rope(x, y, tokens: int, heads: int, head_dim: int, start_position: int, base: float,
         stream=None):
    _check(lib().qb_rope(_ptr(x), x.numel(), _ptr(y), y.numel(), tokens, heads, head_dim,
                         start_position, base, _stream(stream)), RopeError)


# ---------------------------------------------------------------- model --

LINEAR_FORMATS = {"f32": 0, "bf16": 1, "int8": 2}
TABLE_FORMATS = {"f32": 0, "bf16": 1}
_T = {"embedding": 0, "lm_head": 1, "final_norm": 2, "attn_norm": 3, "q": 4, "k": 5, "v": 6,
      "o": 7, "q_bias": 8, "k_bias": 9, "v_bias": 10, "ffn_norm": 11, "gate": 12, "up": 13,
      "down": 14}


class Decoder:
    """A device-resident model (src/model.rs:59-340).

    ``weights`` is the host weight dictionary of ``synthetic.weights`` /
    ``presets.tiny_r_weights``: matrices are float32 arrays or uint16 BF16
    bit patterns.  ``linear_format`` stores the seven per-layer linears as
    "f32", "bf16" or "int8" (per-row absmax, quantized on the device with the
    reference's encode); ``table_format`` stores the embedding/LM-head table
    as "f32" or "bf16"."""

    def __init__(self, config: ModelConfig, weights: dict, linear_format: str = "f32",
                 table_format: str = "f32", device: int = 0, tp=None):
        """tp = (rank, size): this process's tensor-parallel shard (the full
        weight dictionary is passed on every rank; see ``shard``)."""
        self.config = config
        self.linear_format = linear_format
        self.table_format = table_format
        c = _lib.ModelConfigC(config.vocab_size, config.layers, config.hidden_dim,
                              config.query_heads, config.kv_heads, config.head_dim, config.ff_dim,
                              config.max_tokens, config.rope_base, config.norm_epsilon)
        h = C.c_uint64()
        if tp is None:
            _check(lib().qb_model_create(C.byref(c), LINEAR_FORMATS[linear_format],
                                         TABLE_FORMATS[table_format], device, C.byref(h)), ModelError)
        else:
            _check(lib().qb_model_create_tp(C.byref(c), LINEAR_FORMATS[linear_format],
                                            TABLE_FORMATS[table_format], device, int(tp[0]), int(tp[1]),
                                            C.byref(h)), ModelError)
        self.handle = h.value
        self.device = device
        try:
            self._set(-1, "embedding", weights["embedding"])
            if weights.get("lm_head") is not None:
                self._set(-1, "lm_head", weights["lm_head"])
            self._set(-1, "final_norm", weights["final_norm"])
            for i, layer in enumerate(weights["layers"]):
                for k, v in layer.items():
                    if v is not None:
                        self._set(i, k, v)
            _check(lib().qb_model_finalize(self.handle), ModelError)
        except Exception:
            lib().qb_model_free(self.handle)
            self.handle = None
            raise

    def _set(self, layer, name, arr):
        a = np.ascontiguousarray(arr)
        if a.dtype == np.uint16:
            dt = 1
        else:
            a = np.ascontiguousarray(a, dtype=np.float32)
            dt = 0
        _check(lib().qb_model_set_tensor(self.handle, layer, _T[name], dt,
                                         a.ctypes.data_as(C.c_void_p), a.size), ModelError)

    def __del__(self):
        if getattr(self, "handle", None):
            lib().qb_model_free(self.handle)
            self.handle = None

    @classmethod
    def from_safetensors(cls, data: bytes, config: dict, linear_format: str = "f32",
                         table_format: str = "f32", device: int = 0) -> "Decoder":
        """decode_qwen (src/weights.rs:226-264) into a device model: the
        validated BF16 checkpoint in `data` with its HF config.json
        dictionary (tied head; max_tokens = max_position_embeddings)."""
        c, _a, _s = _qwen_config(config)
        h = C.c_uint64()
        buf = C.create_string_buffer(bytes(data), len(data)) if data else None
        _check(lib().qb_model_load_safetensors(buf, len(data), C.byref(c), LINEAR_FORMATS[linear_format],
                                               TABLE_FORMATS[table_format], device, C.byref(h)), LoadError)
        self = cls.__new__(cls)
        self.handle = h.value
        self.device = device
        self.linear_format = linear_format
        self.table_format = table_format
        from .presets import ModelConfig
        hd = config["hidden_size"] // config["num_attention_heads"]
        self.config = ModelConfig(config["vocab_size"], config["num_hidden_layers"], config["hidden_size"],
                                  config["num_attention_heads"], config["num_key_value_heads"], hd,
                                  config["intermediate_size"], config["max_position_embeddings"],
                                  float(config["rope_theta"]), float(config["rms_norm_eps"]), True, True)
        return self

    def shard(self) -> dict:
        """This model's tensor-parallel shard: rank, size and the half-open
        ranges of query heads, KV heads, FFN columns and LM-head rows."""
        i = _lib.TpShard()
        _check(lib().qb_model_tp_info(self.handle, C.byref(i)), ModelError)
        return _shard_dict(i)

    def logical_weight_bytes(self) -> int:
        n = C.c_size_t()
        _check(lib().qb_model_logical_weight_bytes(self.handle, C.byref(n)), ModelError)
        return n.value

    def read_int8(self, layer: int, name: str):
        """Device INT8 values [rows, cols] and row scales of one linear."""
        c = self.config
        rows, cols = {"q": (c.hidden_dim, c.hidden_dim), "k": (c.kv_dim, c.hidden_dim),
                      "v": (c.kv_dim, c.hidden_dim), "o": (c.hidden_dim, c.hidden_dim),
                      "gate": (c.ff_dim, c.hidden_dim), "up": (c.ff_dim, c.hidden_dim),
                      "down": (c.hidden_dim, c.ff_dim)}[name]
        v = np.zeros(rows * cols, dtype=np.int8)
        s = np.zeros(rows, dtype=np.float32)
        _check(lib().qb_model_read_int8(self.handle, layer, _T[name], v.ctypes.data_as(C.c_void_p),
                                        v.size, s.ctypes.data_as(C.c_void_p), s.size), ModelError)
        return v.reshape(rows, cols), s


# -------------------------------------------------------------- session --

KV_DTYPES = {"f32": 0, "bf16": 1}
REFERENCE_BUDGET = 128 * 1024 * 1024


class CachedSession:
    """KV-cached decoding state bound to one Decoder (src/kv_cache.rs:156-475).

    ``budget`` bounds logical KV + workspace bytes like the reference's fixed
    128 MiB (src/kv_cache.rs:184-190); pass 0 for no bound."""

    def __init__(self, model: Decoder, capacity: int, kv_dtype: str = "f32",
                 budget: int = REFERENCE_BUDGET):
        self.model = model
        h = C.c_uint64()
        _check(lib().qb_session_create(model.handle, capacity, KV_DTYPES[kv_dtype], budget,
                                       C.byref(h)), CacheError)
        self.handle = h.value
        self.vocab = model.config.vocab_size

    def __del__(self):
        if getattr(self, "handle", None):
            lib().qb_session_free(self.handle)
            self.handle = None

    def _info(self):
        i = _lib.SessionInfo()
        _check(lib().qb_session_info_get(self.handle, C.byref(i)), CacheError)
        return i

    def processed(self) -> int:
        return self._info().processed

    def capacity(self) -> int:
        return self._info().capacity

    def is_valid(self) -> bool:
        return bool(self._info().valid)

    def logical_bytes(self) -> int:
        return self._info().logical_bytes

    def workspace_bytes(self) -> int:
        return self._info().workspace_bytes

    def reset(self):
        _check(lib().qb_session_reset(self.handle), CacheError)

    def step_withheld(self, token: int, timeout_ns: int) -> None:
        """Fault-path test hook (no counterpart in the reference): one step in
        which the first CTA withholds its first-layer QKV outputs, so the
        polls waiting for them run out after `timeout_ns`.  Raises
        CacheError("DeviceTimeout") and leaves the session invalid until
        reset()."""
        _check(lib().qb_session_step_withheld(self.handle, token, timeout_ns), CacheError)

    def step_into(self, token: int, logits: Optional[np.ndarray]) -> int:
        """Evaluates one token; fills `logits` (float32, vocab width) if given
        and returns the greedy id."""
        am = C.c_uint32()
        if token < 0 or token >= 2**32:
            raise CacheError(9)
        lp = None if logits is None else logits.ctypes.data_as(C.c_void_p)
        _check(lib().qb_session_step(self.handle, token, lp, 0 if logits is None else logits.size,
                                     C.byref(am)), CacheError)
        return am.value

    def step(self, token: int) -> np.ndarray:
        logits = np.zeros(self.vocab, dtype=np.float32)
        self.step_into(token, logits)
        return logits

    def append_into(self, tokens: Sequence[int], logits: Optional[np.ndarray],
                    require_empty: bool = False) -> int:
        ids = np.ascontiguousarray(np.asarray(list(tokens), dtype=np.int64))
        if ids.size and (ids.min() < 0 or ids.max() >= 2**32):
            raise CacheError(9)
        ids = ids.astype(np.uint32)
        am = C.c_uint32()
        lp = None if logits is None else logits.ctypes.data_as(C.c_void_p)
        _check(lib().qb_session_append(self.handle, ids.ctypes.data_as(C.c_void_p) if ids.size else None,
                                       ids.size, lp, 0 if logits is None else logits.size,
                                       C.byref(am), int(require_empty)), CacheError)
        return am.value

    def prefill_into(self, tokens, logits) -> int:
        return self.append_into(tokens, logits, True)

    def append(self, tokens) -> np.ndarray:
        logits = np.zeros(self.vocab, dtype=np.float32)
        self.append_into(tokens, logits)
        return logits

    def prefill(self, tokens) -> np.ndarray:
        logits = np.zeros(self.vocab, dtype=np.float32)
        self.append_into(tokens, logits, True)
        return logits

    def step_profiled(self, token: int):
        """One step with device timestamps (src/kv_cache.rs:309-316).

        Returns (logits, profile).  profile["layers"][l] holds, for each of
        the phases "qkv", "attention", "gate_up", "down": wall ns from the
        moment CTA 0 held this phase's inputs to the moment it held the next
        phase's ("ns"), the slowest CTA's work ("slowest_ns"), the mean CTA's
        work ("mean_ns") and the hand-over latency from the last CTA's finish
        to CTA 0 holding its next inputs ("barrier_ns"; negative when CTA 0's
        inputs did not wait for the last CTA).  Per CTA: "ready_ns" (mean
        over the CTAs of the time from the phase's start to holding its
        inputs), "compute_ns" (mean time from holding the inputs to the
        finish) and "last_ready_ns" (the latest CTA to hold its inputs)."""
        need = C.c_size_t()
        lib().qb_session_step_profiled(self.handle, 0, None, 0, None, None, 0, C.byref(need))
        stamps = np.zeros(need.value, dtype=np.uint64)
        logits = np.zeros(self.vocab, dtype=np.float32)
        am = C.c_uint32()
        _check(lib().qb_session_step_profiled(self.handle, token, logits.ctypes.data_as(C.c_void_p),
                                              logits.size, C.byref(am),
                                              stamps.ctypes.data_as(C.c_void_p), stamps.size,
                                              C.byref(need)), CacheError)
        L = self.model.config.layers
        nb = 4 * L
        grid = (stamps.size - 2) // (2 * nb)
        fin = stamps[:nb * grid].reshape(nb, grid).astype(np.int64)
        rdy = stamps[nb * grid:2 * nb * grid].reshape(nb, grid).astype(np.int64)
        start, end = int(stamps[-2]), int(stamps[-1])
        names = ["qkv", "attention", "gate_up", "down"]
        layers, prev = [], start
        for l in range(L):
            d = {}
            for k, name in enumerate(names):
                i = 4 * l + k
                # inputs of phase i are the outputs of phase i - 1
                r = rdy[i - 1] if i > 0 else np.full(grid, start, dtype=np.int64)
                act = r > 0
                rel = int(rdy[i, 0])
                d[name] = {"ns": int(rel - prev), "slowest_ns": int(fin[i].max() - prev),
                           "mean_ns": float(fin[i].mean() - prev),
                           "barrier_ns": int(rel - fin[i].max()),
                           "ready_ns": float((r[act] - prev).mean()) if act.any() else 0.0,
                           "last_ready_ns": float((r[act] - prev).max()) if act.any() else 0.0,
                           "compute_ns": float((fin[i][act] - r[act]).mean()) if act.any() else 0.0}
                prev = rel
            layers.append(d)
        profile = {"layers": layers, "logits_ns": end - prev, "total_ns": end - start, "argmax": am.value,
                   "finish": fin, "ready": rdy, "start": start, "end": end}
        return logits, profile

    def decode_greedy(self, token: int, steps: int) -> list:
        """`steps` greedy steps on the device, each fed its own argmax."""
        out = np.zeros(steps, dtype=np.uint32)
        _check(lib().qb_session_decode_greedy(self.handle, token, steps,
                                              out.ctypes.data_as(C.c_void_p)), CacheError)
        return [int(v) for v in out]

    def stream(self) -> int:
        p = C.c_void_p()
        _check(lib().qb_session_stream(self.handle, C.byref(p)), CacheError)
        return p.value or 0


# ---------------------------------------------------------------- batch --

# ------------------------------------------------------- checkpoints --

def _qwen_config(config: dict):
    """A HF config.json dictionary as the library's qb_qwen_config (the
    QwenConfig fields of src/weights.rs:9-28); the returned tuple keeps the
    strings alive."""
    archs = [a.encode() for a in config.get("architectures", [])]
    arr = (C.c_char_p * max(1, len(archs)))(*archs)
    c = _lib.QwenConfigC(
        str(config.get("model_type", "")).encode(), str(config.get("hidden_act", "")).encode(),
        str(config.get("torch_dtype", "")).encode(), arr, len(archs),
        int(config.get("vocab_size", 0)), int(config.get("hidden_size", 0)),
        int(config.get("intermediate_size", 0)), int(config.get("num_hidden_layers", 0)),
        int(config.get("num_attention_heads", 0)), int(config.get("num_key_value_heads", 0)),
        int(config.get("max_position_embeddings", 0)), float(config.get("rms_norm_eps", 0.0)),
        float(config.get("rope_theta", 0.0)), int(bool(config.get("tie_word_embeddings", False))),
        int(bool(config.get("use_sliding_window", False))), int(config.get("rope_scaling") is not None))
    return c, arr, archs


class LoadError(QbError):
    """LoadError (src/weights.rs:72-88): Format, UnsupportedConfig,
    MissingTensor, UnexpectedTensor, InvalidShape, InvalidDtype, NonFinite,
    DimensionOverflow, ResourceBudget, Allocation."""


def qwen_tensor_count(config: dict) -> int:
    """tensor_shapes (src/weights.rs:96-187): the config's expected tensor
    count after its checks."""
    c, _a, _s = _qwen_config(config)
    n = C.c_size_t()
    _check(lib().qb_qwen_tensor_count(C.byref(c), C.byref(n)), LoadError)
    return n.value


def inspect_safetensors(data: bytes, config: dict) -> int:
    """inspect_qwen (src/weights.rs:189-221): the number of validated
    tensors of a safetensors file."""
    c, _a, _s = _qwen_config(config)
    n = C.c_size_t()
    buf = C.create_string_buffer(bytes(data), len(data)) if data else None
    _check(lib().qb_safetensors_inspect(buf, len(data), C.byref(c), C.byref(n)), LoadError)
    return n.value


def _shard_dict(i) -> dict:
    return {"rank": i.rank, "size": i.size, "heads": (i.head0, i.head0 + i.heads),
            "kv_heads": (i.kv_head0, i.kv_head0 + i.kv_heads), "ff": (i.ff0, i.ff0 + i.ff),
            "vocab": (i.vocab0, i.vocab0 + i.vocab)}


def tp_shard_of(config: ModelConfig, rank: int, size: int) -> dict:
    """The tensor-parallel shard rank `rank` of `size` holds (host only)."""
    c = _lib.ModelConfigC(config.vocab_size, config.layers, config.hidden_dim, config.query_heads,
                          config.kv_heads, config.head_dim, config.ff_dim, config.max_tokens,
                          config.rope_base, config.norm_epsilon)
    i = _lib.TpShard()
    _check(lib().qb_tp_shard_of(C.byref(c), rank, size, C.byref(i)), ModelError)
    return _shard_dict(i)


class TpComm:
    """A rank's tensor-parallel communicator (no reference counterpart):
    its exchange buffer, opened by the other ranks through CUDA IPC.
    ``exchange(handles)`` receives every rank's ``handle()`` in rank order
    (gathered over any host channel, e.g. torch.distributed)."""

    def __init__(self, device: int, rows: int, hidden: int):
        h = C.c_uint64()
        _check(lib().qb_tp_comm_create(device, rows, hidden, C.byref(h)), CacheError)
        self.handle_id = h.value

    def handle(self) -> bytes:
        buf = (C.c_uint8 * 64)()
        _check(lib().qb_tp_comm_handle(self.handle_id, buf, 64), CacheError)
        return bytes(buf)

    def connect(self, rank: int, handles) -> None:
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        _check(lib().qb_tp_comm_connect(self.handle_id, rank, len(handles), buf, len(blob)), CacheError)

    def __del__(self):
        if getattr(self, "handle_id", None):
            lib().qb_tp_comm_free(self.handle_id)
            self.handle_id = None


class BatchSession:
    """`sequences` independent sequences decoded greedily in lockstep, each
    with its own KV cache of `capacity` positions.  No counterpart in the
    reference (one sequence per CachedSession); each row matches a
    CachedSession fed the same tokens.  With a tensor-parallel shard, pass
    its connected ``comm``; ids are global and ``logits`` holds this rank's
    vocabulary rows."""

    def __init__(self, model: Decoder, sequences: int, capacity: int, kv_dtype: str = "f32", comm=None):
        self.model = model
        self.comm = comm
        h = C.c_uint64()
        if comm is None:
            _check(lib().qb_batch_create(model.handle, sequences, capacity, KV_DTYPES[kv_dtype],
                                         C.byref(h)), CacheError)
        else:
            _check(lib().qb_batch_create_tp(model.handle, comm.handle_id, sequences, capacity,
                                            KV_DTYPES[kv_dtype], C.byref(h)), CacheError)
        self.handle = h.value
        self.sequences = sequences
        if comm is None:
            self.vocab = model.config.vocab_size
        else:
            v0, v1 = model.shard()["vocab"]
            self.vocab = v1 - v0

    def __del__(self):
        if getattr(self, "handle", None):
            lib().qb_batch_free(self.handle)
            self.handle = None

    def _info(self):
        i = _lib.BatchInfo()
        _check(lib().qb_batch_info_get(self.handle, C.byref(i)), CacheError)
        return i

    def processed(self) -> int:
        return self._info().processed

    def capacity(self) -> int:
        return self._info().capacity

    def is_valid(self) -> bool:
        return bool(self._info().valid)

    def reset(self):
        _check(lib().qb_batch_reset(self.handle), CacheError)

    def prefill(self, prompts) -> np.ndarray:
        """prompts [sequences][prompt_len]; returns each row's greedy id after
        its last prompt token."""
        p = np.ascontiguousarray(np.asarray(prompts, dtype=np.uint32))
        if p.ndim != 2 or p.shape[0] != self.sequences:
            raise ValueError(f"prompts must be [{self.sequences}][prompt_len]")
        out = np.zeros(self.sequences, dtype=np.uint32)
        _check(lib().qb_batch_prefill(self.handle, p.ctypes.data_as(C.c_void_p) if p.size else None,
                                      p.shape[1], out.ctypes.data_as(C.c_void_p)), CacheError)
        return out

    def decode_greedy(self, tokens, steps: int) -> np.ndarray:
        """Feeds tokens [sequences], then each row's greedy id; returns the
        greedy ids [steps][sequences]."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        if t.shape != (self.sequences,):
            raise ValueError(f"tokens must be [{self.sequences}]")
        out = np.zeros((steps, self.sequences), dtype=np.uint32)
        _check(lib().qb_batch_decode_greedy(self.handle, t.ctypes.data_as(C.c_void_p), steps,
                                            out.ctypes.data_as(C.c_void_p)), CacheError)
        return out

    def logits(self) -> np.ndarray:
        out = np.zeros((self.sequences, self.vocab), dtype=np.float32)
        _check(lib().qb_batch_logits(self.handle, out.ctypes.data_as(C.c_void_p), out.size), CacheError)
        return out

    def stream(self) -> int:
        p = C.c_void_p()
        _check(lib().qb_batch_stream(self.handle, C.byref(p)), CacheError)
        return p.value or 0


# ----------------------------------------------------------- generation --

class TokenizerError(QbError):
    """TokenizerError (src/tokenizer.rs:27-35): Json, Encoding,
    UnsupportedAssets, EmptyMessages, InvalidToken (the id in .actual),
    InvalidStream."""


class Role:
    """src/tokenizer.rs:8-22."""
    System, User, Assistant = 0, 1, 2


def _out_text(call, cap=1 << 16):
    """Calls call(buf, cap, len_ptr) and grows the buffer once if needed."""
    n = C.c_size_t()
    buf = C.create_string_buffer(cap)
    st = call(buf, cap, C.byref(n))
    if st == 20 and n.value > cap:  # InvalidOutputLength: retry with the reported size
        cap = n.value
        buf = C.create_string_buffer(cap)
        st = call(buf, cap, C.byref(n))
    _check(st, TokenizerError)
    return buf.raw[:n.value].decode("utf-8")


def render_chat(messages, generation_prompt: bool) -> str:
    """render_chat (src/tokenizer.rs:40-63): messages as (Role, content)."""
    n = len(messages)
    roles = (C.c_uint32 * max(n, 1))(*[r for r, _ in messages])
    data = [c.encode() for _, c in messages]
    ptrs = (C.c_char_p * max(n, 1))(*data)
    lens = (C.c_size_t * max(n, 1))(*[len(d) for d in data])
    return _out_text(lambda buf, cap, ln: lib().qb_render_chat(roles, ptrs, lens, n, int(generation_prompt),
                                                                buf, cap, ln))


class Tokenizer:
    """ChatTokenizer (src/tokenizer.rs:64-166) over the host tokenizer of
    the library: ``Tokenizer.load(directory)`` with the reference's checks,
    or ``Tokenizer.from_json(bytes)`` for a bare tokenizer.json."""

    def __init__(self, handle):
        self.handle = handle

    @classmethod
    def from_json(cls, data: bytes) -> "Tokenizer":
        h = C.c_uint64()
        _check(lib().qb_tokenizer_from_json(data, len(data), C.byref(h)), TokenizerError)
        return cls(h.value)

    @classmethod
    def load_files(cls, tokenizer_json: bytes, tokenizer_config: bytes, generation_config: bytes) -> "Tokenizer":
        h = C.c_uint64()
        _check(lib().qb_tokenizer_load_chat(tokenizer_json, len(tokenizer_json), tokenizer_config,
                                            len(tokenizer_config), generation_config, len(generation_config),
                                            C.byref(h)), TokenizerError)
        return cls(h.value)

    @classmethod
    def load(cls, directory) -> "Tokenizer":
        import os
        read = lambda n: open(os.path.join(directory, n), "rb").read()
        return cls.load_files(read("tokenizer.json"), read("tokenizer_config.json"),
                              read("generation_config.json"))

    def __del__(self):
        if getattr(self, "handle", None):
            lib().qb_tokenizer_free(self.handle)
            self.handle = None

    def encode(self, text: str) -> list:
        b = text.encode("utf-8")
        n = C.c_size_t()
        _check(lib().qb_tokenizer_encode(self.handle, b, len(b), None, 0, C.byref(n)) if not b else 0,
               TokenizerError)
        cap = max(1, 2 * len(b) + 8)
        out = (C.c_uint32 * cap)()
        _check(lib().qb_tokenizer_encode(self.handle, b, len(b), out, cap, C.byref(n)), TokenizerError)
        return list(out[:n.value])

    def chat(self, messages, generation_prompt: bool) -> list:
        return self.encode(render_chat(messages, generation_prompt))

    def decode(self, ids, skip_special: bool) -> str:
        a = (C.c_uint32 * max(len(ids), 1))(*ids)
        return _out_text(lambda buf, cap, ln: lib().qb_tokenizer_decode(self.handle, a, len(ids),
                                                                         int(skip_special), buf, cap, ln))

    def stop_tokens(self) -> list:
        out, n = (C.c_uint32 * 8)(), C.c_size_t()
        _check(lib().qb_tokenizer_stop_tokens(self.handle, out, 8, C.byref(n)), TokenizerError)
        return list(out[:n.value])

    def text_stream(self) -> "TextStream":
        h = C.c_uint64()
        _check(lib().qb_tokenizer_stream_create(self.handle, C.byref(h)), TokenizerError)
        return TextStream(h.value, self)


class TextStream:
    """TextStream (src/tokenizer.rs:168-214)."""

    def __init__(self, handle, owner):
        self.handle, self._owner = handle, owner

    def __del__(self):
        if getattr(self, "handle", None):
            lib().qb_tokenizer_stream_free(self.handle)
            self.handle = None

    def push(self, token: int):
        buf, n, has = C.create_string_buffer(4096), C.c_size_t(), C.c_int32()
        _check(lib().qb_tokenizer_stream_push(self.handle, token, buf, 4096, C.byref(n), C.byref(has)),
               TokenizerError)
        return buf.raw[:n.value].decode("utf-8") if has.value else None

    def pending_tokens(self) -> int:
        n = C.c_size_t()
        _check(lib().qb_tokenizer_stream_pending(self.handle, C.byref(n)), TokenizerError)
        return n.value


class SamplingError(QbError):
    """SamplingError (src/sampling.rs:13-18): InvalidParameters, EmptyLogits,
    NonFinite."""


@dataclass(frozen=True)
class Temperature:
    """Sampling::Temperature (src/sampling.rs:7-11)."""
    temperature: float
    top_k: int
    seed: int


class Sampling:
    """Sampling policy (src/sampling.rs:5-12): ``Sampling.Greedy`` or
    ``Sampling.Temperature(temperature, top_k, seed)``."""
    Greedy = "greedy"
    Temperature = Temperature


def _sampling_c(policy):
    if policy == Sampling.Greedy:
        return _lib.SamplingC(0, 1.0, 0, 0)
    if isinstance(policy, Temperature):
        k, seed = int(policy.top_k), int(policy.seed)
        if k < 0 or seed < 0 or seed >= 2**64:
            raise SamplingError(27)
        return _lib.SamplingC(1, float(policy.temperature), min(k, 2**64 - 1), seed)
    raise SamplingError(27)


class Sampler:
    """Sampler (src/sampling.rs:19-110): the ChaCha8 generator on the host,
    the top-k selection and the walk on CUDA device ``device``.  ``sample``
    takes host logits (numpy) or a CUDA float32 tensor on that device."""

    def __init__(self, policy, device: int = 0):
        h = C.c_uint64()
        c = _sampling_c(policy)
        _check(lib().qb_sampler_create(C.byref(c), device, C.byref(h)), SamplingError)
        self.handle = h.value
        self.device = device

    def __del__(self):
        if getattr(self, "handle", None):
            lib().qb_sampler_free(self.handle)
            self.handle = None

    def validate_vocab(self, vocab: int):
        _check(lib().qb_sampler_validate_vocab(self.handle, vocab), SamplingError)

    def reset(self):
        _check(lib().qb_sampler_reset(self.handle), SamplingError)

    def sample(self, logits) -> int:
        out = C.c_uint32()
        if hasattr(logits, "is_cuda") and logits.is_cuda:
            assert logits.dtype.is_floating_point and logits.element_size() == 4 and logits.is_contiguous()
            _check(lib().qb_sampler_sample_device(self.handle, logits.data_ptr(), logits.numel(), C.byref(out)),
                   SamplingError)
        else:
            a = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
            _check(lib().qb_sampler_sample(self.handle, a.ctypes.data_as(C.c_void_p) if a.size else None,
                                           a.size, C.byref(out)), SamplingError)
        return int(out.value)


STOP_REASONS = {0: None, 1: "StopToken", 2: "OutputLimit"}


class CancelFlag:
    """Cooperative cancellation flag (the reference's &AtomicBool)."""

    def __init__(self, value: bool = False):
        self._v = C.c_int32(int(value))

    def store(self, value: bool):
        self._v.value = int(value)

    def load(self) -> bool:
        return bool(self._v.value)

    def ref(self):
        return C.byref(self._v)


class GenerationSession:
    """History plus KV-cached generation (src/generation.rs:98-338), greedy
    or seeded temperature/top-k sampling."""

    def __init__(self, model: Decoder, capacity: int, policy=Sampling.Greedy,
                 stops: Sequence[int] = (), max_new: int = 1, kv_dtype: str = "f32",
                 budget: int = REFERENCE_BUDGET):
        try:
            pc = _sampling_c(policy)
        except SamplingError:
            raise StateError(27)
        st = np.ascontiguousarray(np.asarray(list(stops), dtype=np.int64))
        if st.size and (st.min() < 0 or st.max() >= 2**32):
            raise StateError(27)
        st = st.astype(np.uint32)
        h = C.c_uint64()
        _check(lib().qb_generation_create_sampled(model.handle, capacity, C.byref(pc),
                                                  st.ctypes.data_as(C.c_void_p) if st.size else None,
                                                  st.size, max_new, KV_DTYPES[kv_dtype], budget,
                                                  C.byref(h)), StateError)
        self.handle = h.value
        self.vocab = model.config.vocab_size

    def __del__(self):
        if getattr(self, "handle", None):
            lib().qb_generation_free(self.handle)
            self.handle = None

    @staticmethod
    def _ids(ids):
        a = np.ascontiguousarray(np.asarray(list(ids), dtype=np.int64))
        if a.size and (a.min() < 0 or a.max() >= 2**32):
            a = np.full(a.size, 0xFFFFFFFF, dtype=np.int64)
        return a.astype(np.uint32)

    @staticmethod
    def _cancel(cancel):
        return None if cancel is None else cancel.ref()

    def start(self, prompt):
        self.start_with_cancel(prompt, None)

    def start_with_cancel(self, prompt, cancel: Optional[CancelFlag]):
        p = self._ids(prompt)
        _check(lib().qb_generation_start(self.handle, p.ctypes.data_as(C.c_void_p) if p.size else None,
                                         p.size, self._cancel(cancel)), StateError)

    def next_token(self, cancel: Optional[CancelFlag] = None) -> Optional[int]:
        tok, has = C.c_uint32(), C.c_int32()
        _check(lib().qb_generation_next_token(self.handle, self._cancel(cancel), C.byref(tok),
                                              C.byref(has)), StateError)
        return tok.value if has.value else None

    def append_context(self, suffix, max_new: int, cancel: Optional[CancelFlag] = None):
        s = self._ids(suffix)
        _check(lib().qb_generation_append_context(self.handle,
                                                  s.ctypes.data_as(C.c_void_p) if s.size else None,
                                                  s.size, max_new, self._cancel(cancel)), StateError)

    def replay_history(self, history, max_new: int, cancel: Optional[CancelFlag] = None):
        s = self._ids(history)
        _check(lib().qb_generation_replay_history(self.handle,
                                                  s.ctypes.data_as(C.c_void_p) if s.size else None,
                                                  s.size, max_new, self._cancel(cancel)), StateError)

    def reset(self):
        _check(lib().qb_generation_reset(self.handle), StateError)

    def _info(self):
        i = _lib.GenerationInfo()
        _check(lib().qb_generation_info_get(self.handle, C.byref(i)), StateError)
        return i

    def history(self) -> list:
        n = C.c_size_t()
        _check(lib().qb_generation_history(self.handle, None, 0, C.byref(n)), StateError)
        out = np.zeros(max(n.value, 1), dtype=np.uint32)
        _check(lib().qb_generation_history(self.handle, out.ctypes.data_as(C.c_void_p), n.value,
                                           C.byref(n)), StateError)
        return [int(v) for v in out[:n.value]]

    def processed(self) -> int:
        return self._info().processed

    def generated(self) -> int:
        return self._info().generated

    def is_valid(self) -> bool:
        return bool(self._info().valid)

    def stop_reason(self):
        return STOP_REASONS[self._info().stop_reason]

    def prefix_logits(self) -> Optional[np.ndarray]:
        out = np.zeros(self.vocab, dtype=np.float32)
        st = lib().qb_generation_prefix_logits(self.handle, out.ctypes.data_as(C.c_void_p), out.size)
        if st == 28:
            return None
        _check(st, StateError)
        return out
