"""ctypes wrapper of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The oracle (``qwen_oracle.c``) restates the reference crate's scalar FP32
arithmetic.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may import this module; the product package never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwen_oracle.so")

OK = 0
ZERO_DIMENSION = 1
DIMENSION_OVERFLOW = 2
INVALID_LENGTH = 3
INVALID_GROUP_SIZE = 4
NONFINITE_WEIGHT = 6
UNREPRESENTABLE_SCALE = 7
INVALID_TOKEN = 9
INVALID_EPSILON = 10
NONFINITE = 11
ALL_MASKED = 12
INVALID_CAPACITY = 18
RESOURCE_BUDGET = 19
INVALID_OUTPUT_LENGTH = 20
EMPTY_INPUT = 21
NOT_EMPTY = 22
FULL = 23
INVALID_STATE = 24
CONTEXT_LIMIT = 34
INVALID_PARAMETERS = 27
EMPTY_LOGITS = 31

MAT_NONE, MAT_F32, MAT_BF16, MAT_INT8 = -1, 0, 1, 2
W_EMBEDDING, W_LM_HEAD, W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN = range(9)
V_FINAL_NORM, V_ATTN_NORM, V_FFN_NORM, V_Q_BIAS, V_K_BIAS, V_V_BIAS = range(6)


class Detail(C.Structure):
    _fields_ = [("buffer", C.c_size_t), ("expected", C.c_size_t),
                ("actual", C.c_size_t), ("index", C.c_size_t)]


class Config(C.Structure):
    _fields_ = [(n, C.c_size_t) for n in ("vocab", "layers", "hidden", "query_heads",
                                          "kv_heads", "head_dim", "ff", "max_tokens")] + \
               [("rope_base", C.c_float), ("norm_eps", C.c_float)]


class Matrix(C.Structure):
    _fields_ = [("kind", C.c_int), ("f32", C.c_void_p), ("bf16", C.c_void_p),
                ("q", C.c_void_p), ("scales", C.c_void_p), ("group", C.c_size_t)]


def build():
    """Compile the oracle with its Makefile (gcc, OpenMP, no FMA contraction)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        S = C.c_size_t
        for name, args, res in [
            ("or_linear", [P, S, P, S, P, S, S, S, S, P], C.c_int),
            ("or_linear_lanes4", [P, S, P, S, P, S, S, S, S, P], C.c_int),
            ("or_encode", [C.c_float, C.c_float], C.c_int8),
            ("or_quantize", [P, S, S, S, S, P, P, P], C.c_int),
            ("or_dequantize", [P, P, S, S, S, P], None),
            ("or_linear_int8", [P, S, P, P, P, S, S, S, S, S, C.c_int, P], C.c_int),
            ("or_embedding", [P, S, P, S, P, S, S, S, P], C.c_int),
            ("or_residual_add", [P, S, P, S, P, S, P], C.c_int),
            ("or_rmsnorm", [P, S, P, S, P, S, S, S, C.c_float, P], C.c_int),
            ("or_silu", [P, S, P, S, P], C.c_int),
            ("or_softmax", [P, S, P, S, P, S, S, S, P], C.c_int),
            ("or_rope_table", [C.c_float, S, S, S, P, P], None),
            ("or_rope", [P, S, P, S, S, S, S, S, C.c_float, P], C.c_int),
            ("or_model_new", [P], P),
            ("or_model_free", [P], None),
            ("or_model_set_matrix", [P, C.c_long, C.c_int, P], None),
            ("or_model_set_vector", [P, C.c_long, C.c_int, P], None),
            ("or_trace_len", [P, S], S),
            ("or_forward", [P, P, S, P, P], C.c_int),
            ("or_workspace_bytes", [P, S], S),
            ("or_session_new", [P, S, C.c_int, S, P], C.c_int),
            ("or_session_free", [P], None),
            ("or_session_processed", [P], S),
            ("or_session_is_valid", [P], C.c_int),
            ("or_session_logical_bytes", [P], S),
            ("or_session_workspace_bytes", [P], S),
            ("or_session_reset", [P], None),
            ("or_session_step", [P, S, P, S], C.c_int),
            ("or_session_append", [P, P, S, P, S, C.c_int], C.c_int),
            ("or_session_append_chunked", [P, P, S, P, S, C.c_int, S], C.c_int),
            ("or_set_fast", [C.c_int], None),
            ("or_argmax", [P, S], S),
            ("or_greedy", [P, P, S, P, S, S, P], C.c_long),
            ("or_uncached_greedy", [P, P, S, P, S, S, P], C.c_long),
            ("or_set_threads", [C.c_int], None),
            ("or_get_threads", [], C.c_int),
            ("or_round_bf16", [C.c_float], C.c_float),
            ("or_synthetic_normal", [C.c_uint64, C.c_uint64, S, C.c_double, C.c_int, P], C.c_int),
            ("or_synthetic_tokens", [C.c_uint64, C.c_uint64, S, C.c_uint32, P], C.c_int),
            ("or_chacha_block", [P, C.c_int, P], None),
            ("or_rng_from_seed", [P, P], None),
            ("or_rng_seed", [P, C.c_uint64], None),
            ("or_rng_next_u64", [P], C.c_uint64),
            ("or_rng_next_f64", [P], C.c_double),
            ("or_sampler_init", [P, C.c_int, C.c_float, S, C.c_uint64], C.c_int),
            ("or_sampler_reset", [P], None),
            ("or_sampler_validate_vocab", [P, S], C.c_int),
            ("or_sampler_sample", [P, P, S, P], C.c_int),
        ]:
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def ids_array(ids):
    return np.ascontiguousarray(np.asarray(ids, dtype=np.uint64))


# --------------------------------------------------------------- ops ----

def linear(x, w, tokens, in_dim, out_dim, lanes4=False, y_len=None):
    x, w = f32(x), f32(w)
    y = np.full(tokens * out_dim if y_len is None else y_len, 37.0, dtype=np.float32)
    d = Detail()
    fn = lib().or_linear_lanes4 if lanes4 else lib().or_linear
    s = fn(_p(x), x.size, _p(w), w.size, _p(y), y.size, tokens, in_dim, out_dim, C.byref(d))
    return s, y, d


@dataclass
class Int8Matrix:
    values: np.ndarray  # int8 [out, in]
    scales: np.ndarray  # f32 [out, groups_per_row]
    out_dim: int
    in_dim: int
    group: int

    @property
    def groups_per_row(self):
        return -(-self.in_dim // self.group)

    @property
    def logical_bytes(self):
        return self.values.size + 4 * self.scales.size


def quantize(w, out_dim, in_dim, group):
    w = f32(w)
    gpr = -(-in_dim // group) if group else 0
    values = np.zeros(max(out_dim * in_dim, 1), dtype=np.int8)
    scales = np.zeros(max(out_dim * gpr, 1), dtype=np.float32)
    d = Detail()
    s = lib().or_quantize(_p(w), w.size, out_dim, in_dim, group, _p(values), _p(scales), C.byref(d))
    if s:
        return s, None
    return OK, Int8Matrix(values.reshape(out_dim, in_dim), scales.reshape(out_dim, gpr),
                          out_dim, in_dim, group)


def dequantize(m: Int8Matrix):
    y = np.zeros(m.out_dim * m.in_dim, dtype=np.float32)
    lib().or_dequantize(_p(m.values), _p(m.scales), m.out_dim, m.in_dim, m.group, _p(y))
    return y


def linear_int8(x, m: Int8Matrix, tokens, lanes4=False):
    x = f32(x)
    y = np.zeros(tokens * m.out_dim, dtype=np.float32)
    d = Detail()
    s = lib().or_linear_int8(_p(x), x.size, _p(m.values), _p(m.scales), _p(y), y.size, tokens,
                             m.in_dim, m.out_dim, m.group, int(lanes4), C.byref(d))
    return s, y


def embedding(ids, table, vocab, width):
    ids = ids_array(ids)
    table = f32(table)
    y = np.zeros(ids.size * width, dtype=np.float32)
    s = lib().or_embedding(_p(ids), ids.size, _p(table), table.size, _p(y), y.size, vocab, width, None)
    return s, y


def residual_add(x, r):
    x, r = f32(x), f32(r)
    y = np.zeros_like(x)
    return lib().or_residual_add(_p(x), x.size, _p(r), r.size, _p(y), y.size, None), y


def rmsnorm(x, g, rows, width, eps):
    x, g = f32(x), f32(g)
    y = np.zeros_like(x)
    return lib().or_rmsnorm(_p(x), x.size, _p(g), g.size, _p(y), y.size, rows, width, eps, None), y


def silu(x):
    x = f32(x)
    y = np.zeros_like(x)
    return lib().or_silu(_p(x), x.size, _p(y), y.size, None), y


def softmax(logits, rows, width, mask=None):
    lg = f32(logits)
    y = np.zeros_like(lg)
    m = None if mask is None else np.ascontiguousarray(np.asarray(mask, dtype=np.uint8))
    s = lib().or_softmax(_p(lg), lg.size, _p(m), 0 if m is None else m.size, _p(y), y.size,
                         rows, width, None)
    return s, y


def rope(x, tokens, heads, head_dim, start, base):
    x = f32(x)
    y = np.zeros_like(x)
    s = lib().or_rope(_p(x), x.size, _p(y), y.size, tokens, heads, head_dim, start, base, None)
    return s, y


def rope_table(base, head_dim, start, count):
    half = head_dim // 2
    c = np.zeros(count * half, dtype=np.float32)
    s = np.zeros(count * half, dtype=np.float32)
    lib().or_rope_table(base, head_dim, start, count, _p(c), _p(s))
    return c.reshape(count, half), s.reshape(count, half)


def round_bf16(a):
    a = f32(a)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def set_fast(on=True):
    """Interleaved row evaluation (bit-identical outputs, faster): for the
    parity tests; the timed CPU baseline keeps it off."""
    lib().or_set_fast(int(on))


def set_threads(n):
    lib().or_set_threads(int(n))


def threads():
    return lib().or_get_threads()


# ------------------------------------------------------------- model ----

_MAT_KEYS = {"q": W_Q, "k": W_K, "v": W_V, "o": W_O, "gate": W_GATE, "up": W_UP, "down": W_DOWN}
_VEC_KEYS = {"attn_norm": V_ATTN_NORM, "ffn_norm": V_FFN_NORM, "q_bias": V_Q_BIAS,
             "k_bias": V_K_BIAS, "v_bias": V_V_BIAS}


class Model:
    """An oracle model over host arrays.

    ``weights`` follows the package's host weight dictionary: matrices are
    float32 arrays, uint16 arrays of BF16 bits, or :class:`Int8Matrix`;
    vectors are float32 arrays; ``lm_head`` is optional (tied when absent).
    """

    def __init__(self, config, weights):
        self.config = config
        c = Config(config.vocab_size, config.layers, config.hidden_dim, config.query_heads,
                   config.kv_heads, config.head_dim, config.ff_dim, config.max_tokens,
                   config.rope_base, config.norm_epsilon)
        self._c = c
        self._keep = []
        self.h = lib().or_model_new(C.byref(c))
        self._set_matrix(-1, W_EMBEDDING, weights["embedding"])
        if weights.get("lm_head") is not None:
            self._set_matrix(-1, W_LM_HEAD, weights["lm_head"])
        self._set_vector(-1, V_FINAL_NORM, weights["final_norm"])
        for i, layer in enumerate(weights["layers"]):
            for k, which in _MAT_KEYS.items():
                self._set_matrix(i, which, layer[k])
            for k, which in _VEC_KEYS.items():
                if layer.get(k) is not None:
                    self._set_vector(i, which, layer[k])

    def _set_matrix(self, layer, which, m):
        mat = Matrix()
        if isinstance(m, Int8Matrix):
            q = np.ascontiguousarray(m.values)
            s = np.ascontiguousarray(m.scales, dtype=np.float32)
            self._keep += [q, s]
            mat.kind, mat.q, mat.scales, mat.group = MAT_INT8, q.ctypes.data, s.ctypes.data, m.group
        elif m.dtype == np.uint16:
            a = np.ascontiguousarray(m)
            self._keep.append(a)
            mat.kind, mat.bf16 = MAT_BF16, a.ctypes.data
        else:
            a = f32(m)
            self._keep.append(a)
            mat.kind, mat.f32 = MAT_F32, a.ctypes.data
        lib().or_model_set_matrix(self.h, layer, which, C.byref(mat))

    def _set_vector(self, layer, which, v):
        a = f32(v)
        self._keep.append(a)
        lib().or_model_set_vector(self.h, layer, which, _p(a))

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_model_free(self.h)
            self.h = None

    def forward(self, ids, trace=False):
        ids = ids_array(ids)
        V = self.config.vocab_size
        logits = np.zeros(V, dtype=np.float32)
        tr = None
        if trace:
            tr = np.zeros(lib().or_trace_len(C.byref(self._c), ids.size), dtype=np.float32)
        s = lib().or_forward(self.h, _p(ids), ids.size, _p(logits), _p(tr))
        if s:
            return s, None, None
        return OK, logits, (self._split_trace(tr, ids.size) if trace else None)

    def _split_trace(self, tr, T):
        c = self.config
        h, kv, ff, V = c.hidden_dim, c.kv_heads * c.head_dim, c.ff_dim, c.vocab_size
        out, off = {}, 0

        def take(name, n):
            nonlocal off
            out[name] = tr[off:off + n].copy()
            off += n
        take("embedding", T * h)
        names = [("attention_norm", h), ("query", h), ("key", kv), ("value", kv),
                 ("rotated_query", h), ("rotated_key", kv), ("context", h),
                 ("attention_output", h), ("after_attention", h), ("ffn_norm", h),
                 ("gate", ff), ("up", ff), ("activated_gate", ff), ("product", ff),
                 ("ffn_output", h), ("output", h)]
        for i in range(c.layers):
            for n, w in names:
                take(f"layer_{i}.{n}", T * w)
        take("final_norm", T * h)
        take("logits", T * V)
        return out

    def uncached_greedy(self, prompt, stops, max_new):
        p, st = ids_array(prompt), ids_array(stops)
        out = np.zeros(max(max_new, 1), dtype=np.uint64)
        n = lib().or_uncached_greedy(self.h, _p(p), p.size, _p(st), st.size, max_new, _p(out))
        if n < 0:
            return -n, None
        return OK, [int(v) for v in out[:n]]


class Session:
    """The oracle's CachedSession (src/kv_cache.rs:156-475)."""

    def __init__(self, model: Model, capacity, kv_bf16=False, budget=128 * 1024 * 1024):
        self.model = model
        h = C.c_void_p()
        self.status = lib().or_session_new(model.h, capacity, int(kv_bf16), budget, C.byref(h))
        self.h = h.value if self.status == OK else None

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_session_free(self.h)
            self.h = None

    def step(self, token, logits=None):
        V = self.model.config.vocab_size
        if logits is None:
            logits = np.zeros(V, dtype=np.float32)
        s = lib().or_session_step(self.h, int(token), _p(logits), logits.size)
        return s, logits

    def append(self, tokens, require_empty=False, logits=None):
        t = ids_array(tokens)
        V = self.model.config.vocab_size
        if logits is None:
            logits = np.zeros(V, dtype=np.float32)
        s = lib().or_session_append(self.h, _p(t), t.size, _p(logits), logits.size, int(require_empty))
        return s, logits

    def prefill(self, tokens, logits=None):
        return self.append(tokens, True, logits)

    def append_chunked(self, tokens, require_empty=False, logits=None, chunk=64):
        """append / prefill evaluated layer-major over chunks of `chunk`
        tokens: the same per-token values, only the last token's logits (the
        long prompts of the parity tests)."""
        t = ids_array(tokens)
        V = self.model.config.vocab_size
        if logits is None:
            logits = np.zeros(V, dtype=np.float32)
        s = lib().or_session_append_chunked(self.h, _p(t), t.size, _p(logits), logits.size,
                                            int(require_empty), chunk)
        return s, logits

    def reset(self):
        lib().or_session_reset(self.h)

    @property
    def processed(self):
        return lib().or_session_processed(self.h)

    @property
    def valid(self):
        return bool(lib().or_session_is_valid(self.h))

    @property
    def logical_bytes(self):
        return lib().or_session_logical_bytes(self.h)

    @property
    def workspace_bytes(self):
        return lib().or_session_workspace_bytes(self.h)

    def greedy(self, prompt, max_new, stops=()):
        p, st = ids_array(prompt), ids_array(stops)
        out = np.zeros(max(max_new, 1), dtype=np.uint64)
        n = lib().or_greedy(self.h, _p(p), p.size, _p(st), st.size, max_new, _p(out))
        if n < 0:
            return -n, None
        return OK, [int(v) for v in out[:n]]


class _Rng(C.Structure):
    _fields_ = [("key", C.c_uint32 * 8), ("counter", C.c_uint64), ("buf", C.c_uint32 * 64), ("index", C.c_size_t)]


class _SamplerState(C.Structure):
    _fields_ = [("greedy", C.c_int), ("temperature", C.c_float), ("top_k", C.c_size_t), ("seed", C.c_uint64),
                ("rng", _Rng)]


def chacha_block(words, rounds):
    """The ChaCha block function over a 16-word input state."""
    w = np.ascontiguousarray(words, dtype=np.uint32)
    out = np.zeros(16, dtype=np.uint32)
    lib().or_chacha_block(_p(w), rounds, _p(out))
    return out


class Rng:
    """ChaCha8Rng (rand_chacha 0.9): ``Rng(seed=u64)`` seeds through
    seed_from_u64, ``Rng(key=bytes32)`` through from_seed."""

    def __init__(self, seed=None, key=None):
        self.s = _Rng()
        if key is not None:
            k = np.frombuffer(bytes(key), dtype=np.uint8).copy()
            assert k.size == 32
            lib().or_rng_from_seed(C.byref(self.s), _p(k))
        else:
            lib().or_rng_seed(C.byref(self.s), int(seed))

    def next_u64(self):
        return int(lib().or_rng_next_u64(C.byref(self.s)))

    def next_u32_words(self, n):
        """n keystream words in order (n even)."""
        out = []
        for _ in range(n // 2):
            v = self.next_u64()
            out += [v & 0xFFFFFFFF, v >> 32]
        return out

    def random_f64(self):
        return float(lib().or_rng_next_f64(C.byref(self.s)))


class Sampler:
    """Sampler (src/sampling.rs:19-110): greedy, or seeded temperature/top-k.
    Constructor errors raise ValueError with the status code."""

    def __init__(self, temperature=None, top_k=None, seed=0):
        self.s = _SamplerState()
        greedy = temperature is None
        st = lib().or_sampler_init(C.byref(self.s), int(greedy), 0.0 if greedy else float(temperature),
                                   0 if greedy else int(top_k), int(seed))
        if st:
            raise ValueError(st)

    def validate_vocab(self, vocab):
        return lib().or_sampler_validate_vocab(C.byref(self.s), int(vocab))

    def reset(self):
        lib().or_sampler_reset(C.byref(self.s))

    def sample(self, logits):
        """(status, id)"""
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        out = C.c_size_t(0)
        st = lib().or_sampler_sample(C.byref(self.s), _p(lg) if lg.size else None, lg.size, C.byref(out))
        return st, (int(out.value) if st == OK else None)


def int8_model_weights(cfg, w, linear_format):
    """The oracle's view of a host weight set: for "int8" every per-layer
    linear is quantized per output row by the oracle itself (group = input
    width); embedding/LM-head tables and vectors pass through unchanged."""
    if linear_format != "int8":
        return w
    shapes = dict(q=(cfg.hidden_dim, cfg.hidden_dim), k=(cfg.kv_dim, cfg.hidden_dim),
                  v=(cfg.kv_dim, cfg.hidden_dim), o=(cfg.hidden_dim, cfg.hidden_dim),
                  gate=(cfg.ff_dim, cfg.hidden_dim), up=(cfg.ff_dim, cfg.hidden_dim),
                  down=(cfg.hidden_dim, cfg.ff_dim))
    out = {k: v for k, v in w.items() if k != "layers"}
    out["layers"] = []
    for layer in w["layers"]:
        ql = dict(layer)
        for k, (r, c) in shapes.items():
            a = layer[k]
            f = (a.astype(np.uint32) << 16).view(np.float32) if a.dtype == np.uint16 else f32(a)
            s, q = quantize(f, r, c, c)
            if s:
                raise ValueError(f"oracle quantize failed: {s}")
            ql[k] = q
        out["layers"].append(ql)
    return out


# --------------------------------------------------- synthetic inputs ----
#
# The benchmark workloads' seeded weights and prompts, generated by the
# oracle library itself (or_synthetic_*), so that a CPU-only run (the
# reference arm of bench.py) maps no library of the product.  The stream
# ids and shapes follow the package's synthetic weight dictionary:
# embedding 1, lm_head 2, final_norm 3, layer l: 100 + 16 l + {q 0, k 1,
# v 2, o 3, gate 4, up 5, down 6, q_bias 7, k_bias 8, v_bias 9,
# attn_norm 10, ffn_norm 11}; norm gains 1.0 and biases 0.

STD = 0.02


@dataclass(frozen=True)
class WorkloadConfig:
    """The model shape fields the oracle reads (src/model.rs:12-25)."""
    vocab_size: int
    layers: int
    hidden_dim: int
    query_heads: int
    kv_heads: int
    head_dim: int
    ff_dim: int
    max_tokens: int
    rope_base: float
    norm_epsilon: float
    tied: bool = True
    qkv_bias: bool = False

    @property
    def kv_dim(self):
        return self.kv_heads * self.head_dim


def qwen_0_5b_config(max_tokens):
    return WorkloadConfig(151936, 24, 896, 14, 2, 64, 4864, max_tokens, 1e6, 1e-6, True, True)


def qwen_7b_config(max_tokens):
    return WorkloadConfig(152064, 28, 3584, 28, 4, 128, 18944, max_tokens, 1e6, 1e-6, False, True)


def synthetic_normal(seed, stream, n, std=STD, dtype="f32"):
    out = np.empty(n, dtype=np.float32 if dtype == "f32" else np.uint16)
    s = lib().or_synthetic_normal(seed, stream, n, std, 0 if dtype == "f32" else 1, _p(out))
    if s:
        raise ValueError(f"or_synthetic_normal failed: {s}")
    return out


def synthetic_prompt(vocab, n, seed, stream=7):
    out = np.empty(n, dtype=np.uint32)
    s = lib().or_synthetic_tokens(seed, stream, n, vocab, _p(out))
    if s:
        raise ValueError(f"or_synthetic_tokens failed: {s}")
    return [int(v) for v in out]


def synthetic_layer(cfg, seed, l, dtype="bf16"):
    h, kv, ff = cfg.hidden_dim, cfg.kv_dim, cfg.ff_dim
    shapes = {"q": h * h, "k": kv * h, "v": kv * h, "o": h * h, "gate": ff * h, "up": ff * h, "down": h * ff}
    base = 100 + 16 * l
    layer = {k: synthetic_normal(seed, base + i, shapes[k], STD, dtype)
             for i, k in enumerate(("q", "k", "v", "o", "gate", "up", "down"))}
    layer["attn_norm"] = np.ones(h, dtype=np.float32)
    layer["ffn_norm"] = np.ones(h, dtype=np.float32)
    if cfg.qkv_bias:
        for name, n in (("q_bias", h), ("k_bias", kv), ("v_bias", kv)):
            layer[name] = np.zeros(n, dtype=np.float32)
    return layer


def synthetic_weights(cfg, seed, dtype="bf16"):
    h, V = cfg.hidden_dim, cfg.vocab_size
    w = {"embedding": synthetic_normal(seed, 1, V * h, STD, dtype),
         "final_norm": np.ones(h, dtype=np.float32),
         "layers": [synthetic_layer(cfg, seed, l, dtype) for l in range(cfg.layers)]}
    if not cfg.tied:
        w["lm_head"] = synthetic_normal(seed, 2, V * h, STD, dtype)
    return w
