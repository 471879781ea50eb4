"""Seeded synthetic weights and prompts (no checkpoints, no datasets).

Weights are N(0, 0.02) draws of the library's counter-based generator
(``qb_synthetic_normal``: splitmix64 + Box-Muller, documented in
csrc/synthetic.cpp); RMSNorm gains are 1.0 and Q/K/V biases 0, as the
benchmark configurations specify.  One stream id per tensor:

    embedding 1, lm_head 2, layer l: 100 + 16 l + {q 0, k 1, v 2, o 3,
    gate 4, up 5, down 6, q_bias 7, k_bias 8, v_bias 9,
    attn_norm 10, ffn_norm 11}

``dtype`` selects the host element type of matrices: "f32" (float32) or
"bf16" (uint16 BF16 bit patterns, FP32 draw rounded to nearest-even).
The same host arrays feed the device model and the CPU oracle, so both see
identical weights.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import lib
from .presets import ModelConfig

STD = 0.02
_MAT = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6}


def normal(seed: int, stream: int, n: int, std: float = STD, dtype: str = "f32") -> np.ndarray:
    if dtype == "f32":
        out = np.empty(n, dtype=np.float32)
        code = 0
    elif dtype == "bf16":
        out = np.empty(n, dtype=np.uint16)
        code = 1
    else:
        raise ValueError(dtype)
    st = lib().qb_synthetic_normal(seed, stream, n, std, code, out.ctypes.data_as(C.c_void_p))
    if st:
        raise RuntimeError(f"qb_synthetic_normal failed: {st}")
    return out


def tokens(seed: int, stream: int, n: int, vocab: int) -> np.ndarray:
    out = np.empty(n, dtype=np.uint32)
    st = lib().qb_synthetic_tokens(seed, stream, n, vocab, out.ctypes.data_as(C.c_void_p))
    if st:
        raise RuntimeError(f"qb_synthetic_tokens failed: {st}")
    return out


def prompt(vocab: int, n: int, seed: int, stream: int = 7) -> list:
    """A prompt of n ids uniform over [0, vocab)."""
    return [int(v) for v in tokens(seed, stream, n, vocab)]


def weights(cfg: ModelConfig, seed: int, dtype: str = "bf16", bias_std: float = 0.0,
            norm_std: float = 0.0, lazy: bool = False) -> dict:
    """Host weight dictionary for `cfg` (see module docstring).

    bias_std / norm_std > 0 draw non-trivial biases and norm gains
    (1 + N(0, norm_std)) for tests that must exercise those paths.  With
    lazy=True, "layers" is a sequence that draws each layer when it is
    visited (host memory of one layer at a time, for 7B-sized models).
    """
    h, V = cfg.hidden_dim, cfg.vocab_size
    out = {"embedding": normal(seed, 1, V * h, STD, dtype)}
    if not cfg.tied:
        out["lm_head"] = normal(seed, 2, V * h, STD, dtype)
    out["final_norm"] = _gain(seed, 3, h, norm_std)
    layers = _Layers(cfg, seed, dtype, bias_std, norm_std)
    out["layers"] = layers if lazy else list(layers)
    return out


class _Layers:
    """The layers of `weights`, each drawn when it is visited."""

    def __init__(self, cfg, seed, dtype, bias_std, norm_std):
        self.cfg, self.seed, self.dtype, self.bias_std, self.norm_std = cfg, seed, dtype, bias_std, norm_std

    def __len__(self):
        return self.cfg.layers

    def __getitem__(self, l):
        if not 0 <= l < self.cfg.layers:
            raise IndexError(l)
        cfg, seed = self.cfg, self.seed
        h, kv, ff = cfg.hidden_dim, cfg.kv_dim, cfg.ff_dim
        shapes = {"q": h * h, "k": kv * h, "v": kv * h, "o": h * h, "gate": ff * h, "up": ff * h,
                  "down": h * ff}
        base = 100 + 16 * l
        layer = {k: normal(seed, base + i, shapes[k], STD, self.dtype) for k, i in _MAT.items()}
        layer["attn_norm"] = _gain(seed, base + 10, h, self.norm_std)
        layer["ffn_norm"] = _gain(seed, base + 11, h, self.norm_std)
        if cfg.qkv_bias or self.bias_std > 0:
            for name, i, n in (("q_bias", 7, h), ("k_bias", 8, kv), ("v_bias", 9, kv)):
                layer[name] = (normal(seed, base + i, n, self.bias_std, "f32") if self.bias_std > 0
                               else np.zeros(n, dtype=np.float32))
        return layer

    def __iter__(self):
        for l in range(len(self)):
            yield self[l]


def _gain(seed, stream, n, std):
    if std <= 0:
        return np.ones(n, dtype=np.float32)
    return (1.0 + normal(seed, stream, n, std, "f32")).astype(np.float32)


def as_f32(a: np.ndarray) -> np.ndarray:
    """FP32 values of a host matrix (BF16 bits expand exactly: bits << 16)."""
    if a.dtype == np.uint16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return np.asarray(a, dtype=np.float32)


def to_reference_json(w: dict) -> dict:
    """The reference fixture's JSON weight layout (src/model.rs:27-53)."""
    names = {"attn_norm": "attention_norm", "q": "query", "k": "key", "v": "value",
             "o": "attention_output", "ffn_norm": "ffn_norm", "gate": "gate", "up": "up",
             "down": "down", "q_bias": "query_bias", "k_bias": "key_bias", "v_bias": "value_bias"}
    layers = []
    for layer in w["layers"]:
        layers.append({names[k]: as_f32(v).astype(float).tolist() for k, v in layer.items()})
    return {"embedding": as_f32(w["embedding"]).astype(float).tolist(), "layers": layers,
            "final_norm": as_f32(w["final_norm"]).astype(float).tolist()}
