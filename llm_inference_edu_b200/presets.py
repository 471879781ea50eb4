"""Model configurations of the Qwen2 token loop.

``ModelConfig`` carries the fields of the reference's ``ModelConfig``
(src/model.rs:12-25).  The presets are the shapes the token loop is
exercised on:

* ``tiny_r``  - the reference's tiny JSON fixture (vocab 64, 2 layers,
  hidden 32, 4/2 heads, head_dim 8, ff 64, eps 1e-5, theta 1e4), whose
  weights are an explicit formula (``tiny_r_weights``);
* ``tiny_b``  - the tiny benchmark decoder: vocab 256, 2 layers, hidden 64,
  4/2 heads, head_dim 16, ff 128, eps 1e-6, theta 1e4;
* ``qwen_0_5b`` - Qwen2.5-0.5B shape: vocab 151936 (tied), 24 layers,
  hidden 896, 14/2 heads, head_dim 64, ff 4864, eps 1e-6, theta 1e6;
* ``qwen_7b`` - Qwen2.5-7B shape: vocab 152064 (untied), 28 layers,
  hidden 3584, 28/4 heads, head_dim 128, ff 18944, eps 1e-6, theta 1e6.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, replace

import numpy as np


@dataclass(frozen=True)
class ModelConfig:
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

    def with_max_tokens(self, n: int) -> "ModelConfig":
        return replace(self, max_tokens=n)

    def to_reference_json(self) -> dict:
        d = asdict(self)
        d.pop("tied")
        d.pop("qkv_bias")
        return d

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


def tiny_r(max_tokens: int = 32) -> ModelConfig:
    return ModelConfig(64, 2, 32, 4, 2, 8, 64, max_tokens, 10000.0, 1e-5)


def tiny_b(max_tokens: int = 64) -> ModelConfig:
    return ModelConfig(256, 2, 64, 4, 2, 16, 128, max_tokens, 10000.0, 1e-6)


def qwen_0_5b(max_tokens: int = 32768) -> ModelConfig:
    return ModelConfig(151936, 24, 896, 14, 2, 64, 4864, max_tokens, 1e6, 1e-6, True, True)


def qwen_7b(max_tokens: int = 32768) -> ModelConfig:
    return ModelConfig(152064, 28, 3584, 28, 4, 128, 18944, max_tokens, 1e6, 1e-6, False, True)


def tiny_r_weights() -> dict:
    """The reference's tiny fixture weights.

    Restates the explicit formula of reference/make_tiny_fixture.py:9-30:
    ``values(count, seed)[i] = ((i*17 + seed) % 97 - 48) / 256`` with layer
    seeds ``13 + 29*i`` and norm gains ``1 + values(...)``.  Every value is a
    dyadic rational, exact in FP32.
    """
    def values(count, seed):
        i = np.arange(count, dtype=np.int64)
        return (((i * 17 + seed) % 97 - 48) / 256.0).astype(np.float32)

    layers = []
    for i in range(2):
        seed = 13 + i * 29
        layers.append(dict(
            attn_norm=1 + values(32, seed), q=values(1024, seed + 1), k=values(512, seed + 2),
            v=values(512, seed + 3), o=values(1024, seed + 4), ffn_norm=1 + values(32, seed + 5),
            gate=values(2048, seed + 6), up=values(2048, seed + 7), down=values(2048, seed + 8)))
    return dict(embedding=values(2048, 7), layers=layers, final_norm=1 + values(32, 43))
