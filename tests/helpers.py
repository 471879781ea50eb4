"""Shared builders for the GPU parity tests: one seeded host weight set feeds
both the device model and the CPU oracle."""
import functools

import numpy as np

from llm_inference_edu_b200 import presets, synthetic


def oracle_weights(o, cfg, w, linear_format):
    return o.int8_model_weights(cfg, w, linear_format)


@functools.lru_cache(maxsize=2)
def qwen_host_weights(name, seed, dtype):
    cfg = {"0.5b": presets.qwen_0_5b, "7b": presets.qwen_7b}[name]()
    return synthetic.weights(cfg, seed=seed, dtype=dtype)


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))
