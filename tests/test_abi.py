"""CPU checks of the C-ABI library: it loads without a GPU, exports every
symbol the header declares, and its host-only entry points behave."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def header_symbols():
    text = open(os.path.join(ROOT, "include", "qwen_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from llm_inference_edu_b200 import _lib
    L = C.CDLL(_lib.LIB_PATH)
    syms = header_symbols()
    assert len(syms) >= 40
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    assert set(syms) == set(_lib.SIGNATURES), set(syms) ^ set(_lib.SIGNATURES)


def test_abi_version_and_status_names():
    from llm_inference_edu_b200._lib import lib
    from llm_inference_edu_b200.api import STATUS_NAMES
    assert lib().qb_abi_version() == 1
    for i, name in enumerate(STATUS_NAMES):
        assert lib().qb_status_name(i).decode() == name


def test_host_admission_needs_no_gpu():
    # Validation runs before any device work (src/lib.rs:46-50): zero
    # dimensions and overflow are reported without touching the GPU.
    from llm_inference_edu_b200._lib import lib
    L = lib()
    assert L.qb_linear_f32(None, 0, None, 0, None, 0, 0, 3, 2, None) == 1
    assert L.qb_linear_f32(None, 0, None, 0, None, 0, 2**64 - 1, 2, 1, None) == 2
    assert L.qb_linear_f32(None, 5, None, 6, None, 4, 2, 3, 2, None) == 3
    d = __import__("llm_inference_edu_b200._lib", fromlist=["Detail"]).Detail()
    L.qb_last_detail(C.byref(d))
    assert (d.buffer, d.expected, d.actual) == (0, 6, 5)
    assert L.qb_quantize_int8(None, 0, 1, 1, 0, None, None, None) == 4
    assert L.qb_quantize_int8(None, 0, 1, 1, 257, None, None, None) == 4
    assert L.qb_rope(None, 0, None, 0, 1, 1, 3, 0, 10000.0, None) == 13
    assert L.qb_rope(None, 0, None, 0, 2, 1, 2, 1 << 24, 10000.0, None) == 15
    assert L.qb_rmsnorm(None, 6, None, 3, None, 6, 2, 3, 0.0, None) == 10
    assert L.qb_session_reset(12345) == 26


def test_synthetic_generator_is_deterministic_and_normal():
    from llm_inference_edu_b200 import synthetic
    a = synthetic.normal(1, 5, 100001, 0.02, "f32")
    b = synthetic.normal(1, 5, 100001, 0.02, "f32")
    assert np.array_equal(a, b)
    assert abs(float(a.mean())) < 1e-3 and abs(float(a.std()) - 0.02) < 5e-4
    c = synthetic.normal(1, 5, 100001, 0.02, "bf16")
    f = synthetic.as_f32(c)
    assert np.max(np.abs(f - a)) <= np.max(np.abs(a)) * 2 ** -8
    # A prefix of a longer draw equals the shorter draw (counter-based).
    assert np.array_equal(synthetic.normal(1, 5, 11, 0.02, "f32"), a[:11])
    t = synthetic.tokens(3, 7, 1000, 151936)
    assert t.max() < 151936 and len(set(t.tolist())) > 990


def test_reference_fixture_weights_formula():
    # tiny_r_weights restates reference/make_tiny_fixture.py; spot values
    # from fixtures/tiny-model.json.
    from llm_inference_edu_b200 import presets
    w = presets.tiny_r_weights()
    assert list(w["embedding"][:4]) == [-0.16015625, -0.09375, -0.02734375, 0.0390625]
    assert w["layers"][1]["down"].size == 2048


def test_sampler_policy_admission_needs_no_gpu():
    # Sampler::new (src/sampling.rs:24-42): a temperature that is not finite
    # and positive, or top_k = 0, is InvalidParameters before any device work.
    import llm_inference_edu_b200 as qb
    T = qb.Sampling.Temperature
    for pol in [T(0.0, 1, 0), T(-1.0, 1, 0), T(float("nan"), 1, 0), T(float("inf"), 1, 0), T(1.0, 0, 0)]:
        with pytest.raises(qb.SamplingError) as e:
            qb.Sampler(pol)
        assert e.value.kind == "InvalidParameters"
    from llm_inference_edu_b200._lib import lib, SamplingC
    bad_kind = SamplingC(7, 1.0, 1, 0)
    h = C.c_uint64()
    assert lib().qb_sampler_create(C.byref(bad_kind), 0, C.byref(h)) == 27
    assert lib().qb_sampler_reset(999999) == 26
