"""Small fixed workloads for profiling and examples (synthetic weights).

    python -m llm_inference_edu_b200.workloads batched [--sequences 64] [--prompt 2] [--steps 4]
    python -m llm_inference_edu_b200.workloads decode [--prompt 128] [--steps 8] [--profile]
    python -m llm_inference_edu_b200.workloads long [--prompt 8192] [--steps 128]
    python -m llm_inference_edu_b200.workloads qwen7b [--prompt 512] [--steps 64] [--layers 28]
    python -m llm_inference_edu_b200.workloads sample [--steps 64] [--top-k 40]

Each builds the model on cuda:0 (0.5B INT8 with a BF16 table and KV unless
noted), runs the workload through the public API and prints one line of
timings.  `decode --profile` prints the per-phase device timestamps of the
decode kernel (CachedSession.step_profiled).
"""
from __future__ import annotations

import argparse
import time

import numpy as np

from . import presets, synthetic


def _model(cfg, seed=1, linear="int8"):
    from . import api
    w = synthetic.weights(cfg, seed=seed, dtype="bf16", lazy=True)
    return api.Decoder(cfg, w, linear_format=linear, table_format="bf16")


def _sync():
    import torch
    torch.cuda.synchronize()


def batched(sequences: int, prompt: int, steps: int) -> None:
    from . import api
    cap = prompt + steps + 8
    cfg = presets.qwen_0_5b(cap)
    m = _model(cfg)
    prompts = np.stack([synthetic.prompt(cfg.vocab_size, prompt, seed=100 + r)
                        for r in range(sequences)]).astype(np.uint32)
    b = api.BatchSession(m, sequences, cap, kv_dtype="bf16")
    _sync()
    t0 = time.perf_counter()
    first = b.prefill(prompts)
    _sync()
    t1 = time.perf_counter()
    b.decode_greedy(first, steps)
    _sync()
    t2 = time.perf_counter()
    print(f"batched: {sequences} sequences, prompt {prompt}: prefill {sequences * prompt / (t1 - t0):.0f} tok/s, "
          f"decode {(t2 - t1) * 1e3 / steps:.3f} ms/step (wall)")


def decode(prompt: int, steps: int, profile: bool, linear: str = "int8") -> None:
    from . import api
    cap = prompt + steps + 8
    cfg = presets.qwen_0_5b(cap)
    m = _model(cfg, linear=linear)
    # BF16 linears run with the reference's FP32 cache (the BF16 benchmark leg)
    s = api.CachedSession(m, cap, kv_dtype="bf16" if linear == "int8" else "f32", budget=0)
    tok = s.prefill_into(synthetic.prompt(cfg.vocab_size, prompt, seed=1), None)
    if not profile:
        _sync()
        t0 = time.perf_counter()
        s.decode_greedy(tok, steps)
        _sync()
        print(f"decode: {(time.perf_counter() - t0) * 1e6 / steps:.1f} us/token (wall)")
        return
    keys = ("ns", "mean_ns", "barrier_ns", "ready_ns", "last_ready_ns", "compute_ns")
    acc = {k: np.zeros(len(keys)) for k in ("qkv", "attention", "gate_up", "down")}
    tot = []
    for i in range(steps):
        _, prof = s.step_profiled(tok)
        tok = prof["argmax"]
        if i < 2:
            continue
        tot.append((prof["total_ns"], prof["logits_ns"]))
        for L in prof["layers"]:
            for k, v in L.items():
                acc[k] += np.array([v[x] for x in keys])
    n = (steps - 2) * cfg.layers
    print(f"decode at position ~{prompt}: step {np.mean([t[0] for t in tot]) / 1e3:.1f} us, "
          f"LM head {np.mean([t[1] for t in tot]) / 1e3:.1f} us")
    for k, v in acc.items():
        v = v / n / 1e3
        print(f"  {k:9s} per layer: phase {v[0]:.2f} us, mean CTA work {v[1]:.2f} us, "
              f"hand-over after the last finish {v[2]:.2f} us; per CTA: inputs held after {v[3]:.2f} us "
              f"(last {v[4]:.2f} us), then computes {v[5]:.2f} us")


def long(prompt: int, steps: int) -> None:
    decode(prompt, steps, profile=False)


def qwen7b(prompt: int, steps: int, layers: int = 28) -> None:
    """The 7B shape (fewer layers for a small profiling case)."""
    from dataclasses import replace
    from . import api
    cap = prompt + steps + 8
    cfg = replace(presets.qwen_7b(cap), layers=layers)
    m = _model(cfg, seed=2)
    s = api.CachedSession(m, cap, kv_dtype="bf16", budget=0)
    _sync()
    t0 = time.perf_counter()
    tok = s.prefill_into(synthetic.prompt(cfg.vocab_size, prompt, seed=3), None)
    _sync()
    t1 = time.perf_counter()
    s.decode_greedy(tok, steps)
    _sync()
    t2 = time.perf_counter()
    print(f"qwen7b ({layers} layers): prefill {prompt / (t1 - t0):.0f} tok/s, "
          f"decode {(t2 - t1) * 1e3 / steps:.2f} ms/token (wall)")


def sample(steps: int, top_k: int) -> None:
    """Seeded temperature/top-k sampling (T = 0.8) over Qwen-sized logits
    (151,936 values, N(0, 2.5^2), new per draw) resident on the device; the
    per-draw time includes the host generator and the result's read-back."""
    import torch
    from . import api
    V = 151936
    s = api.Sampler(api.Sampling.Temperature(0.8, top_k, 7))
    g = torch.Generator(device="cuda").manual_seed(3)
    rows = [torch.randn(V, device="cuda", generator=g) * 2.5 for _ in range(8)]
    for i in range(4):
        s.sample(rows[i % 8])
    _sync()
    t0 = time.perf_counter()
    ids = [s.sample(rows[i % 8]) for i in range(steps)]
    _sync()
    print(f"sample: top-k {top_k}, {(time.perf_counter() - t0) * 1e6 / steps:.1f} us/draw (wall), "
          f"last id {ids[-1]}")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("workload", choices=["batched", "decode", "long", "qwen7b", "sample"])
    ap.add_argument("--sequences", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--profile", action="store_true")
    ap.add_argument("--linear", choices=["int8", "bf16"], default="int8")
    ap.add_argument("--top-k", type=int, default=40)
    ap.add_argument("--layers", type=int, default=28)
    a = ap.parse_args(argv)
    if a.workload == "batched":
        batched(a.sequences, a.prompt or 2, a.steps or 4)
    elif a.workload == "decode":
        decode(a.prompt or 128, a.steps or 8, a.profile, a.linear)
    elif a.workload == "long":
        long(a.prompt or 8192, a.steps or 128)
    elif a.workload == "sample":
        sample(a.steps or 64, a.top_k)
    else:
        qwen7b(a.prompt or 512, a.steps or 64, a.layers)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
