"""Benchmark of the Qwen2 token loop on B200.

Workload (one GPU): Qwen2.5-0.5B-shaped decoder, INT8 per-row linears, BF16
embedding/tied head and BF16 KV cache, random N(0, 0.02) weights (seed 1),
a 128-token uniform prompt (seed 1 + rank), then greedy decode at batch 1.
A step is one decode token.  W warm-up steps, then K timed steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

With N > 1 (torchrun, one process per GPU) every rank decodes its own
independent sequence (data parallel, no collectives; weak scaling); the
timed region is bracketed by a barrier and the max over ranks is reported.

`value` is device-timed decode throughput (CUDA events on the session's
stream around K back-to-back steps, each step's argmax feeding the next on
the device).  `e2e` is the same metric through the public generation API
(GenerationSession.next_token: per step a 16-byte host->device control copy
from pinned memory and an 8-byte device->host result read).  The weights
(631 MB) exceed the 126 MB L2, so no flush is needed between steps.

`batched` is the same model decoding 64 independent sequences per GPU in
lockstep (BatchSession: one multi-token forward per step on the tensor
cores), device-timed, with its prompt evaluation rate.  `long_context` is
an 8,192-token prompt (chunked) then greedy decode at that depth.

--impl reference times the reference's CPU token loop on the host: the
oracle (the C restatement of the crate's scalar FP32 arithmetic; the Rust
crate cannot be built here), single-threaded like the crate, on the same
prompt, warm-up and step count as the native arm.  It loads no library of
the product (the oracle draws the same seeded weights itself).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT = 128
SEED = 1
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one
# decode_kernel launch of the INT8 workload, from an ncu capture of this
# kernel (taken at cache position 134; every further cached position adds
# 12,288 bytes of BF16 KV: 24 layers x K and V x 2 KV heads x 64 x 2 B).
NCU_TRAFFIC_BYTES_INT8 = 643_108_608


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--config", default="int8", choices=["int8", "bf16"])
    ap.add_argument("--cpu-steps", type=int, default=6)
    return ap.parse_args()


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS,
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([v.strip() for v in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > i + 2 and s[i + 2].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def algorithmic_bytes(cfg, linear_format, kv_bytes_per_pos, L):
    """HBM bytes one decode step must move: every weight once, the KV of
    all L cached positions once, the new K/V and the logits row."""
    h, kv, ff, V = cfg.hidden_dim, cfg.kv_dim, cfg.ff_dim, cfg.vocab_size
    mats = h * h * 2 + kv * h * 2 + ff * h * 3
    rows = h + 2 * kv + h + 2 * ff + h
    if linear_format == "int8":
        lin = mats + 4 * rows
    else:
        lin = 2 * mats
    per_layer = lin + 4 * (2 * h) + 4 * (h + 2 * kv)
    table = V * h * 2
    return cfg.layers * per_layer + table + 4 * h + L * kv_bytes_per_pos + kv_bytes_per_pos + 4 * V


def native_config(lf, world):
    """The `config` object of the line (shared by both arms)."""
    kv = "bf16" if lf == "int8" else "f32"
    return {"workload": f"qwen2.5-0.5b-shape {lf} batch-1 greedy decode (128-token prompt)",
            "batch_per_gpu": 1, "prompt": PROMPT, "kv": kv, "parallelism": f"dp{world}",
            "l2": "weights 631 MB > 126 MB L2; no flush"}


def ref_decode_rate(token_times):
    """The reference's decode throughput (src/benchmark.rs:85-91): N tokens
    emitted at token_times[0..N); (N - 1) / (t_last - t_first)."""
    if len(token_times) < 2 or token_times[-1] <= token_times[0]:
        return None
    return (len(token_times) - 1) / (token_times[-1] - token_times[0])


def run_reference(args, rank, world):
    """The reference's CPU token loop on this host's cores.

    The Rust crate cannot be built in this image, so its arithmetic runs as
    the oracle (oracle/qwen_oracle.c, the C restatement of the crate's scalar
    FP32 path; nothing of the product is loaded: the oracle draws the same
    seeded weights and prompt itself).  Same workload as the native arm: the
    0.5B model (INT8 per-row linears quantized by the oracle, BF16 table and
    KV), the same 128-token prompt, W warm-up then K timed greedy decode
    steps.  The reference is single-threaded (src/kernels.rs:8), so the
    decode steps run on one thread (`value`); the prompt is evaluated with
    every host thread (not part of the metric) to keep the run short, and
    a few steps on every host thread are reported beside the value."""
    if rank != 0:
        return 0
    import numpy as np

    from oracle import oracle
    lf = args.config
    cap = PROMPT + args.warmup + args.steps + 16
    cfg = oracle.qwen_0_5b_config(cap)
    all_threads = oracle.threads()
    om = oracle.Model(cfg, oracle.int8_model_weights(cfg, oracle.synthetic_weights(cfg, SEED, "bf16"), lf))
    prompt = oracle.synthetic_prompt(cfg.vocab_size, PROMPT, SEED)
    sess = oracle.Session(om, cap, kv_bf16=(lf == "int8"), budget=0)
    t0 = time.perf_counter()
    s, lg = sess.prefill(prompt)
    t_prefill = time.perf_counter() - t0
    if s:
        raise RuntimeError(f"oracle prefill failed: {s}")
    tok = int(np.argmax(lg))
    oracle.set_threads(1)
    for _ in range(args.warmup):
        sess.step(tok, lg)
        tok = int(np.argmax(lg))
    times = [time.perf_counter()]
    for _ in range(args.steps):
        sess.step(tok, lg)
        tok = int(np.argmax(lg))
        times.append(time.perf_counter())
    dt = times[-1] - times[0]
    value = args.steps / dt
    steps_all = min(args.steps, 8)
    oracle.set_threads(all_threads)
    t0 = time.perf_counter()
    for _ in range(steps_all):
        sess.step(tok, lg)
        tok = int(np.argmax(lg))
    rate_all = steps_all / (time.perf_counter() - t0)
    sample = (f"{args.steps} timed greedy decode steps on 1 thread after the 128-token prompt and "
              f"{args.warmup} warm-up steps (oracle: C restatement of the crate's FP32 path)")
    line = {
        "impl": "reference", "metric": "decode_tok_per_s", "value": value, "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32-accumulate/int8-weights" if lf == "int8" else "fp32-accumulate/bf16-weights",
        "data": "synthetic: N(0,0.02) weights seed 1, uniform prompts seed 1+rank",
        "config": native_config(lf, world),
        "decode_tok_per_s_reference_definition": ref_decode_rate(times),
        "prefill_tok_per_s": PROMPT / t_prefill, "prefill_threads": all_threads,
        "value_all_threads": rate_all, "all_threads": all_threads,
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": 1, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_native(args, topo):
    import torch

    import llm_inference_edu_b200 as qb
    from llm_inference_edu_b200 import dp, presets, synthetic

    rank, world, local_rank = topo.rank, topo.world, topo.local_rank
    torch.cuda.set_device(local_rank)
    lf = args.config
    kv = "bf16" if lf == "int8" else "f32"
    cap = PROMPT + args.warmup + args.steps + args.warmup + args.steps + 8
    cfg = presets.qwen_0_5b(cap)
    w = synthetic.weights(cfg, seed=SEED, dtype="bf16")
    model = qb.Decoder(cfg, w, linear_format=lf, table_format="bf16", device=local_rank)
    del w
    prompt = synthetic.prompt(cfg.vocab_size, PROMPT, seed=SEED + rank)
    sess = qb.CachedSession(model, cap, kv_dtype=kv, budget=0)
    stream = torch.cuda.ExternalStream(sess.stream())

    # Prompt evaluation (chunked multi-token path for all but the last token,
    # then one decode step), timed separately.
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    first = sess.prefill_into(prompt, None)
    ev1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = ev0.elapsed_time(ev1)

    tok = first
    ids = sess.decode_greedy(tok, args.warmup)
    tok = ids[-1]
    L0 = sess.processed()
    dp.barrier(topo)
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        ev0.record(stream)
        ids = sess.decode_greedy(tok, args.steps)
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    tok = ids[-1]
    ms = dp.max_over_ranks(topo, ms, device="cuda")

    # End to end through the public generation API (host buffers).
    gen = qb.GenerationSession(model, cap, qb.Sampling.Greedy, [], args.warmup + args.steps + 1,
                               kv_dtype=kv, budget=0)
    gen.start(prompt)
    for _ in range(args.warmup):
        gen.next_token()
    # The generation owns its own session stream; time with wall clock
    # bracketed by device synchronization.
    dp.barrier(topo)
    torch.cuda.synchronize()
    lat = []
    t0 = time.perf_counter()
    times = [t0]
    for _ in range(args.steps):
        a = time.perf_counter()
        gen.next_token()
        times.append(time.perf_counter())
        lat.append(times[-1] - a)
    torch.cuda.synchronize()
    e2e_s = dp.max_over_ranks(topo, time.perf_counter() - t0, device="cuda")
    ref_rate = ref_decode_rate(times)

    batched = run_batched(args, topo, model, cfg, kv)
    batched_split = run_batched(args, topo, model, cfg, kv, per_gpu=max(1, BATCH // topo.world))
    del model
    long_ctx = run_long_context(args, topo, kv) if lf == "int8" else None
    bf16 = run_decode_config(args, topo, "bf16") if lf == "int8" else None
    qwen7b = run_qwen7b(args, topo) if lf == "int8" else None

    if rank != 0:
        return 0
    peak, peak_kind = measured_peaks()
    kv_pos = cfg.layers * 2 * cfg.kv_dim * (2 if kv == "bf16" else 4)
    Lmean = L0 + (args.steps - 1) / 2.0
    bytes_step = algorithmic_bytes(cfg, lf, kv_pos, Lmean)
    step_s = ms / 1000.0 / args.steps
    achieved = bytes_step / step_s / 1e9
    value = world * args.steps / (ms / 1000.0)
    line = {
        "metric": "decode_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32-accumulate/int8-weights" if lf == "int8" else "fp32-accumulate/bf16-weights",
        "data": "synthetic: N(0,0.02) weights seed 1, uniform prompts seed 1+rank",
        "config": native_config(lf, world),
        "prefill_tok_per_s": PROMPT / (prefill_ms / 1000.0),
        "ms_per_token_p50": 1000.0 * statistics.median(lat),
        "decode_tok_per_s_reference_definition": ref_rate,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak,
                     "traffic": NCU_TRAFFIC_BYTES_INT8 if lf == "int8" else None,
                     "bytes_per_step": bytes_step, "peak_source": peak_kind},
        "e2e": {"value": world * args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 16,
                "d2h_bytes_per_step": 8},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "batched": batched,
        "batched_split": batched_split,
        "long_context": long_ctx,
        "bf16": bf16,
        "qwen7b": qwen7b,
    }
    if world == 1:
        line["cpu_baseline"] = cpu_baseline(args)
    print(json.dumps(line), flush=True)
    return 0


BATCH = 64


def run_batched(args, topo, model, cfg, kv, per_gpu=BATCH):
    """Batched greedy decode (BatchSession): `per_gpu` independent sequences
    per GPU (BATCH each, weak scaling; or BATCH // N each, the 64-sequence
    batch split over the N GPUs) with their own 128-token prompts, one
    multi-token forward per step (tensor-core GEMMs).  Device-timed with
    CUDA events on the batch's stream; each decode_greedy call copies its
    tokens host->device and its ids device->host inside the timed region."""
    import numpy as np
    import torch

    import llm_inference_edu_b200 as qb
    from llm_inference_edu_b200 import dp, synthetic

    steps = max(1, args.steps // 4)
    cap = PROMPT + args.warmup + steps + 1
    B = per_gpu
    prompts = np.stack([synthetic.prompt(cfg.vocab_size, PROMPT, seed=1000 + topo.rank * B + s)
                        for s in range(B)]).astype(np.uint32)
    b = qb.BatchSession(model, B, cap, kv_dtype=kv)
    stream = torch.cuda.ExternalStream(b.stream())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    first = b.prefill(prompts)
    ev1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = ev0.elapsed_time(ev1)
    ids = b.decode_greedy(first, args.warmup)
    dp.barrier(topo)
    torch.cuda.synchronize()
    ev0.record(stream)
    ids = b.decode_greedy(ids[-1], steps)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = dp.max_over_ranks(topo, ev0.elapsed_time(ev1), device="cuda")
    del b
    return {"sequences_per_gpu": B, "sequences_total": topo.world * B, "steps": steps,
            "value": topo.world * B * steps / (ms / 1000.0),
            "unit": "tok/s", "ms_per_step": ms / steps,
            "scaling": "weak" if B == BATCH else "strong",
            "prefill_tok_per_s": topo.world * B * PROMPT / (prefill_ms / 1000.0),
            "h2d_bytes_per_call": B * 4, "d2h_bytes_per_call": B * 4 * steps}


LONG_PROMPT = 8192
LONG_STEPS = 128


def run_long_context(args, topo, kv):
    """The long-context variant: an 8,192-token prompt through the chunked
    multi-token path, then 128 greedy tokens through the decode kernel
    (position-split attention), device-timed."""
    import torch

    import llm_inference_edu_b200 as qb
    from llm_inference_edu_b200 import dp, presets, synthetic

    cap = LONG_PROMPT + LONG_STEPS + 8
    cfg = presets.qwen_0_5b(cap)
    w = synthetic.weights(cfg, seed=SEED, dtype="bf16")
    model = qb.Decoder(cfg, w, linear_format="int8", table_format="bf16", device=topo.local_rank)
    del w
    prompt = synthetic.prompt(cfg.vocab_size, LONG_PROMPT, seed=2000 + topo.rank)
    sess = qb.CachedSession(model, cap, kv_dtype=kv, budget=0)
    stream = torch.cuda.ExternalStream(sess.stream())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    first = sess.prefill_into(prompt, None)
    ev1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = dp.max_over_ranks(topo, ev0.elapsed_time(ev1), device="cuda")
    ids = sess.decode_greedy(first, 8)
    dp.barrier(topo)
    torch.cuda.synchronize()
    ev0.record(stream)
    sess.decode_greedy(ids[-1], LONG_STEPS - 8)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = dp.max_over_ranks(topo, ev0.elapsed_time(ev1), device="cuda")
    return {"prompt": LONG_PROMPT, "steps": LONG_STEPS - 8,
            "prefill_tok_per_s": topo.world * LONG_PROMPT / (prefill_ms / 1000.0),
            "value": topo.world * (LONG_STEPS - 8) / (ms / 1000.0), "unit": "tok/s",
            "ms_per_token": ms / (LONG_STEPS - 8)}


def decode_timed(sess, tok, steps, topo):
    """K greedy decode steps on the device, timed with CUDA events on the
    session's stream (max over ranks); returns (ms, first cached position)."""
    import torch

    from llm_inference_edu_b200 import dp
    stream = torch.cuda.ExternalStream(sess.stream())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    L0 = sess.processed()
    dp.barrier(topo)
    torch.cuda.synchronize()
    ev0.record(stream)
    sess.decode_greedy(tok, steps)
    ev1.record(stream)
    torch.cuda.synchronize()
    return dp.max_over_ranks(topo, ev0.elapsed_time(ev1), device="cuda"), L0


def run_decode_config(args, topo, lf):
    """Batch-1 greedy decode of the 0.5B shape with BF16 linears (FP32 KV,
    the reference's cache type): the 128-token prompt, W warm-up then K
    device-timed steps, with its roofline (~988 MB of weights per step)."""
    import llm_inference_edu_b200 as qb
    from llm_inference_edu_b200 import presets, synthetic
    cap = PROMPT + 2 * args.warmup + args.steps + 8
    cfg = presets.qwen_0_5b(cap)
    w = synthetic.weights(cfg, seed=SEED, dtype="bf16")
    model = qb.Decoder(cfg, w, linear_format=lf, table_format="bf16", device=topo.local_rank)
    del w
    kv = "f32"
    sess = qb.CachedSession(model, cap, kv_dtype=kv, budget=0)
    first = sess.prefill_into(synthetic.prompt(cfg.vocab_size, PROMPT, seed=SEED + topo.rank), None)
    ids = sess.decode_greedy(first, args.warmup)
    ms, L0 = decode_timed(sess, ids[-1], args.steps, topo)
    peak, peak_kind = measured_peaks()
    kv_pos = cfg.layers * 2 * cfg.kv_dim * 4
    bytes_step = algorithmic_bytes(cfg, lf, kv_pos, L0 + (args.steps - 1) / 2.0)
    achieved = bytes_step / (ms / 1000.0 / args.steps) / 1e9
    return {"workload": f"qwen2.5-0.5b-shape {lf} linears batch-1 greedy decode (128-token prompt, f32 KV)",
            "steps": args.steps, "value": topo.world * args.steps / (ms / 1000.0), "unit": "tok/s",
            "ms_per_step": ms / args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "bytes_per_step": bytes_step, "peak_source": peak_kind}}


QWEN7B_PROMPT = 512


def qwen7b_shard_bytes(cfg, shard, kv_bytes_per_pos_rank, L, rows):
    """HBM bytes one rank moves per decode step of `rows` sequences: its
    shard's INT8 linears (plus row scales), its LM-head rows (BF16), the
    norms, and the K/V of its KV heads for every sequence's L cached
    positions."""
    h, hd = cfg.hidden_dim, cfg.head_dim
    qd = (shard["heads"][1] - shard["heads"][0]) * hd
    kv = (shard["kv_heads"][1] - shard["kv_heads"][0]) * hd
    ff = shard["ff"][1] - shard["ff"][0]
    nv = shard["vocab"][1] - shard["vocab"][0]
    mats = qd * h + 2 * kv * h + h * qd + 2 * ff * h + h * ff
    rows_sc = qd + 2 * kv + h + 2 * ff + h
    per_layer = mats + 4 * rows_sc + 4 * (2 * h) + 4 * (qd + 2 * kv)
    return cfg.layers * per_layer + nv * h * 2 + 4 * h + rows * (L + 1) * kv_bytes_per_pos_rank


def run_qwen7b(args, topo):
    """The Qwen2.5-7B shape (INT8 per-row linears, untied BF16 head, BF16
    KV), tensor-parallel over the N GPUs of the run (one shard per rank;
    partial sums after o_proj and down summed over NVLink peer memory):
    batch 1 and batch 32 greedy decode after 512-token prompts, each step
    device-timed (max over ranks).  At N = 1 the same model also runs the
    persistent decode kernel (``decode_kernel``)."""
    import numpy as np
    import torch

    import llm_inference_edu_b200 as qb
    from llm_inference_edu_b200 import dp, presets, synthetic, tp
    steps = max(4, args.steps // 4)
    cap = QWEN7B_PROMPT + args.warmup + steps + 8
    cfg = presets.qwen_7b(cap)
    w = synthetic.weights(cfg, seed=2, dtype="bf16", lazy=True)
    model = qb.Decoder(cfg, w, linear_format="int8", table_format="bf16", device=topo.local_rank,
                       tp=(topo.rank, topo.world))
    del w
    shard = model.shard()
    peak, peak_kind = measured_peaks()
    kvh = shard["kv_heads"][1] - shard["kv_heads"][0]
    kv_pos = cfg.layers * 2 * kvh * cfg.head_dim * 2
    out = {"workload": "qwen2.5-7b-shape int8 greedy decode (512-token prompts, bf16 kv)",
           "tp": topo.world, "shard": {k: list(v) if isinstance(v, tuple) else v for k, v in shard.items()}}
    if topo.world == 1:
        sess = qb.CachedSession(model, cap, kv_dtype="bf16", budget=0)
        first = sess.prefill_into(synthetic.prompt(cfg.vocab_size, QWEN7B_PROMPT, seed=3), None)
        ids = sess.decode_greedy(first, args.warmup)
        ms, L0 = decode_timed(sess, ids[-1], steps, topo)
        bytes_step = algorithmic_bytes(cfg, "int8", kv_pos, L0 + (steps - 1) / 2.0)
        achieved = bytes_step / (ms / 1000.0 / steps) / 1e9
        out["decode_kernel_batch1"] = {
            "steps": steps, "value": steps / (ms / 1000.0), "unit": "tok/s", "ms_per_step": ms / steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "bytes_per_step": bytes_step, "peak_source": peak_kind}}
        del sess
    for B in (1, 32):
        b = tp.batch(model, max(256, B), B, cap, "bf16", topo.rank, topo.world)
        prompts = np.stack([synthetic.prompt(cfg.vocab_size, QWEN7B_PROMPT, seed=3 + s)
                            for s in range(B)]).astype(np.uint32)
        stream = torch.cuda.ExternalStream(b.stream())
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dp.barrier(topo)
        torch.cuda.synchronize()
        ev0.record(stream)
        first = b.prefill(prompts)
        ev1.record(stream)
        torch.cuda.synchronize()
        prefill_ms = dp.max_over_ranks(topo, ev0.elapsed_time(ev1), device="cuda")
        ids = b.decode_greedy(first, args.warmup)
        dp.barrier(topo)
        torch.cuda.synchronize()
        ev0.record(stream)
        b.decode_greedy(ids[-1], steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        ms = dp.max_over_ranks(topo, ev0.elapsed_time(ev1), device="cuda")
        L0 = QWEN7B_PROMPT + args.warmup
        bytes_step = qwen7b_shard_bytes(cfg, shard, kv_pos, L0 + (steps - 1) / 2.0, B)
        achieved = bytes_step / (ms / 1000.0 / steps) / 1e9
        out[f"batch{B}"] = {
            "steps": steps, "value": B * steps / (ms / 1000.0), "unit": "tok/s", "ms_per_step": ms / steps,
            "prefill_tok_per_s": B * QWEN7B_PROMPT / (prefill_ms / 1000.0),
            "roofline_per_rank": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                                  "frac": achieved / peak, "bytes_per_step": bytes_step,
                                  "peak_source": peak_kind}}
        del b
    return out


def cpu_baseline(args):
    """The oracle on the host's cores, bounded sample (few decode steps)."""
    r, w = os.pipe()
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference", "--steps",
           str(args.cpu_steps), "--warmup", "1", "--config", args.config,
           "--cpu-steps", str(args.cpu_steps)]
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env).stdout
        d = json.loads(out.strip().splitlines()[-1])
        cb = d["cpu_baseline"]
        cb["prefill_tok_per_s"] = d.get("prefill_tok_per_s")
        return cb
    except Exception as e:  # reported, never fatal
        return {"value": None, "unit": "tok/s", "cores": None, "kind": "port", "sample": f"failed: {e}"}
    finally:
        os.close(r)
        os.close(w)


def main():
    args = parse()
    from llm_inference_edu_b200 import dp
    topo = dp.topology_from_env()
    if args.impl == "reference":
        return run_reference(args, topo.rank, topo.world)
    dp.init(topo, "nccl", timeout_s=600.0)
    try:
        return run_native(args, topo)
    finally:
        dp.shutdown(topo)


if __name__ == "__main__":
    sys.exit(main())
