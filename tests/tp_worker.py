"""One rank of the tensor-parallel parity tests (started by
tests/test_gpu_tp.py with torch.multiprocessing, one process per GPU).  The
ranks exchange their communicator handles over a gloo process group on
127.0.0.1 with a short timeout; each writes its greedy ids and its
vocabulary rows of the logits to `out_dir`."""
import datetime
import os


def build_weights(name):
    from llm_inference_edu_b200 import presets, synthetic
    if name == "0.5b":
        return presets.qwen_0_5b, synthetic.weights(presets.qwen_0_5b(), seed=1, dtype="bf16")
    return presets.qwen_7b, synthetic.weights(presets.qwen_7b(), seed=2, dtype="bf16", lazy=True)


def run(rank, size, port, out_dir, name, prompt_len, steps, sequences, kv):
    import numpy as np
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=size,
                            timeout=datetime.timedelta(seconds=120))
    try:
        torch.cuda.set_device(rank)
        from llm_inference_edu_b200 import api, synthetic, tp
        make_cfg, w = build_weights(name)
        cap = prompt_len + steps + 8
        cfg = make_cfg(cap)
        m = api.Decoder(cfg, w, linear_format="int8", table_format="bf16", device=rank, tp=(rank, size))
        del w
        b = tp.batch(m, max(256, sequences), sequences, cap, kv, rank, size)
        prompts = np.stack([synthetic.prompt(cfg.vocab_size, prompt_len, seed=40 + s)
                            for s in range(sequences)]).astype(np.uint32)
        first = b.prefill(prompts)
        lg0 = b.logits()
        ids = b.decode_greedy(first, steps)
        lg1 = b.logits()
        sh = m.shard()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), first=first, ids=ids, lg0=lg0, lg1=lg1,
                 vocab=np.asarray(sh["vocab"]), heads=np.asarray(sh["heads"]))
        del b
        dist.barrier()
    finally:
        dist.destroy_process_group()
