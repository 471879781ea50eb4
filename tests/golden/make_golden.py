"""Regenerates the committed golden fixtures under tests/golden/.

Run in a container that has the reference checkout:

    python tests/golden/make_golden.py /path/to/llm_inference_edu

Two kinds of files are written:

1. The reference's own golden vectors (``fixtures/t01..t04``, ``t06``,
   ``t25``, ``t28``) copied byte-for-byte.  They were produced by the reference's
   independent NumPy equations and are the vectors its Rust tests assert.
2. ``tinyb-numpy.json``: golden logits and greedy ids for the Tiny-B
   workload (hidden 64, 4/2 heads, head_dim 16, ff 128, vocab 256, 2 layers,
   eps 1e-6, theta 1e4, N(0, 0.02) weights from seed 0), computed by
   importing the reference's own NumPy decoder equations
   (``reference/decoder.py:outputs_for``) on this repository's synthetic
   weights.  The module's NumPy version pin (2.3.2) is bypassed because the
   equations do not depend on it; the weights are handed to it through a
   temporary directory laid out like the reference checkout.
"""
from __future__ import annotations

import importlib
import json
import os
import shutil
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
COPIED = ["t01-inputs.json", "t01-expected.json", "t02-inputs.json", "t02-expected.json",
          "t03-inputs.json", "t03-expected.json", "t04-inputs.json", "t04-expected.json",
          "t25-continuation.json", "t28-tiny-context.json", "t06-tokenizer.json"]


def copy_reference_vectors(ref):
    for name in COPIED:
        shutil.copyfile(os.path.join(ref, "fixtures", name), os.path.join(HERE, name))


def numpy_decoder(ref, model_json):
    """Imports reference/decoder.py with its fixture root pointed at a
    temporary directory holding `model_json` as fixtures/tiny-model.json."""
    sys.path.insert(0, os.path.join(ref, "reference"))
    try:
        decoder = importlib.import_module("decoder")
    finally:
        sys.path.pop(0)
    tmp = tempfile.mkdtemp()
    os.makedirs(os.path.join(tmp, "fixtures"))
    with open(os.path.join(tmp, "fixtures", "tiny-model.json"), "w") as f:
        json.dump(model_json, f)
    decoder.ROOT = type(decoder.ROOT)(tmp)
    return decoder.outputs_for, tmp


def tinyb_vectors(ref):
    sys.path.insert(0, REPO)
    from llm_inference_edu_b200 import presets, synthetic
    cfg = presets.tiny_b()
    w = synthetic.weights(cfg, seed=0, dtype="f32")
    model_json = {"config": cfg.to_reference_json(), "weights": synthetic.to_reference_json(w)}
    outputs_for, tmp = numpy_decoder(ref, model_json)
    real = np.__version__
    np.__version__ = "2.3.2"
    try:
        prompt = synthetic.prompt(cfg.vocab_size, 8, seed=0)
        ids = list(prompt)
        greedy = []
        for _ in range(32):
            logits = outputs_for(ids)["logits"]
            nxt = int(np.argmax(logits[-1]))
            greedy.append(nxt)
            ids.append(nxt)
        full = outputs_for(ids[:-1])["logits"]
    finally:
        np.__version__ = real
        shutil.rmtree(tmp)
    rows = [{"position": p, "logits": full[p].tolist()} for p in (0, 7, 20, len(ids) - 2)]
    out = {"generator": "reference/decoder.py:outputs_for (NumPy FP64 equations)",
           "config": cfg.to_reference_json(), "weight_seed": 0, "prompt": [int(v) for v in prompt],
           "greedy": greedy, "positions": rows, "history": [int(v) for v in ids]}
    with open(os.path.join(HERE, "tinyb-numpy.json"), "w") as f:
        json.dump(out, f)
        f.write("\n")


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    ref = sys.argv[1]
    copy_reference_vectors(ref)
    tinyb_vectors(ref)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
