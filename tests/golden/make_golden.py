"""Regenerates tests/golden/*.json from the oracle (CPU only, seconds).

    python tests/golden/make_golden.py

tiny_greedy.json: the tiny Llama workload (8 layers, d_model 512, 8 x 64
MHA, SwiGLU 1408, vocab 32000, eps 1e-5, theta 1e4; N(0, 0.02) weights with
seed 0, int8 per channel) — a 128-token prompt uniform over [0, 32000) with
seed 1, then 128 greedy tokens, with the top-1 minus top-2 logit margin of
every step.  The GPU engine must reproduce the token stream exactly.
That greedy stream settles on one token (a random-weight model), so the file
also holds the teacher-forced predictions: the prompt fed one token per
decode step, the greedy argmax after each (128 different contexts).
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))

import numpy as np  # noqa: E402
import pyoracle  # noqa: E402

TINY = dict(pyoracle.TINY)


def tiny_greedy():
    m = pyoracle.Model(TINY, 1, seed=0)
    prompt = pyoracle.synth_tokens(1, 128, TINY["vocab"])
    toks, margins = m.generate_greedy(prompt, 128)
    m.reset()
    forced, forced_margins = [], []
    for t in prompt:
        _, last, _ = m.forward(np.array([[t]], np.int64), want_logits=False)
        order = np.argsort(-last[0], kind="stable")
        forced.append(int(pyoracle.argmax(last[0])))
        forced_margins.append(float(last[0][order[0]] - last[0][order[1]]))
    return {
        "config": TINY,
        "weight_seed": 0,
        "prompt_seed": 1,
        "prompt": prompt.tolist(),
        "tokens": toks[0].tolist(),
        "margins": [float(x) for x in margins[0]],
        "forced": forced,
        "forced_margins": forced_margins,
    }


if __name__ == "__main__":
    pyoracle.build()
    with open(os.path.join(HERE, "tiny_greedy.json"), "w") as f:
        json.dump(tiny_greedy(), f, indent=1)
    print("wrote tiny_greedy.json")
