"""Regenerates the large-shape golden files from the oracle (CPU only, minutes).

    python tests/golden/make_golden_7b.py llama7b      # about 10 minutes on 8 cores
    python tests/golden/make_golden_7b.py llama70b     # about 2 minutes on 8 cores

llama7b_decode.json — the benchmarked decode workload: the Llama-7B shape
(32 layers, d_model 4096, 32 x 128 MHA, SwiGLU 11008, vocab 32000, eps 1e-6,
theta 1e4; N(0, 0.02) weights with seed 0, int8 per output channel; KV cache
of 2048 positions), a 512-token prompt uniform over [0, 32000) with seed 0,
then 32 greedy tokens (cache positions 512..543).  For each step it keeps the
greedy token, the top-1 minus top-2 logit margin, max |logit| and the eight
largest logits with their indices, so a test can check the token stream
exactly and the logits within a tolerance of max |logit|.

llama70b_2layer.json — the Llama-70B width cut to 2 layers (d_model 8192,
64 query / 8 kv heads x 128, SwiGLU 28672, vocab 32000, eps 1e-5, theta 5e5;
seed 0 weights), batch 1 and batch 16 (the tensor-parallel workload's batch),
16-token prompts (seed 7 + sequence), 12 greedy tokens, the same per-step
records.

Both models are the same synthetic models the GPU engine draws with
tb_model_init_synthetic (the weight streams are shared; tests check it).
"""
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))

import numpy as np  # noqa: E402
import pyoracle  # noqa: E402

TOP = 8


def step_record(logits_row):
    """Greedy token, margin, max |logit| and the TOP largest logits of one step."""
    order = np.argsort(-logits_row, kind="stable")[:TOP]
    return {
        "token": int(pyoracle.argmax(logits_row)),
        "margin": float(logits_row[order[0]] - logits_row[order[1]]),
        "absmax": float(np.abs(logits_row).max()),
        "top_idx": [int(i) for i in order],
        "top_val": [float(logits_row[i]) for i in order],
    }


def greedy_records(model, prompt, n_new):
    """Prefill prompt [B, S], then n_new greedy steps; per step and row: step_record."""
    B = prompt.shape[0]
    _, last, _ = model.forward(prompt, want_logits=False)
    steps = []
    for _ in range(n_new):
        recs = [step_record(last[b]) for b in range(B)]
        steps.append(recs)
        nxt = np.array([[r["token"]] for r in recs], np.int64)
        _, last, _ = model.forward(nxt, want_logits=False)
    return steps


def llama7b(n_new=32):
    cfg = dict(pyoracle.LLAMA7B)
    t0 = time.time()
    m = pyoracle.Model(cfg, 1, seed=0)
    prompt = pyoracle.synth_tokens(0, 512, cfg["vocab"])
    steps = greedy_records(m, prompt[None, :], n_new)
    m.close()
    return {
        "config": cfg, "weight_seed": 0, "prompt_seed": 0, "prompt_len": 512, "batch": 1,
        "prompt": prompt.tolist(), "steps": [s[0] for s in steps],
        "seconds": round(time.time() - t0, 1),
    }


LLAMA70B_2L = dict(vocab=32000, dim=8192, layers=2, heads=64, kv_heads=8, hidden=28672, max_seq=64,
                   rope_base=500000.0, eps=1e-5)


def llama70b(n_new=12):
    cfg = dict(LLAMA70B_2L)
    out = {"config": cfg, "weight_seed": 0, "prompt_len": 16, "runs": {}}
    t0 = time.time()
    for B in (1, 16):
        m = pyoracle.Model(cfg, B, seed=0)
        prompt = np.stack([pyoracle.synth_tokens(7 + b, 16, cfg["vocab"]) for b in range(B)])
        steps = greedy_records(m, prompt, n_new)
        m.close()
        out["runs"][str(B)] = {"prompt": prompt.tolist(), "steps": steps}
    out["seconds"] = round(time.time() - t0, 1)
    return out


if __name__ == "__main__":
    pyoracle.build()
    pyoracle.set_threads(os.cpu_count() or 1)
    which = sys.argv[1] if len(sys.argv) > 1 else "llama7b"
    if which == "llama7b":
        data, name = llama7b(), "llama7b_decode.json"
    elif which == "llama70b":
        data, name = llama70b(), "llama70b_2layer.json"
    else:
        raise SystemExit("usage: make_golden_7b.py llama7b|llama70b")
    with open(os.path.join(HERE, name), "w") as f:
        json.dump(data, f, indent=0)
    print("wrote", name, data.get("seconds"))
