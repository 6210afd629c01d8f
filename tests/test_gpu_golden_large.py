"""Parity at the benchmarked shapes against the oracle's golden files
(tests/golden/make_golden_7b.py): the Llama-7B shape decoding from position
512 of a 512-token prompt — the workload bench.py times, on the persistent
decode kernel — and the Llama-70B width cut to 2 layers at batch 1 and 16.

Per step: the greedy token equals the oracle's, and the logits at the
oracle's eight largest entries are within LOGIT_TOL * max |logit| of its
values.  Each step feeds the oracle's token (teacher forcing), so one
mismatch is reported where it happens.
"""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
LOGIT_TOL = 1e-3


def load(name):
    with open(os.path.join(HERE, "golden", name)) as f:
        return json.load(f)


def check_step(logits_row, rec, where):
    got = int(np.argmax(logits_row))
    assert got == rec["token"], f"{where}: token {got} != {rec['token']} (oracle margin {rec['margin']:.4g})"
    err = np.abs(logits_row[rec["top_idx"]] - np.array(rec["top_val"], np.float32)).max()
    assert err <= LOGIT_TOL * rec["absmax"], f"{where}: logit error {err:.3g} > {LOGIT_TOL} x {rec['absmax']:.3g}"


def test_llama7b_decode_from_512(tb, cuda):
    """32 greedy steps at cache positions 512..543 of the 7B-shape model (the
    bench workload), through the same decode path the bench times."""
    g = load("llama7b_decode.json")
    m = tb.QuantizedModel(g["config"], batch=1, device=0)
    m.init_synthetic(g["weight_seed"])
    prompt = np.array(g["prompt"], np.int64)[None, :]
    logits, nxt = m.forward(prompt)
    check_step(logits[0], g["steps"][0], "prefill")
    assert int(nxt[0]) == g["steps"][0]["token"]
    persistent = m.launches_per_step == 1
    for k in range(1, len(g["steps"])):
        m.decode(1, start_tokens=np.array([g["steps"][k - 1]["token"]]))
        check_step(m.last_logits()[0], g["steps"][k], f"step {k} (position {511 + k})")
    m.close()
    assert persistent, "the batch-1 7B shape should decode on the persistent kernel"


def test_llama7b_greedy_stream_matches(tb, cuda):
    """Free-running greedy decode (each step feeds the engine's own token),
    the way bench.py and Generate run it: the stream equals the oracle's."""
    g = load("llama7b_decode.json")
    m = tb.QuantizedModel(g["config"], batch=1, device=0)
    m.init_synthetic(g["weight_seed"])
    want = [s["token"] for s in g["steps"]]
    got = m.generate_greedy(np.array(g["prompt"], np.int64)[None, :], len(want))
    m.close()
    assert got[0].tolist() == want


@pytest.mark.parametrize("batch", [1, 16])
def test_llama70b_width_two_layers(tb, cuda, batch):
    """d_model 8192, 64 query / 8 kv heads (GQA), SwiGLU 28672, vocab 32000,
    theta 5e5, 2 layers: batch 1 (the persistent kernel) and batch 16 (the
    tensor-parallel workload's batch on one GPU)."""
    g = load("llama70b_2layer.json")
    run = g["runs"][str(batch)]
    m = tb.QuantizedModel(g["config"], batch=batch, device=0)
    m.init_synthetic(g["weight_seed"])
    logits, _ = m.forward(np.array(run["prompt"], np.int64))
    for b in range(batch):
        check_step(logits[b], run["steps"][0][b], f"prefill row {b}")
    for k in range(1, len(run["steps"])):
        m.decode(1, start_tokens=np.array([r["token"] for r in run["steps"][k - 1]]))
        lg = m.last_logits()
        for b in range(batch):
            check_step(lg[b], run["steps"][k][b], f"step {k} row {b}")
    m.close()
