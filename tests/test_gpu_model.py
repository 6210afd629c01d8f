"""The QuantizedModel engine on the GPU against the oracle: greedy tokens
identical for the stated prefixes, logits within 1e-3 of max |logit|.
"""
import json
import os

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
LOGIT_TOL = 1e-3


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(HERE, "golden", "tiny_greedy.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def tiny_gpu(tb, cuda, golden):
    m = tb.QuantizedModel(golden["config"], batch=1, device=0)
    m.init_synthetic(golden["weight_seed"])
    yield m
    m.close()


def test_tiny_weights_bit_exact(oracle, tiny_gpu, golden):
    ref = oracle.Model(golden["config"], 1, seed=golden["weight_seed"])
    for layer in (0, 3, 7):
        for mat in range(7):
            q, s = tiny_gpu.get_linear(layer, mat, ref.shape(mat))
            np.testing.assert_array_equal(q, ref.q(layer, mat))
            np.testing.assert_array_equal(s.view(np.uint32), ref.scale(layer, mat).view(np.uint32))


def test_tiny_greedy_128_tokens(tiny_gpu, golden):
    """Config 1: 128-token prompt (seed 1), 128 greedy tokens == the oracle's."""
    toks = tiny_gpu.generate_greedy(np.array(golden["prompt"]), 128)
    assert toks[0].tolist() == golden["tokens"]


def test_tiny_teacher_forced_decode(tiny_gpu, golden):
    """The prompt fed one token per CUDA-graph decode step; every argmax == the oracle's."""
    prompt = golden["prompt"]
    tiny_gpu.reset()
    tiny_gpu.forward(np.array([[prompt[0]]]), want_logits=False)
    for t in prompt[1:]:
        tiny_gpu.decode(1, start_tokens=np.array([t]))
    got = tiny_gpu.tokens(len(prompt))[:, 0].tolist()
    assert got == golden["forced"]


def test_tiny_prefill_and_decode_logits(oracle, tiny_gpu, golden):
    ref = oracle.Model(golden["config"], 1, seed=golden["weight_seed"])
    prompt = np.array([golden["prompt"]], np.int64)
    tiny_gpu.reset()
    lg, nxt = tiny_gpu.forward(prompt)
    _, want, _ = ref.forward(prompt, want_logits=False)
    assert rel_err(lg, want) <= LOGIT_TOL
    assert int(nxt[0]) == int(np.argmax(want[0]))
    for t in (17, 31000, 5):
        lg, _ = tiny_gpu.forward(np.array([[t]]))
        _, want, _ = ref.forward(np.array([[t]], np.int64), want_logits=False)
        assert rel_err(lg, want) <= LOGIT_TOL


GQA = dict(vocab=1000, dim=256, layers=3, heads=8, kv_heads=2, hidden=384, max_seq=160, rope_base=500000.0,
           eps=1e-5)


@pytest.mark.parametrize("batch", [1, 3, 12, 16])
def test_gqa_batched_greedy(oracle, tb, cuda, batch):
    """GQA (8 query heads on 2 kv heads, the 70B grouping pattern) and a
    lockstep batch (12 and 16: the fused decode step in groups of 8 rows)."""
    m = tb.QuantizedModel(GQA, batch=batch, device=0)
    m.init_synthetic(5)
    ref = oracle.Model(GQA, batch, seed=5)
    prompt = np.stack([oracle.synth_tokens(7 + b, 40, GQA["vocab"]) for b in range(batch)])
    want, margins = ref.generate_greedy(prompt, 24)
    got = m.generate_greedy(prompt, 24)
    np.testing.assert_array_equal(got, want)
    m.close()


GQA64 = dict(vocab=1000, dim=512, layers=2, heads=8, kv_heads=2, hidden=768, max_seq=160, rope_base=500000.0,
             eps=1e-5)


@pytest.mark.parametrize("batch", [2, 8, 12, 24, 32, 64])
def test_gqa64_batched_greedy(oracle, tb, cuda, batch):
    """head_dim 64 (the captured decode step) on the single-pass tcgen05 GEMV
    projections (RMSNorm fused into the digit kernel)."""
    m = tb.QuantizedModel(GQA64, batch=batch, device=0)
    m.init_synthetic(5)
    ref = oracle.Model(GQA64, batch, seed=5)
    prompt = np.stack([oracle.synth_tokens(7 + b, 40, GQA64["vocab"]) for b in range(batch)])
    want, margins = ref.generate_greedy(prompt, 24)
    got = m.generate_greedy(prompt, 24)
    np.testing.assert_array_equal(got, want)
    m.close()


# d_model 8192 as the 70B shape (64 query / 8 kv heads x 128): too wide for the
# fused lm_head's staged rows, so the captured step takes the fp32 GEMM + key path
WIDE = dict(vocab=1000, dim=8192, layers=1, heads=64, kv_heads=8, hidden=1024, max_seq=64, rope_base=500000.0,
            eps=1e-5)


def test_wide_model_batched_greedy(oracle, tb, cuda):
    batch = 9
    m = tb.QuantizedModel(WIDE, batch=batch, device=0)
    m.init_synthetic(5)
    ref = oracle.Model(WIDE, batch, seed=5)
    prompt = np.stack([oracle.synth_tokens(7 + b, 16, WIDE["vocab"]) for b in range(batch)])
    want, margins = ref.generate_greedy(prompt, 8)
    got = m.generate_greedy(prompt, 8)
    np.testing.assert_array_equal(got, want)
    m.close()


def test_llama7b_shape_prefix(oracle, tb, cuda):
    """7B shape (32 layers, d 4096, 32 x 128, F 11008): 16-token prompt + 4
    greedy tokens == the oracle's, on the same device-generated weights."""
    cfg = dict(oracle.LLAMA7B, max_seq=64)
    m = tb.QuantizedModel(cfg, batch=1, device=0)
    m.init_synthetic(0)
    ref = oracle.Model(cfg, 1, seed=0, generate=False)
    for layer in range(cfg["layers"]):
        for mat in range(7):
            q, s = m.get_linear(layer, mat, ref.shape(mat))
            ref.q(layer, mat)[...] = q
            ref.scale(layer, mat)[...] = s
    # tie the copied weights to the host generator on sample rows
    w = oracle.synth_normal(0, 5 * 8 + 4, 4096, 0.02, offset=123 * 4096)
    _, q_row, s_row = oracle.quantize(w[None, :], 0)
    np.testing.assert_array_equal(ref.q(5, 4)[123], q_row[0])
    ref.embed()[...] = oracle.synth_normal(0, oracle.STREAM_EMBED, 32000 * 4096, 0.02).reshape(32000, 4096)
    ref.lm_head()[...] = oracle.synth_normal(0, oracle.STREAM_LMHEAD, 32000 * 4096, 0.02).reshape(32000, 4096)
    prompt = oracle.synth_tokens(0, 16, 32000)
    want, margins = ref.generate_greedy(prompt[None, :], 4)
    got = m.generate_greedy(prompt[None, :], 4)
    np.testing.assert_array_equal(got, want)
    m.close()


@pytest.mark.parametrize("batch,T,K,P", [(1, 0.8, 20, 0.9), (3, 1.2, 0, 0.0), (12, 0.7, 40, 0.0)])
def test_sampled_generation_matches_oracle(oracle, tb, cuda, batch, T, K, P):
    """QuantizedModel.Generate with the Sampler: the device sampler draws every
    token from the step's logits with the counter generator's uniforms; the
    oracle does the same with the restated Sampler.  Batch 1 runs the
    persistent decode kernel, 3 and 12 the captured multi-kernel step."""
    cfg = GQA64 if batch > 1 else dict(GQA64, heads=8, kv_heads=8)
    m = tb.QuantizedModel(cfg, batch=batch, device=0)
    m.init_synthetic(5)
    ref_w = oracle.Model(cfg, batch, seed=5)
    prompt = np.stack([oracle.synth_tokens(7 + b, 24, cfg["vocab"]) for b in range(batch)])
    want = oracle.generate_sample(ref_w, prompt, 16, T, K, P, seed=3)
    got = m.generate_sample(prompt, 16, T, K, P, seed=3)
    np.testing.assert_array_equal(got, want)
    m.close()
    ref_w.close()


@pytest.mark.parametrize("cfg,batch,group", [("GQA", 1, 128), ("GQA", 3, 128), ("GQA64", 1, 128),
                                             ("GQA64", 12, 256), ("GQA64", 40, 128)])
def test_grouped_model_greedy(oracle, tb, cuda, cfg, batch, group):
    """A model quantized per group (QuantizeModel(m, groupSize)): head_dim 32
    decodes through the per-step grouped DequantizeMatmul, head_dim 64 through
    the captured step's tcgen05 GEMV with per-group scales (batch 1 included);
    the 40-sequence prompt takes the grouped tensor-core GEMM.  Tokens equal
    the grouped oracle's; the synthetic weights and their scales equal the
    oracle's quantization of the same draws."""
    c = GQA if cfg == "GQA" else GQA64
    m = tb.QuantizedModel(c, batch=batch, device=0, group=group)
    m.init_synthetic(5)
    ref = oracle.Model(c, batch, seed=5, group=group)
    for mat in (0, 3, 6):
        q, s = m.get_linear(1, mat, ref.shape(mat))
        np.testing.assert_array_equal(q, ref.q(1, mat))
        np.testing.assert_array_equal(s, ref.scale(1, mat))
    prompt = np.stack([oracle.synth_tokens(7 + b, 40, c["vocab"]) for b in range(batch)])
    want, margins = ref.generate_greedy(prompt, 16)
    got = m.generate_greedy(prompt, 16)
    np.testing.assert_array_equal(got, want)
    m.close()


def test_grouped_model_rejects_ragged_groups(tb, cuda):
    """Every Linear's input width must be a whole number of groups."""
    with pytest.raises(tb.TendoB200Error):
        tb.QuantizedModel(GQA64, batch=1, device=0, group=384)
