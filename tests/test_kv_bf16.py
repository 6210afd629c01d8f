"""The bf16 KV cache option (TB_MODEL_KV_BF16): the oracle's restatement of it
on the CPU, and the engine on the GPU against that restatement.

A bf16 cache is a numerics change against the reference, which stores K and V
in fp32; the option exists to halve the cache bytes the decode attention
streams.  Its oracle rounds each K (after RoPE) and V value to the nearest
even bf16 as it is appended and otherwise computes as the reference does, so
the engine with the option is held to the same bar as without it: greedy
tokens identical to that oracle, logits within 1e-3 of max |logit|.  Against
the fp32-cache oracle the logits move by the rounding (tolerance 2e-2 here).
"""
import numpy as np
import pytest

from conftest import rel_err

GQA = dict(vocab=1000, dim=256, layers=3, heads=8, kv_heads=2, hidden=384, max_seq=160, rope_base=500000.0,
           eps=1e-5)
GQA64 = dict(vocab=1000, dim=512, layers=2, heads=8, kv_heads=2, hidden=768, max_seq=160, rope_base=500000.0,
             eps=1e-5)


def test_round_bf16_matches_torch(oracle):
    import torch

    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 3.0,
        # exact ties between two bf16 values: both parities of the kept bit
        (np.arange(1, 2001, dtype=np.uint32) << 16 | 0x8000).view(np.float32),
        np.array([0.0, -0.0, 1e-38, -1e-40, 3.0e38, -3.4e38, np.inf, -np.inf], np.float32),
    ])
    L = oracle.lib()
    got = np.array([L.or_round_bf16(float(v)) for v in x], np.float32)
    want = torch.from_numpy(x).bfloat16().float().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_oracle_bf16_cache_holds_bf16_values(oracle):
    """With the option the cache holds bf16 values; in layer 0 (same inputs
    either way) they are the fp32 cache's values rounded to nearest even."""
    import torch

    a = oracle.Model(GQA, 2, seed=5)
    b = oracle.Model(GQA, 2, seed=5)
    b.set_kv_bf16(True)
    prompt = np.stack([oracle.synth_tokens(7 + i, 20, GQA["vocab"]) for i in range(2)])
    a.forward(prompt, want_logits=False)
    b.forward(prompt, want_logits=False)
    for layer in range(GQA["layers"]):
        for ca, cb in ((a.kcache(layer), b.kcache(layer)), (a.vcache(layer), b.vcache(layer))):
            got = cb[:, :, :20].copy()
            assert np.all(got.view(np.uint32) & 0xFFFF == 0)
            if layer == 0:
                want = torch.from_numpy(ca[:, :, :20].copy()).bfloat16().float().numpy()
                np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("cfg,batch", [(GQA, 1), (GQA, 3), (GQA64, 1), (GQA64, 8), (GQA64, 32)])
def test_kv_bf16_greedy_matches_oracle(oracle, tb, cuda, cfg, batch):
    """head_dim 32 runs the per-step kernels, head_dim 64 the captured step on
    the tcgen05 GEMV path (batch 1 included); the prompt's prefill writes and
    reads the bf16 cache through the tiled attention."""
    m = tb.QuantizedModel(cfg, batch=batch, device=0, kv_bf16=True)
    m.init_synthetic(5)
    ref = oracle.Model(cfg, batch, seed=5)
    ref.set_kv_bf16(True)
    prompt = np.stack([oracle.synth_tokens(7 + b, 40, cfg["vocab"]) for b in range(batch)])
    want, _ = ref.generate_greedy(prompt, 24)
    got = m.generate_greedy(prompt, 24)
    np.testing.assert_array_equal(got, want)
    m.close()


@pytest.mark.gpu
def test_kv_bf16_logits(oracle, tb, cuda):
    batch = 2
    m = tb.QuantizedModel(GQA64, batch=batch, device=0, kv_bf16=True)
    m.init_synthetic(5)
    ref16 = oracle.Model(GQA64, batch, seed=5)
    ref16.set_kv_bf16(True)
    ref32 = oracle.Model(GQA64, batch, seed=5)
    prompt = np.stack([oracle.synth_tokens(11 + b, 48, GQA64["vocab"]) for b in range(batch)])
    lg, _ = m.forward(prompt)
    _, w16, _ = ref16.forward(prompt, want_logits=False)
    _, w32, _ = ref32.forward(prompt, want_logits=False)
    assert rel_err(lg, w16) <= 1e-3
    assert rel_err(lg, w32) <= 2e-2
    for t in (17, 999, 5):
        step = np.full((batch, 1), t, np.int64)
        lg, _ = m.forward(step)
        _, w16, _ = ref16.forward(step, want_logits=False)
        assert rel_err(lg, w16) <= 1e-3
    m.close()
