"""The oracle against every known-answer test tendo's own suite holds for this
path, plus an independent numpy restatement of the integer/byte arithmetic
(bit-exact) and self-consistency checks of the model restatement.  CPU only.
"""
import math

import numpy as np
import pytest


# --- nn/quantize_test.go -----------------------------------------------------
def test_quantize_per_channel_shapes(oracle):
    # TestQuantize_PerChannel (nn/quantize_test.go:20-60): W [2, 4], scale [2]
    w = np.array([[1, 2, 3, 4], [-1, -2, -3, -4]], np.float32)
    qf, qi, s = oracle.quantize(w, 0)
    assert qf.shape == (2, 4) and qi.shape == (2, 4) and s.shape == (2,)
    # maxAbs 4 -> scale 4/127; q = round(w / scale) = round(w * 31.75)
    np.testing.assert_array_equal(qi[0], [32, 64, 95, 127])
    np.testing.assert_array_equal(qi[1], [-32, -64, -95, -127])
    assert s[0] == np.float32(4.0) / np.float32(127.0)


def test_quantize_per_group_shapes(oracle):
    # TestQuantize_PerGroup (nn/quantize_test.go:62-87): group 4 over K 8 -> scale [N, 2]
    w = (np.arange(16, dtype=np.float32) * np.float32(0.1)).reshape(2, 8)
    _, _, s = oracle.quantize(w, 4)
    assert s.shape == (2, 2)


def test_dequantize_round_trip(oracle):
    # TestDequantize_PerChannel (nn/quantize_test.go:116-158): |deq - w| <= max(2% |w|, 0.1)
    w = np.array([[1.27, 2.54, 3.81, 5.08], [-1.27, -2.54, -3.81, -5.08]], np.float32)
    _, qi, s = oracle.quantize(w, 0)
    deq = oracle.dequantize(qi, s, 0)
    tol = np.maximum(np.abs(w) * 0.02, 0.1)
    assert np.all(np.abs(deq - w) <= tol)


def test_dequantize_per_group_shape(oracle):
    # TestDequantize_PerGroup (nn/quantize_test.go:160-181)
    w = (np.arange(16, dtype=np.float32) * np.float32(0.1)).reshape(2, 8)
    _, qi, s = oracle.quantize(w, 4)
    assert oracle.dequantize(qi, s, 4).shape == (2, 8)


def test_quantize_zero_values(oracle):
    # TestQuantize_ZeroValues (nn/quantize_test.go:183-204): zero rows -> scale 1, q 0, deq 0
    w = np.zeros((2, 4), np.float32)
    _, qi, s = oracle.quantize(w, 0)
    assert np.all(s == 1.0) and np.all(qi == 0)
    assert np.all(oracle.dequantize(qi, s, 0) == 0)


def _np_quantize(w, group):
    """Independent numpy restatement of quantizePerChannel / quantizePerGroup
    (nn/quantize.go:67-187): fp32 maxAbs, fp32 scale, fp32 w / scale, Go's
    math.Round (half away from zero) in fp64, clamp."""
    N, K = w.shape
    g = group or K
    wg = w.reshape(N, K // g, g)
    max_abs = np.abs(wg).max(axis=2).astype(np.float32)
    scale = (max_abs / np.float32(127.0)).astype(np.float32)
    scale[scale == 0] = np.float32(1.0)
    q = (wg / scale[:, :, None]).astype(np.float32).astype(np.float64)
    q = np.sign(q) * np.floor(np.abs(q) + 0.5)
    q = np.clip(q, -128, 127).astype(np.int8).reshape(N, K)
    return q, (scale if group else scale[:, 0])


@pytest.mark.parametrize("group", [0, 32, 128])
def test_quantize_matches_numpy_restatement(oracle, group):
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    w[3] = 0.0  # a zero row
    w[5, 7] = 0.5 * np.float32(w[5].max())  # near-half values exercise rounding
    _, qi, s = oracle.quantize(w, group)
    q2, s2 = _np_quantize(w, group)
    np.testing.assert_array_equal(qi, q2)
    np.testing.assert_array_equal(s.view(np.uint32), s2.astype(np.float32).view(np.uint32))


def test_quantize_rounds_half_away_from_zero(oracle):
    # w / scale lands exactly on .5 when maxAbs = 127 (scale 1): 2.5 -> 3, -2.5 -> -3
    w = np.array([[127.0, 2.5, -2.5, 0.5, -0.5, 126.5]], np.float32)
    _, qi, s = oracle.quantize(w, 0)
    assert s[0] == 1.0
    np.testing.assert_array_equal(qi[0], [127, 3, -3, 1, -1, 127])


# --- nn/rope_test.go -----------------------------------------------------------
def test_rope_position_zero(oracle):
    # TestRoPE_FrequencyValues (nn/rope_test.go:181-213)
    c, s = oracle.rope_tables(4, 4, 10000.0)
    assert np.all(np.abs(c[0] - 1.0) <= 1e-5) and np.all(np.abs(s[0]) <= 1e-5)


def test_rope_tables_follow_reference_formula(oracle):
    # nn/rope.go:28-45: invFreq = 1 / float32(base^(2i/dim)); freq = float32(pos) * invFreq
    dim, max_seq, base = 64, 32, 10000.0
    c, s = oracle.rope_tables(dim, max_seq, base)
    inv = (np.float32(1.0) / np.array([np.float32(math.pow(base, 2 * i / dim)) for i in range(dim // 2)],
                                      np.float32)).astype(np.float32)
    for p in (0, 1, 17, 31):
        f = (np.float32(p) * inv).astype(np.float32)
        np.testing.assert_array_equal(c[p], np.array([np.float32(math.cos(float(x))) for x in f], np.float32))
        np.testing.assert_array_equal(s[p], np.array([np.float32(math.sin(float(x))) for x in f], np.float32))


def test_rope_apply_rotate_half(oracle):
    # rotateHalf (nn/rope.go:141-197): out0 = x0 cos - x1 sin, out1 = x0 sin + x1 cos
    rng = np.random.default_rng(3)
    x = rng.standard_normal((1, 2, 3, 8)).astype(np.float32)
    c, s = oracle.rope_tables(8, 16, 10000.0)
    y = oracle.rope_apply(x, c, s, 5)
    for si in range(3):
        cc, ss = c[5 + si], s[5 + si]
        x0, x1 = x[:, :, si, :4], x[:, :, si, 4:]
        np.testing.assert_array_equal(y[:, :, si, :4], (x0 * cc - x1 * ss).astype(np.float32))
        np.testing.assert_array_equal(y[:, :, si, 4:], (x0 * ss + x1 * cc).astype(np.float32))


# --- activation_test.go --------------------------------------------------------
def test_softmax_known_answers(oracle):
    # TestSoftmax (activation_test.go:114-228)
    for row in ([1, 2, 3], [1000, 1001, 1002]):
        p = oracle.softmax(np.array([row], np.float32))
        assert abs(float(p.sum()) - 1) <= 1e-5
    p = oracle.softmax(np.array([[1, 2, 3], [1, 1, 1]], np.float32))
    assert np.all(np.abs(p.sum(axis=1) - 1) <= 1e-5)
    assert np.all(np.abs(p[1] - 1.0 / 3.0) <= 1e-5)


def test_softmax_masked_entries(oracle):
    p = oracle.softmax(np.array([[0.5, -np.inf, 1.5, -np.inf]], np.float32))
    assert p[0, 1] == 0 and p[0, 3] == 0 and abs(float(p.sum()) - 1) <= 1e-6


def test_silu_zero(oracle):
    # TestSiLU (activation_test.go:315-333)
    assert abs(float(oracle.silu(np.zeros(1, np.float32))[0])) <= 1e-6


def test_silu_formula(oracle):
    # cpu/backend.go:193-198: x * float32(1 / (1 + exp(-float64(x))))
    x = np.array([-3.0, -0.5, 0.25, 2.0, 9.0], np.float32)
    want = np.array([xi * np.float32(1.0 / (1.0 + math.exp(-float(xi)))) for xi in x], np.float32)
    np.testing.assert_array_equal(oracle.silu(x), want)


# --- matrix_test.go --------------------------------------------------------------
def test_matmul_known_answers(oracle):
    # TestMatMul (matrix_test.go:15-60)
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    np.testing.assert_array_equal(oracle.matmul_nn(a, b), [[58, 64], [139, 154]])
    np.testing.assert_array_equal(oracle.matmul_nn(np.array([[1, 2, 3]], np.float32),
                                                   np.array([[4], [5], [6]], np.float32)), [[32]])


def test_dequant_matmul_is_dequantize_then_matmul(oracle):
    # nn/quantize.go:251-258: DequantizeMatmul(x, q, s) == x @ Dequantize(q, s)^T
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((24, 64)) * 0.02).astype(np.float32)
    x = rng.standard_normal((3, 64)).astype(np.float32)
    _, qi, s = oracle.quantize(w, 0)
    y = oracle.dequant_matmul(x, qi, s, 0)
    deq = oracle.dequantize(qi, s, 0)
    np.testing.assert_array_equal(y, oracle.matmul_nt(x, deq))
    # sequential fp32 order: identical to a plain Python left-to-right sum
    for m, n in ((0, 0), (2, 23)):
        acc = np.float32(0)
        for k in range(64):
            acc = np.float32(acc + np.float32(x[m, k] * deq[n, k]))
        assert acc == y[m, n]


def test_rmsnorm_formula(oracle):
    # cpu/backend.go:606-652
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 16)).astype(np.float32)
    w = rng.standard_normal(16).astype(np.float32)
    got = oracle.rmsnorm(x, w, 1e-5)
    for r in range(2):
        ss = np.float32(0)
        for v in x[r]:
            ss = np.float32(ss + np.float32(v * v))
        rms = np.float32(math.sqrt(float(np.float32(ss / np.float32(16)) + np.float32(1e-5))))
        np.testing.assert_array_equal(got[r], ((x[r] / rms).astype(np.float32) * w).astype(np.float32))


def test_argmax_first_index_on_ties(oracle):
    # models/sampling.go:73-83 (strict >)
    assert oracle.argmax(np.array([1, 3, 3, 2], np.float32)) == 1


def test_threads_do_not_change_results(oracle):
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((96, 128)) * 0.02).astype(np.float32)
    x = rng.standard_normal((5, 128)).astype(np.float32)
    _, qi, s = oracle.quantize(w, 0)
    n0 = oracle.get_threads()
    try:
        oracle.set_threads(1)
        y1 = oracle.dequant_matmul(x, qi, s, 0)
        oracle.set_threads(4)
        y4 = oracle.dequant_matmul(x, qi, s, 0)
    finally:
        oracle.set_threads(n0)
    np.testing.assert_array_equal(y1, y4)


SMALL = dict(vocab=512, dim=64, layers=2, heads=4, kv_heads=4, hidden=96, max_seq=64, rope_base=10000.0, eps=1e-5)
SMALL_GQA = dict(SMALL, heads=4, kv_heads=2)


@pytest.mark.parametrize("cfg", [SMALL, SMALL_GQA], ids=["mha", "gqa"])
def test_model_cache_matches_full_recompute(oracle, cfg):
    """Forward(prompt) then Forward(next) with the KV cache equals the last
    position of Forward(prompt + next) without a cache (quantized.go:282-302)."""
    m = oracle.Model(cfg, 1, seed=0)
    toks = np.array([[5, 17, 300, 2, 99, 41]], np.int64)
    _, _, _ = m.forward(toks[:, :5], want_logits=False)
    _, last_cached, _ = m.forward(toks[:, 5:], want_logits=False)
    m.reset()
    full, _, _ = m.forward(toks)
    np.testing.assert_allclose(last_cached[0], full[0, 5], rtol=0, atol=1e-6)


def test_model_batch_rows_are_independent(oracle):
    m2 = oracle.Model(SMALL, 2, seed=1)
    m1 = oracle.Model(SMALL, 1, seed=1)
    toks = np.array([[3, 4, 5, 6], [9, 8, 7, 6]], np.int64)
    _, l2, _ = m2.forward(toks, want_logits=False)
    _, l1, _ = m1.forward(toks[1:], want_logits=False)
    np.testing.assert_array_equal(l2[1], l1[0])


def test_model_rejects_bad_token(oracle):
    m = oracle.Model(SMALL, 1, seed=0)
    with pytest.raises(ValueError):
        m.forward(np.array([[1, SMALL["vocab"]]], np.int64))


def test_oracle_reproduces_golden_fixture(oracle):
    """The committed tiny-model stream (tests/golden/make_golden.py) still comes out of the oracle."""
    import json
    import os

    with open(os.path.join(os.path.dirname(__file__), "golden", "tiny_greedy.json")) as f:
        g = json.load(f)
    m = oracle.Model(g["config"], 1, seed=g["weight_seed"])
    prompt = oracle.synth_tokens(g["prompt_seed"], 128, g["config"]["vocab"])
    assert prompt.tolist() == g["prompt"]
    toks, _ = m.generate_greedy(prompt, 16)
    assert toks[0].tolist() == g["tokens"][:16]


# --- Sampler.Sample (models/sampling.go:47-70): the restatement on cases with
# hand-computed answers ------------------------------------------------------
def test_sampler_restatement_known_answers(oracle):
    import math

    s = oracle.sample
    assert s([0.0, 0.0], r=0.25) == 0 and s([0.0, 0.0], r=0.75) == 1
    # top-k keeps every value tied with the k-th largest (findKthLargest is by value)
    assert s([1.0, 3.0, 3.0, 2.0], top_k=1, r=0.6) == 2
    assert s([1.0, 3.0, 3.0, 2.0], top_k=1, r=0.4) == 1
    # top-p: probabilities 0.5, 0.3, 0.2; P = 0.7 keeps the first two (0.5 + 0.3 >= 0.7),
    # renormalised to 0.625 / 0.375
    lg = [math.log(0.5), math.log(0.3), math.log(0.2)]
    assert s(lg, top_p=0.7, r=0.6) == 0 and s(lg, top_p=0.7, r=0.7) == 1
    assert s(lg, top_p=0.7, r=0.99) == 1  # the masked token is never drawn
    # temperature 2 flattens [0, ln 4] to [0, ln 2]: probabilities 1/3, 2/3
    assert s([0.0, math.log(4.0)], temperature=2.0, r=0.3) == 0
    assert s([0.0, math.log(4.0)], temperature=2.0, r=0.34) == 1
    # r at the very top of [0, 1) still lands on a token
    assert s([5.0, 1.0, 0.0], r=0.9999999) == 2


def test_grouped_model_quantizes_the_same_draws_per_group(oracle):
    """QuantizeModel(m, groupSize): each Linear of the grouped oracle model is
    nn/quantize.go's per-group quantization of the same synthetic draw as the
    per-channel model (stream layer * 8 + matrix), and the projection uses the
    per-group dequantization."""
    m = oracle.Model(SMALL, 1, seed=3, group=32)
    for layer, mat in ((0, 0), (1, 3), (1, 6)):
        N, K = m.shape(mat)
        w = oracle.synth_normal(3, layer * 8 + mat, N * K, 0.02).reshape(N, K)
        _, q, s = oracle.quantize(w, 32)
        np.testing.assert_array_equal(m.q(layer, mat), q)
        np.testing.assert_array_equal(m.scale(layer, mat), s)
    toks = np.array([[3, 4, 5, 6]], np.int64)
    full, _, _ = m.forward(toks)
    assert np.all(np.isfinite(full))
    with pytest.raises(MemoryError):
        oracle.Model(SMALL, 1, seed=3, group=48)  # 64 is not a whole number of groups of 48


def test_reference_sampling_known_answers(oracle):
    """models/sampling_test.go: TestGreedy (:66-107), TestFindKthLargest
    (:185-223) through the top-k mask, TestSortIndicesByValue (:225-238)
    through the top-p cut, TestSampler_Sample_Deterministic (:240-262)."""
    rs = [i / 64.0 for i in range(64)] + [1.0 - 2.0 ** -24]
    # Greedy: first index of the maximum
    for logits, want in (([5.0, 2.0, 1.0, 0.5], 0), ([1.0, 2.0, 3.0, 10.0], 3), ([1.0, 5.0, 2.0], 1),
                         ([-1.0, -0.5, -2.0], 1), ([1.0], 0)):
        assert oracle.argmax(np.array(logits, np.float32)) == want
    # findKthLargest: k = 1 keeps 9.0 only, k = 3 keeps {4, 5, 9}, k >= len keeps every value
    vals = [3.0, 1.0, 4.0, 1.0, 5.0, 9.0]
    assert {oracle.sample(vals, top_k=1, r=r) for r in rs} == {5}
    assert {oracle.sample(vals, top_k=3, r=r) for r in rs} == {2, 4, 5}
    short = [3.0, 1.0, 4.0]
    assert [oracle.sample(short, top_k=10, r=r) for r in rs] == [oracle.sample(short, r=r) for r in rs]
    # sortIndicesByValue: descending order 1, 3, 4, 2, 0; a top-p cut after the
    # third keeps exactly indices {1, 3, 4}, after the first only {1}
    v = np.array([1.0, 5.0, 2.0, 4.0, 3.0], np.float32)
    p = np.exp(v - v.max()) / np.exp(v - v.max()).sum()
    order = [1, 3, 4, 2, 0]
    cut3 = float(p[order[:3]].sum()) - 1e-4
    assert {oracle.sample(v, top_p=cut3, r=r) for r in rs} == {1, 3, 4}
    assert {oracle.sample(v, top_p=1e-4, r=r) for r in rs} == {1}
    # temperature 0.001: always the largest logit
    assert {oracle.sample([1.0, 5.0, 2.0, 3.0], temperature=0.001, r=r) for r in rs} == {1}
