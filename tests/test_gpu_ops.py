"""Kernel parity on the GPU: every op of the path through the C ABI against
the oracle on the same seeded inputs.

Tolerances (stated per test): quantization bits and scales are bit-exact;
the fp32-accumulated GEMV and the fp32 GEMM tiles are within 1e-3 of the
oracle relative to max |Y| (the oracle sums sequentially, the kernels in
parallel trees); elementwise glue within a few ulps.
"""
import math

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3


def _t(a, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def be(tb, cuda):
    return tb.Backend(0)


# --- quantization: bit-exact ------------------------------------------------
@pytest.mark.parametrize("N,K,group", [(64, 256, 0), (37, 1408, 0), (16, 512, 128), (8, 96, 32), (3, 7, 0)])
def test_quantize_bit_exact(oracle, be, cuda, N, K, group):
    rng = np.random.default_rng(N * 1000 + K)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[0] = 0.0  # zero row -> scale 1 (nn/quantize_test.go:183-204)
    if N > 2:
        w[2, : min(K, 5)] = [0.5, -0.5, 1.5, -2.5, 127.0][: min(K, 5)]
    _, q_ref, s_ref = oracle.quantize(w, group)
    qt = be.Quantize(_t(w, cuda), group)
    np.testing.assert_array_equal(_np(qt.data), q_ref)
    np.testing.assert_array_equal(_np(qt.scale).view(np.uint32), s_ref.view(np.uint32))
    deq = be.Dequantize(qt)
    np.testing.assert_array_equal(_np(deq), oracle.dequantize(q_ref, s_ref, group))


def test_quantize_microbench_shape_bit_exact(oracle, be, cuda):
    # configs: W [11008, 4096] N(0, 0.02), seed 42 (rows re-derived on the host)
    w = be.SynthNormal(11008, 4096, 42, 0x7FFF0005, 0.02)
    qt = be.Quantize(w, 0)
    rows = [0, 1, 4095, 11007]
    w_host = np.stack([oracle.synth_normal(42, 0x7FFF0005, 4096, 0.02, offset=r * 4096) for r in rows])
    np.testing.assert_array_equal(_np(w)[rows], w_host)
    _, q_ref, s_ref = oracle.quantize(_np(w), 0)
    np.testing.assert_array_equal(_np(qt.data), q_ref)
    np.testing.assert_array_equal(_np(qt.scale), s_ref)


def test_pack_reference_float_coded_q(oracle, be, cuda):
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((8, 64)) * 0.02).astype(np.float32)
    qf, qi, _ = oracle.quantize(w, 0)
    np.testing.assert_array_equal(_np(be.PackQ(_t(qf, cuda))), qi)
    bad = qf.copy()
    bad[0, 0] = 0.5
    with pytest.raises(ValueError):
        be.PackQ(_t(bad, cuda))


def test_synth_quantized_matches_oracle_model_weights(oracle, be, cuda):
    cfg = dict(vocab=512, dim=64, layers=2, heads=4, kv_heads=2, hidden=96, max_seq=32, rope_base=1e4, eps=1e-5)
    m = oracle.Model(cfg, 1, seed=3)
    for layer in (0, 1):
        for mat in range(7):
            N, K = m.shape(mat)
            q, s = be.SynthQuantized(N, K, 3, layer * 8 + mat)
            np.testing.assert_array_equal(_np(q), m.q(layer, mat))
            np.testing.assert_array_equal(_np(s), m.scale(layer, mat))
    e = be.SynthNormal(512, 64, 3, 0x7FFF0001, 0.02)
    np.testing.assert_array_equal(_np(e), m.embed())


# --- DequantizeMatmul --------------------------------------------------------
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (1, 11008, 4096), (1, 4096, 11008), (2, 1408, 512),
                                   (3, 512, 1408), (8, 4096, 4096), (9, 640, 512), (32, 4096, 4096),
                                   (5, 33, 48), (1, 7, 100), (4, 1003, 4096), (5, 77, 128), (1, 8, 64),
                                   (5, 4096, 4096), (1, 32000, 4096), (1, 8192, 28672), (3, 2000, 11008),
                                   (6, 4096, 4096), (8, 11008, 4096), (10, 1003, 4096), (10, 22016, 4096),
                                   (7, 12288, 4096)])
def test_dequant_matmul_gemv(oracle, be, cuda, M, N, K):
    rng = np.random.default_rng(M * 7 + N + K)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    _, q, s = oracle.quantize(w, 0)
    want = oracle.dequant_matmul(x, q, s, 0)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(s, cuda), 0))
    assert rel_err(got, want) <= GEMV_TOL
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=1e-3 * np.abs(want).max())


@pytest.mark.parametrize("M", [1, 8, 32, 128])
@pytest.mark.parametrize("K", [4096, 11008])
def test_dequant_matmul_digit_split_bound_with_outliers(oracle, be, cuda, M, K):
    """The three-digit split of x on rows with outliers.  Each row of x is
    N(0, 1) with 0.1% of its entries at +-100x the median |x| (the last row
    instead has a single spike), so the row scale s = max|x| / 127 is set by
    the outliers and the ordinary entries keep only the digits' resolution
    (2^-15 s per element).  The product is bounded against a float64 product
    of the same int8 weights: |y - y_ref| <= 4 * 2^-15 * s * scale_n *
    sum_k |q_nk| per element (the digit rounding plus the fp32 conversion of
    the exact s32 sums), whatever path M takes (ring GEMV, tcgen05 GEMV or
    GEMM)."""
    N = 256
    rng = np.random.default_rng(M * 31 + K)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    med = float(np.median(np.abs(x)))
    for m in range(M):
        if m == M - 1:
            idx = rng.integers(0, K, size=1)
        else:
            idx = rng.choice(K, size=max(1, K // 1000), replace=False)
        x[m, idx] = (100.0 * med * rng.choice([-1.0, 1.0], size=idx.size)).astype(np.float32)
    _, q, scale = oracle.quantize(w, 0)
    q = np.asarray(q, dtype=np.int8)
    scale = np.asarray(scale, dtype=np.float32)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(scale, cuda), 0)).astype(np.float64)
    ref = (x.astype(np.float64) @ q.astype(np.float64).T) * scale.astype(np.float64)[None, :]
    s = np.abs(x).max(axis=1).astype(np.float64) / 127.0
    bound = 4.0 * 2.0 ** -15 * s[:, None] * (np.abs(q).astype(np.float64).sum(axis=1) * scale)[None, :]
    err = np.abs(got - ref)
    assert np.all(err <= bound), f"max err / bound = {(err / bound).max():.3f}"


@pytest.mark.parametrize("M,group", [(1, 128), (4, 64), (40, 128)])
def test_dequant_matmul_grouped(oracle, be, cuda, M, group):
    rng = np.random.default_rng(group + M)
    N, K = 256, 512
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    _, q, s = oracle.quantize(w, group)
    want = oracle.dequant_matmul(x, q, s, group)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(s, cuda), group))
    assert rel_err(got, want) <= GEMV_TOL


@pytest.mark.parametrize("M,N,K", [(128, 4096, 4096), (2048, 4096, 4096), (2048, 11008, 4096), (100, 300, 200)])
def test_dequant_matmul_gemm_rows(oracle, be, cuda, M, N, K):
    """Prefill regime: the full product on the GPU, checked on a sample of rows
    (rows are independent; the oracle finishes in seconds)."""
    rng = np.random.default_rng(M + N)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    _, q, s = oracle.quantize(w, 0)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(s, cuda), 0))
    rows = sorted(set([0, 1, M // 2, M - 1] + list(rng.integers(0, M, 4))))
    want = oracle.dequant_matmul(x[rows], q, s, 0)
    assert rel_err(got[rows], want) <= GEMV_TOL


def test_dequant_matmul_float_coded_weights(oracle, be, cuda):
    """The reference's float32-coded q (nn/quantize.go:68) is accepted as is."""
    rng = np.random.default_rng(9)
    w = (rng.standard_normal((64, 128)) * 0.02).astype(np.float32)
    x = rng.standard_normal((1, 128)).astype(np.float32)
    qf, q, s = oracle.quantize(w, 0)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(qf, cuda), _t(s, cuda), 0))
    assert rel_err(got, oracle.dequant_matmul(x, q, s, 0)) <= GEMV_TOL


@pytest.mark.parametrize("K", [512, 500])
def test_matmul_nt_fp32(oracle, be, cuda, K):
    """K % 32 == 0 with aligned rows takes the staged fp32 kernel, K = 500 the
    generic CUDA-core tiles."""
    rng = np.random.default_rng(4)
    a = rng.standard_normal((3, K)).astype(np.float32)
    b = (rng.standard_normal((1000, K)) * 0.02).astype(np.float32)
    assert rel_err(_np(be.MatMulNT(_t(a, cuda), _t(b, cuda))), oracle.matmul_nt(a, b)) <= 1e-5


def test_matmul_nt_fp32_paths_agree_bitwise(be, cuda):
    """The staged kernel and the generic tiles sum in the same order: an operand
    4 bytes off a 16-byte boundary takes the generic path, with the same bits."""
    import torch

    rng = np.random.default_rng(14)
    a = rng.standard_normal((5, 512)).astype(np.float32)
    b = (rng.standard_normal((777, 512)) * 0.02).astype(np.float32)
    fast = _np(be.MatMulNT(_t(a, cuda), _t(b, cuda)))
    flat = torch.empty(a.size + 1, dtype=torch.float32, device=cuda)
    a_off = flat[1:].view(5, 512)  # contiguous, base 4 bytes past a 16-byte boundary
    a_off.copy_(_t(a, cuda))
    assert a_off.data_ptr() % 16 != 0
    slow = _np(be.MatMulNT(a_off, _t(b, cuda)))
    np.testing.assert_array_equal(fast, slow)


# --- glue ops -------------------------------------------------------------------
def test_rmsnorm(oracle, be, cuda):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((5, 4096)).astype(np.float32)
    w = rng.standard_normal(4096).astype(np.float32)
    got = _np(be.RMSNorm(_t(x, cuda), [4096], _t(w, cuda), 1e-6))
    np.testing.assert_allclose(got, oracle.rmsnorm(x, w, 1e-6), rtol=2e-6, atol=1e-6)
    r = rng.standard_normal((5, 4096)).astype(np.float32)
    res, out = be.AddRMSNorm(_t(x, cuda), _t(r, cuda), _t(w, cuda), 1e-6)
    np.testing.assert_array_equal(_np(res), x + r)
    np.testing.assert_allclose(_np(out), oracle.rmsnorm(x + r, w, 1e-6), rtol=2e-6, atol=1e-6)


def test_silu_and_swiglu(oracle, be, cuda):
    rng = np.random.default_rng(6)
    g = (rng.standard_normal(10000) * 3).astype(np.float32)
    u = rng.standard_normal(10000).astype(np.float32)
    np.testing.assert_allclose(_np(be.SiLU(_t(g, cuda))), oracle.silu(g), rtol=1e-6, atol=1e-7)
    assert float(_np(be.SiLU(_t(np.zeros(1, np.float32), cuda)))[0]) == 0.0  # activation_test.go:315-333
    np.testing.assert_allclose(_np(be.SiLUMul(_t(g, cuda), _t(u, cuda))), oracle.silu(g) * u, rtol=1e-6, atol=1e-7)
    np.testing.assert_array_equal(_np(be.Add(_t(g, cuda), _t(u, cuda))), g + u)


def test_embedding_and_argmax(oracle, be, cuda):
    rng = np.random.default_rng(8)
    table = rng.standard_normal((1000, 64)).astype(np.float32)
    ids = np.array([[0, 999, 5, 5]], np.int64)
    np.testing.assert_array_equal(_np(be.Embedding(_t(table, cuda), _t(ids, cuda))), table[ids])
    with pytest.raises(ValueError):
        be.Embedding(_t(table, cuda), _t(np.array([1000], np.int64), cuda))
    v = rng.standard_normal((3, 32000)).astype(np.float32)
    v[1, 17] = v[1, 31000] = 50.0  # tie: first index wins (models/sampling.go:73-83)
    got = _np(be.ArgMax(_t(v, cuda)))
    assert got.tolist() == [oracle.argmax(v[0]), 17, oracle.argmax(v[2])]


def test_rope_apply(oracle, be, cuda):
    rng = np.random.default_rng(10)
    x = rng.standard_normal((2, 4, 5, 128)).astype(np.float32)
    c, s = oracle.rope_tables(128, 64, 10000.0)
    got = _np(be.RoPEApply(_t(x, cuda), _t(c, cuda), _t(s, cuda), 7))
    np.testing.assert_array_equal(got, oracle.rope_apply(x, c, s, 7))


def test_kv_append_rope(oracle, be, cuda):
    import torch

    rng = np.random.default_rng(12)
    B, S, Hkv, D, Ms, pos = 2, 3, 4, 64, 16, 5
    k = rng.standard_normal((B, S, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((B, S, Hkv, D)).astype(np.float32)
    c, s = oracle.rope_tables(D, Ms, 10000.0)
    kc = torch.zeros((B, Hkv, Ms, D), device=cuda)
    vc = torch.zeros((B, Hkv, Ms, D), device=cuda)
    be.KVAppendRoPE(kc, vc, _t(k, cuda), _t(v, cuda), _t(c, cuda), _t(s, cuda), pos)
    kr = oracle.rope_apply(k.transpose(0, 2, 1, 3), c, s, pos)  # [B, Hkv, S, D]
    np.testing.assert_array_equal(_np(kc)[:, :, pos:pos + S], kr)
    np.testing.assert_array_equal(_np(vc)[:, :, pos:pos + S], v.transpose(0, 2, 1, 3))
    assert float(_np(kc)[:, :, :pos].sum()) == 0 and float(_np(kc)[:, :, pos + S:].sum()) == 0


# --- attention ----------------------------------------------------------------------
def _attn_ref(oracle, q, kc, vc, sk):
    """models/llama/quantized.go:319-372 on the host: q [B, Sq, H, D]."""
    B, Sq, H, D = q.shape
    Hkv = kc.shape[1]
    scale = np.float32(1.0) / np.float32(math.sqrt(D))
    out = np.zeros_like(q)
    for b in range(B):
        for h in range(H):
            kh = h // (H // Hkv)
            K = kc[b, kh, :sk]
            V = vc[b, kh, :sk]
            sc = oracle.matmul_nt(q[b, :, h], K) * scale
            for i in range(Sq):
                sc[i, i + (sk - Sq) + 1:] = -np.inf
            p = oracle.softmax(sc)
            out[b, :, h] = oracle.matmul_nn(p, V)
    return out


@pytest.mark.parametrize("B,H,Hkv,D,Sq,sk", [(1, 32, 32, 128, 1, 513), (2, 8, 8, 64, 1, 129), (1, 64, 8, 128, 1, 700),
                                            (3, 4, 2, 128, 1, 1), (1, 8, 8, 64, 128, 128), (2, 4, 4, 128, 37, 90),
                                            (1, 8, 2, 128, 64, 64)])
def test_attention(oracle, be, cuda, B, H, Hkv, D, Sq, sk):
    rng = np.random.default_rng(B * 100 + H + Sq + sk)
    Ms = max(sk, 16) + 8
    q = rng.standard_normal((B, Sq, H, D)).astype(np.float32)
    kc = rng.standard_normal((B, Hkv, Ms, D)).astype(np.float32)
    vc = rng.standard_normal((B, Hkv, Ms, D)).astype(np.float32)
    got = _np(be.Attention(_t(q, cuda), _t(kc, cuda), _t(vc, cuda), sk))
    want = _attn_ref(oracle, q, kc, vc, sk)
    assert rel_err(got, want) <= 1e-4


# --- Sampler.Sample on the device (models/sampling.go:47-70) ----------------
@pytest.mark.parametrize("V,T,K,P", [(32000, 1.0, 0, 0.0), (32000, 0.7, 50, 0.0), (32000, 1.3, 40, 0.9),
                                     (4000, 1.0, 0, 0.9), (32000, 1.0, 1, 0.0), (1000, 0.5, 999, 0.95),
                                     (32000, 1.0, 0, 0.9), (32000, 0.8, 0, 0.5), (32000, 1.0, 0, 0.999),
                                     (32000, 1.0, 20000, 0.97), (40000, 2.0, 0, 0.9)])
def test_sample_matches_oracle(oracle, be, cuda, V, T, K, P):
    rng = np.random.default_rng(V + K)
    B = 6
    logits = (rng.standard_normal((B, V)) * 3).astype(np.float32)
    logits[1, :10] = logits[1].max() + 1.0  # ties at the top
    r = np.array([0.0, 0.5, 0.999999, 0.25, 0.75, 0.1], np.float32)
    got = _np(be.Sample(_t(logits, cuda), _t(r, cuda), T, K, P))
    want = [oracle.sample(logits[b], T, K, P, float(r[b])) for b in range(B)]
    np.testing.assert_array_equal(got, np.array(want))


@pytest.mark.parametrize("P", [0.9, 0.3])
def test_sample_top_p_over_a_flat_vocab(oracle, be, cuda, P):
    """Every probability equal: the cutoff lies thousands of candidates deep,
    across several sorted batches, and the ties keep index order."""
    V = 32000
    logits = np.zeros((3, V), np.float32)
    logits[1, 5:9] = 1e-3  # a few slightly larger values ahead of the ties
    logits[2, ::2] = -50.0  # half the vocabulary with probabilities near zero
    r = np.array([0.5, 0.999, 0.01], np.float32)
    got = _np(be.Sample(_t(logits, cuda), _t(r, cuda), 1.0, 0, P))
    want = [oracle.sample(logits[b], 1.0, 0, P, float(r[b])) for b in range(3)]
    np.testing.assert_array_equal(got, np.array(want))
