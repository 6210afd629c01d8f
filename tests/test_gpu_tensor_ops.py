"""The generic fp32 ops of llama.Backend (tb_fill/binary/where/tril/softmax/
matmul/cat_f32) against restatements of the reference CPU backend on the same
inputs, and the attention op sequence of unchanged models/llama
(models/llama/quantized.go:282-372 with forward.go:345-417) replayed through
them against the fused attention kernel.

Elementwise ops, Where, Tril and Cat are bit-exact.  MatMul sums separately
rounded products in k order, as the oracle's matmul does: bit-exact against
it.  Softmax rounds exp computed in double precision: within 1 ulp of the
restatement (the two libraries' double exp may differ in the last double bit).
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be(tb, cuda):
    return tb.Backend(0)


def _t(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def _np(t):
    return t.detach().cpu().numpy()


def softmax_ref(x, dim):
    """cpu/backend.go:1690-1744 restated: max from -MaxFloat32, exp in float64
    of the float32 difference, a sequential float32 sum, then division."""
    x = np.ascontiguousarray(np.moveaxis(np.asarray(x, np.float32), dim, -1))
    out = np.empty(x.shape, np.float32)
    flat_in = x.reshape(-1, x.shape[-1])
    flat_out = out.reshape(-1, x.shape[-1])
    for r in range(flat_in.shape[0]):
        row = flat_in[r]
        m = np.float32(-np.finfo(np.float32).max)
        for v in row:
            if v > m:
                m = v
        e = np.exp((row - m).astype(np.float64)).astype(np.float32)
        s = np.float32(0)
        for v in e:
            s = np.float32(s + v)
        flat_out[r] = e / s
    return np.moveaxis(out, -1, dim)


def test_fill_tril_where(be, cuda):
    import torch

    f = be.Full(2.5, 3, 4)
    assert _np(f).tolist() == [[2.5] * 4] * 3
    ones = be.Ones(5, 9)
    for k in (-2, 0, 4):
        np.testing.assert_array_equal(_np(be.Tril(ones, k)), np.tril(np.ones((5, 9), np.float32), k))
    rng = np.random.default_rng(0)
    cond = (rng.standard_normal((1, 1, 5, 9)) > 0).astype(np.float32)
    x = rng.standard_normal((2, 3, 5, 9)).astype(np.float32)
    y = be.Full(float("-inf"), 2, 3, 5, 9)
    got = _np(be.Where(_t(cond, cuda), _t(x, cuda), y))
    np.testing.assert_array_equal(got, np.where(cond > 0, x, -np.inf))
    del torch


@pytest.mark.parametrize("shape_a,shape_b", [((4, 7), (4, 7)), ((2, 3, 5, 9), (1,)), ((2, 1, 5, 9), (3, 1, 9)),
                                             ((6, 1), (1, 8))])
def test_binary_broadcast_bit_exact(be, cuda, shape_a, shape_b):
    rng = np.random.default_rng(len(shape_a) * 10 + len(shape_b))
    a = rng.standard_normal(shape_a).astype(np.float32)
    b = (rng.standard_normal(shape_b) + 3.0).astype(np.float32)
    ta, tbb = _t(a, cuda), _t(b, cuda)
    for name, fn in (("Add", np.add), ("Sub", np.subtract), ("Mul", np.multiply), ("Div", np.divide)):
        got = _np(getattr(be, name)(ta, tbb))
        np.testing.assert_array_equal(got, fn(a, b).astype(np.float32), err_msg=name)


def test_binary_on_strided_views(be, cuda):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((4, 6, 8)).astype(np.float32)
    b = rng.standard_normal((8, 6)).astype(np.float32)
    ta = _t(a, cuda).permute(2, 1, 0)  # [8, 6, 4], non-contiguous
    tbb = _t(b, cuda)[:, :, None]      # [8, 6, 1], broadcast last
    got = _np(be.Mul(ta, tbb))
    np.testing.assert_array_equal(got, a.transpose(2, 1, 0) * b[:, :, None])


@pytest.mark.parametrize("shape,dim", [((3, 17), -1), ((2, 4, 5, 300), -1), ((6, 33, 4), 1), ((1, 2, 1, 1), -1)])
def test_softmax_matches_reference_order(be, cuda, shape, dim):
    rng = np.random.default_rng(sum(shape))
    x = (rng.standard_normal(shape) * 4).astype(np.float32)
    if shape[-1] > 5:
        x[..., 3] = -np.inf  # masked entries as the causal mask leaves them
    got = _np(be.Softmax(_t(x, cuda), dim))
    want = softmax_ref(x, dim)
    ulp = np.spacing(np.abs(want).astype(np.float32))
    assert np.all(np.abs(got - want) <= ulp), float(np.abs(got - want).max())


def test_softmax_all_masked_row_matches_reference(be, cuda):
    # the reference divides 0 by a zero sum: NaN, as here
    x = np.full((2, 8), -np.inf, np.float32)
    got = _np(be.Softmax(_t(x, cuda), -1))
    with np.errstate(invalid="ignore"):
        np.testing.assert_array_equal(got, softmax_ref(x, -1))


@pytest.mark.parametrize("M,N,K,batch", [(1, 300, 64, (2, 4)), (5, 7, 33, (3,)), (64, 48, 128, ()), (1, 1, 1, (1,))])
def test_matmul_bit_exact_against_oracle(oracle, be, cuda, M, N, K, batch):
    rng = np.random.default_rng(M * 1000 + N + K)
    a = rng.standard_normal((*batch, M, K)).astype(np.float32)
    b = rng.standard_normal((*batch, K, N)).astype(np.float32)
    got = _np(be.MatMul(_t(a, cuda), _t(b, cuda)))
    want = np.empty_like(got)
    for idx in np.ndindex(*batch):
        want[idx] = oracle.matmul_nn(a[idx], b[idx])
    np.testing.assert_array_equal(got, want)


def test_matmul_transposed_and_broadcast_views(oracle, be, cuda):
    """Q.K^T on a transposed view of a cache and P.V with a broadcast batch
    dimension (the GQA expand), as the reference attention issues them."""
    rng = np.random.default_rng(11)
    q = rng.standard_normal((2, 2, 3, 4, 16)).astype(np.float32)  # [B, Hkv, G, Sq, D]
    k = rng.standard_normal((2, 2, 1, 29, 16)).astype(np.float32)  # [B, Hkv, 1, S, D]
    tq, tk = _t(q, cuda), _t(k, cuda)
    kT = tk.expand(2, 2, 3, 29, 16).transpose(-2, -1)
    got = _np(be.MatMul(tq, kT))
    want = np.empty((2, 2, 3, 4, 29), np.float32)
    for b_ in range(2):
        for h in range(2):
            for g in range(3):
                want[b_, h, g] = oracle.matmul_nt(q[b_, h, g], k[b_, h, 0])
    np.testing.assert_array_equal(got, want)


def test_cat_along_sequence(be, cuda):
    rng = np.random.default_rng(5)
    cache = rng.standard_normal((2, 4, 37, 16)).astype(np.float32)
    new = rng.standard_normal((2, 16, 4, 1)).astype(np.float32)  # a permuted view below
    tn = _t(new, cuda).permute(0, 2, 3, 1)  # [2, 4, 1, 16]
    got = _np(be.Cat([_t(cache, cuda), tn], 2))
    np.testing.assert_array_equal(got, np.concatenate([cache, new.transpose(0, 2, 3, 1)], 2))


@pytest.mark.parametrize("B,H,Hkv,D,P,Sq", [(2, 8, 2, 64, 37, 1), (1, 4, 4, 32, 20, 5), (3, 16, 2, 128, 100, 1)])
def test_reference_attention_sequence_through_the_ops(be, cuda, B, H, Hkv, D, P, Sq):
    """forwardQuantizedAttention after RoPE (quantized.go:282-372): Cat the new
    k / v onto the cache, repeatKVHeads (reshape + expand), Q.K^T on the
    transposed view, Mul by Full(scale), applyCausalMask (Ones, Tril with
    offset Sk - Sq, expand, Full(-inf), Where), Softmax(-1), P.V — every op on
    this library's kernels — against the fused decode/prefill kernel."""
    import torch

    G = H // Hkv
    rng = np.random.default_rng(B * 7 + H + P)
    q = _t(rng.standard_normal((B, H, Sq, D)).astype(np.float32), cuda)
    kcache = _t(rng.standard_normal((B, Hkv, P, D)).astype(np.float32), cuda)
    vcache = _t(rng.standard_normal((B, Hkv, P, D)).astype(np.float32), cuda)
    knew = _t(rng.standard_normal((B, Hkv, Sq, D)).astype(np.float32), cuda)
    vnew = _t(rng.standard_normal((B, Hkv, Sq, D)).astype(np.float32), cuda)
    k = be.Cat([kcache, knew], 2)
    v = be.Cat([vcache, vnew], 2)
    Sk = P + Sq
    # repeatKVHeads: [B, Hkv, S, D] -> [B, Hkv, 1, S, D] -> expand G; the query heads split alike
    kx = k.reshape(B, Hkv, 1, Sk, D).expand(B, Hkv, G, Sk, D)
    vx = v.reshape(B, Hkv, 1, Sk, D).expand(B, Hkv, G, Sk, D)
    q5 = q.reshape(B, Hkv, G, Sq, D)
    scores = be.MatMul(q5, kx.transpose(-2, -1))
    scale = float(np.float32(1.0) / np.float32(math.sqrt(D)))
    scaled = be.Mul(scores, be.Full(scale, 1))
    mask2 = be.Tril(be.Ones(Sq, Sk), Sk - Sq)
    mask = mask2.reshape(1, 1, 1, Sq, Sk).expand(B, Hkv, G, Sq, Sk)
    masked = be.Where(mask, scaled, be.Full(float("-inf"), B, Hkv, G, Sq, Sk))
    attn = be.Softmax(masked, -1)
    out = be.MatMul(attn, vx).reshape(B, H, Sq, D)
    # the fused kernel over a cache holding the same rows
    max_seq = Sk + 3
    kc = torch.zeros((B, Hkv, max_seq, D), dtype=torch.float32, device=cuda)
    vc = torch.zeros_like(kc)
    kc[:, :, :Sk] = k
    vc[:, :, :Sk] = v
    fused = be.Attention(q.permute(0, 2, 1, 3).contiguous(), kc, vc, Sk, scale).permute(0, 2, 1, 3)
    got, want = _np(out), _np(fused)
    assert float(np.abs(got - want).max()) <= 1e-4 * float(np.abs(want).max())
