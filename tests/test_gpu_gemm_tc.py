"""Prefill-regime quantized Linear (M > 32) on the tcgen05 tensor cores,
against the oracle's dequantize-then-matmul (nn/quantize.go:251-258 with the
sequential fp32 sum of cpu/backend.go:1976-2021).

The GEMM splits each activation row into int8 digit rows and sums every
digit row times the raw int8 weights exactly, so its only approximation is
the digit truncation.  Tolerances, relative to max |Y|: three digit rows
(TB_GEMM_I8X3, the default) 1e-4; two digit rows (TB_GEMM_I8X2) 1e-3.  The
oracle's own fp32 summation error is of order 1e-6 at these K.
"""
import ctypes

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = {0: 1e-4, 1: 1e-3}


def _t(a, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def be(tb, cuda):
    return tb.Backend(0)


def _case(oracle, M, N, K, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    _, q, s = oracle.quantize(w, 0)
    return rng, x, q, s


# (M, N, K): M tails (33, 129, 300 rows of 128-row tiles), N tails (300: not a
# multiple of 4 -> scalar epilogue; 1408 = 11 tiles), K tails (1040: a 16-byte
# remainder block read past the end as zeros), the 7B prefill shapes.
SHAPES = [(33, 128, 512), (129, 300, 1040), (300, 1408, 512), (512, 4096, 4096), (512, 4096, 11008),
          (512, 11008, 4096)]


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_tc_matches_oracle(oracle, tb, be, cuda, M, N, K, mode):
    rng, x, q, s = _case(oracle, M, N, K, M * 7 + N + K)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(s, cuda), 0, mode=mode))
    rows = sorted(set([0, M // 2, M - 1] + [int(r) for r in rng.integers(0, M, 5)]))
    want = oracle.dequant_matmul(x[rows], q, s, 0)
    assert rel_err(got[rows], want) <= TOL[mode]


def test_gemm_tc_library_scratch_matches_caller_scratch(oracle, tb, be, cuda):
    """tb_dequant_matmul_i8f32 (library-owned scratch) and the _ws entry point
    run the same kernels: identical bits."""
    import torch

    M, N, K = 200, 1024, 2048
    _, x, q, s = _case(oracle, M, N, K, 5)
    xd, qd, sd = _t(x, cuda), _t(q, cuda), _t(s, cuda)
    a = be.DequantizeMatmul(xd, qd, sd, 0)
    b = torch.empty((M, N), dtype=torch.float32, device=cuda)
    tb.check(tb.lib.tb_dequant_matmul_i8f32(b.data_ptr(), xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), M, N, K, 0,
                                            tb._stream()))
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_gemm_tc_zero_and_extreme_rows(oracle, be, cuda):
    """A zero activation row (scale 1, all digits 0) and rows with one huge
    element (the digit scale follows max |x|) stay within tolerance."""
    M, N, K = 64, 256, 1024
    rng, x, q, s = _case(oracle, M, N, K, 11)
    x[3] = 0.0
    x[7, 5] = 1e4
    x[9] *= 1e-20
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(s, cuda), 0))
    for r in (3, 7, 9, 10):
        want = oracle.dequant_matmul(x[r:r + 1], q, s, 0)
        if r == 3:
            assert np.all(got[r] == 0.0)
        else:
            assert rel_err(got[r:r + 1], want) <= TOL[0]


# per-group scales (nn/quantize.go:126-187) on the tensor-core GEMM, 128 x 64
# tiles with a hand-off per group: M and N tails, groups of one and several
# K blocks, the 7B prefill shapes (86 groups per row at K 11008).
GEMM_GROUP_SHAPES = [(33, 128, 512, 128), (129, 300, 1024, 256), (300, 1408, 512, 512), (512, 4096, 4096, 128),
                     (512, 11008, 4096, 128), (512, 4096, 11008, 128), (200, 4096, 4096, 4096)]


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("M,N,K,g", GEMM_GROUP_SHAPES)
def test_gemm_tc_per_group_matches_oracle(oracle, tb, be, cuda, M, N, K, g, mode):
    assert tb.lib.tb_dequant_matmul_workspace_size(M, N, K, g, mode) > 0  # the tensor-core path
    rng = np.random.default_rng(M + N + K + g)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[:, :g] *= 8.0
    x = rng.standard_normal((M, K)).astype(np.float32)
    _, q, s = oracle.quantize(w, g)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(s, cuda), g, mode=mode))
    rows = sorted(set([0, M // 2, M - 1] + [int(r) for r in rng.integers(0, M, 5)]))
    assert rel_err(got[rows], oracle.dequant_matmul(x[rows], q, s, g)) <= TOL[mode]


def test_gemm_per_group_below_128_takes_cuda_cores(oracle, tb, be, cuda):
    """Groups that are not a multiple of 128 bytes run the CUDA-core GEMM."""
    M, N, K, g = 64, 256, 512, 64
    assert tb.lib.tb_dequant_matmul_workspace_size(M, N, K, g, tb.TB_GEMM_I8X3) == 0
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    _, q, s = oracle.quantize(w, g)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(s, cuda), g))
    assert rel_err(got, oracle.dequant_matmul(x, q, s, g)) <= 1e-3


# --- decode regime (1 <= M <= 32): the stream-K tcgen05 GEMV -----------------
# (M, N, K): the microbench shapes, a down projection (K 11008), N tails (300:
# one partial 128-row tile; 128: a single tile spread over many CTAs) and
# several batch sizes.
GEMV_SHAPES = [(1, 4096, 4096), (1, 11008, 4096), (1, 4096, 11008), (3, 300, 1024), (5, 128, 4096),
               (8, 4096, 4096), (8, 11008, 4096), (17, 1408, 512), (32, 4096, 4096), (32, 11008, 4096)]



@pytest.mark.parametrize("M,N,K", GEMV_SHAPES)
def test_gemv_tc_matches_oracle(oracle, be, cuda, M, N, K):
    rng, x, q, s = _case(oracle, M, N, K, M * 131 + N + K)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(s, cuda), 0))
    want = oracle.dequant_matmul(x, q, s, 0)
    assert rel_err(got, want) <= TOL[0]


def test_gemv_tc_split_tiles_are_deterministic(oracle, be, cuda):
    """Tiles split over several CTAs are summed in integers: repeated calls
    give identical bits."""
    import torch

    M, N, K = 4, 4096, 11008
    _, x, q, s = _case(oracle, M, N, K, 9)
    xd, qd, sd = _t(x, cuda), _t(q, cuda), _t(s, cuda)
    a = be.DequantizeMatmul(xd, qd, sd, 0)
    for _ in range(3):
        assert torch.equal(a, be.DequantizeMatmul(xd, qd, sd, 0))


# per-group scales (nn/quantize.go:126-187) on the same GEMV: (M, N, K, group)
# with one group per 128-byte sub-tile (two per stage), groups spanning
# stages (512, 1024), a stage of one sub-tile (K 384: group 384 = three
# stages), N tails and a single tile spread over many CTAs (128 rows), the
# digit-kernel path (M 17, 32).
GEMV_GROUP_SHAPES = [(1, 4096, 4096, 128), (1, 11008, 4096, 128), (1, 4096, 11008, 128), (3, 300, 1024, 256),
                     (5, 128, 4096, 512), (8, 4096, 4096, 1024), (1, 4096, 384, 384), (17, 1408, 512, 128),
                     (32, 4096, 4096, 128), (2, 11008, 4096, 4096)]


def _group_case(oracle, M, N, K, g, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[:, :g] *= 8.0  # the first group's scales differ from the rest
    x = rng.standard_normal((M, K)).astype(np.float32)
    _, q, s = oracle.quantize(w, g)
    return x, q, s


@pytest.mark.parametrize("M,N,K,g", GEMV_GROUP_SHAPES)
def test_gemv_tc_per_group_matches_oracle(oracle, tb, be, cuda, M, N, K, g):
    assert tb.lib.tb_dequant_matmul_workspace_size(M, N, K, g, tb.TB_GEMM_I8X3) > 0  # the tensor-core path
    x, q, s = _group_case(oracle, M, N, K, g, M * 17 + N + K + g)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(s, cuda), g))
    want = oracle.dequant_matmul(x, q, s, g)
    assert rel_err(got, want) <= TOL[0]


def test_gemv_tc_per_group_is_deterministic_and_library_scratch_agrees(oracle, tb, be, cuda):
    """Split tiles add their fp32 partial rows in CTA order: repeated calls,
    and the library-scratch entry point, give identical bits."""
    import torch

    M, N, K, g = 4, 4096, 11008, 128
    x, q, s = _group_case(oracle, M, N, K, g, 21)
    xd, qd, sd = _t(x, cuda), _t(q, cuda), _t(s, cuda)
    a = be.DequantizeMatmul(xd, qd, sd, g)
    for _ in range(3):
        assert torch.equal(a, be.DequantizeMatmul(xd, qd, sd, g))
    b = torch.empty((M, N), dtype=torch.float32, device=cuda)
    tb.check(tb.lib.tb_dequant_matmul_i8f32(b.data_ptr(), xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), M, N, K, g,
                                            tb._stream()))
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_gemv_per_group_below_128_takes_cuda_cores(oracle, tb, be, cuda):
    """Groups that are not a multiple of 128 bytes run the CUDA-core GEMV."""
    M, N, K, g = 3, 512, 1024, 64
    assert tb.lib.tb_dequant_matmul_workspace_size(M, N, K, g, tb.TB_GEMM_I8X3) == 0
    x, q, s = _group_case(oracle, M, N, K, g, 5)
    got = _np(be.DequantizeMatmul(_t(x, cuda), _t(q, cuda), _t(s, cuda), g))
    assert rel_err(got, oracle.dequant_matmul(x, q, s, g)) <= 1e-4
