"""CPU tests: the synthetic generator against an independent pure-Python
restatement (bit-exact), and the C ABI library: it loads without a GPU,
exports every symbol include/tendo_b200.h declares, validates arguments
before touching the device, and honours host-side fault injection.
"""
import math
import os
import re
import struct
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
M64 = (1 << 64) - 1


def mix64(z):
    z = (z + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def key(seed, stream):
    return mix64(mix64(seed) ^ ((stream * 0xD1B54A32D192ED03) & M64))


def bits(k, c):
    return mix64((k + c * 0x9E3779B97F4A7C15) & M64)


def py_ln(u):
    b = struct.unpack("<Q", struct.pack("<d", u))[0]
    e = ((b >> 52) & 0x7FF) - 1023
    m = struct.unpack("<d", struct.pack("<Q", (b & 0x000FFFFFFFFFFFFF) | 0x3FF0000000000000))[0]
    if m > 1.4142135623730951:
        m *= 0.5
        e += 1
    s = (m - 1.0) / (m + 1.0)
    s2 = s * s
    p = 1.0 / 27.0
    for k in (25, 23, 21, 19, 17, 15, 13, 11, 9, 7, 5, 3):
        p = p * s2 + 1.0 / k
    p = p * s2 + 1.0
    return float(e) * 0.69314718055994530942 + (2.0 * s) * p


def py_sincos(a):
    a2 = a * a
    ps = 1.0 / 25852016738884976640000.0
    for f in (51090942171709440000.0, 121645100408832000.0, 355687428096000.0, 1307674368000.0, 6227020800.0,
              39916800.0, 362880.0, 5040.0, 120.0, 6.0):
        ps = 1.0 / f - ps * a2
    ps = 1.0 - ps * a2
    pc = 1.0 / 1124000727777607680000.0
    for f in (2432902008176640000.0, 6402373705728000.0, 20922789888000.0, 87178291200.0, 479001600.0, 3628800.0,
              40320.0, 720.0, 24.0, 2.0):
        pc = 1.0 / f - pc * a2
    pc = 1.0 - pc * a2
    return a * ps, pc


def py_normal(k, index):
    p = index >> 1
    b1, b2 = bits(k, 2 * p), bits(k, 2 * p + 1)
    u1 = float((b1 >> 11) + 1) * 1.1102230246251565e-16
    u2 = float(b2 >> 11) * 1.1102230246251565e-16
    r = math.sqrt(-2.0 * py_ln(u1))
    t4 = u2 * 4.0
    q = int(t4)
    a = (t4 - float(q)) * 1.5707963267948966
    sn, cs = py_sincos(a)
    c, s = [(cs, sn), (-sn, cs), (-cs, -sn), (sn, -cs)][q & 3]
    return r * (s if index & 1 else c)


def test_generator_matches_python_restatement(oracle):
    for seed, stream in ((0, 0), (42, oracle.STREAM_X), (7, 3 * 8 + 5)):
        n = 257
        got = oracle.synth_normal(seed, stream, n, 0.02, offset=1000)
        k = key(seed, stream)
        want = np.array([np.float32(py_normal(k, 1000 + i) * 0.02) for i in range(n)], np.float32)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_generator_transcendentals_are_accurate():
    for u in (1e-16, 0.001, 0.3, 0.70710678, 0.9999999):
        assert abs(py_ln(u) - math.log(u)) <= 4e-16 * max(1.0, abs(math.log(u)))
    for a in (0.0, 0.1, 0.785, 1.5707):
        s, c = py_sincos(a)
        assert abs(s - math.sin(a)) < 1e-15 and abs(c - math.cos(a)) < 1e-15


def test_generator_distribution(oracle):
    x = oracle.synth_normal(0, 1, 200000, 1.0).astype(np.float64)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1.0) < 0.01
    assert abs(float(((x > 1.0).mean())) - 0.1587) < 0.005


def test_tokens_match(oracle, tb):
    a = oracle.synth_tokens(1, 128, 32000)
    b = tb.synth_tokens(128, 32000, 1)
    np.testing.assert_array_equal(a, b)
    assert a.min() >= 0 and a.max() < 32000 and len(set(a.tolist())) > 100


# --- the C ABI -----------------------------------------------------------------
def _declared_symbols():
    hdr = open(os.path.join(ROOT, "include", "tendo_b200.h")).read()
    return sorted(set(re.findall(r"^TB_API [^(]*?\b(tb_\w+)\s*\(", hdr, re.M)))


def test_library_exports_every_declared_symbol(tb):
    syms = _declared_symbols()
    assert len(syms) >= 35
    for s in syms:
        assert hasattr(tb.lib, s), s
    bound = {n for n, _, _ in tb.SIGNATURES}
    assert set(syms) <= bound, set(syms) - bound


def test_error_strings(tb):
    assert tb.lib.tb_get_error_string(0) == b"success"
    assert tb.lib.tb_get_error_string(6) == b"injected failure"
    assert tb.lib.tb_version() >= 100


def test_argument_validation_needs_no_gpu(tb):
    L = tb.lib
    # K = 0, group not dividing K, negative sizes: rejected before any launch
    assert L.tb_quantize_i8_f32(None, None, None, 4, 0, 0, None) == tb.TB_ERROR_INVALID_ARGUMENT
    assert L.tb_quantize_i8_f32(None, None, None, 4, 10, 3, None) == tb.TB_ERROR_INVALID_ARGUMENT
    assert L.tb_dequant_matmul_i8f32(None, None, None, None, -1, 4, 4, 0, None) == tb.TB_ERROR_INVALID_ARGUMENT
    assert L.tb_dequant_matmul_i8f32(None, None, None, None, 1, 4, 12, 5, None) == tb.TB_ERROR_INVALID_ARGUMENT
    # the tensor-core paths' scratch: none for per-group or CUDA-core modes;
    # digit rows + row scales (+ split-tile partial sums for M <= 32)
    # otherwise; a short workspace is rejected before any launch
    assert L.tb_dequant_matmul_workspace_size(32, 4096, 4096, 0, tb.TB_GEMM_I8X3) >= 3 * 32 * 4096 + 32 * 4
    assert L.tb_dequant_matmul_workspace_size(1, 4096, 4000, 0, tb.TB_GEMM_I8X3) == 0  # K % 128: CUDA-core GEMV
    # per-group GEMM: the digit rows of the tensor-core path, unless a row has more than 128 groups
    assert L.tb_dequant_matmul_workspace_size(64, 4096, 4096, 128, tb.TB_GEMM_I8X3) == 3 * 64 * 4096 + 64 * 4
    assert L.tb_dequant_matmul_workspace_size(64, 4096, 32768, 128, tb.TB_GEMM_I8X3) == 0
    # per-group decode regime: the tensor-core GEMV adds fp32 partial-row slots
    assert L.tb_dequant_matmul_workspace_size(8, 4096, 4096, 128, tb.TB_GEMM_I8X3) > \
        L.tb_dequant_matmul_workspace_size(8, 4096, 4096, 0, tb.TB_GEMM_I8X3)
    assert L.tb_dequant_matmul_workspace_size(8, 4096, 4096, 64, tb.TB_GEMM_I8X3) == 0  # group 64: CUDA cores
    assert L.tb_dequant_matmul_workspace_size(64, 4096, 4096, 0, tb.TB_GEMM_SIMT) == 0
    assert L.tb_dequant_matmul_workspace_size(33, 4096, 4096, 0, tb.TB_GEMM_I8X3) == 3 * 33 * 4096 + 33 * 4
    assert L.tb_dequant_matmul_workspace_size(33, 4096, 4096, 0, tb.TB_GEMM_I8X2) == 2 * 33 * 4096 + 33 * 4
    fake = 4096  # never dereferenced: the size check comes first
    assert L.tb_dequant_matmul_i8f32_ws(fake, fake, fake, fake, 64, 64, 64, 0, tb.TB_GEMM_I8X3, None, 0,
                                        None) == tb.TB_ERROR_INVALID_ARGUMENT
    assert L.tb_dequant_matmul_i8f32_ws(fake, fake, fake, fake, 64, 64, 64, 0, 7, fake, 1 << 20,
                                        None) == tb.TB_ERROR_INVALID_ARGUMENT
    # empty problems are no-ops
    assert L.tb_dequant_matmul_i8f32(None, None, None, None, 0, 4, 16, 0, None) == 0
    assert L.tb_rmsnorm_f32(None, None, None, 0, 8, 1e-5, None) == 0
    # RoPE past MaxSeqLen (nn/rope.go:109-111)
    assert L.tb_rope_apply_f32(None, None, None, None, 1, 1, 4, 8, 10, 12, None) == tb.TB_ERROR_INVALID_ARGUMENT
    # attention needs Sk >= Sq and Sk <= max_seq
    assert L.tb_attention_f32(None, None, None, None, 1, 4, 4, 2, 1, 64, 16, 0.1, None, 0, None) == 1
    assert L.tb_attention_workspace_size(1, 32, 1, 128, 2048) > 0
    assert L.tb_attention_workspace_size(1, 32, 4, 128, 2048) == 0


def test_rope_tables_host_match_oracle(oracle, tb):
    c1, s1 = oracle.rope_tables(128, 64, 10000.0)
    c2, s2 = tb.Backend.RoPETables(128, 64, 10000.0)
    np.testing.assert_array_equal(c1, c2)
    np.testing.assert_array_equal(s1, s2)
    c1, s1 = oracle.rope_tables(128, 16, 500000.0)
    c2, s2 = tb.Backend.RoPETables(128, 16, 500000.0)
    np.testing.assert_array_equal(c1, c2)
    np.testing.assert_array_equal(s1, s2)


def test_fault_injection_returns_status():
    code = (
        "import tendo_b200 as tb\n"
        "r = tb.lib.tb_quantize_i8_f32(None, None, None, 4, 16, 0, None)\n"
        "r2 = tb.lib.tb_rmsnorm_f32(None, None, None, 1, 8, 1e-5, None)\n"
        "print(r, r2)\n")
    env = dict(os.environ, TENDO_B200_INJECT="tb_quantize_i8_f32", PYTHONPATH=ROOT)
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, cwd=ROOT)
    assert out.returncode == 0, out.stderr
    a, b = out.stdout.split()
    assert int(a) == 6  # TB_ERROR_INJECTED, before any device work
    assert int(b) == 1  # not injected: plain argument check (null pointers)


def test_errors_raise_typed_exception(tb):
    with pytest.raises(tb.TendoB200Error) as ei:
        tb.check(tb.TB_ERROR_INVALID_ARGUMENT)
    assert ei.value.code == 1 and "invalid argument" in str(ei.value)


def test_product_never_touches_the_oracle():
    """The library and its Python module import, link and call nothing under oracle/."""
    pkg = os.path.join(ROOT, "tendo_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                text = open(os.path.join(dirpath, f)).read()
                assert "pyoracle" not in text and "liboracle" not in text and "oracle/" not in text, f
