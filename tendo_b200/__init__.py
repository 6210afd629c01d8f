"""tendo_b200 — B200 (sm_100a) kernels for tendo's int8-quantized Llama path.

The product is the C ABI of ``libtendo_b200.so`` (include/tendo_b200.h).  This
module binds it with ctypes for Python callers and tests.  It mirrors the
tendo operator names of the path — ``DequantizeMatmul``, ``Quantize``,
``RMSNorm``, ``SiLU``, ``Add``, ``Embedding``, ``RoPE``, attention — and the
``QuantizedModel`` engine.  PyTorch is used only for device memory and
streams: every op runs a kernel of this library, and there is no CPU or
PyTorch fallback; a missing library raises at import time.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtendo_b200.so")

TB_SUCCESS = 0
TB_ERROR_INVALID_ARGUMENT = 1
TB_ERROR_CUDA = 2
TB_ERROR_NOT_SUPPORTED = 3
TB_ERROR_OUT_OF_MEMORY = 4
TB_ERROR_TIMEOUT = 5
TB_ERROR_INJECTED = 6

TB_GEMM_I8X3 = 0
TB_GEMM_I8X2 = 1
TB_GEMM_SIMT = 2

TB_MODEL_KV_BF16 = 1

TB_BINARY_ADD, TB_BINARY_SUB, TB_BINARY_MUL, TB_BINARY_DIV = 0, 1, 2, 3

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float
_st = ctypes.c_int

# (name, restype, argtypes) of every exported entry point of include/tendo_b200.h
SIGNATURES = [
    ("tb_get_error_string", ctypes.c_char_p, [_st]),
    ("tb_get_last_cuda_error_string", ctypes.c_char_p, []),
    ("tb_version", ctypes.c_int, []),
    ("tb_quantize_i8_f32", _st, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    ("tb_pack_q_f32_to_i8", _st, [_vp, _vp, _i64, _vp, _vp]),
    ("tb_dequantize_i8_f32", _st, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    ("tb_dequant_matmul_i8f32", _st, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    ("tb_dequant_matmul_i8f32_mode", _st, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _st, _vp]),
    ("tb_dequant_matmul_workspace_size", ctypes.c_size_t, [_i64, _i64, _i64, _i64, _st]),
    ("tb_dequant_matmul_i8f32_ws", _st, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _st, _vp, ctypes.c_size_t, _vp]),
    ("tb_matmul_nt_f32", _st, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    ("tb_rmsnorm_f32", _st, [_vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    ("tb_add_rmsnorm_f32", _st, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    ("tb_silu_f32", _st, [_vp, _vp, _i64, _vp]),
    ("tb_silu_mul_f32", _st, [_vp, _vp, _vp, _i64, _vp]),
    ("tb_add_f32", _st, [_vp, _vp, _vp, _i64, _vp]),
    ("tb_rope_tables_host", _st, [_vp, _vp, ctypes.c_int, ctypes.c_int, _f32]),
    ("tb_rope_apply_f32", _st, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    ("tb_kv_append_rope_f32", _st, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    ("tb_fill_f32", _st, [_vp, _f32, _i64, _vp]),
    ("tb_binary_f32", _st, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp]),
    ("tb_where_f32", _st, [_vp, _vp, _vp, _vp, ctypes.c_int, _vp, _vp, _vp, _vp, _vp]),
    ("tb_tril_f32", _st, [_vp, _vp, _i64, _i64, _i64, _vp]),
    ("tb_softmax_f32", _st, [_vp, _vp, ctypes.c_int, _vp, _vp, ctypes.c_int, _vp]),
    ("tb_matmul_f32", _st, [_vp, _vp, _vp, ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                            _vp]),
    ("tb_cat_f32", _st, [_vp, _vp, _vp, ctypes.c_int, _vp, _vp, _vp, _vp, ctypes.c_int, _vp]),
    ("tb_attention_workspace_size", ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64]),
    ("tb_attention_f32", _st,
     [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _vp, ctypes.c_size_t, _vp]),
    ("tb_attention_decode_noalloc_f32", _st, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _vp]),
    ("tb_embedding_f32", _st, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    ("tb_argmax_f32", _st, [_vp, _vp, _i64, _i64, _vp]),
    ("tb_synth_normal_f32", _st, [_vp, _i64, _i64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_double, _vp]),
    ("tb_synth_quantized_i8", _st,
     [_vp, _vp, _i64, _i64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_double, _vp]),
    ("tb_synth_tokens_host", _st, [_vp, _i64, _i64, ctypes.c_uint64]),
    ("tb_model_create", _st, [_vp, _vp, ctypes.c_int]),
    ("tb_model_create_tp", _st, [_vp, _vp, ctypes.c_int, _vp]),
    ("tb_model_create_ex", _st, [_vp, _vp, ctypes.c_int, _vp, ctypes.c_uint32]),
    ("tb_model_create_grouped", _st, [_vp, _vp, ctypes.c_int, _vp, ctypes.c_uint32, _i64]),
    ("tb_sample_f32", _st, [_vp, _vp, _vp, _i64, _i64, ctypes.c_float, _i64, ctypes.c_float, _vp]),
    ("tb_model_generate_sample", _st, [_vp, _vp, _i64, _i64, _i64, ctypes.c_float, _i64, ctypes.c_float,
                                       ctypes.c_uint64, _vp]),
    ("tb_comm_unique_id_bytes", ctypes.c_size_t, []),
    ("tb_comm_unique_id", _st, [_vp, ctypes.c_size_t]),
    ("tb_comm_create", _st, [_vp, _vp, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    ("tb_comm_destroy", _st, [_vp]),
    ("tb_allreduce_sum_f32", _st, [_vp, _vp, _i64, _vp]),
    ("tb_comm_peer_active", ctypes.c_int, [_vp]),
    ("tb_model_destroy", _st, [_vp]),
    ("tb_model_init_synthetic", _st, [_vp, ctypes.c_uint64]),
    ("tb_model_set_linear", _st, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp]),
    ("tb_model_set_tensor", _st, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("tb_model_get_linear", _st, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp]),
    ("tb_model_get_tensor", _st, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("tb_model_bench_kernel", _st, [_vp, ctypes.c_int, ctypes.c_int]),
    ("tb_model_time_kernel", _st, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("tb_model_reset", _st, [_vp]),
    ("tb_model_position", _i64, [_vp]),
    ("tb_model_forward", _st, [_vp, _vp, _i64, _i64, _vp, _vp]),
    ("tb_model_generate_greedy", _st, [_vp, _vp, _i64, _i64, _i64, _vp]),
    ("tb_model_decode", _st, [_vp, _vp, _i64]),
    ("tb_model_tokens", _st, [_vp, _vp, _i64]),
    ("tb_model_set_position", _st, [_vp, _i64]),
    ("tb_model_sync", _st, [_vp]),
    ("tb_model_stream", _vp, [_vp]),
    ("tb_model_launches_per_step", _i64, [_vp]),
    ("tb_model_phase_times", _st, [_vp, _vp, ctypes.c_int, _vp]),
    ("tb_model_unit_times", _st, [_vp, _vp, ctypes.c_int, _vp]),
    ("tb_model_last_logits", _st, [_vp, _vp]),
]


class TendoB200Error(RuntimeError):
    """Mirror of tendo's cuda.CUDAError{Code, Message} (cuda/types.go:7-15)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"tendo_b200: {message} (status {code})")
        self.code = code
        self.message = message


class ShapeError(ValueError):
    """Mirror of tendo.ShapeError (ops.go:232-248)."""


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m tendo_b200.build` (there is no fallback path)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(status: int) -> None:
    if status != TB_SUCCESS:
        msg = lib.tb_get_error_string(status).decode()
        if status == TB_ERROR_CUDA:
            detail = lib.tb_get_last_cuda_error_string().decode()
            if detail:
                msg = f"{msg}: {detail}"
        raise TendoB200Error(status, msg)


# ---------------------------------------------------------------------------
# torch plumbing
# ---------------------------------------------------------------------------
def _torch():
    import torch

    return torch


def _ptr(t) -> int:
    return t.data_ptr() if t is not None else None


def _stream(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _need_cuda_view(*ts):
    """CUDA fp32 tensors of any strides (the strided tensor ops)."""
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ShapeError("tendo_b200 ops take CUDA tensors (DeviceError in tendo terms)")
        if t is not None and t.dtype != _torch().float32:
            raise ShapeError("tendo_b200 tensor ops take float32 tensors")


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ShapeError("tendo_b200 ops take CUDA tensors (DeviceError in tendo terms)")
        if t is not None and not t.is_contiguous():
            raise ShapeError("tendo_b200 ops take contiguous tensors")


@dataclass
class QuantizedTensor:
    """nn.QuantizedTensor (nn/quantize.go:22-37) with int8 storage."""

    data: object  # torch.int8 [N, K]
    scale: object  # torch.float32 [N] or [N, K / group]
    shape: tuple
    group_size: int = 0


def _broadcast_shape(a, b, op):
    """tendo.BroadcastShapes: right-aligned, each pair equal or one of them 1."""
    a, b = tuple(a), tuple(b)
    n = max(len(a), len(b))
    a = (1,) * (n - len(a)) + a
    b = (1,) * (n - len(b)) + b
    out = []
    for x, y in zip(a, b):
        if x != y and x != 1 and y != 1:
            raise ShapeError(f"{op}: shapes {a} and {b} do not broadcast")
        out.append(max(x, y))
    return tuple(out)


def _bcast_strides(out_shape, shape, strides):
    """Element strides of a view of `shape` broadcast to `out_shape` (0 where broadcast)."""
    n = len(out_shape)
    shape, strides = tuple(shape), tuple(strides)
    pad = n - len(shape)
    res = []
    for d in range(n):
        if d < pad or shape[d - pad] == 1 and out_shape[d] != 1:
            res.append(0)
        else:
            res.append(strides[d - pad])
    return res


def _view_arrays(out_shape, t):
    """(shape, strides) ctypes arrays of tensor t viewed at out_shape."""
    n = len(out_shape)
    sh = (ctypes.c_int64 * n)(*out_shape)
    st = (ctypes.c_int64 * n)(*_bcast_strides(out_shape, t.shape, t.stride()))
    return sh, st


class Backend:
    """The ops of tendo's quantized Llama path on this library's kernels.

    Method names and argument meaning follow tendo's Backend interfaces
    (api.go:81-318, nn/quantize.go:251-258, models/llama/forward.go:13-27);
    each call returns a new tensor, as every tendo op does.
    """

    def __init__(self, device: int = 0):
        self.device = device

    # nn/quantize.go:42-187
    def Quantize(self, weight, group_size: int = 0) -> QuantizedTensor:
        torch = _torch()
        _need_cuda(weight)
        if weight.dim() != 2:
            raise ShapeError(f"nn.Quantize: weight must be 2D, got {weight.dim()}D")
        N, K = weight.shape
        if group_size and K % group_size:
            raise ShapeError(f"nn.Quantize: in_features {K} not divisible by group_size {group_size}")
        q = torch.empty((N, K), dtype=torch.int8, device=weight.device)
        s = torch.empty((N, K // group_size) if group_size else (N,), dtype=torch.float32, device=weight.device)
        check(lib.tb_quantize_i8_f32(_ptr(q), _ptr(s), _ptr(weight), N, K, group_size, _stream()))
        return QuantizedTensor(q, s, (N, K), group_size)

    # nn/quantize.go:191-229
    def Dequantize(self, qt: QuantizedTensor):
        torch = _torch()
        N, K = qt.shape
        w = torch.empty((N, K), dtype=torch.float32, device=qt.data.device)
        check(lib.tb_dequantize_i8_f32(_ptr(w), _ptr(qt.data), _ptr(qt.scale), N, K, qt.group_size, _stream()))
        return w

    def PackQ(self, q_f32):
        """float32-coded q (nn/quantize.go:68) -> int8; raises on non-integer values."""
        torch = _torch()
        _need_cuda(q_f32)
        q = torch.empty(q_f32.shape, dtype=torch.int8, device=q_f32.device)
        bad = torch.zeros(1, dtype=torch.int32, device=q_f32.device)
        check(lib.tb_pack_q_f32_to_i8(_ptr(q), _ptr(q_f32), q_f32.numel(), _ptr(bad), _stream()))
        if int(bad.item()):
            raise ShapeError(f"{int(bad.item())} q values are not integers in [-128, 127]")
        return q

    # nn.QuantizedLinearBackend.DequantizeMatmul (nn/quantize.go:251-258; cuda/backend.go:676-721)
    def DequantizeMatmul(self, x, qweight, scale, group_size: int = 0, mode: int = TB_GEMM_I8X3):
        torch = _torch()
        _need_cuda(x, qweight, scale)
        K = x.shape[-1]
        N = qweight.shape[0]
        if qweight.dim() != 2 or qweight.shape[1] != K:
            raise ShapeError(f"dequantize matmul: x [..., {K}] vs qweight {tuple(qweight.shape)}")
        if qweight.dtype != torch.int8:
            qweight = self.PackQ(qweight.contiguous())
        M = x.numel() // K if K else 0
        out = torch.empty((*x.shape[:-1], N), dtype=torch.float32, device=x.device)
        # scratch of the tensor-core path from the caller's allocator (tendo's pool)
        ws_bytes = int(lib.tb_dequant_matmul_workspace_size(M, N, K, group_size, mode))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
        check(lib.tb_dequant_matmul_i8f32_ws(_ptr(out), _ptr(x), _ptr(qweight), _ptr(scale), M, N, K, group_size,
                                             mode, _ptr(ws) if ws is not None else None, ws_bytes, _stream()))
        return out

    # models.Sampler.Sample (models/sampling.go:47-70), one row per sequence
    def Sample(self, logits, uniforms, temperature: float = 1.0, top_k: int = 0, top_p: float = 0.0):
        torch = _torch()
        _need_cuda(logits, uniforms)
        B, V = logits.shape
        out = torch.empty(B, dtype=torch.int64, device=logits.device)
        check(lib.tb_sample_f32(_ptr(out), _ptr(logits), _ptr(uniforms), B, V, float(temperature), int(top_k),
                                float(top_p), _stream()))
        return out

    def MatMulNT(self, a, b):
        """a @ b^T in fp32 (the lm_head projection)."""
        torch = _torch()
        _need_cuda(a, b)
        M, K = a.shape
        N = b.shape[0]
        out = torch.empty((M, N), dtype=torch.float32, device=a.device)
        check(lib.tb_matmul_nt_f32(_ptr(out), _ptr(a), _ptr(b), M, N, K, _stream()))
        return out

    # NormOps.RMSNorm (api.go; cpu/backend.go:606-652)
    def RMSNorm(self, x, normalized_shape, weight, eps: float):
        torch = _torch()
        _need_cuda(x, weight)
        ns = 1
        for d in normalized_shape:
            ns *= d
        out = torch.empty_like(x)
        check(lib.tb_rmsnorm_f32(_ptr(out), _ptr(x), _ptr(weight), x.numel() // ns, ns, eps, _stream()))
        return out

    def AddRMSNorm(self, x, residual, weight, eps: float):
        """(residual + x, RMSNorm(residual + x) * weight) in one pass."""
        torch = _torch()
        _need_cuda(x, residual, weight)
        d = x.shape[-1]
        out = torch.empty_like(x)
        res = torch.empty_like(x)
        check(lib.tb_add_rmsnorm_f32(_ptr(out), _ptr(res), _ptr(x), _ptr(residual), _ptr(weight), x.numel() // d, d,
                                     eps, _stream()))
        return res, out

    def SiLU(self, x):
        torch = _torch()
        _need_cuda(x)
        out = torch.empty_like(x)
        check(lib.tb_silu_f32(_ptr(out), _ptr(x), x.numel(), _stream()))
        return out

    def SiLUMul(self, gate, up):
        torch = _torch()
        _need_cuda(gate, up)
        out = torch.empty_like(gate)
        check(lib.tb_silu_mul_f32(_ptr(out), _ptr(gate), _ptr(up), gate.numel(), _stream()))
        return out

    # ElementwiseOps with broadcasting (cpu/backend.go:257-271, :1511-1560)
    def Add(self, a, b):
        torch = _torch()
        _need_cuda_view(a, b)
        if a.shape == b.shape and a.is_contiguous() and b.is_contiguous():
            out = torch.empty_like(a)
            check(lib.tb_add_f32(_ptr(out), _ptr(a), _ptr(b), a.numel(), _stream()))
            return out
        return self._binary(TB_BINARY_ADD, a, b)

    def Sub(self, a, b):
        return self._binary(TB_BINARY_SUB, a, b)

    def Mul(self, a, b):
        return self._binary(TB_BINARY_MUL, a, b)

    def Div(self, a, b):
        return self._binary(TB_BINARY_DIV, a, b)

    def _binary(self, op, a, b):
        torch = _torch()
        _need_cuda_view(a, b)
        shape = _broadcast_shape(a.shape, b.shape, "binary op")
        out = torch.empty(shape, dtype=torch.float32, device=a.device)
        sh, sa = _view_arrays(shape, a)
        _, sb = _view_arrays(shape, b)
        check(lib.tb_binary_f32(_ptr(out), _ptr(a), _ptr(b), op, len(shape), sh, sa, sb, _stream()))
        return out

    # StorageBackend Full / Ones / Zeros (cpu/backend.go:60-86)
    def Full(self, value: float, *shape):
        torch = _torch()
        out = torch.empty(shape, dtype=torch.float32, device=f"cuda:{self.device}")
        check(lib.tb_fill_f32(_ptr(out), float(value), out.numel(), _stream()))
        return out

    def Ones(self, *shape):
        return self.Full(1.0, *shape)

    def Zeros(self, *shape):
        return self.Full(0.0, *shape)

    # Where (cpu/backend.go:1191-1255): cond > 0 ? x : y, broadcast over all three
    def Where(self, condition, x, y):
        torch = _torch()
        _need_cuda_view(condition, x, y)
        shape = _broadcast_shape(_broadcast_shape(condition.shape, x.shape, "where"), y.shape, "where")
        out = torch.empty(shape, dtype=torch.float32, device=x.device)
        sh, sc = _view_arrays(shape, condition)
        _, sx = _view_arrays(shape, x)
        _, sy = _view_arrays(shape, y)
        check(lib.tb_where_f32(_ptr(out), _ptr(condition), _ptr(x), _ptr(y), len(shape), sh, sc, sx, sy, _stream()))
        return out

    # Tril (cpu/backend.go:1257-1285): 2-D input
    def Tril(self, t, k: int = 0):
        torch = _torch()
        _need_cuda_view(t)
        if t.dim() != 2:
            raise ShapeError("tril: input must be 2D")
        src = t.contiguous()
        out = torch.empty_like(src)
        check(lib.tb_tril_f32(_ptr(out), _ptr(src), t.shape[0], t.shape[1], int(k), _stream()))
        return out

    # Softmax along dim (cpu/backend.go:1690-1744)
    def Softmax(self, t, dim: int = -1):
        torch = _torch()
        _need_cuda_view(t)
        out = torch.empty(t.shape, dtype=torch.float32, device=t.device)
        sh, st = _view_arrays(tuple(t.shape), t)
        check(lib.tb_softmax_f32(_ptr(out), _ptr(t), t.dim(), sh, st, int(dim), _stream()))
        return out

    # MatrixOps.MatMul (cpu/backend.go:281-308): a [..., M, K] @ b [..., K, N], batch dims broadcast
    def MatMul(self, a, b):
        torch = _torch()
        _need_cuda_view(a, b)
        if a.dim() < 2 or b.dim() < 2:
            raise ShapeError("matmul: operands must be at least 2D")
        M, K = a.shape[-2], a.shape[-1]
        K2, N = b.shape[-2], b.shape[-1]
        if K != K2:
            raise ShapeError(f"matmul: inner dimensions {K} and {K2}")
        batch = _broadcast_shape(a.shape[:-2], b.shape[:-2], "matmul")
        out = torch.empty((*batch, M, N), dtype=torch.float32, device=a.device)
        nb = len(batch)
        bs = (ctypes.c_int64 * max(nb, 1))(*batch)
        sa = (ctypes.c_int64 * max(nb, 1))(*_bcast_strides(batch, a.shape[:-2], a.stride()[:-2]))
        sb = (ctypes.c_int64 * max(nb, 1))(*_bcast_strides(batch, b.shape[:-2], b.stride()[:-2]))
        check(lib.tb_matmul_f32(_ptr(out), _ptr(a), _ptr(b), nb, bs, sa, sb, M, N, K, a.stride(-2), a.stride(-1),
                                b.stride(-2), b.stride(-1), _stream()))
        return out

    # Cat along dim (cpu/backend.go:1343-1407)
    def Cat(self, tensors, dim: int):
        torch = _torch()
        out = tensors[0]
        for t in tensors[1:]:
            _need_cuda_view(out, t)
            if out.dim() != t.dim():
                raise ShapeError("cat: ranks differ")
            d = dim % out.dim()
            shape = list(out.shape)
            shape[d] += t.shape[d]
            res = torch.empty(shape, dtype=torch.float32, device=out.device)
            sa_shape, sa = _view_arrays(tuple(out.shape), out)
            sb_shape, sb = _view_arrays(tuple(t.shape), t)
            check(lib.tb_cat_f32(_ptr(res), _ptr(out), _ptr(t), out.dim(), sa_shape, sa, sb_shape, sb, d, _stream()))
            out = res
        return out

    # EmbeddingOps.Embedding (cpu/backend.go:1289-1339)
    def Embedding(self, weight, indices):
        torch = _torch()
        _need_cuda(weight, indices)
        V, d = weight.shape
        out = torch.empty((*indices.shape, d), dtype=torch.float32, device=weight.device)
        bad = torch.zeros(1, dtype=torch.int32, device=weight.device)
        check(lib.tb_embedding_f32(_ptr(out), _ptr(weight), _ptr(indices), indices.numel(), V, d, _ptr(bad),
                                   _stream()))
        if int(bad.item()):
            raise ShapeError(f"embedding: {int(bad.item())} ids outside [0, {V})")
        return out

    def ArgMax(self, x):
        torch = _torch()
        _need_cuda(x)
        n = x.shape[-1]
        out = torch.empty(x.shape[:-1], dtype=torch.int64, device=x.device)
        check(lib.tb_argmax_f32(_ptr(out), _ptr(x), x.numel() // n, n, _stream()))
        return out

    # nn.NewRoPE / RoPE.Apply (nn/rope.go:22-197)
    @staticmethod
    def RoPETables(dim: int, max_seq: int, base: float):
        import numpy as np

        c = np.empty((max_seq, dim // 2), np.float32)
        s = np.empty((max_seq, dim // 2), np.float32)
        check(lib.tb_rope_tables_host(c.ctypes.data, s.ctypes.data, dim, max_seq, base))
        return c, s

    def RoPEApply(self, x, cos_t, sin_t, pos_offset: int):
        """x [B, H, S, D] -> rotated copy at positions pos_offset.. (RoPE.Apply)."""
        torch = _torch()
        _need_cuda(x, cos_t, sin_t)
        B, H, S, D = x.shape
        out = torch.empty_like(x)
        check(lib.tb_rope_apply_f32(_ptr(out), _ptr(x), _ptr(cos_t), _ptr(sin_t), B, H, S, D, pos_offset,
                                    cos_t.shape[0], _stream()))
        return out

    def KVAppendRoPE(self, kcache, vcache, k, v, cos_t, sin_t, pos: int):
        """Cat([cache, new], 2) done in place: k, v [B, S, Hkv, D]; caches [B, Hkv, max_seq, D]."""
        _need_cuda(kcache, vcache, k, v, cos_t, sin_t)
        B, S, Hkv, D = k.shape
        check(lib.tb_kv_append_rope_f32(_ptr(kcache), _ptr(vcache), _ptr(k), _ptr(v), _ptr(cos_t), _ptr(sin_t), B,
                                        Hkv, S, D, pos, kcache.shape[2], _stream()))

    def Attention(self, q, kcache, vcache, sk: int, scale: float | None = None):
        """q [B, Sq, H, D] over the first sk cached positions -> [B, Sq, H, D]."""
        torch = _torch()
        _need_cuda(q, kcache, vcache)
        B, Sq, H, D = q.shape
        Hkv, max_seq = kcache.shape[1], kcache.shape[2]
        if scale is None:
            import math

            scale = float(ctypes.c_float(1.0 / ctypes.c_float(math.sqrt(D)).value).value)
        out = torch.empty_like(q)
        ws_bytes = lib.tb_attention_workspace_size(B, H, Sq, D, max_seq)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=q.device)
        check(lib.tb_attention_f32(_ptr(out), _ptr(q), _ptr(kcache), _ptr(vcache), B, H, Hkv, Sq, sk, D, max_seq,
                                   scale, _ptr(ws), ws_bytes, _stream()))
        return out

    # synthetic workload generator
    def SynthNormal(self, N: int, K: int, seed: int, stream_id: int, std: float):
        torch = _torch()
        w = torch.empty((N, K), dtype=torch.float32, device=f"cuda:{self.device}")
        check(lib.tb_synth_normal_f32(_ptr(w), N, K, seed, stream_id, std, _stream()))
        return w

    def SynthQuantized(self, N: int, K: int, seed: int, stream_id: int, std: float = 0.02):
        torch = _torch()
        q = torch.empty((N, K), dtype=torch.int8, device=f"cuda:{self.device}")
        s = torch.empty((N,), dtype=torch.float32, device=f"cuda:{self.device}")
        check(lib.tb_synth_quantized_i8(_ptr(q), _ptr(s), N, K, seed, stream_id, std, _stream()))
        return q, s


def synth_tokens(n: int, vocab: int, seed: int):
    """Uniform prompt ids in [0, vocab) of the (seed, prompt) stream (host only)."""
    import numpy as np

    ids = np.empty(n, np.int64)
    check(lib.tb_synth_tokens_host(ids.ctypes.data, n, vocab, seed))
    return ids


# Stream ids of the synthetic generator (include/tendo_synth.h).
STREAM_EMBED = 0x7FFF0001
STREAM_LMHEAD = 0x7FFF0002
STREAM_PROMPT = 0x7FFF0003
STREAM_X = 0x7FFF0004
STREAM_W = 0x7FFF0005
MATS_PER_LAYER = 8


class ModelConfig(ctypes.Structure):
    """tb_model_config: llama.Config (models/llama/config.go:5-21) plus the lockstep batch."""

    _fields_ = [
        ("vocab", ctypes.c_int32),
        ("dim", ctypes.c_int32),
        ("layers", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("max_seq", ctypes.c_int32),
        ("rope_base", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("max_batch", ctypes.c_int32),
    ]


class Comm:
    """A tensor-parallel communicator (tb_comm_*: peer memory, NCCL), one per rank.

    ``Comm.from_process_group(device)`` builds it over an initialised
    torch.distributed group: rank 0 makes the unique id and the group
    broadcasts it (any backend, gloo included)."""

    def __init__(self, uid: bytes, rank: int, nranks: int, device: int):
        self.rank, self.nranks, self.device = rank, nranks, device
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(uid, len(uid))
        check(lib.tb_comm_create(ctypes.byref(h), buf, len(uid), rank, nranks, device))
        self.h = h

    @staticmethod
    def unique_id() -> bytes:
        n = int(lib.tb_comm_unique_id_bytes())
        buf = ctypes.create_string_buffer(n)
        check(lib.tb_comm_unique_id(buf, n))
        return buf.raw

    @classmethod
    def from_process_group(cls, device: int):
        import torch.distributed as dist

        rank, world = dist.get_rank(), dist.get_world_size()
        obj = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return cls(obj[0], rank, world, device)

    @property
    def peer(self) -> bool:
        """True when allreduces run over peer memory (tb_comm_peer_active)."""
        return bool(lib.tb_comm_peer_active(self.h))

    def allreduce_sum(self, t, stream=None):
        """In-place fp32 sum over the ranks (tb_allreduce_sum_f32)."""
        check(lib.tb_allreduce_sum_f32(self.h, _ptr(t), t.numel(), _stream(stream)))

    def close(self):
        if getattr(self, "h", None):
            lib.tb_comm_destroy(self.h)
            self.h = None


class QuantizedModel:
    """QuantizedModel (models/llama/quantized.go) on one GPU, B sequences in
    lockstep; with ``comm``, this rank's tensor-parallel share of it.
    ``kv_bf16``: the KV cache in bf16 (TB_MODEL_KV_BF16), half the cache bytes,
    values rounded to nearest even as they are appended.  ``group``: every
    Linear quantized per group of that many input columns (QuantizeModel(m,
    groupSize)); scales [rows, K / group] in set_linear / get_linear."""

    def __init__(self, cfg: dict, batch: int = 1, device: int = 0, comm: "Comm | None" = None,
                 kv_bf16: bool = False, group: int = 0):
        self.cfg = dict(cfg)
        self.B = batch
        self.device = device
        self.comm = comm
        self.kv_bf16 = kv_bf16
        self.group = group
        c = ModelConfig(cfg["vocab"], cfg["dim"], cfg["layers"], cfg["heads"], cfg["kv_heads"], cfg["hidden"],
                        cfg["max_seq"], cfg["rope_base"], cfg["eps"], batch)
        h = ctypes.c_void_p()
        if group:
            check(lib.tb_model_create_grouped(ctypes.byref(h), ctypes.byref(c), device, comm.h if comm else None,
                                              TB_MODEL_KV_BF16 if kv_bf16 else 0, group))
        elif kv_bf16:
            check(lib.tb_model_create_ex(ctypes.byref(h), ctypes.byref(c), device, comm.h if comm else None,
                                         TB_MODEL_KV_BF16))
        elif comm is None:
            check(lib.tb_model_create(ctypes.byref(h), ctypes.byref(c), device))
        else:
            check(lib.tb_model_create_tp(ctypes.byref(h), ctypes.byref(c), device, comm.h))
        self.h = h
        # vocabulary rows of this rank's lm_head (all of them without tensor parallelism)
        self.V_local = cfg["vocab"] // (comm.nranks if comm else 1)

    def close(self):
        if getattr(self, "h", None):
            lib.tb_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_synthetic(self, seed: int = 0):
        check(lib.tb_model_init_synthetic(self.h, seed))

    def set_linear(self, layer: int, mat: int, q, scale):
        import numpy as np

        q = np.ascontiguousarray(q, dtype=np.int8)
        scale = np.ascontiguousarray(scale, dtype=np.float32)
        want = q.shape[0] * (q.shape[1] // self.group if self.group else 1)
        if q.ndim != 2 or scale.size != want:
            raise ShapeError(f"set_linear: scales of a {q.shape} Linear have {want} values, got {scale.size}")
        check(lib.tb_model_set_linear(self.h, layer, mat, q.ctypes.data, scale.ctypes.data))

    def get_linear(self, layer: int, mat: int, shape):
        import numpy as np

        q = np.empty(shape, np.int8)
        s = np.empty((shape[0], shape[1] // self.group) if self.group else shape[0], np.float32)
        check(lib.tb_model_get_linear(self.h, layer, mat, q.ctypes.data, s.ctypes.data))
        return q, s

    def set_tensor(self, which: int, layer: int, host):
        import numpy as np

        a = np.ascontiguousarray(host, dtype=np.float32)
        check(lib.tb_model_set_tensor(self.h, which, layer, a.ctypes.data))

    def get_tensor(self, which: int, layer: int, shape):
        import numpy as np

        a = np.empty(shape, np.float32)
        check(lib.tb_model_get_tensor(self.h, which, layer, a.ctypes.data))
        return a

    def bench_kernel(self, kind: int, layer: int):
        check(lib.tb_model_bench_kernel(self.h, kind, layer))

    def time_kernel(self, kind: int, reps: int = 3) -> float:
        """Average microseconds per launch of one decode-step kernel kind (graph-timed)."""
        us = ctypes.c_float()
        check(lib.tb_model_time_kernel(self.h, kind, reps, ctypes.byref(us)))
        return float(us.value)

    def last_logits(self):
        """Logits [B, V] of the last forward or decode step (ExtractLastLogits)."""
        import numpy as np

        out = np.empty((self.B, self.V_local), np.float32)
        check(lib.tb_model_last_logits(self.h, out.ctypes.data))
        return out

    def reset(self):
        check(lib.tb_model_reset(self.h))

    @property
    def position(self) -> int:
        return int(lib.tb_model_position(self.h))

    def set_position(self, pos: int):
        check(lib.tb_model_set_position(self.h, pos))

    def forward(self, tokens, want_logits: bool = True):
        """Forward of tokens [B, S] (host ints) at the current position: (last_logits [B, V], next [B])."""
        import numpy as np

        t = np.ascontiguousarray(tokens, dtype=np.int64).reshape(self.B, -1)
        logits = np.empty((self.B, self.cfg["vocab"]), np.float32) if want_logits else None
        nxt = np.empty(self.B, np.int64)
        check(lib.tb_model_forward(self.h, t.ctypes.data, self.B, t.shape[1],
                                   logits.ctypes.data if logits is not None else None, nxt.ctypes.data))
        return logits, nxt

    def generate_greedy(self, prompt, n_new: int):
        import numpy as np

        p = np.ascontiguousarray(prompt, dtype=np.int64).reshape(self.B, -1)
        out = np.empty((self.B, n_new), np.int64)
        check(lib.tb_model_generate_greedy(self.h, p.ctypes.data, self.B, p.shape[1], n_new, out.ctypes.data))
        return out

    def generate_sample(self, prompt, n_new: int, temperature: float = 1.0, top_k: int = 0, top_p: float = 0.0,
                        seed: int = 0):
        """Generate with the Sampler, drawn on the device (tb_model_generate_sample)."""
        import numpy as np

        p = np.ascontiguousarray(prompt, dtype=np.int64).reshape(self.B, -1)
        out = np.empty((self.B, n_new), np.int64)
        check(lib.tb_model_generate_sample(self.h, p.ctypes.data, self.B, p.shape[1], n_new, float(temperature),
                                           int(top_k), float(top_p), seed, out.ctypes.data))
        return out

    def decode(self, n_steps: int, start_tokens=None):
        import numpy as np

        st = None
        if start_tokens is not None:
            st = np.ascontiguousarray(start_tokens, dtype=np.int64).reshape(self.B)
        check(lib.tb_model_decode(self.h, st.ctypes.data if st is not None else None, n_steps))

    def tokens(self, count: int):
        import numpy as np

        out = np.empty((count, self.B), np.int64)
        check(lib.tb_model_tokens(self.h, out.ctypes.data, count))
        return out

    def sync(self):
        check(lib.tb_model_sync(self.h))

    @property
    def stream_handle(self) -> int:
        return lib.tb_model_stream(self.h) or 0

    def phase_times(self):
        """Microseconds between the phase stamps of the last persistent decode step."""
        import numpy as np

        buf = np.zeros(4096, np.float64)
        n = ctypes.c_int()
        st = lib.tb_model_phase_times(self.h, buf.ctypes.data, buf.size, ctypes.byref(n))
        if st == TB_ERROR_NOT_SUPPORTED:
            return None
        check(st)
        return buf[: n.value].copy()

    def unit_times(self):
        """Weight-stream units of CTA 0 in the last persistent decode step:
        array [units, 2] of (issued, landed) globaltimer nanoseconds."""
        import numpy as np

        buf = np.zeros(2 * 4096, np.uint64)
        n = ctypes.c_int()
        st = lib.tb_model_unit_times(self.h, buf.ctypes.data, buf.size, ctypes.byref(n))
        if st == TB_ERROR_NOT_SUPPORTED:
            return None
        check(st)
        return buf[: n.value].reshape(-1, 2).copy()

    @property
    def launches_per_step(self) -> int:
        return int(lib.tb_model_launches_per_step(self.h))


MAT_NAMES = ("q", "k", "v", "o", "gate", "up", "down")
