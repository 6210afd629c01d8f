"""Pre-quantized int8 Llama checkpoints in the safetensors format.

tendo's loader reads F32 / F16 / BF16 tensors only (safetensors.go:152-175)
and quantizes every Linear on the host at start-up (nn/quantize.go:42-124).
This module adds the int8 form the quantized path consumes directly: per
Linear an ``I8`` tensor ``<name>.weight`` [N, K] holding the quantized values
and an ``F32`` tensor ``<name>.weight_scale`` [N] (per channel) or
[N, K / group] (per group), under the Hugging Face Llama names tendo already
uses (models/llama/model.go:90-208); embedding, norms and lm_head stay F32.

The file layout is safetensors': an 8-byte little-endian header length, a
JSON header {name: {"dtype", "shape", "data_offsets": [begin, end]}} padded
with spaces to a multiple of 8 bytes, then the raw little-endian data.  Reads
are memory-mapped, so a 70B checkpoint streams to the GPU without a host copy
of the whole file.  A tensor-parallel model loads its shard: rows of the
column-parallel matrices, input columns (and all scales) of the row-parallel
ones.
"""
from __future__ import annotations

import json
import struct

import numpy as np

# safetensors dtype names <-> numpy
_DTYPES = {"I8": np.int8, "U8": np.uint8, "I32": np.int32, "I64": np.int64, "F16": np.float16, "F32": np.float32,
           "F64": np.float64}
_NAMES = {np.dtype(v).str: k for k, v in _DTYPES.items()}

# engine matrix index -> (Hugging Face module name, column-parallel?)
LINEARS = [("self_attn.q_proj", True), ("self_attn.k_proj", True), ("self_attn.v_proj", True),
           ("self_attn.o_proj", False), ("mlp.gate_proj", True), ("mlp.up_proj", True), ("mlp.down_proj", False)]


class CheckpointError(ValueError):
    """A malformed or incompatible checkpoint."""


def write(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Writes `tensors` (name -> numpy array) as one safetensors file."""
    header = {}
    offset = 0
    arrays = []
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr)
        key = a.dtype.str if a.dtype.str in _NAMES else np.dtype(a.dtype).newbyteorder("<").str
        if key not in _NAMES:
            raise CheckpointError(f"{name}: dtype {a.dtype} has no safetensors name")
        header[name] = {"dtype": _NAMES[key], "shape": list(a.shape), "data_offsets": [offset, offset + a.nbytes]}
        offset += a.nbytes
        arrays.append(a)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * (-len(raw) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for a in arrays:
            f.write(a.tobytes())


class SafeTensors:
    """A memory-mapped safetensors file: ``names()``, ``info(name)``, ``get(name)``."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            head = f.read(8)
            if len(head) != 8:
                raise CheckpointError(f"{path}: shorter than the header length field")
            (n,) = struct.unpack("<Q", head)
            raw = f.read(n)
            if len(raw) != n:
                raise CheckpointError(f"{path}: header of {n} bytes is cut short")
            f.seek(0, 2)
            size = f.tell()
        try:
            header = json.loads(raw.decode())
        except ValueError as e:
            raise CheckpointError(f"{path}: header is not JSON: {e}") from None
        self.metadata = header.pop("__metadata__", {})
        self._base = 8 + n
        self._info = {}
        for name, h in header.items():
            dt = h.get("dtype")
            if dt not in _DTYPES:
                raise CheckpointError(f"{name}: unsupported dtype {dt}")
            shape = tuple(int(x) for x in h.get("shape", ()))
            b, e = (int(x) for x in h.get("data_offsets", (0, -1)))
            want = int(np.prod(shape, dtype=np.int64)) * np.dtype(_DTYPES[dt]).itemsize
            if e - b != want or b < 0 or self._base + e > size:
                raise CheckpointError(f"{name}: data_offsets {b}..{e} do not hold {shape} {dt}")
            self._info[name] = (dt, shape, b)
        self._mm = np.memmap(path, dtype=np.uint8, mode="r") if size > self._base else None

    def names(self):
        return list(self._info)

    def info(self, name: str):
        dt, shape, _ = self._info[name]
        return dt, shape

    def get(self, name: str) -> np.ndarray:
        if name not in self._info:
            raise CheckpointError(f"missing tensor {name}")
        dt, shape, b = self._info[name]
        n = int(np.prod(shape, dtype=np.int64)) * np.dtype(_DTYPES[dt]).itemsize
        return self._mm[self._base + b:self._base + b + n].view(_DTYPES[dt]).reshape(shape)


def _linear_name(layer: int, mat: int) -> str:
    return f"model.layers.{layer}.{LINEARS[mat][0]}"


def _shapes(cfg: dict):
    d, H, Hkv, F = cfg["dim"], cfg["heads"], cfg["kv_heads"], cfg["hidden"]
    D = d // H
    return [(H * D, d), (Hkv * D, d), (Hkv * D, d), (d, H * D), (F, d), (F, d), (d, F)]


def export_model(qm, path: str) -> None:
    """Writes the weights of a one-GPU QuantizedModel as a pre-quantized checkpoint."""
    if getattr(qm, "comm", None) is not None:
        raise CheckpointError("export from an unsharded model")
    cfg = qm.cfg
    tensors = {}
    shapes = _shapes(cfg)
    for layer in range(cfg["layers"]):
        for mat in range(7):
            q, s = qm.get_linear(layer, mat, shapes[mat])
            tensors[_linear_name(layer, mat) + ".weight"] = q
            tensors[_linear_name(layer, mat) + ".weight_scale"] = s
        tensors[f"model.layers.{layer}.input_layernorm.weight"] = qm.get_tensor(3, layer, (cfg["dim"],))
        tensors[f"model.layers.{layer}.post_attention_layernorm.weight"] = qm.get_tensor(4, layer, (cfg["dim"],))
    tensors["model.embed_tokens.weight"] = qm.get_tensor(0, 0, (cfg["vocab"], cfg["dim"]))
    tensors["model.norm.weight"] = qm.get_tensor(2, 0, (cfg["dim"],))
    tensors["lm_head.weight"] = qm.get_tensor(1, 0, (cfg["vocab"], cfg["dim"]))
    meta = {k: cfg[k] for k in ("vocab", "dim", "layers", "heads", "kv_heads", "hidden")}
    g = getattr(qm, "group", 0)
    meta["format"] = f"tendo-int8-per-group-{g}" if g else "tendo-int8-per-channel"
    write(path, tensors, meta)


def load_model(qm, path: str) -> None:
    """Uploads a pre-quantized checkpoint into a QuantizedModel (its shard,
    for a tensor-parallel one).  Shapes, dtypes and the scales (per channel,
    or per group for a model made with ``group``) are checked against the
    model's configuration."""
    st = SafeTensors(path)
    cfg = qm.cfg
    comm = getattr(qm, "comm", None)
    r, n = (comm.rank, comm.nranks) if comm is not None else (0, 1)
    shapes = _shapes(cfg)

    def need(name, dtype, shape):
        dt, sh = st.info(name) if name in st._info else (None, None)
        if dt is None:
            raise CheckpointError(f"missing tensor {name}")
        if dt != dtype or tuple(sh) != tuple(shape):
            raise CheckpointError(f"{name}: {dt} {tuple(sh)}, expected {dtype} {tuple(shape)}")
        return st.get(name)

    for layer in range(cfg["layers"]):
        for mat in range(7):
            N, K = shapes[mat]
            base = _linear_name(layer, mat)
            g = getattr(qm, "group", 0)
            q = need(base + ".weight", "I8", (N, K))
            s = need(base + ".weight_scale", "F32", (N, K // g) if g else (N,))
            if LINEARS[mat][1]:  # column-parallel: this rank's output rows
                rows = slice(r * N // n, (r + 1) * N // n)
                qm.set_linear(layer, mat, q[rows], s[rows])
            elif g:  # row-parallel, per group: this rank's input columns and their groups
                cols = slice(r * K // n, (r + 1) * K // n)
                groups = slice(r * (K // g) // n, (r + 1) * (K // g) // n)
                qm.set_linear(layer, mat, q[:, cols], np.ascontiguousarray(s[:, groups]))
            else:  # row-parallel: this rank's input columns, every row's scale
                cols = slice(r * K // n, (r + 1) * K // n)
                qm.set_linear(layer, mat, q[:, cols], s)
        qm.set_tensor(3, layer, need(f"model.layers.{layer}.input_layernorm.weight", "F32", (cfg["dim"],)))
        qm.set_tensor(4, layer, need(f"model.layers.{layer}.post_attention_layernorm.weight", "F32", (cfg["dim"],)))
    V = cfg["vocab"]
    qm.set_tensor(0, 0, need("model.embed_tokens.weight", "F32", (V, cfg["dim"])))
    qm.set_tensor(2, 0, need("model.norm.weight", "F32", (cfg["dim"],)))
    lm = need("lm_head.weight", "F32", (V, cfg["dim"]))
    qm.set_tensor(1, 0, lm[r * V // n:(r + 1) * V // n])
