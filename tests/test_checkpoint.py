"""Pre-quantized int8 checkpoints (tendo_b200/checkpoint.py), host side.

* Files laid out as the reference's own safetensors tests build them
  (safetensors_test.go:19-86: unpadded JSON header, little-endian F32 data)
  read back to the same values.
* Round trips of I8 / F32 / I64 tensors, header metadata, 8-byte padding.
* Malformed files are rejected with CheckpointError.
* Tensor-parallel loading hands every rank the right shard: rows of the
  column-parallel matrices, input columns and all scales of the row-parallel
  ones, rows of the lm_head; embedding and norms whole.
"""
import json
import struct

import numpy as np
import pytest

from tendo_b200 import checkpoint as ck


def _reference_style(path, tensors):
    """The construction of safetensors_test.go:19-86, restated: header
    entries in order, no padding, data appended in the same order."""
    header, data = {}, b""
    for name, (dtype, shape, values) in tensors.items():
        raw = np.asarray(values, dtype="<f4").tobytes()
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [len(data), len(data) + len(raw)]}
        data += raw
    h = json.dumps(header, separators=(",", ":")).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + data)


def test_reads_reference_style_files(tmp_path):
    p = str(tmp_path / "ref.safetensors")
    _reference_style(p, {"weight": ("F32", [2, 3], [1, 2, 3, 4, 5, 6]), "bias": ("F32", [3], [0.5, -1.5, 2.25])})
    st = ck.SafeTensors(p)
    assert sorted(st.names()) == ["bias", "weight"]
    assert st.info("weight") == ("F32", (2, 3))
    np.testing.assert_array_equal(st.get("weight"), np.arange(1, 7, dtype=np.float32).reshape(2, 3))
    np.testing.assert_array_equal(st.get("bias"), np.array([0.5, -1.5, 2.25], np.float32))


def test_round_trip_int8_and_metadata(tmp_path):
    rng = np.random.default_rng(0)
    t = {"q": rng.integers(-128, 128, (7, 33), dtype=np.int8), "s": rng.random(7, dtype=np.float32),
         "ids": np.arange(5, dtype=np.int64), "empty": np.zeros((0, 4), np.float32)}
    p = str(tmp_path / "a.safetensors")
    ck.write(p, t, {"format": "tendo-int8-per-channel", "layers": 2})
    raw = open(p, "rb").read()
    (n,) = struct.unpack("<Q", raw[:8])
    assert n % 8 == 0  # header padded to 8 bytes
    st = ck.SafeTensors(p)
    assert st.metadata == {"format": "tendo-int8-per-channel", "layers": "2"}
    for k, v in t.items():
        got = st.get(k)
        assert got.dtype == v.dtype and got.shape == v.shape
        np.testing.assert_array_equal(got, v)


@pytest.mark.parametrize("bad", ["truncated", "dtype", "offsets", "json"])
def test_malformed_files_are_rejected(tmp_path, bad):
    p = str(tmp_path / "bad.safetensors")
    ck.write(p, {"x": np.ones(4, np.float32)})
    raw = bytearray(open(p, "rb").read())
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n].decode())
    if bad == "truncated":
        raw = raw[:8 + n // 2]
    elif bad == "json":
        raw[8] = ord("#")
    else:
        if bad == "dtype":
            header["x"]["dtype"] = "Q4"
        else:
            header["x"]["data_offsets"] = [0, 12]
        h = json.dumps(header).encode()
        raw = struct.pack("<Q", len(h)) + h + raw[8 + n:]
    open(p, "wb").write(bytes(raw))
    with pytest.raises(ck.CheckpointError):
        ck.SafeTensors(p)


class _Comm:
    def __init__(self, rank, nranks):
        self.rank, self.nranks = rank, nranks


class _FakeModel:
    """Records what load_model uploads (the engine's set_linear / set_tensor)."""

    def __init__(self, cfg, comm):
        self.cfg, self.comm = cfg, comm
        self.lin, self.ten = {}, {}

    def set_linear(self, layer, mat, q, s):
        self.lin[(layer, mat)] = (np.array(q), np.array(s))

    def set_tensor(self, which, layer, a):
        self.ten[(which, layer)] = np.array(a)


CFG = dict(vocab=64, dim=32, layers=2, heads=4, kv_heads=2, hidden=48)


def _checkpoint(path, group=0):
    rng = np.random.default_rng(1)
    t = {}
    for layer in range(CFG["layers"]):
        for mat, (N, K) in enumerate(ck._shapes(CFG)):
            name = ck._linear_name(layer, mat)
            t[name + ".weight"] = rng.integers(-127, 128, (N, K), dtype=np.int8)
            t[name + ".weight_scale"] = rng.random((N, K // group) if group else N, dtype=np.float32)
        t[f"model.layers.{layer}.input_layernorm.weight"] = rng.random(CFG["dim"], dtype=np.float32)
        t[f"model.layers.{layer}.post_attention_layernorm.weight"] = rng.random(CFG["dim"], dtype=np.float32)
    t["model.embed_tokens.weight"] = rng.random((CFG["vocab"], CFG["dim"]), dtype=np.float32)
    t["model.norm.weight"] = rng.random(CFG["dim"], dtype=np.float32)
    t["lm_head.weight"] = rng.random((CFG["vocab"], CFG["dim"]), dtype=np.float32)
    ck.write(path, t)
    return t


@pytest.mark.parametrize("nranks", [1, 2])
def test_tensor_parallel_shards(tmp_path, nranks):
    p = str(tmp_path / "m.safetensors")
    t = _checkpoint(p)
    for r in range(nranks):
        m = _FakeModel(CFG, _Comm(r, nranks) if nranks > 1 else None)
        ck.load_model(m, p)
        for layer in range(CFG["layers"]):
            for mat, (N, K) in enumerate(ck._shapes(CFG)):
                q, s = m.lin[(layer, mat)]
                full_q = t[ck._linear_name(layer, mat) + ".weight"]
                full_s = t[ck._linear_name(layer, mat) + ".weight_scale"]
                if ck.LINEARS[mat][1]:
                    rows = slice(r * N // nranks, (r + 1) * N // nranks)
                    np.testing.assert_array_equal(q, full_q[rows])
                    np.testing.assert_array_equal(s, full_s[rows])
                else:
                    cols = slice(r * K // nranks, (r + 1) * K // nranks)
                    np.testing.assert_array_equal(q, full_q[:, cols])
                    np.testing.assert_array_equal(s, full_s)
        V = CFG["vocab"]
        np.testing.assert_array_equal(m.ten[(1, 0)], t["lm_head.weight"][r * V // nranks:(r + 1) * V // nranks])
        np.testing.assert_array_equal(m.ten[(0, 0)], t["model.embed_tokens.weight"])


def test_shape_mismatch_is_rejected(tmp_path):
    p = str(tmp_path / "m.safetensors")
    _checkpoint(p)
    m = _FakeModel(dict(CFG, hidden=64), None)
    with pytest.raises(ck.CheckpointError):
        ck.load_model(m, p)


@pytest.mark.parametrize("nranks", [1, 2])
def test_grouped_checkpoint_shards(tmp_path, nranks):
    """Per-group scales [N, K / group]: a column-parallel rank takes its rows'
    scales, a row-parallel rank its input columns and the groups over them."""
    group = 8
    p = str(tmp_path / "g.safetensors")
    t = _checkpoint(p, group)
    for r in range(nranks):
        m = _FakeModel(CFG, _Comm(r, nranks) if nranks > 1 else None)
        m.group = group
        ck.load_model(m, p)
        for layer in range(CFG["layers"]):
            for mat, (N, K) in enumerate(ck._shapes(CFG)):
                q, s = m.lin[(layer, mat)]
                full_q = t[ck._linear_name(layer, mat) + ".weight"]
                full_s = t[ck._linear_name(layer, mat) + ".weight_scale"]
                if ck.LINEARS[mat][1]:
                    rows = slice(r * N // nranks, (r + 1) * N // nranks)
                    np.testing.assert_array_equal(q, full_q[rows])
                    np.testing.assert_array_equal(s, full_s[rows])
                else:
                    cols = slice(r * K // nranks, (r + 1) * K // nranks)
                    groups = slice(r * (K // group) // nranks, (r + 1) * (K // group) // nranks)
                    np.testing.assert_array_equal(q, full_q[:, cols])
                    np.testing.assert_array_equal(s, full_s[:, groups])
    m = _FakeModel(CFG, None)  # a per-channel model rejects per-group scales
    with pytest.raises(ck.CheckpointError):
        ck.load_model(m, p)
