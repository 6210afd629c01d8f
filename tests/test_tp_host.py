"""Host-side logic of the tensor-parallel path, on CPU (world_size 2, gloo).

* Vocabulary-split greedy choice: every rank packs its best (logit, global
  index) into one word — the logit's bits made order-preserving in the high
  32 bits, 2^32 - 1 - index in the low ones — and the ranks reduce with max.
  The result must be Greedy's choice over the whole vocabulary, first index
  on ties (models/sampling.go:73-83), ties across shards included.
* The Megatron partition of the quantized Linear (nn/quantize.go:293-312):
  row-parallel shards (input columns) sum to the unsharded product, and
  column-parallel shards (output rows) concatenate to it.
"""
import os
import socket

import numpy as np
import pytest


def packed_key(v, idx):
    b = int(np.float32(v).view(np.uint32))
    b = (~b & 0xFFFFFFFF) if (b & 0x80000000) else (b | 0x80000000)
    return (b << 32) | (0xFFFFFFFF - int(idx))


def unpack_index(k):
    return 0xFFFFFFFF - (k & 0xFFFFFFFF)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, logits, out_dir):
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    V = logits.shape[1]
    vl = V // world
    v0 = rank * vl
    keys = []
    for row in logits:
        shard = row[v0:v0 + vl]
        keys.append(max(packed_key(x, v0 + j) for j, x in enumerate(shard)))
    # gloo reduces signed int64: flip the top bit so signed order is the unsigned order
    t = torch.tensor([k ^ (1 << 63) for k in keys], dtype=torch.uint64).view(torch.int64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    got = [unpack_index((int(x) & 0xFFFFFFFFFFFFFFFF) ^ (1 << 63)) for x in t.tolist()]
    if rank == 0:
        np.save(os.path.join(out_dir, "idx.npy"), np.array(got, np.int64))
    dist.destroy_process_group()


def test_vocab_split_greedy_keys_over_gloo(tmp_path):
    import torch.multiprocessing as mp

    rng = np.random.default_rng(3)
    V = 64
    logits = rng.standard_normal((5, V)).astype(np.float32)
    logits[1, 40] = logits[1, 7] = 9.0       # tie across the two shards: index 7 wins
    logits[2, 3] = logits[2, 5] = 8.0        # tie inside shard 0
    logits[3, :] = -2.0                       # all equal and negative: index 0
    logits[4, 63] = 50.0                      # maximum in the last element of the last shard
    mp.start_processes(_rank, args=(2, _free_port(), logits, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    got = np.load(tmp_path / "idx.npy")
    want = np.array([int(np.argmax(r)) for r in logits])  # numpy: first index on ties
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("tp", [2, 4])
def test_megatron_partition_of_quantized_linear(oracle, tp):
    rng = np.random.default_rng(tp)
    N, K, M = 64, 128, 3
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    _, q, s = oracle.quantize(w, 0)
    full = oracle.dequant_matmul(x, q, s, 0)
    # column-parallel: output rows r N/tp .. (r + 1) N/tp, scales of those rows
    parts = [oracle.dequant_matmul(x, q[r * N // tp:(r + 1) * N // tp], s[r * N // tp:(r + 1) * N // tp], 0)
             for r in range(tp)]
    np.testing.assert_array_equal(np.concatenate(parts, axis=1), full)
    # row-parallel: input columns r K/tp .., full-row scales; the partial products sum to the product
    kl = K // tp
    psum = sum(oracle.dequant_matmul(np.ascontiguousarray(x[:, r * kl:(r + 1) * kl]),
                                     np.ascontiguousarray(q[:, r * kl:(r + 1) * kl]), s, 0) for r in range(tp))
    assert np.abs(psum - full).max() <= 1e-5 * np.abs(full).max()
