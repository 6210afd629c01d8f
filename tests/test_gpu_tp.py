"""Tensor parallelism (the 70B shape's partition) on 2 GPUs against the
oracle's unsharded model: column-parallel Q/K/V, gate/up and lm_head,
row-parallel O and down with an NCCL allreduce of the residual stream, the
greedy token from an allreduce (max) of packed (logit, index) keys.  Greedy
tokens must be identical.  Needs two GPUs; skipped on one."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# head_dim 32: the step-by-step decode path; head_dim 64: the captured fused step
GQA32 = dict(vocab=1000, dim=256, layers=3, heads=8, kv_heads=2, hidden=384, max_seq=160, rope_base=500000.0,
             eps=1e-5)
GQA64 = dict(vocab=1000, dim=512, layers=2, heads=8, kv_heads=2, hidden=768, max_seq=160, rope_base=500000.0,
             eps=1e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("cfg,batch", [(GQA32, 1), (GQA32, 3), (GQA64, 1), (GQA64, 12)])
def test_tp2_greedy_matches_unsharded_oracle(oracle, tb, cuda, tmp_path, cfg, batch):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    import tp_worker

    ref = oracle.Model(cfg, batch, seed=5)
    prompt = np.stack([oracle.synth_tokens(7 + b, 40, cfg["vocab"]) for b in range(batch)])
    want, _ = ref.generate_greedy(prompt, 24)
    out = str(tmp_path / "tokens.npy")
    mp.start_processes(tp_worker.run, args=(2, _free_port(), cfg, batch, 5, prompt, 24, out), nprocs=2,
                       join=True, start_method="spawn")
    np.testing.assert_array_equal(np.load(out), want)


def test_tp2_loads_its_shard_of_a_checkpoint(oracle, tb, cuda, tmp_path):
    """An unsharded pre-quantized checkpoint loaded by two tensor-parallel ranks."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    import tp_worker
    from tendo_b200 import checkpoint as ck

    cfg, batch = GQA64, 3
    src = tb.QuantizedModel(cfg, batch=1, device=0)
    src.init_synthetic(5)
    path = str(tmp_path / "m.safetensors")
    ck.export_model(src, path)
    src.close()
    ref = oracle.Model(cfg, batch, seed=5)
    prompt = np.stack([oracle.synth_tokens(7 + b, 40, cfg["vocab"]) for b in range(batch)])
    want, _ = ref.generate_greedy(prompt, 24)
    out = str(tmp_path / "tokens.npy")
    mp.start_processes(tp_worker.run, args=(2, _free_port(), cfg, batch, 5, prompt, 24, out, path), nprocs=2,
                       join=True, start_method="spawn")
    np.testing.assert_array_equal(np.load(out), want)


def test_tp2_peer_allreduce(tb, cuda, tmp_path):
    """The allreduce kernel over peer memory: exact on integer values, within
    fp32 rounding of the float64 sum on random values, the same bits on both
    ranks, across ragged sizes, both parities and the NCCL path past 4 MB."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    import tp_worker

    out = str(tmp_path / "ar.npy")
    mp.start_processes(tp_worker.run_allreduce, args=(2, _free_port(), out), nprocs=2, join=True,
                       start_method="spawn")
    r0, r1 = np.load(out, allow_pickle=True)
    assert r0["peer"] and r1["peer"]
    for k in r0:
        if k == "peer" or k.endswith("want"):
            continue
        np.testing.assert_array_equal(r0[k], r1[k])  # identical bits on every rank
        if k.endswith("_int"):
            np.testing.assert_array_equal(r0[k], r0[k[:-4] + "_intwant"])
        else:
            np.testing.assert_allclose(r0[k], r0[k[:-5] + "_want"], rtol=1e-6, atol=1e-6)
