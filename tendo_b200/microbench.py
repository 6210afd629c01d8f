"""Quantized Linear microbench: tb_dequant_matmul_i8f32 on one GPU.

    python -m tendo_b200.microbench [--M 1 8 32 128 2048] [--N 4096 11008] [--K 4096] [--iters 20] [--group G]
    python -m tendo_b200.microbench --decode-layers 8 [--tokens 4]
    python -m tendo_b200.microbench --kind attention [--width 70b] [--batch 16] [--position 2048]

W [N, K] is drawn N(0, 0.02) (seed 42) and int8-quantized per output channel
on the device (per group of G input columns with --group G: scales [N, K/G]);
X [M, K] is N(0, 1) (seed 42).  Enough weight copies are
rotated that every launch streams its weights from HBM, not L2 (126 MB).
Prints one JSON line per (M, N): microseconds per launch (CUDA events),
achieved GB/s over the algorithmic bytes N*K + 4N + 4MK + 4MN (4N*K/G for the
scales of --group G; the M <= 32
regime is HBM-bound) and TFLOP/s over 2MNK.

--decode-layers L runs the batch-1 decode step of a Llama-7B-width model cut
to L layers (d 4096, 32x128 heads, F 11008, vocab 32000, KV capacity 1024):
a 512-token prompt, then `--tokens` decode tokens, one persistent-kernel
launch each.  It is the small case for profiling that kernel (about 2.5 GB
on the device at L = 8).

--kind K times one kernel kind of the batched decode step (qkv, attention, o,
gateup, down, lm_head; tb_model_time_kernel: graph-timed, per layer) on one
layer of the 7B or 70B width (70B: d 8192, 64 query / 8 kv heads of 128,
F 28672, KV capacity 4096) at `--batch` sequences whose cache holds
`--position` rows (with `--group G`, a model quantized per group of G).  One
layer of the 70B width with its cache is about 3 GB on the device: the small
case for profiling those kernels.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

import tendo_b200 as tb


def linear_bytes(M, N, K, group=0):
    return N * K + 4 * N * (K // group if group else 1) + 4 * M * K + 4 * M * N


def run(Ms, Ns, K, iters, mode, group=0):
    be = tb.Backend(0)
    dev = torch.device("cuda:0")
    rows = []
    for N in Ns:
        w = be.SynthNormal(N, K, 42, tb.STREAM_W, 0.02)
        qt = be.Quantize(w, group)
        del w
        copies = max(2, math.ceil(400e6 / (N * K)))
        qs = [qt.data] + [qt.data.clone() for _ in range(copies - 1)]
        for M in Ms:
            x = be.SynthNormal(M, K, 42, tb.STREAM_X, 1.0)
            out = torch.empty((M, N), dtype=torch.float32, device=dev)
            st = torch.cuda.current_stream()
            sh = tb._stream(st)

            def launch(i):
                nonlocal sh
                tb.check(tb.lib.tb_dequant_matmul_i8f32_mode(out.data_ptr(), x.data_ptr(), qs[i % copies].data_ptr(),
                                                             qt.scale.data_ptr(), M, N, K, group, mode, sh))

            for i in range(3):
                launch(i)
            torch.cuda.synchronize()
            # the timed launches run from one CUDA graph, so host launch cost is excluded
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                sh = tb._stream(torch.cuda.current_stream())
                for i in range(iters):
                    launch(i)
            graph.replay()
            torch.cuda.synchronize()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(st)
            graph.replay()
            b.record(st)
            torch.cuda.synchronize()
            us = a.elapsed_time(b) * 1000.0 / iters
            byts = linear_bytes(M, N, K, group)
            row = {"M": M, "N": N, "K": K, "group": group, "us": us, "GB_s": byts / (us * 1e-6) / 1e9,
                   "TFLOP_s": 2.0 * M * N * K / (us * 1e-6) / 1e12, "bytes": byts,
                   "regime": "gemv" if M <= 32 else "gemm", "weight_copies": copies}
            rows.append(row)
            print(json.dumps(row), flush=True)
    return rows


def decode_small(layers, tokens):
    cfg = dict(vocab=32000, dim=4096, layers=layers, heads=32, kv_heads=32, hidden=11008, max_seq=1024,
               rope_base=10000.0, eps=1e-6)
    qm = tb.QuantizedModel(cfg, batch=1, device=0)
    qm.init_synthetic(0)
    prompt = tb.synth_tokens(512, cfg["vocab"], 0)
    _, first = qm.forward(prompt[None, :], want_logits=False)
    qm.set_position(512)
    qm.decode(tokens, start_tokens=first)
    qm.sync()
    out = {"layers": layers, "tokens": tokens, "launches_per_token": qm.launches_per_step,
           "first_tokens": qm.tokens(tokens + 1)[:, 0][:4].tolist()}
    print(json.dumps(out), flush=True)
    qm.close()


KINDS = ["qkv", "attention", "o", "gateup", "down", "lm_head"]


def time_kind(kind, width, batch, position, iters, group=0):
    if width == "70b":
        cfg = dict(vocab=32000, dim=8192, layers=1, heads=64, kv_heads=8, hidden=28672, max_seq=4096,
                   rope_base=500000.0, eps=1e-5)
    else:
        cfg = dict(vocab=32000, dim=4096, layers=1, heads=32, kv_heads=32, hidden=11008, max_seq=2048,
                   rope_base=10000.0, eps=1e-6)
    qm = tb.QuantizedModel(cfg, batch=batch, device=0, group=group)
    qm.init_synthetic(0)
    qm.set_position(position)
    us = qm.time_kernel(KINDS.index(kind), iters)
    print(json.dumps({"kind": kind, "width": width, "batch": batch, "position": position, "group": group, "us": us}),
          flush=True)
    qm.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--decode-layers", type=int, default=0)
    ap.add_argument("--tokens", type=int, default=4)
    ap.add_argument("--M", type=int, nargs="+", default=[1, 8, 32, 128, 2048])
    ap.add_argument("--N", type=int, nargs="+", default=[4096, 11008])
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--mode", type=int, default=tb.TB_GEMM_I8X3)
    ap.add_argument("--group", type=int, default=0)
    ap.add_argument("--kind", choices=KINDS, default=None)
    ap.add_argument("--width", choices=["7b", "70b"], default="70b")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--position", type=int, default=2048)
    a = ap.parse_args()
    if a.kind:
        time_kind(a.kind, a.width, a.batch, a.position, a.iters, a.group)
    elif a.decode_layers > 0:
        decode_small(a.decode_layers, a.tokens)
    else:
        run(a.M, a.N, a.K, a.iters, a.mode, a.group)


if __name__ == "__main__":
    main()
