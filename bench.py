"""Benchmark: int8 Llama-7B-shape batch-1 greedy decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (synthetic data of the stated shapes and distributions): 32 layers,
d_model 4096, 32 heads x 128 (MHA), SwiGLU 11008, vocab 32000, RMSNorm eps
1e-6, RoPE theta 1e4; weights N(0, 0.02) seed 0, int8 per output channel;
fp32 embedding and lm_head; batch 1; a 512-token uniform prompt (seed =
rank); KV cache of 2048 fp32 positions.  One step = 256 greedy decode tokens
from position 512 (the prompt's KV state stays resident; each step rewrites
positions 512..767).  `value` = decode tokens/s over all ranks with
everything resident in HBM; `e2e` = the same metric through the public
generate call (host prompt in, host tokens out, prefill included).

N > 1 runs N independent replicas (one process per GPU, no data-path
collective): weak scaling.  `--impl reference` times the CPU restatement of
tendo's path (the oracle) on the host cores for the same metric; under
torchrun only rank 0 runs it.

After the headline measurement the default run also measures, at the same
rank count and in the same process group, the two multi-GPU workloads below
(3 warm-up and min(K, 3) timed steps each) and attaches their lines to the
one JSON line under "multi_gpu_workloads" (`--no-extra` skips them).

    python -m torch.distributed.run --nproc-per-node N bench.py --workload llama70b-tp --gpus N

runs the Llama-70B shape tensor-parallel over the N ranks (N = 1 keeps the
whole model on one GPU): 80 layers, d_model 8192, 64 query / 8 kv heads x
128, SwiGLU 28672, vocab 32000, RoPE theta 5e5, batch 16, KV cache of 4096
positions; one step = 32 greedy tokens per sequence from position 2048.  The
2048-token prompts' KV state is left as zeros instead of prefilled (the
decode kernels read the same bytes whatever they hold; a 70B prefill is not
part of the decode metric), so this workload has no `e2e` or CPU leg.

    python -m torch.distributed.run --nproc-per-node N bench.py --workload llama7b-serving --gpus N

is batched serving of the 7B shape as data-parallel replicas: 64 sequences in
total, 64 / N per GPU, KV cache of 1280 positions, decode from position 1024
(the 1024-token prompts' KV state left as zeros, as above); one step = 32
greedy tokens per sequence; `value` = all ranks' tokens / the slowest rank's
time ("strong" scaling: the 64 sequences are fixed).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(vocab=32000, dim=4096, layers=32, heads=32, kv_heads=32, hidden=11008, max_seq=2048,
           rope_base=10000.0, eps=1e-6)
PROMPT = 512
NEW = 256
METRIC = "int8 Llama-7B decode tok/s (batch 1, greedy)"
WORKLOAD = ("llama7b-int8-decode: 32 layers, d_model 4096, 32x128 MHA, SwiGLU 11008, vocab 32000, int8 per-channel "
            "weights, fp32 activations/KV; batch 1; 512-token prompt; 256 greedy tokens per step; KV 2048 positions")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="default workload only: skip the serving and 70B tensor-parallel lines attached to it")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU baseline sample budget")
    ap.add_argument("--workload", default="llama7b", choices=["llama7b", "llama70b-tp", "llama7b-serving"])
    ap.add_argument("--kv-bf16", action="store_true",
                    help="llama7b-serving only: the bf16 KV cache option (a numerics change; off by default)")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ---------------------------------------------------------------------------
# algorithmic bytes (the roofline numerators)
# ---------------------------------------------------------------------------
def linear_bytes(M, N, K):
    """Quantized Linear: int8 weights + fp32 scales + fp32 x + fp32 y."""
    return N * K + 4 * N + 4 * M * K + 4 * M * N


def kernel_bytes(kind, P):
    c = CFG
    d, H, Hkv, D, F, V = c["dim"], c["heads"], c["kv_heads"], c["dim"] // c["heads"], c["hidden"], c["vocab"]
    if kind == 0:  # qkv (+ norm weight read) + k/v cache writes
        return linear_bytes(1, (H + 2 * Hkv) * D, d) + 4 * d
    if kind == 1:  # attention: K and V rows 0..P, q in, out
        return 2 * Hkv * D * (P + 1) * 4 + 2 * 4 * H * D
    if kind == 2:
        return linear_bytes(1, d, H * D) + 4 * d  # + residual read
    if kind == 3:
        return 2 * F * d + 8 * F + 4 * d + 4 * F + 4 * d
    if kind == 4:
        return linear_bytes(1, d, F) + 4 * d
    if kind == 5:
        return V * d * 4 + 4 * d + 4 * V
    raise ValueError(kind)


KIND_NAMES = ["qkv_rope_gemv", "attention_decode", "o_gemv", "gateup_swiglu_gemv", "down_gemv", "lmhead_gemv"]


def step_bytes(P):
    """Algorithmic bytes of one decode token at cache position P."""
    L = CFG["layers"]
    return sum(L * kernel_bytes(k, P) for k in range(5)) + kernel_bytes(5, P)


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU legs (the oracle): baseline of our arm and the reference arm
# ---------------------------------------------------------------------------
def cpu_decode_sample(model_fill, budget_s, max_tokens=None):
    """Times greedy decode steps of the oracle at positions 512.. on all host
    threads.  model_fill(m) fills the weights.  Returns (tok/s, tokens, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import pyoracle

    pyoracle.build()
    threads = os.cpu_count() or 1
    pyoracle.set_threads(threads)
    m = pyoracle.Model(dict(CFG, max_seq=PROMPT + 64), 1, seed=0, generate=False)
    model_fill(m, pyoracle)
    # The KV state of the 512 prompt positions is left as zeros: attention
    # reads the same bytes whatever they hold, so the cost matches the workload.
    m.set_pos(PROMPT)
    tok = np.array([1], np.int64)
    t0 = time.perf_counter()
    tok = m.decode_step(tok)  # one untimed step (page-in)
    first = time.perf_counter() - t0
    n = max(1, int(budget_s / max(first, 1e-3)))
    if max_tokens:
        n = min(n, max_tokens)
    n = min(n, 60)
    t0 = time.perf_counter()
    for _ in range(n):
        tok = m.decode_step(tok)
    dt = time.perf_counter() - t0
    m.close()
    return n / dt, n, pyoracle.get_threads()


def cpu_planned_workloads(rows_cap=256):
    """The other CPU baseline workloads timed beside the headline, on all host
    threads, with the oracle restatement of tendo's CPU path: the tiny config
    end to end (prefill of its 128-token prompt, then 128 greedy decode steps),
    and the quantized Linear (dequantize then the fp32 product) at K 4096 over
    the decode/prefill grid.  Linear rows are independent, so M 2048 is timed
    on its first rows_cap rows and reported per full call."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import pyoracle

    pyoracle.build()
    pyoracle.set_threads(os.cpu_count() or 1)
    out = {"cores": pyoracle.get_threads(), "kind": "port"}
    cfg = dict(pyoracle.TINY)
    m = pyoracle.Model(cfg, 1, seed=0)
    prompt = pyoracle.synth_tokens(1, 128, cfg["vocab"])
    t0 = time.perf_counter()
    _, last, _ = m.forward(prompt[None, :], want_logits=False)
    t1 = time.perf_counter()
    tok = np.array([int(np.argmax(last[0]))], np.int64)
    for _ in range(128):
        tok = m.decode_step(tok)
    t2 = time.perf_counter()
    m.close()
    out["tiny_end_to_end"] = {"prefill_ms": (t1 - t0) * 1e3, "decode_ms_per_token": (t2 - t1) * 1e3 / 128,
                              "workload": "8 layers, d_model 512, 8x64 MHA, SwiGLU 1408, vocab 32000; batch 1; "
                                          "128-token prompt, 128 greedy tokens"}
    rng = np.random.default_rng(42)
    K = 4096
    grid = []
    for N in (4096, 11008):
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        _, q, sc = pyoracle.quantize(w, 0)
        del w
        for M in (1, 8, 32, 128, 2048):
            rows = min(M, rows_cap)
            x = rng.standard_normal((rows, K)).astype(np.float32)
            reps = max(1, 8 // rows)
            t0 = time.perf_counter()
            for _ in range(reps):
                pyoracle.dequant_matmul(x, q, sc, 0)
            us = (time.perf_counter() - t0) / reps * 1e6 * (M / rows)
            byts = linear_bytes(M, N, K)
            grid.append({"M": M, "N": N, "K": K, "us": us, "GB_s": byts / (us * 1e-6) / 1e9,
                         "GFLOP_s": 2.0 * M * N * K / (us * 1e-6) / 1e9, "rows_timed": rows})
    out["linear_grid"] = grid
    return out


def fill_from_device(qm):
    def fill(m, po):
        for layer in range(CFG["layers"]):
            for mat in range(7):
                q, s = qm.get_linear(layer, mat, m.shape(mat))
                m.q(layer, mat)[...] = q
                m.scale(layer, mat)[...] = s
        m.embed()[...] = qm.get_tensor(0, 0, (CFG["vocab"], CFG["dim"]))
        m.lm_head()[...] = qm.get_tensor(1, 0, (CFG["vocab"], CFG["dim"]))
    return fill


def fill_on_host(m, po):
    """The reference arm draws its own weights on the host (no GPU involved)."""
    import numpy as np

    for layer in range(CFG["layers"]):
        for mat in range(7):
            N, K = m.shape(mat)
            w = po.synth_normal(0, layer * 8 + mat, N * K, 0.02).reshape(N, K)
            _, q, s = po.quantize(w, 0)
            m.q(layer, mat)[...] = q
            m.scale(layer, mat)[...] = s
    V, d = CFG["vocab"], CFG["dim"]
    m.embed()[...] = po.synth_normal(0, po.STREAM_EMBED, V * d, 0.02).reshape(V, d)
    m.lm_head()[...] = po.synth_normal(0, po.STREAM_LMHEAD, V * d, 0.02).reshape(V, d)
    del np


PHASE_NAMES = ["qkv", "attention", "o", "gateup", "down"]


def summarize_phases(us):
    """Per-token microseconds of the persistent decode kernel by phase step
    (CTA 0's view).  A staging interval includes the wait for the previous
    phase's tagged results; attention includes the combine of the splits."""
    L = CFG["layers"]
    if us is None or len(us) < 13 * L + 3:
        return None
    names = ["qkv.stage", "qkv.tiles", "qkv.epi", "attention", "o.stage", "o.tiles", "o.epi", "gateup.stage",
             "gateup.tiles", "gateup.epi", "down.stage", "down.tiles", "down.epi"]
    out = {}
    for l in range(L):
        for k, name in enumerate(names):
            out[name] = out.get(name, 0.0) + float(us[13 * l + k])
    i = 13 * L
    out["lm_head.norm"] = float(us[i])
    out["lm_head.tiles"] = float(us[i + 1])
    out["final.wait"] = float(us[i + 2])
    out["total"] = float(sum(us[: i + 3]))
    return {k: round(v, 1) for k, v in out.items()}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    t0 = time.perf_counter()
    # each "step" of this arm is one decode token (a bounded sample of the 256-token step)
    budget = None
    rate, n, threads = cpu_decode_sample(fill_on_host, budget_s=1e9, max_tokens=args.steps + 0)
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": n, "warmup": 1, "ms_per_step": 1000.0 / rate, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": PROMPT + NEW, "parallelism": "none (CPU)"},
        "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{n} greedy decode tokens at positions 512.. of the 7B workload (one token per "
                                   f"step), oracle restatement of tendo's CPU path, weights drawn on the host"},
        "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0,
    }
    del budget
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import numpy as np
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
        pg = dist
    import tendo_b200 as tb

    qm = tb.QuantizedModel(CFG, batch=1, device=local)
    qm.init_synthetic(0)
    prompt = tb.synth_tokens(PROMPT, CFG["vocab"], rank)
    _, first = qm.forward(prompt[None, :], want_logits=False)
    stream = torch.cuda.ExternalStream(qm.stream_handle, device=dev)

    def step():
        qm.set_position(PROMPT)
        qm.decode(NEW, start_tokens=first)

    for _ in range(max(args.warmup, 0)):
        step()
    qm.sync()
    toks = qm.tokens(NEW + 1)[:, 0]

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    clocks = Clocks(local)
    barrier()
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    qm.sync()
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms_max = float(t.item())
    total_tokens = world * args.steps * NEW
    value = total_tokens / (ms_max / 1000.0)

    # per-kernel timing of the multi-kernel decode step (the path taken when
    # the persistent kernel does not apply: batch > 1, unsupported shapes),
    # same stream, CUDA events, cycling over all layers so weights stream from HBM
    qm.set_position(PROMPT + NEW // 2)  # mean cache length of a step
    kern = {}
    for kind in range(6):
        us = qm.time_kernel(kind, reps=3)
        byts = kernel_bytes(kind, PROMPT + NEW // 2)
        per_step = CFG["layers"] if kind < 5 else 1
        kern[KIND_NAMES[kind]] = {"us": us, "bytes": byts, "GB_s": byts / (us * 1e-6) / 1e9,
                                  "share_est": us * per_step}
    tot = sum(v["share_est"] for v in kern.values())
    for v in kern.values():
        v["share_est"] = v["share_est"] / tot
    dom = max(kern, key=lambda k: kern[k]["share_est"])

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    ms_per_tok = ms_max / (args.steps * NEW)
    model_bytes = statistics.mean(step_bytes(PROMPT + i) for i in range(NEW))
    model_gbs = model_bytes / (ms_per_tok / 1000.0) / 1e9
    persistent = qm.launches_per_step == 1
    if persistent:
        # the whole token is one launch of the persistent decode kernel: its
        # average launch duration is the timed region over the launches in it
        dom = "decode_megakernel"
        dom_gbs = model_gbs
    else:
        dom_gbs = kern[dom]["GB_s"]
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.txt")) as f:
            for line in f:
                parts = line.split("#")[0].split()
                if len(parts) == 2 and parts[0] == dom:
                    traffic = float(parts[1])
    except (OSError, ValueError):
        traffic = None
    roofline = {"bound": "hbm", "achieved": dom_gbs, "peak": hbm_peak, "unit": "GB/s",
                "frac": dom_gbs / hbm_peak, "traffic": traffic, "kernel": dom, "peak_source": peak_src,
                "bytes_per_launch": model_bytes if persistent else kern[dom]["bytes"],
                "launch_us": ms_per_tok * 1000.0 if persistent else kern[dom]["us"],
                "model_achieved": model_gbs, "model_frac": model_gbs / hbm_peak,
                "model_bytes_per_token": model_bytes}

    # e2e: the public generate call, host prompt in, host tokens out (prefill included)
    e2e = None
    if rank == 0 or world > 1:
        reps_e2e = 2
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        barrier()
        a.record(stream)
        for _ in range(reps_e2e):
            out = qm.generate_greedy(prompt[None, :], NEW)
        b.record(stream)
        qm.sync()
        barrier()
        te = torch.tensor([a.elapsed_time(b)], device=dev)
        if pg is not None:
            pg.all_reduce(te, op=pg.ReduceOp.MAX)
        e2e_ms = float(te.item()) / reps_e2e
        e2e = {"value": world * NEW / (e2e_ms / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": PROMPT * 8,
               "d2h_bytes_per_step": NEW * 8, "ms_per_step": e2e_ms,
               "note": "tb_model_generate_greedy: 512-token prefill + 256 greedy tokens, host buffers"}
        assert out[0, 0] == toks[0], "generate_greedy disagrees with the timed decode"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, threads = cpu_decode_sample(fill_from_device(qm), args.cpu_seconds)
        cpu = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{n} greedy decode tokens at positions 512.. of the same 7B workload, oracle restatement "
                         f"of tendo's CPU path on {threads} host threads (weights copied from the device)"}

    cpu_more = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_more = cpu_planned_workloads()

    # the timed tokens against the oracle's golden stream of this workload
    # (tests/golden/llama7b_decode.json: same weights, prompt seed 0)
    parity = None
    if rank == 0:
        with open(os.path.join(ROOT, "tests", "golden", "llama7b_decode.json")) as f:
            gold = [st["token"] for st in json.load(f)["steps"]]
        n_chk = min(len(gold), NEW + 1)
        got = [int(t) for t in toks[:n_chk]]
        if got != gold[:n_chk]:
            raise SystemExit(f"decode tokens differ from the oracle's golden stream: {got} != {gold[:n_chk]}")
        parity = {"fixture": "tests/golden/llama7b_decode.json", "greedy_tokens_checked": n_chk, "match": True}

    phases = summarize_phases(qm.phase_times())
    launches = qm.launches_per_step * NEW * args.steps
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": PROMPT + NEW,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2: 6.5 GB int8 weights + 0.52 GB fp32 lm_head stream per token"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clk, "standalone_kernels": kern, "phases_us": phases, "first_tokens": toks[:8].tolist(),
            "parity": parity,
        }
        if cpu_more is not None:
            line["cpu_workloads"] = cpu_more
    qm.close()
    if not args.no_extra:
        # the multi-GPU workloads at this rank count, in the same process
        # group, after the headline model is freed: serving (64 sequences
        # split over the ranks) and the 70B shape tensor parallel over them
        xs, xw = min(args.steps, 3), 3
        extra = {}
        if SERVE_SEQS % world == 0:
            extra["llama7b-serving"] = measure_serving(args, xs, xw)
        if CFG70["kv_heads"] % world == 0:
            extra["llama70b-tp"] = measure_70b_tp(args, xs, xw)
        if rank == 0:
            line["multi_gpu_workloads"] = extra
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


# ---------------------------------------------------------------------------
# Llama-70B shape, tensor parallel over the ranks
# ---------------------------------------------------------------------------
CFG70 = dict(vocab=32000, dim=8192, layers=80, heads=64, kv_heads=8, hidden=28672, max_seq=4096,
             rope_base=500000.0, eps=1e-5)
B70, PROMPT70, NEW70 = 16, 2048, 32
METRIC70 = "int8 Llama-70B decode tok/s (batch 16, greedy, tensor parallel)"


def step_bytes70(P):
    """Algorithmic bytes of one decode step (16 tokens) of the whole model at
    cache position P: int8 weights + scales, fp32 lm_head, the 16 sequences'
    fp32 KV rows 0..P (summed over the tensor-parallel shards)."""
    c = CFG70
    d, H, Hkv, F, V, L = c["dim"], c["heads"], c["kv_heads"], c["hidden"], c["vocab"], c["layers"]
    D = d // H
    per_layer = (H + 2 * Hkv) * D * d + d * H * D + 2 * F * d + d * F
    scales = (H + 2 * Hkv) * D + d + 2 * F + d
    kv = 2 * Hkv * D * (P + 1) * 4 * B70
    return L * (per_layer + 4 * scales + kv) + V * d * 4


def measure_70b_tp(args, steps, warmup):
    """The 70B tensor-parallel decode over every rank of the (already
    initialised) process group; returns rank 0's JSON line (others: None)."""
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    dev = torch.device("cuda", local)
    import tendo_b200 as tb

    comm = tb.Comm.from_process_group(local) if world > 1 else None
    qm = tb.QuantizedModel(CFG70, batch=B70, device=local, comm=comm)
    qm.init_synthetic(0)
    stream = torch.cuda.ExternalStream(qm.stream_handle, device=dev)
    start = tb.synth_tokens(B70, CFG70["vocab"], 11)

    def step():
        qm.set_position(PROMPT70)
        qm.decode(NEW70, start_tokens=start)

    for _ in range(max(warmup, 0)):
        step()
    qm.sync()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = Clocks(local)
    barrier()
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    qm.sync()
    barrier()
    clk = clocks.stop()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    toks = qm.tokens(NEW70 + 1)[:, 0]
    tokens = steps * NEW70 * B70
    value = tokens / (ms / 1000.0)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    ms_tok = ms / (steps * NEW70)
    byts = statistics.mean(step_bytes70(PROMPT70 + i) for i in range(NEW70))
    achieved = byts / (ms_tok / 1000.0) / 1e9
    line = None
    if rank == 0:
        line = {
            "metric": METRIC70, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
            "config": {"workload": "llama70b-int8-tp-decode: 80 layers, d_model 8192, 64/8 heads x 128 (GQA), SwiGLU "
                                   "28672, vocab 32000; batch 16; decode from position 2048 (prompt KV zeros); "
                                   "32 greedy tokens per step; KV 4096 positions",
                       "global_batch": B70, "seq_len": PROMPT70 + NEW70, "parallelism": f"tp{world}",
                       "l2": "inputs larger than L2: 68 GB int8 weights + 21 GB KV per step"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak * world, "unit": "GB/s",
                         "frac": achieved / (hbm_peak * world), "traffic": None, "kernel": "whole decode step",
                         "bytes_per_token_step": byts, "peak_source": "measured" if "hbm_gbs" in peaks else "fallback"},
            "cpu_baseline": None, "e2e": None, "gpu_launches": None, "clocks": clk, "first_tokens": toks[:8].tolist(),
            "note": "no e2e or CPU leg for this workload: see the module docstring",
        }
    qm.close()
    if comm is not None:
        comm.close()
    if world > 1:
        dist.barrier()
    return line


def run_70b_tp(args):
    import datetime

    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    line = measure_70b_tp(args, args.steps, args.warmup)
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# Llama-7B shape, batched serving as replicas
# ---------------------------------------------------------------------------
SERVE_SEQS, SERVE_PROMPT, SERVE_NEW, SERVE_KV = 64, 1024, 32, 1280
METRIC_SERVE = "int8 Llama-7B batched serving decode tok/s (64 sequences, greedy, replicas)"


def step_bytes_serve(P, seqs, kv_bytes=4):
    """Algorithmic bytes of one decode step of `seqs` sequences on one replica
    at cache position P: the weights once, every sequence's KV rows 0..P
    (kv_bytes per element: 4 fp32, 2 with the bf16 cache option)."""
    c = CFG
    d, H, Hkv, F, V, L = c["dim"], c["heads"], c["kv_heads"], c["hidden"], c["vocab"], c["layers"]
    D = d // H
    w = L * ((H + 2 * Hkv) * D * d + d * H * D + 3 * F * d) + V * d * 4
    kv = L * 2 * Hkv * D * (P + 1) * kv_bytes * seqs
    return w + kv


def measure_serving(args, steps, warmup):
    """The 7B serving decode, 64 sequences split over the ranks of the
    (already initialised) process group; returns rank 0's JSON line."""
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    B = SERVE_SEQS // world
    dev = torch.device("cuda", local)
    import tendo_b200 as tb

    kv16 = bool(getattr(args, "kv_bf16", False))
    qm = tb.QuantizedModel(dict(CFG, max_seq=SERVE_KV), batch=B, device=local, kv_bf16=kv16)
    qm.init_synthetic(0)
    stream = torch.cuda.ExternalStream(qm.stream_handle, device=dev)
    start = tb.synth_tokens(B, CFG["vocab"], 7 + rank)

    def step():
        qm.set_position(SERVE_PROMPT)
        qm.decode(SERVE_NEW, start_tokens=start)

    for _ in range(max(warmup, 0)):
        step()
    qm.sync()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = Clocks(local)
    barrier()
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    qm.sync()
    barrier()
    clk = clocks.stop()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = SERVE_SEQS * SERVE_NEW * steps / (ms / 1000.0)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    ms_tok = ms / (steps * SERVE_NEW)
    per_gpu = statistics.mean(step_bytes_serve(SERVE_PROMPT + i, B, 2 if kv16 else 4) for i in range(SERVE_NEW))
    achieved = per_gpu / (ms_tok / 1000.0) / 1e9
    toks = qm.tokens(SERVE_NEW + 1)[:, 0]
    line = None
    if rank == 0:
        line = {
            "metric": METRIC_SERVE, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8/fp32, bf16 KV" if kv16 else "int8/fp32", "data": "synthetic",
            "config": {"workload": f"llama7b-int8-serving: 64 sequences as {world} replicas of {B}; decode from "
                                   "position 1024 (prompt KV zeros); 32 greedy tokens per step; KV 1280 positions"
                                   + ("; bf16 KV cache option" if kv16 else ""),
                       "global_batch": SERVE_SEQS, "seq_len": SERVE_PROMPT + SERVE_NEW,
                       "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2: 7 GB weights + KV per step"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "traffic": None, "kernel": "whole decode step, per GPU",
                         "bytes_per_token_step_per_gpu": per_gpu,
                         "peak_source": "measured" if "hbm_gbs" in peaks else "fallback"},
            "cpu_baseline": None, "e2e": None, "gpu_launches": None, "clocks": clk, "first_tokens": toks[:8].tolist(),
            "note": "no e2e or CPU leg for this workload: see the module docstring",
        }
    qm.close()
    if world > 1:
        dist.barrier()
    return line


def run_serving(args):
    import datetime

    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    if SERVE_SEQS % world:
        raise SystemExit(f"{SERVE_SEQS} sequences do not split over {world} replicas")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    line = measure_serving(args, args.steps, args.warmup)
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.workload == "llama7b-serving":
        if args.impl == "reference":
            if dist_env()[0] == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference arm runs on the default 7B "
                                  "batch-1 workload; 64 sequences of the CPU restatement take minutes per token"}),
                      flush=True)
            return
        run_serving(args)
        return
    if args.workload == "llama70b-tp":
        if args.impl == "reference":
            if dist_env()[0] == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the 70B shape's CPU restatement needs "
                                  "about 70 GB of host weights and minutes per token; the reference arm runs on the "
                                  "default 7B workload"}), flush=True)
            return
        run_70b_tp(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
