"""One rank of a tensor-parallel run of the engine (launched by
test_gpu_tp.py with torch.multiprocessing, one process per GPU).

Each rank joins a gloo process group (only to hand the NCCL unique id
around), builds its tb_comm and its share of the model, and runs the same
greedy generation; rank 0 reports the tokens."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def run(rank, world, port, cfg, batch, seed, prompt, steps, out_path, ckpt=None):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    import tendo_b200 as tb

    comm = tb.Comm.from_process_group(rank)
    m = tb.QuantizedModel(cfg, batch=batch, device=rank, comm=comm)
    if ckpt:
        from tendo_b200 import checkpoint

        checkpoint.load_model(m, ckpt)  # this rank's shard of the unsharded checkpoint
    else:
        m.init_synthetic(seed)
    toks = m.generate_greedy(np.asarray(prompt, dtype=np.int64), steps)
    m.close()
    dist.barrier()
    comm.close()
    if rank == 0:
        np.save(out_path, toks)
    dist.destroy_process_group()
