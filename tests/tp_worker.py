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


def run_allreduce(rank, world, port, out_path):
    """tb_allreduce_sum_f32 on sizes across the peer kernel's slicing (ragged
    tails, one to 64 CTAs) and past its 4 MB capacity (NCCL), three times each
    so both receive-slot parities are used; rank 0 saves every rank's results."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    import tendo_b200 as tb

    comm = tb.Comm.from_process_group(rank)
    res = {"peer": comm.peer}
    for n in (1, 3, 5, 4096 + 3, 131072, 1 << 20, (1 << 20) + 4):
        for rep in range(3):
            g = torch.Generator().manual_seed(1000 * n + rep)
            full = torch.randn(world, n, generator=g, dtype=torch.float32)
            ints = torch.randint(-1000, 1000, (world, n), generator=g).to(torch.float32)
            a = full[rank].cuda()
            b = ints[rank].cuda()
            comm.allreduce_sum(a)
            comm.allreduce_sum(b)
            torch.cuda.synchronize()
            res[f"{n}_{rep}_rand"] = a.cpu().numpy()
            res[f"{n}_{rep}_want"] = full.double().sum(0).numpy()
            res[f"{n}_{rep}_int"] = b.cpu().numpy()
            res[f"{n}_{rep}_intwant"] = ints.sum(0).numpy()
    got = [None] * world
    dist.all_gather_object(got, res)
    dist.barrier()
    comm.close()
    if rank == 0:
        np.save(out_path, np.array(got, dtype=object), allow_pickle=True)
    dist.destroy_process_group()
