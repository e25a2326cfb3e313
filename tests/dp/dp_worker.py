"""Data-parallel worker for tests/test_dp.py (one process per rank).

With --device cpu it exercises the host-side DP logic over gloo (rank seeds,
unique-id broadcast, max-over-ranks timing); with --device cuda each rank
trains MeshGpt on its own GPU with the library's NCCL all-reduce and writes
its final parameters for the parent test to compare."""

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", choices=["cpu", "cuda"], required=True)
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    import numpy as np
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    if args.device == "cpu":
        dist.init_process_group("gloo", timeout=timedelta(seconds=60))
        from grokking_abmod_b200.data import zipf_batch
        x, _ = zipf_batch(7, rank, 0, 2, 16)
        gathered = [None] * world
        dist.all_gather_object(gathered, x.tobytes())
        box = [b"id-from-rank-0" if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ok = len(set(gathered)) == world and box[0] == b"id-from-rank-0" and float(t.item()) == world
        np.save(f"{args.out}.{rank}.npy", np.array([1 if ok else 0]))
        dist.destroy_process_group()
        return
    from grokking_abmod_b200 import AdamWOptions, GptConfig, MeshGpt, nccl_unique_id
    from grokking_abmod_b200.data import zipf_batch
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    cfg = GptConfig(vocab_size=64, context=64, width=256, heads=4, layers=2)
    model = MeshGpt(rank, cfg, 7)
    box = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    model.attach_nccl(box[0], rank, world)
    opt = AdamWOptions(learning_rate=1e-3, weight_decay=0.1)
    for step in range(3):
        x, y = zipf_batch(11, 0, step, 8 * world, 64)
        n = x.size // world
        model.train_batch_with_optimizer(x[rank * n:(rank + 1) * n], y[rank * n:(rank + 1) * n], 64, opt)
    np.save(f"{args.out}.{rank}.npy", model.parameters())
    model.detach_nccl()
    model.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
