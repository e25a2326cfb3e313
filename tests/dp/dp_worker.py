"""Data-parallel worker for tests/test_dp.py (one process per rank).

--device cpu (gloo): the host-side DP plumbing the bench relies on (rank
seeds, unique-id broadcast, max-over-ranks timing) and the arithmetic of the
library's exact data-parallel loss: every rank's supervised count is summed
first, each rank divides its cross-entropy adjoint by that global count, and
the per-rank gradients and losses are then summed.  The ranks hold different
numbers of supervised targets (answer-only rows on rank 0), so this differs
from averaging per-rank means; each rank saves the combined loss and gradient
of the f64 oracle for the parent to compare with the whole batch.

--device cuda: each rank trains MeshGpt on its own GPU with the library's NCCL
exchange, first through a communicator the library creates from a unique id,
then through a caller-owned communicator, and saves its loss, gradient and
final parameters."""

import argparse
import ctypes
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

# The shared problem: a tiny Mesh GPT and a batch of 2 x 4 sequences whose
# first half (rank 0's share) is supervised only on each sequence's last row.
TINY = dict(vocab_size=9, context=8, width=64, heads=4, layers=1, attention_mesh_depth=2, ffn_mesh_depth=2)
GPU_CFG = dict(vocab_size=64, context=64, width=256, heads=4, layers=2)


def dp_batch(vocab, seqs, seq, world, seed):
    """The whole batch and its rank shares: rank 0's sequences are
    answer-only, the other ranks' are fully supervised."""
    import numpy as np
    from oracle.data import IGNORE_TARGET
    rng = np.random.default_rng(seed)
    x = rng.integers(0, vocab, seqs * seq).astype(np.uint32)
    y = rng.integers(0, vocab, seqs * seq).astype(np.uint32)
    n = x.size // world
    y[:n][np.arange(n) % seq != seq - 1] = IGNORE_TARGET
    return x, y, n


def _nccl():
    lib = ctypes.CDLL("libnccl.so.2")

    class UniqueId(ctypes.Structure):
        _fields_ = [("internal", ctypes.c_char * 128)]

    lib.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, UniqueId, ctypes.c_int]
    lib.ncclCommDestroy.argtypes = [ctypes.c_void_p]
    return lib, UniqueId


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

        # exact DP arithmetic on the oracle
        from oracle.gpt_config import GptConfig
        from oracle.gpt_ref import ReferenceGpt
        from oracle.data import IGNORE_TARGET
        ref = ReferenceGpt(GptConfig(**TINY), seed=7)
        x, y, n = dp_batch(TINY["vocab_size"], 8, 4, world, seed=1)
        xs, ys = x[rank * n:(rank + 1) * n], y[rank * n:(rank + 1) * n]
        local = int((ys != IGNORE_TARGET).sum())
        count = torch.tensor([float(local)], dtype=torch.float64)
        dist.all_reduce(count)                                   # the global supervised count
        loss, grad = ref.loss_and_gradient(xs, ys, 4)            # local means (divided by `local`)
        share = torch.from_numpy(np.concatenate([[loss], grad]) * (local / float(count.item())))
        dist.all_reduce(share)                                   # sum of the ranks' shares
        naive = torch.from_numpy(np.concatenate([[loss], grad]) / world)
        dist.all_reduce(naive)                                   # the mean of per-rank means
        np.save(f"{args.out}.exact.{rank}.npy", share.numpy())
        np.save(f"{args.out}.naive.{rank}.npy", naive.numpy())
        dist.destroy_process_group()
        return

    from grokking_abmod_b200 import AdamWOptions, GptConfig, MeshGpt, nccl_unique_id
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    model = MeshGpt(rank, GptConfig(**GPU_CFG), 7)
    box = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    model.attach_nccl(box[0], rank, world)
    x, y, n = dp_batch(GPU_CFG["vocab_size"], 8 * world, 64, world, seed=3)
    xs, ys = x[rank * n:(rank + 1) * n], y[rank * n:(rank + 1) * n]
    loss, grad = model.loss_and_gradient(xs, ys, 64)
    np.save(f"{args.out}.grad.{rank}.npy", np.concatenate([[loss], grad]))

    # the same evaluation through a caller-owned communicator
    model.detach_nccl()
    nccl, UniqueId = _nccl()
    box = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    uid = UniqueId()
    ctypes.memmove(ctypes.addressof(uid), box[0], 128)
    comm = ctypes.c_void_p()
    assert nccl.ncclCommInitRank(ctypes.byref(comm), world, uid, rank) == 0
    model.attach_nccl_comm(comm.value, world)
    loss2, grad2 = model.loss_and_gradient(xs, ys, 64)
    np.save(f"{args.out}.grad2.{rank}.npy", np.concatenate([[loss2], grad2]))

    opt = AdamWOptions(learning_rate=1e-3, weight_decay=0.1)
    losses = []
    for step in range(3):
        x, y, n = dp_batch(GPU_CFG["vocab_size"], 8 * world, 64, world, seed=10 + step)
        losses.append(model.train_batch_with_optimizer(x[rank * n:(rank + 1) * n], y[rank * n:(rank + 1) * n],
                                                       64, opt))
    np.save(f"{args.out}.{rank}.npy", model.parameters())
    np.save(f"{args.out}.loss.{rank}.npy", np.array(losses))
    model.detach_nccl()
    model.close()
    assert nccl.ncclCommDestroy(comm) == 0
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
