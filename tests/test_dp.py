"""Data parallelism: 2 ranks as separate processes.

CPU (gloo): the host-side DP plumbing the bench relies on, and the
arithmetic of the exact data-parallel loss (global supervised count first,
then a sum of the ranks' shares) with unequal supervised counts per rank,
against the f64 oracle on the whole batch.  GPU (2 devices, NCCL inside the
library): the loss and gradient with unequal supervised counts match one GPU
on the concatenated batch, through a library-owned and a caller-owned
communicator, and the ranks stay bitwise identical while training."""

import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "dp"))
from dp_worker import GPU_CFG, TINY, dp_batch  # noqa: E402


def _launch(device, out, nproc=2):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", "--master-port=29533", os.path.join(HERE, "dp", "dp_worker.py"),
           "--device", device, "--out", out]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    return subprocess.run(["timeout", "-k", "30", "300"] + cmd, capture_output=True, text=True, env=env)


def test_dp_host_plumbing_and_exact_loss_over_gloo(tmp_path):
    res = _launch("cpu", str(tmp_path / "flag"))
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    for r in range(2):
        assert np.load(str(tmp_path / f"flag.{r}.npy"))[0] == 1
    from oracle.gpt_config import GptConfig
    from oracle.gpt_ref import ReferenceGpt
    x, y, _ = dp_batch(TINY["vocab_size"], 8, 4, 2, seed=1)
    loss, grad = ReferenceGpt(GptConfig(**TINY), seed=7).loss_and_gradient(x, y, 4)
    want = np.concatenate([[loss], grad])
    exact = [np.load(str(tmp_path / f"flag.exact.{r}.npy")) for r in range(2)]
    naive = np.load(str(tmp_path / "flag.naive.0.npy"))
    assert exact[0].tobytes() == exact[1].tobytes()
    assert abs(exact[0][0] - loss) <= 1e-12 * abs(loss)
    assert np.abs(exact[0][1:] - grad).max() <= 1e-12 * np.abs(grad).max()
    # averaging per-rank means weights the answer-only rank's few rows too much
    assert np.abs(naive - want).max() > 1e-3 * np.abs(want).max()


@pytest.mark.gpu
def test_dp_matches_single_gpu_with_unequal_supervised_counts(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _launch("cuda", str(tmp_path / "p"))
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    load = lambda name: [np.load(str(tmp_path / f"p.{name}{r}.npy")) for r in range(2)]  # noqa: E731
    g, g2, p, losses = load("grad."), load("grad2."), load(""), load("loss.")
    for pair in (g, g2, p, losses):
        assert pair[0].tobytes() == pair[1].tobytes(), "ranks diverged"
    assert g[0].tobytes() == g2[0].tobytes(), "caller-owned communicator gave a different result"

    from grokking_abmod_b200 import AdamWOptions, GptConfig, MeshGpt
    model = MeshGpt(0, GptConfig(**GPU_CFG), 7)
    x, y, _ = dp_batch(GPU_CFG["vocab_size"], 16, 64, 2, seed=3)
    loss, grad = model.loss_and_gradient(x, y, 64)
    assert abs(g[0][0] - loss) <= 1e-5 * abs(loss), (g[0][0], loss)
    assert np.abs(g[0][1:] - grad).max() <= 1e-4 * np.abs(grad).max()
    opt = AdamWOptions(learning_rate=1e-3, weight_decay=0.1)
    single_losses = []
    for step in range(3):
        x, y, _ = dp_batch(GPU_CFG["vocab_size"], 16, 64, 2, seed=10 + step)
        single_losses.append(model.train_batch_with_optimizer(x, y, 64, opt))
    assert np.allclose(losses[0], single_losses, rtol=1e-5, atol=0)
    single = model.parameters()
    diff = np.abs(single - p[0])
    # Gradients differ from the single-GPU ones only by summation order; AdamW
    # can turn a sign flip of a near-zero gradient into a full lr step, so
    # allow a tiny fraction of such parameters (bounded by 2 * lr * steps).
    assert np.mean(diff > 1e-5 * (1 + np.abs(single))) < 1e-3
    assert diff.max() <= 2 * 1e-3 * 3
