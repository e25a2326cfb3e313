"""Data parallelism: 2 ranks as separate processes.

CPU (gloo): the host-side DP plumbing the bench relies on.  GPU (2 devices,
NCCL inside the library): ranks stay bitwise identical and match one GPU
training on the concatenated batch (gradient average of equal halves)."""

import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _launch(device, out, nproc=2):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", "--master-port=29533", os.path.join(HERE, "dp", "dp_worker.py"),
           "--device", device, "--out", out]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    return subprocess.run(["timeout", "-k", "30", "300"] + cmd, capture_output=True, text=True, env=env)


def test_dp_host_plumbing_over_gloo(tmp_path):
    res = _launch("cpu", str(tmp_path / "flag"))
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    for r in range(2):
        assert np.load(str(tmp_path / f"flag.{r}.npy"))[0] == 1


@pytest.mark.gpu
def test_dp_ranks_identical_and_match_single_gpu(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _launch("cuda", str(tmp_path / "p"))
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    p0, p1 = (np.load(str(tmp_path / f"p.{r}.npy")) for r in range(2))
    assert p0.tobytes() == p1.tobytes()
    from grokking_abmod_b200 import AdamWOptions, GptConfig, MeshGpt
    from grokking_abmod_b200.data import zipf_batch
    model = MeshGpt(0, GptConfig(vocab_size=64, context=64, width=256, heads=4, layers=2), 7)
    for step in range(3):
        x, y = zipf_batch(11, 0, step, 16, 64)
        model.train_batch_with_optimizer(x, y, 64, AdamWOptions(learning_rate=1e-3, weight_decay=0.1))
    single = model.parameters()
    diff = np.abs(single - p0)
    # Gradients differ from the single-GPU ones only by summation order; AdamW
    # can turn a sign flip of a near-zero gradient into a full lr step, so
    # allow a tiny fraction of such parameters (bounded by 2 * lr * steps).
    assert np.mean(diff > 1e-5 * (1 + np.abs(single))) < 1e-3
    assert diff.max() <= 2 * 1e-3 * 3
