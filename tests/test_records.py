"""grok-simple run records (run.txt, loss.csv) against the reference's
archived runs (tests/golden/grok_runs.json, extracted by
tests/golden/extract_grok_runs.py): the metadata that the record writer
derives from a configuration equals the archived file on every field both
write, and loss.csv lines print in the archived format.  Host only."""

import json
import os

import numpy as np
import pytest

from grokking_abmod_b200.gpt import AdamWOptions
from grokking_abmod_b200.records import LOSS_HEADER, loss_line, run_completion, run_metadata, rust_float
from grokking_abmod_b200.simple import SimpleConfig

RUNS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "grok_runs.json")))["runs"]
# fields describing how a run ended, not its configuration
OUTCOME = {"status", "elapsed_seconds", "stop_reason", "completed_steps", "training_examples_seen",
           "completed_epochs", "examples_in_partial_epoch", "first_recorded_train_99_step",
           "first_recorded_validation_99_step"}


def _kv(text):
    return dict(line.split("=", 1) for line in text.splitlines() if "=" in line)


def _config(kv):
    none = lambda key, default: default if kv.get(key, "none") == "none" else kv[key]  # noqa: E731
    arch = kv["architecture"]
    return SimpleConfig(
        architecture=arch, activation=none("activation", "relu"), modulus=int(kv["modulus"]),
        width=int(kv["width"]), depth=int(none("depth", 1)), connectivity=none("connectivity", "neighbor"),
        embedding_mesh_depth=int(kv.get("embedding_mesh_depth", 4)),
        full_mesh_initialization=kv.get("mesh_initialization", "kaiming"),
        mesh_learning_rate_multiplier=int(none("mesh_learning_rate_multiplier", 1)),
        expansion=int(none("expansion", 4)), mesh_depth=int(kv.get("mesh_depth", 4)),
        mesh_output_activation=kv.get("mesh_output_activation") == "true", tied_mesh=kv.get("tied_mesh") == "true",
        encoding=kv["encoding"], decay_factors=int(kv["decay_factors"]))


def _metadata(kv):
    opt = AdamWOptions(learning_rate=float(kv["learning_rate"]), weight_decay=float(kv["weight_decay"]), beta1=0.9,
                       beta2=0.98)
    epochs = None if kv["requested_epochs"] == "none" else int(kv["requested_epochs"])
    stop = None if kv["stop_validation_accuracy"] == "none" else float(kv["stop_validation_accuracy"])
    return _kv(run_metadata(_config(kv), kv["operation"], float(kv["train_fraction"]), int(kv["training_equations"]),
                            int(kv["validation_equations"]), int(kv["seed"]), int(kv["init_seed"]), opt,
                            int(kv["batch"]), int(kv["steps"]), int(kv["report_every"]), epochs, stop))


@pytest.mark.parametrize("run", RUNS, ids=lambda r: r["source"].split("/")[2] + "/" + r["source"].split("/")[-2])
def test_run_metadata_matches_archived_runs(run):
    want = _kv(run["run_txt"])
    got = _metadata(want)
    assert got["status"] == "running"
    missing = sorted(k for k in want if k not in got and k not in OUTCOME)
    assert not missing, f"fields the writer lacks: {missing}"
    differ = {k: (want[k], got[k]) for k in want if k in got and k not in OUTCOME and want[k] != got[k]}
    assert not differ, differ


def test_loss_lines_print_in_the_archived_format():
    for run in RUNS:
        head = run["loss_csv_head"]
        if not head:
            continue
        assert head[0] == LOSS_HEADER
        n_train = int(_kv(run["run_txt"])["training_equations"])
        for line in head[1:]:
            f = line.split(",")
            got = loss_line(int(f[0]), int(f[1]), n_train, *(float(x) for x in f[4:10]), float(f[10]))
            assert got == line, (got, line)


def test_run_completion_and_float_printing():
    assert rust_float(0.001) == "0.001" and rust_float(1.0) == "1" and rust_float(0.5, False) == "0.5"
    assert rust_float(1e-8) == "0.00000001"
    text = run_completion(12.5, "update_budget", 20, 9312, 4656, [None, 20])
    assert _kv(text) == {"elapsed_seconds": "12.500000", "stop_reason": "update_budget", "completed_steps": "20",
                         "training_examples_seen": "9312", "completed_epochs": "2", "examples_in_partial_epoch": "0",
                         "first_recorded_train_99_step": "not_reached", "first_recorded_validation_99_step": "20"}
    assert np.float32(float("0.001000000")) == np.float32(0.001)


@pytest.mark.gpu
def test_train_run_writes_the_archived_records(tmp_path):
    """grok-simple train for 10 updates of the archived cfg1 run (mesh-mlp
    W384 depth 5, butterfly, seed 11, batch 512, report every 10): the step-0
    and step-10 loss.csv lines match the archive (CE to 1e-6 / 2e-5, the
    weight norm to 1e-9 / 2e-5, accuracies to one row), run.txt agrees on every
    configuration field, and every file of the run directory is written."""
    from grokking_abmod_b200.records import PREDICTIONS_HEADER, train_run
    run = next(r for r in RUNS if "000018-mesh-mlp-w384-d5-s11" in r["source"])
    want = _kv(run["run_txt"])
    config = _config(want)
    opt = AdamWOptions(learning_rate=float(want["learning_rate"]), weight_decay=float(want["weight_decay"]),
                       beta1=0.9, beta2=0.98)
    out = str(tmp_path / "run")
    train_run(config, out, operation=want["operation"], train_fraction=float(want["train_fraction"]),
              seed=int(want["seed"]), steps=10, batch=int(want["batch"]), report_every=10, optimizer=opt,
              stop_validation_accuracy=float(want["stop_validation_accuracy"]))
    for name in ("run.txt", "loss.csv", "model.bin", "initial-model.bin", "predictions.csv", "equations.csv",
                 "symbols.csv"):
        assert os.path.exists(os.path.join(out, name)), name
    got = _kv(open(os.path.join(out, "run.txt")).read())
    assert got["status"] == "complete" and got["completed_steps"] == "10" and got["training_examples_seen"] == "4656"
    for k in want:
        if k not in OUTCOME and k not in ("steps", "requested_epochs"):
            assert got[k] == want[k], (k, got[k], want[k])
    lines = open(os.path.join(out, "loss.csv")).read().splitlines()
    assert lines[0] == LOSS_HEADER and len(lines) == 3
    for line, ref, tol, norm_tol in zip(lines[1:], run["loss_csv_head"][1:], (1e-6, 2e-5), (1e-9, 2e-5)):
        g, w = line.split(","), ref.split(",")
        assert g[:4] == w[:4] and g[9] == w[9]
        for i in (4, 5):
            assert abs(float(g[i]) - float(w[i])) <= tol * float(w[i]), (i, g[i], w[i])
        for i in (6, 7):
            assert abs(float(g[i]) - float(w[i])) <= 1.5 / 4656, (i, g[i], w[i])
        assert abs(float(g[8]) - float(w[8])) <= norm_tol * float(w[8]), (g[8], w[8])
    params = np.fromfile(os.path.join(out, "model.bin"), dtype="<f4")
    assert params.size == config.parameter_count()
    pred = open(os.path.join(out, "predictions.csv")).read().splitlines()
    assert pred[0] == PREDICTIONS_HEADER and len(pred) == 1 + 9312
