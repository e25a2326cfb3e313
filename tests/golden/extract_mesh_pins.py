"""Extracts the ``grok_simple_mesh_models`` section of reference_pins.json
from the reference's archived grok-simple runs (``run.txt`` settings and
the ``loss.csv`` lines of step 0 and of a later step).  Run once where the
reference checkout is available; the tests read only the JSON it writes.

    python tests/golden/extract_mesh_pins.py /path/to/reference
"""

import csv
import json
import os
import sys

RUNS = [
    # (archive directory under docs/grokking-results, later step)
    ("residual-mesh/raw/neighbor-w64-b2-m4", 250),
    ("residual-mesh/raw/butterfly-w64-b2-m4", 250),
    ("residual-mesh/raw/butterfly-w64-b4-m4", 250),
    ("residual-mesh/raw/butterfly-w128-b2-m8", 250),
    ("residual-mesh/raw/butterfly-w256-b2-m4", 250),
    ("rotary-neighbor-one-block-128/raw/000001-tied-rotary-residual-mesh-mlp-w128-d1-s11-a01", 10),
    ("rotary-neighbor-one-block-m2-128/raw/000001-tied-rotary-residual-mesh-mlp-w128-d1-s11-a01", 10),
    ("rotary-neighbor-variants/raw/000001-tied-rotary-residual-mesh-mlp-w256-d2-s11-a01", 10),
    ("rotary-neighbor-one-block-m1-square-128/raw/000002-tied-rotary-residual-mesh-mlp-w128-d1-s7-a01", 10),
    ("tied-concat/raw/tied-concat-own-w64-d5-seed7", 250),
]
KEYS = {"architecture": str, "activation": str, "width": int, "depth": int, "connectivity": str,
        "mesh_depth": int, "mesh_output_activation": lambda v: v == "true"}
COLUMNS = ("train_cross_entropy", "validation_cross_entropy", "train_accuracy", "validation_accuracy",
           "weight_l2")


def run(root, path, later):
    base = os.path.join(root, "docs", "grokking-results", path)
    settings = dict(line.strip().split("=", 1) for line in open(os.path.join(base, "run.txt")) if "=" in line)
    config = {k: f(settings[k]) for k, f in KEYS.items() if k in settings}
    if config["architecture"] not in ("residual-mesh-mlp", "tied-concat-residual-mesh-mlp",
                                      "tied-rotary-residual-mesh-mlp"):
        config.pop("mesh_depth", None)
    rows = {int(r["step"]): r for r in csv.DictReader(open(os.path.join(base, "loss.csv")))}
    record = lambda step: [float(rows[step][c]) for c in COLUMNS]
    optimizer = {"operation": settings["operation"], "train_fraction": float(settings["train_fraction"]),
                 "seed": int(settings["seed"]), "batch": int(settings["batch"]),
                 "learning_rate": float(settings["learning_rate"]),
                 "weight_decay": float(settings["weight_decay"]),
                 "beta1": float(settings["betas"].split(",")[0]), "beta2": float(settings["betas"].split(",")[1]),
                 "epsilon": float(settings["epsilon"])}
    return {"config": config, "optimizer": optimizer, "steps": later, "step0": record(0), "later": record(later),
            "source": f"docs/grokking-results/{path}/loss.csv (steps 0 and {later}), run.txt"}


def main():
    root = sys.argv[1]
    pins_path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_pins.json")
    pins = json.load(open(pins_path))
    pins["grok_simple_mesh_models"] = {
        "_about": "Archived grok-simple records of the residual mesh family and the tied-concat mesh MLP "
                  "(one-hot, modulus 97; 10-step warmup; batch 512 with a short epoch tail). Columns: train CE, "
                  "held-out CE, train accuracy, held-out accuracy, weight L2 norm at step 0 and at `steps`.",
        "cases": [run(root, path, later) for path, later in RUNS],
    }
    with open(pins_path, "w") as out:
        json.dump(pins, out, indent=1)
        out.write("\n")


if __name__ == "__main__":
    main()
