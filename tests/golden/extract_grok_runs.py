"""Builds tests/golden/grok_runs.json from the reference's archived
grok-simple run directories (docs/grokking-results/**/run.txt and the first
lines of loss.csv), for the record-writer tests.

Keeps up to three runs per family of configurations that this build trains
(the default embedding initializations; not the unnormalised shared-Neighbor
ablation, which the current reference no longer builds), plus the three
benchmark runs.

    python tests/golden/extract_grok_runs.py /path/to/reference
"""

import glob
import json
import os
import sys

BENCH = ["rotary-dense-relu/raw/w128-seed11",
         "short-plateau-mesh/raw/000018-mesh-mlp-w384-d5-s11-a01",
         "shared-neighbor/pre-norm/raw/000001-shared-neighbor-mesh-mlp-w128-d64-s11-a01"]


def main(reference):
    root = os.path.join(reference, "docs", "grokking-results")
    picked, per_group = [], {}
    paths = sorted(glob.glob(os.path.join(root, "**", "run.txt"), recursive=True))
    bench = {os.path.join(root, b, "run.txt") for b in BENCH}
    for path in sorted(bench) + [p for p in paths if p not in bench]:
        text = open(path).read()
        kv = dict(line.split("=", 1) for line in text.splitlines() if "=" in line)
        if kv.get("model") != "simple" or "shared_embedding_initialization" in kv:
            continue
        if kv.get("dense_embedding_initialization", "uniform-fan-in") != "uniform-fan-in":
            continue
        if kv["architecture"] == "shared-neighbor-mesh-mlp" and kv.get("normalization") == "none":
            continue  # an unnormalised ablation of an earlier version; the current source always pre-normalises
        group = (kv["architecture"], kv.get("encoding"), kv.get("connectivity"), kv.get("tied_mesh"),
                 kv.get("mesh_output_activation"), kv.get("mesh_initialization"))
        if path not in bench and per_group.get(group, 0) >= 3:
            continue
        per_group[group] = per_group.get(group, 0) + 1
        loss_path = os.path.join(os.path.dirname(path), "loss.csv")
        loss = open(loss_path).read().splitlines()[:3] if os.path.exists(loss_path) else []
        picked.append({"source": os.path.relpath(path, reference), "run_txt": text, "loss_csv_head": loss})
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "grok_runs.json")
    json.dump({"runs": picked}, open(out, "w"), indent=1)
    print(f"{len(picked)} runs -> {out}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
