"""The run directory that ``grok-simple train`` writes, from the GPU model.

Host-side mirror of ``src/bin/mesh-gpt/simple.rs:242-652`` (the training loop
and its records) and ``src/bin/mesh-gpt/grokking.rs:511-531,642-672`` (stop
rule, epoch budget, dataset files): ``run.txt`` (metadata written at the
start with ``status=running`` and completed at the end), ``loss.csv`` (one
line per report: losses and accuracies of both complete splits, the weight
norm, the learning rate, elapsed seconds), ``model.bin`` and
``initial-model.bin`` (raw little-endian f32 parameters), ``predictions.csv``
(every equation of both splits under the final weights), ``equations.csv``
and ``symbols.csv``.  Field names, order and number formats follow the
reference's writers; numbers that Rust prints with ``Display`` are printed
as the shortest decimal that round-trips, without an exponent.
"""

import os
import time

import numpy as np

from .data import EquationDataset, EquationSampler
from .gpt import AdamWOptions
from .simple import GpuSimpleModel, SimpleConfig, row_metrics, warmed

MESH_FAMILY = ("mesh-mlp", "full-mesh-mlp", "shared-neighbor-mesh-mlp", "tied-concat-mesh-mlp", "residual-mesh-mlp",
               "tied-concat-residual-mesh-mlp", "tied-rotary-residual-mesh-mlp")
RESIDUAL_MESH = ("residual-mesh-mlp", "tied-concat-residual-mesh-mlp", "tied-rotary-residual-mesh-mlp")
LOSS_HEADER = ("step,training_examples_seen,completed_epochs,examples_in_partial_epoch,train_cross_entropy,"
               "validation_cross_entropy,train_accuracy,validation_accuracy,weight_l2,learning_rate,elapsed_seconds")
PREDICTIONS_HEADER = "split,a,b,answer,prediction,correct,cross_entropy"


def rust_float(x, f32: bool = True) -> str:
    """A float as Rust's ``Display`` prints it: the shortest decimal that
    reads back as the same f32 (or f64), positional, no trailing ``.0``."""
    v = np.float32(x) if f32 else np.float64(x)
    return np.format_float_positional(v, unique=True, trim="-")


def family(c: SimpleConfig) -> str:
    """Groups runs whose size alone varies (simple.rs ``family``)."""
    if c.architecture == "bilinear":
        return f"{c.architecture}-{c.encoding}"
    if c.architecture in MESH_FAMILY:
        rate = "" if c.mesh_learning_rate_multiplier == 1 else f"-mesh-rate-{c.mesh_learning_rate_multiplier}"
        return (f"{c.architecture}-{c.connectivity}{'-tied' if c.tied_mesh else ''}-{c.activation}-{c.encoding}"
                f"{rate}{'-activated-output' if c.mesh_output_activation else ''}")
    if c.decay_factors != 2:
        return f"{c.architecture}-{c.activation}-{c.encoding}-decay-factors-{c.decay_factors}"
    return f"{c.architecture}-{c.activation}-{c.encoding}"


def mesh_stride(c: SimpleConfig, layer: int) -> int:
    """Distance to a unit's second parent (src/simple/mod.rs:179-186)."""
    if c.connectivity == "own":
        return 0
    if c.connectivity == "neighbor":
        return 1
    return 1 << (layer % (c.width.bit_length() - 1))


def mesh_layers(c: SimpleConfig) -> int:
    a = c.architecture
    if a == "full-mesh-mlp":
        return c.depth + 1
    if a == "shared-neighbor-mesh-mlp":
        return c.embedding_mesh_depth + c.depth
    if a in ("mesh-mlp", "tied-concat-mesh-mlp"):
        return max(c.depth - 1, 0)
    if a in RESIDUAL_MESH:
        return c.depth * c.mesh_depth
    return 0


def _full_mesh_fields(c: SimpleConfig):
    """Input bits each full-mesh logit can depend on (src/simple/mod.rs:802-816)."""
    n_in = 2 * c.operand_features()
    layers = [(n_in, c.width, c.operand_features())]
    layers += [(c.width, c.width, mesh_stride(c, layer - 1)) for layer in range(1, c.depth)]
    layers.append((c.width, c.modulus, mesh_stride(c, c.depth - 1)))
    fields = [1 << bit for bit in range(n_in)]
    for inputs, outputs, stride in layers:
        new = []
        for o in range(outputs):
            first = o * inputs // outputs
            new.append(fields[first] | fields[(first + stride) % inputs])
        fields = new
    return [bin(f).count("1") for f in fields]


def _shared_neighbor_coverage(c: SimpleConfig):
    """Input features routed to each readout class (src/simple/mod.rs:822-865)."""
    w, m = c.width, c.modulus

    def combine(fields, stride):
        return [fields[i] | fields[(i + stride) % w] for i in range(w)]
    a, b = [0] * w, [0] * w
    for cls in range(m):
        a[cls] |= 1 << cls
        b[cls] |= 1 << (m + cls)
    for _ in range(c.embedding_mesh_depth):
        a, b = combine(a, 1), combine(b, 1)
    fields = [a[i] | b[i + 1 if i % 2 == 0 else i - 1] for i in range(w)]
    for layer in range(c.depth):
        fields = combine(fields, mesh_stride(c, layer))
    for _ in range(c.embedding_mesh_depth):
        fields = combine(fields, w - 1)
    return [bin(f).count("1") for f in fields[:m]]


def run_metadata(c: SimpleConfig, operation: str, train_fraction: float, n_train: int, n_valid: int, seed: int,
                 init_seed: int, optimizer: AdamWOptions, batch: int, steps: int, report_every: int,
                 epochs=None, stop_validation_accuracy=None) -> str:
    """``run.txt`` as the run starts (simple.rs:287-545, ``status=running``)."""
    a = c.architecture
    mesh = a in MESH_FAMILY
    none = "none"
    normalization = ("pre_rmsnorm_blocks_and_final"
                     if a in ("residual-mlp", "residual-mesh-mlp", "tied-concat-residual-mesh-mlp",
                              "tied-rotary-residual-mesh-mlp", "tied-rotary-residual-dense-mlp",
                              "shared-neighbor-mesh-mlp") else none)
    initialization = {
        "mesh-mlp": "uniform_fan_in_dense_identity_mesh",
        "residual-mesh-mlp": "uniform_fan_in_dense_identity_mesh",
        "tied-concat-mesh-mlp": "uniform_fan_in_embedding_projection_identity_mesh",
        "tied-concat-residual-mesh-mlp": "uniform_fan_in_embedding_projection_identity_mesh",
        "tied-rotary-residual-mesh-mlp": "uniform_fan_in_embedding_identity_mesh",
        "tied-rotary-residual-dense-mlp": "uniform_fan_in_embedding_kaiming_normal_relu_gain_dense",
        "full-mesh-mlp": ("kaiming_normal_two_parent_zero_bias" if c.full_mesh_initialization == "kaiming"
                          else "kaiming_normal_input_output_identity_hidden_zero_bias"),
        "shared-neighbor-mesh-mlp": "near_identity_gaussian_shared_neighbor_kaiming_or_identity_core",
    }.get(a, "uniform_fan_in")
    if a == "mesh-mlp" and c.tied_mesh:
        checkpoint = "raw_f32_le_dense_layers_then_one_tied_mesh_layer"
    else:
        checkpoint = {
            "mesh-mlp": "raw_f32_le_dense_layers_then_mesh_layers",
            "residual-mesh-mlp": "raw_f32_le_dense_layers_then_mesh_layers",
            "tied-concat-mesh-mlp": "raw_f32_le_shared_embedding_projection_then_stored_mesh_layers",
            "tied-concat-residual-mesh-mlp": "raw_f32_le_shared_embedding_projection_then_stored_mesh_layers",
            "tied-rotary-residual-mesh-mlp": "raw_f32_le_shared_embedding_then_mesh_layers",
            "tied-rotary-residual-dense-mlp": "raw_f32_le_shared_embedding_then_dense_branches",
            "full-mesh-mlp": "raw_f32_le_two_parent_layers_unit_weights_then_bias",
            "shared-neighbor-mesh-mlp": "raw_f32_le_shared_neighbor_layers_then_two_parent_core",
        }.get(a, "raw_f32_le_layer_order")
    parameters = c.parameter_count()
    lines = [
        "paper=https://arxiv.org/abs/2201.02177v1", "status=running", "model=simple", f"family={family(c)}",
        f"architecture={a}", f"activation={none if a == 'bilinear' else c.activation}", f"encoding={c.encoding}",
        f"operation={operation}", f"modulus={c.modulus}", f"train_fraction={rust_float(train_fraction, False)}",
        f"training_equations={n_train}", f"validation_equations={n_valid}", f"seed={seed}",
        f"init_seed={init_seed}", "inputs=residue_values", "abstract_symbol_permutation=false", "loss=answer_only",
        f"output_classes={c.modulus}", f"input_features={2 * c.operand_features()}", f"width={c.width}",
        f"depth={none if a == 'bilinear' else c.depth}",
        f"expansion={c.expansion if a == 'residual-mlp' else none}",
        f"connectivity={c.connectivity if mesh else none}", f"mesh_layers={mesh_layers(c)}",
        f"tied_mesh={str(bool(c.tied_mesh)).lower() if mesh else none}", f"parameters={parameters}",
        f"all_parameters={parameters}", f"normalization={normalization}", f"initialization={initialization}",
        f"bias={'true' if a in ('full-mesh-mlp', 'shared-neighbor-mesh-mlp') else 'false'}", "betas=0.9,0.98",
        "epsilon=1e-8", f"learning_rate={rust_float(optimizer.learning_rate)}",
        f"mesh_learning_rate_multiplier={c.mesh_learning_rate_multiplier if mesh else none}",
        f"weight_decay={rust_float(optimizer.weight_decay)}", f"decay_factors={c.decay_factors}",
        "warmup_steps=10", f"batch={batch}", f"steps={steps}", f"report_every={report_every}",
        "evaluation=complete_splits", f"checkpoint={checkpoint}",
        f"requested_epochs={none if epochs is None else epochs}",
        f"steps_per_epoch={-(-n_train // batch)}", "epoch_definition=one_visit_to_every_training_equation",
        "epoch_tail=short_batch",
        f"stop_validation_accuracy={none if stop_validation_accuracy is None else rust_float(stop_validation_accuracy, False)}",
    ]
    if a == "tied-rotary-residual-dense-mlp":
        lines += ["dense_embedding_initialization=uniform-fan-in",
                  f"embedding_initial_variance={1.0 / (3 * c.modulus):.12f}",
                  "embedding_scale_constraint=initialization_only",
                  "dense_branch_initialization=kaiming_normal_variance_2_over_width", "dense_residual=true"]
    if a == "full-mesh-mlp":
        fields = _full_mesh_fields(c)
        lines += ["max_activation_parents=2", "input_projection=two_parent", "readout=two_parent",
                  f"mesh_initialization={c.full_mesh_initialization}",
                  f"readout_min_input_features={min(fields)}", f"readout_max_input_features={max(fields)}"]
    if a == "shared-neighbor-mesh-mlp":
        cover = _shared_neighbor_coverage(c)
        ratio = 0.1 / np.sqrt(c.embedding_mesh_depth)
        lines += ["max_activation_parents=2", f"embedding_mesh_depth={c.embedding_mesh_depth}",
                  "embedding_connectivity=neighbor", "embedding_weight_sharing=a,b,transposed_readout",
                  "operand_rotation=pairwise_b_plus_90_degrees", "readout=transposed_neighbor_chain",
                  f"mesh_initialization={c.full_mesh_initialization}",
                  "shared_embedding_initialization=near-identity",
                  "embedding_initialization=identity_plus_gaussian_mixing_std_0.1_over_sqrt_depth",
                  f"embedding_mixing_strength={ratio:.12f}", "embedding_column_norm_target=none",
                  "embedding_column_normalization=none",
                  "core_structure=pre_rmsnorm_mesh_activation_residual", "final_rmsnorm=true",
                  "rmsnorm_epsilon=1e-5", "input_coverage_excludes_norm_statistics=true",
                  f"readout_min_input_features={min(cover)}", f"readout_max_input_features={max(cover)}"]
    if a in RESIDUAL_MESH:
        lines += [f"mesh_depth={c.mesh_depth}", f"mesh_output_activation={str(bool(c.mesh_output_activation)).lower()}",
                  f"pointwise_activations_per_branch={c.mesh_depth - 1 + int(bool(c.mesh_output_activation))}"]
        if a == "tied-rotary-residual-mesh-mlp":
            lines += ["operand_rotation=pairwise_b_plus_90_degrees", "embedding_roles=a,b,readout"]
    return "\n".join(lines) + "\n"


def run_completion(elapsed: float, stop_reason: str, step: int, trained: int, n_train: int, thresholds) -> str:
    """The lines appended to ``run.txt`` when training ends (simple.rs:625-640)."""
    observed = ["not_reached" if t is None else str(t) for t in thresholds]
    return (f"elapsed_seconds={elapsed:.6f}\nstop_reason={stop_reason}\ncompleted_steps={step}\n"
            f"training_examples_seen={trained}\ncompleted_epochs={trained // n_train}\n"
            f"examples_in_partial_epoch={trained % n_train}\nfirst_recorded_train_99_step={observed[0]}\n"
            f"first_recorded_validation_99_step={observed[1]}\n")


def loss_line(step: int, trained: int, n_train: int, train_ce: float, valid_ce: float, train_acc: float,
              valid_acc: float, weight_l2: float, learning_rate: float, elapsed: float) -> str:
    """One ``loss.csv`` line (simple.rs:781-792); the learning rate is the
    f32 value printed to 9 decimals."""
    return (f"{step},{trained},{trained // n_train},{trained % n_train},{train_ce:.9f},{valid_ce:.9f},"
            f"{train_acc:.9f},{valid_acc:.9f},{weight_l2:.9f},{float(np.float32(learning_rate)):.9f},{elapsed:.6f}")


def write_dataset(directory: str, dataset: EquationDataset) -> None:
    """``equations.csv`` and ``symbols.csv`` (grokking.rs:642-672)."""
    p, tok = dataset.modulus, dataset.residue_tokens
    with open(os.path.join(directory, "equations.csv"), "w") as f:
        f.write("split,pair_id,a,b,answer,input_a_id,operator_id,input_b_id,equals_id,target_id\n")
        for validation in (False, True):
            name = "validation" if validation else "train"
            for a, b, ans in dataset.split(validation):
                f.write(f"{name},{a * p + b},{a},{b},{ans},{tok[a]},{p},{tok[b]},{p + 1},{tok[ans]}\n")
    label = {int(t): str(r) for r, t in enumerate(tok)}
    label[p], label[p + 1] = dataset.operation, "="
    with open(os.path.join(directory, "symbols.csv"), "w") as f:
        f.write("token_id,symbol\n")
        for t in range(p + 2):
            f.write(f"{t},{label[t]}\n")


def train_run(config: SimpleConfig, output: str, operation: str = "div", train_fraction: float = 0.5,
              seed: int = 11, init_seed=None, steps: int = 10000, batch=None, report_every: int = 1000,
              optimizer: AdamWOptions = None, epochs=None, stop_validation_accuracy=None, device: int = 0):
    """``grok-simple train`` on the GPU: writes the run directory and returns
    the recorded (step, train CE, validation CE, train accuracy, validation
    accuracy, weight L2) tuples."""
    if steps == 0 or report_every == 0:
        raise ValueError("steps and report interval must be positive")
    if stop_validation_accuracy is not None and not 0.0 <= stop_validation_accuracy <= 1.0:
        raise ValueError("stop validation accuracy must be in 0..=1")
    optimizer = optimizer or AdamWOptions(learning_rate=1e-3, weight_decay=1.0, beta1=0.9, beta2=0.98)
    config.validate()
    dataset = EquationDataset(config.modulus, operation, train_fraction, seed)
    n_train, n_valid = len(dataset.split(False)), len(dataset.split(True))
    batch = batch if batch is not None else min(512, n_train // 2)
    if not 1 <= batch <= n_train:
        raise ValueError("invalid equation minibatch size")
    if epochs is not None:
        if epochs == 0:
            raise ValueError("epochs, training examples, and batch size must be positive")
        steps = epochs * -(-n_train // batch)
    steps_per_epoch = -(-n_train // batch)
    init_seed = seed if init_seed is None else init_seed
    model = GpuSimpleModel(device, config, init_seed)
    tables = [model.upload_table(*config.encode(dataset.split(v))) for v in (False, True)]
    os.makedirs(output, exist_ok=True)
    write_dataset(output, dataset)
    run_path = os.path.join(output, "run.txt")
    with open(run_path, "w") as f:
        f.write(run_metadata(config, operation, train_fraction, n_train, n_valid, seed, init_seed, optimizer, batch,
                             steps, report_every, epochs, stop_validation_accuracy))
    history = open(os.path.join(output, "loss.csv"), "w")
    history.write(LOSS_HEADER + "\n")
    thresholds = [None, None]
    records = []
    start = time.perf_counter()

    def record(step, trained, lr):
        evaluations = model.evaluate(*tables)
        ces, accs = [], []
        for (logits, preds), table in zip(evaluations, tables):
            ce, _ = row_metrics(logits, table.targets)
            ces.append(float(ce.sum() / table.rows))
            accs.append(float((preds == table.targets).sum()) / table.rows)
        params = model.pinned_parameters()
        norm = float(np.sqrt((params.astype(np.float64) ** 2).sum()))
        elapsed = time.perf_counter() - start
        for i in (0, 1):
            if accs[i] >= 0.99 and thresholds[i] is None:
                thresholds[i] = step
        history.write(loss_line(step, trained, n_train, ces[0], ces[1], accs[0], accs[1], norm, lr, elapsed) + "\n")
        history.flush()
        params.tofile(os.path.join(output, "model.bin"))
        if step == 0:
            params.tofile(os.path.join(output, "initial-model.bin"))
        model.reuse(params)
        for logits, _ in evaluations:
            model.reuse(logits)
        records.append((step, ces[0], ces[1], accs[0], accs[1], norm))
        return accs[1]

    def reached(valid_acc):
        return stop_validation_accuracy is not None and valid_acc >= stop_validation_accuracy

    sampler = EquationSampler(n_train, seed)
    valid_acc = record(0, 0, 0.0)
    step = trained = 0
    epoch, offsets, batches = [], [], None
    while step < steps and not reached(valid_acc):
        if not epoch:
            epoch = sampler.take(batch, min(steps_per_epoch, steps - step))
            offsets = np.cumsum([0] + [len(e) for e in epoch])[:-1].tolist()
            batches = model.upload_batches(tables[0], np.concatenate(epoch))
        rows, offset = len(epoch.pop(0)), offsets.pop(0)
        step += 1
        opt = warmed(optimizer, step)
        model.train_batch(tables[0], batches, offset, rows, opt)
        trained += rows
        if step % report_every == 0 or step == steps:
            valid_acc = record(step, trained, opt.learning_rate)
    history.close()
    stop_reason = "validation_accuracy" if reached(valid_acc) else "update_budget"
    with open(os.path.join(output, "predictions.csv"), "w") as f:
        f.write(PREDICTIONS_HEADER + "\n")
        for (logits, preds), table, validation in zip(model.evaluate(*tables), tables, (False, True)):
            ce, _ = row_metrics(logits, table.targets)
            name = "validation" if validation else "train"
            for (a, b, ans), p, loss in zip(dataset.split(validation), preds, ce):
                f.write(f"{name},{a},{b},{ans},{p},{int(p == ans)},{loss:.9f}\n")
    text = open(run_path).read().replace("status=running", "status=complete")
    with open(run_path, "w") as f:
        f.write(text + run_completion(time.perf_counter() - start, stop_reason, step, trained, n_train, thresholds))
    model.close()
    return records
