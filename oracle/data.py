"""Data generators of the hot path (test infrastructure only).

* Modular-arithmetic equation tables, seeded split, abstract-symbol permutation,
  answer-only batches and the epoch sampler: ``src/gpt/grokking.rs:13-306``.
* The Zipf(1.1) synthetic token stream for the Mesh GPT benchmark shapes.  The
  reference has no Zipf sampler; the harness defines one on the reference's
  ``Random`` (``src/mesh.rs:256-288``): u = unit(); token = smallest rank k
  (1-based) with cdf[k] > u, id k-1, cdf an f64 prefix sum of k^-s / sum.
"""

import numpy as np

from .rng import Random, shuffle

IGNORE_TARGET = 0xFFFFFFFF  # src/gpt/mod.rs:26
EQUATION_CONTEXT = 4  # src/gpt/grokking.rs:9
MAX_ROWS = 131072  # src/gpt/mod.rs:30

OPERATIONS = ["add", "mul", "sub", "div", "mixed", "square-sum", "quadratic",
              "quadratic-linear", "cubic-product", "cubic-mixed"]


def inverse(value: int, modulus: int) -> int:
    """Fermat inverse by square-and-multiply, ``src/gpt/grokking.rs:95-107``."""
    result, base, exponent = 1, value, modulus - 2
    while exponent:
        if exponent % 2 == 1:
            result = result * base % modulus
        base = base * base % modulus
        exponent //= 2
    return result


def apply(op: str, a: int, b: int, p: int) -> int:
    """``src/gpt/grokking.rs:55-67``."""
    if op == "add":
        return (a + b) % p
    if op == "mul":
        return a * b % p
    if op == "sub":
        return (a + p - b) % p
    if op == "div":
        return a * inverse(b, p) % p
    if op == "mixed":
        return a * inverse(b, p) % p if b % 2 == 1 else (a + p - b) % p
    if op == "square-sum":
        return (a * a + b * b) % p
    if op == "quadratic":
        return (a * a + a * b + b * b) % p
    if op == "quadratic-linear":
        return (a * a + a * b + b * b + a) % p
    if op == "cubic-product":
        return (a * a * a + a * b) % p
    if op == "cubic-mixed":
        return (a * a * a + a * b * b + b) % p
    raise ValueError(f"unknown operation: {op}")


def residue_permutation(modulus: int, seed: int) -> list:
    """``src/gpt/grokking.rs:260-265``."""
    tokens = list(range(modulus))
    shuffle(tokens, Random(seed ^ 0x73796D626F6C7301))
    return tokens


class EquationDataset:
    """``src/gpt/grokking.rs:128-186`` (seeded split of the full table)."""

    def __init__(self, modulus: int, op: str, train_fraction: float, seed: int):
        if modulus < 2 or modulus > 254 or any(modulus % d == 0 for d in range(2, modulus)):
            raise ValueError("modulus must be a prime in 2..254")
        if not (0.0 < train_fraction < 1.0):
            raise ValueError("train fraction must be strictly between 0 and 1")
        self.modulus, self.op = modulus, op
        self.residue_tokens = residue_permutation(modulus, seed)
        first_b = 1 if op == "div" else 0
        equations = [(a, b, apply(op, a, b, modulus))
                     for a in range(modulus) for b in range(first_b, modulus)]
        split = int(np.floor(len(equations) * train_fraction))
        if split < 2 or split >= len(equations):
            raise ValueError("split needs two training and one validation equation")
        shuffle(equations, Random(seed ^ 0x73706C6974730002))
        self.training = equations[:split]
        self.validation = equations[split:]

    @property
    def vocab_size(self) -> int:
        return self.modulus + 2

    def split(self, validation: bool):
        return self.validation if validation else self.training

    def batch(self, validation: bool, indices):
        """a, op, b, '=' inputs with only the answer supervised (``:228-257``)."""
        rows = self.split(validation)
        inputs, targets = [], []
        p = self.modulus
        for i in indices:
            a, b, ans = rows[i]
            inputs += [self.residue_tokens[a], p, self.residue_tokens[b], p + 1]
            targets += [IGNORE_TARGET, IGNORE_TARGET, IGNORE_TARGET, self.residue_tokens[ans]]
        return np.array(inputs, dtype=np.uint32), np.array(targets, dtype=np.uint32)


class EquationSampler:
    """Shuffled epochs without replacement, ``src/gpt/grokking.rs:274-306``."""

    def __init__(self, examples: int, seed: int):
        self.indices = list(range(examples))
        self.random = Random(seed ^ 0x6261746368657303)
        self.position = 0
        shuffle(self.indices, self.random)

    def sample(self, batch: int):
        if batch == 0 or batch > len(self.indices):
            raise ValueError("invalid equation minibatch size")
        if self.position == len(self.indices):
            shuffle(self.indices, self.random)
            self.position = 0
        start = self.position
        self.position = min(start + batch, len(self.indices))
        return self.indices[start:self.position]


def warmed_learning_rate(learning_rate: float, step: int) -> np.float32:
    """10-step linear warmup in f32, ``src/bin/mesh-gpt/grokking.rs:524-527``."""
    return np.float32(learning_rate) * (np.float32(min(step, 10)) / np.float32(10.0))


def zipf_cdf(vocab: int, s: float = 1.1) -> np.ndarray:
    # Sequential prefix sums (no pairwise summation) so a C++ loop reproduces
    # every bit: cdf[k] = (sum_{j<=k} j^-s) / (sum_{j<=V} j^-s).
    weights = [float(k) ** -s for k in range(1, vocab + 1)]
    prefix, total = [], 0.0
    for w in weights:
        total += w
        prefix.append(total)
    return np.array(prefix, dtype=np.float64) / total


def zipf_tokens(seed: int, count: int, vocab: int = 64, s: float = 1.1) -> np.ndarray:
    """``count`` Zipf(s) token ids drawn from ``Random(seed)`` by inverse CDF."""
    cdf = zipf_cdf(vocab, s)
    random = Random(seed)
    out = np.empty(count, dtype=np.uint32)
    for i in range(count):
        u = float(random.unit())
        out[i] = int(np.searchsorted(cdf, u, side="right"))
    return np.minimum(out, vocab - 1)


def zipf_batch(base_seed: int, rank: int, step: int, sequences: int, context: int,
               vocab: int = 64):
    """One benchmark batch: ``sequences`` streams of context+1 tokens drawn from
    seed ``base_seed + 1_000_003*rank + step``; inputs are positions 0..T-1 and
    targets positions 1..T of each stream (all supervised)."""
    seed = (base_seed + 1_000_003 * rank + step) & ((1 << 64) - 1)
    stream = zipf_tokens(seed, sequences * (context + 1), vocab).reshape(sequences, context + 1)
    return stream[:, :-1].reshape(-1).copy(), stream[:, 1:].reshape(-1).copy()
