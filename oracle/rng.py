"""SplitMix64 generator of the reference (test infrastructure only).

Restates ``src/mesh.rs:256-288`` (``Random``): ``unit()`` keeps the top 24
bits of the next 64-bit output and divides by 2^24 in f32; ``index(bound)``
rejects the low ``2^64 mod bound`` outputs so the result has no modulo bias.
"""

import numpy as np

MASK = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15


class Random:
    """``src/mesh.rs:256-288``."""

    def __init__(self, seed: int):
        self.state = seed & MASK

    def next_u64(self) -> int:
        # src/mesh.rs:267-274
        self.state = (self.state + GOLDEN) & MASK
        bits = self.state
        bits = ((bits ^ (bits >> 30)) * 0xBF58476D1CE4E5B9) & MASK
        bits = ((bits ^ (bits >> 27)) * 0x94D049BB133111EB) & MASK
        bits ^= bits >> 31
        return bits

    def unit(self) -> np.float32:
        # src/mesh.rs:263-265: ((next >> 40) as u32) as f32 / 16_777_216.0
        return np.float32(self.next_u64() >> 40) / np.float32(16777216.0)

    def index(self, bound: int) -> int:
        # src/mesh.rs:277-287
        assert bound > 0
        threshold = ((-bound) & MASK) % bound
        while True:
            bits = self.next_u64()
            if bits >= threshold:
                return bits % bound


def shuffle(values: list, random: Random) -> None:
    """Fisher-Yates from the back, ``src/gpt/grokking.rs:267-271``."""
    for end in range(len(values) - 1, 0, -1):
        j = random.index(end + 1)
        values[end], values[j] = values[j], values[end]
