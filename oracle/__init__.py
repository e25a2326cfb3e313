"""CPU oracle for the Mesh GPT / grok-simple training hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg (``cpu_baseline`` and ``--impl reference``) may use it, and
there only as the checker or as the timed CPU port of the reference's f64
verify path.

The reference (fxeqxmulfx/grokking_abmod) is Rust + CUDA Oxide and cannot be
built here (no cargo/rustc, un-vendored git crates cuda-core / cuda-device /
cuda-host @ 5276d28f).  Every module restates the published algorithm of one
reference file and cites it by ``path:line``.

Pinning: the integer/data generators and the initial weights are checked bit
for bit against the reference's own unit-test constants (split sizes, parameter
counts, stride tables, known-answer tests); the f64 model is checked against a
pure-Python port of the reference's scalar tape (``tape.py``), finite
differences, and the archived grok-epoch cross-entropies that the reference
publishes in ``docs/cuda-performance.md:238-242``.
"""
