"""Source-level invariants the CUDA code relies on (CPU only).

The grok-simple step graphs chain their kernels with programmatic edges: a
kernel may be scheduled while its predecessor is still running, and only its
first statement, wait_prior_grids() (griddepcontrol.wait), orders it after the
predecessor's writes.  A kernel added to those files without that wait would
race, so every kernel definition there must begin with it.
"""

import os
import re

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "grokking_abmod_b200", "csrc")


def _kernel_bodies(path):
    text = open(path).read()
    for m in re.finditer(r"__global__", text):
        brace = text.index("{", m.end())
        assert ";" not in text[m.end():brace], "declaration without a body"
        yield text[m.end():brace], text[brace + 1:brace + 400]


def test_every_kernel_of_the_step_graphs_waits_for_its_predecessors():
    for name in ("simple_model.cu", "gemm_tc.cu"):
        kernels = list(_kernel_bodies(os.path.join(CSRC, name)))
        assert kernels, name
        for signature, body in kernels:
            first = body.strip().split(";")[0].strip()
            assert first == "wait_prior_grids()", (name, signature.strip()[:80])


def test_no_cluster_multicast_loads():
    # Every kernel may run in a multi-GPU job, and no load there may
    # multicast across a cluster: none of the sources uses the qualifier.
    for name in os.listdir(CSRC):
        assert "multicast::cluster" not in open(os.path.join(CSRC, name)).read(), name
