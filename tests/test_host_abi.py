"""The C ABI library on the host (no GPU): it loads, exports every entry point
that include/meshb200.h declares, and its host-side generators (seeded
initialisation, token codes, equation datasets, sampler, Zipf streams)
reproduce the oracle bit for bit."""

import ctypes
import os
import re

import numpy as np
import pytest

from grokking_abmod_b200 import GptConfig, MeshError, UnsupportedShape, initial_parameters, parameter_count, \
    token_codes
from grokking_abmod_b200 import _lib
from grokking_abmod_b200.data import EquationDataset, EquationSampler, random_units, zipf_batch
from oracle import data as odata
from oracle import gpt_config as ocfg
from oracle.rng import Random

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "meshb200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^int (mb_\w+)\(", text, flags=re.M)))


def test_library_exports_every_declared_entry_point():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 25
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must cover the header exactly"


def test_version_and_errors():
    lib = _lib.load()
    a, b = ctypes.c_int(), ctypes.c_int()
    assert lib.mb_version(ctypes.byref(a), ctypes.byref(b)) == 0
    assert lib.mb_version(None, None) == _lib.MB_ERR_INVALID
    buf = ctypes.create_string_buffer(256)
    assert lib.mb_last_error(buf, 256) == _lib.MB_ERR_INVALID
    assert b"must not be null" in buf.value


def _pairs():
    yield ocfg.GptConfig(), GptConfig()
    for kw in (dict(vocab_size=64, context=256, width=256, heads=4, layers=4),
               dict(vocab_size=99, context=4, width=128),
               dict(vocab_size=7, context=5, width=8, heads=2, layers=2, attention_mesh_depth=3, ffn_mesh_depth=4,
                    connectivity="butterfly"),
               dict(vocab_size=129, width=2, heads=1, layers=1, attention_mesh_depth=2, ffn_mesh_depth=2)):
        yield ocfg.GptConfig(**kw), GptConfig(**kw)


def test_initial_parameters_and_codes_match_oracle_bitwise():
    for oc, pc in _pairs():
        assert parameter_count(pc) == ocfg.Layout(oc).count()
        for seed in (0, 7, 11, 2**63 + 5):
            a = initial_parameters(pc, seed)
            b = ocfg.Layout(oc).initialize(seed)
            assert a.tobytes() == b.tobytes()
        assert token_codes(pc).tobytes() == ocfg.token_codes(oc).tobytes()


def test_config_validation_and_unsupported_shapes():
    with pytest.raises(MeshError):
        parameter_count(GptConfig(heads=3))
    with pytest.raises(MeshError):
        parameter_count(GptConfig(layers=65))
    lib = _lib.load()
    c = GptConfig(width=8, heads=2).to_c()
    assert lib.mb_gpt_validate(ctypes.byref(c)) == _lib.MB_ERR_UNSUPPORTED
    c = GptConfig(vocab_size=64, width=512, heads=8, context=1024, layers=8).to_c()
    assert lib.mb_gpt_validate(ctypes.byref(c)) == 0
    c = GptConfig(vocab_size=64, width=512, heads=4).to_c()  # head width 128
    assert lib.mb_gpt_validate(ctypes.byref(c)) == 0
    c = GptConfig(vocab_size=64, width=512, heads=2).to_c()  # head width 256
    assert lib.mb_gpt_validate(ctypes.byref(c)) == _lib.MB_ERR_UNSUPPORTED


def test_random_units_match_splitmix():
    r = Random(12345)
    expected = np.array([r.unit() for _ in range(1000)], dtype=np.float32)
    assert random_units(12345, 1000).tobytes() == expected.tobytes()


def test_equation_dataset_matches_oracle():
    for p, op, frac, seed in ((97, "add", 0.5, 7), (97, "div", 0.5, 11), (7, "mixed", 0.3, 3),
                              (13, "cubic-mixed", 0.7, 99)):
        a = EquationDataset(p, op, frac, seed)
        b = odata.EquationDataset(p, op, frac, seed)
        assert list(a.residue_tokens) == b.residue_tokens
        assert [tuple(r) for r in a.training] == b.training
        assert [tuple(r) for r in a.validation] == b.validation
        idx = list(range(min(50, len(b.training))))
        xa, ya = a.batch(False, idx)
        xb, yb = b.batch(False, idx)
        assert np.array_equal(xa, xb) and np.array_equal(ya, yb)
    with pytest.raises(MeshError):
        EquationDataset(4, "add", 0.5, 7)
    with pytest.raises(MeshError):
        EquationDataset(7, "add", 1.0, 7)


def test_sampler_matches_oracle():
    a = EquationSampler(25, 7)
    b = odata.EquationSampler(25, 7)
    for _ in range(7):
        assert list(a.sample(12)) == b.sample(12)
    a = EquationSampler(4704, 7).take(512, 12)
    b = odata.EquationSampler(4704, 7)
    for got in a:
        assert list(got) == b.sample(512)


def test_zipf_matches_oracle():
    for seed, rank, step in ((7, 0, 0), (7, 3, 5), (123, 1, 99)):
        xa, ya = zipf_batch(seed, rank, step, 3, 17)
        xb, yb = odata.zipf_batch(seed, rank, step, 3, 17)
        assert np.array_equal(xa, xb) and np.array_equal(ya, yb)


# ------------------------------------------------------------ grok-simple
def _simple_pairs():
    from grokking_abmod_b200.simple import SimpleConfig
    from oracle.simple_ref import SimpleConfig as OracleSimpleConfig
    for kw in (dict(architecture="tied-rotary-residual-dense-mlp", width=128, depth=1),
               dict(architecture="tied-rotary-residual-dense-mlp", modulus=7, width=10, depth=3,
                    activation="square"),
               dict(architecture="mesh-mlp", width=384, depth=5, connectivity="butterfly"),
               dict(architecture="mesh-mlp", modulus=7, width=9, depth=3, connectivity="own"),
               dict(architecture="mesh-mlp", modulus=5, width=16, depth=1),
               dict(architecture="shared-neighbor-mesh-mlp", width=128, depth=64, embedding_mesh_depth=32,
                    full_mesh_initialization="identity-hidden"),
               dict(architecture="shared-neighbor-mesh-mlp", modulus=7, width=8, depth=3, embedding_mesh_depth=2,
                    connectivity="butterfly", mesh_learning_rate_multiplier=3),
               dict(architecture="residual-mesh-mlp", width=64, depth=2, mesh_depth=4),
               dict(architecture="residual-mesh-mlp", modulus=7, width=6, depth=3, mesh_depth=2, connectivity="own"),
               dict(architecture="tied-concat-residual-mesh-mlp", width=128, depth=2, mesh_depth=3,
                    activation="square", connectivity="butterfly"),
               dict(architecture="tied-rotary-residual-mesh-mlp", width=128, depth=1, mesh_depth=1,
                    mesh_output_activation=True, mesh_learning_rate_multiplier=2),
               dict(architecture="tied-concat-mesh-mlp", width=64, depth=5, connectivity="own"),
               dict(architecture="mesh-mlp", width=64, depth=3, connectivity="own", tied_mesh=True),
               dict(architecture="tied-concat-mesh-mlp", modulus=7, width=8, depth=4, tied_mesh=True),
               dict(architecture="mlp", width=512, depth=2, encoding="binary"),
               dict(architecture="residual-mlp", width=128, depth=1, encoding="discrete-log"),
               dict(architecture="bilinear", modulus=13, width=16, encoding="scalar"),
               dict(architecture="mesh-mlp", modulus=3, width=8, depth=2, encoding="discrete-log"),
               dict(architecture="residual-mesh-mlp", modulus=11, width=32, depth=2, mesh_depth=2,
                    encoding="binary"),
               dict(architecture="full-mesh-mlp", width=128, depth=8, connectivity="butterfly", encoding="binary"),
               dict(architecture="full-mesh-mlp", modulus=7, width=8, depth=3, encoding="binary",
                    full_mesh_initialization="identity-hidden")):
        yield OracleSimpleConfig(**kw), SimpleConfig(**kw)


def test_simple_initial_parameters_groups_and_encoding_match_oracle():
    from oracle.simple_ref import encode, initial_parameters as oracle_init
    for oc, pc in _simple_pairs():
        assert pc.parameter_count() == oc.parameter_count()
        assert pc.groups() == oc.groups()
        for seed in (0, 11, 2**63 + 5):
            a, b = pc.initial_parameters(seed), oracle_init(oc, seed)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (oc, seed)
        eq = [(0, 1, 2), (oc.modulus - 1, 0, 1), (3 % oc.modulus, 2, 0)]
        f1, t1 = pc.encode(eq)
        f2, t2 = encode(oc, eq)
        assert np.array_equal(f1, f2) and np.array_equal(t1, t2)


def test_simple_validation_mirrors_the_reference():
    from grokking_abmod_b200.simple import SimpleConfig
    bad = [dict(architecture="shared-neighbor-mesh-mlp", width=64),
           dict(architecture="shared-neighbor-mesh-mlp", width=128, connectivity="own"),
           dict(architecture="tied-rotary-residual-dense-mlp", width=127),
           dict(architecture="mesh-mlp", full_mesh_initialization="identity-hidden"),
           dict(architecture="mesh-mlp", depth=1, mesh_learning_rate_multiplier=2),
           dict(architecture="mesh-mlp", depth=0), dict(architecture="mesh-mlp", depth=65),
           dict(architecture="mesh-mlp", modulus=1), dict(architecture="mesh-mlp", modulus=1025),
           dict(architecture="residual-mesh-mlp", mesh_depth=0), dict(architecture="residual-mesh-mlp", mesh_depth=65),
           dict(architecture="mesh-mlp", mesh_output_activation=True),
           dict(architecture="tied-concat-mesh-mlp", mesh_output_activation=True),
           dict(architecture="tied-rotary-residual-mesh-mlp", width=127),
           dict(architecture="tied-concat-residual-mesh-mlp", width=8193),
           dict(architecture="residual-mesh-mlp", tied_mesh=True), dict(architecture="mlp", tied_mesh=True),
           dict(architecture="tied-rotary-residual-mesh-mlp", encoding="binary"),
           dict(architecture="mlp", modulus=15, encoding="discrete-log"),
           dict(architecture="mlp", decay_factors=1), dict(architecture="mlp", depth=2, decay_factors=3),
           dict(architecture="bilinear", decay_factors=4),
           dict(architecture="full-mesh-mlp"), dict(architecture="full-mesh-mlp", encoding="binary", connectivity="own")]
    for kw in bad:
        with pytest.raises(MeshError):
            SimpleConfig(**kw).validate()
    with pytest.raises(ValueError):
        SimpleConfig(architecture="sparse-mesh-mlp").to_c()
    # src/simple/mod.rs:1446-1760 (parameter counts of the mesh architectures)
    assert SimpleConfig(architecture="residual-mesh-mlp", width=64, depth=2, mesh_depth=4).parameter_count() == 19648
    assert SimpleConfig(architecture="tied-rotary-residual-mesh-mlp", width=128, depth=2,
                        mesh_depth=3).groups() == [12416] + [256] * 6
    assert SimpleConfig(architecture="tied-concat-residual-mesh-mlp", width=128, depth=2,
                        mesh_depth=3).groups() == [12416, 32768] + [256] * 6
    assert SimpleConfig(architecture="tied-concat-mesh-mlp", width=64, depth=5,
                        connectivity="own").groups() == [97 * 64, 128 * 64, 64, 64, 64, 64]
    # the library's own counts for the two dense-only architectures
    assert SimpleConfig(architecture="mlp", modulus=97, width=128, depth=2).parameter_count() == 53632
    assert SimpleConfig(architecture="bilinear", modulus=97, width=16, depth=0).validate().parameter_count() == 4656
    assert SimpleConfig(architecture="mlp", modulus=7, width=9, depth=3).groups() == [14 * 9, 81, 81, 9 * 7]
    with pytest.raises(MeshError):
        SimpleConfig(modulus=7, width=8).encode([(7, 0, 0)])


def test_table_embedding_init_matches_the_oracle_bitwise():
    from oracle.gpt_config import GptConfig as OracleConfig, Layout
    for connectivity in ("neighbor", "butterfly"):
        kw = dict(vocab_size=64, context=70, width=256, heads=4, layers=2, connectivity=connectivity)
        got = initial_parameters(GptConfig(**kw, embedding="table"), 5)
        want = Layout(OracleConfig(**kw, embedding="table")).initialize(5)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert parameter_count(GptConfig(**kw, embedding="table")) == want.size
    with pytest.raises(ValueError):
        GptConfig(embedding="dense").to_c()
