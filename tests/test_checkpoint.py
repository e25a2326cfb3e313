"""Checkpoint formats of the reference (src/gpt/checkpoint.rs:25-196 and
grok-simple's raw model.bin): byte layout, round trips and the reference's
rejections.  Host only, except the model round trip (GPU)."""

import struct

import numpy as np
import pytest

from grokking_abmod_b200 import GptConfig, MeshError, UnsupportedShape, initial_parameters
from grokking_abmod_b200.checkpoint import Checkpoint, load_raw, save_raw


def _expected_bytes(config, characters, params, magic, extra=()):
    head = magic + struct.pack("<7I", config.vocab_size, config.context, config.width, config.heads,
                               config.layers, config.attention_mesh_depth, config.ffn_mesh_depth)
    head += struct.pack(f"<{len(extra)}I", *extra)
    head += struct.pack(f"<{len(characters)}I", *[ord(c) for c in characters])
    return head + np.asarray(params, dtype="<f4").tobytes()


@pytest.mark.parametrize("connectivity,embedding,magic,extra", [
    ("neighbor", "mesh", b"MSHGPT07", ()), ("butterfly", "mesh", b"MSHGPT08", (0, 1)),
    ("neighbor", "table", b"MSHGPT08", (1, 0)), ("butterfly", "table", b"MSHGPT08", (1, 1))])
def test_layout_and_round_trip(tmp_path, connectivity, embedding, magic, extra):
    config = GptConfig(vocab_size=7, context=5, width=8, heads=2, layers=2, attention_mesh_depth=3,
                       ffn_mesh_depth=2, connectivity=connectivity, embedding=embedding)
    chars = "abc=+\U0001F600"
    params = initial_parameters(config, 7)
    path = tmp_path / "model.ckpt"
    Checkpoint(config, chars, params).save(path)
    data = path.read_bytes()
    assert data == _expected_bytes(config, chars, params, magic, extra)
    loaded = Checkpoint.load(path)
    assert loaded.config == config and loaded.characters == chars
    assert np.array_equal(loaded.parameters.view(np.uint32), params.view(np.uint32))


def _write(path, data):
    path.write_bytes(data)
    return path


def test_reference_rejections(tmp_path):
    config = GptConfig(vocab_size=3, context=4, width=4, heads=2, layers=1, attention_mesh_depth=2,
                       ffn_mesh_depth=2)
    params = initial_parameters(config, 1)
    good = _expected_bytes(config, "abc", params, b"MSHGPT07")
    Checkpoint.load(_write(tmp_path / "ok", good))
    for magic, text in ((b"MSHGPT03", "LayerNorm"), (b"MSHGPT06", "token table"), (b"NOTAMESH", "unsupported")):
        with pytest.raises(MeshError, match=text):
            Checkpoint.load(_write(tmp_path / "m", magic + good[8:]))
    with pytest.raises(MeshError, match="trailing"):
        Checkpoint.load(_write(tmp_path / "t", good + b"\0"))
    with pytest.raises(MeshError, match="truncated"):
        Checkpoint.load(_write(tmp_path / "s", good[:-1]))
    with pytest.raises(MeshError, match="unique"):
        Checkpoint.load(_write(tmp_path / "d", _expected_bytes(config, "aab", params, b"MSHGPT07")))
    bad = params.copy()
    bad[3] = np.inf
    with pytest.raises(MeshError, match="finite"):
        Checkpoint.load(_write(tmp_path / "f", _expected_bytes(config, "abc", bad, b"MSHGPT07")))
    with pytest.raises(MeshError, match="MSHGPT07"):
        Checkpoint.load(_write(tmp_path / "8", _expected_bytes(config, "abc", params, b"MSHGPT08", (0, 0))))
    # a table header over mesh-sized parameters: the table layout is shorter
    with pytest.raises(MeshError, match="trailing"):
        Checkpoint.load(_write(tmp_path / "tab", _expected_bytes(config, "abc", params, b"MSHGPT08", (1, 0))))
    with pytest.raises(MeshError, match="embedding"):
        Checkpoint.load(_write(tmp_path / "e", _expected_bytes(config, "abc", params, b"MSHGPT08", (2, 0))))
    with pytest.raises(UnsupportedShape):
        Checkpoint.load(_write(tmp_path / "9", b"MSHGPT09" + good[8:]))
    surrogate = good[:36] + struct.pack("<I", 0xD800) + good[40:]
    with pytest.raises(MeshError, match="character"):
        Checkpoint.load(_write(tmp_path / "u", surrogate))
    with pytest.raises(MeshError, match="do not match"):
        Checkpoint(config, "abcd", params).save(tmp_path / "w")
    with pytest.raises(MeshError, match="finite"):
        Checkpoint(config, "abc", bad).save(tmp_path / "w")


def test_raw_model_bin(tmp_path):
    p = np.random.default_rng(0).standard_normal(101).astype(np.float32)
    save_raw(tmp_path / "model.bin", p)
    assert (tmp_path / "model.bin").read_bytes() == p.astype("<f4").tobytes()
    assert np.array_equal(load_raw(tmp_path / "model.bin", 101), p)
    with pytest.raises(ValueError):
        load_raw(tmp_path / "model.bin", 100)


@pytest.mark.gpu
def test_model_round_trip_through_a_checkpoint(tmp_path):
    from grokking_abmod_b200 import AdamWOptions, MeshGpt
    config = GptConfig(vocab_size=11, context=8, width=64, heads=2, layers=2)
    model = MeshGpt(0, config, 3)
    rng = np.random.default_rng(1)
    x = rng.integers(0, 11, 32).astype(np.uint32)
    y = rng.integers(0, 11, 32).astype(np.uint32)
    model.train_batch_with_optimizer(x, y, 8, AdamWOptions(learning_rate=1e-3))
    Checkpoint.from_model(model, "abcdefghijk").save(tmp_path / "m.ckpt")
    restored = Checkpoint.load(tmp_path / "m.ckpt").model(0)
    assert np.array_equal(restored.logits(x, 8), model.logits(x, 8))
    restored.close()
    model.close()
