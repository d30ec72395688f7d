"""Safetensors checkpoint reading and Qwen3 name binding (CPU).

The reference's tiny Qwen3 fixture is the known-answer case: its config maps to
the model shape and every tensor reads back bit-identical to a direct parse,
in the engine's tensor order.  A sharded copy (index + two shards) and an FP32
copy read back the same bits, and the config rules reject what the reference
rejects.
"""
import json
import os
import shutil
import struct

import numpy as np
import pytest

from dolittle_b200 import checkpoint
from tests import tiny


def _write_safetensors(path, named: dict, dtype="BF16"):
    header, blobs, off = {}, [], 0
    for name, arr in named.items():
        if dtype == "F32":
            data = (arr.astype(np.uint32) << 16).view(np.float32).astype("<f4").tobytes()
        else:
            data = arr.astype("<u2").tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _named():
    return tiny.read_safetensors(os.path.join(tiny.HERE, "model.safetensors"))


def _shape(t):
    return t.shape if t.ndim == 2 else (1, t.shape[0])


def test_tiny_config_maps_to_model_shape():
    cfg = checkpoint.config_from_json(os.path.join(tiny.HERE, "config.json"), "BF16")
    ref = tiny.config()
    assert (cfg.hidden, cfg.query_heads, cfg.kv_heads, cfg.head_width, cfg.mlp_width, cfg.vocabulary,
            cfg.layers) == (ref.hidden, ref.query_heads, ref.kv_heads, ref.head_width, ref.mlp_width,
                            ref.vocabulary, ref.layers)
    assert cfg.epsilon == pytest.approx(ref.epsilon) and cfg.theta == ref.theta


def test_tiny_checkpoint_reads_every_tensor_in_engine_order():
    ck = checkpoint.Checkpoint(tiny.HERE)
    expected = tiny.tensors()
    names = checkpoint.tensor_names(tiny.config().layers)
    assert len(names) == len(expected)
    for name, want in zip(names, expected):
        got = np.asarray(ck.bf16(name, want.shape))
        assert np.array_equal(got, want), name
    assert ck.storage_dtype() == "BF16"


def test_sharded_and_fp32_copies_read_the_same_bits(tmp_path):
    named = _named()
    names = list(named)
    half = len(names) // 2
    d = tmp_path / "sharded"
    d.mkdir()
    _write_safetensors(d / "model-00001-of-00002.safetensors", {n: named[n] for n in names[:half]})
    _write_safetensors(d / "model-00002-of-00002.safetensors", {n: named[n] for n in names[half:]})
    wm = {n: ("model-00001-of-00002.safetensors" if i < half else "model-00002-of-00002.safetensors")
          for i, n in enumerate(names)}
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    shutil.copy(os.path.join(tiny.HERE, "config.json"), d / "config.json")
    ck = checkpoint.Checkpoint(str(d))
    for n in names:
        assert np.array_equal(np.asarray(ck.bf16(n, named[n].shape)), named[n]), n
    # FP32 storage of BF16-exact values rounds back to the same bits.
    f = tmp_path / "f32.safetensors"
    _write_safetensors(f, named, dtype="F32")
    ck32 = checkpoint.Checkpoint(str(f))
    assert ck32.storage_dtype() == "F32"
    for n in names:
        assert np.array_equal(ck32.bf16(n, named[n].shape), named[n]), n


def test_fp32_rounding_is_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9, -2.5, np.inf, -np.inf, 3.4e38], np.float32)
    got = checkpoint._bf16_bits(x)
    assert got.tolist() == [0x3F80, 0x3F80, 0x3F81, 0xC020, 0x7F80, 0xFF80, 0x7F80]
    assert (checkpoint._bf16_bits(np.array([np.nan], np.float32))[0] & 0x7FFF) > 0x7F80


@pytest.mark.parametrize("edit", [{"tie_word_embeddings": True}, {"sliding_window": 128},
                                  {"hidden_act": "gelu"}, {"model_type": "llama"}, {"dtype": "float32"},
                                  {"attention_bias": True}, {"partial_rotary_factor": 0.5}])
def test_config_rules_reject_like_the_reference(tmp_path, edit):
    c = json.load(open(os.path.join(tiny.HERE, "config.json")))
    c.update(edit)
    p = tmp_path / "config.json"
    p.write_text(json.dumps(c))
    with pytest.raises(ValueError):
        checkpoint.config_from_json(str(p), "BF16")


def test_missing_tensor_and_wrong_shape_are_rejected(tmp_path):
    named = _named()
    first = next(iter(named))
    partial = {n: a for n, a in named.items() if n != first}
    f = tmp_path / "partial.safetensors"
    _write_safetensors(f, partial)
    ck = checkpoint.Checkpoint(str(f))
    with pytest.raises(KeyError):
        ck.bf16(first, named[first].shape)
    other = next(iter(partial))
    with pytest.raises(ValueError):
        ck.bf16(other, (partial[other].shape[0] + 1,) + tuple(partial[other].shape[1:]))
