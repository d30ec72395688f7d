"""The reference's tiny Qwen3 fixture (tests/golden/tiny-bf16/) for the tests.

Loads the committed safetensors weights into the role order shared by the
oracle and the product (embedding, final norm, lm_head, then per block:
input norm, q, k, v, q_norm, k_norm, o, post norm, gate, up, down) and the
fixture's expected logits/captures with their per-output tolerances.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tiny-bf16")

HF_GLOBAL = ["model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"]
HF_BLOCK = ["input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
            "self_attn.v_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
            "self_attn.o_proj.weight", "post_attention_layernorm.weight",
            "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"]


def read_safetensors(path: str) -> dict:
    with open(path, "rb") as f:
        blob = f.read()
    n = struct.unpack("<Q", blob[:8])[0]
    header = json.loads(blob[8:8 + n])
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        assert meta["dtype"] == "BF16", name
        a, b = meta["data_offsets"]
        out[name] = np.frombuffer(blob[8 + n + a:8 + n + b], np.uint16).reshape(meta["shape"]).copy()
    return out


def config():
    from oracle.oracle import Config
    c = json.load(open(os.path.join(HERE, "config.json")))
    theta = c.get("rope_theta") or c["rope_parameters"]["rope_theta"]
    return Config(hidden=c["hidden_size"], query_heads=c["num_attention_heads"],
                  kv_heads=c["num_key_value_heads"], head_width=c["head_dim"],
                  mlp_width=c["intermediate_size"], vocabulary=c["vocab_size"],
                  layers=c["num_hidden_layers"], epsilon=c["rms_norm_eps"], theta=float(theta))


def tensors() -> list:
    named = read_safetensors(os.path.join(HERE, "model.safetensors"))
    cfg = config()
    out = [named[n] for n in HF_GLOBAL]
    for layer in range(cfg.layers):
        out += [named[f"model.layers.{layer}.{n}"] for n in HF_BLOCK]
    return out


def fixture() -> dict:
    return json.load(open(os.path.join(HERE, "fixture.json")))


def expected_rows(entry: dict) -> np.ndarray:
    return np.asarray(entry["values"], np.float32).reshape(len(entry["positions"]), entry["width"])
