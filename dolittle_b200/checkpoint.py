"""Qwen3 safetensors checkpoints bound to the engine's tensor order.

Role of the reference's safetensors reader and Qwen3 binding
(src/tensors/formats/safetensors.cpp; src/models/qwen3/checkpoint.cpp:111-152
for the serialized names, :236-300 for the config rules).  A checkpoint is a
single `.safetensors` file or a directory with `config.json` and either
`model.safetensors` or `model.safetensors.index.json` + shards.  Tensors are
read through memory maps one at a time, so host memory stays small.  BF16
storage is bound as is; FP32 storage is rounded to BF16 (nearest even).

The config rules follow the reference: model_type qwen3, SiLU, no attention or
MLP bias, untied embeddings, no sliding window or scaled/partial RoPE, zero
attention dropout, and a declared dtype that matches the storage.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

from .engine import Engine, Qwen3Config

GLOBAL_NAMES = ["model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"]
BLOCK_NAMES = ["input_layernorm", "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
               "self_attn.q_norm", "self_attn.k_norm", "self_attn.o_proj", "post_attention_layernorm",
               "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"]


def tensor_names(layers: int) -> list:
    """Serialized names in the engine's tensor order (dl_engine_tensor_shape)."""
    names = list(GLOBAL_NAMES)
    for block in range(layers):
        names += [f"model.layers.{block}.{n}.weight" for n in BLOCK_NAMES]
    return names


def _bf16_bits(a: np.ndarray) -> np.ndarray:
    """FP32 -> BF16 bits, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    return np.where(nan, (u >> 16) | 0x40, rounded).astype(np.uint16)


class SafetensorsFile:
    """One `.safetensors` file: JSON header, then little-endian tensor data."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            head = f.read(8)
            if len(head) != 8:
                raise ValueError(f"{path}: truncated safetensors header")
            (n,) = struct.unpack("<Q", head)
            if n > 100 * 1024 * 1024:
                raise ValueError(f"{path}: header of {n} bytes is too large")
            self.header = json.loads(f.read(n))
        self.data_offset = 8 + n
        self.metadata = self.header.pop("__metadata__", {})
        size = os.path.getsize(path)
        for name, meta in self.header.items():
            a, b = meta["data_offsets"]
            if not 0 <= a <= b or self.data_offset + b > size:
                raise ValueError(f"{path}: tensor {name} lies outside the file")

    def names(self) -> list:
        return list(self.header)

    def bf16(self, name: str, shape) -> np.ndarray:
        meta = self.header[name]
        if list(meta["shape"]) != list(shape):
            raise ValueError(f"{name}: shape {meta['shape']} != expected {list(shape)}")
        a, b = meta["data_offsets"]
        count = int(np.prod(shape))
        if meta["dtype"] == "BF16":
            if b - a != 2 * count:
                raise ValueError(f"{name}: byte size")
            return np.memmap(self.path, np.uint16, "r", self.data_offset + a, (count,)).reshape(shape)
        if meta["dtype"] == "F32":
            if b - a != 4 * count:
                raise ValueError(f"{name}: byte size")
            return _bf16_bits(np.memmap(self.path, np.float32, "r", self.data_offset + a, (count,))).reshape(shape)
        raise ValueError(f"{name}: dtype {meta['dtype']} (BF16 or F32 required)")


class Checkpoint:
    """A checkpoint file or directory; `bf16(name, shape)` reads one tensor."""

    def __init__(self, path: str):
        self.config_path = None
        if os.path.isdir(path):
            cfg = os.path.join(path, "config.json")
            self.config_path = cfg if os.path.exists(cfg) else None
            index = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(index):
                with open(index) as f:
                    weight_map = json.load(f)["weight_map"]
                files = {fname: SafetensorsFile(os.path.join(path, fname)) for fname in set(weight_map.values())}
                self.where = {name: files[fname] for name, fname in weight_map.items()}
            else:
                single = SafetensorsFile(os.path.join(path, "model.safetensors"))
                self.where = {name: single for name in single.names()}
        else:
            single = SafetensorsFile(path)
            self.where = {name: single for name in single.names()}

    def bf16(self, name: str, shape) -> np.ndarray:
        if name not in self.where:
            raise KeyError(f"checkpoint has no tensor {name}")
        return self.where[name].bf16(name, shape)

    def storage_dtype(self) -> str:
        kinds = {f.header[n]["dtype"] for n, f in self.where.items()}
        if len(kinds) != 1:
            raise ValueError(f"mixed tensor dtypes {sorted(kinds)}")
        return kinds.pop()


def config_from_json(path: str, storage_dtype: str = "BF16") -> Qwen3Config:
    """Qwen3Config from a Hugging Face config.json under the reference's rules."""
    with open(path) as f:
        c = json.load(f)
    if c.get("model_type") != "qwen3":
        raise ValueError("model_type must be qwen3")
    if c.get("architectures", ["Qwen3ForCausalLM"]) != ["Qwen3ForCausalLM"]:
        raise ValueError("unsupported Qwen3 architecture list")
    if c.get("hidden_act") != "silu":
        raise ValueError("hidden_act must be silu")
    for key in ("attention_bias", "mlp_bias", "tie_word_embeddings", "use_sliding_window"):
        if c.get(key, False):
            raise ValueError(f"{key} is unsupported")
    if c.get("rope_scaling") is not None or c.get("sliding_window") is not None:
        raise ValueError("scaled RoPE and sliding windows are unsupported")
    if float(c.get("partial_rotary_factor", 1.0)) != 1.0:
        raise ValueError("partial rotary embeddings are unsupported")
    if float(c.get("attention_dropout", 0.0)) != 0.0:
        raise ValueError("nonzero attention dropout is unsupported")
    want = {"BF16": "bfloat16", "F32": "float32"}.get(storage_dtype)
    for key in ("dtype", "torch_dtype"):
        if key in c and c[key] != want:
            raise ValueError(f"{key} {c[key]} does not match {storage_dtype} storage")
    theta = c.get("rope_theta")
    if theta is None:  # newer transformers write rope_parameters
        rp = c.get("rope_parameters") or {}
        if rp.get("rope_type", "default") != "default":
            raise ValueError("scaled RoPE is unsupported")
        theta = rp.get("rope_theta")
    if theta is None:
        raise ValueError("rope_theta missing")
    heads = int(c["num_attention_heads"])
    return Qwen3Config(hidden=int(c["hidden_size"]), query_heads=heads, kv_heads=int(c["num_key_value_heads"]),
                       head_width=int(c.get("head_dim", int(c["hidden_size"]) // heads)),
                       mlp_width=int(c["intermediate_size"]), vocabulary=int(c["vocab_size"]),
                       layers=int(c["num_hidden_layers"]), epsilon=float(c["rms_norm_eps"]), theta=float(theta))


def load_qwen3(engine: Engine, checkpoint: Checkpoint | str) -> None:
    """Bind every Qwen3 tensor of `checkpoint` into `engine` by name."""
    ck = Checkpoint(checkpoint) if isinstance(checkpoint, str) else checkpoint
    cfg = engine.config
    for index, name in enumerate(tensor_names(cfg.layers)):
        shape = cfg.tensor_shape(index)
        bits = ck.bf16(name, shape if shape[0] != 1 else (shape[1],))
        engine.set_tensor(index, np.ascontiguousarray(bits).reshape(shape))


def open_qwen3(path: str, device: int = 0, capacity: int = 1024, max_rows: int = 8) -> Engine:
    """Engine for a checkpoint directory: config.json + weights."""
    ck = Checkpoint(path)
    if ck.config_path is None:
        raise ValueError("checkpoint directory has no config.json")
    cfg = config_from_json(ck.config_path, ck.storage_dtype())
    engine = Engine(cfg, device=device, capacity=capacity, max_rows=max_rows)
    load_qwen3(engine, ck)
    return engine
