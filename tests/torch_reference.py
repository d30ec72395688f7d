"""Plain PyTorch FP32 reference of the Qwen3 prompt pass.  TEST INFRASTRUCTURE.

It follows the reference's own whole-model oracle policy
(scripts/validation/forward_reference.py:46-107: FP32 arithmetic for every
operation, activations stored in BF16 between operations) over the weights an
engine holds in device memory, and returns every block's output rows.  Its
reduction orders are torch's (FP32 GEMMs with TF32 off), so it is the
independent yardstick against which both the reference-order kernels and the
tensor-core prompt pass are measured.

Rounding points (BF16 storage) follow the reference recipe
(src/models/qwen3/model.cpp:351-388): RMSNorm rounds x*inv then the product
with the weight; projections, RoPE products and sums, attention outputs,
residual adds and the SwiGLU's two products are each rounded to BF16.
"""
from __future__ import annotations

import torch


class _DeviceArray:
    """__cuda_array_interface__ over a device pointer the engine owns."""

    def __init__(self, ptr: int, rows: int, cols: int, row_stride: int):
        self.__cuda_array_interface__ = {"shape": (rows, cols), "typestr": "<i2", "data": (ptr, False),
                                         "strides": (row_stride * 2, 2), "version": 3}


def engine_tensor(engine, cfg, index: int) -> torch.Tensor:
    """A BF16 view (no copy) of resident tensor `index` of an engine."""
    ptr, stride = engine.tensor_device(index)
    rows, cols = cfg.tensor_shape(index)
    return torch.as_tensor(_DeviceArray(ptr, rows, cols, stride), device="cuda").view(torch.bfloat16)


def _bf(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def _rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    inv = torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
    return _bf(_bf(x * inv) * w.float().reshape(-1))


def _linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return _bf(x @ w.float().t())


def _rope(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """x [rows][heads][d]; split-half pairs, cos/sin rounded to storage."""
    d = x.shape[-1]
    half = d // 2
    exponent = (2 * torch.arange(half, dtype=torch.float32, device=x.device)) / d
    inv = (1.0 / torch.pow(torch.tensor(theta, dtype=torch.float64, device=x.device), exponent.double())).float()
    angle = positions.float()[:, None] * inv[None, :]
    c, s = _bf(torch.cos(angle))[:, None, :], _bf(torch.sin(angle))[:, None, :]
    a, b = x[..., :half], x[..., half:]
    return torch.cat([_bf(_bf(a * c) - _bf(b * s)), _bf(_bf(b * c) + _bf(a * s))], dim=-1)


def prompt_blocks(engine, cfg, tokens) -> tuple:
    """Every block's output rows [layers][rows][D] (BF16) and the last row's
    logits [V] (BF16) of one prompt pass from position 0."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.no_grad():
            return _prompt_blocks(engine, cfg, tokens)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _prompt_blocks(engine, cfg, tokens):
    D, H, G, d = cfg.hidden, cfg.query_heads, cfg.kv_heads, cfg.head_width
    n = len(tokens)
    ids = torch.as_tensor([int(t) for t in tokens], dtype=torch.long, device="cuda")
    x = engine_tensor(engine, cfg, 0)[ids].float()
    positions = torch.arange(n, device="cuda")
    causal = torch.ones(n, n, dtype=torch.bool, device="cuda").tril()
    outs = torch.empty((cfg.layers, n, D), dtype=torch.bfloat16, device="cuda")
    scale = 1.0 / (d ** 0.5)
    for l in range(cfg.layers):
        t = [engine_tensor(engine, cfg, 3 + 11 * l + r) for r in range(11)]
        h = _rms_norm(x, t[0], cfg.epsilon)
        q = _linear(h, t[1]).reshape(n, H, d)
        k = _linear(h, t[2]).reshape(n, G, d)
        v = _linear(h, t[3]).reshape(n, G, d)
        q = _rope(_rms_norm(q, t[4], cfg.epsilon), positions, cfg.theta)
        k = _rope(_rms_norm(k, t[5], cfg.epsilon), positions, cfg.theta)
        kk = k.repeat_interleave(H // G, dim=1)      # [n][H][d]
        vv = v.repeat_interleave(H // G, dim=1)
        s = torch.einsum("qhd,khd->hqk", q, kk) * scale
        s = s.masked_fill(~causal[None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        att = _bf(torch.einsum("hqk,khd->qhd", p, vv)).reshape(n, H * d)
        x = _bf(x + _linear(att, t[6]))
        h = _rms_norm(x, t[7], cfg.epsilon)
        g, u = _linear(h, t[8]), _linear(h, t[9])
        act = _bf(_bf(g * torch.sigmoid(g)) * u)
        x = _bf(x + _linear(act, t[10]))
        outs[l] = x.to(torch.bfloat16)
    last = _rms_norm(x[-1:], engine_tensor(engine, cfg, 1), cfg.epsilon)
    logits = _linear(last, engine_tensor(engine, cfg, 2))[0].to(torch.bfloat16)
    return outs, logits
