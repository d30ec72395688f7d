"""Device-memory helpers for the GPU tests (torch is used only as a device
allocator; every computation under test goes through the C ABI)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from oracle import oracle


def torch():
    import torch as _t
    return _t


def to_dev(a: np.ndarray):
    """Host array -> device tensor holding the same bytes."""
    a = np.ascontiguousarray(a)
    t = torch()
    view = {2: np.int16, 4: np.int32, 8: np.int64, 1: np.uint8}[a.dtype.itemsize]
    if a.dtype == np.float32:
        return t.from_numpy(a.copy()).cuda()
    return t.from_numpy(a.view(view).copy()).cuda()


def zeros_dev(shape, itemsize=2):
    t = torch()
    dt = {1: t.uint8, 2: t.int16, 4: t.int32, 8: t.int64}[itemsize]
    return t.zeros(shape, dtype=dt, device="cuda")


def from_dev_u16(t) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


def sync():
    torch().cuda.synchronize()


def rand_bf16(shape, scale=1.0, seed=0) -> np.ndarray:
    from tests import numerics as nm
    rng = np.random.default_rng(seed)
    return nm.f32_to_bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


def ptr(t) -> int:
    return t.data_ptr()


class RefModel:
    """The reference's own kernels (oracle/_ref, compute_86 PTX JIT) run over
    the same device weights as an engine, with their own KV cache."""

    def __init__(self, cfg, tensor_ptrs: list, capacity: int, max_rows: int):
        self.L = oracle.ref_cuda()
        self.cfg = cfg
        self.oc = cfg.c() if hasattr(cfg, "c") else cfg
        self.capacity = capacity
        g = cfg.kv_heads * cfg.head_width
        self.cache = [zeros_dev((capacity, g)) for _ in range(2 * cfg.layers)]
        self._tp = (C.c_void_p * len(tensor_ptrs))(*tensor_ptrs)
        self._cp = (C.c_void_p * len(self.cache))(*[ptr(c) for c in self.cache])
        n = self.L.ref_qwen3_scratch_bytes(C.byref(self._ocfg()), max_rows)
        self.scratch = zeros_dev((n // 2 + 64,))
        self.tokens = zeros_dev((max_rows,), 4)
        self.logits = zeros_dev((cfg.vocabulary,))
        self.max_rows = max_rows

    def _ocfg(self):
        c = self.cfg
        return oracle.OrConfig(c.hidden, c.query_heads, c.kv_heads, c.head_width, c.mlp_width,
                               c.vocabulary, c.layers, c.epsilon, c.theta)

    def forward(self, tokens, first: int, capture_layer: int = -1):
        """BF16 logits bits of the last row, and the captured block output
        rows: [rows][D] for capture_layer >= 0, [layers][rows][D] for -2."""
        tokens = np.ascontiguousarray(tokens, np.uint32)
        rows = tokens.size
        assert rows <= self.max_rows
        self.tokens[:rows].copy_(torch().from_numpy(tokens.view(np.int32)).cuda())
        if capture_layer == -2:
            cap = zeros_dev((self.cfg.layers, rows, self.cfg.hidden))
        else:
            cap = zeros_dev((rows, self.cfg.hidden)) if capture_layer >= 0 else None
        rc = self.L.ref_qwen3_forward(C.byref(self._ocfg()), self._tp, self._cp, self.capacity,
                                      ptr(self.tokens), rows, first, ptr(self.logits), capture_layer,
                                      ptr(cap) if cap is not None else None, ptr(self.scratch), None)
        assert rc == 0
        sync()
        return from_dev_u16(self.logits).copy(), (from_dev_u16(cap).copy() if cap is not None else None)
