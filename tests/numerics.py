"""Shared comparison helpers for the test suite.

compare_elementwise / compare_values restate the reference's test support
(tests/support/numerical.cpp:150-221): an element fails when
|actual - expected| > atol + rtol*|expected|; the whole-tensor check bounds the
maximum absolute error and the relative L2 error.  operand() restates the
deterministic operand generator of tests/gpu/operator_reference.cpp:60-75.
"""
from __future__ import annotations

import math

import numpy as np


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(values) -> np.ndarray:
    """BF16 round-to-nearest-even narrowing (bf16.cpp:48-60)."""
    a = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (a & 0x7FFFFFFF) > 0x7F800000
    r = ((a + 0x7FFF + ((a >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, 0x7FC0, r)
    return r.astype(np.uint16)


def round_bf16(values) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(values))


def operand(shape, seed: int, bf16: bool = True) -> np.ndarray:
    """((i*73 + seed*37) % 257 - 128) / 64, rounded to storage."""
    n = int(np.prod(shape))
    i = np.arange(n, dtype=np.int64)
    v = ((i * 73 + seed * 37) % 257 - 128).astype(np.float32) / np.float32(64)
    v = v.reshape(shape)
    return round_bf16(v) if bf16 else v


def compare_elementwise(expected, actual, atol: float, rtol: float):
    e = np.asarray(expected, np.float64).reshape(-1)
    a = np.asarray(actual, np.float64).reshape(-1)
    assert np.all(np.isfinite(e)), "reference values must be finite"
    finite = np.isfinite(a)
    err = np.abs(a - e)
    bad = (~finite) | (err > atol + rtol * np.abs(e))
    return {"mismatched": int(bad.sum()), "finite": bool(finite.all()),
            "max_abs": float(np.max(np.where(finite, err, np.inf))) if e.size else 0.0,
            "passed": int(bad.sum()) == 0}


def compare_values(expected, actual, max_abs: float, max_rel_l2: float):
    e = np.asarray(expected, np.float64).reshape(-1)
    a = np.asarray(actual, np.float64).reshape(-1)
    if not np.all(np.isfinite(a)):
        return {"finite": False, "max_abs": math.inf, "rel_l2": None, "passed": False}
    d = a - e
    m = float(np.max(np.abs(d))) if d.size else 0.0
    sr = float(np.sum(e * e))
    rel = math.sqrt(float(np.sum(d * d)) / sr) if sr else None
    return {"finite": True, "max_abs": m, "rel_l2": rel,
            "passed": m <= max_abs and (rel is None or rel <= max_rel_l2)}


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    return float(a @ b / (na * nb)) if na and nb else float("nan")


def serial_sum_f32(terms) -> np.float32:
    """Ordinary serial FP32 accumulation (np.cumsum keeps FP32 and order)."""
    t = np.asarray(terms, np.float32).reshape(-1)
    return np.float32(np.cumsum(t, dtype=np.float32)[-1]) if t.size else np.float32(0)
