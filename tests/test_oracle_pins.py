"""Pin the CPU oracle (oracle/dl_oracle.c) before it is trusted.

* BF16 narrowing/widening against the reference's own bf16.cpp (all 65,536
  encodings; ties, specials and random values).
* MT19937-64 against the reference's std::mt19937_64 RandomStream.
* Host selection law against the reference's own Categorical::select on the
  cases of tests/core/test_sampling.cpp:36-165.
* The device selection law (restated from sampling.cu) against the host law on
  the cases of tests/gpu/test_device.cpp:265-352, where the reference asserts
  device == host.
* Every kernel-law op against the reference's independent host equations and
  tolerances (tests/gpu/operator_reference.cpp:167-314).

The _ref libraries are compiled from the reference sources by oracle/Makefile;
tests needing them skip when they were not built.
"""
import numpy as np
import pytest

from oracle import oracle
from tests import numerics as nm

REF_HOST = oracle.ref_host()
needs_ref = pytest.mark.skipif(REF_HOST is None, reason="oracle/_ref not built")


# --------------------------------------------------------------------------
# BF16
# --------------------------------------------------------------------------
@needs_ref
def test_bf16_all_encodings_widen_identically():
    L, R = oracle.lib(), REF_HOST
    for b in range(65536):
        x, y = L.or_bf16_to_float(b), R.ref_bf16_to_float(b)
        assert (x == y) or (np.isnan(x) and np.isnan(y)), b


@needs_ref
def test_bf16_narrowing_matches_reference():
    L, R = oracle.lib(), REF_HOST
    rng = np.random.default_rng(1)
    bits = np.arange(65536, dtype=np.uint32) << 16
    ties = bits + 0x8000              # exact midpoints: round half to even
    near = bits + 0x7FFF
    above = bits + 0x8001
    rand = rng.integers(0, 2**32, 200_000, dtype=np.uint64).astype(np.uint32)
    for words in (bits, ties, near, above, rand):
        values = words.view(np.float32)
        ours = oracle.bf16_from_f32(values)
        theirs = np.array([R.ref_bf16_from_float(float(v)) for v in values[:20000]],
                          dtype=np.uint16)
        assert np.array_equal(ours[:20000], theirs)
        # The numpy restatement used by the tests follows the same law.
        assert np.array_equal(nm.f32_to_bf16_bits(values), ours)


# --------------------------------------------------------------------------
# MT19937-64
# --------------------------------------------------------------------------
@needs_ref
@pytest.mark.parametrize("seed", [0, 7, 42, 7391, 2**63 + 5])
def test_mt19937_64_matches_std(seed):
    ours = oracle.MT64(seed)
    h = REF_HOST.ref_rng_create(seed)
    try:
        for _ in range(1500):               # crosses several 312-word twists
            assert ours() == REF_HOST.ref_rng_next(h)
    finally:
        REF_HOST.ref_rng_destroy(h)


# --------------------------------------------------------------------------
# Selection laws
# --------------------------------------------------------------------------
def _ref_select(logits, categorical, t, k, p, rng):
    import ctypes as C
    tok = C.c_uint32(0)
    rc = REF_HOST.ref_categorical_select(np.ascontiguousarray(logits, np.float32),
                                         len(logits), int(categorical), t, k, p,
                                         rng, C.byref(tok))
    return None if rc else tok.value


@needs_ref
def test_host_law_matches_reference_distribution_contract():
    """tests/core/test_sampling.cpp:56-100 cases, draw by draw."""
    inp = oracle.MT64(7391)
    f32 = np.float32
    for size in (17, 1023, 4096):
        values = np.array([f32(int(inp() % 4001) - 2000) / f32(127.0)
                           for _ in range(size)], np.float32)
        edges = np.array([0.0, -0.0, np.float32(1.4e-45), -np.float32(1.4e-45),
                          -np.inf, 1.0, 1.0], np.float32)
        values[:7] = edges
        for t, k, p in ((1.0, 0, 1.0), (0.6, 0, 0.95), (2.0, 11, 0.7)):
            seed = inp()
            mine, theirs = oracle.MT64(seed), REF_HOST.ref_rng_create(seed)
            try:
                for _ in range(64):
                    expected = _ref_select(values, True, t, k, p, theirs)
                    got = oracle.select_host(values, True, t, k, p, word=mine())
                    assert got == expected
            finally:
                REF_HOST.ref_rng_destroy(theirs)
        zeros = np.where(np.arange(size) % 2 == 1, np.float32(-0.0), np.float32(0.0)).astype(np.float32)
        seed = inp()
        mine, theirs = oracle.MT64(seed), REF_HOST.ref_rng_create(seed)
        try:
            for _ in range(64):
                expected = _ref_select(zeros, True, 1.0, 0, 0.5, theirs)
                assert oracle.select_host(zeros, True, 1.0, 0, 0.5, word=mine()) == expected
        finally:
            REF_HOST.ref_rng_destroy(theirs)


@needs_ref
def test_host_law_fixed_cases_and_rejections():
    """tests/core/test_sampling.cpp:103-160."""
    inf = np.float32(np.inf)
    logits = np.array([-inf, 3, 3, 1], np.float32)
    assert oracle.select_host(logits, False) == 1
    assert oracle.select_host(logits, True, 1.0, 1, 1.0, word=12345) == 1
    assert oracle.select_host(logits, True, 1.0, 0, 0.25, word=2**63) == 1
    uniform = np.zeros(4, np.float32)
    r = oracle.MT64(51)
    w = r()
    u = (w >> 11) * 2.0**-53
    assert oracle.select_host(uniform, True, 1.0, 0, 0.5, word=w) == (0 if u < 0.5 else 1)
    for t, k, p, cat in ((0.0, 0, 1.0, True), (1.0, 5, 1.0, True), (1.0, 0, 0.0, True),
                         (0.5, 0, 1.0, False)):
        assert oracle.select_host(logits, cat, t, k, p) is None
    bad = logits.copy()
    bad[2] = np.nan
    assert oracle.select_host(bad, False) is None
    assert oracle.select_host(np.full(4, -inf, np.float32), False) is None


def _device_cases(n):
    logits = ((np.arange(n) % 97).astype(np.int64) - 48).astype(np.float32) / np.float32(8)
    logits[0] = np.float32(-0.0)
    if n > 1:
        logits[1] = 0.0
        logits[-1] = -np.inf
    return logits


@needs_ref
@pytest.mark.parametrize("n", [1, 513, 151936])
def test_device_law_equals_host_law_on_reference_cases(n):
    """tests/gpu/test_device.cpp:265-330 asserts device == host here."""
    logits = _device_cases(n)
    for categorical in (False, True):
        for k in (0, min(n, 20)):
            for p in (0.01, 0.5, 0.95, 1.0):
                for seed in range(8):
                    if categorical:
                        t, kk, pp = 0.6, k, p
                    else:
                        t, kk, pp = 1.0, 0, 1.0
                    h = REF_HOST.ref_rng_create(seed)
                    try:
                        expected = _ref_select(logits, categorical, t, kk, pp, h)
                    finally:
                        REF_HOST.ref_rng_destroy(h)
                    word = oracle.MT64(seed)() if categorical else 0
                    token, status = oracle.select_device(logits, categorical, t, kk, pp, word)
                    assert status == 0 and token == expected, (categorical, k, p, seed)


@needs_ref
def test_device_law_mt_continuation_700_draws():
    """tests/gpu/test_device.cpp:332-352: seed 42, n=513, 700 draws."""
    logits = _device_cases(513)
    mine, theirs = oracle.MT64(42), REF_HOST.ref_rng_create(42)
    try:
        for _ in range(700):
            expected = _ref_select(logits, True, 0.6, 0, 0.95, theirs)
            token, status = oracle.select_device(logits, True, 0.6, 0, 0.95, mine())
            assert status == 0 and token == expected
    finally:
        REF_HOST.ref_rng_destroy(theirs)


def test_device_law_status_words():
    nan_row = np.array([0.0, np.nan, 1.0], np.float32)
    assert oracle.select_device(nan_row, False)[1] == 1
    # +inf latches status 1 in initialize, then scan_blocks overwrites it with
    # 2 because +inf as the best value leaves no finite weight (sampling.cu:261-275).
    assert oracle.select_device(np.array([0, np.inf], np.float32), True, 1.0, 0, 0.9, 5)[1] == 2
    # A NaN sorts first under the key law and poisons every weight: status 2.
    assert oracle.select_device(np.array([0, np.nan, 1], np.float32), True, 1.0, 0, 0.9, 5)[1] == 2
    masked = np.full(5, -np.inf, np.float32)
    assert oracle.select_device(masked, False) == (0, 2)
    assert oracle.select_device(masked, True, 1.0, 0, 0.9, 5)[1] == 2


# --------------------------------------------------------------------------
# Op laws vs the reference's independent host equations + tolerances
# (tests/gpu/operator_reference.cpp:167-314, BF16 storage).
# --------------------------------------------------------------------------
ORDINARY = (1e-3, 1.6e-2)
f32 = np.float32


@pytest.mark.parametrize("width", [128, 4096])
def test_rms_norm_law_within_reference_tolerance(width):
    x = nm.operand((3, width), 1)
    w = nm.operand((width,), 2)
    expected = np.empty((3, width), np.float32)
    for r in range(3):
        s = nm.serial_sum_f32(x[r] * x[r])
        inv = f32(1) / np.sqrt(s / f32(width) + f32(1e-6), dtype=np.float32)
        expected[r] = nm.round_bf16(nm.round_bf16(x[r] * inv) * w)
    got = nm.bf16_bits_to_f32(oracle.rms_norm(nm.f32_to_bf16_bits(x), nm.f32_to_bf16_bits(w)))
    assert nm.compare_elementwise(expected, got, 1e-2, 1e-2)["passed"]


def test_silu_and_add_laws_within_reference_tolerance():
    x = nm.operand((3, 259), 3)
    up = nm.operand((3, 259), 4)
    x.reshape(-1)[:3] = [-80, 80, 0]
    expected = nm.round_bf16(nm.round_bf16(x / (f32(1) + np.exp(-x))) * up)
    got = nm.bf16_bits_to_f32(oracle.silu_multiply(nm.f32_to_bf16_bits(x), nm.f32_to_bf16_bits(up)))
    assert nm.compare_elementwise(expected, got, *ORDINARY)["passed"]
    got = nm.bf16_bits_to_f32(oracle.add(nm.f32_to_bf16_bits(x), nm.f32_to_bf16_bits(up)))
    assert nm.compare_elementwise(nm.round_bf16(x + up), got, 0, 0)["passed"]


@pytest.mark.parametrize("rows", [1, 9])
@pytest.mark.parametrize("out", [33, 1025])
def test_projection_law_within_reference_tolerance(rows, out):
    x = nm.operand((rows, 128), 5)
    w = nm.operand((out, 128), 6)
    expected = np.empty((rows, out), np.float32)
    for r in range(rows):
        for o in range(out):
            expected[r, o] = nm.serial_sum_f32(x[r] * w[o])
    expected = nm.round_bf16(expected)
    got = nm.bf16_bits_to_f32(oracle.projection(nm.f32_to_bf16_bits(x), nm.f32_to_bf16_bits(w)))
    assert nm.compare_elementwise(expected, got, *ORDINARY)["passed"]


def test_rotary_law_within_reference_tolerance():
    rows, heads, width, first, theta = 3, 2, 128, 4093, 1e6
    x = nm.operand((rows, heads, width), 7)
    expected = np.empty_like(x)
    for r in range(rows):
        for i in range(width // 2):
            freq = f32(theta ** (-2.0 * i / width))
            angle = f32(first + r) * freq
            c = nm.round_bf16(np.cos(angle, dtype=np.float32))
            s = nm.round_bf16(np.sin(angle, dtype=np.float32))
            a, b = x[r, :, i], x[r, :, i + width // 2]
            expected[r, :, i] = nm.round_bf16(nm.round_bf16(a * c) - nm.round_bf16(b * s))
            expected[r, :, i + width // 2] = nm.round_bf16(nm.round_bf16(b * c) + nm.round_bf16(a * s))
    got = nm.bf16_bits_to_f32(oracle.rotary(nm.f32_to_bf16_bits(x), first, theta))
    assert nm.compare_elementwise(expected, got, *ORDINARY)["passed"]


@pytest.mark.parametrize("rows", [1, 37])
def test_attention_law_within_reference_tolerance(rows):
    heads, kv, width = 4, 2, 128
    scale = f32(1.0 / np.sqrt(width))
    q = nm.operand((rows, heads, width), 8)
    k = nm.operand((rows, kv, width), 9)
    v = nm.operand((rows, kv, width), 10)
    expected = np.empty_like(q)
    for r in range(rows):
        for h in range(heads):
            g = h // (heads // kv)
            s = np.array([nm.serial_sum_f32(q[r, h] * k[j, g]) * scale for j in range(r + 1)], np.float32)
            e = np.exp(s - s.max(), dtype=np.float32)
            p = e / nm.serial_sum_f32(e)
            for f in range(width):
                expected[r, h, f] = nm.serial_sum_f32(p * v[: r + 1, g, f])
    expected = nm.round_bf16(expected)
    got = nm.bf16_bits_to_f32(oracle.attention(nm.f32_to_bf16_bits(q), nm.f32_to_bf16_bits(k),
                                               nm.f32_to_bf16_bits(v), 0))
    assert nm.compare_elementwise(expected, got, 3e-2, 2e-2)["passed"]


# --------------------------------------------------------------------------
# Structural laws that hold bit-exactly without elementary functions
# --------------------------------------------------------------------------
def test_projection_is_row_independent_and_partition_exact():
    rng = np.random.default_rng(3)
    x = nm.f32_to_bf16_bits(rng.standard_normal((5, 4096)).astype(np.float32))
    w = nm.f32_to_bf16_bits((rng.standard_normal((2048, 4096)) * 0.02).astype(np.float32))
    full = oracle.projection(x, w)
    for r in range(5):
        assert np.array_equal(oracle.projection(x[r:r + 1], w)[0], full[r])
    # Restate P=16 (I<=4096, O>1024) by hand for one output.
    xf, wf = nm.bf16_bits_to_f32(x[0]), nm.bf16_bits_to_f32(w[7])
    acc = np.zeros(16, np.float32)
    for m in range(4096 // 16):
        acc = (acc + xf[16 * m:16 * m + 16] * wf[16 * m:16 * m + 16]).astype(np.float32)
    for off in (8, 4, 2, 1):
        acc[:off] = (acc[:off] + acc[off:2 * off]).astype(np.float32)
    assert nm.f32_to_bf16_bits(acc[:1])[0] == full[0, 7]


def test_normal_generator_statistics():
    scale = np.float32(0.02 / np.sqrt(8 * (65536.0 ** 2 - 1) / 12))
    v = nm.bf16_bits_to_f32(oracle.fill_normal_bf16(1 << 20, 1, 5, scale))
    assert abs(float(v.mean())) < 1e-4
    assert abs(float(v.std()) - 0.02) < 2e-4
    ids = oracle.uniform_ids(100000, 1, 9, 151936)
    assert ids.max() < 151936 and ids.min() >= 0
