"""Operation parity on the GPU, through the C ABI.

Each sm_100a operation is compared bit-for-bit with the reference's own CUDA
kernel (oracle/_ref/libref_cuda.so: the reference sources compiled for
compute_86 PTX and JIT-compiled on this B200) on identical device inputs, and
with the CPU oracle: bit-exact where the law has no elementary function
(projection, add, embedding), within the reference's own tolerances
(tests/gpu/operator_reference.cpp) otherwise.
"""
import ctypes as C

import numpy as np
import pytest

import dolittle_b200 as dl
from oracle import oracle
from tests import gpu_util as gu
from tests import numerics as nm

pytestmark = pytest.mark.gpu
REF = oracle.ref_cuda()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref/libref_cuda.so not built")
BF = dl.DL_BF16


def _lib():
    return dl.lib()


# ---------------------------------------------------------------------------
# Projection (the decode GEMV law; rows > 1 = prefill rows)
# ---------------------------------------------------------------------------
PROJ_SHAPES = [(1, 4096, 4096), (1, 4096, 1024), (1, 12288, 4096), (1, 4096, 12288),
               (8, 4096, 4096), (3, 4096, 1024), (5, 12288, 4096), (16, 4096, 6144),
               (1, 24, 32), (4, 24, 16), (3, 40, 24), (2, 32, 24), (1, 4096, 151936)]


@pytest.mark.parametrize("rows,I,O", PROJ_SHAPES)
def test_projection_bit_exact(rows, I, O):
    x = gu.rand_bf16((rows, I), 1.0, seed=rows * 7 + I)
    w = gu.rand_bf16((O, I), 0.02, seed=O + 3)
    dx, dw = gu.to_dev(x), gu.to_dev(w)
    mine = gu.zeros_dev((rows, O))
    gu.sync()
    dl.lib().dl_projection(BF, gu.ptr(dx), gu.ptr(dw), gu.ptr(mine), rows, I, O, None, None)
    gu.sync()
    got = gu.from_dev_u16(mine)
    if O <= 16384:
        assert np.array_equal(got, oracle.projection(x, w)), "differs from the CPU law"
    if REF is not None:
        ref = gu.zeros_dev((rows, O))
        assert REF.ref_projection(1, gu.ptr(dx), gu.ptr(dw), gu.ptr(ref), rows, I, O, None, None) == 0
        gu.sync()
        assert np.array_equal(got, gu.from_dev_u16(ref)), "differs from the reference kernel"


def test_projection_positioned_output_appends_rows():
    rows, I, O = 2, 4096, 1024
    x, w = gu.rand_bf16((rows, I), seed=1), gu.rand_bf16((O, I), 0.02, seed=2)
    cache = gu.zeros_dev((16, O))
    pos = gu.to_dev(np.array([5], np.int64))
    dl.lib().dl_projection(BF, gu.ptr(gu.to_dev(x)), gu.ptr(gu.to_dev(w)), gu.ptr(cache), rows, I, O, None,
                           gu.ptr(pos))
    gu.sync()
    got = gu.from_dev_u16(cache)
    assert np.array_equal(got[5:7], oracle.projection(x, w))
    assert not got[:5].any() and not got[7:].any()


# ---------------------------------------------------------------------------
# RMSNorm, RoPE, attention, elementwise
# ---------------------------------------------------------------------------
@needs_ref
@pytest.mark.parametrize("rows,width", [(3, 4096), (40, 128), (5, 24), (8, 8), (2, 12288)])
def test_rms_norm_bit_exact(rows, width):
    x = gu.rand_bf16((rows, width), 1.0, seed=width)
    w = gu.rand_bf16((width,), 0.5, seed=width + 1)
    dx, dw = gu.to_dev(x), gu.to_dev(w)
    mine, ref = gu.zeros_dev((rows, width)), gu.zeros_dev((rows, width))
    assert dl.lib().dl_rms_norm(BF, gu.ptr(dx), gu.ptr(dw), gu.ptr(mine), rows, width, 1e-6, None) == 0
    # The reference uses its warp kernel above 8192 columns and the staged
    # kernel in (128, 8192]; both share one law.
    assert REF.ref_rms_norm(1, gu.ptr(dx), gu.ptr(dw), gu.ptr(ref), rows, width, 1e-6, None) == 0
    gu.sync()
    got = gu.from_dev_u16(mine)
    assert np.array_equal(got, gu.from_dev_u16(ref))
    exp = nm.bf16_bits_to_f32(oracle.rms_norm(x, w))
    assert nm.compare_elementwise(exp, nm.bf16_bits_to_f32(got), 1e-2, 1e-2)["passed"]


@needs_ref
@pytest.mark.parametrize("rows,heads,width,first,theta", [(3, 2, 128, 4093, 1e6), (5, 32, 128, 700, 1e6),
                                                        (4, 4, 8, 9, 1e4)])
def test_rotary_bit_exact(rows, heads, width, first, theta):
    x = gu.rand_bf16((rows, heads, width), 1.0, seed=first)
    dx = gu.to_dev(x)
    mine, ref = gu.zeros_dev(x.shape), gu.zeros_dev(x.shape)
    assert dl.lib().dl_rotary(BF, gu.ptr(dx), gu.ptr(mine), rows, heads, width, first, theta, None, None, 0) == 0
    assert REF.ref_rotary(1, gu.ptr(dx), gu.ptr(ref), rows, heads, width, first, theta, None, None, 0) == 0
    gu.sync()
    assert np.array_equal(gu.from_dev_u16(mine), gu.from_dev_u16(ref))
    exp = nm.bf16_bits_to_f32(oracle.rotary(x, first, theta))
    assert nm.compare_elementwise(exp, nm.bf16_bits_to_f32(gu.from_dev_u16(mine)), 1e-3, 1.6e-2)["passed"]


@needs_ref
@pytest.mark.parametrize("rows,first,H,G,d", [(1, 700, 32, 8, 128), (1, 0, 32, 8, 128), (37, 0, 32, 8, 128),
                                               (16, 300, 32, 8, 128), (6, 3, 4, 2, 8), (1, 2047, 32, 8, 128)])
def test_attention_bit_exact(rows, first, H, G, d):
    total = first + rows
    q = gu.rand_bf16((rows, H, d), 1.0, seed=rows + first)
    k = gu.rand_bf16((total, G, d), 1.0, seed=total)
    v = gu.rand_bf16((total, G, d), 1.0, seed=total + 1)
    dq, dk, dv = gu.to_dev(q), gu.to_dev(k), gu.to_dev(v)
    mine, ref = gu.zeros_dev(q.shape), gu.zeros_dev(q.shape)
    ws = gu.zeros_dev((dl.lib().dl_attention_workspace_bytes(rows, H, total) // 2 + 8,))
    scale = gu.zeros_dev((2,), 4)
    assert REF.ref_attention_scale(gu.ptr(scale), d, None) == 0
    assert dl.lib().dl_attention(BF, gu.ptr(dq), gu.ptr(dk), gu.ptr(dv), gu.ptr(mine), rows, H, G, d, None,
                                 first, None, total, gu.ptr(scale), gu.ptr(ws)) == 0
    assert REF.ref_attention(1, gu.ptr(dq), gu.ptr(dk), gu.ptr(dv), gu.ptr(ref), rows, H, G, d, None, first,
                             None, total, gu.ptr(scale)) == 0
    gu.sync()
    got = gu.from_dev_u16(mine)
    assert np.array_equal(got, gu.from_dev_u16(ref))
    exp = nm.bf16_bits_to_f32(oracle.attention(q, k, v, first))
    assert nm.compare_elementwise(exp, nm.bf16_bits_to_f32(got), 3e-2, 2e-2)["passed"]


@needs_ref
def test_add_silu_embedding_bit_exact():
    n = 3 * 259
    g = gu.rand_bf16((n,), 3.0, seed=1)
    u = gu.rand_bf16((n,), 1.0, seed=2)
    g[:3] = nm.f32_to_bf16_bits(np.array([-80, 80, 0], np.float32))
    dg, du = gu.to_dev(g), gu.to_dev(u)
    for fn, rf, law in ((dl.lib().dl_add, REF.ref_add, oracle.add),
                        (dl.lib().dl_silu_multiply, REF.ref_silu_multiply, oracle.silu_multiply)):
        mine, ref = gu.zeros_dev((n,)), gu.zeros_dev((n,))
        assert fn(BF, gu.ptr(dg), gu.ptr(du), gu.ptr(mine), n, None) == 0
        assert rf(1, gu.ptr(dg), gu.ptr(du), gu.ptr(ref), n, None) == 0
        gu.sync()
        assert np.array_equal(gu.from_dev_u16(mine), gu.from_dev_u16(ref))
        exp = nm.bf16_bits_to_f32(law(g, u))
        assert nm.compare_elementwise(exp, nm.bf16_bits_to_f32(gu.from_dev_u16(mine)), 1e-3, 1.6e-2)["passed"]
    table = gu.rand_bf16((37, 24), 1.0, seed=5)
    ids = np.array([3, 0, 36, 7], np.uint32)
    out = gu.zeros_dev((4, 24))
    assert dl.lib().dl_embedding(BF, gu.ptr(gu.to_dev(ids)), gu.ptr(gu.to_dev(table)), gu.ptr(out), 4, 24,
                                 None) == 0
    gu.sync()
    assert np.array_equal(gu.from_dev_u16(out), table[ids])


@needs_ref
@pytest.mark.parametrize("rows,first", [(1, 511), (8, 16)])
def test_qk_norm_rope_append_matches_reference_composition(rows, first):
    H, G, d, theta, eps = 32, 8, 128, 1e6, 1e-6
    qr = gu.rand_bf16((rows, H, d), 1.0, seed=11)
    kr = gu.rand_bf16((rows, G, d), 1.0, seed=12)
    qw = gu.rand_bf16((d,), 0.5, seed=13)
    kw = gu.rand_bf16((d,), 0.5, seed=14)
    dqr, dkr, dqw, dkw = map(gu.to_dev, (qr, kr, qw, kw))
    inv = gu.zeros_dev((d // 2,), 4)
    assert dl.lib().dl_rope_inverse_frequency(gu.ptr(inv), d, theta, None) == 0
    pos = gu.to_dev(np.array([first], np.int64))
    q_out, cache = gu.zeros_dev((rows, H, d)), gu.zeros_dev((first + rows + 4, G, d))
    assert dl.lib().dl_qk_norm_rope_append(gu.ptr(dqr), gu.ptr(dkr), gu.ptr(dqw), gu.ptr(dkw), gu.ptr(inv),
                                           gu.ptr(q_out), gu.ptr(cache), gu.ptr(pos), rows, H, G, d, eps,
                                           None) == 0
    # Reference composition: rms_norm(q) -> rotary(q); rms_norm(k) -> rotary(k) positioned into the cache.
    q2, k2 = gu.zeros_dev(qr.shape), gu.zeros_dev(kr.shape)
    rq, rcache = gu.zeros_dev(qr.shape), gu.zeros_dev((first + rows + 4, G, d))
    assert REF.ref_rms_norm(1, gu.ptr(dqr), gu.ptr(dqw), gu.ptr(q2), rows * H, d, eps, None) == 0
    assert REF.ref_rotary(1, gu.ptr(q2), gu.ptr(rq), rows, H, d, first, theta, None, None, 0) == 0
    assert REF.ref_rms_norm(1, gu.ptr(dkr), gu.ptr(dkw), gu.ptr(k2), rows * G, d, eps, None) == 0
    assert REF.ref_rotary(1, gu.ptr(k2), gu.ptr(rcache), rows, G, d, first, theta, None, None, 1) == 0
    gu.sync()
    assert np.array_equal(gu.from_dev_u16(q_out), gu.from_dev_u16(rq))
    assert np.array_equal(gu.from_dev_u16(cache), gu.from_dev_u16(rcache))


# ---------------------------------------------------------------------------
# Sampler: device law vs the reference's DeviceCategorical on the same rows
# ---------------------------------------------------------------------------
def _device_cases(n):
    logits = ((np.arange(n) % 97).astype(np.int64) - 48).astype(np.float32) / np.float32(8)
    logits[0] = np.float32(-0.0)
    if n > 1:
        logits[1] = 0.0
        logits[-1] = -np.inf
    return logits


class _Sampler:
    def __init__(self, n, bf16):
        self.h = C.c_void_p()
        assert dl.lib().dl_sampler_create(n, BF if bf16 else dl.DL_F32, C.byref(self.h)) == 0

    def submit(self, row_dev, settings, bits):
        res = C.c_void_p()
        s = settings.c()
        assert dl.lib().dl_sampler_submit(self.h, gu.ptr(row_dev), C.byref(s), bits, None, C.byref(res)) == 0
        return self._read(res)

    def _read(self, res):
        gu.sync()
        out = (C.c_uint32 * 2)()
        cudart = C.CDLL("libcudart.so.12")   # the runtime the product library links
        assert cudart.cudaMemcpy(out, C.c_void_p(res.value), 8, 2) == 0
        return out[0], out[1]

    def close(self):
        dl.lib().dl_sampler_destroy(self.h)


@needs_ref
# 8449 keys = 33 radix blocks + 1: uneven block segments in the offset scan.
@pytest.mark.parametrize("n", [1, 513, 8449, 151936])
@pytest.mark.parametrize("bf16", [True, False])
def test_sampler_matches_reference_device_sampler(n, bf16):
    logits = _device_cases(n)
    row = gu.to_dev(nm.f32_to_bf16_bits(logits) if bf16 else logits)
    smp = _Sampler(n, bf16)
    try:
        for categorical in (False, True):
            for k in (0, min(n, 20)):
                for p in (0.01, 0.5, 0.95, 1.0):
                    for seed in range(4):
                        if categorical:
                            st = dl.Settings(dl.SelectionMode.categorical, 0.6, k, p)
                        else:
                            st = dl.Settings()
                        bits = oracle.MT64(seed)() if categorical else 0
                        got = smp.submit(row, st, bits)
                        ref = np.zeros(2, np.uint32)
                        assert REF.ref_device_select(np.ascontiguousarray(logits), n, int(bf16), int(categorical),
                                                     st.temperature, st.top_k, st.top_p, bits, ref) == 0
                        assert got == (int(ref[0]), int(ref[1])), (categorical, k, p, seed)
                        law = oracle.select_device(logits, categorical, st.temperature, st.top_k, st.top_p, bits)
                        assert got == law
    finally:
        smp.close()


@needs_ref
def test_sampler_owned_stream_matches_reference_700_draws():
    n = 513
    logits = _device_cases(n)
    row = gu.to_dev(logits)
    smp = _Sampler(n, False)
    st = dl.Settings(dl.SelectionMode.categorical, 0.6, 0, 0.95)
    s = st.c()
    assert dl.lib().dl_sampler_start(smp.h, C.byref(s), 42, None, 0, None) == 0
    ref = np.zeros(2 * 700, np.uint32)
    assert REF.ref_device_sequence(np.ascontiguousarray(logits), n, 0, 0.6, 0, 0.95, 42, 700, ref) == 0
    try:
        for i in range(700):
            res = C.c_void_p()
            assert dl.lib().dl_sampler_submit_next(smp.h, gu.ptr(row), None, C.byref(res)) == 0
            assert smp._read(res) == (int(ref[2 * i]), int(ref[2 * i + 1]))
    finally:
        smp.close()


def test_sampler_status_words_on_nonfinite_rows():
    smp = _Sampler(3, False)
    try:
        assert smp.submit(gu.to_dev(np.array([0, np.nan, 1], np.float32)), dl.Settings(), 0)[1] == 1
        assert smp.submit(gu.to_dev(np.full(3, -np.inf, np.float32)), dl.Settings(), 0) == (0, 2)
    finally:
        smp.close()


# ---------------------------------------------------------------------------
# Steering edit and injection normalisation (bit-exact vs the CPU law: no
# elementary functions beyond the correctly rounded sqrt)
# ---------------------------------------------------------------------------
def test_intervene_and_injection_bit_exact_vs_law():
    D, rows, first, selected = 4096, 3, 198, 200
    h = gu.rand_bf16((rows, D), 1.0, seed=21)
    u = np.random.default_rng(22).standard_normal(D).astype(np.float32)
    u /= np.linalg.norm(u)
    dh = gu.to_dev(h)
    state = gu.zeros_dev((2,), 4)
    pos = gu.to_dev(np.array([first], np.int64))
    assert dl.lib().dl_intervene(gu.ptr(dh), gu.ptr(gu.to_dev(u)), gu.ptr(pos), gu.ptr(state), D, selected, rows,
                                 4.0, None) == 0
    gu.sync()
    exp = h.copy()
    st = np.zeros(2, np.uint32)
    oracle.lib().or_intervene(exp, u, D, selected, first, rows, 4.0, st)
    assert np.array_equal(gu.from_dev_u16(dh), exp)
    assert gu.torch().equal(state.cpu(), gu.torch().tensor([0, 1], dtype=gu.torch().int32))
    # Injection: (h/||h||)*150 into the marker row.
    src = gu.rand_bf16((D,), 1.0, seed=23)
    out, norm, status = gu.zeros_dev((D,)), gu.zeros_dev((1,), 4), gu.zeros_dev((1,), 4)
    assert dl.lib().dl_normalize_injection(gu.ptr(gu.to_dev(src)), gu.ptr(out), gu.ptr(norm), gu.ptr(status), D,
                                           150.0, None) == 0
    gu.sync()
    exp2 = np.empty(D, np.uint16)
    nrm = C.c_float()
    assert oracle.lib().or_normalize_injection(src, exp2, D, 150.0, C.byref(nrm)) == 0
    assert np.array_equal(gu.from_dev_u16(out), exp2)


# ---------------------------------------------------------------------------
# Philox4x32-10 draw source (selectable; the reference's stream is MT19937-64)
# ---------------------------------------------------------------------------
def test_sampler_philox_stream_matches_law_and_is_deterministic():
    """Draw k of row 0 comes from the Philox block at counter k under key
    seed; each selection equals the device law (oracle) given that word.
    Same seed -> same sequence; another seed -> another sequence."""
    n = 8449
    logits = _device_cases(n)
    row = gu.to_dev(nm.f32_to_bf16_bits(logits))
    st = dl.Settings(dl.SelectionMode.categorical, 0.7, 0, 0.9)

    def run(seed, draws):
        smp = _Sampler(n, True)
        try:
            assert dl.lib().dl_sampler_set_engine(smp.h, dl.DL_RNG_PHILOX4X32_10) == 0
            s = st.c()
            assert dl.lib().dl_sampler_start(smp.h, C.byref(s), seed, None, 0, None) == 0
            # The engine is fixed once the stream is seeded.
            assert dl.lib().dl_sampler_set_engine(smp.h, dl.DL_RNG_MT19937_64) != 0
            out = []
            for _ in range(draws):
                res = C.c_void_p()
                assert dl.lib().dl_sampler_submit_next(smp.h, gu.ptr(row), None, C.byref(res)) == 0
                out.append(smp._read(res))
            return out
        finally:
            smp.close()

    bf = nm.bf16_bits_to_f32(nm.f32_to_bf16_bits(logits))
    a = run(7, 64)
    for k, got in enumerate(a):
        want = oracle.select_device(bf, True, st.temperature, st.top_k, st.top_p, oracle.philox_word(7, k))
        assert got == want, k
    assert run(7, 64) == a
    assert run(8, 64) != a


def test_engine_generation_with_philox_draws_matches_law():
    """A categorical generation through the engine's device loop with the
    Philox source: every selected token equals the device law on that step's
    logits with draw k of the stream seeded with the generation's seed."""
    cfg = dl.Qwen3Config(hidden=256, query_heads=4, kv_heads=2, head_width=64, mlp_width=512,
                         vocabulary=1000, layers=2)
    e = dl.Engine(cfg, capacity=64, max_rows=8)
    e.init_random(3, 0.02)
    e.set_sampler_engine(dl.DL_RNG_PHILOX4X32_10)
    st = dl.Settings(dl.SelectionMode.categorical, 0.9, 0, 0.95)
    prompt = oracle.uniform_ids(9, 1, 3, cfg.vocabulary)
    g = e.generate(prompt, 12, settings=st, seed=11, want_logits=True)
    assert g.status == 0 and len(g.tokens) == 12
    for k in range(12):
        want = oracle.select_device(nm.bf16_bits_to_f32(g.logits[k]), True, st.temperature, st.top_k, st.top_p,
                                    oracle.philox_word(11, k))
        assert g.tokens[k] == want[0], k
    # The reference's MT19937-64 stream stays the default (and selectable).
    e.set_sampler_engine(dl.DL_RNG_MT19937_64)
    g2 = e.generate(prompt, 12, settings=st, seed=11, want_logits=True)
    mt = oracle.MT64(11)
    for k in range(12):
        want = oracle.select_device(nm.bf16_bits_to_f32(g2.logits[k]), True, st.temperature, st.top_k, st.top_p, mt())
        assert g2.tokens[k] == want[0], k
    e.close()
