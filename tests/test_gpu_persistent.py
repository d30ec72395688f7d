"""The persistent decode step (one cooperative kernel per token) against the
per-operation decode kernels and the reference kernels.

Both decode paths compute the reference's arithmetic, so every generated
token, every step's logits, the KV cache, block captures and steering edits
must be bit-identical between them; the 8B-shaped case is also checked
directly against the reference's own kernels.
"""
import numpy as np
import pytest

import dolittle_b200 as dl
from oracle import oracle
from tests import gpu_util as gu
from tests import numerics as nm

pytestmark = pytest.mark.gpu
REF = oracle.ref_cuda()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref/libref_cuda.so not built")


def _engine(cfg, capacity, seed=1, max_rows=8):
    e = dl.Engine(cfg, capacity=capacity, max_rows=max_rows)
    e.init_random(seed, 0.02)
    return e


def _run(e, path, prompt, n, **kw):
    e.set_decode_path(path)
    return e.generate(prompt, n, want_logits=True, **kw)


def _kv(e, cfg, count):
    return [e.read_kv(l, v, 0, count) for l in range(cfg.layers) for v in (False, True)]


SHAPES = [
    dl.Qwen3Config(layers=2),
    # Other GQA group / widths: group 4 with 16 heads, group 2, ragged vocabulary.
    dl.Qwen3Config(hidden=1024, query_heads=16, kv_heads=4, head_width=128, mlp_width=3072, vocabulary=5003,
                   layers=3),
    dl.Qwen3Config(hidden=512, query_heads=8, kv_heads=4, head_width=64, mlp_width=1536, vocabulary=777,
                   layers=2),
]


@pytest.mark.parametrize("cfg", SHAPES, ids=["8b-2blocks", "d1024-g4", "d512-g2-w64"])
def test_persistent_greedy_matches_kernel_path(cfg):
    cap = 200
    e = _engine(cfg, cap)
    prompt = oracle.uniform_ids(45, 1, 201, cfg.vocabulary)
    kern = _run(e, dl.DL_DECODE_KERNELS, prompt, 40)
    kv_kern = _kv(e, cfg, 45 + 39)
    pers = _run(e, dl.DL_DECODE_PERSISTENT, prompt, 40)
    assert pers.status == 0 and kern.status == 0
    assert pers.kernels_per_decode_step == 1
    assert pers.tokens == kern.tokens
    assert np.array_equal(pers.logits, kern.logits)
    for a, b in zip(kv_kern, _kv(e, cfg, 45 + 39)):
        assert np.array_equal(a, b)


def test_persistent_capture_and_steering_match_kernel_path():
    cfg = dl.Qwen3Config(layers=3)
    cap = 160
    e = _engine(cfg, cap)
    prompt = oracle.uniform_ids(30, 1, 202, cfg.vocabulary)
    rng = np.random.default_rng(5)
    u = rng.standard_normal(cfg.hidden).astype(np.float32)
    u /= np.linalg.norm(u)
    out = {}
    for path in (dl.DL_DECODE_KERNELS, dl.DL_DECODE_PERSISTENT):
        e.set_capture(1)
        e.set_intervention(1, 36, 4.0, u)   # a decode row: the edit lands inside the step kernel
        g = _run(e, path, prompt, 20)
        out[path] = (g, e.read_capture(0, 30 + 19))
        e.set_intervention(-1)
        e.set_capture(-1)
    (gk, ck), (gp, cp) = out[dl.DL_DECODE_KERNELS], out[dl.DL_DECODE_PERSISTENT]
    assert gk.tokens == gp.tokens
    assert np.array_equal(gk.logits, gp.logits)
    assert np.array_equal(ck, cp)


def test_persistent_capture_without_edit_matches_kernel_path():
    cfg = dl.Qwen3Config(layers=2)
    e = _engine(cfg, 128)
    prompt = oracle.uniform_ids(20, 1, 203, cfg.vocabulary)
    caps = []
    for path in (dl.DL_DECODE_KERNELS, dl.DL_DECODE_PERSISTENT):
        e.set_capture(0)
        _run(e, path, prompt, 12)
        caps.append(e.read_capture(0, 31))
    assert np.array_equal(caps[0], caps[1])


def test_persistent_categorical_matches_kernel_path():
    cfg = dl.Qwen3Config(layers=2)
    e = _engine(cfg, 160)
    prompt = oracle.uniform_ids(25, 1, 204, cfg.vocabulary)
    s = dl.Settings(dl.SelectionMode.categorical, temperature=0.7, top_p=0.9)
    a = _run(e, dl.DL_DECODE_KERNELS, prompt, 30, settings=s, seed=7)
    b = _run(e, dl.DL_DECODE_PERSISTENT, prompt, 30, settings=s, seed=7)
    assert a.tokens == b.tokens
    assert np.array_equal(a.logits, b.logits)


@needs_ref
def test_persistent_decode_bit_exact_vs_reference_kernels():
    cfg = dl.Qwen3Config(layers=2)
    cap = 128
    e = _engine(cfg, cap)
    prompt = oracle.uniform_ids(33, 1, 205, cfg.vocabulary)
    out = _run(e, dl.DL_DECODE_PERSISTENT, prompt, 24)
    ref = gu.RefModel(cfg, [_contig(e, cfg, i) for i in range(cfg.tensor_count())], cap, 64)
    logits, _ = ref.forward(prompt, 0)
    pos = len(prompt)
    for i in range(24):
        assert np.array_equal(out.logits[i], logits), i
        t = oracle.select_host(nm.bf16_bits_to_f32(logits), False)
        assert t == out.tokens[i]
        if i + 1 < 24:
            logits, _ = ref.forward([t], pos)
            pos += 1


_KEEP = []


def _contig(e, cfg, i):
    p, stride = e.tensor_device(i)
    if stride != cfg.tensor_shape(i)[1]:
        t = gu.to_dev(e.get_tensor(i))
        _KEEP.append(t)
        return gu.ptr(t)
    return p
