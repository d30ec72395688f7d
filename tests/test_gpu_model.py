"""Whole-model parity on the GPU.

* The reference's tiny Qwen3 fixture (tests/golden/tiny-bf16): logits and
  captures within the fixture's tolerances, the fixture's greedy IDs, and
  bit-identical logits to the reference's own kernels run on the same weights.
* A Qwen3-8B-shaped model (full widths, two blocks, seeded weights): prompt
  pass and decode steps bit-identical to the reference kernels (logits, KV
  cache, captures), greedy IDs identical, chunking invariance.
* Full Qwen3-8B (36 blocks, BASELINE config 2 shape): greedy token sequence
  identical to the reference kernels for the whole generation.
"""
import numpy as np
import pytest

import dolittle_b200 as dl
from oracle import oracle
from tests import gpu_util as gu
from tests import numerics as nm
from tests import tiny

pytestmark = pytest.mark.gpu
REF = oracle.ref_cuda()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref/libref_cuda.so not built")


def _tiny_engine(capacity=64, max_rows=8):
    c = tiny.config()
    cfg = dl.Qwen3Config(c.hidden, c.query_heads, c.kv_heads, c.head_width, c.mlp_width, c.vocabulary,
                         c.layers, c.epsilon, c.theta)
    e = dl.Engine(cfg, capacity=capacity, max_rows=max_rows)
    e.load_tensors(tiny.tensors())
    return cfg, e


def _ref_for(engine, cfg, capacity, max_rows):
    """Reference kernels over the engine's own device weights; tensors the
    engine stores strided (interleaved gate/up rows) get contiguous copies."""
    ptrs, keep = [], []
    for i in range(cfg.tensor_count()):
        p, stride = engine.tensor_device(i)
        if stride != cfg.tensor_shape(i)[1]:
            t = gu.to_dev(engine.get_tensor(i))
            keep.append(t)
            p = gu.ptr(t)
        ptrs.append(p)
    ref = gu.RefModel(cfg, ptrs, capacity, max_rows)
    ref.keep = keep
    return ref


@needs_ref
def test_tiny_fixture_rows_match_reference_kernels_and_fixture():
    cfg, e = _tiny_engine()
    ref = _ref_for(e, cfg, 64, 8)
    fx = tiny.fixture()
    for case in fx["cases"]:
        e.reset()
        ref = _ref_for(e, cfg, 64, 8)
        toks = case["token_ids"]
        logits = []
        for p, t in enumerate(toks):
            mine = e.consume_view([t])
            theirs, _ = ref.forward([t], p)
            assert np.array_equal(mine, theirs), (case["name"], p)
            logits.append(nm.bf16_bits_to_f32(mine))
        lp = case["logit_positions"]
        tol = case["logits"]["tolerance"]
        r = nm.compare_values(tiny.expected_rows(case["logits"]), np.stack(logits)[lp],
                              tol["max_absolute_error"], tol["max_relative_l2"])
        assert r["passed"], r


def test_tiny_fixture_greedy_generation():
    cfg, e = _tiny_engine()
    gen = tiny.fixture()["generation"]
    toks = gen["reference"]["token_ids"]
    prompt = toks[:gen["prompt_tokens"]]
    out = e.generate(prompt, gen["max_new_tokens"])
    assert prompt + out.tokens == toks
    assert out.status == 0


def _model_8b_shape(layers, capacity, max_rows=8, seed=1):
    cfg = dl.Qwen3Config(layers=layers)
    e = dl.Engine(cfg, capacity=capacity, max_rows=max_rows)
    e.init_random(seed, 0.02)
    return cfg, e


def test_seeded_weights_match_host_generator():
    cfg = dl.Qwen3Config(hidden=256, query_heads=4, kv_heads=2, head_width=64, mlp_width=512,
                         vocabulary=1000, layers=2)
    e = dl.Engine(cfg, capacity=32, max_rows=4)
    e.init_random(7, 0.02)
    scale = np.float32(0.02 / np.sqrt(8 * (65536.0 ** 2 - 1) / 12))
    for i in range(cfg.tensor_count()):
        shape = cfg.tensor_shape(i)
        got = e.get_tensor(i)
        if shape[0] == 1:
            assert np.all(got == nm.f32_to_bf16_bits(np.ones(1, np.float32))[0])
        else:
            exp = oracle.fill_normal_bf16(shape[0] * shape[1], 7, i, scale).reshape(shape)
            assert np.array_equal(got, exp), i


@needs_ref
def test_8b_shape_prefill_and_decode_bit_exact_vs_reference_kernels():
    cap = 256
    cfg, e = _model_8b_shape(2, cap)
    ref = _ref_for(e, cfg, cap, 32)
    prompt = oracle.uniform_ids(21, 1, 101, cfg.vocabulary)
    e.set_capture(1)
    mine = e.consume_view(prompt)
    theirs, cap_ref = ref.forward(prompt, 0, capture_layer=1)
    assert np.array_equal(mine, theirs)
    assert np.array_equal(e.read_capture(0, 21), cap_ref)
    for layer in range(2):
        for values in (False, True):
            rc = gu.from_dev_u16(ref.cache[2 * layer + int(values)])[:21]
            assert np.array_equal(e.read_kv(layer, values, 0, 21), rc)
    # Decode rows: each step's logits and the greedy IDs.
    pos = 21
    tok = int(np.argmax(nm.bf16_bits_to_f32(mine)))
    for _ in range(12):
        mine = e.consume_view([tok])
        theirs, _ = ref.forward([tok], pos)
        assert np.array_equal(mine, theirs), pos
        pos += 1
        tok = oracle.select_host(nm.bf16_bits_to_f32(mine), False)


@needs_ref
def test_8b_shape_generation_graph_matches_reference_greedy():
    cap = 160
    cfg, e = _model_8b_shape(2, cap)
    prompt = oracle.uniform_ids(37, 1, 102, cfg.vocabulary)
    out = e.generate(prompt, 40, want_logits=True)
    assert out.status == 0 and len(out.tokens) == 40
    ref = _ref_for(e, cfg, cap, 64)
    logits, _ = ref.forward(prompt, 0)
    tokens, pos = [], len(prompt)
    for i in range(40):
        assert np.array_equal(out.logits[i], logits), i
        t = oracle.select_host(nm.bf16_bits_to_f32(logits), False)
        tokens.append(t)
        if i + 1 < 40:
            logits, _ = ref.forward([t], pos)
            pos += 1
    assert tokens == out.tokens


def test_fast_prefill_within_tolerance_of_parity_prefill():
    """The tcgen05 prompt pass (tensor-core accumulation order) against the
    parity prompt pass: the 36-block fixture tolerance (max-abs <= 0.0625 x
    peak, relative L2 <= 0.03, forward_reference.py:153-162) on the logits
    and on the KV cache, cosine > 0.999."""
    cap = 200
    cfg, e = _model_8b_shape(2, cap, max_rows=160)
    prompt = oracle.uniform_ids(150, 1, 104, cfg.vocabulary)
    parity = nm.bf16_bits_to_f32(e.consume_view(prompt, dl.DL_PREFILL_PARITY))
    kv_parity = [e.read_kv(l, v, 0, 150) for l in range(2) for v in (False, True)]
    e.reset()
    fast = nm.bf16_bits_to_f32(e.consume_view(prompt, dl.DL_PREFILL_FAST))
    peak = float(np.max(np.abs(parity)))
    r = nm.compare_values(parity, fast, max(1e-4, 0.0625 * peak), 0.03)
    assert r["passed"], r
    assert nm.cosine(parity, fast) > 0.999
    for a, (l, v) in zip(kv_parity, [(l, v) for l in range(2) for v in (False, True)]):
        b = nm.bf16_bits_to_f32(e.read_kv(l, v, 0, 150))
        a = nm.bf16_bits_to_f32(a)
        assert nm.cosine(a, b) > 0.999
        assert nm.compare_values(a, b, max(1e-4, 0.0625 * float(np.max(np.abs(a)))), 0.03)["passed"]
    # Decode continues from the fast cache through the graph.
    out = e.generate(prompt, 4, prefill=dl.DL_PREFILL_FAST)
    assert out.status == 0 and len(out.tokens) == 4


def test_fast_prefill_chunks_within_tolerance_of_parity_prefill():
    """Fast prompt pass in 128-row chunks (later chunks attend cached keys
    through the tensor-core attention) against the parity pass: same
    tolerance as the single-chunk case."""
    cap = 320
    cfg, e = _model_8b_shape(2, cap, max_rows=128)
    prompt = oracle.uniform_ids(300, 1, 105, cfg.vocabulary)
    parity = nm.bf16_bits_to_f32(e.consume_view(prompt, dl.DL_PREFILL_PARITY))
    e.reset()
    fast = nm.bf16_bits_to_f32(e.consume_view(prompt, dl.DL_PREFILL_FAST))
    peak = float(np.max(np.abs(parity)))
    r = nm.compare_values(parity, fast, max(1e-4, 0.0625 * peak), 0.03)
    assert r["passed"], r
    assert nm.cosine(parity, fast) > 0.999


@needs_ref
def test_chunked_prefill_is_bit_invariant():
    cap = 64
    cfg, e = _model_8b_shape(2, cap, max_rows=8)
    prompt = oracle.uniform_ids(19, 1, 103, cfg.vocabulary)
    whole = e.consume_view(prompt)
    kv_whole = [e.read_kv(l, v, 0, 19) for l in range(2) for v in (False, True)]
    e.reset()
    e.consume_view(prompt[:3])
    e.consume_view(prompt[3:11])
    split = e.consume_view(prompt[11:])
    assert np.array_equal(whole, split)
    assert all(np.array_equal(a, e.read_kv(l, v, 0, 19))
               for a, (l, v) in zip(kv_whole, [(l, v) for l in range(2) for v in (False, True)]))


@needs_ref
def test_full_qwen3_8b_config2_greedy_tokens_identical_to_reference():
    """BASELINE config 2 shape: 36 blocks, V=151936, seeded weights (seed 1),
    512 uniform prompt IDs, 256 greedy decode steps.  The whole generated
    sequence must equal the reference kernels' sequence."""
    prompt_len, steps = 512, 256
    cap = prompt_len + steps + 8
    cfg, e = _model_8b_shape(36, cap, seed=1)
    prompt = oracle.uniform_ids(prompt_len, 1, 0, cfg.vocabulary)
    out = e.generate(prompt, steps + 1)
    assert out.status == 0 and len(out.tokens) == steps + 1
    ref = _ref_for(e, cfg, cap, prompt_len)
    logits, _ = ref.forward(prompt, 0)
    tokens, pos = [], prompt_len
    for i in range(steps + 1):
        t = oracle.select_host(nm.bf16_bits_to_f32(logits), False)
        tokens.append(t)
        if i < steps:
            logits, _ = ref.forward([t], pos)
            pos += 1
    first_diff = next((i for i, (a, b) in enumerate(zip(tokens, out.tokens)) if a != b), None)
    assert first_diff is None, f"first divergence at generated index {first_diff}"
