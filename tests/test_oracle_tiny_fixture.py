"""Pin the oracle's whole-model composition against the reference's own
Python oracle (scripts/validation/forward_reference.py), whose outputs are
committed in tests/golden/tiny-bf16 (regenerate with make_tiny_fixture.py).

The oracle runs the reference kernel laws row by row with a KV cache (the
reference's cached path); the fixture is an independent FP32 policy, so the
comparison uses the fixture's own per-output tolerances (max-abs bound and
relative L2, forward_reference.py:153-162) and reports cosine similarity.
Greedy generation must reproduce the fixture's four generated IDs.
"""
import numpy as np
import pytest

from oracle import oracle
from tests import numerics as nm
from tests import tiny


def _run_rows(model, tokens):
    """Feed tokens one row at a time; return per-position logits and every
    block output (captures) as FP32."""
    cfg = model.cfg
    logits, caps = [], []
    for p, t in enumerate(tokens):
        out, cap = model.forward([t], p, logits=True, capture_layer=-2)
        logits.append(nm.bf16_bits_to_f32(out))
        caps.append(nm.bf16_bits_to_f32(cap[:, 0, :]))
    return np.stack(logits), np.stack(caps)       # [P][V], [P][L][D]


def _check_case(case, logits, caps, embed):
    lp = case["logit_positions"]
    res = nm.compare_values(tiny.expected_rows(case["logits"]),
                            logits[lp], case["logits"]["tolerance"]["max_absolute_error"],
                            case["logits"]["tolerance"]["max_relative_l2"])
    assert res["passed"], res
    for cap in case["captures"]:
        pos, block = cap["positions"], cap["block"]
        if cap["boundary"] == "block_output":
            got = caps[pos, block]
        elif block == 0:
            got = embed[pos]
        else:
            got = caps[pos, block - 1]
        tol = cap["tolerance"]
        r = nm.compare_values(tiny.expected_rows(cap), got, tol["max_absolute_error"],
                              tol["max_relative_l2"])
        assert r["passed"], (cap["boundary"], block, r)
        assert nm.cosine(tiny.expected_rows(cap), got) > 0.999


@pytest.fixture(scope="module")
def tiny_model():
    cfg = tiny.config()
    return cfg, tiny.tensors()


@pytest.mark.parametrize("name", ["full", "prefix", "alternate"])
def test_oracle_matches_reference_fixture_cases(tiny_model, name):
    cfg, tensors = tiny_model
    fx = tiny.fixture()
    case = next(c for c in fx["cases"] if c["name"] == name)
    model = oracle.OracleModel(cfg, tensors, capacity=64)
    logits, caps = _run_rows(model, case["token_ids"])
    embed = nm.bf16_bits_to_f32(tensors[0])[case["token_ids"]]
    _check_case(case, logits, caps, embed)


def test_oracle_greedy_generation_matches_reference_fixture(tiny_model):
    cfg, tensors = tiny_model
    gen = tiny.fixture()["generation"]
    ref = gen["reference"]
    prompt = ref["token_ids"][:gen["prompt_tokens"]]
    model = oracle.OracleModel(cfg, tensors, capacity=64)
    out, _ = model.forward(prompt, 0)                 # prefill as one chunk
    tokens = list(prompt)
    for _ in range(gen["max_new_tokens"]):
        tok = oracle.select_host(nm.bf16_bits_to_f32(out), False)
        tokens.append(tok)
        out, _ = model.forward([tok], len(tokens) - 1)
    assert tokens == ref["token_ids"]
    # The cached trace (all rows) within the fixture's tolerances.
    model2 = oracle.OracleModel(cfg, tensors, capacity=64)
    logits, caps = _run_rows(model2, ref["token_ids"])
    embed = nm.bf16_bits_to_f32(tensors[0])[ref["token_ids"]]
    _check_case(ref, logits, caps, embed)


def test_prefill_chunking_is_bit_invariant(tiny_model):
    """Reference contract: cached chunks equal the uncached pass byte for byte
    (tests/gpu/test_generation.cpp:462-560)."""
    cfg, tensors = tiny_model
    toks = [(i * 7 + 3) % 37 for i in range(17)]
    a = oracle.OracleModel(cfg, tensors, capacity=64)
    whole, cap_a = a.forward(toks, 0, capture_layer=-2)
    b = oracle.OracleModel(cfg, tensors, capacity=64)
    b.forward(toks[:3], 0)
    b.forward(toks[3:10], 3)
    split, _ = b.forward(toks[10:], 10)
    assert np.array_equal(whole, split)
    assert all(np.array_equal(a.cache[i], b.cache[i]) for i in range(len(a.cache)))
