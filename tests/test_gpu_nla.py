"""NLA pair paths on the GPU: checkpoint loading, verbalizer (AV) injection
and the reconstructor (AR) forward-only head.

* A checkpoint directory opens into an engine that reproduces the tiny
  fixture's greedy IDs.
* Injection at a marker position equals running the same prompt with that
  token's embedding row replaced by the injection law's vector (the oracle's
  BF16((h/||h||)*scale)), bit for bit.
* Reconstruction equals the oracle: the last position's block output
  (no final norm) through the D x D head under the projection law.
"""
import ctypes as C

import numpy as np
import pytest

import dolittle_b200 as dl
from dolittle_b200 import checkpoint
from oracle import oracle
from tests import tiny

pytestmark = pytest.mark.gpu


def test_open_qwen3_reproduces_the_tiny_fixture():
    e = checkpoint.open_qwen3(tiny.HERE, capacity=64, max_rows=8)
    gen = tiny.fixture()["generation"]
    toks = gen["reference"]["token_ids"]
    prompt = toks[:gen["prompt_tokens"]]
    out = e.generate(prompt, gen["max_new_tokens"])
    assert prompt + out.tokens == toks


def _engine(cfg, cap=64):
    e = dl.Engine(cfg, capacity=cap, max_rows=8)
    e.init_random(3, 0.02)
    return e


def _oracle_injection(h, scale):
    out = np.empty_like(h)
    norm = C.c_float()
    status = oracle.lib().or_normalize_injection(np.ascontiguousarray(h), out, h.size, scale, C.byref(norm))
    assert status == 0
    return out


@pytest.mark.parametrize("path", [dl.DL_DECODE_PERSISTENT, dl.DL_DECODE_KERNELS])
def test_injection_equals_embedding_row_replacement(path):
    cfg = dl.Qwen3Config(hidden=1024, query_heads=16, kv_heads=4, head_width=128, mlp_width=3072, vocabulary=2048,
                         layers=2)
    e = _engine(cfg)
    e.set_decode_path(path)
    marker, p = 2047, 7
    prompt = [int(t) % 2000 for t in oracle.uniform_ids(20, 2, 7, cfg.vocabulary)]
    prompt[p] = marker
    rng = np.random.default_rng(11)
    h = (rng.standard_normal(cfg.hidden).astype(np.float32) * 3).astype(np.float32)
    h_bits = (h.view(np.uint32) >> 16).astype(np.uint16)
    e.set_injection(p, h_bits, 150.0)
    injected = e.consume_view(prompt)
    gen_injected = e.generate(prompt, 6)
    # The same prompt with the marker's embedding row replaced by the law's vector.
    e.set_injection(-1)
    emb = e.get_tensor(0)
    emb[marker] = _oracle_injection(h_bits, 150.0)
    e.set_tensor(0, emb)
    e.reset()
    replaced = e.consume_view(prompt)
    assert np.array_equal(injected, replaced)
    assert e.generate(prompt, 6).tokens == gen_injected.tokens


def test_injection_rejects_a_zero_source():
    cfg = dl.Qwen3Config(hidden=1024, query_heads=16, kv_heads=4, head_width=128, mlp_width=3072, vocabulary=2048,
                         layers=1)
    e = _engine(cfg)
    with pytest.raises(dl.DolittleError):
        e.set_injection(3, np.zeros(cfg.hidden, np.uint16), 150.0)


def test_reconstruction_head_matches_oracle():
    cfg = dl.Qwen3Config(hidden=1024, query_heads=16, kv_heads=4, head_width=128, mlp_width=3072, vocabulary=2048,
                         layers=2)
    e = _engine(cfg)
    head = oracle.fill_normal_bf16(cfg.hidden * cfg.hidden, 9, 0, np.float32(0.02 / np.sqrt(8 * (65536.0 ** 2 - 1) / 12)))
    head = head.reshape(cfg.hidden, cfg.hidden)
    e.set_reconstruction_head(head)
    prompt = oracle.uniform_ids(17, 3, 1, cfg.vocabulary)
    got = e.reconstruct(prompt)
    ocfg = oracle.Config(cfg.hidden, cfg.query_heads, cfg.kv_heads, cfg.head_width, cfg.mlp_width, cfg.vocabulary,
                         cfg.layers, cfg.epsilon, cfg.theta)
    model = oracle.OracleModel(ocfg, [e.get_tensor(i) for i in range(cfg.tensor_count())], capacity=32)
    _, cap = model.forward(prompt, 0, logits=False, capture_layer=cfg.layers - 1)
    want = oracle.projection(cap[-1:], head)[0]
    assert np.array_equal(got, want)
    # A second call starts a fresh sequence: same result.
    assert np.array_equal(e.reconstruct(prompt), got)
