"""Device-side generation loop (the reference's DeviceSequence role): one
graph with a conditional WHILE node replays the decode step on the device,
journaling every selection as a 32-byte event in mapped host memory.

* The loop selects exactly the tokens of the host-driven generate() (greedy
  and categorical, both decode paths).
* A stop ID ends the loop on the device: the journal's terminal event says
  EOS, and no step runs past it.
* A cancel request ends it early with reason CANCELLED; a budget of one
  selection ends it at once with reason LIMIT.
"""
import numpy as np
import pytest

import dolittle_b200 as dl
from oracle import oracle

pytestmark = pytest.mark.gpu


def _engine(layers=2, cap=160):
    cfg = dl.Qwen3Config(hidden=1024, query_heads=16, kv_heads=4, head_width=128, mlp_width=3072,
                         vocabulary=5003, layers=layers)
    e = dl.Engine(cfg, capacity=cap, max_rows=8)
    e.init_random(4, 0.02)
    return cfg, e


def _journal(e, n):
    return [e.collect(i, 10000) for i in range(n)]


@pytest.mark.parametrize("path", [dl.DL_DECODE_PERSISTENT, dl.DL_DECODE_KERNELS])
@pytest.mark.parametrize("categorical", [False, True])
def test_device_loop_matches_generate(path, categorical):
    cfg, e = _engine()
    e.set_decode_path(path)
    prompt = oracle.uniform_ids(30, 1, 301, cfg.vocabulary)
    st = dl.Settings(dl.SelectionMode.categorical, 0.8, 0, 0.9) if categorical else dl.Settings()
    ref = e.generate(prompt, 25, settings=st, seed=11)
    e.start(prompt, 25, settings=st, seed=11)
    ev = _journal(e, 27)
    out = e.drain()
    assert out.tokens == ref.tokens
    assert ev[0].kind == dl.DL_EVENT_CONSUMED and ev[0].count == 30
    for k in range(1, 26):
        assert ev[k].kind == dl.DL_EVENT_SELECTED and ev[k].count == k and ev[k].token == ref.tokens[k - 1]
        assert ev[k].status == 0
    assert ev[26].kind == dl.DL_EVENT_TERMINAL and ev[26].reason == dl.DL_REASON_LIMIT and ev[26].count == 25
    assert out.decode_steps == 24


def test_stop_id_ends_the_loop_on_the_device():
    cfg, e = _engine()
    prompt = oracle.uniform_ids(20, 1, 302, cfg.vocabulary)
    free = e.generate(prompt, 30).tokens
    stop = free[9]  # the 10th selection is a stop ID
    first = free.index(stop)
    e.start(prompt, 30, stop_ids=[stop])
    ev = e.collect(first + 2, 10000)
    out = e.drain()
    assert out.tokens == free[:first + 1]
    assert ev.kind == dl.DL_EVENT_TERMINAL and ev.reason == dl.DL_REASON_EOS and ev.token == stop
    assert e.collect(first + 3, 0) is None  # nothing after the terminal event
    assert e.position == len(prompt) + first  # no step ran past the stop


def test_cancel_request_and_limit_of_one():
    cfg, e = _engine(layers=4, cap=600)
    prompt = oracle.uniform_ids(16, 1, 303, cfg.vocabulary)
    e.start(prompt, 560)
    assert e.collect(3, 10000).kind == dl.DL_EVENT_SELECTED
    e.request_stop()
    out = e.drain()
    n = len(out.tokens)
    assert n < 560
    term = e.collect(n + 1, 0)
    assert term.kind == dl.DL_EVENT_TERMINAL and term.reason == dl.DL_REASON_CANCELLED and term.count == n
    e.start(prompt, 1)
    out = e.drain()
    assert len(out.tokens) == 1
    term = e.collect(2, 0)
    assert term.kind == dl.DL_EVENT_TERMINAL and term.reason == dl.DL_REASON_LIMIT


def test_start_while_running_is_rejected():
    cfg, e = _engine()
    prompt = oracle.uniform_ids(10, 1, 304, cfg.vocabulary)
    e.start(prompt, 50)
    with pytest.raises(dl.DolittleError):
        e.start(prompt, 5)
    e.drain()
    with pytest.raises(dl.DolittleError):
        e.drain()
