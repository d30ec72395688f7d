"""Steered and unsteered continuations as one batch.

The server captures block `layer`'s output and adds a fixed-strength
steering vector there for every position >= first, for chosen sequences
(dl_serve_set_steering).  The reference edits one row once
(src/kernels/cuda/steering.cu:106-159, one-shot count decode.cu:177-184);
its strength is beta = alpha * ||h[p]|| of the edited row.  Here beta is
computed the same way from the source sequence's row p, so:

* the steered rows of the prompt equal the oracle's fixed-strength law on the
  unsteered rows (blocks up to `layer` are unaffected by the edits), bit for
  bit, and row p equals the reference's one-row edit of it (or_intervene);
* the unsteered sequence is bit-identical to a run without steering (rows of
  a lockstep batch do not interact);
* the first decode row, where both sequences see the same token, is edited by
  the same law through the decode step's graph.
"""
import numpy as np
import pytest

import dolittle_b200 as dl
from dolittle_b200.serve import Server
from oracle import oracle

pytestmark = pytest.mark.gpu


def _cfg():
    return dl.Qwen3Config(hidden=1024, query_heads=16, kv_heads=4, head_width=128, mlp_width=3072,
                          vocabulary=2048, layers=3)


def _unit(width, seed):
    u = np.random.Generator(np.random.Philox(seed)).standard_normal(width).astype(np.float32)
    return (u / np.linalg.norm(u)).astype(np.float32)


def _run(cfg, prompts, steps, layer, steer=None, settings=None):
    srv = Server(cfg, batch=prompts.shape[0], capacity=prompts.shape[1] + steps + 8, chunk_rows=16)
    srv.init_random(4, 0.02)
    srv.set_capture(layer)
    if steer is not None:
        srv.set_steering(layer, **steer)
    first = srv.prefill(prompts, settings or dl.Settings(), seed=7)
    res = srv.decode(steps, want_logits=True)
    cap = [srv.read_capture(b, 0, prompts.shape[1] + steps) for b in range(prompts.shape[0])]
    beta = srv.steering_strength() if steer is not None else None
    srv.close()
    return first, res, cap, beta


def test_batch_of_steered_and_unsteered_rows_follows_the_law():
    cfg = _cfg()
    P, steps, layer, p0, alpha = 40, 6, 1, 20, 4.0
    prompt = oracle.uniform_ids(P, 1, 31, cfg.vocabulary)
    prompts = np.stack([prompt, prompt])           # sequence 0 unsteered, 1 steered
    u = _unit(cfg.hidden, 7)
    f0, r0, c0, _ = _run(cfg, prompts, steps, layer)
    steer = dict(first_position=p0, strength=alpha, direction=u, sequences=[1], source_sequence=0,
                 source_position=p0)
    f1, r1, c1, beta = _run(cfg, prompts, steps, layer, steer)
    # beta from sequence 0's row p0 with the one-row edit's norm law.
    assert np.float32(beta) == oracle.steer_beta(c0[0][p0], alpha)
    # The unsteered sequence is untouched, prompt and decode.
    assert np.array_equal(c1[0], c0[0])
    assert np.array_equal(r1.logits[:, 0], r0.logits[:, 0]) and int(f1[0]) == int(f0[0])
    # Prompt rows of the steered sequence: unchanged before p0, the law after.
    assert np.array_equal(c1[1][:p0], c0[1][:p0])
    st, want = oracle.steer_rows(c0[1][:P], u, 0, p0, np.float32(beta))
    assert st == 0
    assert np.array_equal(c1[1][:P], want)
    # Row p0 is exactly the reference's one-row edit of that row.
    row = c0[1][p0:p0 + 1].copy()
    state = np.zeros(2, np.uint32)
    oracle.lib().or_intervene(row, u, cfg.hidden, p0, p0, 1, alpha, state)
    assert state[0] == 0 and np.array_equal(c1[1][p0], row[0])
    # First decode row (position P): if both sequences selected the same
    # token, its pre-edit row at block `layer` is the same in both (blocks up
    # to `layer` never see an edit), so the steered row is the law on the
    # unsteered one.
    if int(f1[1]) == int(f1[0]):
        st, want = oracle.steer_rows(c1[0][P:P + 1], u, P, p0, np.float32(beta))
        assert np.array_equal(c1[1][P], want[0])
    # The steering changed the continuation's logits.
    assert not np.array_equal(r1.logits[:, 1], r1.logits[:, 0])


def test_decode_rows_are_steered_through_the_step_graph():
    """Steering from the first decode position only: the prompts are
    identical, so both sequences select the same greedy token and compute
    the same pre-edit row at position P; the steered sequence's captured row
    there is the law applied to the unsteered one (fixed beta)."""
    cfg = _cfg()
    P, steps, layer = 24, 3, 2
    prompt = oracle.uniform_ids(P, 1, 32, cfg.vocabulary)
    prompts = np.stack([prompt, prompt, prompt])
    u = _unit(cfg.hidden, 8)
    beta = np.float32(3.25)
    steer = dict(first_position=P, strength=float(beta), direction=u, sequences=[1, 2])
    first, res, cap, got_beta = _run(cfg, prompts, steps, layer, steer)
    assert np.float32(got_beta) == beta
    assert int(first[0]) == int(first[1]) == int(first[2])
    assert np.array_equal(cap[1][:P], cap[0][:P])
    st, want = oracle.steer_rows(cap[0][P:P + 1], u, P, P, beta)
    assert st == 0
    assert np.array_equal(cap[1][P], want[0]) and np.array_equal(cap[2][P], want[0])
    assert np.array_equal(cap[1], cap[2])        # same input, same edits


def test_steering_arguments_are_checked():
    cfg = _cfg()
    srv = Server(cfg, batch=2, capacity=32, chunk_rows=16)
    u = _unit(cfg.hidden, 9)
    with pytest.raises(dl.DolittleError):   # a steered sequence before the strength source
        srv.set_steering(1, first_position=4, strength=2.0, direction=u, sequences=[0], source_sequence=1,
                         source_position=4)
    with pytest.raises(dl.DolittleError):
        srv.set_steering(7, first_position=4, strength=2.0, direction=u, sequences=[1])
    bad = u.copy()
    bad[3] = np.nan
    with pytest.raises(dl.DolittleError):
        srv.set_steering(1, first_position=4, strength=2.0, direction=bad, sequences=[1])
    srv.set_steering(-1)
    srv.close()
