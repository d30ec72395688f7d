"""Tensor-parallel host logic on CPU: the slice layout every rank holds, and
the NCCL id exchange over a two-rank gloo group (stand-in server; the id
factory is the only library call and is replaced here)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import dolittle_b200 as dl
from dolittle_b200 import serve


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_slices_tile_every_tensor_exactly_once(size):
    cfg = dl.Qwen3Config(layers=2)
    per_rank = [serve.tp_slices(cfg, r, size) for r in range(size)]
    for i in range(cfg.tensor_count()):
        rows, cols = cfg.tensor_shape(i)
        pieces = [p[i] for p in per_rank]
        if all(p == (rows, cols, 0, 0) for p in pieces):
            continue  # replicated
        covered = set()
        for r, c, r0, c0 in pieces:
            assert (r == rows) != (c == cols), (i, pieces)  # cut along exactly one dimension
            span = range(r0, r0 + r) if c == cols else range(c0, c0 + c)
            assert not covered & set(span)
            covered |= set(span)
        assert covered == set(range(rows if pieces[0][1] == cols else cols)), i


def test_slices_follow_kv_head_groups():
    cfg = dl.Qwen3Config(layers=1)
    q, k, v, o, gate, down = 3 + 1, 3 + 2, 3 + 3, 3 + 6, 3 + 8, 3 + 10
    s = serve.tp_slices(cfg, 1, 4)
    assert s[q] == (1024, 4096, 1024, 0)       # query heads 8..15
    assert s[k] == s[v] == (256, 4096, 256, 0)  # KV heads 2..3 (the same GQA groups)
    assert s[o] == (4096, 1024, 0, 1024)
    assert s[gate] == (3072, 4096, 3072, 0)
    assert s[down] == (4096, 3072, 0, 3072)
    assert s[2] == (37984, 4096, 37984, 0)     # vocabulary head rows 37984..75967
    assert s[0] == (151936, 4096, 0, 0)         # the embedding stays whole
    with pytest.raises(ValueError):
        serve.tp_slices(cfg, 0, 3)


class _FakeServer:
    def __init__(self, rank):
        self.got = None
        self.rank = rank
        self.peers = None

    def connect(self, nccl_id):
        self.got = nccl_id

    def ipc_handle(self):
        return bytes([self.rank]) * 64

    def connect_peers(self, handles):
        self.peers = handles


def _rank_main(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        srv = _FakeServer(rank)
        made = []
        got = serve.connect_group(srv, dist, make_id=lambda: made.append(1) or bytes(range(128)))
        assert srv.got == got == bytes(range(128))
        assert srv.peers == b"".join(bytes([r]) * 64 for r in range(world))  # every rank's handle, rank order
        assert made == ([1] if rank == 0 else [])  # only rank 0 makes the id
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_nccl_id_reaches_every_rank():
    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)


def _plan(batch, kv_heads, capacity, sms=148):
    import ctypes as C
    splits, lead = C.c_int(-1), C.c_int(-1)
    assert dl.lib().dl_attention_decode_batched_plan(batch, kv_heads, capacity, sms, C.byref(splits),
                                                     C.byref(lead)) == 0
    return splits.value, lead.value


def test_attention_plan_choices():
    """The batched decode attention's key ranges (host arithmetic, no GPU):
    batch 32 x 8 KV heads is 256 units on 296 CTA slots of a 148-SM B200.
    At 8K context a long first range per unit plus a short second one beats
    even ranges; at 2K one range per unit stays; under two-way tensor
    parallelism (4 local KV heads) two even ranges fill the slots."""
    splits, lead = _plan(32, 8, 8192 + 32 * 6 + 8)  # the config-5 bench's capacity
    assert splits == 2 and 850 < lead < 1000, (splits, lead)
    assert _plan(32, 8, 2048 + 32 * 6 + 8) == (1, 0)
    assert _plan(32, 4, 2048 + 32 * 6 + 8) == (2, 0)
    assert _plan(56, 4, 2048)[0] == 2 and _plan(56, 4, 2048)[1] > 0  # the GPU test's server shape
    # More units than slots: even ranges only.
    for cap in (512, 2048, 8192, 32768):
        assert _plan(128, 8, cap)[1] == 0
    # One unit: many even ranges, never the leading form.
    s1, l1 = _plan(1, 8, 9216)
    assert l1 == 0 and s1 > 1


def test_attention_plan_rejects_bad_arguments():
    import ctypes as C
    L = dl.lib()
    out = C.c_int()
    assert L.dl_attention_decode_batched_plan(32, 8, 2048, 148, None, C.byref(out)) != 0
    assert L.dl_attention_decode_batched_plan(0, 8, 2048, 148, C.byref(out), C.byref(out)) != 0
    assert L.dl_attention_decode_batched_plan(32, 8, 2048, 0, C.byref(out), C.byref(out)) != 0
