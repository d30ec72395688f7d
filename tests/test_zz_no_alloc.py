"""dl_attention_fixed_scratch: attention without any device allocation.

Callers that cannot allocate device memory (a host that owns every device
allocation in its own arena, or a plugin whose process allocator forbids
cudaMalloc) use this entry point; it keeps the attention scores in a fixed
array inside the library.  The test calls it twice in a row through the C ABI
and checks each result against dl_attention with a caller-provided workspace
(the results must be identical: same kernels, same arithmetic), with the
query position given on the host and read from device memory against a
larger key capacity (the decode layout), that the calls leave the device's
free memory unchanged, and that a request beyond the fixed array's size is
rejected before any launch.

This file is collected last on purpose, and it sets up everything it needs
itself, so it passes both alone in a fresh process and after the other tests.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _rand_bf16(shape, seed):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal(shape).astype(np.float32).view(np.uint32).astype(np.uint64)
    return (((a + 0x7FFF + ((a >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16).copy()).cuda()


def _host(t):
    return t.cpu().numpy().view(np.uint16)


def _run_pair(case_seed, rows, first, H=32, G=8, d=128, capacity=None):
    """dl_attention (caller workspace) and dl_attention_fixed_scratch on the
    same inputs.  capacity=None: the query position is `first`, given on the
    host, and the key capacity is first + rows.  Otherwise the cache holds
    `capacity` key rows and the position is read from device memory."""
    import torch

    import dolittle_b200 as dl
    L = dl.lib()
    total = first + rows if capacity is None else capacity
    q, k, v = (_rand_bf16(s, case_seed + i) for i, s in
               enumerate([(rows, H, d), (total, G, d), (total, G, d)]))
    dq, dk, dv = _dev(q), _dev(k), _dev(v)
    with_ws = torch.zeros((rows, H, d), dtype=torch.int16, device="cuda")
    fixed = torch.full((rows, H, d), -1, dtype=torch.int16, device="cuda")
    ws = torch.zeros(L.dl_attention_workspace_bytes(rows, H, total) // 2 + 8, dtype=torch.int16, device="cuda")
    scale = torch.zeros(2, dtype=torch.float32, device="cuda")
    pos = torch.tensor([first], dtype=torch.int64, device="cuda")
    dev_pos = pos.data_ptr() if capacity is not None else None
    host_first = 0 if capacity is not None else first
    assert L.dl_attention_scale(scale.data_ptr(), d, None) == 0
    assert L.dl_attention(dl.DL_BF16, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), with_ws.data_ptr(), rows, H, G,
                          d, None, host_first, dev_pos, total, scale.data_ptr(), ws.data_ptr()) == 0
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    rc = L.dl_attention_fixed_scratch(dl.DL_BF16, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), fixed.data_ptr(),
                                      rows, H, G, d, None, host_first, dev_pos, total)
    assert rc == 0, L.dl_last_error()
    torch.cuda.synchronize()
    free_after = torch.cuda.mem_get_info()[0]
    return _host(with_ws), _host(fixed), free_before - free_after


def test_fixed_scratch_attention_matches_workspace_attention_twice():
    # A first call loads the library's device module (and with it the fixed
    # array) if nothing has yet; the calls after it must allocate nothing.
    _run_pair(7, rows=2, first=30)
    # Two calls in a row: the second reuses the array the first left behind.
    a, b, grew = _run_pair(101, rows=1, first=700)
    assert np.array_equal(a, b) and grew == 0
    a, b, grew = _run_pair(202, rows=9, first=40)
    assert np.array_equal(a, b) and grew == 0


def test_fixed_scratch_attention_device_position_and_capacity():
    # Decode layout: a cache of 1024 key rows, the query row's position read
    # from device memory; then a 5-row chunk at position 300.
    _run_pair(5, rows=1, first=10, capacity=64)
    a, b, grew = _run_pair(303, rows=1, first=517, capacity=1024)
    assert np.array_equal(a, b) and grew == 0
    a, b, grew = _run_pair(404, rows=5, first=300, capacity=1024)
    assert np.array_equal(a, b) and grew == 0


def test_fixed_scratch_rejects_requests_above_its_size():
    import torch

    import dolittle_b200 as dl
    L = dl.lib()
    cap = 1 << 20   # DL_ATTENTION_FIXED_SCRATCH_SCORES
    rows, H, G, d = 64, 32, 8, 128
    first = cap // (rows * H)           # rows * H * (first + rows) > cap
    dummy = torch.zeros(16, dtype=torch.int16, device="cuda")
    p = dummy.data_ptr()
    rc = L.dl_attention_fixed_scratch(dl.DL_BF16, p, p, p, p, rows, H, G, d, None, first, None, first + rows)
    assert rc == dl._lib.DL_INVALID_ARGUMENT
    assert b"fixed scratch" in L.dl_last_error()
    # Sizes whose product would wrap a 64-bit count are rejected too.
    rc = L.dl_attention_fixed_scratch(dl.DL_BF16, p, p, p, p, 1 << 62, H, G, d, None, 0, None, 1)
    assert rc == dl._lib.DL_INVALID_ARGUMENT
