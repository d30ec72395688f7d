"""dl_attention_fixed_scratch: attention without any device allocation.

Callers that cannot allocate device memory (a host that owns every device
allocation in its own arena, or a plugin whose process allocator forbids
cudaMalloc) use this entry point; it keeps the attention scores in a fixed
array inside the library.  The test calls it twice in a row through the C ABI
and checks each result against dl_attention with a caller-provided workspace
(the results must be identical: same kernels, same arithmetic), and that a
request beyond the fixed array's size is rejected before any launch.

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


def _run_pair(case_seed, rows, first, H=32, G=8, d=128):
    import torch

    import dolittle_b200 as dl
    L = dl.lib()
    total = first + rows
    q, k, v = (_rand_bf16(s, case_seed + i) for i, s in
               enumerate([(rows, H, d), (total, G, d), (total, G, d)]))
    dq, dk, dv = _dev(q), _dev(k), _dev(v)
    with_ws = torch.zeros((rows, H, d), dtype=torch.int16, device="cuda")
    fixed = torch.full((rows, H, d), -1, dtype=torch.int16, device="cuda")
    ws = torch.zeros(L.dl_attention_workspace_bytes(rows, H, total) // 2 + 8, dtype=torch.int16, device="cuda")
    scale = torch.zeros(2, dtype=torch.float32, device="cuda")
    assert L.dl_attention_scale(scale.data_ptr(), d, None) == 0
    assert L.dl_attention(dl.DL_BF16, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), with_ws.data_ptr(), rows, H, G,
                          d, None, first, None, total, scale.data_ptr(), ws.data_ptr()) == 0
    rc = L.dl_attention_fixed_scratch(dl.DL_BF16, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), fixed.data_ptr(),
                                      rows, H, G, d, None, first, None, total)
    assert rc == 0, L.dl_last_error()
    torch.cuda.synchronize()
    return _host(with_ws), _host(fixed)


def test_fixed_scratch_attention_matches_workspace_attention_twice():
    # Two calls in a row: the second reuses the array the first left behind.
    a, b = _run_pair(101, rows=1, first=700)
    assert np.array_equal(a, b)
    a, b = _run_pair(202, rows=9, first=40)
    assert np.array_equal(a, b)


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
