"""Steering direction from two reconstructions (DeviceDirection).

Reference: src/kernels/cuda/steering.cu:68-98 (kernel) and :200-258
(DeviceDirection::submit/finish), interface src/inference/steering/device.h:
30-48.  direction = (edited - original) / ||edited - original|| in FP32, the
norm from 8 lanes of serially added rounded squares (lane L owns features
L + 8k), the lane sums added 0..7, sqrt_rn, each quotient div_rn; status 1
and no output on a zero or non-finite norm.

CPU: the oracle's restatement against an independent NumPy FP32 one.
GPU: dl_direction through the C ABI bit for bit against the reference's own
DeviceDirection (oracle/_ref) and the oracle, on BF16 and FP32
reconstructions, ragged widths, the zero-difference and non-finite cases.
"""
import numpy as np
import pytest

from oracle import oracle
from tests import numerics as nm


def _numpy_law(original, edited):
    a = nm.bf16_bits_to_f32(original) if original.dtype == np.uint16 else original.astype(np.float32)
    b = nm.bf16_bits_to_f32(edited) if edited.dtype == np.uint16 else edited.astype(np.float32)
    delta = (b - a).astype(np.float32)
    sq = (delta * delta).astype(np.float32)
    lanes = [nm.serial_sum_f32(sq[l::8]) for l in range(8)]
    total = nm.serial_sum_f32(np.array(lanes, np.float32))
    norm = np.float32(np.sqrt(np.float64(total)))  # sqrt of an FP32 value, correctly rounded
    if not np.isfinite(norm) or norm == 0:
        return 1, None
    return 0, (delta / norm).astype(np.float32)


def _inputs(width, seed, bf16):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal(width).astype(np.float32) * 3
    b = a + rng.standard_normal(width).astype(np.float32) * 0.25
    if bf16:
        return nm.f32_to_bf16_bits(a), nm.f32_to_bf16_bits(b)
    return a, b


@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("width", [1, 7, 4096, 4100, 9000])
def test_oracle_direction_matches_numpy_law(bf16, width):
    a, b = _inputs(width, width, bf16)
    st, d = oracle.direction(a, b)
    want_st, want = _numpy_law(a, b)
    assert st == want_st == 0
    assert np.array_equal(d.view(np.uint32), want.view(np.uint32))


def test_oracle_direction_status_cases():
    a, _ = _inputs(64, 1, True)
    st, d = oracle.direction(a, a)
    assert st == 1 and np.isnan(d).all()
    f, g = _inputs(64, 2, False)
    g[5] = np.inf
    assert oracle.direction(f, g)[0] == 1


def _dl_direction(a, b):
    import torch

    import dolittle_b200 as dl
    L = dl.lib()
    bf16 = a.dtype == np.uint16
    view = np.int16 if bf16 else np.float32
    da = torch.from_numpy(np.ascontiguousarray(a).view(view).copy()).cuda()
    db = torch.from_numpy(np.ascontiguousarray(b).view(view).copy()).cuda()
    out = torch.full((a.size,), float("nan"), dtype=torch.float32, device="cuda")
    status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    rc = L.dl_direction(dl.DL_BF16 if bf16 else dl.DL_F32, da.data_ptr(), db.data_ptr(), a.size, out.data_ptr(),
                        status.data_ptr(), None)
    assert rc == 0, L.dl_last_error()
    torch.cuda.synchronize()
    return int(status.item()), out.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("width", [1, 13, 4096, 4100, 9000])
def test_direction_bit_exact_vs_reference_and_oracle(bf16, width):
    ref = oracle.ref_cuda()
    a, b = _inputs(width, 100 + width, bf16)
    st, d = _dl_direction(a, b)
    ost, od = oracle.direction(a, b)
    assert st == ost == 0
    assert np.array_equal(d.view(np.uint32), od.view(np.uint32))
    if ref is None:
        pytest.skip("oracle/_ref/libref_cuda.so not built")
    rst, rd = oracle.ref_direction(a, b)
    assert rst == 0
    assert np.array_equal(d.view(np.uint32), rd.view(np.uint32))


@pytest.mark.gpu
def test_direction_status_zero_and_nonfinite_difference():
    ref = oracle.ref_cuda()
    for bf16 in (True, False):
        a, _ = _inputs(4096, 3, bf16)
        st, d = _dl_direction(a, a.copy())
        assert st == 1 and np.isnan(d).all()      # output untouched
        if ref is not None:
            assert oracle.ref_direction(a, a.copy())[0] == 1
    f, g = _inputs(4096, 4, False)
    g[100] = np.inf
    assert _dl_direction(f, g)[0] == 1
    if ref is not None:
        assert oracle.ref_direction(f, g)[0] == 1


@pytest.mark.gpu
def test_direction_rejects_bad_arguments():
    import dolittle_b200 as dl
    from dolittle_b200 import _lib
    L = dl.lib()
    assert L.dl_direction(dl.DL_BF16, None, None, 16, None, None, None) == _lib.DL_INVALID_ARGUMENT
    assert L.dl_direction(7, 16, 16, 16, 16, 16, None) == _lib.DL_UNSUPPORTED
