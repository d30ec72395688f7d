"""tcgen05 causal prefill attention (the fast prompt pass) against a PyTorch
FP32 reference of causal GQA attention on the same BF16 inputs.

The kernel rounds the probabilities and the output to BF16 (tensor-core
operands), so the bar is a tolerance: max |error| <= 1.5 % of max |ref| and
cosine similarity > 0.9999, stated per case below.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import dolittle_b200 as dl

pytestmark = pytest.mark.gpu
MAX_ABS_FRAC = 0.015
MIN_COSINE = 0.9999


def reference(q, k, v, first):
    """q [rows][Hq][d], k/v [keys][Hkv][d] (FP32): causal GQA softmax attention."""
    rows, hq, d = q.shape
    hkv = k.shape[1]
    group = hq // hkv
    keys = first + rows
    kk = k[:keys].repeat_interleave(group, dim=1)  # [keys][Hq][d]
    vv = v[:keys].repeat_interleave(group, dim=1)
    s = torch.einsum("rhd,khd->hrk", q, kk) / np.sqrt(d)
    pos = torch.arange(rows, device=q.device)[:, None] + first
    mask = torch.arange(keys, device=q.device)[None, :] > pos
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hrk,khd->rhd", p, vv)


CASES = [
    # rows, first, capacity, Hq, Hkv
    (150, 0, 160, 32, 8),      # two ragged query tiles, two key blocks
    (512, 0, 512, 32, 8),      # config 2 prompt
    (100, 200, 320, 32, 8),    # a later chunk: keys 0..299
    (1, 37, 64, 32, 8),        # one row
    (130, 0, 130, 8, 4),       # GQA group 2
    (64, 0, 64, 16, 16),       # no grouping
]


@pytest.mark.parametrize("rows,first,cap,hq,hkv", CASES)
def test_tc_attention_matches_fp32_reference(rows, first, cap, hq, hkv):
    torch.manual_seed(rows * 7 + first)
    d = 128
    q = torch.randn(rows, hq, d, device="cuda").to(torch.bfloat16)
    k = torch.randn(cap, hkv, d, device="cuda").to(torch.bfloat16)
    v = torch.randn(cap, hkv, d, device="cuda").to(torch.bfloat16)
    out = torch.zeros(rows, hq, d, device="cuda", dtype=torch.bfloat16)
    L = dl.lib()
    ws = torch.zeros(L.dl_attention_prefill_fast_workspace_bytes(hkv, d, cap), device="cuda", dtype=torch.uint8)
    st = torch.cuda.current_stream().cuda_stream
    dl._lib.check(L.dl_attention_prefill_fast(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), rows, hq,
                                               hkv, d, st, first, cap, ws.data_ptr()))
    torch.cuda.synchronize()
    ref = reference(q.float(), k.float(), v.float(), first)
    got = out.float()
    err = (got - ref).abs().max().item()
    peak = ref.abs().max().item()
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    assert err <= MAX_ABS_FRAC * peak, (err, peak)
    assert cos > MIN_COSINE, cos


def test_tc_attention_rejects_unsupported_shapes():
    L = dl.lib()
    p = C.c_void_p(1)
    # head width 64 is not supported by the tensor-core path
    assert L.dl_attention_prefill_fast(p, p, p, p, 4, 8, 4, 64, None, 0, 16, p) == dl._lib.DL_UNSUPPORTED
    # keys beyond the capacity
    assert L.dl_attention_prefill_fast(p, p, p, p, 10, 8, 4, 128, None, 10, 16, p) == dl._lib.DL_INVALID_ARGUMENT
