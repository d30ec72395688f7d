"""tcgen05/TMEM GEMM (fast prefill projections) against a PyTorch FP32
reference of the same op: Y = X W^T accumulated in FP32, rounded to BF16.

The tensor-core summation order differs from the reference's strided FP32
chains, so the check is the reference's BF16 projection tolerance
(atol 1e-3, rtol 1.6e-2; tests/gpu/operator_reference.cpp) plus a
relative-L2 bound, and nearly all elements must round identically.
"""
import numpy as np
import pytest

import dolittle_b200 as dl
from tests import numerics as nm

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


def _case(M, N, K, seed, scale_w=0.02):
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * scale_w).to(torch.bfloat16)
    return x, w


@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (77, 1024, 4096), (128, 256, 12288),
                                   (512, 6144, 4096), (300, 128, 64), (1, 256, 128)])
def test_gemm_store_matches_fp32_reference(M, N, K):
    torch = _torch()
    x, w = _case(M, N, K, seed=M + N + K)
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    assert dl.lib().dl_gemm_bf16(x.data_ptr(), K, w.data_ptr(), y.data_ptr(), N, M, N, K, 0, None) == 0, \
        dl.lib().dl_last_error()
    torch.cuda.synchronize()
    ref = (x.float() @ w.float().T)
    got = y.float()
    r = nm.compare_elementwise(ref.cpu().numpy(), got.cpu().numpy(), 1e-3, 1.6e-2)
    assert r["passed"], r
    same = (ref.to(torch.bfloat16) == y).float().mean().item()
    assert same > 0.97, same
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel < 4e-3, rel


def test_gemm_residual_and_swiglu_epilogues():
    torch = _torch()
    M, D, F = 96, 512, 256
    x, w = _case(M, D, D, seed=5)
    res = torch.randn(M, D, device="cuda").to(torch.bfloat16)
    out = res.clone()
    assert dl.lib().dl_gemm_bf16(x.data_ptr(), D, w.data_ptr(), out.data_ptr(), D, M, D, D, 1, None) == 0
    torch.cuda.synchronize()
    proj = (x.float() @ w.float().T).to(torch.bfloat16).float()
    ref = (res.float() + proj).to(torch.bfloat16).float()
    r = nm.compare_elementwise(ref.cpu().numpy(), out.float().cpu().numpy(), 1e-2, 1.6e-2)
    assert r["passed"], r
    # SwiGLU on interleaved (gate, up) rows.
    xg, wgu = _case(M, 2 * F, D, seed=6)
    act = torch.empty(M, F, device="cuda", dtype=torch.bfloat16)
    assert dl.lib().dl_gemm_bf16(xg.data_ptr(), D, wgu.data_ptr(), act.data_ptr(), F, M, 2 * F, D, 3, None) == 0
    torch.cuda.synchronize()
    yy = (xg.float() @ wgu.float().T).to(torch.bfloat16).float()
    g, u = yy[:, 0::2], yy[:, 1::2]
    ref2 = ((g * torch.sigmoid(g)).to(torch.bfloat16).float() * u).to(torch.bfloat16).float()
    r2 = nm.compare_elementwise(ref2.cpu().numpy(), act.float().cpu().numpy(), 1e-2, 3e-2)
    assert r2["passed"], r2


@pytest.mark.parametrize("M,N,K,epi,tile_m,tile_n,parts", [
    (512, 4096, 4096, 0, 0, 0, 0), (512, 4096, 12288, 1, 0, 0, 0), (200, 6144, 4096, 0, 0, 0, 0),
    (512, 4096, 4096, 1, 128, 256, 3), (300, 4096, 4096, 0, 128, 128, 4), (512, 4096, 12288, 1, 128, 128, 2),
    (129, 2048, 1024, 0, 128, 256, 4), (512, 2048, 4096, 3, 128, 128, 3),
    # 256 x 256 tiles on CTA pairs (tcgen05 cta_group::2)
    (512, 4096, 4096, 0, 256, 256, 1), (300, 2048, 4096, 1, 256, 256, 1), (512, 4096, 12288, 1, 256, 256, 2),
    (700, 4096, 2048, 3, 256, 256, 3), (2048, 6144, 4096, 0, 256, 0, 1)])
def test_gemm_split_k_matches_fp32_reference_and_unsplit(M, N, K, epi, tile_m, tile_n, parts):
    """Split-K (up to 4 K parts summed in FP32 in part order by the last
    finisher) and single-SM or CTA-pair tiles, chosen by the library or
    pinned, against the FP32 reference: same tolerance as the unsplit
    kernel, and repeated runs are bit-identical (the order of the parts is
    fixed)."""
    torch = _torch()
    x, w = _case(M, N, K, seed=M + K + epi)
    ncols = N // 2 if epi == 3 else N
    res = torch.randn(M, N, device="cuda").to(torch.bfloat16) if epi == 1 else None
    L = dl.lib()
    ws = torch.empty(L.dl_gemm_bf16_split_workspace_bytes(M, N), device="cuda", dtype=torch.uint8)
    n_t = ((M + 127) // 128) * (N // 128)
    tickets = torch.zeros(n_t, device="cuda", dtype=torch.int32)
    outs = []
    for _ in range(2):
        y = res.clone() if epi == 1 else torch.empty(M, ncols, device="cuda", dtype=torch.bfloat16)
        assert L.dl_gemm_bf16_config(x.data_ptr(), K, w.data_ptr(), y.data_ptr(), ncols, M, N, K, epi, None,
                                     ws.data_ptr(), tickets.data_ptr(), n_t, tile_m, tile_n, parts) == 0, \
            L.dl_last_error()
        torch.cuda.synchronize()
        outs.append(y)
    assert torch.equal(outs[0], outs[1])
    assert int(tickets.abs().sum()) == 0
    proj = x.float() @ w.float().T
    got = outs[0].float()
    if epi == 3:
        yy = proj.to(torch.bfloat16).float()
        g, u = yy[:, 0::2], yy[:, 1::2]
        ref = ((g * torch.sigmoid(g)).to(torch.bfloat16).float() * u).to(torch.bfloat16).float()
        r = nm.compare_elementwise(ref.cpu().numpy(), got.cpu().numpy(), 1e-2, 3e-2)
        assert r["passed"], r
        return
    ref = (res.float() + proj.to(torch.bfloat16).float()).to(torch.bfloat16).float() if epi == 1 else proj
    if epi == 1:
        # Residual epilogue: round(res + round(acc)) rounds twice, so a
        # different (tensor-core) accumulation can move round(acc) by one
        # BF16 ulp of the projection and the sum by one ulp of the result:
        # bound 2 ulp of the larger magnitude (ulp = 2^(e-7) on [2^e, 2^(e+1))).
        mag = torch.maximum(proj.abs(), ref.abs()).clamp_min(1e-30)
        ulp = torch.exp2(torch.floor(torch.log2(mag)) - 7)
        assert bool(((got - ref).abs() <= 2 * ulp + 1e-3).all())
    else:
        r = nm.compare_elementwise(ref.cpu().numpy(), got.cpu().numpy(), 1e-3, 1.6e-2)
        assert r["passed"], r
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel < 4e-3, rel


def test_gemm_rejects_unsupported_shapes():
    torch = _torch()
    x = torch.zeros(8, 100, device="cuda", dtype=torch.bfloat16)
    assert dl.lib().dl_gemm_bf16(x.data_ptr(), 100, x.data_ptr(), x.data_ptr(), 128, 8, 128, 100, 0,
                                 None) == dl._lib.DL_UNSUPPORTED


@pytest.mark.parametrize("M,N,K,epi,bn", [(512, 6144, 4096, 0, 256), (512, 4096, 12288, 1, 256),
                                          (200, 2048, 4096, 3, 256), (512, 4096, 4096, 1, 128),
                                          (77, 1024, 1024, 0, 128)])
def test_gemm_streamk_matches_fp32_reference_and_repeats_bit_identically(M, N, K, epi, bn):
    """Stream-K (parts = -1): every CTA takes an equal share of the k-steps;
    tiles cut between CTAs are summed in k order by the CTA holding their last
    k-step.  Store / residual / SwiGLU epilogues against the FP32 reference;
    two runs bit-identical (fixed sum order)."""
    torch = _torch()
    L = dl.lib()
    x, w = _case(M, N, K, seed=3 * M + N + K)
    cols = N // 2 if epi == 3 else N
    base = torch.randn(M, cols, device="cuda").to(torch.bfloat16)
    ws = torch.empty(L.dl_gemm_bf16_split_workspace_bytes(M, N), device="cuda", dtype=torch.uint8)
    n_t = ((M + 255) // 256) * 2 * (N // 128)
    tickets = torch.zeros(n_t, device="cuda", dtype=torch.int32)
    outs = []
    for _ in range(2):
        y = base.clone()
        rc = L.dl_gemm_bf16_config(x.data_ptr(), K, w.data_ptr(), y.data_ptr(), cols, M, N, K, epi, None,
                                   ws.data_ptr(), tickets.data_ptr(), n_t, 128, bn, -1)
        assert rc == 0, L.dl_last_error()
        torch.cuda.synchronize()
        outs.append(y)
    assert torch.equal(outs[0], outs[1])
    assert int(tickets.abs().sum().item()) == 0   # every finisher reset its ticket
    proj = x.float() @ w.float().T
    got = outs[0].float()
    if epi == 0:
        r = nm.compare_elementwise(proj.cpu().numpy(), got.cpu().numpy(), 1e-3, 1.6e-2)
    elif epi == 1:
        # round(old + round(proj)): a one-ulp flip of the inner rounding is
        # relative to |proj|, not to the (possibly cancelled) sum.
        pb = proj.to(torch.bfloat16).float()
        ref = (base.float() + pb).to(torch.bfloat16).float()
        err = (got - ref).abs()
        bound = 1e-2 + 2.0 ** -6 * torch.maximum(ref.abs(), pb.abs())  # one ulp of each rounding
        r = {"mismatched": int((err > bound).sum().item()), "max_abs": float(err.max().item())}
        r["passed"] = r["mismatched"] == 0
    else:
        yy = proj.to(torch.bfloat16).float()
        gg, uu = yy[:, 0::2], yy[:, 1::2]
        ref = ((gg * torch.sigmoid(gg)).to(torch.bfloat16).float() * uu).to(torch.bfloat16).float()
        r = nm.compare_elementwise(ref.cpu().numpy(), got.cpu().numpy(), 1e-2, 3e-2)
    assert r["passed"], r
