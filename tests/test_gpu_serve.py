"""Batched serving (lockstep batches, tensor-parallel slices) on one GPU.

* Split-K GEMM for few rows and the batched flash-decoding attention against
  PyTorch FP32 references of the same ops.
* Server (B sequences at once, tcgen05 projections, online-softmax
  attention) against the single-sequence engine's reference-law path on
  the same seeded weights: logits within the fast-path tolerance used for
  the tensor-core prompt pass, and the same greedy continuations.
* Tensor-parallel slices: ranks of one group generate exactly the matching
  rows / columns of the full seeded tensors.
"""
import numpy as np
import pytest

import dolittle_b200 as dl
from dolittle_b200.serve import Server, tp_slices
from oracle import oracle
from tests import numerics as nm

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


@pytest.mark.parametrize("M,N,K,epi", [(32, 6144, 4096, 0), (32, 4096, 12288, 1), (7, 2048, 4096, 3),
                                       (32, 1024, 512, 0)])
def test_gemm_parts_matches_fp32_reference(M, N, K, epi):
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    L = dl.lib()
    ws = torch.empty(L.dl_gemm_bf16_parts_workspace_bytes(M, N, K, 0) // 4 + 1, device="cuda", dtype=torch.float32)
    proj = (x.float() @ w.float().T)
    if epi == 3:
        out = torch.empty(M, N // 2, device="cuda", dtype=torch.bfloat16)
        ld = N // 2
    else:
        out = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16) if epi == 1 else \
            torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ld = N
    before = out.clone()
    assert L.dl_gemm_bf16_parts(x.data_ptr(), K, w.data_ptr(), out.data_ptr(), ld, M, N, K, epi, 0, ws.data_ptr(),
                                None) == 0, L.dl_last_error()
    torch.cuda.synchronize()
    if epi == 0:
        ref = proj
        r = nm.compare_elementwise(ref.cpu().numpy(), out.float().cpu().numpy(), 1e-3, 1.6e-2)
    elif epi == 1:
        ref = (before.float() + proj.to(torch.bfloat16).float()).to(torch.bfloat16).float()
        r = nm.compare_elementwise(ref.cpu().numpy(), out.float().cpu().numpy(), 1e-2, 1.6e-2)
    else:
        yy = proj.to(torch.bfloat16).float()
        gg, uu = yy[:, 0::2], yy[:, 1::2]
        ref = ((gg * torch.sigmoid(gg)).to(torch.bfloat16).float() * uu).to(torch.bfloat16).float()
        r = nm.compare_elementwise(ref.cpu().numpy(), out.float().cpu().numpy(), 1e-2, 3e-2)
    assert r["passed"], r
    # The parts are added in a fixed order: repeated runs are bit-identical.
    again = before.clone()
    assert L.dl_gemm_bf16_parts(x.data_ptr(), K, w.data_ptr(), again.data_ptr(), ld, M, N, K, epi, 0,
                                ws.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert torch.equal(again, out)


@pytest.mark.parametrize("B,Hq,Hkv,count,cap", [(3, 8, 2, 201, 256), (2, 32, 8, 1000, 1024), (4, 4, 1, 5, 64),
                                                (1, 32, 8, 9216, 9216), (32, 32, 8, 8000, 8192),
                                                (32, 32, 8, 100, 8192)])
def test_attention_decode_batched_matches_fp32_reference(B, Hq, Hkv, count, cap):
    """The last two cases take the leading-range plan on a 148-SM B200 (256
    (sequence, KV head) units on 296 CTA slots): a long first key range per
    unit and a short second one; at 100 keys the second range is empty."""
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(B * 100 + count)
    G = Hkv * 128
    # Arena per sequence: K plane [cap][G], then V plane [cap][G].
    kv = torch.randn(B, 2, cap, G, device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn(B, Hq, 128, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.tensor([count - 1], device="cuda", dtype=torch.int64)
    out = torch.empty(B, Hq * 128, device="cuda", dtype=torch.bfloat16)
    L = dl.lib()
    ws_bytes = L.dl_attention_decode_batched_workspace_bytes(B, Hq, Hkv, cap)
    if B * Hkv == 256 and torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert ws_bytes == B * Hq * 2 * 130 * 4  # two ranges per unit
    ws = torch.empty(ws_bytes // 4 + 1, device="cuda", dtype=torch.float32)
    assert L.dl_attention_decode_batched(q.data_ptr(), kv.data_ptr(), 2 * cap * G, 0, cap * G, pos.data_ptr(), B, Hq,
                                         Hkv, cap, out.data_ptr(), ws.data_ptr(), None) == 0, L.dl_last_error()
    torch.cuda.synchronize()
    k = kv[:, 0, :count].float().view(B, count, Hkv, 128)
    v = kv[:, 1, :count].float().view(B, count, Hkv, 128)
    grp = Hq // Hkv
    k = k.repeat_interleave(grp, dim=2)
    v = v.repeat_interleave(grp, dim=2)
    s = torch.einsum("bhd,bjhd->bhj", q.float(), k) / np.sqrt(128.0)
    p = torch.softmax(s, dim=-1)
    ref = torch.einsum("bhj,bjhd->bhd", p, v).reshape(B, Hq * 128)
    r = nm.compare_elementwise(ref.cpu().numpy(), out.float().cpu().numpy(), 2e-3, 1.6e-2)
    assert r["passed"], r


def _small_cfg(layers=2):
    return dl.Qwen3Config(hidden=1024, query_heads=16, kv_heads=4, head_width=128, mlp_width=3072,
                          vocabulary=2048, layers=layers)


def _close(ref_bits, got_bits):
    ref = nm.bf16_bits_to_f32(ref_bits)
    got = nm.bf16_bits_to_f32(got_bits)
    peak = float(np.max(np.abs(ref)))
    r = nm.compare_values(ref, got, max(1e-4, 0.0625 * peak), 0.03)
    return r["passed"] and nm.cosine(ref, got) > 0.999, r


def test_server_matches_single_sequence_engine():
    """Three sequences through the server (prompt in 16-row chunks, 5 decode
    steps) against each sequence alone through the engine's reference-law
    path, fed the server's tokens: logits within the fast-path tolerance."""
    cfg = _small_cfg()
    B, P, steps, cap = 3, 40, 5, 64
    srv = Server(cfg, batch=B, capacity=cap, chunk_rows=16)
    srv.init_random(3, 0.02)
    eng = dl.Engine(cfg, capacity=cap, max_rows=8)
    eng.init_random(3, 0.02)
    prompts = np.stack([oracle.uniform_ids(P, 7 + b, 0, cfg.vocabulary) for b in range(B)])
    first = srv.prefill(prompts)
    res = srv.decode(steps, want_logits=True)
    assert srv.position == P + steps
    agree = 0
    for b in range(B):
        eng.reset()
        logits = eng.consume_view(prompts[b])
        agree += int(np.argmax(nm.bf16_bits_to_f32(logits)) == int(first[b]))
        tokens = [int(first[b])] + [int(t) for t in res.tokens[:, b]]
        for i in range(steps):
            ref = eng.consume_view([tokens[i]])
            ok, r = _close(ref, res.logits[i, b])
            assert ok, (b, i, r)
            agree += int(np.argmax(nm.bf16_bits_to_f32(ref)) == tokens[i + 1])
    # Greedy choices: the server's own argmax, and (nearly always) the engine's.
    assert agree >= B * (steps + 1) - 1, agree


@pytest.mark.parametrize("capture_layer", [-1, 1])
def test_fused_decode_step_gives_the_same_bits_as_separate_kernels(capture_layer):
    """The fused step (the qkv split-K sums, QK-norm/RoPE and the KV append
    inside the attention kernel, which also merges its own splits; the o /
    down sums folded into residual + RMSNorm; chained programmatic launches)
    against the step as separate kernels: tokens,
    logits and the captured block output identical, with fewer launches.  A
    captured block keeps its separate residual epilogue (the hook sits between
    the residual add and the next norm)."""
    cfg = _small_cfg(3)
    B, P, steps = 3, 40, 6
    prompts = np.stack([oracle.uniform_ids(P, 70 + b, 0, cfg.vocabulary) for b in range(B)])
    runs = []
    for fused in (True, False):
        srv = Server(cfg, batch=B, capacity=64, chunk_rows=16)
        srv.init_random(11, 0.02)
        if capture_layer >= 0:
            srv.set_capture(capture_layer)
        srv.set_step_fusion(fused)
        first = srv.prefill(prompts, dl.Settings(dl.SelectionMode.categorical, 0.9, 0, 0.95), seed=5)
        res = srv.decode(steps, want_logits=True)
        cap = [srv.read_capture(b, 0, P + steps) for b in range(B)] if capture_layer >= 0 else []
        runs.append((first, res, cap))
        srv.close()
    (f1, r1, c1), (f0, r0, c0) = runs
    assert np.array_equal(f1, f0)
    assert np.array_equal(r1.tokens, r0.tokens)
    assert np.array_equal(r1.logits, r0.logits)
    for a, b in zip(c1, c0):
        assert np.array_equal(a, b)
    # 5 launches fewer per block (the qkv sum, QK-norm/RoPE/append, the
    # attention combine, two norms), 4 on the captured block.
    saved = 5 * cfg.layers - (1 if capture_layer >= 0 else 0)
    assert r0.kernels_per_decode_step - r1.kernels_per_decode_step == saved, (r0.kernels_per_decode_step,
                                                                               r1.kernels_per_decode_step)


def test_leading_range_attention_plan_in_the_decode_step():
    """56 sequences x 4 KV heads (224 units on 296 CTA slots of a 148-SM
    B200) at capacity 2048 take the leading-range attention plan: the fused
    step gives the same bits as the separate kernels, and the first decode
    step's logits of three of the sequences match a batch-3 server (even
    splits) within the fast-path tolerance."""
    torch = _torch()
    L = dl.lib()
    cfg = _small_cfg(2)
    B, P, cap, steps = 56, 1900, 2048, 4
    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert L.dl_attention_decode_batched_workspace_bytes(B, cfg.query_heads, cfg.kv_heads, cap) == \
            B * cfg.query_heads * 2 * 130 * 4
    prompts = np.stack([oracle.uniform_ids(P, 300 + b, 0, cfg.vocabulary) for b in range(B)])
    greedy = dl.Settings()
    runs = []
    for fused in (True, False):
        srv = Server(cfg, batch=B, capacity=cap, chunk_rows=512)
        srv.init_random(17, 0.02)
        srv.set_step_fusion(fused)
        first = srv.prefill(prompts, greedy)
        runs.append((first, srv.decode(steps, want_logits=True)))
        srv.close()
    (f1, r1), (f0, r0) = runs
    assert np.array_equal(f1, f0)
    assert np.array_equal(r1.tokens, r0.tokens)
    assert np.array_equal(r1.logits, r0.logits)
    small = Server(cfg, batch=3, capacity=cap, chunk_rows=512)
    small.init_random(17, 0.02)
    fs = small.prefill(prompts[:3], greedy)
    rs = small.decode(1, want_logits=True)
    small.close()
    assert np.array_equal(fs, f1[:3])
    for b in range(3):
        ok, r = _close(rs.logits[0, b], r1.logits[0, b])
        assert ok, (b, r)


def test_server_greedy_tokens_are_the_argmax_of_its_logits():
    cfg = _small_cfg(1)
    srv = Server(cfg, batch=2, capacity=48, chunk_rows=32)
    srv.init_random(5, 0.02)
    prompts = np.stack([oracle.uniform_ids(20, 40 + b, 0, cfg.vocabulary) for b in range(2)])
    srv.prefill(prompts)
    res = srv.decode(6, want_logits=True)
    for i in range(6):
        for b in range(2):
            assert int(res.tokens[i, b]) == int(np.argmax(nm.bf16_bits_to_f32(res.logits[i, b])))


def test_tensor_parallel_slices_match_full_tensors():
    cfg = _small_cfg(1)
    eng = dl.Engine(cfg, capacity=16, max_rows=4)
    eng.init_random(9, 0.02)
    tp = 2
    for rank in range(tp):
        srv = Server(cfg, batch=1, capacity=16, chunk_rows=8, tp_rank=rank, tp_size=tp)
        srv.init_random(9, 0.02)
        layout = tp_slices(cfg, rank, tp)
        for i in range(cfg.tensor_count()):
            rows, cols, r0, c0 = srv.slice_shape(i)
            assert (rows, cols, r0, c0) == layout[i], i
            full = eng.get_tensor(i)
            assert np.array_equal(srv.get_tensor(i), full[r0:r0 + rows, c0:c0 + cols]), (rank, i)
        srv.close()
    # set_tensor keeps the same slice of a host tensor.
    srv = Server(cfg, batch=1, capacity=16, chunk_rows=8, tp_rank=1, tp_size=2)
    idx = 3 + 6  # block 0 o_proj: column slice
    full = np.arange(np.prod(cfg.tensor_shape(idx)), dtype=np.uint32).astype(np.uint16).reshape(cfg.tensor_shape(idx))
    srv.set_tensor(idx, full)
    rows, cols, r0, c0 = srv.slice_shape(idx)
    half_q = cfg.query_heads * cfg.head_width // 2
    assert (r0, c0, rows, cols) == (0, half_q, cfg.hidden, half_q)
    assert np.array_equal(srv.get_tensor(idx), full[:, c0:c0 + cols])


def test_server_rejects_bad_shapes():
    cfg = _small_cfg(1)
    with pytest.raises(dl.DolittleError):
        Server(cfg, batch=1, capacity=16, chunk_rows=8, tp_rank=0, tp_size=3)   # 3 does not divide 4 KV heads
    srv = Server(cfg, batch=2, capacity=16, chunk_rows=8)
    with pytest.raises(dl.DolittleError):
        srv.decode(1)   # decode before prefill
    with pytest.raises(dl.DolittleError):
        srv.prefill(np.zeros((2, 16), np.uint32))  # prompt fills the capacity


def test_batched_categorical_selection_follows_the_device_law():
    """One sampler launch per kernel serves every row: row b's selections
    equal the device law on its own logits with the words of the MT19937-64
    stream seeded with seed + b (the prompt pass's selection used word 0)."""
    cfg = _small_cfg(1)
    B, seed = 3, 7
    srv = Server(cfg, batch=B, capacity=48, chunk_rows=32)
    srv.init_random(6, 0.02)
    prompts = np.stack([oracle.uniform_ids(16, 90 + b, 0, cfg.vocabulary) for b in range(B)])
    st = dl.Settings(dl.SelectionMode.categorical, 0.8, 0, 0.95)
    srv.prefill(prompts, st, seed=seed)
    res = srv.decode(5, want_logits=True)
    for b in range(B):
        mt = oracle.MT64(seed + b)
        mt()
        for i in range(5):
            logits = nm.bf16_bits_to_f32(res.logits[i, b])
            token, status = oracle.select_device(logits, True, 0.8, 0, 0.95, mt())
            assert status == 0 and token == int(res.tokens[i, b]), (b, i)
