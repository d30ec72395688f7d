"""One rank of the tensor-parallel serving check (launched by
tests/test_gpu_serve_tp.py through torch.distributed.run).

Every rank holds its slice of the same seeded weights (TP over KV-head
groups); the o_proj / down_proj partial sums meet in the NCCL all-reduce.
Rank 0 also runs the whole model on one GPU (TP = 1) and compares: every
decode step's logits within the fast-path tolerance and the same greedy
tokens on every rank.  Prints one JSON line on rank 0; exit status 0 = pass.
"""
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import dolittle_b200 as dl  # noqa: E402
from dolittle_b200.serve import Server, connect_group  # noqa: E402
from oracle import oracle  # noqa: E402
from tests import numerics as nm  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    layers = int(os.environ.get("TP_LAYERS", "2"))
    cfg = dl.Qwen3Config(hidden=1024, query_heads=16, kv_heads=4, head_width=128, mlp_width=3072,
                         vocabulary=2048, layers=layers)
    B, P, steps, cap = 2, 40, 6, 64
    prompts = np.stack([oracle.uniform_ids(P, 70 + b, 0, cfg.vocabulary) for b in range(B)])
    srv = Server(cfg, batch=B, capacity=cap, chunk_rows=16, device=rank, tp_rank=rank, tp_size=world)
    srv.init_random(11, 0.02)
    connect_group(srv, dist)
    first = srv.prefill(prompts)
    res = srv.decode(steps, want_logits=True)
    got = [first.tolist(), res.tokens.tolist()]
    everyone = [None] * world
    dist.all_gather_object(everyone, got)
    ok = all(e == got for e in everyone)
    report = {"ranks_agree": ok}
    if rank == 0:
        ref = Server(cfg, batch=B, capacity=cap, chunk_rows=16, device=0)
        ref.init_random(11, 0.02)
        first_ref = ref.prefill(prompts)
        out_ref = ref.decode(steps, want_logits=True)
        worst = 0.0
        close = True
        for i in range(steps):
            for b in range(B):
                a = nm.bf16_bits_to_f32(out_ref.logits[i, b])
                g = nm.bf16_bits_to_f32(res.logits[i, b])
                peak = float(np.max(np.abs(a)))
                r = nm.compare_values(a, g, max(1e-4, 0.0625 * peak), 0.03)
                close = close and r["passed"] and nm.cosine(a, g) > 0.999
                worst = max(worst, float(np.max(np.abs(a - g))) / max(peak, 1e-6))
        same_tokens = (first_ref.tolist() == first.tolist()) and np.array_equal(out_ref.tokens, res.tokens)
        report.update({"logits_close": close, "worst_rel_max_abs": worst, "same_greedy_tokens": bool(same_tokens),
                       "tp": world})
        ok = ok and close
        ref.close()
        print(json.dumps(report), flush=True)
    srv.close()
    flag = torch.tensor([1 if ok else 0])
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    return 0 if int(flag.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
