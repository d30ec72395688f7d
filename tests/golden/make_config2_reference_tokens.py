#!/usr/bin/env python3
"""Regenerate tests/golden/config2_reference_tokens.json on a GPU box.

    python tests/golden/make_config2_reference_tokens.py [output path]

The reference's own CUDA kernels (oracle/_ref/libref_cuda.so: its sources
compiled for compute_86 PTX, JIT-compiled by the driver) run BASELINE config 2
exactly as bench.py does: full Qwen3-8B (36 blocks, V=151936) with the seeded
BF16 weights of seed 1 (~N(0, 0.02), norms 1), the bench's 512-token prompt,
then 256 greedy decode steps, composed in the reference recipe order
(src/models/qwen3/model.cpp:343-409) with the reference host selection law
(src/inference/sampling/categorical.cpp:146-201) on the BF16 logits.  The
product engine only holds the weights in device memory; every number comes
from the reference kernels.  The output (prompt + 257 selected IDs) lets
bench.py report, without running any checker, whether its pipelines
reproduce the reference's greedy sequence.
"""
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
OUT = Path(__file__).resolve().parent / "config2_reference_tokens.json"


def main() -> None:
    import numpy as np

    import bench
    import dolittle_b200 as dl
    from oracle import oracle
    from tests import gpu_util as gu
    from tests import numerics as nm

    cfg = dl.QWEN3_8B
    cap = bench.PROMPT + bench.DECODE + 8
    e = dl.Engine(cfg, capacity=cap, max_rows=8)
    e.init_random(bench.SEED, 0.02)
    ptrs, keep = [], []
    for i in range(cfg.tensor_count()):
        p, stride = e.tensor_device(i)
        if stride != cfg.tensor_shape(i)[1]:
            t = gu.to_dev(e.get_tensor(i))
            keep.append(t)
            p = gu.ptr(t)
        ptrs.append(p)
    ref = gu.RefModel(cfg, ptrs, cap, bench.PROMPT)
    prompt = bench.prompt_ids(cfg.vocabulary)
    logits, _ = ref.forward(prompt, 0)
    tokens, pos = [], bench.PROMPT
    for i in range(bench.DECODE + 1):
        t = oracle.select_host(nm.bf16_bits_to_f32(logits), False)
        tokens.append(int(t))
        if i < bench.DECODE:
            logits, _ = ref.forward([t], pos)
            pos += 1
    rec = {"what": "reference CUDA kernels (compute_86 PTX JIT), config 2 greedy sequence",
           "seed": bench.SEED, "prompt": [int(v) for v in prompt], "tokens": tokens,
           "generator": os.path.relpath(__file__, ROOT)}
    out = Path(sys.argv[1]) if len(sys.argv) > 1 else OUT
    out.write_text(json.dumps(rec) + "\n")
    print(json.dumps({"written": str(out), "first_tokens": tokens[:8]}))


if __name__ == "__main__":
    main()
