#!/usr/bin/env python3
"""Regenerate tests/golden/tiny-bf16/ from the reference's own Python oracle.

Run in the development container, where the reference tree is mounted,
with DOLITTLE_REFERENCE naming it (else BASELINE.json's reference_path):

    DOLITTLE_REFERENCE=<reference tree> python tests/golden/make_tiny_fixture.py

It imports scripts/validation/forward_reference.py from the reference and
calls its generate(kind="tiny-bf16", device="cpu") directly.  That function
builds the reference's independent tiny Qwen3 (3 blocks, D=24, Hq=4, Hkv=2,
d=8, F=40, V=37, theta 1e4, seed 20261018; forward_reference.py:230-240),
runs its FP32 one-row-projection / per-query-attention policy, and writes
config.json, model.safetensors and fixture.json (logits and block captures
with the reference's own tolerances).  The script's main() pins Transformers
4.57.3; this container has a later Transformers, so generate() is called
directly and the version actually used is recorded in fixture.json.  Nothing
at test time reads the reference tree: only the committed outputs.
"""
import importlib
import json
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "tiny-bf16"


def main() -> None:
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
    from oracle.oracle import reference_tree
    ref = reference_tree()
    if ref is None:
        raise SystemExit("set DOLITTLE_REFERENCE to the reference source tree")
    REFERENCE = Path(ref)
    sys.path.insert(0, str(REFERENCE / "scripts" / "validation"))
    fr = importlib.import_module("forward_reference")
    import torch
    torch.set_num_threads(8)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    OUT.mkdir(parents=True, exist_ok=True)
    for stale in OUT.iterdir():
        stale.unlink()
    env = fr.environment("cpu")
    fr.generate(OUT, "tiny-bf16", None, None, env, "cpu")
    fixture = json.loads((OUT / "fixture.json").read_text())
    print(json.dumps({"written": sorted(p.name for p in OUT.iterdir()),
                      "cases": [c["name"] for c in fixture["cases"]],
                      "generation_tokens": fixture["generation"]["reference"]["token_ids"]}))


if __name__ == "__main__":
    main()
