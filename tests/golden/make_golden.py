#!/usr/bin/env python3
"""Regenerate the golden fixtures in this folder from the potpori reference checkout.

    python tests/golden/make_golden.py --reference <potpori checkout>

Source: the reference's own golden vectors in ``tests/fixtures/dspark_tiny`` (made by its
``tools/make_dspark_fixture.py`` with transformers): a 6-layer tiny Qwen3 target
(hidden 16, intermediate 32, 4 query / 2 KV heads of width 4, vocab 64, RoPE theta 1e4,
tied embeddings; BF16 matrices, F32 norms), transformers' logits for every position of a
59-token sequence, the outputs of layers 0, 2 and 4 for every position ("features"), the
11-token prompt and its greedy continuation. The reference checks its own forward against
them at 2e-3 (``src/qwen/cpu_check.rs:244-284``).

Written here (copied value for value, nothing recomputed):
  dspark_tiny_target.safetensors    the target's parameters as stored by the reference
  dspark_tiny_expected.safetensors  target_logits [59, 64] F32, features [59, 48] F32
  dspark_tiny.json                  target config, prompt, sequence, next_tokens
The DSpark drafter and its outputs are not copied: the drafter is outside this project.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil

from safetensors.torch import load_file, save_file

HERE = os.path.dirname(os.path.abspath(__file__))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True,
                    help="root of the potpori repository checkout")
    args = ap.parse_args()
    src = os.path.join(args.reference, "tests", "fixtures", "dspark_tiny")

    shutil.copyfile(os.path.join(src, "target.safetensors"),
                    os.path.join(HERE, "dspark_tiny_target.safetensors"))

    expected = load_file(os.path.join(src, "expected.safetensors"))
    save_file(
        {"target_logits": expected["target_logits"], "features": expected["features"]},
        os.path.join(HERE, "dspark_tiny_expected.safetensors"),
    )

    with open(os.path.join(src, "expected.json")) as f:
        meta = json.load(f)
    with open(os.path.join(src, "config.json")) as f:
        drafter_cfg = json.load(f)
    out = {
        "source": "potpori tests/fixtures/dspark_tiny (reference golden vectors)",
        "target": meta["target"],
        "feature_layers": drafter_cfg["target_layer_ids"],
        "prompt": meta["prompt"],
        "sequence": meta["sequence"],
        "next_tokens": meta["next_tokens"],
    }
    with open(os.path.join(HERE, "dspark_tiny.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
