"""Writes the goldens of the MID synthetic model (tests/golden/mid_golden.json).

MID (swiftlet_b200.configs.MID) is the 35B layout shrunk to hidden 512 and 4
layers; its weights come from the counter-based synthetic generator (seed
MID_SEED), so the checkpoint itself is only a config.json that the tests
write to a temporary directory. Every linear module of MID takes the integer
tensor-core decode kernels (the ones the bench times), which the reference's
tiny fixtures do not reach.

The goldens are produced by the CPU oracle (oracle/, the restatement of
QwenCPUModel.swift): an 8-id prompt drawn from numpy's PCG64 with the same
seed, the logits after the prompt, 32 greedy continuation tokens and, per
greedy step, the margin between the best and the second-best logit.

Usage: python tests/golden/make_mid_golden.py
"""
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from swiftlet_b200 import formats  # noqa: E402
from swiftlet_b200.configs import MID, MID_SEED  # noqa: E402

OUT = os.path.join(HERE, "mid_golden.json")


def mid_checkpoint(dirname: str) -> str:
    """The MID synthetic checkpoint (config.json only) in `dirname`."""
    return formats.write_synthetic(dirname, MID, seed=MID_SEED)


def mid_prompt() -> list[int]:
    return np.random.default_rng(MID_SEED).integers(0, MID["vocab_size"], 8).tolist()


def generate(model_dir: str) -> dict:
    cpu = oracle.OracleModel(model_dir)
    st = oracle.DecodeState()
    prompt = mid_prompt()
    logits = cpu.step(prompt, st)
    out = {"seed": MID_SEED, "prompt": prompt, "prompt_logits": [float(v) for v in logits]}
    greedy, margins = [], []
    for _ in range(32):
        s = np.sort(logits)
        margins.append(float(s[-1] - s[-2]))
        t = int(np.argmax(logits))
        greedy.append(t)
        logits = cpu.step([t], st)
    out["greedy_32"] = greedy
    out["margins"] = margins
    return out


def main() -> None:
    with tempfile.TemporaryDirectory() as d:
        g = generate(mid_checkpoint(d))
    with open(OUT, "w") as f:
        json.dump(g, f)
    print(f"wrote {OUT}: greedy {g['greedy_32'][:8]}..., min margin {min(g['margins']):.4f}")


if __name__ == "__main__":
    main()
