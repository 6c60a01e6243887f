"""The MID goldens (tests/golden/mid_golden.json) are what the CPU oracle
computes on the MID synthetic model: the committed prompt logits, 32 greedy
tokens and margins are regenerated here and must agree."""
import json
import os

import numpy as np

from conftest import GOLDEN
from golden.make_mid_golden import generate, mid_checkpoint, mid_prompt


def test_oracle_reproduces_mid_goldens(tmp_path):
    g = json.load(open(os.path.join(GOLDEN, "mid_golden.json")))
    assert g["prompt"] == mid_prompt()
    fresh = generate(mid_checkpoint(str(tmp_path / "mid")))
    assert fresh["greedy_32"] == g["greedy_32"]
    assert np.abs(np.array(fresh["prompt_logits"]) - np.array(g["prompt_logits"])).max() < 1e-6
    # the greedy chain is decided by a clear margin: a GPU result within the
    # logit tolerance cannot flip it
    assert min(g["margins"]) > 0.02
