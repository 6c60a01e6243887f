"""BASELINE config 1 (tiny hybrid, q4 group 64 bf16): prompt logits within
2e-2 max-abs and 1e-3 relative-L2 of the oracle goldens, per-layer top-k
expert ids identical, and 32 greedy tokens identical."""
import json
import os

import numpy as np
import pytest

import oracle
import swiftlet_b200 as swl
from conftest import GOLDEN, TINY_BASELINE

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def golden():
    return json.load(open(os.path.join(GOLDEN, "tiny_baseline_golden.json")))


def test_prompt_logits_and_32_greedy_tokens(golden):
    gpu = swl.QwenCUDAModel(TINY_BASELINE)
    st = swl.DecodeState(64)
    logits = gpu.step(golden["prompt"], st)
    ref = np.array(golden["prompt_logits"], np.float32)
    assert np.abs(logits - ref).max() < 2e-2
    assert np.linalg.norm(logits - ref) / np.linalg.norm(ref) < 1e-3
    out = []
    for _ in range(32):
        best = int(np.argmax(logits))
        out.append(best)
        logits = gpu.step([best], st)
    assert out == golden["greedy_32"]


def test_topk_ids_per_layer_at_first_position(golden):
    cpu = oracle.OracleModel(TINY_BASELINE)
    gpu = swl.QwenCUDAModel(TINY_BASELINE)
    caps = cpu.forward(golden["prompt"][:1])
    h = caps["embed"][0]
    for layer in range(cpu.L):
        out, ids, w = gpu.debug_layer(swl.DecodeState(8), layer, h)
        assert ids.tolist() == golden["topk_ids_per_layer"][layer][0], layer
        assert np.abs(out - caps["layers"][layer][0]).max() < 1e-4
        h = caps["layers"][layer][0]
