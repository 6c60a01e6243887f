"""The CUDA model reproduces the CPU oracle on the reference's tiny fixtures
(MetalModelTests.swift:15-81, QpackTests.swift:68-121): logits within 2e-3
and identical greedy tokens, for int4 / f32 models, both DeltaNet layouts,
and the .qpack container path."""
import json
import os

import numpy as np
import pytest

import oracle
import swiftlet_b200 as swl
from conftest import REF_FIXTURES
from swiftlet_b200 import formats

pytestmark = pytest.mark.gpu
TOKENS = [1, 5, 9, 42, 7]


def compare(model_dir, oracle_dir=None, tokens=TOKENS, budget=0.0):
    cpu = oracle.OracleModel(oracle_dir or model_dir)
    gpu = swl.QwenCUDAModel(model_dir, cache_budget_gb=budget)
    cs, gs = oracle.DecodeState(), swl.DecodeState(64)
    for t in tokens:
        cl = cpu.step([t], cs)
        gl = gpu.step([t], gs)
    assert gs.position == len(tokens)
    assert np.abs(cl - gl).max() < 2e-3
    assert int(np.argmax(cl)) == int(np.argmax(gl))
    return gpu


@pytest.mark.parametrize("name", ["tiny-model-q4", "tiny-model", "tiny-model-q35"])
def test_gpu_matches_oracle(name):
    compare(os.path.join(REF_FIXTURES, name))


@pytest.mark.parametrize("name,fixture", [("tiny-model-q4", "tiny_forward_q4"), ("tiny-model", "tiny_forward"),
                                          ("tiny-model-q35", "tiny_forward_q35")])
def test_gpu_greedy_matches_mlx_fixture(name, fixture):
    # greedy_next_tokens[i] is the argmax after consuming tokens[0..i].
    man = json.load(open(os.path.join(REF_FIXTURES, fixture + ".json")))
    gpu = swl.QwenCUDAModel(os.path.join(REF_FIXTURES, name))
    st = swl.DecodeState(64)
    got = [int(np.argmax(gpu.step([t], st))) for t in man["tokens"]]
    assert got == man["greedy_next_tokens"]


def test_gpu_qpack_container_matches_oracle(tmp_path):
    src = os.path.join(REF_FIXTURES, "tiny-model-q4")
    out = str(tmp_path / "tiny-q4.qpack")
    formats.repack(src, out)
    gpu = compare(out, oracle_dir=src, tokens=[1, 5, 9, 42, 7, 99], budget=0.05)
    stats = gpu.expert_cache
    assert stats.hits + stats.misses > 0
    assert stats.stride % formats.PAGE_ALIGNMENT == 0


def test_prefill_matches_token_by_token():
    d = os.path.join(REF_FIXTURES, "tiny-model")
    gpu = swl.QwenCUDAModel(d)
    tokens = [1, 5, 9, 42, 7, 99, 3, 17, 64, 2]
    a = swl.DecodeState(64)
    la = gpu.step(tokens[:6], a)
    for t in tokens[6:]:
        la = gpu.step([t], a)
    b = swl.DecodeState(64)
    for t in tokens:
        lb = gpu.step([t], b)
    assert a.position == b.position == len(tokens)
    assert np.abs(la - lb).max() < 1e-5
    full = oracle.OracleModel(d).forward(tokens, capture_layers=False)["logits"][-1]
    assert np.abs(la - full).max() < 2e-3


def test_interleaved_states_do_not_interfere():
    # Device state is per sequence (the reference keeps one GPU state per model).
    d = os.path.join(REF_FIXTURES, "tiny-model-q4")
    gpu = swl.QwenCUDAModel(d)
    s1, s2, s3 = swl.DecodeState(64), swl.DecodeState(64), swl.DecodeState(64)
    seq_a, seq_b = [1, 5, 9, 42], [7, 99, 3, 17]
    for x, y in zip(seq_a, seq_b):
        la = gpu.step([x], s1)
        lb = gpu.step([y], s2)
    for x in seq_a:
        ref = gpu.step([x], s3)
    assert np.abs(la - ref).max() == 0.0
    cpu = oracle.OracleModel(d)
    cs = oracle.DecodeState()
    for y in seq_b:
        cl = cpu.step([y], cs)
    assert np.abs(lb - cl).max() < 2e-3


def test_token_out_of_range_is_rejected():
    gpu = swl.QwenCUDAModel(os.path.join(REF_FIXTURES, "tiny-model-q4"))
    st = swl.DecodeState(8)
    with pytest.raises(swl.SwiftletError) as e:
        gpu.step([128], st)
    assert e.value.code == swl.SWL_ERR_INVALID
    assert st.position == 0
    gpu.step(list(range(8)), st)
    with pytest.raises(swl.SwiftletError) as e:
        gpu.step([1], st)
    assert e.value.code == swl.SWL_ERR_CAPACITY


def test_dequant_is_bit_exact():
    d = os.path.join(REF_FIXTURES, "tiny-model-q4")
    cpu = oracle.OracleModel(d)
    gpu = swl.QwenCUDAModel(d)
    for mod, rows, cols in [("model.embed_tokens", (0, 128), 64), ("model.layers.0.linear_attn.in_proj_qkvz", (0, 96), 64),
                            ("model.layers.3.self_attn.o_proj", (0, 64), 64),
                            ("model.layers.2.mlp.switch_mlp.down_proj", (64, 256), 32)]:
        a = cpu.dequant(mod, rows[0], rows[1], cols)
        b = gpu.debug_dequant(mod, rows[0], rows[1], cols)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), mod


def test_long_context_matches_oracle():
    # 200 positions: the attention layer splits the context over several
    # chunks (and sub-tiles) whose partial softmax results are combined.
    d = os.path.join(REF_FIXTURES, "tiny-model-q4")
    cpu = oracle.OracleModel(d)
    gpu = swl.QwenCUDAModel(d)
    cs, gs = oracle.DecodeState(), swl.DecodeState(256)
    vocab = json.load(open(os.path.join(d, "config.json")))["vocab_size"]
    rng = np.random.default_rng(5)
    toks = [int(t) for t in rng.integers(0, vocab, 200)]
    for i, t in enumerate(toks):
        cl = cpu.step([t], cs)
        gl = gpu.step([t], gs)
        if i % 25 == 24 or i == len(toks) - 1:
            assert np.abs(cl - gl).max() < 2e-3, i
            assert int(np.argmax(cl)) == int(np.argmax(gl)), i
