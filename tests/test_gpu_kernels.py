"""Kernel-level parity of the MLX-affine GEMV (the decode path's weight
streamer) against the CPU oracle, on the reference's LCG construction
(MetalKernelTests.swift:21-77) and on decode-path shapes."""
import numpy as np
import pytest

import oracle
import swiftlet_b200 as swl
from test_oracle_fixtures import lcg_gemv_case

pytestmark = pytest.mark.gpu


def _bf16(a):
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("sdtype", ["f32", "bf16", "f16"])
def test_gemv_matches_oracle_on_reference_case(bits, sdtype):
    packed, scales, biases, x = lcg_gemv_case(bits)
    if sdtype == "bf16":
        scales, biases = _bf16(scales), _bf16(biases)
    elif sdtype == "f16":
        scales, biases = scales.astype(np.float16), biases.astype(np.float16)
    ref = oracle.gemv_affine(packed, scales, biases, 48, 128, 32, bits, x)
    y = swl.gemv_affine(packed, scales, biases, 48, 128, 32, bits, x)
    assert np.abs(y - ref).max() < 1e-3   # the reference's tolerance


@pytest.mark.parametrize("bits,out,inn,group", [(4, 512, 2048, 64), (4, 2048, 512, 64), (4, 1000, 4096, 64),
                                                (8, 256, 2048, 64), (4, 333, 2048, 128), (8, 77, 512, 32)])
def test_gemv_matches_oracle_on_decode_shapes(bits, out, inn, group):
    rng = np.random.default_rng(out * 7 + inn)
    per = 32 // bits
    packed = rng.integers(0, 2**32, size=out * inn // per, dtype=np.uint64).astype(np.uint32)
    scales = _bf16(np.abs(rng.normal(0, 0.01, out * inn // group)))
    biases = _bf16(rng.normal(0, 0.01, out * inn // group))
    x = rng.normal(0, 1, inn).astype(np.float32)
    ref = oracle.gemv_affine(packed, scales, biases, out, inn, group, bits, x)
    y = swl.gemv_affine(packed, scales, biases, out, inn, group, bits, x)
    scale = np.abs(ref).max() + 1e-6
    assert np.abs(y - ref).max() / scale < 1e-5


def random_affine(rng, out, inn, group, bits, sdtype="bf16"):
    per = 32 // bits
    packed = rng.integers(0, 2**32, size=out * inn // per, dtype=np.uint64).astype(np.uint32)
    s = np.abs(rng.normal(0, 0.01, out * inn // group)).astype(np.float32)
    b = rng.normal(0, 0.01, out * inn // group).astype(np.float32)
    if sdtype == "bf16":
        s, b = _bf16(s), _bf16(b)
    return packed, s, b


@pytest.mark.parametrize("bits,hidden,inter,group,sdtype", [(4, 2048, 512, 64, "bf16"), (8, 2048, 512, 64, "bf16"),
                                                            (4, 64, 32, 32, "f32"), (4, 1024, 256, 128, "bf16")])
def test_expert_swiglu_matches_oracle(bits, hidden, inter, group, sdtype):
    rng = np.random.default_rng(hidden + inter + bits)
    gate = random_affine(rng, inter, hidden, group, bits, sdtype)
    up = random_affine(rng, inter, hidden, group, bits, sdtype)
    down = random_affine(rng, hidden, inter, group, bits, sdtype)
    x = rng.normal(0, 1, hidden).astype(np.float32)
    ref = oracle.expert_swiglu(gate, up, down, hidden, inter, group, bits, x)
    y = swl.expert_swiglu(gate, up, down, hidden, inter, group, bits, x)
    assert np.abs(y - ref).max() / (np.abs(ref).max() + 1e-6) < 1e-5


def _delta_inputs(rng, T, Hk, Hv, Dk, Dv):
    """Inputs as the decode path forms them: k unit-norm, q of norm 1/sqrt(dk)
    (RMSNorm scaled 1/sqrt(dk) and 1/dk), g = exp(-exp(A) softplus(a)),
    beta = sigmoid(b) (QwenCPUModel.swift:423-458)."""
    q = rng.normal(0, 1, (T, Hk, Dk)).astype(np.float32)
    k = rng.normal(0, 1, (T, Hk, Dk)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True) * np.sqrt(Dk)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.normal(0, 1, (T, Hv, Dv)).astype(np.float32)
    a_log = rng.uniform(0, 1, Hv)
    g = np.exp(-np.exp(a_log) * np.log1p(np.exp(rng.normal(0, 1, (T, Hv))))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.normal(0, 1, (T, Hv))))).astype(np.float32)
    state = rng.normal(0, 0.1, (Hv, Dv, Dk)).astype(np.float32)
    return q, k, v, g, beta, state


@pytest.mark.parametrize("T", [1, 64, 65, 130, 4096])
def test_chunked_delta_rule_matches_sequential_oracle(T):
    """The chunk-parallel prompt kernel (64-token chunks, triangular solve)
    against the oracle's token-by-token recurrence (MetalKernelTests.swift:
    194-220 construction): outputs and final state within 1e-4 relative."""
    Hk, Hv, Dk, Dv = 2, 4, 128, 128
    q, k, v, g, beta, state = _delta_inputs(np.random.default_rng(T), T, Hk, Hv, Dk, Dv)
    y_ref, s_ref = oracle.gated_delta(q, k, v, g, beta, state, T, Hk, Hv, Dk, Dv)
    y, s = swl.gated_delta(q, k, v, g, beta, state, T, Hk, Hv, Dk, Dv)
    assert np.abs(y - y_ref).max() / (np.abs(y_ref).max() + 1e-6) < 1e-4
    assert np.abs(s - s_ref).max() / (np.abs(s_ref).max() + 1e-6) < 1e-4
