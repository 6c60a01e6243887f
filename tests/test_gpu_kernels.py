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
