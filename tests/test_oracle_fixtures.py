"""The CPU oracle reproduces the reference's mlx-generated fixtures with the
reference's own tolerances (Tests/SwiftletCoreTests/FixtureForwardTests.swift,
IncrementalDecodeTests.swift, MetalKernelTests.swift)."""
import hashlib
import json
import os

import numpy as np
import pytest
from safetensors.numpy import load_file

import oracle
from conftest import REF_FIXTURES


def _fix(name):
    return load_file(os.path.join(REF_FIXTURES, name + ".safetensors"))


def _greedy(name):
    return json.load(open(os.path.join(REF_FIXTURES, name + ".json")))["greedy_next_tokens"]


def test_fixture_copies_match_recorded_digests():
    for line in open(os.path.join(REF_FIXTURES, "SHA256SUMS")):
        digest, rel = line.split()
        assert hashlib.sha256(open(os.path.join(REF_FIXTURES, rel), "rb").read()).hexdigest() == digest, rel


@pytest.mark.parametrize("model,fixture", [("tiny-model", "tiny_forward"), ("tiny-model-q35", "tiny_forward_q35")])
def test_forward_matches_mlx_layer_by_layer(model, fixture):
    # FixtureForwardTests.swift:21-82: per-layer from the reference input 5e-4,
    # end-to-end logits 0.05, greedy ids identical.
    m = oracle.OracleModel(os.path.join(REF_FIXTURES, model))
    f = _fix(fixture)
    toks = f["input_ids"].reshape(-1)
    caps = m.forward(toks)
    assert np.abs(caps["embed"] - f["embed"][0]).max() < 1e-6
    for i in range(m.L):
        ref_in = f["embed"][0] if i == 0 else f["layer_%02d" % (i - 1)][0]
        out = m.layer_forward(ref_in, i)
        assert np.abs(out - f["layer_%02d" % i][0]).max() < 5e-4, f"layer {i}"
    assert np.abs(caps["logits"] - f["logits"].reshape(len(toks), -1)).max() < 0.05
    assert caps["greedy"] == _greedy(fixture)


def test_quantized_forward_matches_mlx():
    # FixtureForwardTests.swift:86-102: int4 group-32 f32-scale fixture, 2e-3.
    m = oracle.OracleModel(os.path.join(REF_FIXTURES, "tiny-model-q4"))
    f = _fix("tiny_forward_q4")
    toks = f["input_ids"].reshape(-1)
    caps = m.forward(toks, capture_layers=False)
    assert np.abs(caps["logits"] - f["logits"].reshape(len(toks), -1)).max() < 2e-3
    assert caps["greedy"] == _greedy("tiny_forward_q4")


def test_incremental_matches_whole_sequence():
    # IncrementalDecodeTests.swift:15-40.
    m = oracle.OracleModel(os.path.join(REF_FIXTURES, "tiny-model"))
    tokens = [1, 5, 9, 42, 7, 99, 3, 17, 64, 2]
    full = m.forward(tokens, capture_layers=False)["logits"][-1]
    st = oracle.DecodeState()
    logits = m.step(tokens[:6], st)
    for t in tokens[6:]:
        logits = m.step([t], st)
    assert st.position == len(tokens)
    assert np.abs(logits - full).max() < 1e-4
    st2 = oracle.DecodeState()
    for t in tokens:
        logits = m.step([t], st2)
    assert np.abs(logits - full).max() < 1e-4


def test_greedy_continuation_is_deterministic():
    # IncrementalDecodeTests.swift:42-63.
    m = oracle.OracleModel(os.path.join(REF_FIXTURES, "tiny-model-q4"))

    def gen():
        st = oracle.DecodeState()
        logits = m.step([1, 5, 9], st)
        out = []
        for _ in range(8):
            best = int(np.argmax(logits))
            out.append(best)
            logits = m.step([best], st)
        return out

    a, b = gen(), gen()
    assert a == b and len(a) == 8


class Rand:
    """The reference's LCG (MetalKernelTests.swift:8-16)."""

    def __init__(self, seed):
        self.s = seed

    def next32(self):
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        return self.s >> 32

    def float(self):
        return np.float32(np.float32(self.next32()) / np.float32(4294967295.0) * np.float32(2) - np.float32(1))


def lcg_gemv_case(bits, seed=42, O=48, I=128, group=32):
    per = 32 // bits
    rng = Rand(seed)
    packed = np.array([rng.next32() for _ in range(O * I // per)], np.uint32)
    scales = np.array([rng.float() * np.float32(0.1) for _ in range(O * I // group)], np.float32)
    biases = np.array([rng.float() * np.float32(0.05) for _ in range(O * I // group)], np.float32)
    x = np.array([rng.float() for _ in range(I)], np.float32)
    return packed, scales, biases, x


def numpy_gemv(packed, scales, biases, O, I, group, bits, x):
    per = 32 // bits
    w = packed.reshape(O, I // per)
    q = np.stack([(w >> np.uint32(bits * j)) & np.uint32((1 << bits) - 1) for j in range(per)], -1).reshape(O, I)
    s = np.repeat(scales.reshape(O, I // group), group, axis=1)
    b = np.repeat(biases.reshape(O, I // group), group, axis=1)
    return ((s * q.astype(np.float32) + b) * x).sum(1, dtype=np.float64)


@pytest.mark.parametrize("bits", [4, 8])
def test_gemv_oracle_on_reference_lcg_case(bits):
    # MetalKernelTests.swift:21-77 construction (f32 and bf16 scales), 1e-3.
    packed, scales, biases, x = lcg_gemv_case(bits)
    ref = numpy_gemv(packed, scales, biases, 48, 128, 32, bits, x)
    y = oracle.gemv_affine(packed, scales, biases, 48, 128, 32, bits, x)
    assert np.abs(y - ref).max() < 1e-3
    sb = (scales.view(np.uint32) >> 16).astype(np.uint16)
    bb = (biases.view(np.uint32) >> 16).astype(np.uint16)
    ref_b = numpy_gemv(packed, (sb.astype(np.uint32) << 16).view(np.float32), (bb.astype(np.uint32) << 16).view(np.float32),
                       48, 128, 32, bits, x)
    yb = oracle.gemv_affine(packed, sb, bb, 48, 128, 32, bits, x)
    assert np.abs(yb - ref_b).max() < 1e-3


def test_gated_delta_oracle_on_reference_lcg_case():
    # MetalKernelTests.swift:79-128: T=5, Hk=2, Hv=4, Dk=32, Dv=8; 1e-4.
    T, Hk, Hv, Dk, Dv = 5, 2, 4, 32, 8
    rng = Rand(7)
    q = [rng.float() for _ in range(T * Hk * Dk)]
    k = [rng.float() for _ in range(T * Hk * Dk)]
    v = [rng.float() for _ in range(T * Hv * Dv)]
    g = [abs(rng.float()) * np.float32(0.9) for _ in range(T * Hv)]
    beta = [abs(rng.float()) for _ in range(T * Hv)]
    s0 = [rng.float() * np.float32(0.1) for _ in range(Hv * Dv * Dk)]
    y, st = oracle.gated_delta(q, k, v, g, beta, s0, T, Hk, Hv, Dk, Dv)
    # float64 restatement of the recurrence
    S = np.array(s0, np.float64).reshape(Hv, Dv, Dk)
    Y = np.zeros((T, Hv, Dv))
    qa, ka = np.array(q).reshape(T, Hk, Dk), np.array(k).reshape(T, Hk, Dk)
    va, ga, ba = np.array(v).reshape(T, Hv, Dv), np.array(g).reshape(T, Hv), np.array(beta).reshape(T, Hv)
    for t in range(T):
        for hv in range(Hv):
            hk = hv // (Hv // Hk)
            S[hv] *= ga[t, hv]
            kv = S[hv] @ ka[t, hk]
            d = (va[t, hv] - kv) * ba[t, hv]
            S[hv] += np.outer(d, ka[t, hk])
            Y[t, hv] = S[hv] @ qa[t, hk]
    assert np.abs(y - Y.reshape(-1)).max() < 1e-4
    assert np.abs(st - S.reshape(-1)).max() < 1e-4


def test_route_gap_is_smallest_topk_margin():
    # The oracle's near-tie measure used to screen parity inputs: the smallest
    # (p_k - p_k+1) / p_k over every routed row since the last reset.
    m = oracle.OracleModel(os.path.join(REF_FIXTURES, "tiny-model"))
    m.route_gap(reset=True)
    assert m.route_gap() == float("inf")
    rng = np.random.default_rng(3)
    x = rng.standard_normal((6, m.D)).astype(np.float32)
    _, ids, pp, probs = m.moe_forward(x, 0)
    s = -np.sort(-probs, axis=1)
    want = ((s[:, m.K - 1] - s[:, m.K]) / s[:, m.K - 1]).min()
    got = m.route_gap(reset=True)
    assert abs(got - want) <= 1e-6 * max(1.0, abs(want)), (got, want)
    assert m.route_gap() == float("inf")
