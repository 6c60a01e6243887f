"""The sampler restatement (oracle/sampling.py) against a second reading of
SwiftletSession.sample (SwiftletSession.swift:226-273) that keeps the
reference's control flow: the replace-the-minimum top-k scan over a fixed
candidate set, the sort, the top-p loop and the walk of u * sum. Tie-free
seeded rows, so both must pick the same token."""
import numpy as np
import pytest

from oracle import sampling

F = np.float32


def control_flow_reading(x, u, temperature, top_k, top_p):
    V = len(x)
    if temperature <= 0:
        best = 0
        for v in range(1, V):
            if x[v] > x[best]:
                best = v
        return best
    k = max(1, min(top_k, V))
    cand = list(range(k))
    mn = min(range(k), key=lambda i: (x[cand[i]], i))
    for v in range(k, V):
        if x[v] > x[cand[mn]]:
            cand[mn] = v
            mn = min(range(k), key=lambda i: (x[cand[i]], i))
    top = sorted(((c, x[c]) for c in cand), key=lambda t: -t[1])
    probs = [np.exp(F(F(t[1] - top[0][1]) / F(temperature)), dtype=F) for t in top]
    s = F(0)
    for p in probs:
        s = F(s + p)
    if top_p < 1:
        cum, cut = F(0), len(probs)
        for i, p in enumerate(probs):
            cum = F(cum + F(p / s))
            if cum >= F(top_p):
                cut = i + 1
                break
        top, probs = top[:cut], probs[:cut]
        s = F(0)
        for p in probs:
            s = F(s + p)
    r = F(F(u) * s)
    for i, p in enumerate(probs):
        r = F(r - p)
        if r <= 0:
            return top[i][0]
    return top[0][0]


@pytest.mark.parametrize("temperature,top_k,top_p", [(0.7, 20, 0.8), (0.0, 20, 0.8), (1.0, 5, 1.0), (0.3, 64, 0.95)])
def test_restatement_follows_reference_control_flow(temperature, top_k, top_p):
    rng = np.random.default_rng(11)
    for _ in range(40):
        x = rng.normal(0, 2, 200).astype(F)
        counts = (rng.random(200) < 0.1) * rng.integers(1, 4, 200)
        u = float(rng.random())
        adj = dict(suppress=[3, 7], eos=[199], ban_eos=True, counts=counts, presence=1.5, frequency=0.5)
        got, _ = sampling.sample_row(x, u, temperature, top_k, top_p, **adj)
        want = control_flow_reading(sampling.adjusted_logits(x, **adj), u, temperature, top_k, top_p)
        assert got == want


def test_penalty_and_suppression():
    x = np.zeros(8, F)
    x[2], x[5] = 3.0, 2.0
    counts = np.zeros(8, np.int64)
    counts[2] = 2
    y = sampling.adjusted_logits(x, suppress=[0], eos=[7], ban_eos=True, counts=counts, presence=1.5, frequency=0.5)
    assert y[0] == -np.inf and y[7] == -np.inf and y[2] == F(3.0 - (1.5 + 0.5 * 2))
    assert sampling.sample_row(x, 0.5, 0.0, 20, 0.8, counts=counts, presence=1.5, frequency=0.5)[0] == 5
