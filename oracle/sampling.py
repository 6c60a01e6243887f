"""CPU restatement of Swiftlet's token sampler — TEST INFRASTRUCTURE ONLY.

Follows ``SwiftletSession.sample`` (Sources/SwiftletCore/SwiftletSession.swift
:226-273) step by step, in float32 and in the reference's sequential order:
suppressed ids and (when EOS is banned) the EOS ids set to -inf (:228-231);
presence/frequency penalty for every seen token (:232-236); temperature <= 0
takes the first maximum (:238-242); otherwise the top-k candidates (:244-254),
sorted by logit (:255), weights exp((l - l0) / T) (:256), top-p cut (:258-268)
and the walk of u * sum down the weights (:269-273), where u replaces
``Float.random(in: 0..<1)`` so that the draw is reproducible.

Ties at the k-th logit and in the sort are resolved toward the lower id (the
reference's replace-the-minimum scan and its unstable sort leave them
unspecified); seeded random logits have none. Parity unpinned: the reference
ships no sampling fixtures (its sampler is random), so this restatement is
checked against the reference's code by reading, and the GPU kernel against
this restatement. Only tests/ import it.
"""
from __future__ import annotations

import numpy as np

F = np.float32


def adjusted_logits(logits, suppress=(), eos=(), ban_eos=False, counts=None, presence=0.0, frequency=0.0):
    """SwiftletSession.swift:227-236 on one row (float32 copy)."""
    x = np.array(logits, dtype=F, copy=True)
    for t in suppress:
        x[t] = -np.inf
    if ban_eos:
        for t in eos:
            x[t] = -np.inf
    if counts is not None and (presence != 0 or frequency != 0):
        for t in np.nonzero(counts)[0]:
            pen = F(F(presence) + F(F(frequency) * F(counts[t])))
            x[t] = F(x[t] - pen)
    return x


def sample_row(logits, u, temperature, top_k, top_p, **adj):
    """Returns (token, margin): margin is how far the decision stood from a
    float32 boundary (the walk's remainder and the top-p comparison), for
    tests that skip rows whose choice a last-ulp exp difference could flip."""
    x = adjusted_logits(logits, **adj)
    V = x.shape[0]
    if temperature <= 0:
        return int(np.argmax(x)), np.inf  # np.argmax: first maximum
    k = max(1, min(int(top_k), V))
    order = np.lexsort((np.arange(V), -x.astype(np.float64)))[:k]  # logit desc, id asc
    vals = x[order]
    T = F(temperature)
    probs = np.array([np.exp(F(F(v - vals[0]) / T), dtype=F) for v in vals], dtype=F)
    s = F(0)
    for p in probs:
        s = F(s + p)
    cut = k
    margin = np.inf
    if top_p < 1:
        cum = F(0)
        for i in range(k):
            cum = F(cum + F(probs[i] / s))
            margin = min(margin, abs(float(cum) - float(top_p)))
            if cum >= F(top_p):
                cut = i + 1
                break
        s = F(0)
        for p in probs[:cut]:
            s = F(s + p)
    r = F(F(u) * s)
    for i in range(cut):
        r = F(r - probs[i])
        margin = min(margin, abs(float(r)) / max(float(s), 1e-30))
        if r <= 0:
            return int(order[i]), margin
    return int(order[0]), margin
