"""On-device sampling (swl_sample_device) against the CPU restatement of
SwiftletSession.sample (oracle/sampling.py) on 64 rows of a 151,936-token
vocabulary: suppressed ids, EOS banned in every other row, presence and
frequency penalties from per-row counts, and the reference's default options
(temperature 0.7, top-k 20, top-p 0.8) besides greedy, wide top-k and top-1
settings. The chosen ids must be equal on every row whose decision stands
further than 1e-5 from a float32 boundary (where a last-ulp difference of
exp could flip it); nearly every row qualifies."""
import numpy as np
import pytest

import swiftlet_b200 as swl
from oracle import sampling

pytestmark = pytest.mark.gpu

V, S = 151936, 64


@pytest.fixture(scope="module")
def rows():
    import torch
    rng = np.random.default_rng(5)
    logits = rng.normal(0, 3, (S, V)).astype(np.float32)
    counts = ((rng.random((S, V)) < 2e-4) * rng.integers(1, 5, (S, V))).astype(np.int32)
    suppress = np.array([0, 17, 151643, 151935], np.int32)
    eos = np.array([151645, 151643, 5], np.int32)
    ban = (np.arange(S) % 2).astype(np.int32)
    u = rng.random(S).astype(np.float32)
    dev = {k: torch.from_numpy(v).cuda() for k, v in
           dict(logits=logits, counts=counts, suppress=suppress, eos=eos, ban=ban, u=u).items()}
    return dict(logits=logits, counts=counts, suppress=suppress, eos=eos, ban=ban, u=u, dev=dev)


@pytest.mark.parametrize("temperature,top_k,top_p,pres,freq", [
    (0.7, 20, 0.8, 1.5, 0.5), (0.0, 20, 0.8, 1.5, 0.5), (1.0, 1024, 1.0, 0.0, 0.0), (0.9, 1, 0.5, 0.0, 0.0),
    (1.3, 300, 0.95, 0.2, 0.1)])
def test_sampled_ids_match_restatement(rows, temperature, top_k, top_p, pres, freq):
    import torch
    d = rows["dev"]
    out = torch.full((S,), -1, dtype=torch.int32, device="cuda")
    swl.sample_device(d["logits"].data_ptr(), S, V, V, temperature=temperature, top_k=top_k, top_p=top_p,
                      presence_penalty=pres, frequency_penalty=freq, d_suppress=d["suppress"].data_ptr(),
                      n_suppress=len(rows["suppress"]), d_eos=d["eos"].data_ptr(), n_eos=len(rows["eos"]),
                      d_ban_eos=d["ban"].data_ptr(), d_counts=d["counts"].data_ptr(), d_uniform=d["u"].data_ptr(),
                      d_out=out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    checked = 0
    for i in range(S):
        want, margin = sampling.sample_row(
            rows["logits"][i], float(rows["u"][i]), temperature, top_k, top_p, suppress=rows["suppress"],
            eos=rows["eos"], ban_eos=bool(rows["ban"][i]), counts=rows["counts"][i], presence=pres, frequency=freq)
        if margin > 1e-5:
            checked += 1
            assert got[i] == want, (i, got[i], want, margin)
    assert checked >= S - 3


def test_counts_update_and_greedy_feedback(rows):
    import torch
    d = rows["dev"]
    counts = d["counts"].clone()
    out = torch.empty(S, dtype=torch.int32, device="cuda")
    for _ in range(2):
        swl.sample_device(d["logits"].data_ptr(), S, V, V, temperature=0.0, d_counts=counts.data_ptr(),
                          update_counts=True, d_out=out.data_ptr())
    torch.cuda.synchronize()
    first = int(np.argmax(rows["logits"][0]))
    c = counts.cpu().numpy()
    # greedy without penalties picks the plain argmax twice
    assert int(out[0]) == first and c[0, first] == rows["counts"][0, first] + 2


def test_rejects_wide_top_k():
    import torch
    x = torch.zeros((1, V), device="cuda")
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    u = torch.zeros(1, device="cuda")
    with pytest.raises(swl.SwiftletError):
        swl.sample_device(x.data_ptr(), 1, V, V, temperature=1.0, top_k=2048, d_uniform=u.data_ptr(),
                          d_out=out.data_ptr())
