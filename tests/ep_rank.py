"""One rank of the expert-parallel parity check (run by tests/test_gpu_ep.py).

Usage: python tests/ep_rank.py <model_dir> <rank> <world> <id_hex> <tokens_per_rank> <steps> <out_json>

The rank opens the checkpoint twice on GPU `rank`: a plain model (the whole
MoE on this GPU, the batched path the single-GPU tests pin to the oracle) and
an expert-parallel one that computes only its share of the routed experts and
exchanges partial sums with the other ranks over NCCL. Both prefill the same
seeded prompts, then decode `steps` greedy tokens (fed from the plain model's
argmax so both see the same inputs); the logits of every step are compared
within the logit tolerances of the batched parity tests (2e-2 max-abs, 1e-3
relative-L2).
"""
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
# torch first: its libnccl.so.2 is then the one the library's dlopen() finds,
# the same NCCL build as the test process that made the communicator id
import torch  # noqa: E402,F401
import swiftlet_b200 as swl  # noqa: E402

MAX_ABS, REL_L2 = 2e-2, 1e-3


def main() -> int:
    d, rank, world, id_hex, tpr, steps, out = sys.argv[1:8]
    rank, world, tpr, steps = int(rank), int(world), int(tpr), int(steps)
    plain = swl.QwenCUDAModel(d, device=rank)
    ep = swl.QwenCUDAModel(d, device=rank)
    ep.ep_init(rank, world, bytes.fromhex(id_hex), tpr)
    on, r, w, lo, hi = ep.ep_info()
    V = plain.config.vocab_size
    rng = np.random.default_rng(1000 + rank)
    # prompts of 2+ tokens: a prompt call stays on the rank on every rank alike
    # (a call of one token per sequence would be a decode call, which exchanges)
    prompts = [rng.integers(0, V, int(n)).tolist() for n in rng.integers(2, 7, tpr)]
    ps = [plain.new_state(64) for _ in prompts]
    es = [ep.new_state(64) for _ in prompts]
    ref = plain.step_batch(prompts, ps)
    got = ep.step_batch(prompts, es)
    worst_abs, worst_rel, same_greedy = 0.0, 0.0, True
    for step in range(steps + 1):
        for i in range(tpr):
            err = float(np.abs(got[i] - ref[i]).max())
            rel = float(np.linalg.norm(got[i] - ref[i]) / (np.linalg.norm(ref[i]) + 1e-30))
            worst_abs, worst_rel = max(worst_abs, err), max(worst_rel, rel)
            same_greedy = same_greedy and int(np.argmax(got[i])) == int(np.argmax(ref[i]))
        if step == steps:
            break
        toks = [[int(np.argmax(r_))] for r_ in ref]
        ref = plain.step_batch(toks, ps)
        got = ep.step_batch(toks, es)
    res = {"rank": rank, "world": world, "ep_on": on, "expert_lo": lo, "expert_hi": hi, "max_abs": worst_abs,
           "rel_l2": worst_rel, "same_greedy": same_greedy,
           "positions": [s.position for s in es] == [s.position for s in ps]}
    with open(out, "w") as f:
        json.dump(res, f)
    ep.close()
    plain.close()
    ok = on and worst_abs < MAX_ABS and worst_rel < REL_L2 and res["positions"]
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
