"""One rank of the expert-parallel failure-path check (run by tests/test_gpu_ep.py).

Usage: python tests/ep_stall.py <model_dir> <rank> <world> <id_hex> <flag_dir> <out_json>

Both ranks join the group (SWL_EP_TIMEOUT_MS set by the test), prefill and
run two decode steps together. Then rank 1 stops taking part: it stays alive
(its memory stays valid) but makes no further call until rank 0 has written
`done` to flag_dir. Rank 0 makes a third decode step, whose exchange has no
partner: the library's watchdog must abort the communicator after the
timeout, that call and the next must fail with SWL_ERR_CUDA instead of
waiting forever, and the model must still close.
"""
import json
import os
import sys
import time

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import torch  # noqa: E402,F401  (torch's libnccl.so.2 first)
import swiftlet_b200 as swl  # noqa: E402


def main() -> int:
    d, rank, world, id_hex, flags, out = sys.argv[1:7]
    rank, world = int(rank), int(world)
    tpr = 2
    m = swl.QwenCUDAModel(d, device=rank)
    m.ep_init(rank, world, bytes.fromhex(id_hex), tpr)
    V = m.config.vocab_size
    rng = np.random.default_rng(7 + rank)
    states = [m.new_state(64) for _ in range(tpr)]
    logits = m.step_batch([rng.integers(0, V, 3).tolist() for _ in range(tpr)], states)
    for _ in range(2):
        logits = m.step_batch([[int(np.argmax(l))] for l in logits], states)
    res = {"rank": rank}
    if rank == 1:
        # stop answering, but stay alive until rank 0 is through
        t0 = time.time()
        while not os.path.exists(os.path.join(flags, "done")) and time.time() - t0 < 120:
            time.sleep(0.1)
        res["waited_s"] = time.time() - t0
    else:
        t0 = time.time()
        codes = []
        for _ in range(2):
            try:
                m.step_batch([[int(np.argmax(l))] for l in logits], states)
                codes.append(0)
            except swl.SwiftletError as e:
                codes.append(e.code)
                res.setdefault("message", str(e))
        res["codes"] = codes
        res["elapsed_s"] = time.time() - t0
        open(os.path.join(flags, "done"), "w").close()
    for s in states:
        s.free()
    m.close()
    res["closed"] = True
    with open(out, "w") as f:
        json.dump(res, f)
    return 0


if __name__ == "__main__":
    sys.exit(main())
