"""One rank of the expert-parallel failure-path check (run by tests/test_gpu_ep.py).

Usage: python tests/ep_stall.py <model_dir> <rank> <world> <id_hex> <flag_dir> <store_port> <out_json>

Both ranks join the group with a liveness callback on a shared
torch.distributed TCPStore (a heartbeat per step, 5 s limit), prefill and run
two decode steps together. Then rank 1 stops taking part: it stays alive but
makes no further call until rank 0 has written `done` to flag_dir. Rank 0
makes a third decode step: its liveness check finds rank 1 missing, so the
library must refuse that step with SWL_ERR_CUDA before launching anything,
refuse the next one at once, and still close the model.
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
    d, rank, world, id_hex, flags, port, out = sys.argv[1:8]
    rank, world = int(rank), int(world)
    import datetime
    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", int(port), world, rank == 0, timeout=datetime.timedelta(seconds=60))
    tpr = 2
    m = swl.QwenCUDAModel(d, device=rank)
    m.ep_init(rank, world, bytes.fromhex(id_hex), tpr)
    m.ep_set_liveness(swl.ep_store_liveness(store, rank, world, timeout_s=5.0))
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
    if rank == 0:  # the store's host leaves last
        time.sleep(1.0)
    return 0


if __name__ == "__main__":
    sys.exit(main())
