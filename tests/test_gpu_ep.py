"""Expert parallelism (swl_ep_init): the routed experts of every layer split
by id over two GPUs, NCCL all-gather of the tokens' quantised MoE inputs and
router logits, reduce-scatter of the partial sums; decode steps replayed as
CUDA graphs that hold the NCCL calls, and launched directly
(SWL_EP_NO_GRAPH=1). Each rank runs as its own
process (tests/ep_rank.py) and checks its sequences' logits against the same
checkpoint stepped by the single-GPU batched path, which the other batched
tests pin to the CPU oracle: 2e-2 max-abs, 1e-3 relative-L2, greedy ids
identical."""
import json
import os
import subprocess
import sys

import pytest

import swiftlet_b200 as swl
from conftest import ROOT, TINY_BASELINE
from swiftlet_b200 import formats
from swiftlet_b200.configs import NEXT_80B, with_layers

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("shape,graph", [("tiny", True), ("80b", True), ("80b", False)])
def test_expert_parallel_matches_single_gpu(shape, graph, tmp_path):
    world = 2
    if _gpus() < world:
        pytest.skip("expert parallelism needs two GPUs")
    d = TINY_BASELINE if shape == "tiny" else formats.write_synthetic(
        str(tmp_path / "80b"), with_layers(NEXT_80B, 4), seed=99)
    ep_id = swl.ep_unique_id().hex()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SWL_EP_NO_GRAPH="0" if graph else "1")
    outs = [str(tmp_path / f"rank{r}.json") for r in range(world)]
    procs = [subprocess.Popen([sys.executable, os.path.join(ROOT, "tests", "ep_rank.py"), d, str(r), str(world),
                               ep_id, "4", "6", outs[r]], env=env, cwd=ROOT) for r in range(world)]
    rcs = []
    try:
        for p in procs:
            rcs.append(p.wait(timeout=300))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
                p.wait()
    res = [json.load(open(o)) for o in outs if os.path.exists(o)]
    assert rcs == [0] * world, (rcs, res)
    assert [r["expert_lo"] for r in res] == [0, res[0]["expert_hi"]]
    for r in res:
        assert r["ep_on"] and r["positions"] and r["same_greedy"], r


def test_a_peer_that_stops_answering_is_reported_not_waited_for(tmp_path):
    """The failure path: rank 1 stops making calls after two steps (alive,
    nothing of it in flight); rank 0's liveness callback (a heartbeat on a
    TCPStore) finds it missing before the next exchange, so rank 0's calls
    fail with SWL_ERR_CUDA without launching anything, and both ranks still
    close their models (NVLS off, plain peer transfers)."""
    import socket
    world = 2
    if _gpus() < world:
        pytest.skip("expert parallelism needs two GPUs")
    with socket.socket() as s_:
        s_.bind(("127.0.0.1", 0))
        port = s_.getsockname()[1]
    ep_id = swl.ep_unique_id().hex()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    outs = [str(tmp_path / f"rank{r}.json") for r in range(world)]
    procs = [subprocess.Popen([sys.executable, os.path.join(ROOT, "tests", "ep_stall.py"), TINY_BASELINE, str(r),
                               str(world), ep_id, str(tmp_path), str(port), outs[r]], env=env, cwd=ROOT)
             for r in range(world)]
    rcs = []
    try:
        for p in procs:
            rcs.append(p.wait(timeout=240))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
                p.wait()
    res = {r["rank"]: r for r in (json.load(open(o)) for o in outs if os.path.exists(o))}
    assert rcs == [0] * world, (rcs, res)
    r0 = res[0]
    assert r0["codes"] == [swl.SWL_ERR_CUDA, swl.SWL_ERR_CUDA], r0
    assert "peer left or stopped" in r0["message"]
    assert r0["elapsed_s"] < 30, r0
    assert r0["closed"] and res[1]["closed"]
