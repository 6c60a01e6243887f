"""The expert-parallel MoE partition, restated on two gloo ranks on CPU.

The library splits a batched decode step's MoE block over ranks this way
(csrc/batch.cu k_broute / k_bcombine_ep, csrc/model.cu enqueue_batch,
csrc/ep_nccl.cpp): every rank all-gathers its tokens' MoE inputs and router
logits; routes all tokens with the softmax / top-k / renorm of
QwenCPUModel.swift:506-521; computes only the routed experts it owns,
[r * E / W, (r + 1) * E / W), for every token that picked one; adds, for its
own tokens only, the gated shared expert and the residual; and a sum
reduce-scatter hands each rank its own tokens' new residual rows.

Here each step is restated with numpy on dequantised weights of the tiny
baseline model and torch.distributed (gloo) collectives, and the result must
equal the oracle's single-rank MoE (QwenCPUModel.swift:500-569) plus the
residual for every token of every rank."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT, TINY_BASELINE

T_PER_RANK = 3


def owned_range(rank: int, world: int, experts: int) -> tuple[int, int]:
    """Experts rank `rank` computes (Model::ep_lo / ep_hi in csrc/model.cu)."""
    return rank * experts // world, (rank + 1) * experts // world


def route(logits: np.ndarray, k: int, norm_topk: bool):
    """Max-subtracted softmax, insertion top-k with ties to the lower id, and
    renormalisation (QwenCPUModel.swift:506-521)."""
    p = np.exp(logits - logits.max())
    p = p / p.sum()
    ids = []
    for e in range(len(p)):  # insertion: a later id enters only on a strictly larger value
        pos = len(ids)
        while pos > 0 and p[e] > p[ids[pos - 1]]:
            pos -= 1
        ids.insert(pos, e)
        del ids[k:]
    w = p[ids]
    if norm_topk:
        w = w / w.sum()
    return np.array(ids), w.astype(np.float32)


def silu(v):
    return v / (1.0 + np.exp(-v))


def _rank(rank: int, world: int, port: int, layer: int, q) -> None:
    import sys
    sys.path.insert(0, ROOT)
    import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cpu = oracle.OracleModel(TINY_BASELINE)
        D, E, K = cpu.D, cpu.E, cpu.K
        inter = cpu.cfg("moe_intermediate_size")
        sinter = cpu.cfg("shared_expert_intermediate_size")
        pre = f"model.layers.{layer}.mlp."
        deq = lambda mod, r0, r1, cols: cpu.dequant(pre + mod, r0, r1, cols)
        router = deq("gate", 0, E, D)
        sgate = deq("shared_expert_gate", 0, 1, D)
        # this rank's tokens: normalised MoE inputs and residual rows
        rng = np.random.default_rng(1000 + rank)
        x_own = rng.normal(0, 1, (T_PER_RANK, D)).astype(np.float32)
        h_own = rng.normal(0, 1, (T_PER_RANK, D)).astype(np.float32)
        logit_own = np.concatenate([x_own @ router.T, x_own @ sgate.T], axis=1).astype(np.float32)
        # (1) all-gather of every rank's inputs and router logits
        xs = [torch.zeros(T_PER_RANK, D) for _ in range(world)]
        ls = [torch.zeros(T_PER_RANK, E + 1) for _ in range(world)]
        dist.all_gather(xs, torch.from_numpy(x_own))
        dist.all_gather(ls, torch.from_numpy(logit_own))
        X = torch.cat(xs).numpy()
        LG = torch.cat(ls).numpy()
        N = world * T_PER_RANK
        lo, hi = owned_range(rank, world, E)
        own_lo, own_hi = rank * T_PER_RANK, (rank + 1) * T_PER_RANK
        # (2) routing of all N tokens; slots only for owned experts,
        # expert-major with tokens ascending (k_broute)
        picks = [route(LG[t, :E], K, bool(cpu.cfg("norm_topk_prob"))) for t in range(N)]
        slot_of = -np.ones((N, K), np.int64)
        slot_tok = []
        for e in range(lo, hi):
            for t in range(N):
                for j in range(K):
                    if picks[t][0][j] == e:
                        slot_of[t, j] = len(slot_tok)
                        slot_tok.append((t, e))
        # (3) owned experts' SwiGLU for the tokens in their slots
        y_slot = np.zeros((len(slot_tok), D), np.float32)
        for s, (t, e) in enumerate(slot_tok):
            g = deq("switch_mlp.gate_proj", e * inter, (e + 1) * inter, D)
            u = deq("switch_mlp.up_proj", e * inter, (e + 1) * inter, D)
            dn = deq("switch_mlp.down_proj", e * D, (e + 1) * D, inter)
            y_slot[s] = dn @ (silu(g @ X[t]) * (u @ X[t]))
        sg = deq("shared_expert.gate_proj", 0, sinter, D)
        su = deq("shared_expert.up_proj", 0, sinter, D)
        sd = deq("shared_expert.down_proj", 0, D, sinter)
        # (4) partial sums (k_bcombine_ep): this rank's picks of every token,
        # plus the shared expert and the residual of its own tokens
        part = np.zeros((N, D), np.float32)
        for t in range(N):
            for j in range(K):
                if slot_of[t, j] >= 0:
                    part[t] += picks[t][1][j] * y_slot[slot_of[t, j]]
            if own_lo <= t < own_hi:
                gate = 1.0 / (1.0 + np.exp(-LG[t, E]))
                part[t] += gate * (sd @ (silu(sg @ X[t]) * (su @ X[t]))) + h_own[t - own_lo]
        # (5) reduce-scatter: rank r receives the sum of rows [r*T, (r+1)*T)
        out = torch.zeros(T_PER_RANK, D)
        dist.reduce_scatter(out, [torch.from_numpy(part[r * T_PER_RANK:(r + 1) * T_PER_RANK]) for r in range(world)])
        # the oracle's single-rank MoE of the same tokens
        ref, ids, _, _ = cpu.moe_forward(x_own, layer)
        own_ids = [sorted(picks[t][0].tolist()) for t in range(own_lo, own_hi)]
        q.put((rank, out.numpy(), ref + h_own, own_ids, [sorted(r) for r in ids.tolist()], hi - lo))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layer", [0, 3])
def test_two_rank_partition_equals_single_rank_moe(layer):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, layer, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = {}
    for _ in ps:
        rank, out, ref, ids, ref_ids, owned = q.get(timeout=180)
        got[rank] = (out, ref, ids, ref_ids, owned)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sum(v[4] for v in got.values()) == 8  # the ranks' expert ranges cover E once
    for rank, (out, ref, ids, ref_ids, _) in got.items():
        assert ids == ref_ids, rank
        assert np.abs(out - ref).max() / (np.abs(ref).max() + 1e-6) < 1e-5, rank
