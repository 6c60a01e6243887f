#!/usr/bin/env python
"""Decode benchmark of the Qwen3.6-35B-A3B-shaped q4 model on B200.

Workload: 40 layers (3 gated-DeltaNet : 1 gated GQA),
hidden 2048, vocab 151936, 256 experts top-8 + 1 shared (intermediate 512),
every linear MLX-affine 4-bit group-64 with bf16 scales/biases, random-init
weights generated on the device from a seed (synthetic checkpoint), a
512-token seeded prompt, then greedy single-stream decode (B=1). One "step"
is one decoded token; `value` is tokens/s with the token feedback kept in
HBM, `e2e` is the same through the host API (swl_step: H2D token, D2H
logits, host argmax). Weights streamed per token (~1.7 GB) exceed the
126 MB L2, so no flush is needed between steps.

`--impl reference` times the reference's CPU algorithm (the C++ restatement
in oracle/) on the host cores on a bounded sample of the same workload.
With N > 1 ranks every rank runs an independent replica (batch-1 decode does
not shard); value = tokens of all ranks / max elapsed over ranks.

`--model 80b` runs BASELINE config 5 alone: 64 sequences of ragged seeded
prompts, then batched greedy decode. Under torchrun with `--ep` the 64
sequences are split over the ranks and the routed experts of every layer are
split by id (swl_ep_init: NCCL all-gather + reduce-scatter per layer), so the
total work is fixed ("scaling": "strong"); without it each rank runs its own
64 sequences as a replica.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "35B-A3B q4 decode tok/s (B=1; B=64 under batched)"
PROMPT_SEED = 4242
MODEL_SEED = 35


def model_dir(tmp: str, layers: int | None = None, model: str = "35b") -> str:
    from swiftlet_b200 import formats
    from swiftlet_b200.configs import NEXT_80B, Q35_35B, with_layers
    base = NEXT_80B if model == "80b" else Q35_35B
    cfg = with_layers(base, layers) if layers else base
    return formats.write_synthetic(os.path.join(tmp, f"synth-{model}"), cfg, seed=MODEL_SEED)


def algorithmic_bytes_per_token(cfg, ctx: float) -> dict:
    """Bytes one decoded token must move: every dense weight except the
    embedding table (one row), K routed + 1 shared expert per layer, the
    f32 delta state read + written, the conv ring, and the f32 KV cache."""
    D, L, V = cfg.hidden_size, cfg.num_hidden_layers, cfg.vocab_size

    def q4(out, inn, gs=64):
        return out * inn // 2 + out * (inn // gs) * 4

    nv, nk, dk, dv = cfg.linear_num_value_heads, cfg.linear_num_key_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
    key, val = nk * dk, nv * dv
    conv = 2 * key + val
    H, KVH, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    E, K, I, SI = cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
    expert = q4(I, D) * 2 + q4(D, I)
    shared = q4(SI, D) * 2 + q4(D, SI)
    n_delta = sum(1 for i in range(L) if cfg.is_linear_layer(i))
    n_attn = L - n_delta
    b = {
        "delta_proj": n_delta * (q4(conv, D) + q4(val, D) + 2 * q4(nv, D) + q4(D, val)),
        "attn_proj": n_attn * (q4(2 * H * hd, D) + 2 * q4(KVH * hd, D) + q4(D, H * hd)),
        "router": L * (q4(E, D) + q4(1, D)),
        "experts": L * (K * expert + shared),
        "delta_state": n_delta * 2 * nv * dv * dk * 4,
        "conv_ring": n_delta * cfg.linear_conv_kernel_dim * conv * 4,
        "kv": n_attn * (ctx * 2 * KVH * hd * 4),
        "lm_head": q4(V, D),
        "embed_row": D // 2 + (D // 64) * 4,
    }
    b["total"] = sum(b.values())
    b["expert_blob"] = expert
    return b


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a region."""

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p)), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def profile_traffic() -> dict:
    p = os.path.join(ROOT, "profiles", "traffic.json")
    return json.load(open(p)) if os.path.exists(p) else {}


def cpu_decode_sample(mdir: str, n_steps: int, warm: int = 1) -> dict:
    """The oracle (C++ restatement of QwenCPUModel) decoding on all host threads."""
    import numpy as np
    import oracle
    oracle.set_threads(os.cpu_count() or 1)
    cpu = oracle.OracleModel(mdir, retain_all_layers=True)
    st = oracle.DecodeState()
    logits = cpu.step([7], st)
    for _ in range(warm):
        logits = cpu.step([int(np.argmax(logits))], st)
    t0 = time.perf_counter()
    for _ in range(n_steps):
        logits = cpu.step([int(np.argmax(logits))], st)
    dt = time.perf_counter() - t0
    return {"value": n_steps / dt, "unit": "tok/s", "cores": oracle.max_threads(), "kind": "port",
            "sample": f"{n_steps} greedy decode steps after a 1-token prompt and {warm} warm-up step(s), same 35B-shaped "
                      "synthetic model; dense weights retained as f32, experts dequantised per call "
                      "(QwenCPUModel with retainAllLayers=true)",
            "seconds": dt}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps = min(args.steps, 6)
    warm = min(args.warmup, 1)
    with tempfile.TemporaryDirectory() as tmp:
        cb = cpu_decode_sample(model_dir(tmp), steps, warm)
    line = {"metric": METRIC, "value": cb["value"], "unit": "tok/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warm, "requested_steps": args.steps, "ms_per_step": 1000.0 / cb["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "qwen3.6-35b-a3b shape, q4 g64 bf16, B=1 greedy decode (CPU sample)",
                       "global_batch": 1, "parallelism": "none (host cores)"},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def max_over_ranks(values, dist, device) -> list:
    """Elapsed times of this rank -> their maximum over all ranks (every rank
    runs the same collective: a replica run is as slow as its slowest GPU)."""
    import torch
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def replica_rate(world: int, units_per_rank: float, max_ms: float) -> float:
    """Whole-job throughput of `world` replicas: all units over the slowest
    rank's time."""
    return world * units_per_rank / (max_ms / 1000.0)


def expected_unique_experts(E: int, K: int, B: int) -> float:
    """Expected distinct experts per layer when B tokens each pick K of E
    uniformly (the synthetic router's logits are i.i.d.)."""
    return E * (1.0 - (1.0 - K / E) ** B)


def batched_decode(model, cfg, stream, args, rank, local, dist) -> dict:
    """B sequences, each with its own seeded prompt of args.batch_prompt
    tokens (run through the batched rounds), then greedy decode with the
    tokens fed back on the device; e2e through swl_step_batch (H2D tokens,
    D2H logits of every sequence, host argmax)."""
    import numpy as np
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    ep = bool(args.ep) and world > 1
    B = args.batch // world if ep else args.batch
    if ep:
        # expert parallelism: args.batch sequences in all, B per rank; every
        # decode step routes all ranks' tokens over the experts split by id
        import swiftlet_b200 as swl
        model.ep_init(rank, world, swl.ep_unique_id_broadcast(rank), B)
    steps, e2e_steps = args.batch_steps, min(args.batch_steps, 8)
    rng = np.random.default_rng(PROMPT_SEED + 1000 + rank)
    # prompt lengths: all args.batch_prompt, or uniform in [batch_prompt, batch_prompt_max] (ragged)
    hi = max(args.batch_prompt, args.batch_prompt_max or 0)
    lens = rng.integers(args.batch_prompt, hi + 1, B) if hi > args.batch_prompt else np.full(B, args.batch_prompt)
    extra = args.warmup + steps + e2e_steps + 8
    states = [model.new_state(max_ctx=int(n) + extra) for n in lens]
    prompts = [rng.integers(0, cfg.vocab_size, int(n)).astype(np.int32) for n in lens]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    ev[0].record(stream)
    logits = model.step_batch(prompts, states)
    ev[1].record(stream)
    torch.cuda.synchronize()
    prefill_ms = ev[0].elapsed_time(ev[1])
    tok = torch.tensor(np.argmax(logits, axis=1).astype(np.int32), device=f"cuda:{local}")
    for _ in range(args.warmup):
        model.step_batch_device(states, tok.data_ptr(), 0, tok.data_ptr())
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ev[2].record(stream)
        for _ in range(steps):
            model.step_batch_device(states, tok.data_ptr(), 0, tok.data_ptr())
        ev[3].record(stream)
        torch.cuda.synchronize()
    ms = ev[2].elapsed_time(ev[3])
    host = tok.cpu().numpy().tolist()
    ev[4].record(stream)
    for _ in range(e2e_steps):
        lg = model.step_batch([[t] for t in host], states)
        host = np.argmax(lg, axis=1).tolist()
    ev[5].record(stream)
    torch.cuda.synchronize()
    e2e_ms = ev[4].elapsed_time(ev[5])
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], dist, f"cuda:{local}")
    for s in states:
        s.free()
    bt = algorithmic_bytes_per_token(cfg, float(np.mean(lens)) + args.warmup + steps / 2)
    L = cfg.num_hidden_layers
    # distinct routed experts this rank reads per layer: of all E for its own
    # B tokens, or of its E / world for every rank's tokens
    uniq = (expected_unique_experts(cfg.num_experts, cfg.num_experts_per_tok, B * world) / world if ep else
            expected_unique_experts(cfg.num_experts, cfg.num_experts_per_tok, B))
    per_seq = bt["delta_state"] + bt["conv_ring"] + bt["kv"] + bt["embed_row"]
    dense = bt["total"] - bt["experts"] - per_seq
    step_bytes = dense + L * (uniq + 1) * bt["expert_blob"] + B * per_seq
    peaks, peak_kind = measured_peaks()
    hbm = float(peaks["hbm_gbs"])
    step_s = ms / steps / 1000.0
    return {
        "B": B, "value": replica_rate(world, B * steps, ms), "unit": "tok/s", "steps": steps,
        "expert_parallel": {"world": world, "sequences_per_rank": B,
                            "collectives_per_layer": "NCCL all-gather (digits, router logits) + reduce-scatter"}
        if ep else None,
        "ms_per_step": ms / steps, "prompt": args.batch_prompt if hi == args.batch_prompt else [args.batch_prompt, hi],
        "prefill": {"tokens": int(lens.sum()), "ms": prefill_ms,
                    "tok_s": float(lens.sum()) / (prefill_ms / 1000.0),
                    "mode": "packed launches of up to 64 tokens, an equal share per sequence"},
        "step_roofline": {"bound": "hbm", "bytes_per_step": step_bytes, "achieved": step_bytes / step_s / 1e9,
                          "peak": hbm, "unit": "GB/s", "frac": step_bytes / step_s / 1e9 / hbm,
                          "peak_kind": peak_kind,
                          "bytes": "dense weights once + (expected distinct routed experts %.1f + shared) blobs per "
                                   "layer + per-sequence delta state r/w, conv ring and f32 KV" % uniq},
        "e2e": {"value": replica_rate(world, B * e2e_steps, e2e_ms), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B * cfg.vocab_size},
        "gpu_launches_per_step": 3 + 11 * L + 3,
        "clocks": clk.summary(),
    }


def run_ours(args) -> None:
    import numpy as np
    import torch
    import swiftlet_b200 as swl

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    tmp = tempfile.mkdtemp()
    mdir = model_dir(tmp, args.layers, args.model)
    model = swl.QwenCUDAModel(mdir, device=local)
    cfg = model.config
    stream = torch.cuda.Stream()
    model.set_stream(stream.cuda_stream)
    if args.batch_only or args.model == "80b":
        # the batched leg alone: profiling, or the 80B-shaped ragged batch
        # (replicas per GPU, or with --ep the routed
        # experts split over the GPUs)
        res = batched_decode(model, cfg, stream, args, rank, local, dist)
        model.close()
        if rank == 0:
            line = {"metric": METRIC, "batched": res, "profiling_only": True}
            if args.model == "80b":
                ep = bool(args.ep) and world > 1
                line = {"metric": "80B-A3B q4 ragged batched decode tok/s (B=%d %s)"
                                  % (args.batch, "over all GPUs, expert-parallel" if ep else "per GPU"),
                        "value": res["value"],
                        "unit": "tok/s", "n_gpus": world, "steps": res["steps"], "warmup": args.warmup,
                        "ms_per_step": res["ms_per_step"], "higher_is_better": True,
                        "scaling": "strong" if ep else "weak",
                        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                        "config": {"workload": "qwen3-next-80b-a3b shape (48 layers, 512 experts top-10 + shared), q4 "
                                               "g64, %d sequences with seeded prompts of ragged length %s"
                                               % (args.batch, "split over the GPUs" if ep else "per GPU"),
                                   "parallelism": ("ep%d (routed experts by id, sequences data-parallel)" % world)
                                   if ep else "replica x%d" % world},
                        "batched": res}
            print(json.dumps(line), flush=True)
        if dist:
            dist.destroy_process_group()
        return
    rng = np.random.default_rng(PROMPT_SEED + rank)
    prompt = rng.integers(0, cfg.vocab_size, args.prompt).astype(np.int32)
    e2e_steps = min(args.steps, 32)
    st = model.new_state(max_ctx=args.prompt + args.warmup + args.steps + e2e_steps + 8)

    # prefill (reported separately)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    ev[0].record(stream)
    logits = model.step(prompt, st)
    ev[1].record(stream)
    torch.cuda.synchronize()
    prefill_ms = ev[0].elapsed_time(ev[1])

    a = torch.tensor([int(np.argmax(logits))], dtype=torch.int32, device=f"cuda:{local}")
    b = torch.empty_like(a)
    bufs = [a, b]

    def dev_step(i):
        src, dst = bufs[i & 1], bufs[(i + 1) & 1]
        model.step_device(src.data_ptr(), 1, st, 0, dst.data_ptr())

    i = 0
    for _ in range(args.warmup):
        dev_step(i); i += 1
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ev[2].record(stream)
        for _ in range(args.steps):
            dev_step(i); i += 1
        ev[3].record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = ev[2].elapsed_time(ev[3])

    # end to end through the public host API
    tok = int(bufs[i & 1].item())
    ev[4].record(stream)
    for _ in range(e2e_steps):
        lg = model.step([tok], st)
        tok = int(np.argmax(lg))
    ev[5].record(stream)
    torch.cuda.synchronize()
    e2e_ms = ev[4].elapsed_time(ev[5])

    # batched decode: args.batch sequences advancing together through the
    # batched kernels (one weight stream per step for all of them)
    bres = None
    if args.batch > 1:
        bres = batched_decode(model, cfg, stream, args, rank, local, dist)

    # roofline of the dominant kernels: the fused expert GEMV pair, swept over all layers
    sweep_iters = 4
    sweep_ms, bytes_layer, sweep_launches = model.bench_expert_sweep(sweep_iters)
    ms, e2e_ms, sweep_ms = max_over_ranks([ms, e2e_ms, sweep_ms], dist, f"cuda:{local}")
    if rank != 0:
        model.close()
        if dist:
            dist.destroy_process_group()
        return

    peaks, peak_kind = measured_peaks()
    hbm = float(peaks["hbm_gbs"])
    ctx_mean = args.prompt + args.warmup + args.steps / 2
    bt = algorithmic_bytes_per_token(cfg, ctx_mean)
    value = replica_rate(world, args.steps, ms)
    per_launch_s = sweep_ms / 1000.0 / (sweep_iters * cfg.num_hidden_layers)
    achieved = bytes_layer / per_launch_s / 1e9
    traffic = profile_traffic().get("moe_expert_pair_bytes_per_layer")
    launches_per_token = 2 + 6 * cfg.num_hidden_layers
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "weights": "u4 MLX-affine g64, bf16 scales/biases", "data": "synthetic",
        "config": {"workload": "qwen3.6-35b-a3b shape (%d layers, hidden 2048, 256 experts top-8 + shared, "
                               "vocab 151936), q4 g64, B=1 greedy decode after a %d-token prompt"
                               % (cfg.num_hidden_layers, args.prompt),
                   "model": "Q35_35B synthetic seed %d" % MODEL_SEED, "global_batch": world, "seq_len": args.prompt,
                   "parallelism": "replica x%d" % world if world > 1 else "single GPU",
                   "l2": "no flush: each token streams ~1.7 GB of weights, far above the 126 MB L2"},
        "prefill": {"tokens": args.prompt, "ms": prefill_ms, "tok_s": args.prompt / (prefill_ms / 1000.0),
                    "mode": "chunked: launches of up to 64 prompt tokens through the batched kernels"},
        "step_roofline": {"bound": "hbm", "bytes_per_token": bt["total"], "achieved": bt["total"] * value / world / 1e9,
                          "peak": hbm, "unit": "GB/s", "frac": bt["total"] * value / world / 1e9 / hbm,
                          "peak_kind": peak_kind},
        "roofline": {"kernel": "k_igateup + k_idown (8 routed + 1 shared expert, one layer)", "bound": "hbm",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "bytes_per_launch_pair": bytes_layer, "avg_pair_us": per_launch_s * 1e6,
                     "traffic": traffic, "peak_kind": peak_kind},
        "e2e": {"value": replica_rate(world, e2e_steps, e2e_ms), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * cfg.vocab_size},
        "gpu_launches": launches_per_token * args.steps,
        "clocks": clk.summary(),
    }
    if bres is not None:
        line["batched"] = bres
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_decode_sample(mdir, 2, 1)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    model.close()
    print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=64, help="sequences of the batched-decode leg (<= 1: skip it)")
    ap.add_argument("--batch-prompt", type=int, default=128)
    ap.add_argument("--batch-steps", type=int, default=32)
    ap.add_argument("--batch-prompt-max", type=int, default=None,
                    help="ragged prompts: lengths uniform in [--batch-prompt, this]")
    ap.add_argument("--model", default="35b", choices=["35b", "80b"],
                    help="80b: the Qwen3-Next-80B-shaped batched leg alone (BASELINE config 5 per GPU)")
    ap.add_argument("--ep", action="store_true",
                    help="batched leg with expert parallelism over the ranks (--batch sequences in all)")
    ap.add_argument("--batch-only", action="store_true",
                    help="profiling only: run the batched leg alone and print its numbers")
    ap.add_argument("--layers", type=int, default=None,
                    help="profiling only: same shapes with fewer layers (keeps ncu captures to a few GB)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
