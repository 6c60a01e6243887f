#!/usr/bin/env python
"""Decode benchmark of the Qwen3.6-35B-A3B / Qwen3-Next-80B-A3B-shaped q4 models on B200.

One GPU (the default): the line's `value` is single-stream greedy decode
(B=1) of the 35B shape: 40 layers (3 gated-DeltaNet : 1 gated GQA), hidden
2048, vocab 151936, 256 experts top-8 + 1 shared (intermediate 512), every
linear MLX-affine 4-bit group-64 with bf16 scales/biases, random-init
weights generated on the device from a seed (synthetic checkpoint), a
512-token seeded prompt. One "step" is one decoded token; `value` is tokens/s
with the token feedback kept in HBM, `e2e` is the same through the host API
(swl_step: H2D token, D2H logits, host argmax). Weights streamed per token
(~1.7 GB) exceed the 126 MB L2, so no flush is needed between steps. The same
line carries the other measurements of the metric:
  * `b64`: 64 sequences of the 35B shape decoding together (batched kernels);
  * `expert_gemv`: the expert GEMV/GEMM sweeps over all 40 layers at B = 1, 8
    and 64, for 4-bit and 8-bit experts, against their algorithmic bytes;
  * `deltanet`: the DeltaNet decode step of the 80B shape at B = 1 and 64;
  * `batched`: the 80B shape with 64 sequences of seeded ragged prompts
    (lengths uniform in [128, 8192]), batched greedy decode, world 1.

Several GPUs (torchrun, one rank per GPU): the line is that last workload
split over the ranks by expert parallelism: the 64 sequences (the same
prompt lengths whatever the rank count) are divided among the ranks and the
routed experts of every layer are split by id (swl_ep_init: NCCL all-gather
+ reduce-scatter per MoE layer); `value` is all ranks' tokens over the
slowest rank's time and `batched.expert_parallel.world` is the rank count,
so `batched.value` compares across rank counts ("scaling": "strong").

`--impl reference` times the reference's CPU algorithm (the C++ restatement
in oracle/) on the host cores on a bounded sample of the same workload.
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


def model_dir(tmp: str, layers: int | None = None, model: str = "35b", bits: int = 4) -> str:
    from swiftlet_b200 import formats
    from swiftlet_b200.configs import NEXT_80B, Q35_35B, with_layers
    base = NEXT_80B if model == "80b" else Q35_35B
    cfg = with_layers(base, layers) if layers else base
    return formats.write_synthetic(os.path.join(tmp, f"synth-{model}-q{bits}"), cfg, seed=MODEL_SEED, bits=bits)


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


def cpu_decode_sample(mdir: str, n_steps: int, warm: int = 1, label: str = "35B") -> dict:
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
            "sample": f"{n_steps} greedy decode steps of one sequence after a 1-token prompt and {warm} warm-up "
                      f"step(s), same {label}-shaped synthetic model; dense weights retained as f32, experts "
                      "dequantised per call (QwenCPUModel with retainAllLayers=true; the reference steps "
                      "sequences one at a time, so this is also its batched rate)",
            "seconds": dt}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return
    multi = world > 1
    steps = min(args.steps, 4 if multi else 6)
    warm = min(args.warmup, 1)
    with tempfile.TemporaryDirectory() as tmp:
        cb = cpu_decode_sample(model_dir(tmp, None, "80b" if multi else "35b"), steps, warm,
                               "80B" if multi else "35B")
    if multi:
        metric = "80B-A3B q4 ragged batched decode tok/s (%d sequences over all GPUs, expert-parallel)" % args.batch
        config = {"workload": "qwen3-next-80b-a3b shape, q4 g64 bf16, batched decode (CPU sample: the reference "
                              "steps one sequence at a time)", "parallelism": "none (host cores)"}
    else:
        metric = METRIC
        config = {"workload": "qwen3.6-35b-a3b shape, q4 g64 bf16, B=1 greedy decode (CPU sample)",
                  "global_batch": 1, "parallelism": "none (host cores)"}
    line = {"metric": metric, "value": cb["value"], "unit": "tok/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warm, "requested_steps": args.steps, "ms_per_step": 1000.0 / cb["value"],
            "higher_is_better": True, "scaling": "strong" if multi else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference", "config": config,
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


def prompt_lengths(args) -> "np.ndarray":
    """The batched workload's prompt lengths: all args.batch_prompt, or seeded
    uniform in [batch_prompt, batch_prompt_max]; the same list whatever the
    number of ranks (rank r of N takes sequences [r * B / N, (r + 1) * B / N))."""
    import numpy as np
    hi = max(args.batch_prompt, args.batch_prompt_max or 0)
    if hi == args.batch_prompt:
        return np.full(args.batch, args.batch_prompt)
    return np.random.default_rng(PROMPT_SEED + 1000).integers(args.batch_prompt, hi + 1, args.batch)


def batched_decode(model, cfg, stream, args, rank, local, dist, ep: bool, steps: int, deltanet: bool = False) -> dict:
    """args.batch sequences with seeded prompts (run through packed batched
    launches), then greedy decode with the tokens fed back on the device; e2e
    through swl_step_batch (H2D tokens, D2H logits of every sequence, host
    argmax). With `ep` the sequences are split over the ranks and the routed
    experts by id (every decode step routes all ranks' tokens)."""
    import numpy as np
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    ep = ep and world > 1
    B = args.batch // world if ep else args.batch
    if ep:
        import swiftlet_b200 as swl
        model.ep_init(rank, world, swl.ep_unique_id_broadcast(rank), B)
    e2e_steps = min(steps, 8)
    all_lens = prompt_lengths(args)
    first = rank * B if ep else 0
    lens = all_lens[first:first + B]
    extra = args.warmup + steps + e2e_steps + 8
    states = [model.new_state(max_ctx=int(n) + extra) for n in lens]
    prompts = [np.random.default_rng(PROMPT_SEED + 2000 + first + i).integers(0, cfg.vocab_size, int(n)).astype(np.int32)
               for i, n in enumerate(lens)]
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
    if ep:
        model.ep_timing(reset=True)
    with ClockSampler(local) as clk:
        ev[2].record(stream)
        for _ in range(steps):
            model.step_batch_device(states, tok.data_ptr(), 0, tok.data_ptr())
        ev[3].record(stream)
        torch.cuda.synchronize()
    ms = ev[2].elapsed_time(ev[3])
    # with SWL_EP_TIMING=1 and SWL_EP_NO_GRAPH=1: this rank's collective time
    # (CUDA events around each exchange, waits for peers included)
    ep_t = model.ep_timing() if ep else None
    host = tok.cpu().numpy().tolist()
    ev[4].record(stream)
    for _ in range(e2e_steps):
        lg = model.step_batch([[t] for t in host], states)
        host = np.argmax(lg, axis=1).tolist()
    ev[5].record(stream)
    torch.cuda.synchronize()
    e2e_ms = ev[4].elapsed_time(ev[5])
    ms, e2e_ms, prefill_ms = max_over_ranks([ms, e2e_ms, prefill_ms], dist, f"cuda:{local}")
    delta = deltanet_sweeps(model, cfg, states) if deltanet else None
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
    hi = int(all_lens.max())
    res = {
        "B": B * (world if ep else 1), "sequences_per_rank": B, "value": replica_rate(world if ep else 1, B * steps, ms),
        "unit": "tok/s", "steps": steps, "warmup": args.warmup,
        "expert_parallel": {"world": world if ep else 1, "sequences_per_rank": B,
                            "experts_per_rank": cfg.num_experts // (world if ep else 1),
                            "collectives_per_layer": "NCCL all-gather (digits, router logits) + reduce-scatter"
                            if ep else "none (one rank holds every expert)"},
        "ms_per_step": ms / steps,
        "prompt": args.batch_prompt if hi == args.batch_prompt else [args.batch_prompt, args.batch_prompt_max],
        "prefill": {"tokens": int(all_lens.sum()) if ep else int(lens.sum()), "ms": prefill_ms,
                    "tok_s": float(all_lens.sum() if ep else lens.sum()) / (prefill_ms / 1000.0),
                    "mode": "packed launches of up to 64 tokens, an equal share per sequence; each rank prefills "
                            "its own sequences"},
        "step_roofline": {"bound": "hbm", "bytes_per_step_per_rank": step_bytes,
                          "achieved": step_bytes / step_s / 1e9, "peak": hbm, "unit": "GB/s",
                          "frac": step_bytes / step_s / 1e9 / hbm, "peak_kind": peak_kind,
                          "bytes": "dense weights once + (expected distinct routed experts %.1f + shared) blobs per "
                                   "layer + per-sequence delta state r/w, conv ring and f32 KV" % uniq},
        "e2e": {"value": replica_rate(world if ep else 1, B * e2e_steps, e2e_ms), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B * cfg.vocab_size},
        "gpu_launches_per_step": 3 + 11 * L + 3,
        "clocks": clk.summary(),
    }
    if ep_t:
        coll = max_over_ranks([ep_t["collective_ms"] / max(1, ep_t["steps"])], dist, f"cuda:{local}")[0]
        res["ep_timing"] = {"collective_ms_per_step_max_over_ranks": coll,
                            "collectives_per_step": ep_t["collectives"] / max(1, ep_t["steps"]),
                            "rank0_step_ms": ep_t["step_ms"] / max(1, ep_t["steps"]),
                            "mode": "SWL_EP_NO_GRAPH=1 (steps launched directly, CUDA events around each exchange)"}
    if delta:
        res["deltanet"] = delta
    return res


def deltanet_sweeps(model, cfg, states) -> dict:
    """DeltaNet decode step of every DeltaNet layer of this model's shape:
    B = len(states) from the last batched step,
    and B = 1 on one state after one swl_step; bytes are the f32 state read
    and written plus the small per-token vectors."""
    import numpy as np
    peaks, peak_kind = measured_peaks()
    hbm = float(peaks["hbm_gbs"])
    out = {}
    iters = 8
    ms, byts, launches = model.bench_delta_sweep(len(states), iters)
    per_launch = ms / launches
    out["B%d" % len(states)] = {"us_per_layer": per_launch * 1000.0, "bytes_per_layer": byts * iters / launches,
                                "achieved": byts * iters / (ms / 1000.0) / 1e9, "peak": hbm,
                                "frac": byts * iters / (ms / 1000.0) / 1e9 / hbm, "unit": "GB/s",
                                "peak_kind": peak_kind}
    st = model.new_state(max_ctx=64)
    model.step([7, 8], st)
    model.step([9], st)
    ms, byts, launches = model.bench_delta_sweep(1, iters * 8)
    per_launch = ms / launches
    out["B1"] = {"us_per_layer": per_launch * 1000.0, "bytes_per_layer": byts * iters * 8 / launches,
                 "achieved": byts * iters * 8 / (ms / 1000.0) / 1e9, "peak": hbm,
                 "frac": byts * iters * 8 / (ms / 1000.0) / 1e9 / hbm, "unit": "GB/s", "peak_kind": peak_kind}
    st.free()
    # chunked-parallel prompt recurrence: one sequence of 4096 tokens
    import swiftlet_b200 as swl
    T = 4096
    ms, fl = swl.bench_gated_delta(T, cfg.linear_num_key_heads, cfg.linear_num_value_heads,
                                   cfg.linear_key_head_dim, cfg.linear_value_head_dim, 10)
    tf = fl / (ms / 1000.0) / 1e12
    out["prefill_4096"] = {"us_per_layer": ms * 100.0, "tflops": tf,
                           "tok_s_per_layer": T * 10 / (ms / 1000.0),
                           "kernel": "k_delta_wy (64-token chunks, f32 CUDA cores)",
                           "of_bf16_peak": tf / (float(peaks["bf16_tflops"])),
                           "flops": "per chunk and value head 2 x (2 C^2 dk + 2 C dk dv + 2 C^2 dv + C dk dv), C = 64"}
    out["note"] = ("graph of the decode recurrence (conv, norms, gating, delta rule) over all %d DeltaNet layers, "
                   "timed with CUDA events; state [%d, %d, %d] f32 per sequence and layer"
                   % (sum(1 for i in range(cfg.num_hidden_layers) if cfg.is_linear_layer(i)),
                      cfg.linear_num_value_heads, cfg.linear_value_head_dim, cfg.linear_key_head_dim))
    return out


def expert_gemv_leg(tmp, local, bits: int, stream, model=None) -> dict:
    """Expert GEMV/GEMM sweeps over all 40 layers of the 35B shape (distinct
    weights per layer, so nothing stays in L2): B = 1 through the single-token
    expert kernels, B = 8 and 64 through the batched grouped GEMMs; bytes are
    the distinct routed experts the routing picked plus the shared expert (and
    router for the batched block)."""
    import numpy as np
    import swiftlet_b200 as swl
    own = model is None
    if own:
        model = swl.QwenCUDAModel(model_dir(tmp, None, "35b", bits), device=local)
        model.set_stream(stream.cuda_stream)
    cfg = model.config
    peaks, peak_kind = measured_peaks()
    hbm = float(peaks["hbm_gbs"])
    out = {}
    st = model.new_state(max_ctx=64)
    model.step([11, 12, 13], st)
    model.step([14], st)
    iters = 4
    ms, bytes_layer, _ = model.bench_expert_sweep(iters)
    per_s = ms / 1000.0 / (iters * cfg.num_hidden_layers)
    out["B1"] = {"achieved": bytes_layer / per_s / 1e9, "peak": hbm, "frac": bytes_layer / per_s / 1e9 / hbm,
                 "unit": "GB/s", "us_per_layer": per_s * 1e6, "distinct_experts_per_layer": cfg.num_experts_per_tok + 1,
                 "kernels": "k_igateup + k_idown (integer tensor-core GEMV)"}
    st.free()
    rng = np.random.default_rng(PROMPT_SEED + 77)
    for B in (8, 64):
        states = [model.new_state(max_ctx=16) for _ in range(B)]
        model.step_batch([[int(t)] for t in rng.integers(0, cfg.vocab_size, B)], states)
        model.step_batch([[int(t)] for t in rng.integers(0, cfg.vocab_size, B)], states)
        ms, byts, uniq, _ = model.bench_moe_sweep(B, iters)
        sec = ms / 1000.0 / iters
        out["B%d" % B] = {"achieved": byts / sec / 1e9, "peak": hbm, "frac": byts / sec / 1e9 / hbm, "unit": "GB/s",
                          "us_per_layer": sec * 1e6 / cfg.num_hidden_layers,
                          "distinct_experts_per_layer": uniq / cfg.num_hidden_layers + 1,
                          "kernels": "k_broute + k_bgemm gate/up and down + k_bcombine (grouped GEMMs)"}
        for s in states:
            s.free()
    if own:
        model.close()
    out["weights"] = "q%d g64, bf16 scales/biases; expert blob %d B" % (bits, 1769472 if bits == 4 else 3342336)
    return out


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
    stream = torch.cuda.Stream()
    if world > 1 or args.model == "80b" or args.batch_only:
        # the 80B-shaped ragged batch (expert-parallel over the ranks), or
        # the batched leg alone (profiling)
        model = swl.QwenCUDAModel(model_dir(tmp, args.layers, args.model if args.batch_only else "80b"), device=local)
        model.set_stream(stream.cuda_stream)
        cfg = model.config
        res = batched_decode(model, cfg, stream, args, rank, local, dist, ep=world > 1, steps=args.steps)
        model.close()
        if rank == 0:
            line = {"metric": "80B-A3B q4 ragged batched decode tok/s (%d sequences over all GPUs, expert-parallel)"
                              % args.batch,
                    "value": res["value"], "unit": "tok/s", "n_gpus": world, "steps": res["steps"],
                    "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
                    "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                    "config": {"workload": "qwen3-next-80b-a3b shape (48 layers, 512 experts top-10 + shared), q4 "
                                           "g64, %d sequences with seeded prompts of ragged length, split over the "
                                           "GPUs" % args.batch,
                               "parallelism": "ep%d (routed experts by id, sequences data-parallel)" % world,
                               "l2": "no flush: each step streams tens of GB of weights, state and KV"},
                    "e2e": res["e2e"], "gpu_launches": res["gpu_launches_per_step"] * res["steps"],
                    "clocks": res["clocks"], "batched": res}
            if args.batch_only:
                line["profiling_only"] = True
            print(json.dumps(line), flush=True)
        if dist:
            dist.destroy_process_group()
        return
    mdir = model_dir(tmp, args.layers, "35b")
    model = swl.QwenCUDAModel(mdir, device=local)
    cfg = model.config
    model.set_stream(stream.cuda_stream)
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
    with ClockSampler(local) as clk:
        ev[2].record(stream)
        for _ in range(args.steps):
            dev_step(i); i += 1
        ev[3].record(stream)
        torch.cuda.synchronize()
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

    # roofline of the dominant kernels: the fused expert GEMV pair, swept over all layers
    sweep_iters = 4
    sweep_ms, bytes_layer, sweep_launches = model.bench_expert_sweep(sweep_iters)

    # 64 sequences of the 35B shape advancing together (one weight stream per step)
    b64 = None
    if args.batch > 1:
        b64_args = argparse.Namespace(**vars(args))
        b64_args.batch_prompt, b64_args.batch_prompt_max = 128, None
        b64 = batched_decode(model, cfg, stream, b64_args, rank, local, None, ep=False, steps=args.batch_steps)
    gemv = {"q4": expert_gemv_leg(tmp, local, 4, stream, model)} if not args.no_gemv else None
    model.close()
    if gemv is not None:
        gemv["q8"] = expert_gemv_leg(tmp, local, 8, stream)

    peaks, peak_kind = measured_peaks()
    hbm = float(peaks["hbm_gbs"])
    ctx_mean = args.prompt + args.warmup + args.steps / 2
    bt = algorithmic_bytes_per_token(cfg, ctx_mean)
    value = args.steps / (ms / 1000.0)
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
                   "model": "Q35_35B synthetic seed %d" % MODEL_SEED, "global_batch": 1, "seq_len": args.prompt,
                   "parallelism": "single GPU",
                   "l2": "no flush: each token streams ~1.7 GB of weights, far above the 126 MB L2"},
        "prefill": {"tokens": args.prompt, "ms": prefill_ms, "tok_s": args.prompt / (prefill_ms / 1000.0),
                    "mode": "chunked: launches of up to 64 prompt tokens through the batched kernels"},
        "step_roofline": {"bound": "hbm", "bytes_per_token": bt["total"], "achieved": bt["total"] * value / 1e9,
                          "peak": hbm, "unit": "GB/s", "frac": bt["total"] * value / 1e9 / hbm,
                          "peak_kind": peak_kind},
        "roofline": {"kernel": "k_igateup + k_idown (8 routed + 1 shared expert, one layer)", "bound": "hbm",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "bytes_per_launch_pair": bytes_layer, "avg_pair_us": per_launch_s * 1e6,
                     "traffic": traffic, "traffic_source": "ncu capture committed in profiles/traffic.json "
                                                          "(per launch pair; not re-measured in this run)",
                     "peak_kind": peak_kind},
        "e2e": {"value": e2e_steps / (e2e_ms / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * cfg.vocab_size},
        "gpu_launches": launches_per_token * args.steps,
        "clocks": clk.summary(),
    }
    if b64 is not None:
        line["b64"] = b64
    if gemv is not None:
        line["expert_gemv"] = gemv
    if not args.no_80b:
        # the 80B-shaped ragged batch on this one GPU (the multi-GPU runs
        # split the same workload by expert parallelism), with the DeltaNet
        # step sweeps of that shape
        m80 = swl.QwenCUDAModel(model_dir(tmp, args.layers, "80b"), device=local)
        m80.set_stream(stream.cuda_stream)
        line["batched"] = batched_decode(m80, m80.config, stream, args, rank, local, None, ep=False,
                                         steps=args.batch_steps, deltanet=True)
        line["deltanet"] = line["batched"].pop("deltanet")
        m80.close()
    if not args.no_cpu_baseline:
        cb = cpu_decode_sample(mdir, 2, 1)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), flush=True)


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
    ap.add_argument("--batch-prompt-max", type=int, default=8192,
                    help="80B batch: prompt lengths uniform in [--batch-prompt, this]")
    ap.add_argument("--model", default="35b", choices=["35b", "80b"],
                    help="80b: the Qwen3-Next-80B-shaped ragged batch alone")
    ap.add_argument("--ep", action="store_true", help="accepted for compatibility: several ranks always split "
                                                      "the 80B batch by expert parallelism")
    ap.add_argument("--no-gemv", action="store_true", help="skip the expert GEMV/GEMM sweeps")
    ap.add_argument("--no-80b", action="store_true", help="skip the 80B-shaped ragged batch on one GPU")
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
