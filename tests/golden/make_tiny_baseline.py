"""Writes the BASELINE tiny checkpoint and its oracle goldens.

The checkpoint (tests/golden/tiny-baseline/) is the 4-layer tiny hybrid of
swiftlet_b200.configs.TINY: weights N(0, 0.02) from numpy's PCG64 with a
fixed seed, every linear MLX-affine quantised to 4 bits with group 64 and
bf16 scales/biases. Modules whose in-dim is 32 (expert and shared
down_proj) use a per-module {group_size: 32} override recorded in
config.json, the same mechanism as Checkpoint.swift:41-46.

Quantiser (affine min/max): scale = (max - min) / 15, bias = min, both
rounded to bf16; q = clamp(round((w - bias) / scale), 0, 15), packed
low-nibble-first into uint32 words. Parity is defined against these bytes.

The goldens (tiny_baseline_golden.json) are produced by the CPU oracle
(oracle/): the 8-id prompt, the logits after the prompt, per-layer top-k
expert ids for the prompt, and 32 greedy continuation tokens.

Usage: python tests/golden/make_tiny_baseline.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from swiftlet_b200.configs import TINY  # noqa: E402
from swiftlet_b200.formats import write_safetensors  # noqa: E402

SEED = 20240601
OUT = os.path.join(HERE, "tiny-baseline")


def bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_val(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def quantize(w: np.ndarray, gs: int):
    rows, cols = w.shape[-2], w.shape[-1]
    lead = w.shape[:-2]
    g = w.reshape(*lead, rows, cols // gs, gs).astype(np.float32)
    mn, mx = g.min(-1), g.max(-1)
    scale_b = bf16_bits((mx - mn) / 15.0)
    bias_b = bf16_bits(mn)
    s, b = bf16_val(scale_b), bf16_val(bias_b)
    q = np.clip(np.round((g - b[..., None]) / np.where(s == 0, 1, s)[..., None]), 0, 15).astype(np.uint32)
    q = q.reshape(*lead, rows, cols // 8, 8)
    packed = np.zeros(q.shape[:-1], np.uint32)
    for j in range(8):
        packed |= q[..., j] << np.uint32(4 * j)
    return packed, scale_b.reshape(*lead, rows, cols // gs), bias_b.reshape(*lead, rows, cols // gs)


def main() -> None:
    rng = np.random.default_rng(SEED)
    c = TINY
    D, V, E, I, SI = c["hidden_size"], c["vocab_size"], c["num_experts"], c["moe_intermediate_size"], c["shared_expert_intermediate_size"]
    nk, nv, dk, dv, K = c["linear_num_key_heads"], c["linear_num_value_heads"], c["linear_key_head_dim"], c["linear_value_head_dim"], c["linear_conv_kernel_dim"]
    H, KVH, hd = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
    keyDim, valueDim = nk * dk, nv * dv
    convDim = 2 * keyDim + valueDim
    tensors = []
    overrides = {}

    def lin(name, shape):
        w = rng.normal(0.0, 0.02, size=shape).astype(np.float32)
        gs = 64 if shape[-1] % 64 == 0 else 32
        if gs != 64:
            overrides[name] = {"group_size": gs, "bits": 4}
        p, s, b = quantize(w, gs)
        tensors.append((name + ".weight", "U32", list(p.shape), p.tobytes()))
        tensors.append((name + ".scales", "BF16", list(s.shape), s.tobytes()))
        tensors.append((name + ".biases", "BF16", list(b.shape), b.tobytes()))

    def plain(name, arr):
        tensors.append((name, "BF16", list(arr.shape), bf16_bits(arr).tobytes()))

    lin("model.embed_tokens", (V, D))
    lin("lm_head", (V, D))
    plain("model.norm.weight", 1.0 + 0.05 * rng.standard_normal(D).astype(np.float32))
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}."
        plain(p + "input_layernorm.weight", 1.0 + 0.05 * rng.standard_normal(D).astype(np.float32))
        plain(p + "post_attention_layernorm.weight", 1.0 + 0.05 * rng.standard_normal(D).astype(np.float32))
        if (i + 1) % c["full_attention_interval"] != 0:
            lin(p + "linear_attn.in_proj_qkvz", (2 * keyDim + 2 * valueDim, D))
            lin(p + "linear_attn.in_proj_ba", (2 * nv, D))
            plain(p + "linear_attn.conv1d.weight", 0.3 * rng.standard_normal((convDim, K, 1)).astype(np.float32))
            plain(p + "linear_attn.A_log", rng.uniform(0, 1, nv).astype(np.float32))
            plain(p + "linear_attn.dt_bias", 0.5 * rng.standard_normal(nv).astype(np.float32))
            plain(p + "linear_attn.norm.weight", 1.0 + 0.05 * rng.standard_normal(dv).astype(np.float32))
            lin(p + "linear_attn.out_proj", (D, valueDim))
        else:
            lin(p + "self_attn.q_proj", (2 * H * hd, D))
            lin(p + "self_attn.k_proj", (KVH * hd, D))
            lin(p + "self_attn.v_proj", (KVH * hd, D))
            lin(p + "self_attn.o_proj", (D, H * hd))
            plain(p + "self_attn.q_norm.weight", 1.0 + 0.05 * rng.standard_normal(hd).astype(np.float32))
            plain(p + "self_attn.k_norm.weight", 1.0 + 0.05 * rng.standard_normal(hd).astype(np.float32))
        lin(p + "mlp.gate", (E, D))
        lin(p + "mlp.switch_mlp.gate_proj", (E, I, D))
        lin(p + "mlp.switch_mlp.up_proj", (E, I, D))
        lin(p + "mlp.switch_mlp.down_proj", (E, D, I))
        lin(p + "mlp.shared_expert.gate_proj", (SI, D))
        lin(p + "mlp.shared_expert.up_proj", (SI, D))
        lin(p + "mlp.shared_expert.down_proj", (D, SI))
        lin(p + "mlp.shared_expert_gate", (1, D))
    os.makedirs(OUT, exist_ok=True)
    write_safetensors(os.path.join(OUT, "model.safetensors"), sorted(tensors))
    cfg = dict(c)
    cfg["quantization"] = {"group_size": 64, "bits": 4, **overrides}
    with open(os.path.join(OUT, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2, sort_keys=True)

    # Goldens from the CPU oracle.
    import oracle
    prompt = [int(t) for t in np.random.default_rng(SEED + 1).integers(0, V, 8)]
    m = oracle.OracleModel(OUT)
    st = oracle.DecodeState()
    logits = m.step(prompt, st)
    prompt_logits = logits.tolist()
    greedy = []
    for _ in range(32):
        best = int(np.argmax(logits))
        greedy.append(best)
        logits = m.step([best], st)
    caps = m.forward(prompt)
    picks = caps["picks"].tolist()   # [layer][position][k] of the whole-prompt pass
    golden = {"seed": SEED, "prompt": prompt, "prompt_logits": prompt_logits, "greedy_32": greedy,
              "topk_ids_per_layer": picks, "generator": "tests/golden/make_tiny_baseline.py"}
    with open(os.path.join(HERE, "tiny_baseline_golden.json"), "w") as f:
        json.dump(golden, f)
    print("greedy:", greedy)


if __name__ == "__main__":
    main()
