"""Container formats: .qpack repack round trip (QpackTests.swift:15-63) and
the synthetic checkpoint generator's definition."""
import json
import os
import struct

import numpy as np
import pytest

import oracle
from conftest import REF_FIXTURES, TINY_BASELINE
from swiftlet_b200 import formats
from swiftlet_b200.configs import TINY, Q35_35B, with_layers


def test_qpack_repack_round_trip(tmp_path):
    src = os.path.join(REF_FIXTURES, "tiny-model-q4")
    out = str(tmp_path / "tiny-q4.qpack")
    layout = formats.repack(src, out)
    cfg = json.load(open(os.path.join(src, "config.json")))
    assert layout["expertCount"] == cfg["num_experts"]
    assert layout["layerCount"] == cfg["num_hidden_layers"]
    assert layout["expertStride"] % formats.PAGE_ALIGNMENT == 0
    tensors = formats.load_checkpoint(src)
    for layer in (0, cfg["num_hidden_layers"] - 1):
        for expert in (0, 3, cfg["num_experts"] - 1):
            blob = formats.read_expert(out, layer, expert)
            for s in layout["sections"]:
                _, _, raw = tensors[f"model.layers.{layer}.mlp.switch_mlp.{s['name']}"]
                assert blob[s["offset"]:s["offset"] + s["size"]] == raw[expert * s["size"]:(expert + 1) * s["size"]]
    dense = formats.read_safetensors(os.path.join(out, "model.safetensors"))
    for name in ("model.embed_tokens.weight", "model.layers.0.input_layernorm.weight", "model.layers.0.mlp.gate.scales",
                 "model.layers.3.self_attn.q_norm.weight"):
        assert dense[name] == tensors[name]
    assert "model.layers.0.mlp.switch_mlp.gate_proj.weight" not in dense
    sec = {s["name"]: s for s in layout["sections"]}
    assert sec["gate_proj.weight"]["shape"] == [cfg["moe_intermediate_size"], cfg["hidden_size"] // 8]
    man = json.load(open(os.path.join(out, "manifest.json")))
    assert man["magic"] == "QPACK" and man["quantBits"] == 4


def test_qpack_short_read_is_an_error(tmp_path):
    out = str(tmp_path / "c.qpack")
    formats.repack(os.path.join(REF_FIXTURES, "tiny-model-q4"), out)
    p = os.path.join(out, "packed_experts", "layer_00.bin")
    data = open(p, "rb").read()
    open(p, "wb").write(data[:-100])
    with pytest.raises(IOError):
        formats.read_expert(out, 0, 7)


def test_tiny_baseline_records_group_override():
    cfg = json.load(open(os.path.join(TINY_BASELINE, "config.json")))
    q = cfg["quantization"]
    assert q["group_size"] == 64 and q["bits"] == 4
    assert q["model.layers.0.mlp.switch_mlp.down_proj"] == {"group_size": 32, "bits": 4}
    assert q["model.layers.0.mlp.shared_expert.down_proj"] == {"group_size": 32, "bits": 4}


# --- synthetic generator: an independent numpy restatement -----------------
GAMMA = 0x9E3779B97F4A7C15
M64 = (1 << 64) - 1


def _mix(z):
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9 & M64
    z = (z ^ (z >> 27)) * 0x94D049BB133111EB & M64
    return z ^ (z >> 31)


def _key(name, seed):
    h = 0xCBF29CE484222325
    for c in name.encode():
        h = ((h ^ c) * 0x100000001B3) & M64
    return h ^ ((seed * GAMMA) & M64)


def _hash(key, i):
    return _mix((key + (i + 1) * GAMMA) & M64)


def _bf16(f):
    u = int(np.float32(f).view(np.uint32))
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFFFFFF
    return u >> 16


def test_synthetic_bytes_match_independent_restatement(tmp_path):
    d = formats.write_synthetic(str(tmp_path / "syn"), with_layers(TINY, 4), seed=1234, group_size=32)
    m = oracle.OracleModel(d)
    f32 = np.float32
    # packed words
    name = "model.layers.1.mlp.switch_mlp.up_proj.weight"
    raw = np.frombuffer(m.tensor_bytes(name, 100, 140), np.uint32)
    k = _key(name, 1234)
    assert [int(x) for x in raw] == [_hash(k, i) & 0xFFFFFFFF for i in range(100, 140)]
    # scales and biases (4-bit: qstd = sqrt(255/12))
    mod = "model.layers.2.linear_attn.in_proj_qkvz"
    s0 = f32(0.02 / 4.6097722286464435)
    ks, kb = _key(mod + ".scales", 1234), _key(mod + ".biases", 1234)
    sc = np.frombuffer(m.tensor_bytes(mod + ".scales", 0, 30), np.uint16)
    bi = np.frombuffer(m.tensor_bytes(mod + ".biases", 0, 30), np.uint16)
    for i in range(30):
        u = f32(_hash(ks, i) >> 40) * f32(5.9604644775390625e-08)
        s = (u * f32(0.5) + f32(0.75)) * s0
        assert int(sc[i]) == _bf16(s)
        sq = np.array([_bf16(s) << 16], np.uint32).view(np.float32)[0]
        h = _hash(kb, i)
        n = f32(sum((h >> (16 * j)) & 0xFFFF for j in range(4)) - 131070) * f32(2.6429039e-05)
        b = sq * f32(-7.5) + n * f32(np.float32(0.1 * 0.02))
        assert int(bi[i]) == _bf16(b)
    # a norm weight
    nm = "model.layers.0.input_layernorm.weight"
    kn = _key(nm, 1234)
    vals = np.frombuffer(m.tensor_bytes(nm, 0, 16), np.uint16)
    for i in range(16):
        h = _hash(kn, i)
        n = f32(sum((h >> (16 * j)) & 0xFFFF for j in range(4)) - 131070) * f32(2.6429039e-05)
        assert int(vals[i]) == _bf16(f32(1.0) + n * f32(0.05))


def test_synthetic_35b_shape_tensor_table(tmp_path):
    d = formats.write_synthetic(str(tmp_path / "s35"), with_layers(Q35_35B, 4), seed=7)
    m = oracle.OracleModel(d)
    assert m.tensor_info("model.layers.0.mlp.switch_mlp.gate_proj.weight") == ("U32", [256, 512, 256])
    assert m.tensor_info("model.layers.0.mlp.switch_mlp.down_proj.scales") == ("BF16", [256, 2048, 8])
    assert m.tensor_info("model.layers.0.linear_attn.in_proj_qkv.weight") == ("U32", [8192, 256])
    assert m.tensor_info("model.layers.3.self_attn.q_proj.weight") == ("U32", [8192, 256])
    assert m.tensor_info("lm_head.scales") == ("BF16", [151936, 32])
