"""Host-side container tools: safetensors read/write and .qpack repacking.

The .qpack layout follows Swiftlet's container (Sources/SwiftletCore/
Qpack.swift:3-16, repacker :64-166): ``manifest.json``, ``config.json``, a
dense ``model.safetensors`` (every tensor except the routed experts), and
``packed_experts/layout.json`` + ``layer_XX.bin`` holding one fixed-stride
blob per expert (gate/up/down x weight/scales/biases, 16 KiB-aligned stride).
"""
from __future__ import annotations

import json
import os
import shutil
import struct

import numpy as np

PAGE_ALIGNMENT = 16_384
DTYPE_SIZE = {"F32": 4, "I32": 4, "U32": 4, "F16": 2, "BF16": 2, "I16": 2, "U16": 2, "F64": 8, "I64": 8, "U64": 8,
              "I8": 1, "U8": 1}


def read_safetensors(path: str) -> dict[str, tuple[str, list[int], bytes]]:
    """name -> (dtype, shape, raw bytes)."""
    with open(path, "rb") as f:
        data = f.read()
    (n,) = struct.unpack("<Q", data[:8])
    header = json.loads(data[8:8 + n])
    start = 8 + n
    out = {}
    for name, ent in header.items():
        if name == "__metadata__":
            continue
        a, b = ent["data_offsets"]
        out[name] = (ent["dtype"], list(ent["shape"]), data[start + a:start + b])
    return out


def write_safetensors(path: str, tensors: list[tuple[str, str, list[int], bytes]]) -> None:
    """Writes (name, dtype, shape, raw bytes) entries in the given order."""
    header = {}
    off = 0
    for name, dtype, shape, raw in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
    hb = json.dumps(header, separators=(",", ":")).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for _, _, _, raw in tensors:
            f.write(raw)


def load_checkpoint(ckpt_dir: str) -> dict[str, tuple[str, list[int], bytes]]:
    idx = os.path.join(ckpt_dir, "model.safetensors.index.json")
    if os.path.exists(idx):
        files = sorted(set(json.load(open(idx))["weight_map"].values()))
        out = {}
        for fn in files:
            out.update(read_safetensors(os.path.join(ckpt_dir, fn)))
        return out
    return read_safetensors(os.path.join(ckpt_dir, "model.safetensors"))


def repack(ckpt_dir: str, out_dir: str) -> dict:
    """Repacks an mlx-lm checkpoint into a .qpack container; returns the layout."""
    cfg_all = json.load(open(os.path.join(ckpt_dir, "config.json")))
    cfg = cfg_all.get("text_config", cfg_all)
    E, L = cfg["num_experts"], cfg["num_hidden_layers"]
    interval = cfg.get("full_attention_interval", 4)
    tensors = load_checkpoint(ckpt_dir)

    def resolve(name):
        if name in tensors:
            return name
        return "language_model." + name if "language_model." + name in tensors else name

    os.makedirs(os.path.join(out_dir, "packed_experts"), exist_ok=True)
    sections = []
    off = 0
    for proj in ("gate_proj", "up_proj", "down_proj"):
        for part in ("weight", "scales", "biases"):
            name = resolve(f"model.layers.0.mlp.switch_mlp.{proj}.{part}")
            if name not in tensors:
                continue
            dtype, shape, _ = tensors[name]
            if shape[0] != E:
                raise ValueError(f"bad expert tensor shape: {name}")
            per = int(np.prod(shape[1:])) * DTYPE_SIZE[dtype]
            sections.append({"name": f"{proj}.{part}", "dtype": dtype, "shape": shape[1:], "offset": off, "size": per})
            off += per
    stride = (off + PAGE_ALIGNMENT - 1) // PAGE_ALIGNMENT * PAGE_ALIGNMENT
    layout = {"expertCount": E, "layerCount": L, "expertStride": stride, "sections": sections,
              "linearLayers": [(i + 1) % interval != 0 for i in range(L)]}
    files = {}
    for layer in range(L):
        blob = bytearray(stride * E)
        for s in sections:
            _, _, raw = tensors[resolve(f"model.layers.{layer}.mlp.switch_mlp.{s['name']}")]
            for e in range(E):
                blob[e * stride + s["offset"]: e * stride + s["offset"] + s["size"]] = raw[e * s["size"]:(e + 1) * s["size"]]
        fn = "layer_%02d.bin" % layer
        with open(os.path.join(out_dir, "packed_experts", fn), "wb") as f:
            f.write(blob)
        files["packed_experts/" + fn] = len(blob)
    lay = json.dumps(layout, sort_keys=True, indent=2).encode()
    with open(os.path.join(out_dir, "packed_experts", "layout.json"), "wb") as f:
        f.write(lay)
    files["packed_experts/layout.json"] = len(lay)
    dense = [(n, *tensors[n]) for n in sorted(tensors)
             if ".mlp.switch_mlp." not in n and not n.startswith("mtp.") and ".mtp." not in n
             and not n.startswith("vision_tower.") and "model.visual" not in n]
    write_safetensors(os.path.join(out_dir, "model.safetensors"), dense)
    files["model.safetensors"] = os.path.getsize(os.path.join(out_dir, "model.safetensors"))
    for aux in ("config.json", "tokenizer.json", "tokenizer_config.json", "vocab.json", "merges.txt",
                "added_tokens.json", "special_tokens_map.json", "chat_template.jinja"):
        src = os.path.join(ckpt_dir, aux)
        if os.path.exists(src):
            shutil.copyfile(src, os.path.join(out_dir, aux))
            files[aux] = os.path.getsize(src)
    q = cfg_all.get("quantization", {})
    manifest = {"magic": "QPACK", "version": 1, "modelName": cfg.get("model_type", "qwen3_next"),
                "sourceCheckpoint": os.path.basename(os.path.normpath(ckpt_dir)),
                "quantBits": q.get("bits"), "quantGroupSize": q.get("group_size"), "files": files}
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f, sort_keys=True, indent=2)
    return layout


def read_expert(container: str, layer: int, expert: int) -> bytes:
    """One expert blob by a single positioned read (QpackExpertReader.readExpert, Qpack.swift:185-197)."""
    layout = json.load(open(os.path.join(container, "packed_experts", "layout.json")))
    stride = layout["expertStride"]
    path = os.path.join(container, "packed_experts", "layer_%02d.bin" % layer)
    fd = os.open(path, os.O_RDONLY)
    try:
        data = os.pread(fd, stride, expert * stride)
    finally:
        os.close(fd)
    if len(data) != stride:
        raise IOError(f"short read: layer {layer} expert {expert}")
    return data


def write_synthetic(out_dir: str, config: dict, seed: int, bits: int = 4, group_size: int = 64,
                    overrides: dict | None = None, weight_std: float = 0.02) -> str:
    """Writes a synthetic checkpoint: config.json with a "synthetic" block.

    The weights are defined by the counter-based generator in
    swiftlet_b200/csrc/synth.cu and generated on the device at open.
    """
    os.makedirs(out_dir, exist_ok=True)
    cfg = dict(config)
    q = {"group_size": group_size, "bits": bits}
    for k, v in (overrides or {}).items():
        q[k] = v
    cfg["quantization"] = q
    cfg["synthetic"] = {"seed": int(seed), "scheme": "swl-synth-v1", "weight_std": weight_std,
                        "scale_dtype": "bf16", "plain_dtype": "bf16"}
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    return out_dir


def write_hashes(container: str) -> dict:
    """hashes.json for a container (verify_container.py --write-hashes): the
    SHA-256 of every file except dot-files and hashes.json itself."""
    import hashlib
    out = {}
    for r, _, files in os.walk(container):
        for f in files:
            rel = os.path.relpath(os.path.join(r, f), container)
            if rel.startswith(".") or rel == "hashes.json":
                continue
            h = hashlib.sha256()
            with open(os.path.join(container, rel), "rb") as fh:
                for chunk in iter(lambda: fh.read(1 << 22), b""):
                    h.update(chunk)
            out[rel] = h.hexdigest()
    with open(os.path.join(container, "hashes.json"), "w") as f:
        json.dump({"files": dict(sorted(out.items()))}, f, indent=1)
    return out
