"""Per-kernel timeline of batch-1 decode steps.

Opens a synthetic checkpoint of the 35B shape (or the 80B shape) with the
library's per-CTA trace on (``SWL_TRACE``), decodes a few greedy tokens after a
short prompt, and summarises one traced token kernel kind by kernel kind:

* ``critical``: end of the kind's launch minus end of the launch before it,
  averaged over layers (the kind's share of the token's time);
* ``staging``: median over CTAs of input staging after the dependency wait
  (normalisation, digit table);
* ``loop``: median over CTAs of the tile loop (weights reduced on the tensor
  cores, including any wait for weight tiles still in flight);
* ``tail``: median over CTAs of the epilogue after the loop.

Every CTA of a traced launch appends one record {tag, block, start, waited,
staged, looped, end} (globaltimer ns); the tag is 16 * (layer + 1) + kind for
the layer kernels, 1 for the embedding and 8 for lm_head.

    python -m swiftlet_b200.timeline [--model 35b|80b] [--layers N] [--csv PATH]
"""
from __future__ import annotations

import argparse
import collections
import csv
import os
import statistics
import tempfile

KINDS = {1: "embed", 2: "in_proj", 3: "mixer", 4: "out_proj", 5: "router", 6: "gate/up", 7: "down", 8: "lm_head"}


def summarise(path: str) -> str:
    """Per-kind table of the second traced token of a trace CSV."""
    rows = [{k: int(v) for k, v in r.items()} for r in csv.DictReader(open(path))]
    rows.sort(key=lambda r: r["start_ns"])
    embeds = [r["start_ns"] for r in rows if r["tag"] == 1 and r["block"] == 0]
    if len(embeds) < 2:
        raise RuntimeError("the trace holds fewer than two tokens")
    lo, hi = embeds[-2], embeds[-1]
    launches = collections.defaultdict(list)
    for r in rows:
        if lo <= r["start_ns"] < hi:
            launches[r["tag"]].append(r)
    order = sorted(launches, key=lambda t: max(r["end_ns"] for r in launches[t]))
    agg = collections.defaultdict(lambda: {"n": 0, "crit": 0.0, "stage": [], "loop": [], "tail": []})
    prev_end = None
    for tag in order:
        g = launches[tag]
        end = max(r["end_ns"] for r in g)
        a = agg[KINDS.get(tag % 16 if tag >= 16 else tag, str(tag))]
        a["n"] += 1
        if prev_end is not None and tag != 1:  # the embedding overlaps the previous token's lm_head
            a["crit"] += (end - prev_end) / 1e3
        prev_end = end
        for r in g:
            if r["staged_ns"]:
                a["stage"].append((r["staged_ns"] - r["waited_ns"]) / 1e3)
            if r["looped_ns"]:
                a["loop"].append((r["looped_ns"] - (r["staged_ns"] or r["waited_ns"])) / 1e3)
                a["tail"].append((r["end_ns"] - r["looped_ns"]) / 1e3)
    first = min(min(r["start_ns"] for r in launches[t]) for t in order)
    out = [f"token: {(prev_end - first) / 1e3:.1f} us over {len(order)} launches",
           "| kernel | launches | critical us per launch | staging us | loop us | tail us |",
           "|---|---|---|---|---|---|"]
    med = lambda v: f"{statistics.median(v):.2f}" if v else "-"
    for kind, a in agg.items():
        out.append(f"| {kind} | {a['n']} | {a['crit'] / a['n']:.2f} | {med(a['stage'])} | {med(a['loop'])} | "
                   f"{med(a['tail'])} |")
    return "\n".join(out)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", default="35b", choices=["35b", "80b"])
    ap.add_argument("--layers", type=int, default=None, help="layers of the synthetic model (default: all)")
    ap.add_argument("--prompt", type=int, default=64)
    ap.add_argument("--csv", default=None, help="also keep the raw trace here")
    args = ap.parse_args()
    os.environ.setdefault("SWL_TRACE", "400000")  # records; read when the model opens
    import numpy as np

    import swiftlet_b200 as swl
    from swiftlet_b200 import formats
    from swiftlet_b200.configs import NEXT_80B, Q35_35B, with_layers

    base = NEXT_80B if args.model == "80b" else Q35_35B
    cfg = with_layers(base, args.layers) if args.layers else base
    with tempfile.TemporaryDirectory() as tmp:
        d = formats.write_synthetic(os.path.join(tmp, "synth"), cfg, seed=35, bits=4)
        m = swl.QwenCUDAModel(d)
        st = swl.DecodeState(args.prompt + 64)
        rng = np.random.default_rng(1)
        lg = m.step(rng.integers(0, m.config.vocab_size, args.prompt).tolist(), st)
        for _ in range(5):  # warm-up tokens, traced into the void
            lg = m.step([int(np.argmax(lg))], st)
        m.trace_dump(os.devnull)
        for _ in range(3):
            lg = m.step([int(np.argmax(lg))], st)
        path = args.csv or os.path.join(tmp, "trace.csv")
        m.trace_dump(path)
        print(summarise(path))


if __name__ == "__main__":
    main()
