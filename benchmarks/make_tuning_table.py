"""Builds the fused collectives' tuning table from measured sweeps.

Input: JSON documents written by ``benchmarks/allreduce_sweep.py --algos
oneshot twoshot --out FILE`` (one per world size; any bitwidths and formats).
For every (world, bits, format) the one-shot threshold is the largest packed
message size per rank at which one-shot was at least as fast as two-shot and
above which two-shot won at every measured size (the crossover, read from
the large end so that one noisy small-size sample does not cut it short); a
format where two-shot wins at every size gets threshold 0.  When one-shot
still wins at the largest measured size, that size is the threshold.  Writes the table
read by ``bitscom_b200.tuning`` (``BITSCOM_TUNING_FILE`` or the shipped
``bitscom_b200/tuning/b200.json``), keeping the table's other keys.

    python benchmarks/make_tuning_table.py sweep_w2.json sweep_w4.json sweep_w8.json \\
        --out bitscom_b200/tuning/b200.json
"""

from __future__ import annotations

import argparse
import json
import os
from collections import defaultdict


def crossover(rows):
    """{(world, bits, fmt): oneshot_max_packed_bytes} from sweep rows."""
    times = defaultdict(dict)  # key -> {packed_bytes: {algo: ms}}
    for r in rows:
        if r.get("impl") != "ours" or r.get("algo") not in ("oneshot", "twoshot"):
            continue
        n = r["bytes_fp32"] // 4
        packed = n * r["bits"] // 8
        times[(r["world"], r["bits"], r["fmt"])].setdefault(packed, {})[r["algo"]] = r["ms"]
    out = {}
    for key, by_size in times.items():
        best = 0
        for packed in sorted(by_size, reverse=True):
            t = by_size[packed]
            if "oneshot" not in t or "twoshot" not in t:
                continue
            if t["oneshot"] <= t["twoshot"]:
                best = packed
                break
        out[key] = best
    return out


def main():
    p = argparse.ArgumentParser()
    p.add_argument("sweeps", nargs="+")
    p.add_argument("--out", required=True)
    p.add_argument("--device", default="NVIDIA B200")
    args = p.parse_args()
    rows, sources = [], []
    for f in args.sweeps:
        with open(f, encoding="utf-8") as fh:
            doc = json.load(fh)
        rows += doc["rows"]
        sources.append({"file": os.path.basename(f), "command": doc.get("command"), "clocks": doc.get("clocks")})
    table = {}
    if os.path.exists(args.out):
        with open(args.out, encoding="utf-8") as fh:
            table = json.load(fh)
    cross = crossover(rows)
    old = [e for e in table.get("entries", []) if (e["world"], e["bits"], e.get("fmt", "int")) not in cross]
    new = [{"world": w, "bits": b, "fmt": f, "oneshot_max_packed_bytes": v}
           for (w, b, f), v in sorted(cross.items())]
    table["device"] = args.device
    table["entries"] = old + new
    table["entries_how"] = ("benchmarks/allreduce_sweep.py --algos oneshot twoshot (EF + SR, CUDA-event time, max over "
                            "ranks); threshold = largest packed bytes per rank up to which one-shot was never slower")
    table["entries_sources"] = sources
    with open(args.out, "w", encoding="utf-8") as fh:
        json.dump(table, fh, indent=1)
        fh.write("\n")
    for e in new:
        print(e)


if __name__ == "__main__":
    main()
