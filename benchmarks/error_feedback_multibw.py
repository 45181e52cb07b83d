"""Runs the EF comparison at several bitwidths and summarises the EF gain.

Counterpart of reference benchmarks/error_feedback_multibw.py: one
subprocess per bitwidth (fresh process state), then a summary table of the
no-EF / EF cumulative-error ratio and the final TinyMLP losses.

    python benchmarks/error_feedback_multibw.py --bitwidths 2 4 8 --out-dir outputs
"""

from __future__ import annotations

import argparse
import csv
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--bitwidths", type=int, nargs="+", default=[2, 4, 8])
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--train-steps", type=int, default=160)
    p.add_argument("--vec-size", type=int, default=1 << 20)
    p.add_argument("--device", default=None)
    p.add_argument("--out-dir", default="ef_outputs")
    args = p.parse_args()
    os.makedirs(args.out_dir, exist_ok=True)
    summary = []
    for b in args.bitwidths:
        cmd = [sys.executable, os.path.join(HERE, "error_feedback_comparison.py"), "--bitwidth", str(b),
               "--steps", str(args.steps), "--train-steps", str(args.train_steps), "--vec-size", str(args.vec_size),
               "--out-dir", args.out_dir]
        if args.device:
            cmd += ["--device", args.device]
        subprocess.run(cmd, check=True)
        with open(os.path.join(args.out_dir, f"ef_benefit_curve_bw{b}.csv")) as fh:
            rows = list(csv.DictReader(fh))
        with open(os.path.join(args.out_dir, f"ef_training_curve_bw{b}.csv")) as fh:
            trows = list(csv.DictReader(fh))
        last = rows[-1]
        noef, ef = float(last["noef_rel_error"]), float(last["ef_rel_error"])
        summary.append({"bitwidth": b, "noef_rel_error": noef, "ef_rel_error": ef,
                        "error_ratio_noef_over_ef": noef / max(ef, 1e-12),
                        "final_loss_noef": float(trows[-1]["loss_noef"]), "final_loss_ef": float(trows[-1]["loss_ef"])})
    with open(os.path.join(args.out_dir, "ef_multibitwidth_summary.csv"), "w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=list(summary[0]))
        w.writeheader()
        w.writerows(summary)
    for s in summary:
        print(s)


if __name__ == "__main__":
    main()
