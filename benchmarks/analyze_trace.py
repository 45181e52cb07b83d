"""CLI: communication share of a torch.profiler Chrome trace over a stable window.

    python benchmarks/analyze_trace.py trace.json --skip-steps 1 --keep-steps 3 --gpu-only
"""

from __future__ import annotations

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bitscom_b200.utils.trace import analyze, load_events, step_window, time_window  # noqa: E402


def main():
    p = argparse.ArgumentParser()
    p.add_argument("trace")
    p.add_argument("--skip-steps", type=int, default=1)
    p.add_argument("--keep-steps", type=int, default=0)
    p.add_argument("--skip-ratio", type=float, default=None, help="use a time window instead of profiler steps")
    p.add_argument("--gpu-only", action="store_true")
    p.add_argument("--top-k", type=int, default=15)
    args = p.parse_args()
    ev = load_events(args.trace)
    win = time_window(ev, args.skip_ratio) if args.skip_ratio is not None else step_window(ev, args.skip_steps, args.keep_steps)
    res = analyze(ev, win, gpu_only=args.gpu_only, top_k=args.top_k)
    print(json.dumps({k: v for k, v in res.items() if k != "top_ops"}))
    for name, us in res["top_ops"]:
        print(f"{us:12.1f} us  {name}")


if __name__ == "__main__":
    main()
