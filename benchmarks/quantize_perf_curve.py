"""quantize_tensor latency: CPU vs GPU, 2^10 .. 2^23 elements.

Counterpart of reference benchmarks/quantize_perf_curve.py (its published
curve: benchmarks/outputs/quantize_curve_bw4.csv).  GPU timings use CUDA
events around `iters` calls (the reference timed with perf_counter around a
device sync); the public API returns a Python float scale, so every call
includes one device->host read, as in the reference.  Also reports the
sync-free fused compress (quantise + pack on the device) for comparison.

    python benchmarks/quantize_perf_curve.py --bitwidth 4 --out quantize_curve_bw4.csv
"""

from __future__ import annotations

import argparse
import csv
import os
import statistics
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bitscom_b200.ops.quant import quantize_pack  # noqa: E402
from bitscom_b200.quantization import quantize_tensor  # noqa: E402


def cpu_ms(x, bits, warmup, iters):
    for _ in range(warmup):
        quantize_tensor(x, bits)
    samples = []
    for _ in range(iters):
        t0 = time.perf_counter()
        quantize_tensor(x, bits)
        samples.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(samples)


def gpu_ms(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--bitwidth", type=int, default=4)
    p.add_argument("--min-pow2", type=int, default=10)
    p.add_argument("--max-pow2", type=int, default=23)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iters", type=int, default=30)
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--out", default=None)
    args = p.parse_args()
    rows = []
    for k in range(args.min_pow2, args.max_pow2 + 1):
        n = 1 << k
        x = torch.linspace(-1.0, 1.0, n)
        xg = x.cuda()
        c = float("nan") if args.no_cpu else cpu_ms(x, args.bitwidth, 2, max(3, args.iters // 5))
        g = gpu_ms(lambda: quantize_tensor(xg, args.bitwidth), args.warmup, args.iters)
        f = gpu_ms(lambda: quantize_pack(xg, args.bitwidth), args.warmup, args.iters)
        rows.append({"numel": n, "cpu_ms": c, "gpu_ms": g, "gpu_fused_compress_ms": f,
                     "speedup_gpu_vs_cpu": c / g, "gpu_melems_per_s": n / 1e6 / (g / 1e3)})
        print(f"n=2^{k:2d} cpu={c:9.4f} ms gpu={g:8.4f} ms fused={f:8.4f} ms", flush=True)
    if args.out:
        with open(args.out, "w", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=list(rows[0]))
            w.writeheader()
            w.writerows(rows)


if __name__ == "__main__":
    main()
