"""Single-GPU kernel cases for timing and Nsight Compute captures.

    python benchmarks/kernel_case.py --op allreduce --n 67108864 --bits 4 --ef
    python benchmarks/kernel_case.py --op compress --n 67108864 --bits 4

Runs `--warmup` untimed calls then `--iters` calls timed with CUDA events on
the launching stream (synchronised on both sides), and prints one JSON line
with the per-call time and the achieved HBM bandwidth from the algorithmic
byte count (the minimum bytes the op must move).  The op runs on a one-rank
communicator, so the fused all-reduce executes every local phase (quantise,
pack, store, dequantise-reduce, requantise, unpack) with loopback stores.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bitscom_b200 as bitscom  # noqa: E402
from bitscom_b200.parallel.comm import Communicator  # noqa: E402


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--op", choices=["allreduce", "reduce_scatter", "all_gather", "compress", "decompress", "ef_roundtrip",
                                    "standalone"],
                   default="allreduce")
    p.add_argument("--n", type=int, default=1 << 26)
    p.add_argument("--bits", type=int, default=4)
    p.add_argument("--fmt", default="int")
    p.add_argument("--dtype", default="float32")
    p.add_argument("--ef", action="store_true")
    p.add_argument("--res-dtype", default="float32", choices=["float32", "bfloat16"])
    p.add_argument("--sr", action="store_true")
    p.add_argument("--algo", default="twoshot")
    p.add_argument("--max-ctas", type=int, default=0)
    p.add_argument("--lag", type=int, default=None, help="schedule lag of the fused kernel (-1 automatic, 0 phase-major)")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=10)
    args = p.parse_args()

    torch.cuda.set_device(0)
    dt = getattr(torch, args.dtype)
    esz = torch.tensor([], dtype=dt).element_size()
    x = (torch.randn(args.n, device="cuda") * 1e-3).to(dt)
    res = torch.zeros(args.n, device="cuda", dtype=getattr(torch, args.res_dtype)) if args.ef else None
    rsz = 4 if args.res_dtype == "float32" else 2
    comm = None
    if args.op in ("allreduce", "reduce_scatter", "all_gather"):
        comm = Communicator.create_local(0, workspace_bytes=max(256 << 20, 4 * args.n * args.bits // 8))
        if args.lag is not None:
            comm.set_schedule_lag(args.lag)
    packed = bitscom.compress_tensor(x, args.bits)
    res_sa = torch.zeros(args.n, device="cuda") if args.op == "standalone" else None
    out = torch.empty_like(x)

    def call():
        if args.op == "allreduce":
            comm.all_reduce(x, out=out, bits=args.bits, fmt=args.fmt, residual=res, stochastic_rounding=args.sr,
                            algo=args.algo, max_ctas=args.max_ctas)
        elif args.op == "reduce_scatter":
            comm.reduce_scatter(out, x, bits=args.bits, fmt=args.fmt, residual=res, max_ctas=args.max_ctas)
        elif args.op == "all_gather":
            comm.all_gather(out, x, bits=args.bits, fmt=args.fmt, residual=res, max_ctas=args.max_ctas)
        elif args.op == "compress":
            bitscom.compress_tensor(x, args.bits, stochastic_rounding=args.sr)
        elif args.op == "decompress":
            bitscom.decompress_tensor(packed)
        elif args.op == "standalone":
            # every standalone kernel once: absmax + quantise (int16), pack,
            # unpack, int16 dequantise, fused compress, fused decompress, EF roundtrip
            from bitscom_b200.quantization import dequantize_tensor, pack_lowbit, quantize_tensor, unpack_lowbit

            q, scale = quantize_tensor(x, args.bits)
            pk, _ = pack_lowbit(q, args.bits)
            q2 = unpack_lowbit(pk, args.bits, x.numel())
            dequantize_tensor(q2, scale, dtype=x.dtype, shape=x.shape)
            bitscom.compress_tensor(x, args.bits)
            bitscom.decompress_tensor(packed)
            bitscom.ef_roundtrip(x, res_sa, args.bits)
        else:
            bitscom.ef_roundtrip(x, res, args.bits, stochastic_rounding=args.sr)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.iters):
        call()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.iters
    n = args.n
    packed_b = n * args.bits / 8
    if args.op == "allreduce":
        # read x (+ read/write residual) + write out, plus packed store+load of both phases
        alg = n * esz * 2 + (2 * n * rsz if args.ef else 0) + 4 * packed_b
    elif args.op in ("reduce_scatter", "all_gather"):
        alg = n * esz * 2 + (2 * n * rsz if args.ef else 0) + 2 * packed_b
    elif args.op == "compress":
        alg = 2 * n * esz + packed_b  # absmax pass + quantise pass + packed write
    elif args.op == "decompress":
        alg = packed_b + n * esz
    elif args.op == "standalone":
        alg = 0  # a mix of kernels: only the per-kernel profile is meaningful
    else:
        alg = 3 * n * esz + (2 * n * rsz if args.ef else 0)
    print(json.dumps({"op": args.op, "n": n, "bits": args.bits, "fmt": args.fmt, "dtype": args.dtype, "ef": args.ef, "res_dtype": args.res_dtype if args.ef else None,
                      "sr": args.sr, "algo": args.algo, "ms": round(ms, 5), "alg_bytes": int(alg),
                      "alg_GBs": round(alg / (ms * 1e6), 1)}))


if __name__ == "__main__":
    main()
