"""Low-bit all-reduce sweep: fp32-equivalent bus bandwidth vs message size.

The sweep configuration named in BASELINE.json: per-rank seeded fp32 gradient-like tensors ~N(0, 1e-3)
with 1% outliers ~N(0, 1e-1), sizes 1 KB .. 1 GB in powers of two, bitwidths
1/2/4/8 (+ fp8 block-scaled), error feedback on, stochastic rounding, at
2/4/8 GPUs; compared with NCCL fp32 all-reduce and the reference's low-bit
all-reduce (its LowBitGroup path over NCCL).

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        benchmarks/allreduce_sweep.py --min-kb 1 --max-mb 1024 --bits 4

Timing: CUDA events on the launching stream around `iters` back-to-back
calls after `warmup` calls, barrier + synchronize on both sides, max over
ranks.  busBW = 2 (W-1)/W * fp32 bytes / time (the nccl-tests convention),
so a low-bit all-reduce that moves fewer bytes shows as a higher
fp32-equivalent bandwidth.  Rank 0 prints one JSON line per (impl, bits,
algo, size); with ``--out FILE`` it also writes one JSON document with every
row and the clock record (nvidia-smi samples of every GPU of the run, taken
while the sweep ran: median SM clock under load, throttle reasons).
``--algos oneshot twoshot`` times both fused algorithms at every size (the
input of the tuning table); the default, ``auto``, times the automatic choice.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def gradient_like(n: int, rank: int, device) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(1234 + rank)
    x = torch.randn(n, generator=g) * 1e-3
    k = max(1, n // 100)
    idx = torch.randint(0, n, (k,), generator=g)
    x[idx] = torch.randn(k, generator=g) * 1e-1
    return x.to(device)


def time_fn(fn, warmup: int, iters: int, world: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    if world > 1:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--min-kb", type=float, default=1)
    p.add_argument("--max-mb", type=float, default=256)
    p.add_argument("--bits", type=int, nargs="+", default=[4])
    p.add_argument("--fp8", action="store_true", help="also run the E4M3 8-bit format")
    p.add_argument("--impls", nargs="+", default=["ours", "nccl"], choices=["ours", "nccl", "reference", "reference_ef"])
    p.add_argument("--no-ef", action="store_true")
    p.add_argument("--residual-dtype", choices=["float32", "bfloat16"], default="float32",
                   help="element type of our error-feedback residual")
    p.add_argument("--no-sr", action="store_true")
    p.add_argument("--algos", nargs="+", default=["auto"], choices=["auto", "oneshot", "twoshot"])
    p.add_argument("--out", default=None, help="rank 0 writes every row plus the clock record to this JSON file")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--max-ctas", type=int, default=0)
    p.add_argument("--lag", type=int, nargs="+", default=[-1],
                   help="schedule lags to sweep (-1 automatic, 0 phase-major)")
    p.add_argument("--spi", type=int, nargs="+", default=[0],
                   help="sub-chunks per work item to sweep (0 automatic)")
    args = p.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29561")
    kw = {} if world > 1 else {"init_method": "tcp://127.0.0.1:%s" % os.environ["MASTER_PORT"], "rank": 0, "world_size": 1}
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local), **kw)

    from bitscom_b200.parallel.comm import Communicator

    comm = Communicator.for_group(None, local) if world > 1 else Communicator.create_local(local)
    ref_group = None
    ref_pg = None
    if "reference" in args.impls or "reference_ef" in args.impls:
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        import bitscom as ref_bitscom  # the reference package
        from bitscom.api import LowBitGroup as RefGroup
    if "reference_ef" in args.impls:
        # The reference's error-feedback path: its C++ lowbit backend (one
        # bitwidth per process), reached through dist.all_reduce.
        ref_bitscom.init(bitwidth=args.bits[0], error_feedback=not args.no_ef)
        ref_pg = dist.new_group(backend="lowbit")

    from bitscom_b200.utils.clocks import ClockSampler

    sampler = ClockSampler(list(range(world)) if rank == 0 else [local]).__enter__()
    rows = []
    sizes = []
    s = int(args.min_kb * 1024)
    while s <= int(args.max_mb * 2**20):
        sizes.append(s)
        s *= 2
    formats = [(b, "int") for b in args.bits] + ([(8, "e4m3")] if args.fp8 else [])
    for nbytes in sizes:
        n = max(1, nbytes // 4)
        x0 = gradient_like(n, rank, "cuda")
        buf = x0.clone()
        bus_factor = 2.0 * (world - 1) / world if world > 1 else 1.0
        runs = [(impl, lag, spi, algo) for impl in args.impls for lag in (args.lag if impl == "ours" else [None])
                for spi in (args.spi if impl == "ours" else [None])
                for algo in (args.algos if impl == "ours" else [None])]
        for impl, lag, spi, algo in runs:
            if lag is not None:
                comm.set_schedule_lag(lag)
            if spi is not None:
                comm.set_sub_per_item(spi)
            for bits, fmt in formats if impl != "nccl" else [(32, "fp32")]:
                if impl == "nccl":
                    fn = lambda: dist.all_reduce(buf)
                elif impl == "ours":
                    res = None if args.no_ef else torch.zeros(n, device="cuda", dtype=getattr(torch, args.residual_dtype))
                    counter = [0]

                    def fn(res=res, bits=bits, fmt=fmt, counter=counter):
                        counter[0] += 1
                        comm.all_reduce(buf, bits=bits, fmt=fmt, residual=res,
                                        stochastic_rounding=not args.no_sr and fmt == "int",
                                        offset=counter[0], algo=algo, max_ctas=args.max_ctas)
                elif impl == "reference_ef":
                    if fmt != "int" or bits != args.bits[0] or n % world:
                        continue
                    fn = lambda: dist.all_reduce(buf, group=ref_pg)
                else:
                    if fmt != "int":
                        continue
                    ref_group = RefGroup(bitwidth=bits, process_group=dist.group.WORLD,
                                         stochastic_rounding=not args.no_sr)
                    fn = lambda g=ref_group: g.all_reduce(buf)
                buf.copy_(x0)
                ms = time_fn(fn, args.warmup, args.iters, world)
                # accuracy of one call vs the exact fp32 sum
                buf.copy_(x0)
                exact = x0.clone()
                dist.all_reduce(exact)
                buf.copy_(x0)
                if impl == "ours":
                    comm.all_reduce(buf, bits=bits, fmt=fmt, algo=algo)
                else:
                    fn()
                torch.cuda.synchronize()
                rel = float((buf - exact).norm() / exact.norm().clamp_min(1e-30))
                rel_t = torch.tensor([rel], device="cuda")
                if world > 1:
                    dist.all_reduce(rel_t, op=dist.ReduceOp.MAX)
                if rank == 0:
                    row = {
                        "impl": impl, "bits": bits, "fmt": fmt, "world": world, "bytes_fp32": n * 4,
                        **({"algo": algo} if algo is not None else {}),
                        "ms": round(ms, 5), "busbw_fp32_equiv_GBs": round(bus_factor * n * 4 / (ms * 1e6), 2),
                        "algbw_GBs": round(n * 4 / (ms * 1e6), 2), "rel_err": float(rel_t.item()),
                        "ef": not args.no_ef and impl == "ours", "sr": not args.no_sr and impl != "nccl",
                        **({"residual_dtype": args.residual_dtype} if impl == "ours" and not args.no_ef else {}),
                        **({"lag": lag} if lag is not None and len(args.lag) > 1 else {}),
                        **({"spi": spi} if spi is not None and len(args.spi) > 1 else {}),
                    }
                    rows.append(row)
                    print(json.dumps(row), flush=True)
        del x0, buf
    dist.barrier()
    sampler.__exit__(None, None, None)
    if rank == 0 and args.out:
        doc = {
            "command": " ".join(sys.argv),
            "world": world,
            "timing": "CUDA events around iters back-to-back calls after warmup calls, max over ranks",
            "clocks": sampler.summary(),
            "rows": rows,
        }
        with open(args.out, "w", encoding="utf-8") as fh:
            json.dump(doc, fh, indent=1)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
