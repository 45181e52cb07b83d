"""Headline benchmark: DDP training throughput with 4-bit error-feedback
low-bit gradient all-reduce.

Config (the DDP benchmark configuration named in BASELINE.json): ResNet-18 CIFAR-style (3x3 stem, no max-pool,
10-way head), DDP with the low-bit comm hook at 4-bit + error feedback, bf16
autocast, SGD momentum 0.9, synthetic 32x32x3 fp32 images ~N(0,1) with labels
uniform over 10 classes, batch 256 per GPU, seed 0.  Weak scaling: every GPU
trains on its own 256 images per step.

    python bench.py --gpus 1 --steps 20 --warmup 5
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        --master-port 29500 bench.py --gpus 8 --steps 20 --warmup 5
    python bench.py --impl reference ...      # the reference package, same config

Reported (rank 0, one JSON line):
  value      samples/s of the whole job, device-timed with CUDA events over K
             steps with inputs resident on the device (rotating pool larger
             than L2), max over ranks;
  e2e.value  samples/s through the same public API with, every step, an H2D
             copy of the batch from pinned host memory and a D2H read of the
             loss, also device-timed and max over ranks.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import sys
import time

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "DDP samples/s (ResNet-18 CIFAR, 4-bit EF low-bit all-reduce)"
BASELINE_VALUE = None  # the reference publishes no ResNet-18 DDP number
L2_BYTES = 126 * 2**20
POOL = 48  # distinct input batches cycled through (48 x 3 MiB > L2)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--batch", type=int, default=256)
    p.add_argument("--bits", type=int, default=4)
    p.add_argument("--bucket-mb", type=float, default=25.0)
    p.add_argument("--max-ctas", type=int, default=None,
                   help="CTAs of each fused launch (default: the hook's default; 0 = two per SM)")
    p.add_argument("--algo", default="auto", choices=["auto", "oneshot", "twoshot"])
    p.add_argument("--hook", default="lowbit", choices=["lowbit", "none"],
                   help="diagnostic: 'none' runs DDP's own fp32 NCCL all-reduce")
    p.add_argument("--broadcast-buffers", action="store_true",
                   help="broadcast BatchNorm buffers from rank 0 before every forward (DDP's default); off by default "
                        "because the reference's training loop synchronises gradients only")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cudnn-benchmark", action="store_true",
                   help="both arms: keep cuDNN's heuristic algorithm choice (default: benchmark mode)")
    p.add_argument("--eager", action="store_true",
                   help="our arm: run the step eagerly instead of replaying it as one CUDA graph")
    p.add_argument("--ref-path", choices=["ef", "python"], default="ef",
                   help="reference arm: its C++ error-feedback backend path, or its Python LowBitGroup path")
    return p.parse_args()


# ----------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------
def setup(args):
    # Torch-level setting shared by both arms: cuDNN picks the fastest
    # convolution algorithms for these fixed shapes during the warm-up steps.
    torch.backends.cudnn.benchmark = not args.no_cudnn_benchmark
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29517")
    return rank, world, local


# Group used for timing barriers and max-over-ranks reductions: plain NCCL, so
# the reference arm (whose backend implements neither barrier nor MAX) is
# timed the same way as ours.
_AUX = None


def aux_group():
    global _AUX
    if _AUX is None:
        _AUX = dist.new_group(backend="nccl")
    return _AUX


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=aux_group())
    return float(t.item())


def barrier_sync(world):
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(group=aux_group(), device_ids=[torch.cuda.current_device()])
    torch.cuda.synchronize()


def make_data(rank, batch, device):
    g = torch.Generator().manual_seed(0 + rank)
    # Images are stored NHWC (channels-last): the model sees x.permute(0, 3, 1, 2),
    # a channels_last NCHW view, so no layout conversion runs per step.
    xs = torch.randn(POOL, batch, 32, 32, 3, generator=g)
    ys = torch.randint(0, 10, (POOL, batch), generator=g)
    return xs, ys


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------
def build_ours(args, rank, world, local):
    sys.path.insert(0, ROOT)
    import bitscom_b200 as bitscom
    from bitscom_b200.models import resnet18_cifar

    kw = {} if world > 1 else {"init_method": "tcp://127.0.0.1:%s" % os.environ["MASTER_PORT"], "rank": 0, "world_size": 1}
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local), **kw)
    torch.manual_seed(0)
    model = resnet18_cifar(10).cuda().to(memory_format=torch.channels_last)
    # For whole-step graph capture DDP is built on a side stream (PyTorch's
    # capture recipe for DDP); harmless in eager mode.
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ddp = nn.parallel.DistributedDataParallel(
            model, device_ids=[local], bucket_cap_mb=args.bucket_mb, gradient_as_bucket_view=True,
            process_group=dist.group.WORLD,
        )
    torch.cuda.current_stream().wait_stream(side)
    if args.hook == "lowbit":
        extra = {} if args.max_ctas is None else {"max_ctas": args.max_ctas}
        state = bitscom.register_lowbit_hook(ddp, bitwidth=args.bits, error_feedback=True, algo=args.algo, **extra)
    else:  # diagnostic: DDP's own fp32 NCCL all-reduce
        state = bitscom.LowBitHookState()
    ddp.broadcast_buffers = args.broadcast_buffers
    opt = torch.optim.SGD(ddp.parameters(), lr=0.1, momentum=0.9, fused=True)

    def step(x, y):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = F.cross_entropy(ddp(x.permute(0, 3, 1, 2)), y)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=False)
        return loss

    def launches():
        n = 0
        for c in state._comms.values():
            if c is not None:
                n += c.stats()["launches"]
        return n

    _MODEL[0] = model
    _COMMS[0] = state._comms
    return step, launches, "bitscom_b200 DDP comm hook (fused sm_100a NVLink kernel)"


# ----------------------------------------------------------------------------
# reference arm: the unmodified reference package from baseline/_ref
# ----------------------------------------------------------------------------
def build_reference(args, rank, world, local):
    ref_path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_path, "bitscom")):
        return None, None, "reference not installed in baseline/_ref"
    sys.path.insert(0, ref_path)
    import bitscom  # the reference package
    import torchvision

    kw = {} if world > 1 else {"init_method": "tcp://127.0.0.1:%s" % os.environ["MASTER_PORT"], "rank": 0, "world_size": 1}
    if args.ref_path == "ef":
        # The reference's error-feedback path: its C++ `lowbit` backend with
        # error_feedback=True, reached through dist.all_reduce (reference
        # README; cpp/src/process_group_lowbit.cc:153-328).  DDP cannot drive
        # it (its Work future completes before the second phase), so
        # gradients go through persistent flat buckets — persistent so the
        # residual, keyed by tensor identity, carries across steps — padded to
        # a multiple of the world size as that path requires.
        bitscom.init(bitwidth=args.bits, error_feedback=True)
        dist.init_process_group("lowbit", timeout=datetime.timedelta(seconds=120), **kw)
        group = None
    else:
        # The reference's Python path: LowBitGroup over an NCCL group (no EF).
        from bitscom.api import LowBitGroup

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), **kw)
        group = LowBitGroup(bitwidth=args.bits, process_group=dist.group.WORLD)
    torch.manual_seed(0)
    model = torchvision.models.resnet18(num_classes=10)
    model.conv1 = nn.Conv2d(3, 64, 3, 1, 1, bias=False)
    model.maxpool = nn.Identity()
    model = model.cuda().to(memory_format=torch.channels_last)
    for p in model.parameters():  # same initial weights on every rank
        dist.broadcast(p.data, 0)
    # Same torch optimizer settings as our arm (fused SGD is a torch choice,
    # not library work).
    opt = torch.optim.SGD(model.parameters(), lr=0.1, momentum=0.9, fused=True)
    cap = int(args.bucket_mb * 2**20 / 4)
    params = [p for p in model.parameters()]
    buckets, cur, size = [], [], 0
    for p in reversed(params):  # gradient-ready order, as DDP buckets them
        if cur and size + p.numel() > cap:
            buckets.append(cur)
            cur, size = [], 0
        cur.append(p)
        size += p.numel()
    if cur:
        buckets.append(cur)
    flats = []
    for b in buckets:
        n = sum(p.numel() for p in b)
        flats.append(torch.zeros(n + (-n) % world, device="cuda"))

    def sync_grads():
        for b, flat in zip(buckets, flats):
            off = 0
            for p in b:
                flat[off : off + p.numel()].copy_(p.grad.reshape(-1))
                off += p.numel()
            if group is None:
                dist.all_reduce(flat)  # synchronous: waits on the reference's Work (runs its second phase)
            else:
                group.all_reduce(flat, async_op=False)
            flat.div_(world)
            off = 0
            for p in b:
                p.grad.copy_(flat[off : off + p.numel()].view(p.grad.shape))
                off += p.numel()

    def step(x, y):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = F.cross_entropy(model(x.permute(0, 3, 1, 2)), y)
        loss.backward()
        sync_grads()
        opt.step()
        opt.zero_grad(set_to_none=False)
        return loss

    _MODEL[0] = model
    desc = ("reference bitscom lowbit backend, error feedback, dist.all_reduce per persistent bucket after backward"
            if group is None else "reference bitscom LowBitGroup over NCCL, bucketed after backward (no EF)")
    return step, (lambda: 0), desc


_MODEL = [None]  # the trained module of the arm (for the replica check)
_COMMS = [None]  # our arm: the hook's communicators (for kernel timing)


def replicas_identical(world: int):
    """After the run: do all ranks hold bit-identical parameters?  (float64
    sum and sum of squares of every parameter, gathered over ranks.)"""
    if world == 1 or _MODEL[0] is None:
        return None
    with torch.no_grad():
        v = torch.stack([torch.stack([p.double().sum(), p.double().square().sum()]) for p in _MODEL[0].parameters()])
    allv = [torch.empty_like(v) for _ in range(world)]
    dist.all_gather(allv, v, group=aux_group())
    return bool(all(torch.equal(allv[0], a) for a in allv[1:]))


def fused_kernel_ms(step, xs_dev, ys_dev, n, world):
    """Device time of the fused collective launches per eager step (CUDA
    events around every launch), over n untimed steps; max over ranks."""
    comms = [c for c in (_COMMS[0] or {}).values() if c is not None]
    if not comms:
        return None
    for c in comms:
        c.native.reset_stats()
        c.set_timing(True)
    for i in range(n):
        step(xs_dev[i % POOL], ys_dev[i % POOL])
    torch.cuda.synchronize()
    ms = 0.0
    for c in comms:
        st = c.stats()
        ms += st["kernel_ms"]
        c.set_timing(False)
    return max_over_ranks(ms / n, world)


# ----------------------------------------------------------------------------
def timed(step, xs_dev, ys_dev, steps, world, e2e_host=None, bufs=None):
    """Device-timed K steps; with e2e_host=(xs_pinned, ys_pinned) each step
    copies its batch H2D from pinned memory (into `bufs`, e.g. a captured
    graph's static inputs) and reads the loss back D2H."""
    loss_host = torch.empty(steps, dtype=torch.float32, pin_memory=True)
    xbuf, ybuf = bufs if bufs is not None else (torch.empty_like(xs_dev[0]), torch.empty_like(ys_dev[0]))
    barrier_sync(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(steps):
        j = i % POOL
        if e2e_host is not None:
            xbuf.copy_(e2e_host[0][j], non_blocking=True)
            ybuf.copy_(e2e_host[1][j], non_blocking=True)
            loss = step(xbuf, ybuf)
            loss_host[i : i + 1].copy_(loss.detach().float().view(1), non_blocking=True)
        else:
            step(xs_dev[j], ys_dev[j])
    t1.record()
    barrier_sync(world)
    ms = t0.elapsed_time(t1)
    if e2e_host is not None:
        assert torch.isfinite(loss_host).all(), "non-finite loss"
    return ms, loss_host


def main():
    args = parse()
    rank, world, local = setup(args)
    if args.impl == "reference":
        try:
            step, launches, desc = build_reference(args, rank, world, local)
        except Exception as exc:  # pragma: no cover - depends on the reference build
            step, desc = None, f"reference failed to start: {exc!r}"[:300]
        if step is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": desc}))
            return
    else:
        step, launches, desc = build_ours(args, rank, world, local)

    xs, ys = make_data(rank, args.batch, "cuda")
    xs_dev, ys_dev = xs.cuda(), ys.cuda()
    xs_pin, ys_pin = xs.pin_memory(), ys.pin_memory()

    # Clock samples (nvidia-smi, every 100 ms) from the warm-up steps through
    # the timed regions: the same workload runs throughout, and a timed
    # region of a few steps alone can end before the first sample.
    from bitscom_b200.utils.clocks import ClockSampler

    cs = ClockSampler(list(range(world)) if rank == 0 else [local], period_ms=100).__enter__()
    graph = args.impl == "ours" and not args.eager and args.hook == "lowbit"
    bufs = None
    kernel_ms = None
    per_step_launches = None
    if graph:
        # Whole-step CUDA graph (forward, backward with the fused all-reduce
        # launches of the DDP hook, optimizer): eager DDP warm-up on a side
        # stream, then one capture.  Untimed.
        from bitscom_b200.parallel.graphs import DDP_EAGER_WARMUP, GraphedStep

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(DDP_EAGER_WARMUP):
                step(xs_dev[i % POOL], ys_dev[i % POOL])
            # Fused-kernel device time per step, from eager warm-up steps
            # (launches inside a replayed graph are not timed).
            kernel_ms = fused_kernel_ms(step, xs_dev, ys_dev, 5, world)
        torch.cuda.current_stream().wait_stream(side)
        barrier_sync(world)
        la = launches()
        try:
            gstep = GraphedStep(step, [xs_dev[0], ys_dev[0]], warmup=0)
            ok = 1.0
        except Exception as exc:  # keep the run alive: every rank falls back to the eager step
            print(f"[bench] CUDA-graph capture failed ({exc!r}); timing the eager step", file=sys.stderr)
            gstep, ok = None, 0.0
        ok = -max_over_ranks(-ok, world)  # min over ranks
        if ok > 0:
            step = gstep
            per_step_launches = launches() - la
            bufs = tuple(step.static_inputs)
            desc += ", whole step replayed as one CUDA graph"
        else:
            graph = False

    for i in range(args.warmup):
        step(xs_dev[i % POOL], ys_dev[i % POOL])
    barrier_sync(world)

    l0 = launches()
    ms, _ = timed(step, xs_dev, ys_dev, args.steps, world)
    l1 = launches()
    if per_step_launches is not None:  # replays do not pass through the host
        l1 = l0 + per_step_launches * args.steps
    ms = max_over_ranks(ms, world)
    e2e = None
    if not args.no_e2e:
        ms_e2e, _ = timed(step, xs_dev, ys_dev, args.steps, world, e2e_host=(xs_pin, ys_pin), bufs=bufs)
        ms_e2e = max_over_ranks(ms_e2e, world)
        img_bytes = xs[0].numel() * xs.element_size() + ys[0].numel() * ys.element_size()
        e2e = {
            "value": round(args.batch * world * args.steps / (ms_e2e / 1e3), 2),
            "unit": "samples/s",
            "ms_per_step": round(ms_e2e / args.steps, 4),
            "h2d_bytes_per_step": int(img_bytes),
            "d2h_bytes_per_step": 4,
        }
    if args.impl == "ours" and not graph and args.hook == "lowbit":
        kernel_ms = fused_kernel_ms(step, xs_dev, ys_dev, 5, world)
    identical = replicas_identical(world)
    value = args.batch * world * args.steps / (ms / 1e3)
    cs.__exit__(None, None, None)
    clocks = cs.summary()
    if rank == 0:
        out = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "samples/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": (round(value / BASELINE_VALUE, 4) if BASELINE_VALUE else None),
            "dtype": "bf16",
            "data": "synthetic (N(0,1) 32x32x3 images, uniform labels; random-init weights)",
            "config": {
                "model": "resnet18_cifar",
                "global_batch": args.batch * world,
                "per_gpu_batch": args.batch,
                "seq_len": None,
                "image": [3, 32, 32],
                "parallelism": f"dp{world}",
                "comm": (f"{args.bits}-bit error-feedback low-bit all-reduce, {args.bucket_mb} MB buckets"
                         if args.hook == "lowbit" or args.impl == "reference"
                         else f"fp32 NCCL all-reduce (diagnostic), {args.bucket_mb} MB buckets"),
                "optimizer": "SGD momentum 0.9 (fused)",
                "cudnn_benchmark": not args.no_cudnn_benchmark,
                "buffer_sync": ("DDP broadcast of BatchNorm buffers every forward" if args.broadcast_buffers
                                else "none (gradients only, as in the reference's loop)"),
                "l2": f"rotating pool of {POOL} device-resident batches ({POOL * 3} MiB > 126 MiB L2)",
                "implementation": desc,
                "cuda_graph": graph,
            },
            "clocks": {"sm_mhz": clocks.get("sm_mhz"), "sm_max_mhz": clocks.get("sm_max_mhz"), "reasons": clocks.get("reasons")},
            "gpu_launches": int(l1 - l0),
        }
        if kernel_ms is not None:
            out["fused_kernel_ms_per_step"] = round(kernel_ms, 4)
            out["fused_kernel_ms_note"] = "device time of the fused all-reduce launches of one eager step (CUDA events), max over ranks"
        if identical is not None:
            out["replicas_identical"] = identical
        if args.impl == "reference":
            out["impl"] = "reference"
        if e2e is not None:
            out["e2e"] = e2e
        print(json.dumps(out), flush=True)
    if dist.is_initialized():
        if world > 1:
            dist.barrier(group=aux_group(), device_ids=[torch.cuda.current_device()])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
