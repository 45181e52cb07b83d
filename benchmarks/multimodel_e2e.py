"""Multi-model end-to-end training: ResNet-50, BERT, GPT-2 with low-bit
gradient all-reduce (no SR / SR) vs fp32 NCCL.

Counterpart of reference benchmarks/multimodel_stochastic_e2e_curve.py
(published: multimodel_*_loss_curve_bw4.csv, multimodel_throughput_summary_bw4.csv).
Differences by design: gradients go through the DDP comm hook (one fused
kernel per bucket, overlapped with backward) instead of a hand-built bucket
loop after backward (`--sync bucketed` restores that loop with persistent
buckets, GradBucketer over LowBitGroup.all_reduce); the no-compression mode
is a real fp32 all-reduce;
timing is device-side (CUDA events, max over ranks).

The ResNet-50 configuration named in BASELINE.json (ResNet-50 ImageNet shape, 2-bit EF + SR, 25 MB buckets,
batch 128/GPU):

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        benchmarks/multimodel_e2e.py --models resnet50 --bitwidth 2 --modes lowbit_sr \
        --batch 128 --image 224 --num-classes 1000 --steps 20

Options: --profile-trace DIR writes a Chrome trace of a few steps per run
(analyse with benchmarks/analyze_trace.py).
"""

from __future__ import annotations

import argparse
import csv
import datetime
import json
import math
import os
import sys

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bitscom_b200 as bitscom  # noqa: E402
from bitscom_b200.models import gpt2_small_test, resnet50  # noqa: E402


def build(name, args):
    if name == "resnet50":
        return resnet50(args.num_classes).to(memory_format=torch.channels_last)
    if name == "gpt2":
        return gpt2_small_test(n_positions=max(512, args.seq))
    if name == "bert":
        from transformers import BertConfig, BertForSequenceClassification

        cfg = BertConfig(vocab_size=30522, hidden_size=256, num_hidden_layers=4, num_attention_heads=4,
                         intermediate_size=1024, max_position_embeddings=512, num_labels=2)
        return BertForSequenceClassification(cfg)
    raise ValueError(name)


def batches(name, args, rank, device):
    g = torch.Generator(device="cpu").manual_seed(17 + 10_000 * rank)
    out = []
    for _ in range(8):
        if name == "resnet50":
            y = torch.randint(0, args.num_classes, (args.batch,), generator=g)
            x = torch.randn(args.batch, 3, args.image, args.image, generator=g)
            out.append((x.to(device).contiguous(memory_format=torch.channels_last), y.to(device)))
        elif name == "bert":
            ids = torch.randint(0, 30522, (args.batch, args.seq), generator=g)
            lab = torch.randint(0, 2, (args.batch,), generator=g)
            ids[:, 0] = lab + 101  # learnable cue
            out.append((ids.to(device), lab.to(device)))
        else:
            start = torch.randint(0, 512, (args.batch, 1), generator=g)
            ids = (start + torch.arange(args.seq + 1).unsqueeze(0)) % 512
            out.append((ids.to(device), None))
    return out


def loss_of(name, model, batch):
    x, y = batch
    if name == "resnet50":
        return F.cross_entropy(model(x), y)
    if name == "bert":
        return model(input_ids=x, labels=y).loss
    _, loss = model(x[:, :-1], x[:, 1:])
    return loss


def run(name, mode, args, rank, world, device):
    torch.manual_seed(args.seed)
    model = build(name, args).to(device)
    ddp = nn.parallel.DistributedDataParallel(model, device_ids=[device.index], bucket_cap_mb=args.bucket_mb,
                                              gradient_as_bucket_view=True)
    bucketer = None
    if mode != "no_compression":
        sr = mode == "lowbit_sr"
        if args.sync == "ddp_hook":
            bitscom.register_lowbit_hook(ddp, bitwidth=args.bitwidth, error_feedback=not args.no_ef,
                                         stochastic_rounding=sr)
        else:
            from bitscom_b200.parallel.bucketing import GradBucketer

            group = bitscom.LowBitGroup(bitwidth=args.bitwidth, stochastic_rounding=sr, error_feedback=not args.no_ef)
            bucketer = GradBucketer(model.parameters(), group, bucket_mb=args.bucket_mb)
    opt = torch.optim.AdamW(model.parameters(), lr=args.lr, weight_decay=0.01, fused=True)
    warm = max(1, int(args.steps * 0.1))
    sched = torch.optim.lr_scheduler.LambdaLR(
        opt, lambda s: (s + 1) / warm if s < warm else 0.1 + 0.45 * (1 + math.cos(math.pi * (s - warm) / max(1, args.steps - warm))))
    data = batches(name, args, rank, device)
    losses = []
    prof = None
    if args.profile_trace and rank == 0:
        prof = torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA],
                                      schedule=torch.profiler.schedule(wait=1, warmup=1, active=3, repeat=1))
        prof.__enter__()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    for step in range(args.steps):
        if step == args.warmup:
            torch.cuda.synchronize()
            dist.barrier()
            a.record()
        batch = data[step % len(data)]
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = loss_of(name, ddp if bucketer is None else model, batch)
        loss.backward()
        if bucketer is not None:  # reference-style: backward without DDP, then bucketed low-bit all-reduce
            bucketer.sync()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        sched.step()
        opt.zero_grad(set_to_none=False)
        losses.append(loss.detach().float())
        if prof is not None:
            prof.step()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / max(1, args.steps - args.warmup)
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if prof is not None:
        prof.__exit__(None, None, None)
        os.makedirs(args.profile_trace, exist_ok=True)
        prof.export_chrome_trace(os.path.join(args.profile_trace, f"trace_{name}_{mode}_bw{args.bitwidth}.json"))
    lt = torch.stack(losses)
    dist.all_reduce(lt)
    return (lt / world).tolist(), float(t.item())


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--models", nargs="+", default=["resnet50", "bert", "gpt2"], choices=["resnet50", "bert", "gpt2"])
    p.add_argument("--modes", nargs="+", default=["lowbit_no_sr", "lowbit_sr", "no_compression"])
    p.add_argument("--bitwidth", type=int, default=4)
    p.add_argument("--no-ef", action="store_true")
    p.add_argument("--sync", choices=["ddp_hook", "bucketed"], default="ddp_hook")
    p.add_argument("--steps", type=int, default=40)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--image", type=int, default=224)
    p.add_argument("--num-classes", type=int, default=20)
    p.add_argument("--seq", type=int, default=64)
    p.add_argument("--bucket-mb", type=float, default=25.0)
    p.add_argument("--lr", type=float, default=2e-4)
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--out-dir", default=None)
    p.add_argument("--profile-trace", default=None)
    args = p.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29591")
    kw = {} if world > 1 else {"init_method": "tcp://127.0.0.1:%s" % os.environ["MASTER_PORT"], "rank": 0, "world_size": 1}
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device, **kw)
    summary = []
    for name in args.models:
        curves = {}
        for mode in args.modes:
            losses, ms = run(name, mode, args, rank, world, device)
            curves[mode] = losses
            sps = args.batch * world / (ms / 1e3)
            summary.append({"model": name, "method": mode, "avg_step_time_ms": ms, "throughput_samples_per_s": sps,
                            "final_loss": losses[-1]})
            if rank == 0:
                print(json.dumps(summary[-1]), flush=True)
        if rank == 0 and args.out_dir:
            os.makedirs(args.out_dir, exist_ok=True)
            with open(os.path.join(args.out_dir, f"multimodel_{name}_loss_curve_bw{args.bitwidth}.csv"), "w", newline="") as fh:
                w = csv.writer(fh)
                w.writerow(["step"] + [f"loss_{m}" for m in args.modes])
                for i in range(args.steps):
                    w.writerow([i + 1] + [curves[m][i] for m in args.modes])
    if rank == 0 and args.out_dir:
        with open(os.path.join(args.out_dir, f"multimodel_throughput_summary_bw{args.bitwidth}.csv"), "w", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=list(summary[0]))
            w.writeheader()
            w.writerows(summary)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
