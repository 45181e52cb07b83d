"""Stochastic-rounding end-to-end curve: TinyMLP trained with low-bit gradient
all-reduce without SR, with SR, and without compression.

Counterpart of reference benchmarks/stochastic_rounding_e2e_curve.py
(published: benchmarks/outputs/e2e_loss_curve_stochastic_vs_nocompress_bw4.csv).
Same workload as that script, so the curves compare: TinyMLP 256-512-512-10;
each rank owns a fixed dataset of 8192 N(0,1) inputs (generator seed
data_seed + 100000 * rank) labelled by the argmax of one linear teacher shared
by all ranks (seed data_seed + 9999); batches of 128 are read sequentially
with wrap-around; per-parameter LowBitGroup.all_reduce and division by the
world size; SGD momentum 0.9, lr 0.05, gradient clipping 1.0.  The "no
compression" run here is a real fp32 all-reduce (the reference's ran its
4-bit C++ path).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        benchmarks/stochastic_rounding_e2e.py --bitwidth 4 --steps 160 --out curve.csv
"""

from __future__ import annotations

import argparse
import csv
import datetime
import os
import sys

import torch
import torch.distributed as dist
import torch.nn as nn

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bitscom_b200 import LowBitGroup  # noqa: E402
from bitscom_b200.models import tiny_mlp_sr  # noqa: E402


def local_dataset(args, rank):
    """Fixed per-rank inputs labelled by a linear teacher common to all ranks."""
    g = torch.Generator(device="cpu").manual_seed(args.data_seed + 100_000 * rank)
    tg = torch.Generator(device="cpu").manual_seed(args.data_seed + 9999)
    x = torch.randn(args.dataset_size, 256, generator=g)
    w = torch.randn(256, 10, generator=tg)
    b = torch.randn(10, generator=tg)
    return x, torch.argmax(x @ w + b, dim=1)


def batch_at(step, args, data, device):
    x, y = data
    n = x.size(0)
    idx = (torch.arange(args.batch) + (step * args.batch) % n) % n
    return x[idx].to(device), y[idx].to(device)


def run(mode, args, rank, world, device):
    torch.manual_seed(args.seed)
    model = tiny_mlp_sr().to(device)
    opt = torch.optim.SGD(model.parameters(), lr=args.lr, momentum=0.9)
    group = None
    if mode != "nocompress":
        group = LowBitGroup(bitwidth=args.bitwidth, stochastic_rounding=(mode == "sr"))
    data = local_dataset(args, rank)
    losses = []
    for step in range(args.steps):
        x, y = batch_at(step, args, data, device)
        loss = nn.functional.cross_entropy(model(x), y)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        for p in model.parameters():
            if group is None:
                dist.all_reduce(p.grad)
            else:
                group.all_reduce(p.grad)
            p.grad.div_(world)
        if args.grad_clip_norm > 0:
            torch.nn.utils.clip_grad_norm_(model.parameters(), args.grad_clip_norm)
        opt.step()
        lt = loss.detach().clone()
        dist.all_reduce(lt)
        losses.append(float(lt.item()) / world)
    return losses


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--bitwidth", type=int, default=4)
    p.add_argument("--steps", type=int, default=160)
    p.add_argument("--batch", type=int, default=128)
    p.add_argument("--lr", type=float, default=0.05)
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--data-seed", type=int, default=7)
    p.add_argument("--dataset-size", type=int, default=8192)
    p.add_argument("--grad-clip-norm", type=float, default=1.0)
    p.add_argument("--out", default=None)
    args = p.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(local)
    device = torch.device("cuda", local) if cuda else torch.device("cpu")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29581")
    kw = {} if world > 1 else {"init_method": "tcp://127.0.0.1:%s" % os.environ["MASTER_PORT"], "rank": 0, "world_size": 1}
    dist.init_process_group("nccl" if cuda else "gloo", timeout=datetime.timedelta(seconds=120), **kw)
    curves = {m: run(m, args, rank, world, device) for m in ("nosr", "sr", "nocompress")}
    if rank == 0:
        last = {m: c[-1] for m, c in curves.items()}
        print(f"bw={args.bitwidth} world={world} loss@{args.steps}: no-SR={last['nosr']:.4f} "
              f"SR={last['sr']:.4f} fp32={last['nocompress']:.4f}")
        if args.out:
            with open(args.out, "w", newline="") as fh:
                w = csv.writer(fh)
                w.writerow(["step", "loss_lowbit_no_sr", "loss_lowbit_sr", "loss_no_compression"])
                for i in range(args.steps):
                    w.writerow([i + 1, curves["nosr"][i], curves["sr"][i], curves["nocompress"][i]])
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
