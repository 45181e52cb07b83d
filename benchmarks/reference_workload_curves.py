"""Loss curves on the reference's own multi-model workloads, on GPUs.

The reference publishes BERT and GPT-2 loss curves of its 4-bit low-bit
all-reduce at world size 2 (benchmarks/outputs/multimodel_{bert,gpt2}_loss_
curve_bw4.csv, produced by benchmarks/multimodel_stochastic_e2e_curve.py).
A loss curve only compares on the same workload, so this script rebuilds
that workload with the same settings (the steps below follow the
reference's script; the code is this repository's own):

* models: Hugging Face ``GPT2LMHeadModel`` (vocab 50257, 256 hidden, 4
  layers, 4 heads, 512 positions) and ``BertForSequenceClassification``
  (vocab 30522, 256 hidden, 4 layers, 4 heads, 1024 intermediate, 2 labels),
  one model per mode, built one after another from seed 2026;
* data, per rank: GPT-2 sequences ``(start + arange(64)) % 512`` with
  ``start`` uniform in [0, 512); BERT uniform token ids with the label
  written into position 0 as token ``label + 101``; 1024 samples per rank
  (CPU generator seeded ``17 + rank * 30000`` / ``17 + rank * 20000``), read
  in order, 4 samples per step;
* training: fp32, AdamW (betas 0.9/0.999, eps 1e-8, weight decay 0.01;
  lr 2e-4 GPT-2, 2.5e-4 BERT), linear warm-up over 8 % of the steps then a
  cosine decay to 5 % of the lr, gradient clipping at 0.8; after backward
  the gradients are all-reduced in flat buckets of up to 4,000,000 elements
  (``GradBucketer`` over ``LowBitGroup.all_reduce``) and divided by the
  world size; the logged loss is the mean over ranks.

Modes: ``lowbit_no_sr`` / ``lowbit_sr`` (4-bit, no error feedback: the
reference's LowBitGroup path has none), ``lowbit_ef`` (4-bit with error
feedback), ``no_compression`` (fp32 NCCL all-reduce).  Our 4-bit all-reduce
is the fused kernel with 1024-element block scales; the reference's uses one
scale per rank and tensor.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        benchmarks/reference_workload_curves.py --models gpt2 bert --steps 240 --out-dir outputs
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

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bitscom_b200 import LowBitGroup  # noqa: E402
from bitscom_b200.parallel.bucketing import GradBucketer  # noqa: E402

MODES = ["lowbit_no_sr", "lowbit_sr", "no_compression", "lowbit_ef"]
LR = {"gpt2": 2e-4, "bert": 2.5e-4}


def build_model(name):
    if name == "gpt2":
        from transformers import GPT2Config, GPT2LMHeadModel

        return GPT2LMHeadModel(GPT2Config(vocab_size=50257, n_embd=256, n_layer=4, n_head=4, n_positions=512))
    from transformers import BertConfig, BertForSequenceClassification

    return BertForSequenceClassification(BertConfig(
        vocab_size=30522, hidden_size=256, num_hidden_layers=4, num_attention_heads=4, intermediate_size=1024,
        max_position_embeddings=512, num_labels=2))


def build_data(name, rank, size=1024, seq=64, base_seed=17):
    g = torch.Generator(device="cpu")
    if name == "gpt2":
        g.manual_seed(base_seed + rank * 30_000)
        starts = torch.randint(0, 512, (size, 1), generator=g, dtype=torch.int64)
        ids = (starts + torch.arange(seq, dtype=torch.int64).unsqueeze(0)) % 512
        return {"input_ids": ids, "attention_mask": torch.ones(size, seq, dtype=torch.int64)}
    g.manual_seed(base_seed + rank * 20_000)
    ids = torch.randint(0, 30522, (size, seq), generator=g, dtype=torch.int64)
    labels = torch.randint(0, 2, (size,), generator=g, dtype=torch.int64)
    ids[:, 0] = labels + 101
    return {"input_ids": ids, "attention_mask": torch.ones(size, seq, dtype=torch.int64), "labels": labels}


def batch_at(data, step, bs):
    n = next(iter(data.values())).size(0)
    s = ((step - 1) * bs) % n
    out = {}
    for k, v in data.items():
        out[k] = v[s:s + bs] if s + bs <= n else torch.cat([v[s:], v[: s + bs - n]])
    return out


def train(name, mode, model, data, args, world, device):
    model.train().to(device)
    group = None
    if mode != "no_compression":
        group = LowBitGroup(bitwidth=args.bitwidth, stochastic_rounding=(mode == "lowbit_sr"),
                            error_feedback=(mode == "lowbit_ef"))
    opt = torch.optim.AdamW(model.parameters(), lr=LR[name], betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    warm = max(1, int(args.steps * 0.08))

    def lr_at(i):
        if i < warm:
            return (i + 1) / warm
        prog = (i - warm) / max(1, args.steps - warm)
        return 0.05 + 0.95 * 0.5 * (1.0 + math.cos(math.pi * prog))

    sched = torch.optim.lr_scheduler.LambdaLR(opt, lr_at)
    bucketer = None if group is None else GradBucketer(model.parameters(), group, bucket_mb=4_000_000 * 4 / 2**20)
    losses = []
    for step in range(1, args.steps + 1):
        b = {k: v.to(device, non_blocking=True) for k, v in batch_at(data, step, args.batch).items()}
        opt.zero_grad(set_to_none=False)
        if name == "gpt2":
            loss = model(input_ids=b["input_ids"], attention_mask=b["attention_mask"], labels=b["input_ids"]).loss
        else:
            loss = model(input_ids=b["input_ids"], attention_mask=b["attention_mask"], labels=b["labels"]).loss
        loss.backward()
        if group is None:
            for p in model.parameters():
                if p.grad is not None:
                    dist.all_reduce(p.grad)
                    p.grad.div_(world)
        else:
            bucketer.sync()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 0.8)
        opt.step()
        sched.step()
        lt = loss.detach().float().view(1)
        dist.all_reduce(lt)
        losses.append(float(lt.item()) / world)
    return losses


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--models", nargs="+", default=["gpt2", "bert"], choices=["gpt2", "bert"])
    p.add_argument("--modes", nargs="+", default=MODES, choices=MODES)
    p.add_argument("--bitwidth", type=int, default=4)
    p.add_argument("--steps", type=int, default=240)
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--out-dir", default=None)
    args = p.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    for name in args.models:
        torch.manual_seed(args.seed)
        torch.cuda.manual_seed_all(args.seed)
        models = {m: build_model(name) for m in MODES}  # built in mode order from one seed
        data = build_data(name, rank)
        curves = {}
        for mode in args.modes:
            curves[mode] = train(name, mode, models[mode], data, args, world, device)
            if rank == 0:
                print(json.dumps({"model": name, "mode": mode, "bitwidth": args.bitwidth, "world": world,
                                  "final_loss": curves[mode][-1], "steps": args.steps}), flush=True)
        if rank == 0 and args.out_dir:
            os.makedirs(args.out_dir, exist_ok=True)
            path = os.path.join(args.out_dir, f"refworkload_{name}_loss_curve_bw{args.bitwidth}.csv")
            with open(path, "w", newline="") as fh:
                w = csv.writer(fh)
                w.writerow(["step"] + [f"loss_{m}" for m in args.modes])
                for i in range(args.steps):
                    w.writerow([i + 1] + [curves[m][i] for m in args.modes])
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
