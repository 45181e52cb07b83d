"""GPT-2 medium, sharded data parallel with low-bit gradient reduce-scatter and
low-bit parameter all-gather (the sharded configuration named in BASELINE.json).

24 layers, d_model 1024, 16 heads, vocab 50257, seq 1024; bf16 autocast; 8-bit
reduce-scatter of gradients and 8-bit all-gather of parameters with error
feedback; tokens uniform random in [0, 50257); micro-batch 8 per GPU;
random-init weights; AdamW.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        benchmarks/gpt2_fsdp.py --steps 10 --warmup 3
    ... --comm nccl        # fp32 NCCL reduce-scatter / all-gather (baseline)
    ... --fsdp2            # PyTorch FSDP2 (fully_shard per block) on a `lowbit`
                           # process group (or on NCCL with --comm nccl)

Two sharding engines: ``LowBitShardedDP`` (this library's ZeRO-3-style
wrapper: fp32 master shard per rank, low-bit gradient reduce-scatter and
parameter all-gather once per step) and, with ``--fsdp2``, PyTorch's FSDP2
with ``fully_shard`` on every transformer block and the root: its per-block
all-gathers (prefetched during forward and backward) and gradient
reduce-scatters go through the `lowbit` backend's ``_allgather_base`` /
``_reduce_scatter_base``, i.e. the fused 8-bit kernels, with FSDP2's own
overlap.

Prints one JSON line (rank 0): tokens/s of the whole job, device-timed with
CUDA events, max over ranks, the mean loss of the last timed step, and the
clock record of the timed region.
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

from bitscom_b200.models import gpt2_medium, gpt2_small_test  # noqa: E402
from bitscom_b200.parallel.fsdp import LowBitShardedDP  # noqa: E402


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--micro-batch", type=int, default=8)
    p.add_argument("--seq", type=int, default=1024)
    p.add_argument("--bits", type=int, default=8)
    p.add_argument("--fp8", action="store_true")
    p.add_argument("--comm", choices=["lowbit", "nccl"], default="lowbit")
    p.add_argument("--small", action="store_true", help="4-layer test model")
    p.add_argument("--fsdp2", action="store_true", help="PyTorch FSDP2 fully_shard per block")
    p.add_argument("--fsdp2-comms", choices=["custom", "backend"], default="custom",
                   help="low-bit FSDP2 collectives: per-module custom comms on an NCCL group (error feedback per "
                        "module) or the `lowbit` backend's fused RS/AG under FSDP2's default comms")
    p.add_argument("--no-ef", action="store_true")
    args = p.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29571")
    kw = {} if world > 1 else {"init_method": "tcp://127.0.0.1:%s" % os.environ["MASTER_PORT"], "rank": 0, "world_size": 1}
    lowbit = args.comm == "lowbit"
    if args.fsdp2 and lowbit and args.fsdp2_comms == "backend":
        import bitscom_b200 as bitscom

        bitscom.init(bitwidth=args.bits, error_feedback=not args.no_ef, force_lowbit=True, fp8=args.fp8)
        backend = "lowbit"
    else:
        backend = "nccl"
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local), **kw)

    torch.manual_seed(0)
    model = (gpt2_small_test() if args.small else gpt2_medium()).cuda()
    if args.fsdp2:
        run_fsdp2(model, args, world, rank, lowbit)
        return
    sdp = LowBitShardedDP(
        model,
        lambda ps: torch.optim.AdamW(ps, lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True),
        rs_bits=args.bits if lowbit else 16,
        ag_bits=args.bits if lowbit else 16,
        fp8=args.fp8,
        error_feedback=lowbit,
        use_fused=lowbit,
    )
    vocab = model.cfg.vocab_size
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    pool = [torch.randint(0, vocab, (args.micro_batch, args.seq + 1), device="cuda", generator=g) for _ in range(4)]

    def step(i):
        tok = pool[i % len(pool)]
        with torch.autocast("cuda", dtype=torch.bfloat16):
            _, loss = sdp(tok[:, :-1], tok[:, 1:])
        loss.backward()
        sdp.step()
        return loss

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(args.steps):
        loss = step(i)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    tokens = args.micro_batch * args.seq * world * args.steps
    if rank == 0:
        print(json.dumps({
            "metric": "GPT-2 medium sharded-DP tokens/s", "value": round(tokens / (ms / 1e3), 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
            "dtype": "bf16", "data": "synthetic uniform tokens", "loss": float(loss.item()),
            "config": {"model": "gpt2_small_test" if args.small else "gpt2_medium", "micro_batch": args.micro_batch,
                       "seq_len": args.seq, "comm": f"{args.bits}-bit EF low-bit RS/AG" if lowbit else "fp32 NCCL RS/AG",
                       "fmt": "e4m3" if args.fp8 else "int", "parallelism": f"zero3-dp{world}"},
        }), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def run_fsdp2(model, args, world, rank, lowbit):
    from torch.distributed.device_mesh import DeviceMesh
    from torch.distributed.fsdp import fully_shard

    from bitscom_b200.utils.clocks import ClockSampler

    mesh = DeviceMesh.from_group(dist.group.WORLD, "cuda")
    for blk in model.blocks:
        fully_shard(blk, mesh=mesh)
    fully_shard(model, mesh=mesh)
    comms = None
    if lowbit and args.fsdp2_comms == "custom":
        from bitscom_b200.parallel.fsdp2 import enable_lowbit_fsdp2

        comms = enable_lowbit_fsdp2(model, bits=args.bits, fmt="e4m3" if args.fp8 else "int",
                                    error_feedback=not args.no_ef, group=dist.group.WORLD)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    vocab = model.cfg.vocab_size
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    pool = [torch.randint(0, vocab, (args.micro_batch, args.seq + 1), device="cuda", generator=g) for _ in range(4)]

    def step(i):
        tok = pool[i % len(pool)]
        with torch.autocast("cuda", dtype=torch.bfloat16):
            _, loss = model(tok[:, :-1], tok[:, 1:])
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    with ClockSampler(list(range(world)) if rank == 0 else [int(os.environ.get("LOCAL_RANK", "0"))]) as cs:
        a.record()
        for i in range(args.steps):
            loss = step(i)
        b.record()
        torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    lt = loss.detach().float().view(1)
    dist.all_reduce(lt)
    stats = {}
    if lowbit and comms is None:
        stats = dict(dist.group.WORLD._get_backend(torch.device("cuda")).stats())
    elif comms is not None:
        stats = {"fused_all_gathers": sum(a.fused_calls for a, _ in comms.values()),
                 "fused_reduce_scatters": sum(r.fused_calls for _, r in comms.values()),
                 "fsdp_modules": len(comms)}
    tokens = args.micro_batch * args.seq * world * args.steps
    if rank == 0:
        print(json.dumps({
            "metric": "GPT-2 medium FSDP2 tokens/s", "value": round(tokens / (ms / 1e3), 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
            "dtype": "bf16", "data": "synthetic uniform tokens", "loss": float(lt.item()) / world,
            "clocks": cs.summary(), "backend_stats": stats,
            "config": {"model": "gpt2_small_test" if args.small else "gpt2_medium", "micro_batch": args.micro_batch,
                       "seq_len": args.seq, "engine": "FSDP2 fully_shard per block",
                       "comm": ((f"{args.bits}-bit low-bit RS/AG, " +
                                 ("per-module custom comms" + ("" if args.no_ef else ", EF on gradients")
                                  if comms is not None else "lowbit backend" + ("" if args.no_ef else ", EF")))
                                if lowbit else "fp32 NCCL RS/AG"),
                       "fmt": "e4m3" if args.fp8 else "int", "parallelism": f"fsdp2-dp{world}"},
        }), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
