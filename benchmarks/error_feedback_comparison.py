"""Error-feedback benefit: cumulative quantisation error and TinyMLP training.

Counterpart of reference benchmarks/error_feedback_comparison.py (published
curves: benchmarks/outputs/ef_benefit_curve_bw{2,4,8}.csv and
ef_training_curve_bw{2,4,8}.csv).

(a) cumulative-error curve: each step draws g ~ N(0, 0.05^2) of `vec_size`
    elements; the no-EF path accumulates dequant(quant(g)), the EF path
    accumulates dequant(quant(g + r)) and carries r; reported is
    ||sum_hat - sum|| / ||sum|| per step.
(b) TinyMLP (64-128-128-10), SGD, gradients quantised in place per parameter
    with / without EF.

Uses the fused ef_roundtrip kernel on CUDA (one pass: add residual, quantise,
dequantise, write residual; the reference's per-tensor scale) and the
identical CPU path otherwise.  With ``--fused`` the roundtrip is instead the
fused all-reduce's own encode (1024-element block scales) on a one-rank
communicator (one-shot: one quantisation with the residual, then decode), and
``--residual-dtype bfloat16`` stores that residual in bf16, so the EF curves
of the collective's fp32 and bf16 residuals can be compared (CUDA only).

    python benchmarks/error_feedback_comparison.py --bitwidth 4 --out-dir outputs
    python benchmarks/error_feedback_comparison.py --bitwidth 4 --fused --residual-dtype bfloat16
"""

from __future__ import annotations

import argparse
import csv
import os
import sys

import torch
import torch.nn as nn

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bitscom_b200.models import TinyMLP  # noqa: E402
from bitscom_b200.quantization import ef_roundtrip as _ef_roundtrip_ref  # noqa: E402

_FUSED = {"comm": None, "res_dtype": torch.float32}


def ef_roundtrip(g, residual, bits):
    """dequant(quant(g + residual)), residual updated in place when given."""
    comm = _FUSED["comm"]
    if comm is None:
        return _ef_roundtrip_ref(g, residual, bits)
    out = torch.empty_like(g)
    comm.all_reduce(g.contiguous(), out=out, bits=bits, residual=residual, algo="oneshot")
    return out


def new_residual(n, device):
    return torch.zeros(n, device=device, dtype=_FUSED["res_dtype"])


def ef_benefit_curve(device, bits, steps, vec_size, seed):
    torch.manual_seed(seed)
    true_cum = torch.zeros(vec_size, device=device)
    noef_cum = torch.zeros_like(true_cum)
    ef_cum = torch.zeros_like(true_cum)
    res = new_residual(vec_size, device)
    rows = []
    for step in range(1, steps + 1):
        g = torch.randn(vec_size, device=device) * 0.05
        true_cum += g
        noef_cum += ef_roundtrip(g, None, bits)
        ef_cum += ef_roundtrip(g, res, bits)
        d = true_cum.norm().item() + 1e-12
        rows.append((step, (noef_cum - true_cum).norm().item() / d, (ef_cum - true_cum).norm().item() / d))
    return rows


def toy_batch(batch, device):
    x = torch.randn(batch, 64, device=device)
    w = torch.linspace(-1.0, 1.0, 64, device=device).unsqueeze(1).repeat(1, 10)
    return x, torch.argmax(x @ w, dim=1)


def train(device, bits, steps, lr, batch, seed, use_ef):
    torch.manual_seed(seed)
    model = TinyMLP().to(device)
    opt = torch.optim.SGD(model.parameters(), lr=lr)
    crit = nn.CrossEntropyLoss()
    res = {}
    losses = []
    for _ in range(steps):
        x, y = toy_batch(batch, device)
        opt.zero_grad(set_to_none=True)
        loss = crit(model(x), y)
        loss.backward()
        with torch.no_grad():
            for i, p in enumerate(model.parameters()):
                r = None
                if use_ef:
                    r = res.setdefault(i, new_residual(p.numel(), device))
                p.grad.copy_(ef_roundtrip(p.grad.reshape(-1), r, bits).view_as(p.grad))
        opt.step()
        losses.append(float(loss.item()))
    return losses


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--bitwidth", type=int, default=2)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--vec-size", type=int, default=1 << 20)
    p.add_argument("--train-steps", type=int, default=160)
    p.add_argument("--batch-size", type=int, default=256)
    p.add_argument("--lr", type=float, default=0.05)
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    p.add_argument("--out-dir", default=None)
    p.add_argument("--fused", action="store_true", help="the fused collective's block-scaled encode (CUDA)")
    p.add_argument("--residual-dtype", default="float32", choices=["float32", "bfloat16"])
    args = p.parse_args()
    dev = torch.device(args.device)
    if args.fused:
        from bitscom_b200.parallel.comm import Communicator

        _FUSED["comm"] = Communicator.create_local(dev.index or 0)
        _FUSED["res_dtype"] = getattr(torch, args.residual_dtype)
    elif args.residual_dtype != "float32":
        raise SystemExit("--residual-dtype needs --fused")
    rows = ef_benefit_curve(dev, args.bitwidth, args.steps, args.vec_size, args.seed)
    l0 = train(dev, args.bitwidth, args.train_steps, args.lr, args.batch_size, args.seed, False)
    l1 = train(dev, args.bitwidth, args.train_steps, args.lr, args.batch_size, args.seed, True)
    last = rows[min(len(rows), 160) - 1]
    tag = f"fused_{args.residual_dtype}_" if args.fused else ""
    print(f"{tag}bw={args.bitwidth} rel. cumulative error @{last[0]}: noEF={last[1]:.4g} EF={last[2]:.4g}; "
          f"TinyMLP loss @{len(l0)}: noEF={l0[-1]:.4g} EF={l1[-1]:.4g}")
    if args.out_dir:
        os.makedirs(args.out_dir, exist_ok=True)
        with open(os.path.join(args.out_dir, f"{tag}ef_benefit_curve_bw{args.bitwidth}.csv"), "w", newline="") as fh:
            w = csv.writer(fh)
            w.writerow(["step", "noef_rel_error", "ef_rel_error"])
            w.writerows(rows)
        with open(os.path.join(args.out_dir, f"{tag}ef_training_curve_bw{args.bitwidth}.csv"), "w", newline="") as fh:
            w = csv.writer(fh)
            w.writerow(["step", "loss_noef", "loss_ef"])
            w.writerows([(i + 1, a, b) for i, (a, b) in enumerate(zip(l0, l1))])


if __name__ == "__main__":
    main()
