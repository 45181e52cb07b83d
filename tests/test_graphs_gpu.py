"""Whole-step CUDA-graph capture of DDP training with the low-bit comm hook
(bitscom_b200.parallel.graphs.GraphedStep), world size 1 on one GPU."""

import datetime
import os

import pytest
import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _pg():
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29655")
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))


def _make(seed=0):
    torch.manual_seed(seed)
    model = nn.Sequential(nn.Linear(64, 256), nn.ReLU(), nn.Linear(256, 256), nn.ReLU(), nn.Linear(256, 10)).cuda()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ddp = nn.parallel.DistributedDataParallel(model, device_ids=[0], gradient_as_bucket_view=True,
                                                  broadcast_buffers=False, bucket_cap_mb=0.1)
    torch.cuda.current_stream().wait_stream(side)
    return model, ddp


def test_graphed_ddp_step_matches_eager(cuda):
    import bitscom_b200 as bitscom
    from bitscom_b200.parallel.graphs import DDP_EAGER_WARMUP, GraphedStep

    _pg()
    try:
        g = torch.Generator().manual_seed(1)
        batches = [(torch.randn(128, 64, generator=g).cuda(), torch.randint(0, 10, (128,), generator=g).cuda())
                   for _ in range(6)]

        def build():
            model, ddp = _make()
            state = bitscom.register_lowbit_hook(ddp, bitwidth=4, error_feedback=True)
            opt = torch.optim.SGD(ddp.parameters(), lr=0.05, momentum=0.9)

            def step(x, y):
                loss = F.cross_entropy(ddp(x), y)
                loss.backward()
                opt.step()
                opt.zero_grad(set_to_none=False)
                return loss

            return model, state, step

        # eager: warm-up steps on batch 0, then batches 1..5
        m_e, s_e, step_e = build()
        for _ in range(DDP_EAGER_WARMUP):
            step_e(*batches[0])
        for x, y in batches[1:]:
            step_e(x, y)
        torch.cuda.synchronize()

        m_g, s_g, step_g = build()
        gs = GraphedStep(step_g, batches[0], warmup=DDP_EAGER_WARMUP)
        comm = next(c for c in s_g._comms.values() if c is not None)
        e0 = comm.native.device_epoch()
        launches = comm.stats()["launches"]
        res_before = {k: v.clone() for k, v in s_g.residuals.items()}
        for x, y in batches[1:]:
            gs(x, y)
        torch.cuda.synchronize()
        comm.check()
        # every replay ran the captured all-reduce launches (host stats do not move)
        assert comm.stats()["launches"] == launches
        per_step = len(s_g.residuals)
        assert comm.native.device_epoch() == e0 + per_step * (len(batches) - 1)
        assert any(not torch.equal(res_before[k], v) for k, v in s_g.residuals.items())
        for pe, pg in zip(m_e.parameters(), m_g.parameters()):
            torch.testing.assert_close(pg, pe, rtol=1e-4, atol=1e-5)
    finally:
        dist.destroy_process_group()
