"""Fused low-bit collectives across GPUs (one process per GPU, NCCL for the
plumbing).  Bit-exact against the CPU model of the block-scaled format; needs
at least two CUDA devices.  NVLS is disabled (these tests include a bounded
wait that runs out on purpose)."""

import datetime
import os

import pytest
import torch
import torch.distributed as dist

from . import wire_emulator as emu
from .dist_utils import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ENV = {"NCCL_NVLS_ENABLE": "0", "BITSCOM_WORKSPACE_MB": "128"}


def _need(n=2):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} CUDA devices")


def _init(rank, world, backend="nccl"):
    torch.cuda.set_device(rank)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))


def _x(n, rank, seed=0, dtype=torch.float32):
    g = torch.Generator().manual_seed(1000 * seed + rank)
    x = torch.randn(n, generator=g) * 1e-3
    idx = torch.randint(0, n, (max(1, n // 100),), generator=g)
    x[idx] = torch.randn(idx.numel(), generator=g) * 1e-1
    return x.to(dtype)


def _w_allreduce(rank, world, cases):
    from bitscom_b200.parallel.comm import Communicator

    _init(rank, world)
    comm = Communicator.for_group(None, rank)
    assert comm is not None, "peer-to-peer workspace unavailable"
    outs = []
    for (n, bits, algo, fmt, ef, dtype) in cases:
        x = _x(n, rank, seed=bits + n, dtype=getattr(torch, dtype))
        t = x.cuda()
        r = (torch.randn(n, generator=torch.Generator().manual_seed(rank)) * 1e-4) if ef else None
        rg = r.cuda() if ef else None
        comm.all_reduce(t, bits=bits, algo=algo, fmt=fmt, residual=rg, post_scale=1.0 / world)
        torch.cuda.synchronize()
        comm.check()
        outs.append((x, r, t.cpu(), rg.cpu() if ef else None))
    assert comm.check_canaries() == 0, "a launch wrote outside its workspace slots"
    dist.destroy_process_group()
    return outs


CASES = [
    (1000, 4, "oneshot", "int", False, "float32"),
    (1000, 4, "twoshot", "int", False, "float32"),
    (300001, 4, "twoshot", "int", True, "float32"),
    (300001, 2, "twoshot", "int", True, "float32"),
    (65536, 1, "twoshot", "int", False, "float32"),
    (65536, 8, "oneshot", "int", True, "float32"),
    (123457, 12, "twoshot", "int", False, "float32"),
    (123457, 16, "twoshot", "int", False, "float32"),
    (100000, 8, "twoshot", "e4m3", False, "float32"),
    (100000, 4, "twoshot", "int", False, "bfloat16"),
    (77777, 1, "twoshot", "sign", True, "float32"),
]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_allreduce_matches_model(world):
    _need(world)
    res = run_ranks(_w_allreduce, world, (CASES,), env=ENV, timeout=300)
    for ci, (n, bits, algo, fmt, ef, dtype) in enumerate(CASES):
        inputs = [res[r][ci][0].float() for r in range(world)]
        residuals = [res[r][ci][1] for r in range(world)] if ef else None
        model = emu.allreduce_two_shot if algo == "twoshot" else emu.allreduce_one_shot
        exp, new_res = model(inputs, bits, residuals=residuals, post_scale=1.0 / world, fmt=fmt)
        for r in range(world):
            got = res[r][ci][2]
            assert torch.equal(got, exp.to(got.dtype)), (ci, r)
            if ef:
                assert torch.equal(res[r][ci][3], new_res[r]), (ci, r)


@pytest.mark.parametrize("world", [2, 8])
def test_fused_allreduce_matches_model_warp_specialised(world):
    """The same cases on the warp-specialised kernel (producer warp waits on
    the peers' flags and stages packed data by bulk copies)."""
    _need(world)
    res = run_ranks(_w_allreduce, world, (CASES,), env={**ENV, "BITSCOM_KERNEL": "ws", "BITSCOM_TIMEOUT_MS": "20000"},
                    timeout=300)
    for ci, (n, bits, algo, fmt, ef, dtype) in enumerate(CASES):
        inputs = [res[r][ci][0].float() for r in range(world)]
        residuals = [res[r][ci][1] for r in range(world)] if ef else None
        model = emu.allreduce_two_shot if algo == "twoshot" else emu.allreduce_one_shot
        exp, new_res = model(inputs, bits, residuals=residuals, post_scale=1.0 / world, fmt=fmt)
        for r in range(world):
            got = res[r][ci][2]
            assert torch.equal(got, exp.to(got.dtype)), (ci, r)
            if ef:
                assert torch.equal(res[r][ci][3], new_res[r]), (ci, r)


def _w_bucket_series(rank, world, n, iters, max_ctas):
    from bitscom_b200.parallel.comm import Communicator

    _init(rank, world)
    comm = Communicator.for_group(None, rank)
    outs = []
    res = torch.zeros(n, device="cuda")
    xs = [_x(n, rank, seed=70 + i) for i in range(iters)]
    for x in xs:
        t = x.cuda()
        comm.all_reduce(t, bits=4, algo="twoshot", residual=res, post_scale=1.0 / world, max_ctas=max_ctas)
        outs.append(t.cpu())
    torch.cuda.synchronize()
    comm.check()
    dist.destroy_process_group()
    return xs, outs


@pytest.mark.parametrize("variant", ["reg", "ws"])
@pytest.mark.parametrize("max_ctas", [32, 0])
def test_bucket_sized_series_matches_model(variant, max_ctas):
    """DDP-bucket-sized two-shot launches (6.5M elements, 4-bit EF) back to
    back, with the hook's restricted grid and a full grid: every call on every
    rank equals the model, residuals carried across calls."""
    _need(2)
    world, n, iters = 2, 6_500_000, 4
    res = run_ranks(_w_bucket_series, world, (n, iters, max_ctas),
                    env={**ENV, "BITSCOM_KERNEL": variant, "BITSCOM_TIMEOUT_MS": "20000"}, timeout=300)
    residuals = [torch.zeros(n) for _ in range(world)]
    for i in range(iters):
        exp, residuals = emu.allreduce_two_shot([res[r][0][i] for r in range(world)], 4, residuals=residuals,
                                                post_scale=1.0 / world)
        for r in range(world):
            assert torch.equal(res[r][1][i], exp), (i, r)


def _w_rs_ag(rank, world):
    from bitscom_b200.parallel.comm import Communicator

    _init(rank, world)
    comm = Communicator.for_group(None, rank)
    n = 50001
    x = _x(n * world, rank, seed=3)
    out = torch.empty(n, device="cuda")
    comm.reduce_scatter(out, x.cuda(), bits=8, post_scale=1.0)
    s = _x(n, rank, seed=4)
    g = torch.empty(n * world, device="cuda")
    comm.all_gather(g, s.cuda(), bits=8)
    torch.cuda.synchronize()
    dist.destroy_process_group()
    return x, out.cpu(), s, g.cpu()


def test_fused_reduce_scatter_all_gather():
    _need(2)
    res = run_ranks(_w_rs_ag, 2, env=ENV)
    xs = [r[0] for r in res]
    rs = emu.reduce_scatter(xs, 8)
    ag = emu.all_gather([r[2] for r in res], 8)
    for r in range(2):
        assert torch.equal(res[r][1], rs[r])
        assert torch.equal(res[r][3], ag)


def _w_backend(rank, world):
    import bitscom_b200 as bitscom

    bitscom._ext._C.install_crash_backtrace()
    bitscom.init(bitwidth=4, error_feedback=True, algo="twoshot")
    torch.cuda.set_device(rank)
    dist.init_process_group("lowbit", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    x = _x(200000, rank, seed=9).cuda()
    t = x.clone()
    w = dist.all_reduce(t, async_op=True)
    fut_val = w.get_future().wait()[0]
    w.wait()
    torch.cuda.synchronize()
    be = dist.group.WORLD._get_backend(torch.device("cuda"))
    st = dict(be.stats())
    # reduce-scatter / all-gather through the backend (8-bit-compressible with force_lowbit off: 4-bit)
    rs_in = _x(2 * 8192, rank, seed=10).cuda()
    rs_out = torch.empty(8192, device="cuda")
    dist.reduce_scatter_tensor(rs_out, rs_in)
    ag_out = torch.empty(2 * 8192, device="cuda")
    dist.all_gather_into_tensor(ag_out, rs_out)
    b = torch.full((4,), float(rank), device="cuda")
    dist.broadcast(b, src=1)
    dist.barrier()
    torch.cuda.synchronize()
    st2 = dict(be.stats())
    dist.destroy_process_group()
    return x.cpu(), t.cpu(), fut_val.cpu(), st, st2, b.cpu()


def test_lowbit_backend_fused_path():
    _need(2)
    res = run_ranks(_w_backend, 2, env=ENV)
    inputs = [res[r][0] for r in range(2)]
    zeros = [torch.zeros_like(i) for i in inputs]
    exp, _ = emu.allreduce_two_shot(inputs, 4, residuals=zeros)
    for r in range(2):
        x, t, fv, st, st2, b = res[r]
        assert torch.equal(t, exp) and torch.equal(fv, exp)
        assert st["fused_calls"] == 1 and st["staged_calls"] == 0
        assert st2["fused_calls"] == 3 and torch.equal(b, torch.ones(4))


def _w_ddp(rank, world, lowbit=True):
    import bitscom_b200 as bitscom
    from bitscom_b200.models import resnet18_cifar

    _init(rank, world)
    torch.manual_seed(0)
    model = resnet18_cifar(10).cuda()
    ddp = torch.nn.parallel.DistributedDataParallel(model, device_ids=[rank], bucket_cap_mb=5)
    state = bitscom.register_lowbit_hook(ddp, bitwidth=4, error_feedback=True) if lowbit else None
    opt = torch.optim.SGD(ddp.parameters(), lr=0.05, momentum=0.9)
    g = torch.Generator(device="cuda").manual_seed(rank)
    for _ in range(5):
        x = torch.randn(32, 3, 32, 32, device="cuda", generator=g)
        y = torch.randint(0, 10, (32,), device="cuda", generator=g)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = torch.nn.functional.cross_entropy(ddp(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
    torch.cuda.synchronize()
    p = torch.cat([q.detach().float().view(-1) for q in model.parameters()]).cpu()
    launches = sum(c.stats()["launches"] for c in state._comms.values() if c is not None) if lowbit else 0
    dist.destroy_process_group()
    return p, launches


def test_ddp_hook_replicas_stay_identical():
    """4-bit EF DDP: replicas bit-identical, and the training trajectory
    tracks fp32 DDP (the parameter update of 5 steps points the same way)."""
    _need(2)
    res = run_ranks(_w_ddp, 2, env=ENV, timeout=300)
    fp = run_ranks(_w_ddp, 2, (False,), env=ENV, timeout=300)
    assert torch.equal(res[0][0], res[1][0])
    assert res[0][1] > 5
    torch.manual_seed(0)
    from bitscom_b200.models import resnet18_cifar

    p0 = torch.cat([q.detach().float().view(-1) for q in resnet18_cifar(10).parameters()])
    d_lb, d_fp = res[0][0] - p0, fp[0][0] - p0
    cos = float(torch.dot(d_lb, d_fp) / (d_lb.norm() * d_fp.norm()))
    rel = float((d_lb - d_fp).norm() / d_fp.norm())
    assert cos > 0.75 and rel < 0.8, (cos, rel)  # measured on 2 B200s: cos 0.84


def _w_timeout(rank, world):
    from bitscom_b200.parallel.comm import Communicator

    _init(rank, world)
    comm = Communicator.for_group(None, rank)
    comm.set_timeout(0.5)
    t = torch.randn(100000, device="cuda")
    comm.all_reduce(t, bits=4, algo="twoshot")  # a healthy call first
    torch.cuda.synchronize()
    comm.check()
    if rank == 1:
        comm.native.set_fault_skip_signal(True)  # this rank drops its flags
    dist.barrier()
    comm.all_reduce(t, bits=4, algo="twoshot")
    torch.cuda.synchronize()
    status = comm.status()
    try:
        comm.check()
        raised = False
    except RuntimeError:
        raised = True
    ok = float(torch.ones(4, device="cuda").sum())  # context still healthy
    dist.barrier()
    dist.destroy_process_group()
    return status, raised, ok


def test_peer_timeout_is_reported_not_hung():
    _need(2)
    res = run_ranks(_w_timeout, 2, env=ENV, timeout=120)
    for status, raised, ok in res:
        assert ok == 4.0
    assert res[0][0] != 0 and res[0][1]  # rank 0 waited on rank 1's dropped flags


def _w_pipeline(rank, world):
    from bitscom_b200 import LowBitGroup

    _init(rank, world)
    local = None
    for r in range(world):
        g = dist.new_group([r])
        if r == rank:
            local = g
    x = (torch.linspace(-1.0, 1.0, 100003) + rank * 0.01).cuda()
    exp = x.clone()
    dist.all_reduce(exp)
    grp = LowBitGroup(bitwidth=4)
    y = x.clone()
    grp.all_reduce(y, local_group=local, inter_group=dist.group.WORLD, chunk_size=30000)
    ga = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(ga, y)
    torch.cuda.synchronize()
    dist.destroy_process_group()
    return y.cpu(), exp.cpu(), [a.cpu() for a in ga]


def test_pipeline_a_on_gpus():
    """Pipeline-A with singleton local groups (every rank a leader, the
    reference's own test topology): the dual-stream schedule runs every chunk
    through the inter stage, the fused one-shot 4-bit all-reduce of that
    chunk (30000 elements, 15 KB packed: below the one-shot threshold), so the
    result equals the block model chunk by chunk, bit for bit, on every rank."""
    _need(2)
    world = 2
    res = run_ranks(_w_pipeline, world, env=ENV)
    xs = [(torch.linspace(-1.0, 1.0, 100003) + r * 0.01) for r in range(world)]
    exp = torch.cat([
        emu.allreduce_one_shot([x[s:s + 30000] for x in xs], 4)[0] for s in range(0, 100003, 30000)
    ])
    y, fp, ga = res[0]
    assert torch.equal(ga[0], ga[1])
    assert torch.equal(y, exp)
    assert (y - fp).abs().max() / fp.abs().max() < 0.1  # and it tracks the fp32 sum


def _w_sdp(rank, world):
    from bitscom_b200.models import gpt2_small_test
    from bitscom_b200.parallel.fsdp import LowBitShardedDP

    _init(rank, world)
    torch.manual_seed(0)
    model = gpt2_small_test(n_positions=128).cuda()
    sdp = LowBitShardedDP(model, lambda ps: torch.optim.AdamW(ps, lr=1e-3), rs_bits=8, ag_bits=8)
    g = torch.Generator(device="cuda").manual_seed(rank)
    losses = []
    for _ in range(20):
        start = torch.randint(0, 512, (8, 1), device="cuda", generator=g)
        tok = (start + torch.arange(65, device="cuda")) % 512
        with torch.autocast("cuda", dtype=torch.bfloat16):
            _, loss = sdp(tok[:, :-1], tok[:, 1:])
        loss.backward()
        sdp.step()
        losses.append(float(loss))
    torch.cuda.synchronize()
    fp = sdp.flat_param.cpu()
    dist.destroy_process_group()
    return fp, losses


def test_sharded_dp_replicas_identical():
    _need(2)
    res = run_ranks(_w_sdp, 2, env=ENV, timeout=300)
    assert torch.equal(res[0][0], res[1][0])  # every rank decodes the same gathered bytes
    assert res[0][1][-1] < res[0][1][0]


def _w_graph(rank, world):
    from bitscom_b200.parallel.comm import Communicator

    _init(rank, world)
    comm = Communicator.for_group(None, rank)
    comm.set_timeout(10.0)
    n = 300001
    xs = [_x(n, rank, seed=60 + i) for i in range(3)]
    static = torch.zeros(n, device="cuda")
    res = torch.zeros(n, device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        comm.all_reduce(static, bits=4, algo="twoshot", residual=res, post_scale=1.0 / world)
        comm.all_reduce(static, bits=8, algo="oneshot", post_scale=1.0)
    outs = []
    for x in xs:
        static.copy_(x.cuda())
        g.replay()
        outs.append(static.cpu())
    torch.cuda.synchronize()
    comm.check()
    del g
    dist.destroy_process_group()
    return xs, outs


def test_graph_replay_across_ranks_matches_model():
    """Two collectives captured in one CUDA graph and replayed three times on
    every rank: the device-side epochs keep the ranks in step and error
    feedback carries across replays."""
    _need(2)
    world = 2
    res = run_ranks(_w_graph, world, env=ENV, timeout=300)
    residuals = [torch.zeros(300001) for _ in range(world)]
    for i in range(3):
        inputs = [res[r][0][i] for r in range(world)]
        mid, residuals = emu.allreduce_two_shot(inputs, 4, residuals=residuals, post_scale=1.0 / world)
        exp, _ = emu.allreduce_one_shot([mid] * world, 8)
        for r in range(world):
            assert torch.equal(res[r][1][i], exp), (i, r)


class _Scale(torch.nn.Module):
    """y = x * w with a flat weight: the gradient of sum(y) is x exactly, so
    the reduce-scatter input is known bit-for-bit; forward records the
    unsharded weight FSDP2 all-gathered."""

    def __init__(self, n):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.zeros(n))
        self.seen = None

    def forward(self, x):
        self.seen = self.weight.detach().clone()
        return x * self.weight


def _w_fsdp2(rank, world, n):
    import bitscom_b200 as bitscom
    from torch.distributed.device_mesh import DeviceMesh
    from torch.distributed.fsdp import fully_shard

    bitscom.init(bitwidth=8, error_feedback=False, force_lowbit=True)
    torch.cuda.set_device(rank)
    dist.init_process_group("lowbit", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    mesh = DeviceMesh.from_group(dist.group.WORLD, "cuda")
    model = _Scale(n).cuda()
    w0 = _x(n, 0, seed=21)  # the same full weight on every rank before sharding
    with torch.no_grad():
        model.weight.copy_(w0.cuda())
    fully_shard(model, mesh=mesh)
    x = _x(n, rank, seed=22).cuda()
    loss = model(x).sum()
    loss.backward()
    torch.cuda.synchronize()
    seen = model.seen.cpu()
    grad_shard = model.weight.grad.to_local().cpu()
    be = dist.group.WORLD._get_backend(torch.device("cuda"))
    st = dict(be.stats())
    dist.destroy_process_group()
    return w0, x.cpu(), seen, grad_shard, st


def test_fsdp2_step_on_lowbit_group_matches_model():
    """FSDP2 (fully_shard) on a `lowbit` process group on GPUs: its parameter
    all-gather and gradient reduce-scatter run the fused 8-bit kernels
    (backend counters), and the unsharded weight and the averaged gradient
    shard equal the wire model bit-for-bit on every rank."""
    _need(2)
    world, n = 2, 8192 * 6
    res = run_ranks(_w_fsdp2, world, (n,), env=ENV, timeout=300)
    w0 = res[0][0]
    shard = n // world
    exp_w = emu.all_gather([w0[r * shard:(r + 1) * shard] for r in range(world)], 8)
    exp_g = emu.reduce_scatter([res[r][1] for r in range(world)], 8, post_scale=1.0 / world)
    for r in range(world):
        _, _, seen, grad_shard, st = res[r]
        assert torch.equal(seen, exp_w), r
        assert torch.equal(grad_shard, exp_g[r]), r
        assert st["fused_calls"] >= 2, st  # at least one all-gather and one reduce-scatter


def _w_fsdp2_custom(rank, world, n):
    from torch.distributed.device_mesh import DeviceMesh
    from torch.distributed.fsdp import fully_shard

    from bitscom_b200.parallel.fsdp2 import enable_lowbit_fsdp2

    _init(rank, world)  # a plain NCCL group: the low-bit collectives come from the custom comms
    mesh = DeviceMesh.from_group(dist.group.WORLD, "cuda")
    model = _Scale(n).cuda()
    w0 = _x(n, 0, seed=21)
    with torch.no_grad():
        model.weight.copy_(w0.cuda())
    fully_shard(model, mesh=mesh)
    comms = enable_lowbit_fsdp2(model, bits=8, error_feedback=False, group=dist.group.WORLD)
    x = _x(n, rank, seed=22).cuda()
    model(x).sum().backward()
    torch.cuda.synchronize()
    seen = model.seen.cpu()
    grad_shard = model.weight.grad.to_local().cpu()
    ag, rs = comms[""]
    dist.destroy_process_group()
    return w0, x.cpu(), seen, grad_shard, (ag.fused_calls, rs.fused_calls)


def test_fsdp2_custom_lowbit_comms_match_model():
    """FSDP2 on an NCCL group with this library's low-bit all-gather and
    reduce-scatter installed per FSDP module: same bit-exact model as above."""
    _need(2)
    world, n = 2, 8192 * 6
    res = run_ranks(_w_fsdp2_custom, world, (n,), env=ENV, timeout=300)
    w0 = res[0][0]
    shard = n // world
    exp_w = emu.all_gather([w0[r * shard:(r + 1) * shard] for r in range(world)], 8)
    exp_g = emu.reduce_scatter([res[r][1] for r in range(world)], 8, post_scale=1.0 / world)
    for r in range(world):
        _, _, seen, grad_shard, (n_ag, n_rs) = res[r]
        assert torch.equal(seen, exp_w), r
        assert torch.equal(grad_shard, exp_g[r]), r
        assert n_ag >= 1 and n_rs == 1


def test_ddp_hook_replicas_identical_warp_specialised():
    """The DDP hook on the warp-specialised kernel (restricted grid while
    backward runs, full grid for the last bucket): replicas bit-identical."""
    _need(2)
    res = run_ranks(_w_ddp, 2, env={**ENV, "BITSCOM_KERNEL": "ws", "BITSCOM_TIMEOUT_MS": "20000"}, timeout=300)
    assert torch.equal(res[0][0], res[1][0])
    assert res[0][1] > 5
