"""Multi-process tests on CPU ranks (gloo): the staged low-bit all-reduce of
LowBitGroup and of the native ``lowbit`` backend against the reference's
arithmetic, pipeline-A, the DDP hook, backend forwarding, futures, and host
failure detection.  Mirrors reference tests/test_lowbit_allreduce_reference.py
and tests/test_pipeline_a_correctness.py, which needed 2 GPUs."""

import datetime
import os

import pytest
import torch
import torch.distributed as dist

from . import ref_oracle
from .dist_utils import run_ranks

CASES = [
    {"name": "linspace_nondiv_bw4", "bitwidth": 4, "numel": 1031, "pattern": "linspace", "seed": 11},
    {"name": "random_nondiv_bw2", "bitwidth": 2, "numel": 4099, "pattern": "random", "seed": 23},
    {"name": "alternating_div_bw1", "bitwidth": 1, "numel": 2048, "pattern": "alternating", "seed": 37},
    {"name": "small_range_div_bw4", "bitwidth": 4, "numel": 512, "pattern": "small_range", "seed": 41},
    {"name": "sparse_spikes_nondiv_bw2", "bitwidth": 2, "numel": 777, "pattern": "sparse_spikes", "seed": 53},
]


def make_input(rank, case):
    n, pat, seed = case["numel"], case["pattern"], case["seed"]
    if pat == "linspace":
        return torch.linspace(-2.5, 3.0, n) + rank * 0.037
    if pat == "random":
        g = torch.Generator().manual_seed(seed + rank)
        return torch.randn(n, generator=g) * 1.5 + rank * 0.031
    if pat == "alternating":
        idx = torch.arange(n)
        return torch.where(idx % 2 == 0, 1.0, -1.0) * (1.0 + 0.1 * rank)
    if pat == "small_range":
        idx = torch.arange(n, dtype=torch.float32)
        return 0.02 * torch.sin(idx / 7.0) + 0.015 * torch.cos(idx / 13.0) + rank * 0.002
    x = torch.zeros(n)
    pos = torch.arange(rank, n, 17)
    x[pos] = torch.linspace(-3.0, 3.0, pos.numel())
    return x


def c8_oracle(ref, inputs, bits):
    """Reference Python low-bit all-reduce (one scale per rank), composed from
    the reference's own quantisation functions."""
    W = len(inputs)
    n = inputs[0].numel()
    pad = (W - n % W) % W
    flats = [torch.cat([x, torch.zeros(pad)]) for x in inputs]
    shard = flats[0].numel() // W
    packed, scales = [], []
    for f in flats:
        q, s = ref.quantize_tensor(f, bits)
        packed.append([ref.pack_lowbit(p, bits)[0] for p in q.split(shard)])
        scales.append(s)
    outs = []
    for o in range(W):
        acc = torch.zeros(shard)
        for s in range(W):
            acc.add_(ref.dequantize_tensor(ref.unpack_lowbit(packed[s][o], bits, shard), scales[s]))
        q, sc = ref.quantize_tensor(acc, bits)
        outs.append(ref.dequantize_tensor(ref.unpack_lowbit(ref.pack_lowbit(q, bits)[0], bits, shard), sc))
    return torch.cat(outs)[:n]


def c15_oracle(inputs, bits, residuals=None):
    """Reference C++ low-bit all-reduce (per-shard float32 scales, error
    feedback on the sent values), restated with torch ops."""
    qmin, qmax = (0, 1) if bits == 1 else (-(1 << (bits - 1)), (1 << (bits - 1)) - 1)
    W = len(inputs)
    n = inputs[0].numel()
    pad = (W - n % W) % W

    def q_shard(x):
        amax = x.abs().max()
        s = torch.where(amax == 0, torch.ones(()), amax / float(qmax))
        q = torch.round(x / s).clamp(qmin, qmax)
        return q * s

    deq, new_res = [], []
    for r, x in enumerate(inputs):
        c = x.float() + (residuals[r] if residuals is not None else 0)
        cp = torch.cat([c, torch.zeros(pad)])
        d = torch.cat([q_shard(p) for p in cp.view(W, -1)])
        deq.append(d)
        new_res.append((cp - d)[:n])
    shard = deq[0].numel() // W
    outs = []
    for o in range(W):
        acc = torch.zeros(shard)
        for s in range(W):
            acc = acc + deq[s][o * shard : (o + 1) * shard]
        outs.append(q_shard(acc))
    return torch.cat(outs)[:n], new_res


# ----------------------------------------------------------------------------
# workers (module level: spawned processes import them)
# ----------------------------------------------------------------------------
def _init_gloo(rank, world):
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))


def _w_lowbitgroup(rank, world, case):
    from bitscom_b200 import LowBitGroup

    _init_gloo(rank, world)
    x = make_input(rank, case)
    g = LowBitGroup(bitwidth=case["bitwidth"])
    y = x.clone()
    g.all_reduce(y)
    dist.destroy_process_group()
    return x, y


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_lowbitgroup_staged_matches_reference(case):
    ref = ref_oracle.load()
    res = run_ranks(_w_lowbitgroup, 2, (case,))
    inputs = [r[0] for r in res]
    exp = c8_oracle(ref, inputs, case["bitwidth"])
    for _, y in res:
        assert (y - exp).abs().max() < 1e-6


def _w_sr(rank, world):
    from bitscom_b200 import LowBitGroup

    _init_gloo(rank, world)
    case = {"numel": 4099, "pattern": "random", "seed": 101}
    x = make_input(rank, case)
    g = LowBitGroup(bitwidth=4, stochastic_rounding=True)
    torch.manual_seed(1000 + rank)
    a = x.clone()
    g.all_reduce(a)
    torch.manual_seed(2000 + rank)
    b = x.clone()
    g.all_reduce(b)
    ga = [torch.empty_like(a) for _ in range(world)]
    dist.all_gather(ga, a)
    dist.destroy_process_group()
    return a, b, ga


def test_lowbitgroup_stochastic_rounding():
    res = run_ranks(_w_sr, 2)
    a, b, ga = res[0]
    assert (a - b).abs().max() > 0
    assert torch.isfinite(a).all() and torch.isfinite(b).all()
    assert (ga[0] - ga[1]).abs().max() < 1e-6  # every rank decodes the same bytes


def _w_backend(rank, world, bits, ef):
    import bitscom_b200 as bitscom

    bitscom.init(bitwidth=bits, error_feedback=ef)
    dist.init_process_group("lowbit", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    case = {"numel": 4099, "pattern": "random", "seed": 7}
    x = make_input(rank, case)
    outs = []
    t = x.clone()
    for _ in range(3):  # residual carried across calls for the same tensor
        t.copy_(x)
        w = dist.all_reduce(t, async_op=True)
        fut = w.get_future()
        w.wait()
        outs.append((t.clone(), fut.value()[0].clone()))
    # forwarded collectives
    b = torch.arange(4.0) * (rank + 1)
    dist.broadcast(b, src=1)
    gl = [torch.empty(2) for _ in range(world)]
    dist.all_gather(gl, torch.full((2,), float(rank)))
    dist.barrier()
    mx = torch.tensor([float(rank)])
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    be = dist.group.WORLD._get_backend(torch.device("cpu"))
    stats = dict(be.stats())
    dist.destroy_process_group()
    return x, outs, b, gl, mx, stats


@pytest.mark.parametrize("bits,ef", [(4, False), (2, True), (1, False)])
def test_native_backend_staged_path(bits, ef):
    res = run_ranks(_w_backend, 2, (bits, ef), env={"BITSCOM_TEST_DUMP_AFTER": os.environ.get("BITSCOM_TEST_DUMP_AFTER", "")})
    inputs = [r[0] for r in res]
    residuals = [torch.zeros(inputs[0].numel()) for _ in inputs] if ef else None
    for step in range(3):
        exp, new_res = c15_oracle(inputs, bits, residuals)
        for r in range(2):
            got, fut_val = res[r][1][step]
            assert (got - exp).abs().max() < 1e-5, (step, r)
            assert torch.equal(fut_val, got)
        if ef:
            residuals = new_res
    x, outs, b, gl, mx, stats = res[0]
    assert torch.equal(b, torch.arange(4.0) * 2)
    assert torch.equal(gl[1], torch.ones(2)) and float(mx) == 1.0
    assert stats["staged_calls"] == 3 and stats["forwarded_calls"] >= 4
    assert stats["residuals"] == (1 if ef else 0)


def _w_pipeline(rank, world, local_quantize):
    from bitscom_b200 import LowBitGroup

    _init_gloo(rank, world)
    local_group = None
    for r in range(world):  # singleton local groups: every rank is a leader
        g = dist.new_group([r])
        if r == rank:
            local_group = g
    x = torch.linspace(-1.0, 1.0, 257) + rank * 0.01
    exp = x.clone()
    dist.all_reduce(exp)
    grp = LowBitGroup(bitwidth=4)
    y = x.clone()
    grp.all_reduce(y, local_group=local_group, inter_group=dist.group.WORLD, chunk_size=63,
                   local_quantize=local_quantize)
    ga = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(ga, y)
    dist.destroy_process_group()
    return y, exp, ga


@pytest.mark.parametrize("local_quantize", [False, True])
def test_pipeline_a_correctness(local_quantize):
    res = run_ranks(_w_pipeline, 2, (local_quantize,))
    y, exp, ga = res[0]
    assert (ga[0] - ga[1]).abs().max() < 1e-6
    err = (y - exp).abs().max()
    assert err < 1.5 and err / exp.abs().max() < 0.2


def _w_ddp(rank, world):
    import bitscom_b200 as bitscom
    from bitscom_b200.models import TinyMLP, toy_batch

    _init_gloo(rank, world)
    torch.manual_seed(0)
    model = TinyMLP()
    ddp = torch.nn.parallel.DistributedDataParallel(model)
    state = bitscom.register_lowbit_hook(ddp, bitwidth=4, error_feedback=True)
    opt = torch.optim.SGD(ddp.parameters(), lr=0.05)
    g = torch.Generator().manual_seed(rank)
    losses = []
    for _ in range(30):
        x, y = toy_batch(64, 64, 10, "cpu", generator=g)
        loss = torch.nn.functional.cross_entropy(ddp(x), y)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss))
    params = torch.cat([p.detach().view(-1) for p in model.parameters()])
    sd = state.state_dict()
    dist.destroy_process_group()
    return losses, params, sd["calls"]


def test_ddp_hook_on_cpu_ranks():
    res = run_ranks(_w_ddp, 2)
    (l0, p0, c0), (l1, p1, c1) = res
    assert torch.equal(p0, p1)  # identical replicas after low-bit averaging
    assert sum(l0[-5:]) < sum(l0[:5]) and c0 == c1 and c0 > 0


def _w_failure(rank, world):
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    t = torch.ones(4)
    if rank == 1:
        return "skipped"  # never joins the collective, exits between steps
    try:
        dist.all_reduce(t)
    except Exception as exc:
        return f"raised: {type(exc).__name__}"
    return "completed"


def test_missing_rank_is_detected_by_timeout():
    res = run_ranks(_w_failure, 2, timeout=60)
    assert res[1] == "skipped"
    assert res[0].startswith("raised")


def _w_fsdp2(rank, world, backend, custom=False):
    import torch.nn as nn
    from torch.distributed.device_mesh import DeviceMesh
    from torch.distributed.fsdp import fully_shard

    if backend == "lowbit":
        import bitscom_b200 as bitscom

        bitscom.init(bitwidth=4, error_feedback=False)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    mesh = DeviceMesh.from_group(dist.group.WORLD, "cpu")
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(64, 128), nn.ReLU(), nn.Linear(128, 10))
    fully_shard(model[0], mesh=mesh)
    fully_shard(model, mesh=mesh)
    comms = {}
    if custom:
        from bitscom_b200.parallel.fsdp2 import enable_lowbit_fsdp2

        comms = enable_lowbit_fsdp2(model, bits=8)
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    g = torch.Generator().manual_seed(rank)
    losses = []
    for _ in range(4):
        x, y = torch.randn(32, 64, generator=g), torch.randint(0, 10, (32,), generator=g)
        loss = nn.functional.cross_entropy(model(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
        losses.append(float(loss.detach()))
    stats = {}
    if backend == "lowbit":
        stats = dict(dist.group.WORLD._get_backend(torch.device("cpu")).stats())
    if custom:
        stats = {"modules": sorted(comms), "fused": sum(a.fused_calls + r.fused_calls for a, r in comms.values())}
    dist.destroy_process_group()
    return losses, stats


def test_fsdp2_runs_over_lowbit_backend():
    """FSDP2 (fully_shard) on a `lowbit` process group: its reduce-scatter and
    all-gather reach the backend's tensor overrides, which forward CPU tensors
    to the inner gloo group (the fused low-bit kernels take CUDA tensors), so
    training matches plain gloo exactly."""
    ref = run_ranks(_w_fsdp2, 2, ("gloo",))
    got = run_ranks(_w_fsdp2, 2, ("lowbit",))
    for r in range(2):
        assert got[r][0] == ref[r][0]
    assert got[0][1]["forwarded_calls"] > 0


def test_fsdp2_custom_comms_install_and_fall_back_on_cpu():
    """enable_lowbit_fsdp2 installs one all-gather / reduce-scatter pair per
    FSDP module; CPU tensors fall back to the group's own collectives, so
    training matches plain gloo exactly (the fused path is tested on GPUs)."""
    ref = run_ranks(_w_fsdp2, 2, ("gloo",))
    got = run_ranks(_w_fsdp2, 2, ("gloo", True))
    for r in range(2):
        assert got[r][0] == ref[r][0]
    assert got[0][1] == {"modules": ["", "0"], "fused": 0}


def _w_bucketer(rank, world, bits):
    import torch.nn as nn

    from bitscom_b200 import LowBitGroup
    from bitscom_b200.parallel.bucketing import GradBucketer

    _init_gloo(rank, world)
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(32, 64), nn.ReLU(), nn.Linear(64, 64), nn.ReLU(), nn.Linear(64, 5))
    bk = GradBucketer(model.parameters(), LowBitGroup(bitwidth=bits, error_feedback=True), bucket_mb=0.01)
    g = torch.Generator().manual_seed(100 + rank)
    x, y = torch.randn(16, 32, generator=g), torch.randint(0, 5, (16,), generator=g)
    nn.functional.cross_entropy(model(x), y).backward()
    views_ok = all(
        any(buf.data_ptr() <= p.grad.data_ptr() < buf.data_ptr() + buf.numel() * buf.element_size() for buf in bk.buffers)
        for p in model.parameters()
    )
    local = [p.grad.clone() for p in model.parameters()]
    bk.sync()
    synced = [p.grad.clone() for p in model.parameters()]
    bk.zero_grad()
    zeroed = all(float(p.grad.abs().sum()) == 0.0 for p in model.parameters())
    dist.destroy_process_group()
    return bk.num_buckets(), views_ok, local, synced, zeroed


@pytest.mark.parametrize("bits", [16, 4])
def test_grad_bucketer(bits):
    res = run_ranks(_w_bucketer, 2, (bits,))
    nb, views_ok, _, _, zeroed = res[0]
    assert nb > 1 and views_ok and zeroed
    for i in range(len(res[0][2])):
        mean = (res[0][2][i] + res[1][2][i]) / 2
        a, b = res[0][3][i], res[1][3][i]
        assert torch.equal(a, b)  # every rank holds the same reduced gradient
        if bits == 16:  # >= 8 bits: full-precision all-reduce
            torch.testing.assert_close(a, mean, rtol=1e-6, atol=1e-7)
        else:
            assert float((a - mean).norm()) <= 0.5 * float(mean.norm()) + 1e-6


def _w_backend_views(rank, world):
    import bitscom_b200 as bitscom

    bitscom.init(bitwidth=4, error_feedback=False)
    dist.init_process_group("lowbit", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    g = torch.Generator().manual_seed(40 + rank)
    base = torch.randn(64, 65, generator=g)
    base_in = base.clone()
    t = base.t()  # non-contiguous view
    assert not t.is_contiguous()
    dist.all_reduce(t)
    b16 = (torch.randn(3001, generator=g) * 0.1).to(torch.bfloat16)
    b16_in = b16.clone()
    dist.all_reduce(b16)
    dist.destroy_process_group()
    return base_in, t.clone(), b16_in, b16


def test_native_backend_staged_path_views_and_bf16():
    """The staged (CPU) path on a non-contiguous view and on bf16 tensors:
    values reduced in logical element order, results written back in place
    and rounded to the tensor's dtype."""
    res = run_ranks(_w_backend_views, 2)
    exp, _ = c15_oracle([r[0].t().reshape(-1) for r in res], 4)
    exp16, _ = c15_oracle([r[2].float() for r in res], 4)
    for r in range(2):
        assert (res[r][1].reshape(-1) - exp).abs().max() < 1e-5
        assert res[r][3].dtype == torch.bfloat16
        assert torch.equal(res[r][3], exp16.to(torch.bfloat16))


def _w_rs_ag_tensor(rank, world):
    from bitscom_b200 import LowBitGroup

    _init_gloo(rank, world)
    grp = LowBitGroup(bitwidth=4)
    g = torch.Generator().manual_seed(70 + rank)
    x = torch.randn(2 * 1000, generator=g)
    rs = torch.empty(1000)
    grp.reduce_scatter_tensor(rs, x)
    rs_avg = torch.empty(1000)
    grp.reduce_scatter_tensor(rs_avg, x, average=True)
    ag = torch.empty(2 * 2000)
    grp.all_gather_into_tensor(ag, x)
    dist.destroy_process_group()
    return x, rs, rs_avg, ag


def test_lowbitgroup_tensor_rs_ag_on_cpu():
    """Without the fused kernel (CPU tensors) the tensor reduce-scatter and
    all-gather quantise each rank's input with the reference's per-tensor
    4-bit roundtrip and then reduce / gather in full precision."""
    from bitscom_b200.quantization import roundtrip_tensor

    res = run_ranks(_w_rs_ag_tensor, 2)
    q = [roundtrip_tensor(r[0], 4) for r in res]
    total = q[0] + q[1]
    for r in range(2):
        torch.testing.assert_close(res[r][1], total[r * 1000 : (r + 1) * 1000], rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(res[r][2], total[r * 1000 : (r + 1) * 1000] / 2, rtol=1e-6, atol=1e-6)
        assert torch.equal(res[r][3], torch.cat(q))


def _w_sharded_dp(rank, world):
    import torch.nn as nn

    from bitscom_b200.parallel.fsdp import LowBitShardedDP

    _init_gloo(rank, world)
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(32, 64), nn.ReLU(), nn.Linear(64, 4))
    sdp = LowBitShardedDP(model, lambda ps: torch.optim.AdamW(ps, lr=1e-2), rs_bits=8, ag_bits=8, use_fused=False)
    g = torch.Generator().manual_seed(rank)
    w = torch.randn(32, 4, generator=torch.Generator().manual_seed(123))

    def batch():
        x = torch.randn(64, 32, generator=g)
        return x, (x @ w).argmax(1)

    losses = []
    for _ in range(30):
        x, y = batch()
        loss = nn.functional.cross_entropy(sdp(x), y)
        loss.backward()
        sdp.step()
        losses.append(float(loss.detach()))
    ck = sdp.state_dict_shard()
    sdp.load_state_dict_shard(ck)
    flat = sdp.flat_param.clone()
    dist.destroy_process_group()
    return losses, flat, sdp.shard, sdp.numel


def test_sharded_dp_on_cpu_ranks():
    """LowBitShardedDP without the fused kernels (gloo reduce-scatter and
    all-gather after the reference's quantisation roundtrip): the ranks'
    working parameters stay identical, training makes progress, and a
    checkpoint restores every rank's working copy."""
    res = run_ranks(_w_sharded_dp, 2)
    (l0, f0, shard, numel), (l1, f1, _, _) = res
    assert torch.equal(f0, f1)
    assert shard * 2 >= numel and shard % 8192 == 0
    assert sum(l0[-5:]) / 5 < l0[0] - 0.2 and sum(l1[-5:]) / 5 < l1[0] - 0.2
