"""Fused collective kernels on one GPU (world size 1: every phase runs, the
peer stores loop back to the own workspace), checked bit-for-bit against the
CPU model of the block-scaled format, plus the bounded-wait error path."""

import pytest
import torch

from bitscom_b200.parallel.comm import Communicator

from . import wire_emulator as emu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def comm():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return Communicator.create_local(0, workspace_bytes=64 << 20)


def _x(n, seed=0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, generator=g) * 1e-3
    idx = torch.randint(0, n, (max(1, n // 100),), generator=g)
    x[idx] = torch.randn(idx.numel(), generator=g) * 1e-1
    return x.to(dtype)


@pytest.mark.parametrize("bits", [1, 2, 4, 8, 12, 16])
@pytest.mark.parametrize("algo", ["twoshot", "oneshot"])
@pytest.mark.parametrize("n", [1, 1000, 8192, 50001])
def test_allreduce_matches_model(comm, bits, algo, n):
    x = _x(n, seed=bits + n)
    t = x.cuda()
    comm.all_reduce(t, bits=bits, algo=algo, post_scale=0.5)
    torch.cuda.synchronize()
    comm.check()
    model = emu.allreduce_two_shot if algo == "twoshot" else emu.allreduce_one_shot
    exp, _ = model([x], bits, post_scale=0.5)
    assert torch.equal(t.cpu(), exp)


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("algo", ["twoshot", "oneshot"])
def test_allreduce_error_feedback(comm, bits, algo):
    n = 123457
    x = _x(n, seed=bits)
    r = torch.randn(n) * 1e-4
    t, rg = x.cuda(), r.cuda()
    comm.all_reduce(t, bits=bits, algo=algo, residual=rg)
    torch.cuda.synchronize()
    model = emu.allreduce_two_shot if algo == "twoshot" else emu.allreduce_one_shot
    exp, res = model([x], bits, residuals=[r])
    assert torch.equal(t.cpu(), exp)
    assert torch.equal(rg.cpu(), res[0])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_allreduce_low_precision_io(comm, dtype):
    x = _x(77777, seed=5, dtype=dtype)
    t = x.cuda()
    out = torch.empty_like(t)
    comm.all_reduce(t, out=out, bits=4)
    torch.cuda.synchronize()
    exp, _ = emu.allreduce_two_shot([x.float()], 4)
    assert out.dtype == dtype
    assert torch.equal(out.cpu(), exp.to(dtype))
    assert torch.equal(t.cpu(), x)  # input untouched when out is given


def test_allreduce_e4m3(comm):
    x = _x(40000, seed=11)
    t = x.cuda()
    comm.all_reduce(t, bits=8, fmt="e4m3")
    torch.cuda.synchronize()
    exp, _ = emu.allreduce_two_shot([x], 8, fmt="e4m3")
    assert torch.equal(t.cpu(), exp)
    assert (t.cpu() - x).abs().max() <= x.abs().max() / 8  # 3 mantissa bits


@pytest.mark.parametrize("bits", [4, 8])
def test_reduce_scatter_and_all_gather(comm, bits):
    n = 20000
    x = _x(n, seed=bits)
    out = torch.empty(n, device="cuda")
    comm.reduce_scatter(out, x.cuda(), bits=bits, post_scale=1.0)
    g = torch.empty(n, device="cuda")
    comm.all_gather(g, x.cuda(), bits=bits)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), emu.reduce_scatter([x], bits)[0])
    assert torch.equal(g.cpu(), emu.all_gather([x], bits))


def test_segmented_large_message(comm):
    cap = comm.native.max_elems_per_launch(0, 16)
    n = cap + 12345
    x = _x(n, seed=1)
    t = x.cuda()
    before = comm.stats()["launches"]
    comm.all_reduce(t, bits=16, algo="twoshot")
    torch.cuda.synchronize()
    assert comm.stats()["launches"] - before == 2
    exp1, _ = emu.allreduce_two_shot([x[:cap]], 16)
    exp2, _ = emu.allreduce_two_shot([x[cap:]], 16)
    assert torch.equal(t.cpu(), torch.cat([exp1, exp2]))


def test_stochastic_rounding_reproducible_and_unbiased(comm):
    x = torch.full((1 << 16,), 0.3)
    x[::1024] = 1.0  # every block: amax 1 -> 2-bit scale 1
    a, b, c = x.cuda(), x.cuda(), x.cuda()
    comm.all_reduce(a, bits=2, algo="oneshot", stochastic_rounding=True, seed=5, offset=1)
    comm.all_reduce(b, bits=2, algo="oneshot", stochastic_rounding=True, seed=5, offset=1)
    comm.all_reduce(c, bits=2, algo="oneshot", stochastic_rounding=True, seed=5, offset=2)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and not torch.equal(a, c)
    mask = torch.ones_like(x, dtype=torch.bool)
    mask[::1024] = False
    assert abs(float(a.cpu()[mask].mean()) - 0.3) < 0.01


def test_back_to_back_launches_many_epochs(comm):
    x = _x(300000, seed=2)
    exp, _ = emu.allreduce_two_shot([x], 4)
    for _ in range(20):
        t = x.cuda()
        comm.all_reduce(t, bits=4, algo="twoshot", max_ctas=7)
    torch.cuda.synchronize()
    assert torch.equal(t.cpu(), exp)


def test_timeout_returns_error_status_without_faulting(cuda):
    """A wait that nothing will satisfy: this rank drops its own signals, the
    kernel gives up after the bounded wait and reports through the status word."""
    c = Communicator.create_local(0, workspace_bytes=64 << 20)
    c.set_timeout(0.2)
    c.native.set_fault_skip_signal(True)
    t = torch.randn(100000, device="cuda")
    c.all_reduce(t, bits=4, algo="twoshot")
    torch.cuda.synchronize()
    assert c.status() != 0
    with pytest.raises(RuntimeError, match="did not signal"):
        c.check()
    with pytest.raises(RuntimeError, match="broken"):
        c.all_reduce(t, bits=4)
    # the CUDA context is still healthy
    y = torch.ones(10, device="cuda") * 2
    assert float(y.sum()) == 20.0


def test_segmented_reduce_scatter_and_all_gather(comm):
    """Shards larger than one launch are processed as column segments."""
    cap_ag = comm.native.max_elems_per_launch(3, 8)
    n = cap_ag + 5 * 8192 + 77
    x = _x(n, seed=21)
    g = torch.empty(n, device="cuda")
    r = torch.zeros(n, device="cuda")
    comm.all_gather(g, x.cuda(), bits=8, residual=r)
    out = torch.empty(n, device="cuda")
    comm.reduce_scatter(out, x.cuda(), bits=8)
    torch.cuda.synchronize()
    assert torch.equal(g.cpu(), emu.all_gather([x], 8))
    assert torch.equal(out.cpu(), emu.reduce_scatter([x], 8)[0])
    # residual of the gather = x - dequant(quant(x))
    assert torch.equal(r.cpu(), x - emu.all_gather([x], 8))


def test_sharded_dp_single_rank_trains(cuda):
    import datetime
    import os

    import torch.distributed as dist

    from bitscom_b200.models import gpt2_small_test
    from bitscom_b200.parallel.fsdp import LowBitShardedDP

    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29653")
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    model = gpt2_small_test(n_positions=128).cuda()
    sdp = LowBitShardedDP(model, lambda ps: torch.optim.AdamW(ps, lr=1e-3), rs_bits=8, ag_bits=8)
    start = torch.randint(0, 512, (8, 1), device="cuda")
    tok = (start + torch.arange(65, device="cuda")) % 512
    losses = []
    for _ in range(30):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            _, loss = sdp(tok[:, :-1], tok[:, 1:])
        loss.backward()
        sdp.step()
        losses.append(float(loss))
    assert losses[-1] < losses[0] - 1.0
    assert torch.isfinite(sdp.flat_param).all()
    # working parameters = decoded master (+ the all-gather residual keeps the difference small)
    lo = sdp.rank * sdp.shard
    diff = (sdp.flat_param[lo : lo + sdp.shard] - sdp.master.detach()).abs().max()
    assert float(diff) < 0.02 * float(sdp.master.detach().abs().max())
    dist.destroy_process_group()


@pytest.mark.parametrize("algo", ["twoshot", "oneshot"])
def test_graph_replay_matches_eager_and_advances_device_epoch(cuda, algo):
    """A captured launch replayed K times equals K eager launches bit for bit
    (error feedback carried across them) and advances the device-side epoch."""
    n = 200003
    xs = [_x(n, seed=40 + i) for i in range(4)]
    ce = Communicator.create_local(0, workspace_bytes=64 << 20)
    r_e = torch.zeros(n, device="cuda")
    outs_e = []
    for x in xs:
        t = x.cuda()
        ce.all_reduce(t, bits=4, algo=algo, residual=r_e, post_scale=0.5)
        outs_e.append(t.clone())

    c = Communicator.create_local(0, workspace_bytes=64 << 20)
    c.set_timeout(5.0)
    static = torch.zeros(n, device="cuda")
    r_g = torch.zeros(n, device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        c.all_reduce(static, bits=4, algo=algo, residual=r_g, post_scale=0.5)
    torch.cuda.synchronize()
    e0 = c.native.device_epoch()
    outs_g = []
    for x in xs:
        static.copy_(x.cuda())
        g.replay()
        outs_g.append(static.clone())
    torch.cuda.synchronize()
    c.check()
    assert c.native.device_epoch() == e0 + len(xs)
    for a, b in zip(outs_e, outs_g):
        assert torch.equal(a, b)
    assert torch.equal(r_e, r_g)
    # eager launches after the replays still find fresh epochs
    t = xs[0].cuda()
    c.all_reduce(t, bits=4, algo=algo)
    torch.cuda.synchronize()
    c.check()
    assert c.native.device_epoch() == e0 + len(xs) + 1


def test_graph_replays_draw_fresh_stochastic_rounding(cuda):
    c = Communicator.create_local(0, workspace_bytes=64 << 20)
    c.set_timeout(5.0)
    x = torch.full((1 << 16,), 0.3, device="cuda")
    x[::1024] = 1.0  # block absmax 1.0: 0.3 sits between two 2-bit codes
    static = x.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        c.all_reduce(static, bits=2, algo="oneshot", stochastic_rounding=True, seed=3)
    outs = []
    for _ in range(2):
        static.copy_(x)
        g.replay()
        outs.append(static.clone())
    torch.cuda.synchronize()
    c.check()
    assert not torch.equal(outs[0], outs[1])
    mask = torch.ones_like(x, dtype=torch.bool)
    mask[::1024] = False
    for o in outs:  # unbiased
        assert abs(float(o[mask].mean()) - 0.3) < 0.01


@pytest.mark.parametrize("algo", ["twoshot", "oneshot"])
def test_allreduce_bf16_residual(comm, algo):
    """bf16 error-feedback residual: read as bf16, summed in fp32, the new
    residual rounded to bf16 (round to nearest even)."""
    n = 123457
    x = _x(n, seed=77)
    r = (torch.randn(n) * 1e-4).to(torch.bfloat16)
    t, rg = x.cuda(), r.cuda()
    comm.all_reduce(t, bits=4, algo=algo, residual=rg)
    torch.cuda.synchronize()
    model = emu.allreduce_two_shot if algo == "twoshot" else emu.allreduce_one_shot
    exp, res = model([x], 4, residuals=[r.float()])
    assert torch.equal(t.cpu(), exp)
    assert rg.dtype == torch.bfloat16
    assert torch.equal(rg.cpu(), res[0].to(torch.bfloat16))


def test_sharded_dp_checkpoint_roundtrip(cuda):
    import datetime
    import os

    import torch.distributed as dist

    from bitscom_b200.models import gpt2_small_test
    from bitscom_b200.parallel.fsdp import LowBitShardedDP

    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29657")
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
    try:
        tok = (torch.randint(0, 512, (4, 1), device="cuda") + torch.arange(33, device="cuda")) % 512

        def make():
            torch.manual_seed(0)
            return LowBitShardedDP(gpt2_small_test(n_positions=64).cuda(), lambda ps: torch.optim.AdamW(ps, lr=1e-3),
                                   rs_bits=8, ag_bits=8, residual_dtype=torch.bfloat16)

        def train(sdp, k):
            out = []
            for _ in range(k):
                _, loss = sdp(tok[:, :-1], tok[:, 1:])
                loss.backward()
                sdp.step()
                out.append(float(loss))
            return out

        a = make()
        train(a, 3)
        ck = a.state_dict_shard()
        ref = train(a, 3)
        b = make()
        b.load_state_dict_shard(ck)
        got = train(b, 3)
        # same trajectory (attention backward may use atomics: allow rounding noise)
        for x, y in zip(got, ref):
            assert abs(x - y) <= 1e-3 * abs(y)
        torch.testing.assert_close(b.master.detach(), a.master.detach(), rtol=1e-3, atol=1e-4)
    finally:
        dist.destroy_process_group()


def test_workspace_guard_bytes_intact(comm):
    """Runs after the other tests that share the module communicator: no
    launch wrote into the guard bytes after the flag arrays or at the end of a
    data region."""
    x = torch.randn(comm.native.max_elems_per_launch(0, 1), device="cuda")  # the largest 1-bit two-shot launch
    comm.all_reduce(x, bits=1, algo="twoshot")
    comm.all_reduce(x[: 1 << 20], bits=16, algo="oneshot")
    torch.cuda.synchronize()
    assert comm.check_canaries() == 0


def test_launch_timing_in_stats(cuda):
    c = Communicator.create_local(0, workspace_bytes=64 << 20)
    c.set_timing(True)
    t = torch.randn(1 << 20, device="cuda")
    for _ in range(3):
        c.all_reduce(t, bits=4, algo="twoshot")
    torch.cuda.synchronize()
    s = c.stats()
    assert s["launches"] == 3 and s["timed_launches"] == 3
    assert s["kernel_ms"] > 0.0
    c.set_timing(False)
    c.all_reduce(t, bits=4)
    torch.cuda.synchronize()
    assert c.stats()["timed_launches"] == 3


@pytest.mark.parametrize("algo", ["twoshot", "oneshot"])
@pytest.mark.parametrize("n", [1000, 50001, 3 * 8192 + 5])
def test_sign_1bit_allreduce_matches_model(comm, algo, n):
    """Opt-in sign-magnitude 1-bit format (mean-|x| block scale) with error
    feedback, bit-exact against the CPU model."""
    x = _x(n, seed=90 + n)
    r = torch.randn(n) * 1e-4
    t, rg = x.cuda(), r.cuda()
    comm.all_reduce(t, bits=1, fmt="sign", algo=algo, residual=rg, post_scale=0.5)
    torch.cuda.synchronize()
    comm.check()
    model = emu.allreduce_two_shot if algo == "twoshot" else emu.allreduce_one_shot
    exp, res = model([x], 1, residuals=[r], post_scale=0.5, fmt="sign")
    assert torch.equal(t.cpu(), exp)
    assert torch.equal(rg.cpu(), res[0])


def test_sign_1bit_reduce_scatter_all_gather(comm):
    n = 20001
    x = _x(n, seed=11)
    out = torch.empty(n, device="cuda")
    comm.reduce_scatter(out, x.cuda(), bits=1, fmt="sign")
    g = torch.empty(n, device="cuda")
    comm.all_gather(g, x.cuda(), bits=1, fmt="sign")
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), emu.reduce_scatter([x], 1, fmt="sign")[0])
    assert torch.equal(g.cpu(), emu.all_gather([x], 1, fmt="sign"))


def test_launches_on_two_streams_are_ordered():
    """One communicator used from two streams (a DDP hook's comm stream and a
    LowBitGroup call on the current stream): each launch waits for the
    previous one, so the shared workspace and counters are never used by two
    launches at once; every result is bit-exact against the model."""
    c = Communicator.create_local(0, workspace_bytes=64 << 20)
    side = torch.cuda.Stream()
    cur = torch.cuda.current_stream()
    xs = [_x(4_000_000 if i % 2 == 0 else 50_001, seed=100 + i) for i in range(6)]
    rs = [torch.randn(x.numel()) * 1e-4 for x in xs]
    ts = [x.cuda() for x in xs]
    rgs = [r.cuda() for r in rs]
    side.wait_stream(cur)
    for i, (t, rg) in enumerate(zip(ts, rgs)):
        with torch.cuda.stream(side if i % 2 == 0 else cur):
            c.all_reduce(t, bits=4, residual=rg, algo="twoshot")
    cur.wait_stream(side)
    torch.cuda.synchronize()
    c.check()
    for x, r, t, rg in zip(xs, rs, ts, rgs):
        exp, res = emu.allreduce_two_shot([x], 4, residuals=[r])
        assert torch.equal(t.cpu(), exp)
        assert torch.equal(rg.cpu(), res[0])


@pytest.fixture(scope="module")
def variant_pair():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    ws = Communicator.create_local(0, workspace_bytes=64 << 20)
    ws.set_kernel_variant("ws")
    reg = Communicator.create_local(0, workspace_bytes=64 << 20)
    reg.set_kernel_variant("reg")
    assert ws.kernel_variant == "ws" and reg.kernel_variant == "reg"
    return ws, reg


@pytest.mark.parametrize("op", ["twoshot", "oneshot", "reduce_scatter", "all_gather"])
@pytest.mark.parametrize("bits,fmt", [(1, "int"), (1, "sign"), (2, "int"), (4, "int"), (8, "e4m3"), (12, "int"), (16, "int")])
@pytest.mark.parametrize("dtype,res_dtype", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                             (torch.float16, None)])
@pytest.mark.parametrize("offset", [0, 1])
def test_warp_specialised_kernel_matches_register_kernel(variant_pair, op, bits, fmt, dtype, res_dtype, offset):
    """The warp-specialised kernel (bulk-copy stage ring) and the register
    kernel produce identical outputs and residuals; offset 1 makes every
    pointer unaligned, so the staged path falls back to direct loads."""
    ws, reg = variant_pair
    n = 3 * 8192 * 5 + 4097
    base = _x(n + offset, seed=bits * 7 + offset, dtype=dtype).cuda()
    results = []
    for c in (ws, reg):
        x = base[offset:]
        r = None
        if res_dtype is not None:
            r = (torch.randn(n + offset, generator=torch.Generator().manual_seed(3)) * 1e-4).to(res_dtype).cuda()[offset:]
        if op in ("twoshot", "oneshot"):
            out = torch.empty(n + offset, dtype=dtype, device="cuda")[offset:]
            c.all_reduce(x, out=out, bits=bits, fmt=fmt, residual=r, algo=op, post_scale=0.5,
                         stochastic_rounding=(fmt == "int"), seed=7, offset=3)
        elif op == "reduce_scatter":
            out = torch.empty(n + offset, dtype=dtype, device="cuda")[offset:]
            c.reduce_scatter(out, x, bits=bits, fmt=fmt, residual=r, stochastic_rounding=(fmt == "int"), seed=7)
        else:
            out = torch.empty(n + offset, dtype=dtype, device="cuda")[offset:]
            c.all_gather(out, x, bits=bits, fmt=fmt, residual=r)
        torch.cuda.synchronize()
        c.check()
        results.append((out.cpu(), None if r is None else r.cpu()))
    assert torch.equal(results[0][0], results[1][0])
    if res_dtype is not None:
        assert torch.equal(results[0][1], results[1][1])


def test_warp_specialised_kernel_large_twoshot_matches_model(variant_pair):
    """Large sizes stage many sub-chunks per CTA: compare a multi-item launch
    against the CPU model."""
    ws, _ = variant_pair
    n = 8192 * 600 + 123
    x = _x(n, seed=42)
    r = torch.randn(n) * 1e-4
    t, rg = x.cuda(), r.cuda()
    ws.all_reduce(t, bits=4, residual=rg, algo="twoshot")
    torch.cuda.synchronize()
    ws.check()
    exp, res = emu.allreduce_two_shot([x], 4, residuals=[r])
    assert torch.equal(t.cpu(), exp)
    assert torch.equal(rg.cpu(), res[0])
