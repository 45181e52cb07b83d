"""LowBitGroup dispatch with a fake torch.distributed (reference
tests/test_api.py covers the same behaviour for the reference package)."""

from types import SimpleNamespace

import pytest
import torch

from bitscom_b200.api import LowBitGroup


class DummyWork:
    def __init__(self):
        self.wait_called = 0

    def wait(self):
        self.wait_called += 1
        return True


@pytest.fixture
def fake_dist(monkeypatch):
    calls = {}
    default_group = object()

    def fake_a2a_single(output, input, group=None, async_op=False):
        calls.setdefault("all_to_all_single", []).append(group)
        output.copy_(input)
        return DummyWork()

    def fake_all_gather_into_tensor(output, input, group=None, async_op=False):
        calls.setdefault("all_gather_into_tensor", []).append(group)
        output.copy_(input.repeat(output.numel() // input.numel()))
        return DummyWork()

    def make(name):
        def _fn(*args, **kwargs):
            calls[name] = {"args": args, "kwargs": kwargs}
            return DummyWork()

        return _fn

    t = "bitscom_b200.api.dist"
    monkeypatch.setattr(f"{t}.distributed_c10d._get_default_group", lambda: default_group)
    monkeypatch.setattr(f"{t}.get_rank", lambda group=None: 1)
    monkeypatch.setattr(f"{t}.get_world_size", lambda group=None: 8)
    for name in ("all_reduce", "all_gather", "reduce_scatter", "broadcast"):
        monkeypatch.setattr(f"{t}.{name}", make(name))
    monkeypatch.setattr(f"{t}.all_to_all_single", fake_a2a_single)
    monkeypatch.setattr(f"{t}.all_gather_into_tensor", fake_all_gather_into_tensor)
    return SimpleNamespace(calls=calls, default_group=default_group)


def test_uses_default_group(fake_dist):
    g = LowBitGroup(bitwidth=4)
    assert g.pg is fake_dist.default_group and g.rank == 1 and g.world_size == 8


@pytest.mark.parametrize("bad", [0, 3, 15, 17])
def test_rejects_unsupported_bitwidth(bad):
    with pytest.raises(ValueError):
        LowBitGroup(bitwidth=bad, process_group=object())


def test_all_reduce_sync_waits(fake_dist):
    g = LowBitGroup(bitwidth=8, process_group=object())
    assert g.all_reduce(torch.ones(16), async_op=False) is None
    assert fake_dist.calls["all_reduce"]["kwargs"]["async_op"] is True


def test_all_reduce_async_returns_work(fake_dist):
    g = LowBitGroup(bitwidth=8, process_group=object())
    assert isinstance(g.all_reduce(torch.ones(16), async_op=True), DummyWork)


def test_simulate_quantization_changes_values(fake_dist):
    g = LowBitGroup(bitwidth=2, process_group=object(), simulate_quantization=True)
    t = torch.linspace(-1.0, 1.0, 128)
    before = t.clone()
    # 2-bit on world 8 takes the low-bit path; force the fp branch with MAX
    g.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    assert not torch.equal(before, t)


def test_compress_decompress_methods(fake_dist):
    g = LowBitGroup(bitwidth=8, process_group=object())
    x = torch.randn(32)
    y = g.decompress(g.compress(x))
    assert y.shape == x.shape and y.dtype == x.dtype


def test_lowbit_path_uses_two_all_to_all_and_two_all_gathers(fake_dist, monkeypatch):
    monkeypatch.setattr("bitscom_b200.api.dist.get_world_size", lambda group=None: 2)
    monkeypatch.setattr("bitscom_b200.api.dist.get_rank", lambda group=None: 0)
    g = LowBitGroup(bitwidth=4, process_group=object())
    t = torch.tensor([0.0, 1.0])
    g.all_reduce(t)
    assert "all_reduce" not in fake_dist.calls
    assert len(fake_dist.calls["all_to_all_single"]) == 2
    assert len(fake_dist.calls["all_gather_into_tensor"]) == 2


def test_non_sum_falls_back_to_regular_allreduce(fake_dist, monkeypatch):
    monkeypatch.setattr("bitscom_b200.api.dist.get_world_size", lambda group=None: 2)
    g = LowBitGroup(bitwidth=4, process_group=object())
    g.all_reduce(torch.tensor([0.0, 1.0]), op=torch.distributed.ReduceOp.MAX)
    assert "all_reduce" in fake_dist.calls


def test_non_divisible_numel_is_handled(fake_dist, monkeypatch):
    monkeypatch.setattr("bitscom_b200.api.dist.get_world_size", lambda group=None: 2)
    g = LowBitGroup(bitwidth=4, process_group=object())
    t = torch.tensor([0.0, 1.0, 2.0])
    g.all_reduce(t)
    assert t.shape == (3,)


def test_pipeline_a_dispatch(fake_dist, monkeypatch):
    monkeypatch.setattr("bitscom_b200.api.dist.get_world_size", lambda group=None: 2)
    called = {}

    def fake_pipeline(self, tensor, *, local_group, inter_group, chunk_size, local_quantize):
        called.update(chunk_size=chunk_size, local_quantize=local_quantize)
        tensor.add_(1.0)

    monkeypatch.setattr("bitscom_b200.api.LowBitGroup._hierarchical_lowbit_allreduce_pipeline_a", fake_pipeline)
    g = LowBitGroup(bitwidth=4, process_group=object())
    t = torch.tensor([0.0, 1.0])
    g.all_reduce(t, local_group=object(), inter_group=object(), chunk_size=32)
    assert called == {"chunk_size": 32, "local_quantize": False}
    assert torch.allclose(t, torch.tensor([1.0, 2.0]))


def test_local_group_only_uses_full_precision(fake_dist, monkeypatch):
    monkeypatch.setattr("bitscom_b200.api.dist.get_world_size", lambda group=None: 2)
    g = LowBitGroup(bitwidth=4, process_group=object())
    local = object()
    g.all_reduce(torch.tensor([0.0, 1.0]), local_group=local, inter_group=None, chunk_size=16)
    assert fake_dist.calls["all_reduce"]["kwargs"]["group"] is local


def test_local_group_only_quantized_path(fake_dist, monkeypatch):
    monkeypatch.setattr("bitscom_b200.api.dist.get_world_size", lambda group=None: 2)
    seen = {}

    def fake_group_reduce(self, flat, group):
        seen["group"] = group
        return flat + 2.0

    monkeypatch.setattr("bitscom_b200.api.LowBitGroup._lowbit_allreduce_via_alltoall_group", fake_group_reduce)
    g = LowBitGroup(bitwidth=4, process_group=object())
    local = object()
    t = torch.tensor([0.0, 1.0])
    g.all_reduce(t, local_group=local, local_quantize=True)
    assert seen["group"] is local and torch.allclose(t, torch.tensor([2.0, 3.0]))


def test_dual_stream_guard():
    g = LowBitGroup.__new__(LowBitGroup)
    assert g._should_use_dual_stream_pipeline(is_cuda=True, local_size=8, global_size=8) is False
    assert g._should_use_dual_stream_pipeline(is_cuda=True, local_size=4, global_size=8) is True
    assert g._should_use_dual_stream_pipeline(is_cuda=False, local_size=4, global_size=8) is False


def test_staged_allreduce_matches_reference_arithmetic(fake_dist, monkeypatch):
    """With the identity all-to-all / all-gather fakes (every rank = rank 0's
    data), the staged path must equal the reference's C8 arithmetic."""
    from . import ref_oracle

    ref = ref_oracle.load()
    monkeypatch.setattr("bitscom_b200.api.dist.get_world_size", lambda group=None: 1)
    x = torch.randn(1031)
    g = LowBitGroup(bitwidth=4, process_group=object())
    out = g._staged_allreduce(x, object(), None)
    q, s = ref.quantize_tensor(x, 4)
    d = ref.dequantize_tensor(q, s)
    q2, s2 = ref.quantize_tensor(d, 4)
    exp = ref.dequantize_tensor(q2, s2)
    assert torch.equal(out, exp)


def test_error_feedback_residual_persists(fake_dist, monkeypatch):
    monkeypatch.setattr("bitscom_b200.api.dist.get_world_size", lambda group=None: 2)
    g = LowBitGroup(bitwidth=2, process_group=object(), error_feedback=True)
    t = torch.randn(64)
    g.all_reduce(t.clone(), ef_key="bucket0")
    r = g._residuals["bucket0"].clone()
    assert r.abs().sum() > 0
    g.all_reduce(t.clone(), ef_key="bucket0")
    assert not torch.equal(r, g._residuals["bucket0"])


@pytest.mark.parametrize("use_key", [False, True])
def test_error_feedback_checkpoint_resume_is_bit_identical(fake_dist, monkeypatch, use_key):
    """A LowBitGroup restored from state_dict() continues exactly like the
    uninterrupted run: residuals come back under their ef_key, or by order
    of first use for tensors all-reduced without a key (new tensor objects
    in the resumed process)."""
    monkeypatch.setattr("bitscom_b200.api.dist.get_world_size", lambda group=None: 2)
    torch.manual_seed(0)
    grads = [[torch.randn(257), torch.randn(64)] for _ in range(4)]
    kw = {"bitwidth": 2, "process_group": object(), "error_feedback": True, "stochastic_rounding": True}

    def run(group, steps, bufs):
        outs = []
        for step in steps:
            for i, buf in enumerate(bufs):
                buf.copy_(grads[step][i])
                group.all_reduce(buf, ef_key=(f"b{i}" if use_key else None))
                outs.append(buf.clone())
        return outs

    full = LowBitGroup(**kw)
    exp = run(full, range(4), [torch.empty(257), torch.empty(64)])
    first = LowBitGroup(**kw)
    got = run(first, range(2), [torch.empty(257), torch.empty(64)])
    ck = first.state_dict()
    resumed = LowBitGroup(**kw)
    resumed.load_state_dict(ck)
    got += run(resumed, range(2, 4), [torch.empty(257), torch.empty(64)])  # new buffers
    assert len(got) == len(exp)
    for a, b in zip(got, exp):
        assert torch.equal(a, b)
    assert resumed.state_dict()["calls"] == full.state_dict()["calls"]


def test_hook_residuals_follow_bucket_parameters():
    """Hook residuals are keyed by bucket index and parameter signature: a
    rebuilt bucket with the same size but another parameter order starts from
    zero (and the stale residual of that index is dropped); a checkpoint
    restores residuals under the same keys."""
    from bitscom_b200.parallel.hooks import LowBitHookState

    params = [torch.nn.Parameter(torch.zeros(3)), torch.nn.Parameter(torch.zeros(3)), torch.nn.Parameter(torch.zeros(4))]

    class Bucket:
        def __init__(self, idx, ps):
            self._i, self._p = idx, ps

        def index(self):
            return self._i

        def parameters(self):
            return self._p

    s = LowBitHookState()
    s.set_parameter_order(params)
    b0 = Bucket(0, [params[0], params[1]])
    buf = torch.zeros(6)
    r = s.residual(0, buf, s.bucket_signature(b0))
    r.fill_(1.0)
    assert s.bucket_signature(b0) == (0, 1)
    assert torch.equal(s.residual(0, buf, s.bucket_signature(b0)), torch.ones(6))
    b0r = Bucket(0, [params[1], params[0]])  # rebuilt: same size, other order
    r2 = s.residual(0, buf, s.bucket_signature(b0r))
    assert torch.equal(r2, torch.zeros(6)) and len(s.residuals) == 1
    r2.fill_(2.0)
    t = LowBitHookState()
    t.set_parameter_order(params)
    t.load_state_dict(s.state_dict())
    assert torch.equal(t.residual(0, buf, t.bucket_signature(b0r)), torch.full((6,), 2.0))
    u = LowBitHookState()  # no parameter order: shapes stand in for indices
    assert u.bucket_signature(b0) == ((3,), (3,))
