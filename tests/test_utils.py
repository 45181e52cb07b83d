"""Trace analyzer, EF-benchmark arithmetic and the sharded-DP module on CPU."""

import json
import os
import subprocess
import sys

import pytest
import torch

from bitscom_b200.utils.trace import analyze, step_window

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _trace():
    ev = []
    for i in range(4):
        t0 = i * 1000
        ev.append({"ph": "X", "name": f"ProfilerStep#{i}", "ts": t0, "dur": 900})
        ev.append({"ph": "X", "name": "aten::conv2d", "ts": t0 + 10, "dur": 500, "cat": "cpu_op"})
        ev.append({"ph": "X", "name": "lowbit_coll_kernel<float, 4, 0>", "ts": t0 + 600, "dur": 200, "cat": "kernel"})
        ev.append({"ph": "X", "name": "nccl:broadcast", "ts": t0 + 820, "dur": 50, "cat": "cpu_op"})
    return ev


def test_trace_window_and_comm_share():
    ev = _trace()
    w = step_window(ev, skip_steps=1, keep_steps=2)
    assert w.start_us == 1000 and w.end_us == 2900
    res = analyze(ev, w)
    assert res["total_op_us"] == 2 * 750 and res["comm_us"] == 2 * 250
    assert abs(res["comm_share"] - 250 / 750) < 1e-9
    gpu = analyze(ev, w, gpu_only=True)
    assert gpu["comm_share"] == 1.0


def test_trace_cli(tmp_path):
    path = tmp_path / "t.json"
    path.write_text(json.dumps({"traceEvents": _trace()}))
    out = subprocess.run([sys.executable, os.path.join(ROOT, "benchmarks", "analyze_trace.py"), str(path)],
                         capture_output=True, text=True, check=True).stdout
    assert json.loads(out.splitlines()[0])["comm_us"] == 3 * 250


def test_ef_benefit_curve_cpu_shows_ef_gain():
    sys.path.insert(0, os.path.join(ROOT, "benchmarks"))
    from error_feedback_comparison import ef_benefit_curve

    rows = ef_benefit_curve(torch.device("cpu"), 4, 40, 1 << 14, 0)
    assert rows[-1][2] < rows[-1][1] / 3  # EF cumulative error far below no-EF


def test_graphed_step_rejects_bad_inputs():
    import pytest
    import torch

    from bitscom_b200.parallel.graphs import GraphedStep

    with pytest.raises(ValueError):
        GraphedStep(lambda: None, [])
    with pytest.raises(ValueError):
        GraphedStep(lambda x: x, [torch.zeros(3)])  # CPU tensors cannot be captured


def test_hook_state_residual_dtype():
    import pytest
    import torch

    from bitscom_b200.parallel.hooks import LowBitHookState

    s = LowBitHookState(residual_dtype=torch.bfloat16)
    buf = torch.zeros(10)
    r = s.residual(0, buf)
    assert r.dtype == torch.bfloat16 and r.numel() == 10
    s.residual_dtype = torch.float32
    assert s.residual(0, buf).dtype == torch.float32  # converted on the next use
    with pytest.raises(ValueError):
        LowBitHookState(residual_dtype=torch.float16)


def test_tuning_table_thresholds(tmp_path, monkeypatch):
    import json

    from bitscom_b200 import tuning

    tuning.load_table.cache_clear()
    assert tuning.oneshot_max_bytes(8) == 524288  # shipped B200 table
    assert tuning.oneshot_max_bytes(3) == tuning.load_table()["default_oneshot_max_packed_bytes"]
    f = tmp_path / "t.json"
    f.write_text(json.dumps({"oneshot_max_packed_bytes": {"2": 1234}, "default_oneshot_max_packed_bytes": 99}))
    monkeypatch.setenv("BITSCOM_TUNING_FILE", str(f))
    tuning.load_table.cache_clear()
    assert tuning.oneshot_max_bytes(2) == 1234
    assert tuning.oneshot_max_bytes(8) == 99
    monkeypatch.setenv("BITSCOM_TUNING_FILE", str(tmp_path / "missing.json"))
    tuning.load_table.cache_clear()
    assert tuning.oneshot_max_bytes(2) == tuning.FALLBACK_ONESHOT_MAX_BYTES
    tuning.load_table.cache_clear()


def test_tuning_table_entries(tmp_path, monkeypatch):
    """Per (world, bits, format) entries: selected by world size, formats
    mapped to the native codes, missing values as -1."""
    import json

    from bitscom_b200 import tuning

    f = tmp_path / "t.json"
    f.write_text(json.dumps({"entries": [
        {"world": 8, "bits": 4, "fmt": "int", "oneshot_max_packed_bytes": 65536, "ws_min_packed_bytes": 1 << 24},
        {"world": 8, "bits": 8, "fmt": "e4m3", "oneshot_max_packed_bytes": 131072},
        {"world": 2, "bits": 2, "fmt": "int", "ws_min_packed_bytes": 0},
    ]}))
    monkeypatch.setenv("BITSCOM_TUNING_FILE", str(f))
    tuning.load_table.cache_clear()
    assert tuning.entries(8) == [(4, 0, 65536, 1 << 24), (8, 1, 131072, -1)]
    assert tuning.entries(2) == [(2, 0, -1, 0)]
    assert tuning.entries(4) == []
    tuning.load_table.cache_clear()


def test_sign_block_model_scale_and_error():
    """CPU model of the sign-magnitude 1-bit format: the block scale is the
    mean |x| (summed in the kernel's order), and on N(0, 1) data one 1-bit
    sign pass has relative L2 error sqrt(1 - 2/pi) ~ 0.60, far below the
    reference's unsigned 1-bit codes, which zero every negative value."""
    import math

    import torch

    from tests import wire_emulator as emu

    g = torch.Generator().manual_seed(0)
    x = torch.randn(64 * 1024, generator=g)
    scale = emu._block_mean_abs(x.view(-1, 1024)).view(-1)
    torch.testing.assert_close(scale, x.view(-1, 1024).abs().mean(dim=1), rtol=1e-5, atol=0)
    d = emu.block_quant(x, 1, "sign")
    assert torch.equal(d.abs().view(-1, 1024), scale.unsqueeze(1).expand(-1, 1024))
    rel = float((d - x).norm() / x.norm())
    assert abs(rel - math.sqrt(1 - 2 / math.pi)) < 0.01
    rel_unsigned = float((emu.block_quant(x, 1, "int") - x).norm() / x.norm())
    assert rel_unsigned > rel + 0.1


def test_clock_sampler_summary_from_rows():
    """The clock summary attached to bench lines: median SM clock over samples
    under load, the max clock, and every throttle reason seen active."""
    from bitscom_b200.utils.clocks import ClockSampler

    cs = ClockSampler([0])
    cs.rows = [
        ["0", "1965", "1965", "300", "5", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"],
        ["0", "1800", "1965", "990", "100", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
        ["0", "1700", "1965", "995", "99", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
        ["0", "1750", "1965", "998", "97", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"],
    ]
    s = cs.summary()
    assert s["sm_mhz"] == 1750 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]
    assert ClockSampler([0]).summary()["reasons"] == ["unsampled"]


def test_trace_ranges_only_while_profiling():
    import contextlib

    import torch

    from bitscom_b200.parallel.comm import _trace_range
    from bitscom_b200.utils.trace import is_comm

    assert isinstance(_trace_range("all_reduce"), contextlib.nullcontext)
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU]) as prof:
        with _trace_range("all_reduce"):
            torch.ones(3).add_(1)
    names = [e.name for e in prof.events()]
    assert "lowbit:all_reduce" in names and is_comm("lowbit:all_reduce")


def test_info_entry_point_runs():
    from bitscom_b200.__main__ import info

    d = info()
    assert d["bitscom_b200"] and "tuning" in d and isinstance(d["devices"], list)


def test_tuning_table_crossover_from_sweep_rows():
    """make_tuning_table: the one-shot threshold is the largest packed size
    at which one-shot won with two-shot winning at every larger size (an
    isolated small-size loss does not cut it short); always-two-shot formats
    get 0."""
    import importlib.util
    from pathlib import Path

    path = Path(__file__).resolve().parents[1] / "benchmarks" / "make_tuning_table.py"
    spec = importlib.util.spec_from_file_location("make_tuning_table", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)

    def row(algo, mb, ms, bits=4, fmt="int", world=8):
        return {"impl": "ours", "algo": algo, "bits": bits, "fmt": fmt, "world": world,
                "bytes_fp32": mb << 20, "ms": ms}

    rows = [row("oneshot", 1, 0.03), row("twoshot", 1, 0.02),  # a noisy small-size sample
            row("oneshot", 2, 0.02), row("twoshot", 2, 0.02),
            row("oneshot", 4, 0.05), row("twoshot", 4, 0.03),
            row("oneshot", 8, 0.06), row("twoshot", 8, 0.05),
            row("oneshot", 1, 0.03, bits=8, fmt="e4m3"), row("twoshot", 1, 0.02, bits=8, fmt="e4m3"),
            {"impl": "nccl", "bits": 32, "fmt": "fp32", "world": 8, "bytes_fp32": 1 << 20, "ms": 0.01}]
    cross = mod.crossover(rows)
    assert cross == {(8, 4, "int"): (2 << 20) // 4 * 4 // 8, (8, 8, "e4m3"): 0}
