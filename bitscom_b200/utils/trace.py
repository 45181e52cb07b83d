"""Chrome-trace analysis: communication share over a stable window of steps.

Counterpart of reference benchmarks/analyze_trace_stable_window.py: load a
``torch.profiler`` Chrome trace, pick a window of ``ProfilerStep#`` events
(skipping warm-up steps), sum the duration of complete ("X") events that fall
inside it, and attribute communication by name prefix.  The prefix set adds
this library's markers (``lowbit:`` record_function ranges of the backend and
the ``lowbit_coll_kernel`` / quantisation kernels) to NCCL's and gloo's.
"""

from __future__ import annotations

import json
from collections import Counter
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence

COMM_PREFIXES = ("nccl:", "gloo:", "lowbit:", "ncclDevKernel", "ncclKernel", "lowbit_coll_kernel",
                 "quantize_ref_kernel", "unpack_ref_kernel", "ef_roundtrip_kernel", "absmax_kernel")


@dataclass
class Window:
    start_us: float
    end_us: float

    @property
    def span_us(self) -> float:
        return self.end_us - self.start_us


def load_events(path: str) -> List[dict]:
    with open(path, encoding="utf-8") as fh:
        data = json.load(fh)
    return data.get("traceEvents", []) if isinstance(data, dict) else data


def complete_events(events: Iterable[dict]) -> List[dict]:
    out = [e for e in events if e.get("ph") == "X" and "ts" in e and "dur" in e]
    out.sort(key=lambda e: e["ts"])
    return out


def step_window(events: Sequence[dict], skip_steps: int = 1, keep_steps: int = 0) -> Window:
    steps = [e for e in complete_events(events) if str(e.get("name", "")).startswith("ProfilerStep")]
    if not steps:
        raise RuntimeError("no ProfilerStep events in trace")
    if skip_steps >= len(steps):
        raise RuntimeError(f"skip_steps={skip_steps} but the trace has {len(steps)} steps")
    last = len(steps) - 1 if keep_steps <= 0 else min(len(steps) - 1, skip_steps + keep_steps - 1)
    return Window(float(steps[skip_steps]["ts"]), float(steps[last]["ts"] + steps[last]["dur"]))


def time_window(events: Sequence[dict], skip_ratio: float = 0.2) -> Window:
    ops = complete_events(events)
    if not ops:
        raise RuntimeError("no complete events in trace")
    t0 = float(ops[0]["ts"])
    t1 = float(max(e["ts"] + e["dur"] for e in ops))
    return Window(t0 + (t1 - t0) * min(max(skip_ratio, 0.0), 0.95), t1)


def is_comm(name: str, prefixes: Sequence[str] = COMM_PREFIXES) -> bool:
    return any(name.startswith(p) or p in name for p in prefixes)


def analyze(events: Sequence[dict], window: Optional[Window] = None, *, gpu_only: bool = False,
            prefixes: Sequence[str] = COMM_PREFIXES, top_k: int = 15) -> Dict:
    """Summed op time inside the window, communication share, top ops."""
    if window is None:
        try:
            window = step_window(events)
        except RuntimeError:
            window = time_window(events)
    totals: Counter = Counter()
    comm = 0.0
    total = 0.0
    for e in complete_events(events):
        if e["ts"] < window.start_us or e["ts"] + e["dur"] > window.end_us:
            continue
        if gpu_only and e.get("cat") not in ("kernel", "gpu_memcpy", "gpu_memset"):
            continue
        name = str(e.get("name", ""))
        if name.startswith("ProfilerStep"):
            continue
        d = float(e["dur"])
        totals[name] += d
        total += d
        if is_comm(name, prefixes):
            comm += d
    return {
        "window_us": window.span_us,
        "total_op_us": total,
        "comm_us": comm,
        "comm_share": comm / total if total else 0.0,
        "top_ops": totals.most_common(top_k),
    }
