"""Tuning table of the fused collectives.

The table is a JSON file (``b200.json`` beside this module, or the file named
by ``BITSCOM_TUNING_FILE``) with

* ``oneshot_max_packed_bytes``: per world size, the largest packed message,
  in bytes per rank, for which the one-shot all-reduce is chosen
  automatically (larger messages use the two-shot form);
* ``entries``: per (world size, bitwidth, wire format) overrides measured on
  the device: ``oneshot_max_packed_bytes`` and ``ws_min_packed_bytes`` (the
  packed size from which the warp-specialised kernel runs instead of the
  register kernel; -1 or absent: never).

* ``schedule_lag``: per world size, the chunk-group lag of the fused
  kernel's work order (0: phase-major).

``BITSCOM_ALGO=oneshot|twoshot``, ``BITSCOM_KERNEL=ws|reg`` and
``BITSCOM_SCHED_LAG`` override the automatic choices altogether (read by the
native communicator).
"""

from __future__ import annotations

import json
import os
from functools import lru_cache
from typing import Optional

_DEFAULT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "b200.json")
FALLBACK_ONESHOT_MAX_BYTES = 512 << 10


@lru_cache(maxsize=8)
def load_table(path: Optional[str] = None) -> dict:
    path = path or os.environ.get("BITSCOM_TUNING_FILE") or _DEFAULT
    with open(path, encoding="utf-8") as fh:
        table = json.load(fh)
    if not isinstance(table, dict):
        raise ValueError(f"tuning table {path} is not a JSON object")
    return table


def oneshot_max_bytes(world: int, path: Optional[str] = None) -> int:
    """Automatic one-shot/two-shot threshold (packed bytes per rank) for `world` ranks."""
    try:
        table = load_table(path)
    except (OSError, ValueError):
        return FALLBACK_ONESHOT_MAX_BYTES
    per_world = table.get("oneshot_max_packed_bytes", {})
    v = per_world.get(str(int(world)), table.get("default_oneshot_max_packed_bytes", FALLBACK_ONESHOT_MAX_BYTES))
    return int(v)


FMTS = {"int": 0, "e4m3": 1, "sign": 2}


def entries(world: int, path: Optional[str] = None):
    """[(bits, fmt_code, oneshot_max_bytes, ws_min_bytes)] of the table's
    per-format entries for ``world`` ranks (-1 = no value)."""
    try:
        table = load_table(path)
    except (OSError, ValueError):
        return []
    out = []
    for e in table.get("entries", []):
        if int(e.get("world", -1)) != int(world):
            continue
        out.append((int(e["bits"]), FMTS[e.get("fmt", "int")], int(e.get("oneshot_max_packed_bytes", -1)),
                    int(e.get("ws_min_packed_bytes", -1))))
    return out


def schedule_lag(world: int, path: Optional[str] = None) -> Optional[int]:
    """Measured schedule lag for ``world`` ranks, or None (keep the default)."""
    try:
        table = load_table(path)
    except (OSError, ValueError):
        return None
    v = table.get("schedule_lag", {}).get(str(int(world)))
    return None if v is None else int(v)
