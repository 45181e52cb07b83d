"""``python -m bitscom_b200``: what this installation can do on this machine.

Prints the package and extension versions, where the native extension was
loaded from, the CUDA devices with their SM count, the peer-access matrix
(the fused collectives need every pair of ranks on one node to reach each
other's memory), and the tuning table in use.  Reads state only.
"""

from __future__ import annotations

import json
import sys


def info() -> dict:
    import torch

    from . import __version__, _ext
    from .tuning import load_table

    out = {
        "bitscom_b200": __version__,
        "torch": torch.__version__,
        "extension": getattr(_ext._C, "__file__", None) if _ext.HAS_EXT else f"not loaded: {_ext.IMPORT_ERROR!r}",
        "cuda_available": torch.cuda.is_available(),
        "devices": [],
        "peer_access": [],
    }
    if torch.cuda.is_available():
        n = torch.cuda.device_count()
        for d in range(n):
            p = torch.cuda.get_device_properties(d)
            out["devices"].append({"index": d, "name": p.name, "sm_count": p.multi_processor_count,
                                   "memory_gb": round(p.total_memory / 2**30, 1), "capability": f"{p.major}.{p.minor}"})
        out["peer_access"] = [[a == b or torch.cuda.can_device_access_peer(a, b) for b in range(n)] for a in range(n)]
    try:
        out["tuning"] = load_table()
    except (OSError, ValueError) as exc:
        out["tuning"] = f"unavailable: {exc!r}"
    import os

    out["kernel"] = {
        "variant": os.environ.get("BITSCOM_KERNEL", "auto (register kernel unless a tuning entry selects the "
                                                     "warp-specialised one)"),
        "algo": os.environ.get("BITSCOM_ALGO", "auto"),
        "workspace_mb": int(os.environ.get("BITSCOM_WORKSPACE_MB", "256")),
    }
    ref = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref",
                       "bitscom_b200_install.json")
    if os.path.exists(ref):
        with open(ref, encoding="utf-8") as fh:
            out["reference_build"] = json.load(fh)
    return out


def main(argv=None) -> int:
    json.dump(info(), sys.stdout, indent=1)
    sys.stdout.write("\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
