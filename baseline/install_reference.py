"""Builds the reference implementation (Aerithy/bitscom) from its own source
into ``baseline/_ref`` of this repository.

The reference arm of ``bench.py`` and the byte-compatibility oracle of the
tests (``tests/ref_oracle.py``) import the reference from there.  Steps:

1. the source location is ``reference_path`` of ``BASELINE.json`` (or
   ``--src`` / ``BITSCOM_REFERENCE_SRC``);
2. the source tree is copied to a staging directory under the system temp
   dir, and every shipped binary in the copy (``*.so``, ``*.pyc``,
   ``__pycache__``) is deleted first, so nothing that was not built here is
   ever installed or loaded;
3. the copy is built and installed with pip, offline::

       pip install --no-index --no-build-isolation --no-deps \\
           --find-links /opt/wheelhouse --target baseline/_ref <staging copy>

   with ``TORCH_CUDA_ARCH_LIST=10.0`` (the reference's setup.py passes no
   architecture of its own) and the system compiler (``/usr/bin/gcc``,
   ``/usr/bin/g++``): an image's default compiler wrapper that falls back to a
   static ``libstdc++.a`` gives each module a private C++ runtime that crashes
   the reference's backend on its first formatted integer.  ``--no-deps``
   because the reference declares ``torch>=2.0``, which the offline
   wheelhouse does not carry (the image's torch is used);
4. the result is checked (``bitscom/_lowbit_c*.so`` present, ``bitscom``
   importable) and a stamp file records the source and the build.

Usage::

    python baseline/install_reference.py            # no-op when already built
    python baseline/install_reference.py --force     # rebuild

Returns exit code 0 on success; on failure prints one line that starts with
``reference install failed:`` and exits 1.
"""

from __future__ import annotations

import argparse
import glob
import json
import os
import shutil
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TARGET = os.path.join(ROOT, "baseline", "_ref")
STAMP = os.path.join(TARGET, "bitscom_b200_install.json")
WHEELHOUSE = "/opt/wheelhouse"


def reference_source(cli: str | None = None) -> str | None:
    """Location of the reference's source tree: CLI, env, then BASELINE.json."""
    if cli:
        return cli
    env = os.environ.get("BITSCOM_REFERENCE_SRC")
    if env:
        return env
    try:
        with open(os.path.join(ROOT, "BASELINE.json"), encoding="utf-8") as f:
            return json.load(f).get("reference_path")
    except (OSError, ValueError):
        return None


def installed() -> bool:
    """True when baseline/_ref holds a reference build made from source here."""
    pkg = os.path.join(TARGET, "bitscom")
    return (os.path.isfile(os.path.join(pkg, "quantization.py"))
            and bool(glob.glob(os.path.join(pkg, "_lowbit_c*.so")))
            and os.path.isfile(STAMP))


def _strip_binaries(tree: str) -> list[str]:
    removed = []
    for dirpath, dirnames, filenames in os.walk(tree):
        for d in list(dirnames):
            if d == "__pycache__" or d.endswith(".egg-info") or d == "build":
                shutil.rmtree(os.path.join(dirpath, d))
                removed.append(os.path.join(dirpath, d))
                dirnames.remove(d)
        for fn in filenames:
            if fn.endswith((".so", ".pyc", ".pyo", ".o", ".a", ".cubin", ".fatbin")):
                os.remove(os.path.join(dirpath, fn))
                removed.append(os.path.join(dirpath, fn))
    return removed


def install(src: str, force: bool = False, jobs: int | None = None, quiet: bool = False) -> None:
    if installed() and not force:
        if not quiet:
            print(f"reference already built in {TARGET}")
        return
    if not src or not os.path.isfile(os.path.join(src, "setup.py")):
        raise RuntimeError(f"no reference source tree with a setup.py at {src!r}")
    stage_root = tempfile.mkdtemp(prefix="bitscom_ref_src_")
    stage = os.path.join(stage_root, "bitscom")
    try:
        # third_party holds only empty submodule mount points in the reference.
        shutil.copytree(src, stage, ignore=shutil.ignore_patterns("third_party", ".git"))
        removed = _strip_binaries(stage)
        if os.path.isdir(TARGET):
            shutil.rmtree(TARGET)
        os.makedirs(os.path.dirname(TARGET), exist_ok=True)
        env = dict(os.environ)
        env["TORCH_CUDA_ARCH_LIST"] = "10.0"
        env["MAX_JOBS"] = str(jobs or min(8, os.cpu_count() or 4))
        for var, path in (("CC", "/usr/bin/gcc"), ("CXX", "/usr/bin/g++")):
            if os.path.exists(path):
                env[var] = path
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps"]
        if os.path.isdir(WHEELHOUSE):
            cmd += ["--find-links", WHEELHOUSE]
        cmd += ["--target", TARGET, stage]
        t0 = time.time()
        proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
        if proc.returncode != 0:
            tail = (proc.stdout + proc.stderr)[-4000:]
            raise RuntimeError(f"pip exited {proc.returncode}:\n{tail}")
        pkg = os.path.join(TARGET, "bitscom")
        sos = sorted(os.path.basename(p) for p in glob.glob(os.path.join(pkg, "_lowbit_*.so")))
        if not any(s.startswith("_lowbit_c") and not s.startswith("_lowbit_cuda") for s in sos):
            raise RuntimeError(f"build finished but {pkg} holds no _lowbit_c extension (found {sos})")
        with open(STAMP, "w", encoding="utf-8") as f:
            json.dump({
                "source": os.path.abspath(src),
                "built": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
                "seconds": round(time.time() - t0, 1),
                "extensions": sos,
                "shipped_binaries_removed_before_build": len(removed),
                "command": " ".join(cmd[:-1] + ["<staging copy of the source>"]),
                "env": {k: env[k] for k in ("TORCH_CUDA_ARCH_LIST", "CC", "CXX") if k in env},
            }, f, indent=1)
        if not quiet:
            print(f"reference built from {src} into {TARGET}: {', '.join(sos)}")
    finally:
        shutil.rmtree(stage_root, ignore_errors=True)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--src", default=None, help="reference source tree (default: BASELINE.json reference_path)")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args(argv)
    try:
        install(reference_source(args.src), force=args.force, jobs=args.jobs)
    except Exception as exc:
        print(f"reference install failed: {exc}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
