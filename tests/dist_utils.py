"""Helpers to run a test body on several spawned CPU ranks (gloo) or GPU ranks."""

from __future__ import annotations

import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _pack(obj):
    """Tensors -> numpy so results survive the child's exit (no shared memory)."""
    import torch

    if isinstance(obj, torch.Tensor):
        t = obj.detach().cpu()
        if t.dtype in (torch.bfloat16, torch.float16):
            return ("__tensor__", t.view(torch.int16).numpy().copy(), str(t.dtype))
        return ("__tensor__", t.numpy().copy(), str(t.dtype))
    if isinstance(obj, (list, tuple)):
        return type(obj)(_pack(o) for o in obj)
    if isinstance(obj, dict):
        return {k: _pack(v) for k, v in obj.items()}
    return obj


def _unpack(obj):
    import torch

    if isinstance(obj, tuple) and len(obj) == 3 and obj[0] == "__tensor__":
        t = torch.from_numpy(obj[1])
        if obj[2] in ("torch.bfloat16", "torch.float16"):
            t = t.view(getattr(torch, obj[2].split(".")[1]))
        return t
    if isinstance(obj, (list, tuple)):
        return type(obj)(_unpack(o) for o in obj)
    if isinstance(obj, dict):
        return {k: _unpack(v) for k, v in obj.items()}
    return obj


def _entry(rank, world, port, fn, args, q, env):
    import faulthandler

    faulthandler.enable(all_threads=True)  # a hard crash prints the Python stacks
    if env.get("BITSCOM_TEST_DUMP_AFTER"):  # debugging aid: dump stacks of a hung rank
        faulthandler.dump_traceback_later(float(env["BITSCOM_TEST_DUMP_AFTER"]), exit=False)
    os.environ.update(env)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    os.environ["LOCAL_RANK"] = str(rank)
    try:
        q.put((rank, True, _pack(fn(rank, world, *args))))
    except BaseException as exc:  # report every failure to the parent
        q.put((rank, False, "".join(traceback.format_exception(exc))))
        raise SystemExit(1)


def run_ranks(fn, world: int = 2, args=(), timeout: float = 180.0, env=None, allow_fail=()):
    """Run ``fn(rank, world, *args)`` on ``world`` spawned processes; returns
    the per-rank results (raises with the child traceback on failure)."""
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q, dict(env or {}))) for r in range(world)]
    for p in procs:
        p.start()
    # Drain results while the children run: a child cannot exit while its
    # queued result is still in the pipe.
    import time

    results, errors = {}, {}
    deadline = time.time() + timeout
    while len(results) + len(errors) < world and time.time() < deadline:
        if not q.empty():
            r, ok, val = q.get()
            if ok:
                results[r] = _unpack(val)
            else:
                errors[r] = val
            continue
        if all(not p.is_alive() for p in procs) and q.empty():
            break
        time.sleep(0.05)
    for p in procs:
        p.join(max(1.0, deadline - time.time()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join(5)
    for r, val in errors.items():
        if r not in allow_fail:
            raise AssertionError(f"rank {r} failed:\n{val}")
        results[r] = RuntimeError(val)
    if alive:
        raise AssertionError(f"{len(alive)} rank(s) did not finish within {timeout}s")
    for r, p in enumerate(procs):
        if r not in results and r not in allow_fail:
            raise AssertionError(f"rank {r} exited with code {p.exitcode} without a result")
    return [results.get(r) for r in range(world)]
