"""Spawn helpers for multi-process tests: every child gets RANK/WORLD_SIZE/
MASTER_* (127.0.0.1, a free port), the parent joins with a deadline and kills
stragglers, so a protocol deadlock fails the test instead of hanging it."""
import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn, args, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        fn(rank, world, *args)
        q.put((rank, None))
    except BaseException:  # noqa: BLE001 - reported to the parent
        q.put((rank, traceback.format_exc()))


def run(fn, world: int, args=(), timeout: float = 300.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q)) for r in range(world)]
    for p in procs:
        p.start()
    errors = {}
    import time

    deadline = time.time() + timeout
    got = 0
    while got < world and time.time() < deadline:
        try:
            rank, err = q.get(timeout=max(0.1, deadline - time.time()))
        except Exception:  # noqa: BLE001 - queue timeout
            break
        got += 1
        if err:
            errors[rank] = err
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.time()))
    for p in procs:
        if p.is_alive():
            p.kill()
            errors.setdefault(-1, "rank did not finish before the deadline")
    if got < world:
        errors.setdefault(-2, f"only {got}/{world} ranks reported")
    if errors:
        raise AssertionError("\n".join(f"rank {r}: {e}" for r, e in sorted(errors.items())))
