"""Spawn helpers for multi-process tests: every child gets RANK/WORLD_SIZE/
MASTER_* (127.0.0.1), the parent joins with a deadline and kills stragglers,
so a protocol deadlock fails the test instead of hanging it. The parent hosts
the rendezvous store on a port it has already bound and every child attaches
to it as a client (as under torchrun's agent), so no child races another
process for a free port."""
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
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      TORCHELASTIC_USE_AGENT_STORE="True")
    try:
        fn(rank, world, *args)
        q.put((rank, None))
    except BaseException:  # noqa: BLE001 - reported to the parent
        q.put((rank, traceback.format_exc()))


def run(fn, world: int, args=(), timeout: float = 300.0):
    import datetime

    import torch.distributed as dist

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    # The store server binds port 0 itself: the port is held from the start.
    store = dist.TCPStore("127.0.0.1", 0, world, is_master=True, wait_for_workers=False,
                          timeout=datetime.timedelta(seconds=timeout))
    port = store.port
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
