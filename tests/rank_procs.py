"""Spawned rank processes for the multi-GPU tests, ended without signals.

The ranks of these tests map their all-reduce areas through torch symmetric
memory, which binds them to an NVLink multicast object where the NVSwitch
offers one; a rank ended while bound to such an object can fault the other
ranks' GPUs. So nothing here terminates or kills a rank. Each worker gets a
``stop`` event as its last argument and calls ``check_stop(stop)`` between
its device calls. Past the deadline the helper sets the event, waits for the
ranks to raise out of their loop, close their communicators and exit (every
device wait in the library is bounded at about a second and every process
group has a timeout, so a rank still alive at the deadline is stuck in host
code and can be told to stop), and fails the test. A rank that still does not
exit is named in the failure and left running.
"""
from __future__ import annotations

import time

import pytest

STOP_GRACE_S = 180.0


class StopRequested(RuntimeError):
    pass


def check_stop(stop) -> None:
    """Call between device calls in a worker: raises once the test's deadline passed."""
    if stop is not None and stop.is_set():
        raise StopRequested("the test's deadline passed: stopping this rank")


def run_ranks(target, world: int, args: tuple, timeout: float) -> dict:
    """Run ``target(rank, world, *args, results, stop)`` on ranks 0..world-1
    (spawn context) and return {rank: result} from the shared dict."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        stop = ctx.Event()
        procs = [ctx.Process(target=target, args=(r, world, *args, results, stop)) for r in range(world)]
        for p in procs:
            p.start()
        deadline = time.monotonic() + timeout
        for p in procs:
            p.join(timeout=max(0.0, deadline - time.monotonic()))
        late = [r for r, p in enumerate(procs) if p.is_alive()]
        if late:
            stop.set()
            grace = time.monotonic() + STOP_GRACE_S
            for p in procs:
                p.join(timeout=max(0.0, grace - time.monotonic()))
        stuck = [r for r, p in enumerate(procs) if p.is_alive()]
        res = dict(results)
    if stuck:
        pytest.fail(f"ranks {stuck} did not exit {STOP_GRACE_S:.0f} s after the stop request; left running "
                    "(they may hold NVLink multicast memory, so they are not killed)")
    if late:
        pytest.fail(f"ranks {late} were still running after {timeout:.0f} s and stopped on request: {res}")
    codes = [p.exitcode for p in procs]
    assert all(c == 0 for c in codes), codes
    return res
