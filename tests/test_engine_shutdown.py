"""How the engine ends its TP workers, on the CPU (no GPU, no real workers):
a worker turns SIGTERM into an orderly exit (its cleanup runs), an idle worker
leaves on its own when rank 0's process is gone, and LLMEngine._reap kills a
worker that ignores the stop request only when no rank holds memory that may
be bound to an NVLink multicast object."""
import multiprocessing as mp
import os
import signal
import time
from types import SimpleNamespace

import pytest


def _sigterm_child(marker):
    from kavor_b200.engine.llm_engine import _stop_requested

    signal.signal(signal.SIGTERM, _stop_requested)
    try:
        with open(marker + ".ready", "w"):
            pass
        while True:
            time.sleep(0.05)
    finally:  # reached through SystemExit, as ModelRunner.loop's abandon() is
        with open(marker, "w") as f:
            f.write("cleaned up")


def test_sigterm_becomes_an_orderly_exit(tmp_path):
    marker = str(tmp_path / "m")
    p = mp.get_context("spawn").Process(target=_sigterm_child, args=(marker,), daemon=True)
    p.start()
    deadline = time.monotonic() + 60
    while not os.path.exists(marker + ".ready") and time.monotonic() < deadline:
        time.sleep(0.05)
    p.terminate()  # SIGTERM
    p.join(timeout=30)
    assert p.exitcode == 1  # SystemExit with a message
    assert open(marker).read() == "cleaned up"


def _idle_worker(marker):
    import threading

    from kavor_b200.engine.model_runner import ModelRunner

    # should the product code never notice its parent is gone, the test still leaves no process behind
    guard = threading.Timer(120.0, lambda: os._exit(3))
    guard.daemon = True
    guard.start()

    ev = mp.get_context("spawn").Event()  # never set: rank 0 sends nothing
    runner = SimpleNamespace(event=ev, rank=1, shm=None)
    try:
        ModelRunner.read_shm(runner)
    except SystemExit as e:
        with open(marker, "w") as f:
            f.write(str(e))


def _rank0(marker):
    ctx = mp.get_context("spawn")
    w = ctx.Process(target=_idle_worker, args=(marker,))  # non-daemonic: outlives this process
    w.start()
    with open(marker + ".pid", "w") as f:
        f.write(str(w.pid))
    os._exit(0)  # rank 0 gone without sending "exit"


def test_idle_worker_leaves_when_rank0_is_gone(tmp_path):
    marker = str(tmp_path / "w")
    r0 = mp.get_context("spawn").Process(target=_rank0, args=(marker,))
    r0.start()
    r0.join(timeout=60)
    deadline = time.monotonic() + 60
    while not os.path.exists(marker) and time.monotonic() < deadline:
        time.sleep(0.1)
    assert "rank 0's process exited" in open(marker).read()


class _Stuck:
    """A worker process that ignores every stop request."""

    def __init__(self):
        self.name, self.calls = "worker-1", []

    def is_alive(self):
        return True

    def join(self, timeout=None):
        self.calls.append("join")

    def terminate(self):
        self.calls.append("terminate")

    def kill(self):
        self.calls.append("kill")


@pytest.mark.parametrize("kill_ok", [False, True])
def test_reap_never_kills_a_rank_that_may_hold_multicast_memory(monkeypatch, kill_ok, caplog):
    from kavor_b200.engine import llm_engine

    monkeypatch.setattr(llm_engine, "WORKER_EXIT_TIMEOUT", 0.0)
    monkeypatch.setattr(llm_engine, "WORKER_STOP_TIMEOUT", 0.0)
    w = _Stuck()
    engine = SimpleNamespace(ps=[w], _kill_ok=kill_ok)
    llm_engine.LLMEngine._reap(engine, graceful=True)
    assert "terminate" in w.calls  # the stop request (SIGTERM) is always sent
    assert ("kill" in w.calls) == kill_ok
    if not kill_ok:
        assert "left running" in caplog.text
