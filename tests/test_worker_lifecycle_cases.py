"""Worker engine lifecycle under the scenarios the reference's runtime lifecycle tests pin
(python/lake/runtime/tests/test_lifecycle.py:31-215): the capacity signal of a serving worker,
stop on a worker that never started (and stop twice), stop with requests in flight, a stop
whose wait runs out while a step is still running (the requests stay with the loop, which fails
them when it exits), submit after stop, a step failure that ends the loop, and submit racing
stop (it finishes or raises, never hangs)."""
import threading
import time

import pytest

from lake_b200.engine.llm_engine import LLMEngine
from lake_b200.pool.types import PoolError, PoolErrorCode
from lake_b200.runtime.config import RoleConfig, WorkerState
from lake_b200.runtime.worker_engine import WorkerEngine


def _worker(start=True, **cfg):
    eng = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=128, max_model_len=512, num_blocks=64)
    we = WorkerEngine(RoleConfig(device="cpu", model_backend="mock", **cfg), engine=eng)
    if start:
        we.start()
    return we


def _submit_in_thread(we, rid, n_new=3, prompt=(1, 2, 3, 4, 5)):
    out = {}

    def run():
        try:
            out["result"] = we.submit(rid, list(prompt), n_new, timeout_s=30)
        except Exception as e:  # noqa: BLE001 - the test inspects it
            out["error"] = e

    t = threading.Thread(target=run)
    t.start()
    return t, out


def test_a_serving_worker_reports_its_capacity():
    we = _worker(served_model_name="public-llm")
    try:
        sig = we.capacity_signal()
        assert sig.state == WorkerState.SERVING and sig.role == "hybrid"
        assert (sig.max_running_reqs, sig.remaining_slots, sig.inflight_reqs) == (4, 4, 0)
        assert sig.served_model_name == "public-llm" and sig.model_loaded and sig.model_warmed
    finally:
        we.stop()
    assert we.state == WorkerState.TERMINATE


def test_stop_on_a_worker_that_never_started_and_stop_twice():
    we = _worker(start=False)
    we.stop()
    assert we.state == WorkerState.TERMINATE
    we.stop()
    assert we.state == WorkerState.TERMINATE
    with pytest.raises(PoolError):
        we.submit("late", [1, 2, 3], 1)


def test_stop_fails_a_request_left_in_flight():
    we = _worker()
    real = we.engine.step
    we.engine.step = lambda: time.sleep(0.01) or real()  # 200 tokens take ~2 s
    t, out = _submit_in_thread(we, "orphan", n_new=200)
    time.sleep(0.1)
    we.stop(drain=False, timeout_s=10)
    t.join(10)
    assert not t.is_alive()
    assert isinstance(out.get("error"), PoolError) and "stopped" in str(out["error"])
    assert we.state == WorkerState.TERMINATE


def test_a_stop_that_times_out_leaves_in_flight_requests_to_the_loop():
    we = _worker()
    entered, release = threading.Event(), threading.Event()
    real = we.engine.step

    def stuck():
        entered.set()
        while not release.is_set():  # a long step that does not look at the stop flag
            time.sleep(0.01)
        return real()

    we.engine.step = stuck
    t, out = _submit_in_thread(we, "stuck", n_new=20)
    assert entered.wait(5)
    we.stop(drain=False, timeout_s=0.05)
    assert we._thread.is_alive() and "stuck" in we._inflight  # noqa: SLF001 - nothing cleared under a live step
    assert not out and we.state == WorkerState.DRAIN
    with pytest.raises(PoolError):  # but nothing new is accepted
        we.submit("new", [1, 2, 3], 1)
    release.set()
    we._thread.join(5)  # noqa: SLF001
    t.join(5)
    assert isinstance(out.get("error"), PoolError) and "stopped" in str(out["error"])
    assert we._inflight == {} and we.state == WorkerState.TERMINATE  # noqa: SLF001


def test_submit_after_stop_raises_at_once():
    we = _worker()
    we.stop()
    t0 = time.monotonic()
    with pytest.raises(PoolError) as e:
        we.submit("late", [1, 2, 3, 4], 1)
    assert e.value.code == PoolErrorCode.CAPACITY and time.monotonic() - t0 < 1.0


def test_a_step_exception_ends_the_loop_and_later_submits_raise():
    we = _worker()

    def boom():
        raise RuntimeError("fatal forward")

    we.engine.step = boom
    t, out = _submit_in_thread(we, "fatal")
    t.join(10)
    we._thread.join(5)  # noqa: SLF001
    assert not we._thread.is_alive()  # noqa: SLF001
    assert "fatal forward" in str(out["error"])
    with pytest.raises(PoolError) as e:
        we.submit("after-fatal", [1, 2, 3, 4], 1)
    assert e.value.code == PoolErrorCode.DOWNSTREAM
    we.stop(drain=False)


@pytest.mark.parametrize("round_", range(5))
def test_submit_racing_stop_finishes_or_raises(round_):
    we = _worker()
    barrier = threading.Barrier(2)
    out = {}

    def run():
        barrier.wait()
        try:
            out["result"] = we.submit("race", list(range(1, 9)), 1, timeout_s=None)
        except PoolError as e:
            out["error"] = e

    t = threading.Thread(target=run)
    t.start()
    barrier.wait()
    if round_ % 2:
        time.sleep(0.001 * round_)
    we.stop(drain=False, timeout_s=5)
    t.join(5)
    assert not t.is_alive(), "submit hung after stop"
    assert ("result" in out) != ("error" in out)
