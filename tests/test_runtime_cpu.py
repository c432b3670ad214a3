"""Runtime layer on CPU: role config, lifecycle, mode selection, the worker engine
loop and the WorkerService gRPC facade (python/lake/runtime tests' behaviour)."""
import threading
from concurrent import futures

import grpc
import pytest

from lake_b200.api import proto
from lake_b200.engine.llm_engine import LLMEngine
from lake_b200.pool.types import PoolError, PoolErrorCode, PrefixHint
from lake_b200.runtime.config import (ExecMode, RoleConfig, WorkerLifecycle, WorkerRole, WorkerState,
                                      full_local_hit, select_exec_mode)
from lake_b200.runtime.worker import WorkerServicer
from lake_b200.runtime.worker_engine import WorkerEngine


def tiny_engine(**kw):
    args = dict(max_running=4, max_batched_tokens=128, max_model_len=512, num_blocks=64)
    args.update(kw)
    return LLMEngine("tiny", device="cpu", **args)


def test_role_config_env(monkeypatch):
    monkeypatch.setenv("LAKE_WORKER_ROLE", "DECODE")
    monkeypatch.setenv("LAKE_MAX_RUNNING_REQS", "32")
    monkeypatch.setenv("LAKE_MAX_NUM_SCHEDULED_TOKENS", "bogus")
    monkeypatch.setenv("LAKE_ENABLE_DRAFTER", "yes")
    cfg = RoleConfig.from_env()
    assert cfg.role == WorkerRole.DECODE and cfg.max_running_reqs == 32
    assert cfg.max_num_scheduled_tokens == 8192 and cfg.enable_drafter
    monkeypatch.setenv("LAKE_WORKER_ROLE", "nonsense")
    assert RoleConfig.from_env().role == WorkerRole.HYBRID
    with pytest.raises(ValueError):
        RoleConfig(max_running_reqs=0)


def test_lifecycle_order():
    lc = WorkerLifecycle()
    assert not lc.accepting
    lc.warm()
    assert lc.state == WorkerState.WARM and not lc.accepting
    lc.ready()
    lc.serve()
    assert lc.accepting
    with pytest.raises(ValueError):
        lc.advance(WorkerState.BOOT)
    lc.drain()
    assert not lc.accepting
    lc.terminate()
    assert lc.state == WorkerState.TERMINATE


def test_select_exec_mode():
    assert select_exec_mode(PrefixHint(computed_tokens=32, local_hit=True), 64, WorkerRole.HYBRID) == ExecMode.D_DIRECT
    assert select_exec_mode(PrefixHint(reused_blocks=2), 64, WorkerRole.PREFILL, bw_gbps=0.5) == ExecMode.COLOCATED
    assert select_exec_mode(PrefixHint(), 64, WorkerRole.PREFILL) == ExecMode.PD_DISAGG
    assert select_exec_mode(PrefixHint(), 64, WorkerRole.HYBRID) == ExecMode.COLOCATED
    assert full_local_hit(PrefixHint(computed_tokens=64, local_hit=True), 64)
    assert not full_local_hit(PrefixHint(computed_tokens=32, local_hit=True), 64)


@pytest.mark.parametrize("overlap", [False, True])  # overlapped steps resolve the last token one step later
def test_worker_engine_concurrent_submit(overlap):
    eng = tiny_engine(overlap=overlap)
    ref = tiny_engine()
    prompts = [[(7 * i + j) % 1000 for j in range(20 + i)] for i in range(6)]
    want = ref.generate(prompts, max_new_tokens=5)
    we = WorkerEngine(RoleConfig(device="cpu", model_backend="mock"), engine=eng)
    we.start()
    assert we.state == WorkerState.SERVING
    got = [None] * len(prompts)

    def run(i):
        got[i] = we.submit(f"r{i}", prompts[i], 5).output_tokens

    ts = [threading.Thread(target=run, args=(i,)) for i in range(len(prompts))]
    [t.start() for t in ts]
    [t.join(60) for t in ts]
    assert got == want
    sig = we.capacity_signal()
    assert sig.inflight_reqs == 0 and sig.model_warmed and sig.remaining_slots == 4
    we.stop()
    assert we.state == WorkerState.TERMINATE
    with pytest.raises(PoolError) as e:
        we.submit("late", [1, 2, 3], 2)
    assert e.value.code == PoolErrorCode.CAPACITY


def test_worker_engine_step_failure_fails_inflight():
    eng = tiny_engine()
    we = WorkerEngine(RoleConfig(device="cpu", model_backend="mock"), engine=eng)
    we.start()
    real_step = eng.step

    def bad_step():
        raise RuntimeError("device lost")

    eng.step = bad_step
    with pytest.raises(PoolError) as e:
        we.submit("x", [1, 2, 3, 4], 3, timeout_s=30)
    assert e.value.code == PoolErrorCode.DOWNSTREAM and "device lost" in str(e.value)
    with pytest.raises(PoolError) as e:
        we.submit("y", [1, 2, 3], 3, timeout_s=30)
    assert e.value.code == PoolErrorCode.DOWNSTREAM
    eng.step = real_step
    we.stop(drain=False)


def test_worker_grpc_generate_and_error_mapping():
    eng = tiny_engine()
    ref = tiny_engine()
    prompt = list(range(40))
    want = ref.generate([prompt], max_new_tokens=4)[0]
    we = WorkerEngine(RoleConfig(device="cpu", model_backend="mock"), engine=eng)
    we.start()
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=4))
    proto.add_service(server, "WorkerService", WorkerServicer(we))
    port = server.add_insecure_port("127.0.0.1:0")
    server.start()
    pb = proto.messages()
    try:
        with grpc.insecure_channel(f"127.0.0.1:{port}") as ch:
            stub = proto.Stub(ch, "WorkerService")
            resp = stub.Generate(pb.GenerateRequest(request_id="g1", prompt_tokens=prompt, max_new_tokens=4),
                                 timeout=60)
            assert list(resp.output_tokens) == want and resp.mode == "COLOCATED"
            # same prompt again: the radix prefix cache serves the full blocks
            resp2 = stub.Generate(pb.GenerateRequest(request_id="g2", prompt_tokens=prompt, max_new_tokens=4,
                                                     exec_mode="D_DIRECT", computed_tokens=32, local_hit=True),
                                  timeout=60)
            assert list(resp2.output_tokens) == want and resp2.reused_blocks == 2 and resp2.mode == "D_DIRECT"
            with pytest.raises(grpc.RpcError) as e:
                stub.Generate(pb.GenerateRequest(request_id="g3", max_new_tokens=4), timeout=30)
            assert e.value.code() == grpc.StatusCode.INVALID_ARGUMENT
            we.lifecycle.drain()
            with pytest.raises(grpc.RpcError) as e:
                stub.Generate(pb.GenerateRequest(request_id="g4", prompt_tokens=[1, 2], max_new_tokens=1),
                              timeout=30)
            assert e.value.code() == grpc.StatusCode.RESOURCE_EXHAUSTED
    finally:
        server.stop(0)
        we.stop(drain=False)


def test_kernel_timeout_maps_to_pool_timeout():
    """A step that failed because a kernel's bounded wait ran out (a peer GPU stopped answering)
    surfaces as PoolError TIMEOUT; other kernel errors as DOWNSTREAM (both UNAVAILABLE at gRPC)."""
    from lake_b200.ops.core import KernelError
    from lake_b200.pool.types import PoolErrorCode
    from lake_b200.runtime.worker_engine import _step_error_code

    assert _step_error_code(KernelError(0, 2)) == PoolErrorCode.TIMEOUT
    assert _step_error_code(KernelError(0, 1)) == PoolErrorCode.TIMEOUT
    assert _step_error_code(KernelError(0, 3)) == PoolErrorCode.DOWNSTREAM
    assert _step_error_code(ValueError("x")) == PoolErrorCode.DOWNSTREAM
    assert "peer flag wait timed out" in str(KernelError(1, 2))


def test_stop_without_drain_fails_every_orphaned_request():
    """Stopping mid-flight (no drain) ends every waiting submitter with an error instead of leaving
    it blocked, and the worker refuses new work (reference: test_lifecycle stop races)."""
    import time

    eng = tiny_engine()
    we = WorkerEngine(RoleConfig(device="cpu", model_backend="mock"), engine=eng)
    we.start()
    real_step = eng.step

    def slow_step():
        time.sleep(0.05)
        return real_step()

    eng.step = slow_step
    results = [None] * 6

    def run(i):
        try:
            results[i] = we.submit(f"s{i}", [(i + j) % 900 for j in range(30)], 200, timeout_s=60)
        except PoolError as e:
            results[i] = e

    ts = [threading.Thread(target=run, args=(i,)) for i in range(6)]
    [t.start() for t in ts]
    time.sleep(0.3)
    we.stop(drain=False, timeout_s=30)
    [t.join(30) for t in ts]
    assert not any(t.is_alive() for t in ts)
    assert all(r is not None for r in results)
    assert any(isinstance(r, PoolError) for r in results)  # 200 tokens at 50 ms/step cannot finish
    assert we.state == WorkerState.TERMINATE
    with pytest.raises(PoolError):
        we.submit("after", [1, 2, 3], 2)


def test_pd_pair_serves_pd_disagg_requests(tmp_path):
    """The PD serving pair (prefill process + decode worker with WorkerService): a PD_DISAGG
    request is prefilled by the prefill process into the decode worker's arena and decoded there;
    the tokens equal a colocated engine's, and a COLOCATED request runs on the decode worker."""
    import os
    import signal
    import socket
    import subprocess
    import sys
    import time

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, LAKE_MODEL_BACKEND="mock", LAKE_DEVICE="cpu", LAKE_MAX_RUNNING_REQS="8",
               LAKE_LOG="WARNING")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    proc = subprocess.Popen([sys.executable, "-m", "lake_b200.runtime.pd_pair", "--bind", f"127.0.0.1:{port}"],
                            cwd=root, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    pb = proto.messages()
    try:
        ch = grpc.insecure_channel(f"127.0.0.1:{port}")
        grpc.channel_ready_future(ch).result(timeout=120)
        stub = proto.Stub(ch, "WorkerService")
        prompt = [(5 * j + 3) % 1000 for j in range(50)]
        t0 = time.time()
        while True:  # the worker answers once it has warmed up
            try:
                resp = stub.Generate(pb.GenerateRequest(request_id="pd1", prompt_tokens=prompt, max_new_tokens=6,
                                                        exec_mode="PD_DISAGG"), timeout=60)
                break
            except grpc.RpcError:
                if time.time() - t0 > 120:
                    raise
                time.sleep(0.5)
        want = tiny_engine().generate([prompt], max_new_tokens=6)[0]
        assert resp.mode == "PD_DISAGG" and list(resp.output_tokens) == want
        other = [(7 * j + 1) % 1000 for j in range(40)]
        r2 = stub.Generate(pb.GenerateRequest(request_id="c1", prompt_tokens=other, max_new_tokens=4,
                                              exec_mode="COLOCATED"), timeout=60)
        assert r2.mode == "COLOCATED" and list(r2.output_tokens) == tiny_engine().generate([other], 4)[0]
        ch.close()
    finally:
        proc.send_signal(signal.SIGTERM)
        try:
            out, _ = proc.communicate(timeout=60)
        except subprocess.TimeoutExpired:
            proc.kill()
            out, _ = proc.communicate()
    assert proc.returncode == 0, out[-2000:]


def test_worker_metrics_histograms_and_request_trace(tmp_path):
    """Finished requests feed the worker's TTFT/TPOT/queue/e2e histograms and token counters,
    the Prometheus endpoint serves them, and LAKE_TRACE_OUT gets one line per request."""
    import json
    import urllib.request

    from lake_b200.runtime.config import RoleConfig
    from lake_b200.runtime.metrics import serve_metrics
    from lake_b200.runtime.worker_engine import WorkerEngine

    we = WorkerEngine(RoleConfig(device="cpu", model_backend="mock", max_num_scheduled_tokens=128, num_blocks=64,
                                 enable_overlap=False), node_id="w-metrics")
    we.metrics.trace_path = str(tmp_path / "trace.jsonl")
    we.start()
    try:
        for i in range(3):
            we.submit(f"r{i}", list(range(1 + i, 40 + i)), 4)
        server = serve_metrics(we.metrics, "127.0.0.1:0")
        port = server[0].server_port if isinstance(server, tuple) else server.server_port
        text = urllib.request.urlopen(f"http://127.0.0.1:{port}/metrics", timeout=10).read().decode()
    finally:
        we.stop(drain=False)
    assert 'lake_worker_ttft_seconds_count{mode="COLOCATED"} 3.0' in text
    assert 'lake_worker_tpot_seconds_count{mode="COLOCATED"} 3.0' in text
    assert "lake_worker_output_tokens_total 12.0" in text
    assert "lake_worker_running_requests" in text
    recs = [json.loads(l) for l in open(tmp_path / "trace.jsonl")]
    assert [r["request_id"] for r in recs] == ["r0", "r1", "r2"]
    assert all(r["t_arrival"] <= r["t_admitted"] <= r["t_first_token"] <= r["t_finish"] for r in recs)
    assert all(r["output_tokens"] == 4 and r["node"] == "w-metrics" for r in recs)
