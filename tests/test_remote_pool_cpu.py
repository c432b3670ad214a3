"""The KV pool on the serving path: workers whose storage agent is the remote pool agent
(control plane + kv-pool byte service over gRPC). A prompt finished on worker A is written
back to the pool; worker B, which never saw it, pulls those prefix blocks at admission,
prefills only the rest and produces the same tokens as a worker that recomputes everything.
Also: the pull budget, bytes the byte store lost, and finishes held by the step fence."""
from concurrent import futures

import grpc
import numpy as np
import pytest

from lake_b200.api import proto
from lake_b200.services.controlplane import ControlPlane
from lake_b200.services.kvpool import serve as serve_kvpool

pb = proto.messages()


@pytest.fixture
def pool_services():
    cp = ControlPlane()
    cp_server = grpc.server(futures.ThreadPoolExecutor(max_workers=8), options=proto.message_options())
    proto.add_service(cp_server, "ControlPlaneService", cp)
    cp_port = cp_server.add_insecure_port("127.0.0.1:0")
    cp_server.start()
    kv_server, kv_port = serve_kvpool("127.0.0.1:0", max_workers=8)
    yield cp, f"127.0.0.1:{cp_port}", f"127.0.0.1:{kv_port}"
    cp.stop()
    cp_server.stop(0)
    kv_server.stop(0)


def _cfg():
    from lake_b200.runtime.config import RoleConfig

    return RoleConfig(model_backend="mock", served_model_name="tiny", device="cpu", max_running_reqs=4,
                      max_num_scheduled_tokens=128, max_model_length=512, num_blocks=64, enable_overlap=False)


def _worker(cp_addr, kv_addr, node, **kw):
    from lake_b200.runtime.worker import remote_pool_factory
    from lake_b200.runtime.worker_engine import WorkerEngine

    we = WorkerEngine(_cfg(), node_id=node, pool_factory=remote_pool_factory(cp_addr, kv_addr, node, "tiny", **kw))
    we.start()
    return we


def _prompt(n, seed):
    return np.random.default_rng(seed).integers(0, 1024, n).tolist()


def _reference_tokens(prompt, n):
    from lake_b200.runtime.worker_engine import build_engine

    return build_engine(_cfg()).generate([prompt], max_new_tokens=n)[0]


def test_worker_b_reuses_blocks_worker_a_wrote_back(pool_services):
    cp, cp_addr, kv_addr = pool_services
    a = _worker(cp_addr, kv_addr, "wA")
    b = _worker(cp_addr, kv_addr, "wB")
    try:
        shared = _prompt(200, 1)  # 12 full blocks
        ra = a.submit("r-a", shared, 5)
        agent_a = a.pool.agent
        assert agent_a.stats["written_blocks"] >= 12
        from lake_b200.engine.block_pool import chain_block_hashes

        hashes = chain_block_hashes(shared, 16, full_only=True)
        assert cp.auth.lookup_prefix("tiny", "", 1, hashes, "wB").hit_length == 12
        follow = shared + _prompt(37, 2)
        rb = b.submit("r-b", follow, 6)
        agent_b = b.pool.agent
        assert agent_b.stats["pulled_blocks"] >= 12  # from the kv-pool, not B's own HBM cache
        assert rb.reused_blocks >= 12
        assert rb.output_tokens == _reference_tokens(follow, 6)
        assert ra.output_tokens == _reference_tokens(shared, 5)
        # every reference taken while pulling was released, and B's barrier completed
        assert cp.auth.barrier_completed("r-b")
    finally:
        a.stop(drain=False)
        b.stop(drain=False)


def test_pull_budget_stops_the_pull_and_the_rest_is_recomputed(pool_services):
    _, cp_addr, kv_addr = pool_services
    a = _worker(cp_addr, kv_addr, "wA")
    b = _worker(cp_addr, kv_addr, "wB", pull_budget_ms=5.0)
    try:
        shared = _prompt(180, 3)
        a.submit("r-a", shared, 3)
        ticks = iter(range(0, 10**6, 10))
        b.pool.agent.clock = lambda: next(ticks) / 1000.0  # 10 ms per reading: the budget is spent at once
        follow = shared + _prompt(20, 4)
        rb = b.submit("r-b", follow, 4)
        assert b.pool.agent.stats["budget_stops"] == 1 and b.pool.agent.stats["pulled_blocks"] == 0
        assert rb.output_tokens == _reference_tokens(follow, 4)
    finally:
        a.stop(drain=False)
        b.stop(drain=False)


def test_blocks_the_byte_store_lost_are_recomputed(pool_services):
    cp, cp_addr, kv_addr = pool_services
    a = _worker(cp_addr, kv_addr, "wA")
    b = _worker(cp_addr, kv_addr, "wB")
    try:
        shared = _prompt(150, 5)
        a.submit("r-a", shared, 3)
        # drop the bytes of the 4th block from the kv-pool: the authority still lists it
        kv = proto.Stub(grpc.insecure_channel(kv_addr, options=proto.message_options()), "TcpDataService")
        from lake_b200.engine.block_pool import chain_block_hashes

        hashes = chain_block_hashes(shared, 16, full_only=True)
        kv.PutBlocks(pb.PutBlocksRequest(node_id="kv-pool", blocks=[pb.OpaqueBlock(
            id=pb.KVBlockID(model_id="tiny", block_hash=hashes[3], pool_kind=1, scope="public"), data=b"x")]))
        follow = shared + _prompt(10, 6)
        rb = b.submit("r-b", follow, 4)
        st = b.pool.agent.stats
        assert st["pulled_blocks"] == 3 and st["missing_bytes"] == 1
        assert rb.output_tokens == _reference_tokens(follow, 4)
    finally:
        a.stop(drain=False)
        b.stop(drain=False)


def test_finish_inside_an_open_step_is_held_until_done(pool_services):
    from lake_b200.pool.agents.remote import connect
    from lake_b200.pool.types import FinishRequest, ForwardMode, PoolError, PreparePlan, ReqIoSet
    from lake_b200.runtime.worker_engine import build_engine

    cp, cp_addr, kv_addr = pool_services
    eng = build_engine(_cfg())
    agent = connect(eng, cp_addr, kv_addr, node_id="wA", model_id="tiny")
    prompt = _prompt(40, 7)
    rid = eng.add_request(prompt, max_new_tokens=2)
    while eng.has_unfinished():
        eng.step()
    plan = PreparePlan(9, ForwardMode.DECODE, [], [ReqIoSet("other", 0, 1)], {"other": 1}, 0, False)
    agent.prepare_step(plan)
    with pytest.raises(PoolError):
        agent.prepare_step(plan)  # one open step at a time
    agent.on_request_finished(FinishRequest(rid, "wA"))
    assert agent.stats["written_blocks"] == 0 and not cp.auth.barrier_completed(rid)
    with pytest.raises(PoolError):
        agent.done(8)
    agent.done(9)
    assert agent.stats["written_blocks"] == 2 and cp.auth.barrier_completed(rid)
