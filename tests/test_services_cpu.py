"""ControlPlaneService over gRPC on the C++ authority (behaviour of the
reference's rust/controlplane/src/lib.rs handler tests)."""
import threading
from concurrent import futures

import grpc
import pytest

from lake_b200.api import proto
from lake_b200.engine.block_pool import chain_block_hashes
from lake_b200.services.controlplane import ControlPlane, FileCheckpointStore

pb = proto.messages()
M = "llama"


@pytest.fixture
def cp_stub():
    warm = []
    now = [0.0]
    cp = ControlPlane(warmup_sink=lambda node, ids: warm.append((node, len(ids))), lease_ttl_ms=1000,
                      clock=lambda: now[0])
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=8))
    proto.add_service(server, "ControlPlaneService", cp)
    port = server.add_insecure_port("127.0.0.1:0")
    server.start()
    ch = grpc.insecure_channel(f"127.0.0.1:{port}")
    stub = proto.Stub(ch, "ControlPlaneService")
    stub.RegisterModel(pb.RegisterModelRequest(model=pb.ModelDescriptor(
        model_id=M, num_layers=2, block_spec=pb.BlockSpec(block_tokens=16, bytes_per_block=1000), hash_algo=1,
        quota=pb.Quota(soft_bytes=4000, hard_bytes=6000))), timeout=10)
    yield cp, stub, warm, now
    cp.stop()
    ch.close()
    server.stop(0)


def chain(n, seed=0):
    return chain_block_hashes(list(range(seed, seed + 16 * n)), 16)


def reg_req(hashes, node="n0", tier=1):
    return pb.RegisterBlocksRequest(node_id=node, prefix_hashes=hashes, blocks=[
        pb.BlockMeta(id=pb.KVBlockID(model_id=M, block_hash=h, pool_kind=1), block_kind=1,
                     locations=[pb.Location(tier=tier, node_id=node, segment_id=1, offset=i * 1000)])
        for i, h in enumerate(hashes)])


def test_register_lookup_locate(cp_stub):
    cp, stub, warm, _ = cp_stub
    hs = chain(3)
    assert stub.RegisterBlocks(reg_req(hs), timeout=10).ok
    r = stub.LookupPrefix(pb.LookupPrefixRequest(model_id=M, prefix_hashes=hs + chain(1, seed=999),
                                                 requester_node_id="n0", pool_kind=1), timeout=10)
    assert r.hit_length == 3 and all(b.local_hit for b in r.blocks)
    r2 = stub.LookupPrefix(pb.LookupPrefixRequest(model_id=M, prefix_hashes=hs, requester_node_id="n1",
                                                  pool_kind=1), timeout=10)
    assert r2.hit_length == 3 and not r2.all_local_hit
    loc = stub.Locate(pb.LocateRequest(ids=[pb.KVBlockID(model_id=M, block_hash=hs[1], pool_kind=1)]), timeout=10)
    assert loc.blocks[0].locations[0].offset == 1000


def test_hard_quota_backpressure(cp_stub):
    cp, stub, _, _ = cp_stub
    hs = chain(7)
    a = stub.AdmitRegisterBlocks(reg_req(hs), timeout=10)
    assert not a.ok and a.backpressure.deficit_bytes > 0 and "admission rejected" in a.err
    assert stub.AdmitRegisterBlocks(reg_req(hs[:3]), timeout=10).ok
    q = stub.GetModelQuota(pb.GetModelQuotaRequest(model_id=M), timeout=10)
    assert q.ok and q.quota.hard_bytes == 6000 and q.used_bytes == 0
    bad = stub.GetModelQuota(pb.GetModelQuotaRequest(model_id="nope"), timeout=10)
    assert not bad.ok and "unknown namespace" in bad.err


def test_report_ref_all_or_nothing(cp_stub):
    cp, stub, _, _ = cp_stub
    hs = chain(2)
    stub.RegisterBlocks(reg_req(hs), timeout=10)
    kid = pb.KVBlockID(model_id=M, block_hash=hs[0], pool_kind=1)
    assert stub.ReportRef(iter([pb.RefDelta(id=kid, kind=1, delta=2, node_id="n0")]), timeout=10).ok
    bad = stub.ReportRef(iter([pb.RefDelta(id=kid, kind=1, delta=-1, node_id="n0"),
                               pb.RefDelta(id=kid, kind=3, delta=-1, node_id="n0")]), timeout=10)
    assert not bad.ok
    from lake_b200.services import convert as C
    assert cp.auth.refs_by_kind(C.kid_in(kid)) == (2, 0)


def test_subscribe_view_snapshot_live_and_resume(cp_stub):
    cp, stub, _, _ = cp_stub
    stub.RegisterBlocks(reg_req(chain(2)), timeout=10)
    call = stub.SubscribeView(pb.SubscribeRequest(subscriber_id="r1"), timeout=20)
    it = iter(call)
    snap = next(it)
    assert snap.seq == 0 and len(snap.events) == 2
    anchor = next(it)
    assert anchor.seq == 1 and not anchor.events
    stub.RegisterBlocks(reg_req(chain(1, seed=500), node="n1"), timeout=10)
    live = next(it)
    assert live.seq == 2 and live.events[0].kind == 0 and live.events[0].locations[0].node_id == "n1"
    call.cancel()
    # resume from seq 1: only the missed update is replayed
    call2 = stub.SubscribeView(pb.SubscribeRequest(subscriber_id="r1", resume_from_seq=1), timeout=20)
    u = next(iter(call2))
    assert u.seq == 2
    call2.cancel()


def test_checkpoint_file_roundtrip(tmp_path, cp_stub):
    cp, stub, _, _ = cp_stub
    cp.checkpoints = FileCheckpointStore(str(tmp_path / "cp" / "snap.bin"))
    hs = chain(3)
    stub.RegisterBlocks(reg_req(hs), timeout=10)
    s = stub.SaveCheckpoint(pb.SaveCheckpointRequest(), timeout=10)
    assert s.ok and s.snapshot.seq == 1 and len(s.snapshot.blocks) == 3
    assert stub.DiscardBlocks(pb.DiscardBlocksRequest(ids=[s.snapshot.blocks[0].meta.id]), timeout=10).ok
    assert cp.auth.block_count(M, "") < 3
    assert stub.RestoreCheckpoint(pb.RestoreCheckpointRequest(), timeout=10).ok
    assert cp.auth.block_count(M, "") == 3
    r = stub.LookupPrefix(pb.LookupPrefixRequest(model_id=M, prefix_hashes=hs, requester_node_id="n0",
                                                 pool_kind=1), timeout=10)
    assert r.hit_length == 3


def test_lease_and_dead_node_reap(cp_stub):
    cp, stub, _, now = cp_stub
    stub.RegisterBlocks(reg_req(chain(2), node="n7"), timeout=10)
    acks = list(stub.Lease(iter([pb.LeaseHeartbeat(op=0, node_id="n7", segment_id=1),
                                 pb.LeaseHeartbeat(op=2, node_id="n7"),
                                 pb.LeaseHeartbeat(op=2, node_id="ghost")]), timeout=10))
    assert [a.granted for a in acks] == [True, True, False] and acks[0].ttl_ms == 1000
    assert cp.reap_expired_leases() == []
    now[0] = 5.0
    assert cp.reap_expired_leases() == ["n7"]
    r = stub.LookupPrefix(pb.LookupPrefixRequest(model_id=M, prefix_hashes=chain(2), requester_node_id="n7",
                                                 pool_kind=1), timeout=10)
    assert r.hit_length == 0 or not r.all_local_hit


def test_shard_ring_and_hits(cp_stub):
    cp, stub, warm, _ = cp_stub
    j = stub.JoinShardNode(pb.JoinShardNodeRequest(node_id="a", vnode_count=8), timeout=10)
    assert j.ok and any(n.node_id == "a" for n in j.map.nodes)
    j2 = stub.JoinShardNode(pb.JoinShardNodeRequest(node_id="b", vnode_count=8), timeout=10)
    assert j2.ok and len(j2.map.nodes) == 2
    d = stub.DrainShardNode(pb.DrainShardNodeRequest(node_id="a"), timeout=10)
    assert d.ok and any(n.draining for n in d.map.nodes if n.node_id == "a")
    assert stub.RemoveShardNode(pb.RemoveShardNodeRequest(node_id="a"), timeout=10).ok
    g = stub.GetShardMap(pb.GetShardMapRequest(), timeout=10)
    assert [n.node_id for n in g.map.nodes] == ["b"]
    assert stub.PauseBackground(pb.PauseBackgroundRequest(paused=True), timeout=10).ok
    assert cp.auth.background_paused()
    t = stub.TriggerDefrag(pb.TriggerDefragRequest(model_id=M, pool_kind=1, mode=3, slot_bytes=1000), timeout=10)
    assert t.ok
    rec = stub.ReconcileOrphans(pb.ReconcileOrphansRequest(dead_node_id="zz"), timeout=10)
    assert rec.ok and rec.refs_cleared == 0


# ---------------------------------------------------------------- transfer / kv-pool / agent
@pytest.fixture
def data_stub():
    from lake_b200.services.agent_service import AgentServer
    from lake_b200.services.transfer import TcpDataServer, TransferServer

    placed = []
    ts = TransferServer()
    tcp = TcpDataServer(ts.store)
    ag = AgentServer("n0", place=lambda ids, node: placed.append((len(ids), node)))
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=8))
    proto.add_service(server, "TransferService", ts)
    proto.add_service(server, "TcpDataService", tcp)
    proto.add_service(server, "AgentService", ag)
    port = server.add_insecure_port("127.0.0.1:0")
    server.start()
    ch = grpc.insecure_channel(f"127.0.0.1:{port}")
    yield ts, ag, placed, proto.Stub(ch, "TransferService"), proto.Stub(ch, "TcpDataService"), \
        proto.Stub(ch, "AgentService")
    ch.close()
    server.stop(0)


def kid(h):
    return pb.KVBlockID(model_id=M, block_hash=h, pool_kind=1, revision="r1", scope="public")


def test_transfer_batch_status_and_tier_check(data_stub):
    ts, _, _, stub, _, _ = data_stub
    src = ts.engine.open_segment("src", 4096)
    dst = ts.engine.open_segment("dst", 4096)
    ts.engine.write_segment(src, 100, b"hello world")
    ack = stub.SubmitTransfer(pb.TransferBatchRequest(reqs=[pb.TransferRequest(
        source=pb.Location(tier=2, node_id="n0", segment_id=src, offset=100), target_segment_id=dst,
        target_offset=7, length=11)]), timeout=10)
    st = stub.GetTransferStatus(pb.TransferStatusRequest(batch_id=ack.batch_id, task_id=0), timeout=10)
    assert st.state == 2 and st.bytes_done == 11
    assert ts.engine.read_segment(dst, 7, 11) == b"hello world"
    assert stub.FreeBatch(pb.FreeBatchRequest(batch_id=ack.batch_id), timeout=10).ok
    assert not stub.FreeBatch(pb.FreeBatchRequest(batch_id=ack.batch_id), timeout=10).ok
    for bad in (pb.Location(tier=4, segment_id=src), pb.Location(tier=0, segment_id=src)):
        with pytest.raises(grpc.RpcError) as e:
            stub.SubmitTransfer(pb.TransferBatchRequest(reqs=[pb.TransferRequest(
                source=bad, target_segment_id=dst, length=1)]), timeout=10)
        assert e.value.code() == grpc.StatusCode.INVALID_ARGUMENT
    with pytest.raises(grpc.RpcError):  # out of range: rejected before any byte moves
        stub.SubmitTransfer(pb.TransferBatchRequest(reqs=[pb.TransferRequest(
            source=pb.Location(tier=1, segment_id=src, offset=4000), target_segment_id=dst, length=200)]),
            timeout=10)
    assert ts.engine.batch_count() == 0


def test_tcp_data_and_pull_policies(data_stub):
    ts, _, _, stub, tcp, _ = data_stub
    a = tcp.PutBlocks(pb.PutBlocksRequest(node_id="n0", blocks=[pb.OpaqueBlock(id=kid(b"h0"), data=b"AAAA"),
                                                                 pb.OpaqueBlock(id=kid(b"h1"), data=b"BBBBBB"),
                                                                 pb.OpaqueBlock(data=b"noid")]), timeout=10)
    assert not a.ok and "skipped 1 block" in a.err
    g = tcp.GetBlocks(pb.GetBlocksRequest(ids=[kid(b"h1"), kid(b"zz")]), timeout=10)
    assert len(g.blocks) == 1 and g.blocks[0].data == b"BBBBBB"
    p = stub.Pull(pb.PullRequest(ids=[kid(b"h0"), kid(b"zz"), kid(b"h1")], policy=0, requester_node_id="n1"),
                  timeout=10)
    assert p.pulled_length == 2 and p.completed
    assert ts.engine.read_segment(ts.pull_segment(p.handle), 0, 10) == b"AAAABBBBBB"
    with pytest.raises(grpc.RpcError) as e:
        stub.Pull(pb.PullRequest(ids=[kid(b"h0"), kid(b"zz")], policy=1), timeout=10)
    assert e.value.code() == grpc.StatusCode.NOT_FOUND
    t = stub.Pull(pb.PullRequest(ids=[kid(b"h0"), kid(b"h1")], policy=2, budget_ms=1), timeout=10)
    assert t.pulled_length == 1 and not t.completed
    n_seg = ts.engine.segment_count()
    assert stub.FreePull(pb.FreePullRequest(handle=p.handle), timeout=10).ok
    assert ts.engine.segment_count() == n_seg - 1
    assert not stub.FreePull(pb.FreePullRequest(handle=p.handle), timeout=10).ok


def test_publish_seq_fence_and_dedup(data_stub):
    ts, _, _, stub, _, _ = data_stub
    sl = [pb.LayerSlice(id=kid(b"h0"), layer_idx=3, offset=0, length=100),
          pb.LayerSlice(id=kid(b"h0"), layer_idx=3, offset=100, length=50)]
    assert stub.Publish(pb.PublishRequest(slices=sl, seq=2, request_id="r"), timeout=10).ok
    assert stub.Publish(pb.PublishRequest(slices=sl[:1], seq=2, request_id="r"), timeout=10).ok  # resend
    assert ts.published_layer_bytes("r", b"h0", 3) == 150
    late = stub.Publish(pb.PublishRequest(slices=sl, seq=1, request_id="r"), timeout=10)
    assert not late.ok and "overlap fence" in late.err
    assert stub.Publish(pb.PublishRequest(slices=sl, seq=1, request_id="other"), timeout=10).ok
    assert ts.publish_stream_count == 2
    assert stub.FreePublish(pb.FreePublishRequest(request_id="r"), timeout=10).ok
    assert not stub.FreePublish(pb.FreePublishRequest(request_id="r"), timeout=10).ok


def test_agent_dispatch_report_load_backpressure(data_stub):
    from lake_b200 import _host as H

    _, ag, placed, _, _, stub = data_stub
    with pytest.raises(grpc.RpcError) as e:
        stub.Dispatch(pb.DispatchRequest(mode="PD_DISAGG"), timeout=10)
    assert e.value.code() == grpc.StatusCode.INVALID_ARGUMENT
    assert stub.Dispatch(pb.DispatchRequest(mode="PD_DISAGG", target_node_id="n0"), timeout=10).ok
    s = H.BackpressureSignal()
    s.model_id, s.deficit_bytes, s.reason = M, 123, "HARD_QUOTA"
    ag.bp.record(s)
    acks = list(stub.ReportLoad(iter([pb.LoadReport(node_id="n0", queue_len=3, in_flight=2, remaining_cap=5)] * 3),
                                timeout=10))
    assert len(acks) == 3 and acks[0].backpressure.deficit_bytes == 123
    assert ag.load_report_count == 3 and ag.last_loads["n0"] == (3, 2, 5) and ag.dispatch_count == 1
    assert stub.PlaceBlocks(pb.PlaceBlocksRequest(ids=[kid(b"h0"), kid(b"h1")], target_node_id="n2"), timeout=10).ok
    assert placed == [(2, "n2")]


def test_byte_store_lru_bound():
    from lake_b200 import _host as H

    s = H.ByteStore(100)
    for i in range(5):
        s.put(bytes([i]), b"x" * 30)
    assert len(s) == 3 and s.bytes == 90 and s.evictions == 2
    assert s.get(bytes([0])) is None and s.get(bytes([4])) == b"x" * 30


def test_subscribe_view_lagging_subscriber_gets_a_fresh_snapshot(monkeypatch):
    """A subscriber whose queue overflows is resynchronised: the next message is a seq-0
    snapshot holding every block, then an anchor at the latest seq; stale queued updates are
    dropped (reference behaviour: lib.rs subscribe_view, lag -> resnapshot)."""
    from lake_b200.services import controlplane as cpmod

    monkeypatch.setattr(cpmod, "SUBSCRIBER_QUEUE", 2)
    cp = ControlPlane()
    cp.RegisterModel(pb.RegisterModelRequest(model=pb.ModelDescriptor(
        model_id=M, num_layers=2, block_spec=pb.BlockSpec(block_tokens=16, bytes_per_block=1000), hash_algo=1,
        quota=pb.Quota(soft_bytes=10 ** 9, hard_bytes=2 * 10 ** 9))), None)
    gen = cp.SubscribeView(pb.SubscribeRequest(subscriber_id="slow"), None)
    snap = next(gen)
    assert snap.seq == 0 and not snap.events
    for k in range(5):  # five commits into a queue of two
        cp.RegisterBlocks(reg_req(chain(1, seed=1000 * k)), None)
    resync = next(gen)
    assert resync.seq == 0 and len(resync.events) == 5
    anchor = next(gen)
    assert anchor.seq == cp.auth.last_seq() and not anchor.events
    cp.RegisterBlocks(reg_req(chain(1, seed=9000)), None)
    live = next(gen)
    assert live.seq == anchor.seq + 1 and len(live.events) == 1
    gen.close()
    cp.stop()


def test_warmup_sink_runs_outside_the_lock():
    """The warm-up sink of a shard join is called after the control-plane lock is released, so a
    sink that calls back into the service from another thread does not deadlock (reference:
    lib.rs 'sink delivered outside lock')."""
    from lake_b200.services.controlplane import ControlPlane

    done = []
    cp_box = []

    def sink(node, ids):
        t = threading.Thread(target=lambda: done.append(cp_box[0].GetShardMap(pb.GetShardMapRequest(), None)))
        t.start()
        t.join(timeout=5)
        done.append(("joined", not t.is_alive(), len(ids)))

    cp = ControlPlane(warmup_sink=sink)
    cp_box.append(cp)
    cp.RegisterModel(pb.RegisterModelRequest(model=pb.ModelDescriptor(
        model_id=M, num_layers=2, block_spec=pb.BlockSpec(block_tokens=16, bytes_per_block=1000), hash_algo=1,
        quota=pb.Quota(soft_bytes=10 ** 9, hard_bytes=2 * 10 ** 9))), None)
    cp.JoinShardNode(pb.JoinShardNodeRequest(node_id="a", vnode_count=8), None)
    hs = [h for k in range(24) for h in chain(1, seed=1000 * k)]
    for h in hs:
        cp.RegisterBlocks(reg_req([h], node="a"), None)
    for _ in range(5):
        cp.ReportHits(pb.ReportHitsRequest(node_id="a", ids=[pb.KVBlockID(model_id=M, block_hash=h, pool_kind=1)
                                                             for h in hs]), None)
    r = cp.JoinShardNode(pb.JoinShardNodeRequest(node_id="b", vnode_count=8), None)
    assert r.ok
    joined = [d for d in done if isinstance(d, tuple)]
    assert joined and all(ok for _, ok, _ in joined) and joined[0][2] > 0
    cp.stop()


def test_standalone_kvpool_service_roundtrip():
    from lake_b200.services import kvpool

    server, port = kvpool.serve("127.0.0.1:0", max_workers=2)
    ch = grpc.insecure_channel(f"127.0.0.1:{port}")
    try:
        tcp = proto.Stub(ch, "TcpDataService")
        assert tcp.PutBlocks(pb.PutBlocksRequest(node_id="n0", blocks=[pb.OpaqueBlock(id=kid(b"k0"), data=b"xyz")]),
                             timeout=10).ok
        g = tcp.GetBlocks(pb.GetBlocksRequest(ids=[kid(b"k0"), kid(b"missing")]), timeout=10)
        assert [b.data for b in g.blocks] == [b"xyz"]
    finally:
        ch.close()
        server.stop(0)
