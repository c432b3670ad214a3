"""Request router: OpenAI-style chat HTTP front -> node pick -> mode select ->
priority admission -> AgentService.Dispatch -> WorkerService.Generate.

Per request: prompt text from the user/system messages is tokenized by the
mock tokenizer (one id per character, ``ord(c) % 10000 + 1``, padded with 42
to a multiple of 8; an empty prompt becomes ids 1..8) unless the body carries
``prompt_token_ids``; the token ids are chain-hashed into 16-token block
hashes; the routing key is the X-Lake-Session-Id header or the prefix anchor
hash; the node is picked by the C++ affinity/HRW core (mirror L0 score with an
in-flight guard, integer HRW cold path). Each attempt recomputes the reuse
hint (mirror prefix lookup, authority LookupPrefix when the mirror misses) and
the execution mode (PD_DISAGG / COLOCATED / D_DIRECT with the bandwidth
gate), dispatches to the node's agent and calls Generate on the node's worker.
Admission runs through the C++ priority queue: higher priority first, FIFO
within one; a higher-priority arrival preempts the lowest running request,
which is cancelled and requeued (its KV stays in the pool, so the rerun hits
the prefix). Models the agent reported under hard-quota backpressure are
paused, not dropped.

Background loops: view sync (SubscribeView into the C++ mirror; resume from
the mirror's last seq after a gap or disconnect), load sync (ReportLoad bidi
stream: the queue snapshot goes up, backpressure comes back), and the
autoscale tick (reap draining nodes, flush hot-block hits to ReportHits, and -
when enabled - scale out with JoinShardNode / in with DrainShardNode).

Reference parity: go/router/server.go:193-541 (handler, error mapping, mock
tokenizer), modeselect.go:58-125, affinity.go, pq.go, viewsync.go,
loadsync.go, autoscale.go:339-473.
"""
from __future__ import annotations

import asyncio
import bisect
import logging
import os
import time
import uuid
from dataclasses import dataclass, field

import grpc
import grpc.aio

from .. import _host as H
from ..api import proto
from ..services import convert as C

LOG = logging.getLogger("lake_b200.router")
pb = proto.messages()
BLOCK_SIZE = 16
MAX_BODY = 1 << 20
LATENCY_BOUNDS_S = (0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0, 30.0)
ROLE = {"hybrid": H.Role.HYBRID, "prefill": H.Role.PREFILL, "decode": H.Role.DECODE}


def tokenize_mock(text: str) -> list[int]:
    text = text.strip()
    if not text:
        return list(range(1, 9))
    out = [ord(c) % 10000 + 1 for c in text]
    while len(out) % 8:
        out.append(42)
    return out


def detokenize_mock(tokens) -> str:
    return "mock:" + ",".join(str(t) for t in tokens)


@dataclass
class RouterConfig:
    worker_addr: str = "127.0.0.1:50053"
    agent_addr: str = "127.0.0.1:50054"
    cp_addr: str = "127.0.0.1:50051"
    node_role: str = "hybrid"
    max_inflight: int = 1
    autoscale: bool = False
    affinity_guard: int = 8
    path_bw_gbps: dict = field(default_factory=dict)  # path class -> GB/s
    workers: dict = field(default_factory=dict)  # node id -> worker address
    request_timeout_s: float = 30.0
    block_size: int = BLOCK_SIZE
    max_reroutes: int = 1

    @classmethod
    def from_env(cls) -> "RouterConfig":
        c = cls(worker_addr=os.environ.get("LAKE_WORKER_ADDR", "127.0.0.1:50053"),
                agent_addr=os.environ.get("LAKE_AGENT_ADDR", "127.0.0.1:50054"),
                cp_addr=os.environ.get("LAKE_CP_ADDR", "127.0.0.1:50051"),
                node_role=os.environ.get("LAKE_NODE_ROLE", "hybrid"),
                max_inflight=int(os.environ.get("LAKE_MAX_INFLIGHT", "1") or 1),
                autoscale=os.environ.get("LAKE_AUTOSCALE", "") in ("1", "true"))
        # LAKE_WORKER_NODES="worker-0=host:port,worker-1=host:port": several workers behind one router
        for item in filter(None, (x.strip() for x in os.environ.get("LAKE_WORKER_NODES", "").split(","))):
            node, _, addr = item.partition("=")
            if node and addr:
                c.workers[node] = addr
        return c


class Preempted(Exception):
    pass


class RouterError(Exception):
    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


def map_grpc_error(op: str, e: Exception) -> RouterError:
    if isinstance(e, grpc.aio.AioRpcError) or isinstance(e, grpc.RpcError):
        code = e.code()
        if code == grpc.StatusCode.INVALID_ARGUMENT:
            return RouterError(400, f"{op} request invalid")
        if code in (grpc.StatusCode.UNAVAILABLE, grpc.StatusCode.DEADLINE_EXCEEDED):
            return RouterError(503, f"{op} upstream unavailable")
        if code == grpc.StatusCode.RESOURCE_EXHAUSTED:
            return RouterError(503, f"{op} upstream at capacity")
    return RouterError(502, f"{op} upstream failed")


class Router:
    def __init__(self, cfg: RouterConfig | None = None):
        self.cfg = cfg or RouterConfig()
        self.mirror = H.ViewMirror()
        self.nodes = H.NodeRegistry(list(self.cfg.workers) or ["worker-0"])
        self.pq = H.PQScheduler(self.cfg.max_inflight * max(1, self.nodes.count()))
        self.scaler = H.Autoscaler(H.AutoscaleConfig())
        self.hot = H.HotSet(256)
        self.mode_counts: dict[str, int] = {}
        self.stats = {"requests": 0, "errors": 0, "hit_blocks": 0, "total_blocks": 0, "local_hit_blocks": 0,
                      "reusable_blocks": 0, "preemptions": 0, "reroutes": 0, "latency_sum_s": 0.0}
        self.latency_buckets = [0] * (len(LATENCY_BOUNDS_S) + 1)
        self.last_ready_latency_s = 0.0
        self._waiters: dict[int, asyncio.Future] = {}
        self._running: dict[int, object] = {}  # ticket -> in-flight grpc call (cancelled on preemption)
        self._tasks: list[asyncio.Task] = []
        self._channels: dict[str, grpc.aio.Channel] = {}

    # ---------------------------------------------------------------- clients
    def _chan(self, addr: str) -> grpc.aio.Channel:
        ch = self._channels.get(addr)
        if ch is None:
            ch = self._channels[addr] = grpc.aio.insecure_channel(addr)
        return ch

    def stub(self, service: str, addr: str) -> proto.Stub:
        return proto.Stub(self._chan(addr), service)

    @property
    def cp(self):
        return self.stub("ControlPlaneService", self.cfg.cp_addr)

    @property
    def agent(self):
        return self.stub("AgentService", self.cfg.agent_addr)

    def worker(self, node: str):
        return self.stub("WorkerService", self.cfg.workers.get(node, self.cfg.worker_addr))

    async def start(self) -> None:
        self._tasks = [asyncio.create_task(self._view_sync()), asyncio.create_task(self._load_sync()),
                       asyncio.create_task(self._autoscale_loop()), asyncio.create_task(self._pump_loop())]

    async def close(self) -> None:
        for t in self._tasks:
            t.cancel()
        for t in self._tasks:
            try:
                await t
            except (asyncio.CancelledError, Exception):
                pass
        for ch in self._channels.values():
            await ch.close()

    # ---------------------------------------------------------------- admission
    def _pump(self) -> None:
        for t in self.pq.start_eligible():
            f = self._waiters.pop(t, None)
            if f is not None and not f.done():
                f.set_result(True)

    async def _pump_loop(self) -> None:
        while True:  # backpressure expiry re-opens paused models
            await asyncio.sleep(0.05)
            self._pump()

    def _preempt(self, ticket: int) -> None:
        call = self._running.get(ticket)
        self.stats["preemptions"] += 1
        if call is not None:
            call.cancel()

    async def admit_and_run(self, priority: int, model: str, exec_fn, timeout_s: float):
        loop = asyncio.get_running_loop()
        deadline = loop.time() + timeout_s
        ticket, pre = self.pq.submit(priority, model)
        if pre is not None:
            self._preempt(pre)
        while True:
            fut = loop.create_future()
            self._waiters[ticket] = fut
            self._pump()
            try:
                await asyncio.wait_for(fut, max(0.0, deadline - loop.time()))
            except (asyncio.TimeoutError, asyncio.CancelledError):
                self._waiters.pop(ticket, None)
                self.pq.cancel(ticket)
                raise RouterError(503, "request timed out in queue")
            try:
                res = await exec_fn(ticket)
            except Preempted:
                self.pq.finish(ticket, True)  # requeued under the same ticket
                continue
            except BaseException:
                self.pq.finish(ticket, False)
                self._pump()
                raise
            self.pq.finish(ticket, False)
            self._pump()
            return res

    # ---------------------------------------------------------------- routing
    def path_bandwidth(self, node: str) -> float:
        return float(self.cfg.path_bw_gbps.get("same_az", 0.0))

    async def prefix_hint(self, model: str, hashes: list[bytes], prompt_len: int, node: str) -> H.PrefixHint:
        if not hashes or prompt_len <= 0:
            return H.PrefixHint()
        blocks = self.mirror.prefix_lookup(model, "", 1, hashes, node)
        bs = self.cfg.block_size
        if not blocks:
            try:
                resp = await self.cp.LookupPrefix(pb.LookupPrefixRequest(
                    model_id=model, prefix_hashes=hashes, requester_node_id=node, pool_kind=1), timeout=2.0)
            except Exception:
                return H.PrefixHint()  # authority unreachable: treat as cold, do not block
            local = 0
            for b in resp.blocks:
                if not b.local_hit:
                    break
                local += 1
            self.hot.add(node, [C.kid_in(b.id) for b in resp.blocks])
            return H.PrefixHint(min(resp.hit_length * bs, prompt_len), resp.hit_length, local, local > 0)
        self.hot.add(node, [H.KVBlockID(model, b.hash, 1) for b in blocks])
        local = 0
        for b in blocks:
            if not b.local_hit:
                break
            local += 1
        return H.PrefixHint(min(len(blocks) * bs, prompt_len), len(blocks), local, local > 0)

    async def generate(self, model: str, tokens: list[int], max_new: int, priority: int = 0,
                       session: bytes = b"", rid: str | None = None) -> dict:
        """Route and run one request. A node whose worker answers UNAVAILABLE (a failed or
        draining worker: the F4 signal) is skipped and the request re-dispatched to the next
        ready node, up to cfg.max_reroutes times; the reuse hint and mode are recomputed for
        the new node."""
        rid = rid or uuid.uuid4().hex
        hashes = H.chain_block_hashes(tokens, self.cfg.block_size, True)
        key = session or H.prefix_anchor(hashes)
        node = H.pick_node(self.nodes, self.mirror, model, hashes, key, self.cfg.affinity_guard)
        tried = [node]
        for attempt in range(self.cfg.max_reroutes + 1):
            try:
                return await self._generate_on(node, model, tokens, hashes, max_new, priority,
                                               rid if attempt == 0 else f"{rid}-n{attempt}")
            except RouterError as e:
                alt = [n for n in self.nodes.ready_ids() if n not in tried]
                if e.status != 503 or attempt == self.cfg.max_reroutes or not alt:
                    raise
                node = alt[0]
                tried.append(node)
                self.stats["reroutes"] += 1
        raise RouterError(503, "no node available")

    async def _generate_on(self, node: str, model: str, tokens: list[int], hashes: list[bytes], max_new: int,
                           priority: int, rid: str) -> dict:
        t0 = time.perf_counter()
        self.nodes.inc_inflight(node)
        attempt = [0]
        last_hint = [H.PrefixHint()]
        try:
            async def exec_fn(ticket):
                attempt[0] += 1
                req_id = rid if attempt[0] == 1 else f"{rid}-r{attempt[0]}"
                hint = await self.prefix_hint(model, hashes, len(tokens), node)
                last_hint[0] = hint
                mode = H.select_exec_mode(hint, len(tokens), ROLE.get(self.cfg.node_role, H.Role.HYBRID),
                                          self.path_bandwidth(node))
                mode_s = mode.name
                if attempt[0] == 1:
                    self.mode_counts[mode_s] = self.mode_counts.get(mode_s, 0) + 1
                try:
                    ack = await self.agent.Dispatch(pb.DispatchRequest(
                        mode=mode_s, target_node_id=node, hints={"request_id": req_id, "model_id": model}),
                        timeout=self.cfg.request_timeout_s)
                except grpc.aio.AioRpcError as e:
                    raise map_grpc_error("Dispatch", e)
                if ack.HasField("backpressure") and ack.backpressure.model_id:
                    self.pq.set_backpressure(ack.backpressure.model_id)
                if not ack.ok:
                    raise RouterError(502, "Dispatch rejected")
                call = self.worker(node).Generate(pb.GenerateRequest(
                    request_id=req_id, model_id=model, prompt_tokens=tokens, max_new_tokens=max_new,
                    requester_node_id=node, exec_mode=mode_s, computed_tokens=hint.computed_tokens,
                    reused_blocks=hint.reused_blocks, local_hit=hint.local_hit), timeout=self.cfg.request_timeout_s)
                self._running[ticket] = call
                try:
                    return await call
                except asyncio.CancelledError:
                    if call.cancelled() and ticket in self._running:
                        raise Preempted()
                    raise
                except grpc.aio.AioRpcError as e:
                    if e.code() == grpc.StatusCode.CANCELLED:
                        raise Preempted()
                    raise map_grpc_error("Generate", e)
                finally:
                    self._running.pop(ticket, None)

            gen = await self.admit_and_run(priority, model, exec_fn, self.cfg.request_timeout_s)
        except RouterError:
            self.stats["errors"] += 1
            raise
        finally:
            self.nodes.dec_inflight(node)
        st = self.stats
        st["requests"] += 1
        st["total_blocks"] += len(hashes)
        st["hit_blocks"] += gen.reused_blocks
        st["reusable_blocks"] += last_hint[0].reused_blocks
        st["local_hit_blocks"] += last_hint[0].local_hit_blocks
        lat = time.perf_counter() - t0
        st["latency_sum_s"] += lat
        self.latency_buckets[bisect.bisect_left(LATENCY_BOUNDS_S, lat)] += 1
        return {"request_id": rid, "node": node, "output_tokens": list(gen.output_tokens),
                "reused_blocks": gen.reused_blocks, "prefill_blocks": gen.prefill_blocks, "mode": gen.mode}

    # ---------------------------------------------------------------- metrics
    def hit_rate(self) -> float:
        t = self.stats["total_blocks"]
        return self.stats["hit_blocks"] / t if t else 0.0

    def local_hit_rate(self) -> float:
        t = self.stats["reusable_blocks"]
        return self.stats["local_hit_blocks"] / t if t else 0.0

    def metrics_text(self) -> str:
        st = self.stats
        lines = [
            "# TYPE lake_router_requests_total counter", f"lake_router_requests_total {st['requests']}",
            "# TYPE lake_router_errors_total counter", f"lake_router_errors_total {st['errors']}",
            "# TYPE lake_router_preemptions_total counter", f"lake_router_preemptions_total {st['preemptions']}",
            "# TYPE lake_router_reroutes_total counter", f"lake_router_reroutes_total {st['reroutes']}",
            "# TYPE lake_router_latency_seconds_sum counter", f"lake_router_latency_seconds_sum {st['latency_sum_s']:.6f}",
            "# TYPE lake_router_prefix_hit_rate gauge", f"lake_router_prefix_hit_rate {self.hit_rate():.6f}",
            "# TYPE lake_router_local_hit_rate gauge", f"lake_router_local_hit_rate {self.local_hit_rate():.6f}",
            "# TYPE lake_router_queue_len gauge", f"lake_router_queue_len {self.pq.queue_len()}",
            "# TYPE lake_router_in_flight gauge", f"lake_router_in_flight {self.pq.in_flight()}",
            "# TYPE lake_router_nodes gauge", f"lake_router_nodes {self.nodes.count()}",
            "# TYPE lake_router_mirror_blocks gauge", f"lake_router_mirror_blocks {self.mirror.size()}",
            "# TYPE lake_router_mode_total counter",
        ]
        for m, n in sorted(self.mode_counts.items()):
            lines.append(f'lake_router_mode_total{{mode="{m}"}} {n}')
        lines.append("# TYPE lake_router_request_seconds histogram")
        cum = 0
        for b, n in zip(LATENCY_BOUNDS_S + (float("inf"),), self.latency_buckets):
            cum += n
            le = "+Inf" if b == float("inf") else f"{b}"
            lines.append(f'lake_router_request_seconds_bucket{{le="{le}"}} {cum}')
        lines.append(f"lake_router_request_seconds_count {cum}")
        lines.append(f"lake_router_request_seconds_sum {st['latency_sum_s']:.6f}")
        return "\n".join(lines) + "\n"

    # ---------------------------------------------------------------- background loops
    async def _view_sync(self, reconnect_s: float = 0.2) -> None:
        while True:
            gap = False
            try:
                call = self.cp.SubscribeView(pb.SubscribeRequest(subscriber_id="router",
                                                                 resume_from_seq=self.mirror.last_seq()))
                async for u in call:
                    if self.mirror.apply(C.update_in(u)) != 0:
                        gap = True  # missed updates: resume from the mirror's seq right away
                        call.cancel()
                        break
            except asyncio.CancelledError:
                raise
            except Exception as e:
                LOG.debug("view sync: %s", e)
            if not gap:
                await asyncio.sleep(reconnect_s)

    async def _load_sync(self, interval_s: float = 1.0) -> None:
        while True:
            try:
                call = self.agent.ReportLoad()

                async def reader():
                    async for ack in call:
                        if ack.HasField("backpressure") and ack.backpressure.model_id:
                            self.pq.set_backpressure(ack.backpressure.model_id)

                rt = asyncio.create_task(reader())
                try:
                    while not rt.done():
                        s = self.pq.load_snapshot("router")
                        await call.write(pb.LoadReport(node_id=s.node_id, queue_len=s.queue_len,
                                                       in_flight=s.in_flight, remaining_cap=s.remaining_cap))
                        await asyncio.sleep(interval_s)
                finally:
                    rt.cancel()
                    call.cancel()
            except asyncio.CancelledError:
                raise
            except Exception as e:
                LOG.debug("load sync: %s", e)
            await asyncio.sleep(1.0)

    async def _autoscale_loop(self, interval_s: float = 2.0) -> None:
        while True:
            await asyncio.sleep(interval_s)
            try:
                await self.autoscale_tick()
            except asyncio.CancelledError:
                raise
            except Exception as e:
                LOG.warning("autoscale tick: %s", e)

    async def autoscale_tick(self) -> None:
        await self._reap_draining()
        for node, ids in self.hot.drain().items():
            if node and ids:
                try:
                    await self.cp.ReportHits(pb.ReportHitsRequest(node_id=node, ids=[C.kid_out(k) for k in ids]),
                                             timeout=2.0)
                except Exception as e:
                    LOG.warning("report hits for %s failed: %s", node, e)
        if not self.cfg.autoscale:
            return
        d = self.scaler.evaluate(time.monotonic(), int(self.pq.queue_len()), int(self.pq.in_flight()),
                                 self.nodes.count())
        if d != H.ScaleDecision.NONE:
            await self.apply_scale(d)

    def _sync_capacity(self) -> None:
        self.pq.set_max_inflight(max(1, self.cfg.max_inflight) * max(1, self.nodes.count()))

    async def apply_scale(self, d) -> None:
        if d == H.ScaleDecision.SCALE_OUT:
            nid = self.nodes.next_id()
            t0 = time.perf_counter()
            resp = await self.cp.JoinShardNode(pb.JoinShardNodeRequest(node_id=nid), timeout=5.0)
            if not resp.ok:
                raise RuntimeError(f"JoinShardNode rejected: {resp.err}")
            self.nodes.add(nid)
            self._sync_capacity()
            self.last_ready_latency_s = time.perf_counter() - t0
        elif d == H.ScaleDecision.SCALE_IN:
            victim = self.nodes.last_ready()
            if not victim or not self.nodes.mark_draining(victim):
                return
            try:
                resp = await self.cp.DrainShardNode(pb.DrainShardNodeRequest(node_id=victim), timeout=5.0)
                if not resp.ok:
                    raise RuntimeError(resp.err)
            except Exception:
                self.nodes.unmark_draining(victim)  # drain did not run: capacity is kept
                self._sync_capacity()
                raise
            self._sync_capacity()
            await self._reap_draining()

    async def _reap_draining(self) -> None:
        for nid in self.nodes.draining():
            try:
                ack = await self.cp.RemoveShardNode(pb.RemoveShardNodeRequest(node_id=nid), timeout=2.0)
            except Exception:
                continue
            if ack.ok:
                self.nodes.remove(nid)
