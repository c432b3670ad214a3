"""Public serving API of one engine instance (one GPU, or the CPU oracle path).

    eng = LLMEngine("llama3-8b", device="cuda")
    rid = eng.add_request(prompt_token_ids, max_new_tokens=256)
    while eng.has_unfinished():
        for out in eng.step():
            ...

Each ``step()`` schedules a batch, stages its metadata through pinned host
memory, runs the model on the GPU and reads the sampled tokens back.
"""
from __future__ import annotations

import itertools
import time
from dataclasses import dataclass, field

import torch

from ..models.config import ModelConfig, get_config
from ..utils.trace import nvtx
from ..models.llama import DecoderLM
from .block_pool import BlockPool
from .model_runner import ModelRunner
from .request import Request, RequestStatus, SamplingParams
from .scheduler import Scheduler, SchedulerConfig, SchedulerOutput


@dataclass
class EngineConfig:
    model: str | ModelConfig = "llama3-8b"
    device: str = "cuda"
    max_running: int = 256
    max_batched_tokens: int = 8192
    long_prefill_threshold: int = 0
    max_model_len: int = 8192
    num_blocks: int = 0  # 0 = size from free memory
    kv_mem_fraction: float = 0.90
    enable_prefix_cache: bool = True
    use_cuda_graphs: bool = True
    seed: int = 0
    block_size: int = 16
    model_overrides: dict = field(default_factory=dict)
    # Arena other processes can map: a /dev/shm file on the CPU path, its own IPC-exportable
    # cudaMalloc allocation on the GPU (decode instances of PD-split)
    shared_arena: bool = False
    # Tensor parallel: (rank, world, process group for the handle exchange); every rank of the
    # group runs an engine with the same requests and makes the same scheduling decisions.
    tp: tuple | None = None
    weight_dtype: str = "bf16"  # "fp8": block-scaled e4m3 projection weights (W8A16 GEMMs)
    # Expert parallel (MoE): (rank, world, process group). Each rank serves its own requests and
    # steps in lockstep with the group (a step with no work still runs the expert exchange).
    ep: tuple | None = None
    # Overlapped scheduling: step() launches step n+1 before it waits for step n, so host
    # scheduling and metadata packing hide behind the device. A step's tokens are returned by
    # the following step() call. Not combined with a storage pool or expert parallel.
    overlap: bool = False
    # Inter-token latency target (ms): the scheduler caps the prefill tokens of mixed steps so
    # the step period stays under it (wall-clock feedback, so single-rank engines only: ranks of
    # a TP or EP group must schedule identically). 0 = off.
    itl_target_ms: float = 0.0
    # "native": this package's kernels; "library": the same model from library ops (cuBLAS, torch
    # SDPA, NCCL all_reduce, peer page copies; models/library.py), the benchmark comparator.
    # The library model runs eagerly (no CUDA graphs); with tp its group must be an NCCL group.
    model_impl: str = "native"
    # Speculative decoding (greedy): up to `spec_tokens` draft tokens per decode request from
    # prompt lookup (an earlier occurrence of the last `spec_ngram` tokens), verified in one
    # chunk per request. Steps with drafts run synchronously (no overlap).
    spec_tokens: int = 0
    spec_ngram: int = 3
    # Checkpoint: a safetensors file or directory (HF names). A model given as a directory with
    # config.json and safetensors shards loads both; otherwise weights are random-init.
    weights: str | None = None


@dataclass
class StepOutput:
    rid: str
    new_tokens: list[int]
    finished: bool


def alloc_arena(cfg: ModelConfig, num_blocks: int, device, dtype, block_size: int = 16) -> torch.Tensor:
    """Page-first KV arena [num_blocks, layers, 2, kv_heads, block_size, head_dim] (zero-filled)."""
    return torch.zeros(num_blocks, cfg.n_layers, 2, cfg.n_kv_heads, block_size, cfg.head_dim, dtype=dtype,
                       device=device)


def _local_kv_cfg(cfg: ModelConfig, world: int) -> ModelConfig:
    """The per-rank view of a tensor-parallel model's KV geometry."""
    import dataclasses

    return dataclasses.replace(cfg, n_kv_heads=cfg.n_kv_heads // world, n_q_heads=cfg.n_q_heads // world)


def page_bytes(cfg: ModelConfig, block_size: int = 16, elem: int = 2) -> int:
    return cfg.n_layers * 2 * cfg.n_kv_heads * block_size * cfg.head_dim * elem


class LLMEngine:
    def __init__(self, model: str | ModelConfig = "llama3-8b", device: str = "cuda", **kw):
        ec = EngineConfig(model=model, device=device, **kw)
        self.ec = ec
        cfg = model if isinstance(model, ModelConfig) else get_config(model, **ec.model_overrides)
        self.cfg = cfg
        self.device = torch.device(device)
        dtype = torch.float32 if self.device.type == "cpu" else torch.bfloat16
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        maxb = (ec.max_model_len + ec.block_size - 1) // ec.block_size
        max_tokens = ec.max_batched_tokens + ec.max_running
        self.tp_world = 1
        weights = ec.weights
        if weights is None and isinstance(model, str) and not isinstance(model, ModelConfig):
            from ..models.checkpoint import has_checkpoint

            weights = model if has_checkpoint(model) else None
        init = "zeros" if weights else "random"
        if ec.model_impl == "library":
            from ..models.library import LibraryLM

            tp = ec.tp if ec.tp is not None and ec.tp[1] > 1 else None
            full = DecoderLM(cfg, "cpu", torch.bfloat16, init="zeros", weights=weights).w if weights else None
            self.model = LibraryLM(cfg, self.device, dtype, seed=ec.seed, tp=tp, weights=full)
            ec.use_cuda_graphs = False
            self._arena_cfg = cfg
            if tp is not None:
                self.tp_world = tp[1]
                max_tokens += tp[1]
                cfg = self._arena_cfg = _local_kv_cfg(cfg, tp[1])
        elif ec.tp is not None and ec.tp[1] > 1:
            from ..models.llama_tp import TPDecoderLM
            from ..parallel.tp import TPGroup

            rank, world, pg = ec.tp
            self.tp_world = world
            max_tokens += world  # rows padded to a multiple of the group size
            self.tp_group = TPGroup(rank, world, self.device, max_tokens, cfg.hidden,
                                    ec.max_running * (1 + ec.spec_tokens), group=pg, status=None)
            full = None
            if weights:  # the whole checkpoint on the host, then this rank's shard
                full = DecoderLM(cfg, "cpu", torch.bfloat16, init="zeros", weights=weights).w
            self.model = TPDecoderLM(cfg, self.tp_group, self.device, seed=ec.seed, weight_dtype=ec.weight_dtype,
                                     full_weights=full)
            cfg = self._arena_cfg = _local_kv_cfg(cfg, world)
        elif ec.ep is not None and ec.ep[1] > 1:
            from ..parallel.ep import EPGroup

            rank, world, pg = ec.ep
            self.ep_group = EPGroup(rank, world, self.device, max_tokens, cfg.hidden, cfg.n_experts, cfg.top_k,
                                    group=pg)
            self.model = DecoderLM(cfg, self.device, dtype, seed=ec.seed, ep=self.ep_group, init=init,
                                   weights=weights)
            self._arena_cfg = cfg
        else:
            self.model = DecoderLM(cfg, self.device, dtype, seed=ec.seed, init=init, weights=weights)
            self._arena_cfg = cfg
            if ec.weight_dtype == "fp8" and self.device.type == "cuda":
                self.model.quantize_fp8()
                # fp8 GEMMs at prefill sizes run W8A8: the activations' e4m3 workspace for the largest step
                from ..ops._ext import native

                native().gemm_w8a8_reserve(max_tokens, max(cfg.hidden, cfg.q_size, cfg.intermediate))
        num_blocks = ec.num_blocks
        if not num_blocks:
            if self.device.type == "cuda":
                # leave room for activations / graphs: size the runner first, then the arena
                self.runner = None
                free, _ = torch.cuda.mem_get_info(self.device)
                act = max_tokens * (cfg.hidden * 4 + cfg.q_size * 4 + cfg.intermediate * 2) + 2 * 1024**3
                if ec.model_impl == "library":  # unfused intermediates + the decode batch's gathered K/V
                    act += max_tokens * cfg.intermediate * 8 + 2 * page_bytes(cfg, ec.block_size) // cfg.n_layers \
                        * ec.max_running * maxb
                num_blocks = int((free - act) * ec.kv_mem_fraction) // page_bytes(cfg, ec.block_size)
            else:
                num_blocks = 256
        self.arena_path = None
        shape = (num_blocks, cfg.n_layers, 2, cfg.n_kv_heads, ec.block_size, cfg.head_dim)
        cfg = self.cfg
        if ec.shared_arena and self.device.type == "cpu":
            from ..parallel.peer import alloc_shared_cpu_arena

            self.arena, self.arena_path = alloc_shared_cpu_arena(shape, dtype)
        elif ec.shared_arena:
            from ..parallel.peer import alloc_ipc_arena

            self.arena = alloc_ipc_arena(shape, dtype, self.device)
        else:
            self.arena = torch.zeros(shape, dtype=dtype, device=self.device)
        self.pool = BlockPool(num_blocks, ec.block_size, ec.enable_prefix_cache)
        single = self.tp_world == 1 and not (ec.ep and ec.ep[1] > 1)
        self.scheduler = Scheduler(self.pool, SchedulerConfig(ec.max_running, ec.max_batched_tokens,
                                                              ec.long_prefill_threshold, ec.max_model_len, maxb,
                                                              ec.spec_tokens, ec.spec_ngram,
                                                              ec.itl_target_ms if single else 0.0))
        self.runner = ModelRunner(self.model, self.arena, max_tokens, ec.max_running, maxb,
                                  ec.use_cuda_graphs, ec.block_size,
                                  row_multiple=self.tp_world, max_samples=ec.max_running * (1 + ec.spec_tokens))
        if ec.ep is not None and ec.ep[1] > 1:
            self.runner.lazy_capture = False
        self.requests: dict[str, Request] = {}
        self.peer_arenas: list = []  # decode arenas of a prefill instance serving several (set_peer_arenas)
        self.pool_iface = None  # PoolIface (storage-pool fences), attached by attach_pool
        self.overlap = ec.overlap and not (ec.ep and ec.ep[1] > 1) and ec.spec_tokens == 0
        self.inflight = None  # (SchedulerOutput, runner handle) of the launched, unfinished step
        self._drained: list[StepOutput] = []
        if self.overlap:
            self.runner.relay = True
            self.scheduler.before_preempt = self._drain
        self._ids = itertools.count()
        self.step_count = 0
        self.last_step: SchedulerOutput | None = None

    # ------------------------------------------------------------ requests
    def add_request(self, prompt: list[int], max_new_tokens: int = 16, rid: str | None = None,
                    params: SamplingParams | None = None, arrival: float | None = None) -> str:
        rid = rid or f"req-{next(self._ids)}"
        p = params or SamplingParams(max_new_tokens=max_new_tokens)
        req = Request(rid=rid, prompt=list(prompt), params=p)
        if arrival is not None:
            req.arrival = arrival
        self.scheduler.add(req)
        self.requests[rid] = req
        return rid

    def attach_pool(self, pool) -> None:
        """Route every step through a storage-pool interface (lake_b200.pool.PoolIface).
        An agent with ``prefetch(req)`` is called at admission, right before the prefix
        lookup, to bring pool-resident prefix pages back into HBM."""
        self.pool_iface = pool
        prefetch = getattr(pool.agent, "prefetch", None)
        self.scheduler.on_admit = prefetch if callable(prefetch) else None
        mirror = getattr(pool.agent, "mirror_arena", None)
        if mirror is not None and self.runner.peer_arena is None and self.tp_world == 1:
            # the agent's host slab becomes the QKV epilogue's second target (kernel write-behind);
            # graphs captured before this point do not write it and are dropped
            self.runner.mirror_arena = mirror
            self.runner.graphs.clear()
            self.runner.graph_launches.clear()

    def abort(self, rid: str) -> bool:
        return self.scheduler.abort(rid)

    # ------------------------------------------------------------ disaggregation hooks
    def reserve_blocks(self, n_tokens: int) -> list[int] | None:
        """Pages for a request another instance will prefill into this arena (None if full)."""
        n = (n_tokens + self.ec.block_size - 1) // self.ec.block_size
        if not self.pool.can_alloc(n):
            return None
        return self.pool.alloc(n)

    def release_blocks(self, blocks: list[int]) -> None:
        self.pool.release(blocks)

    def adopt_prefilled(self, rid: str, prompt: list[int], first_token: int, block_ids: list[int],
                        max_new_tokens: int, arrival: float | None = None) -> Request:
        """Decode side of PD-split: the prompt's KV was written into `block_ids` by a prefill
        instance, which also sampled `first_token`."""
        now = time.perf_counter()
        req = Request(rid=rid, prompt=list(prompt), params=SamplingParams(max_new_tokens=max_new_tokens))
        if arrival is not None:
            req.arrival = arrival
        req.block_ids = list(block_ids)
        req.output = [int(first_token)]
        req.first_token_time = now
        req.token_times.append(now)
        self.requests[rid] = req
        if req.should_stop():
            req.status = RequestStatus.FINISHED
            req.finish_time = now
            self.pool.release(req.block_ids)
            req.block_ids = []
            return req
        self.scheduler.adopt(req)
        return req

    def add_remote_prefill(self, prompt: list[int], remote_blocks: list[int], rid: str | None = None,
                           arrival: float | None = None, dest: int = 0) -> str:
        """Prefill side of PD-split: compute the prompt, write its K/V into the decode
        instance's pages `remote_blocks` (runner.peer_arena, or with several decode instances
        attached through set_peer_arenas, the arena of instance `dest`) and sample the first
        token."""
        if self.runner.peer_arena is None and not self.peer_arenas:
            raise RuntimeError("no peer arena attached (parallel.pd attaches the decode instance's arena)")
        if self.peer_arenas and not 0 <= dest < len(self.peer_arenas):
            raise ValueError(f"destination {dest} not among the {len(self.peer_arenas)} attached decode arenas")
        rid = self.add_request(prompt, max_new_tokens=1, rid=rid, arrival=arrival)
        req = self.requests[rid]
        req.remote_blocks = list(remote_blocks)
        req.meta["pd_dest"] = dest
        return rid

    def set_peer_arenas(self, arenas: list) -> None:
        """A prefill instance serving several decode instances: their arenas, indexed by the
        `dest` of add_remote_prefill. Each step then holds remote prefills of one destination
        only (the scheduler groups them) and its K/V stores go to that destination's arena."""
        self.peer_arenas = list(arenas)
        self.runner.peer_arena = self.peer_arenas[0] if self.peer_arenas else None
        self.scheduler.group_of = ((lambda r: r.meta.get("pd_dest") if r.remote_blocks is not None else None)
                                   if len(self.peer_arenas) > 1 else None)

    def _select_peer(self, out: SchedulerOutput) -> None:
        """Point the runner at the destination arena of this step's remote prefills."""
        if len(self.peer_arenas) > 1:
            for ch in out.prefill:
                if ch.req.remote_blocks is not None:
                    self.runner.peer_arena = self.peer_arenas[ch.req.meta.get("pd_dest", 0)]
                    return

    def _copy_cached_to_peer(self, out: SchedulerOutput) -> None:
        """Prefix pages served from this instance's cache are not recomputed, so their
        K/V go to the peer arena by a page copy (NVLink P2P on the GPU)."""
        src, dst = [], []
        for ch in out.prefill:
            r = ch.req
            if r.remote_blocks is None or not r.num_cached or r.meta.get("peer_copied"):
                continue
            nb = r.num_cached // self.ec.block_size
            src += r.block_ids[:nb]
            dst += r.remote_blocks[:nb]
            r.meta["peer_copied"] = True
        if not src:
            return
        if hasattr(self.model, "copy_pages"):  # library comparator: peer memcpy per page run
            self.model.copy_pages(self.arena, self.runner.peer_arena, src, dst)
            return
        from .. import ops

        dev = self.arena.device
        ops.page_copy(self.arena, self.runner.peer_arena, torch.tensor(src, device=dev),
                      torch.tensor(dst, device=dev), page_bytes(self._arena_cfg, self.ec.block_size,
                                                                self.arena.element_size()))

    def has_unfinished(self) -> bool:
        return self.scheduler.has_work() or self.inflight is not None

    # ------------------------------------------------------------ stepping
    def step(self) -> list[StepOutput]:
        with nvtx("engine.step"):
            return self._step()

    def _step(self) -> list[StepOutput]:
        if self.overlap and self.pool_iface is None:
            return self._step_overlap()
        out = self.scheduler.schedule()
        self.last_step = out
        if out.is_empty:
            if self.ec.ep is not None and self.ec.ep[1] > 1:
                self.runner.execute_null()  # the group's expert exchange needs every rank
                self.step_count += 1
            return []
        bitmask = self._bitmask(out)
        self._select_peer(out)
        if self.runner.peer_arena is not None:
            self._copy_cached_to_peer(out)
        if self.pool_iface is not None:
            self.pool_iface.prepare_step(out)  # ready fence
            try:
                sampled = self.runner.execute(out, bitmask)
            finally:
                self.pool_iface.done(out.step_id)  # compute fence
        else:
            sampled = self.runner.execute(out, bitmask)
        now = time.perf_counter()
        finished = self.scheduler.update(out, sampled, now)
        if self.pool_iface is not None:
            for r in finished:
                self.pool_iface.on_request_finished(r, self.cfg.name)
        self.step_count += 1
        # one output per sampling chunk: its token, or every verified token of a verify chunk
        return [StepOutput(ch.req.rid, list(ch.accepted), ch.req.finished)
                for ch in out.chunks if ch.sample and ch.accepted]

    # ------------------------------------------------------------ overlapped stepping
    def _step_overlap(self) -> list[StepOutput]:
        """Schedule and launch step n+1, then finish step n (wait, fill in its tokens) and
        return step n's outputs. Steps with token bitmasks run synchronously."""
        out = self.scheduler.schedule()  # may drain the in-flight step to preempt
        self.last_step = out
        # a drain during scheduling may have finished (stop token) requests it had already placed
        out.decode = [c for c in out.decode if c.req.status == RequestStatus.RUNNING]
        out.prefill = [c for c in out.prefill if c.req.status == RequestStatus.RUNNING]
        res, self._drained = self._drained, []
        if out.is_empty:
            return res + self._finish_inflight()
        bitmask = self._bitmask(out)
        if bitmask is not None:
            res += self._finish_inflight()  # the masks apply to the tokens after the in-flight ones
        self._select_peer(out)
        if self.runner.peer_arena is not None:
            self._copy_cached_to_peer(out)
        handle = self.runner.launch(out, bitmask)
        res += self._finish_inflight()
        self.scheduler.advance(out)
        self.inflight = (out, handle)
        self.step_count += 1
        if bitmask is not None:
            res += self._finish_inflight()
        return res

    def _finish_inflight(self) -> list[StepOutput]:
        if self.inflight is None:
            return []
        out, handle = self.inflight
        self.inflight = None
        sampled = self.runner.collect(handle)
        applied = self.scheduler.resolve(out, sampled, time.perf_counter())
        return [StepOutput(r.rid, [tok], r.finished) for r, tok in applied]

    def _drain(self) -> None:
        """Scheduler hook before a preemption: finish the in-flight step now."""
        self._drained += self._finish_inflight()

    def _bitmask(self, out: SchedulerOutput):
        rows = [c.req.bitmask for c in out.chunks if c.sample]
        if not any(r is not None for r in rows):
            return None
        words = (self.cfg.vocab + 31) // 32
        bm = torch.full((len(rows), words), -1, dtype=torch.int32)
        for i, r in enumerate(rows):
            if r is not None:
                bm[i] = torch.as_tensor(r, dtype=torch.int32)
        return bm.to(self.device, non_blocking=True)

    def generate(self, prompts: list[list[int]], max_new_tokens: int = 16) -> list[list[int]]:
        rids = [self.add_request(p, max_new_tokens) for p in prompts]
        while self.has_unfinished():
            self.step()
        return [self.requests[r].output for r in rids]

    # ------------------------------------------------------------ metrics
    def metrics(self) -> dict:
        fin = [r for r in self.requests.values() if r.status == RequestStatus.FINISHED]
        ttft = sorted(x for x in (r.ttft() for r in fin) if x is not None)
        tpot = sorted(x for x in (r.tpot() for r in fin) if x is not None)

        def p50(xs):
            return xs[len(xs) // 2] if xs else None

        return {"finished": len(fin), "ttft_p50_s": p50(ttft), "tpot_p50_s": p50(tpot),
                "prefix_hit_blocks": self.pool.stats["hits"], "pool": self.pool.residency(),
                "h2d_bytes": self.runner.h2d_bytes, "d2h_bytes": self.runner.d2h_bytes}
